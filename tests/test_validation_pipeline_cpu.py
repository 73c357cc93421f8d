"""End to end on CPU with the tiny model: four training arms with model-only saves through the train CLI, a packed
held-out set, held-out evaluation of every checkpoint, the summary tables and the verdict."""
import contextlib
import io
import json
import os

import torch


def _corpus(root, n_files=3, docs=30):
    os.makedirs(os.path.join(root, "json"), exist_ok=True)
    os.makedirs(os.path.join(root, "shard", "web"), exist_ok=True)
    files = []
    for i in range(n_files):
        rel = f"shard/web/{i:05d}.jsonl"
        with open(os.path.join(root, rel), "w") as f:
            for d in range(docs):
                f.write(json.dumps({"text": f"document {i}.{d}: the cat sat on the mat\n\nand then it slept"}) + "\n")
        files.append(rel)
    json.dump(files, open(os.path.join(root, "json", "web.json"), "w"))
    json.dump([{"name": "web", "weight": 1.0}], open(os.path.join(root, "json", "train.json"), "w"))


def test_paired_validation_pipeline(tmp_path):
    from faster_yoco_b200.cli import train as T
    from faster_yoco_b200.data.tokenizers import ByteTokenizer
    from faster_yoco_b200.validation import analyze, eval_ckpt, heldout, verdict
    data = str(tmp_path / "data")
    _corpus(data)
    V = str(tmp_path / "val")
    for arm, seed, kernels in (("opt", 1, "torch"), ("ref", 1, "torch"), ("ref_s2", 2, "torch"),
                               ("opt_s2", 2, "torch")):
        out = os.path.join(V, arm)
        os.makedirs(out, exist_ok=True)
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            rc = T.main([data, "--arch", "yoco_tiny", "--task", "gpt", "--tiktoken-model", "byte",
                         "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len",
                         "--batch-read-ahead", "8", "--log-interval", "2", "--warmup-updates", "2",
                         "--save-dir", os.path.join(out, "ckpt"), "--save-model-only", "--save-interval-updates", "2",
                         "--max-update", "4", "--seed", str(seed), "--cpu", "--kernels", kernels])
        assert rc == 0
        with open(os.path.join(out, "train.log"), "w") as f:
            f.write(buf.getvalue())
        assert sorted(os.listdir(os.path.join(out, "ckpt"))) == ["model_000002.pt", "model_000004.pt"]
    # held-out set: two sources, packed like the training loader
    hd = str(tmp_path / "held")
    os.makedirs(hd)
    for name, txt in (("fineweb_edu", "held out prose number {}"), ("codeparrot", "def held_{}():\n    return {}")):
        with open(os.path.join(hd, f"heldout_{name}.jsonl"), "w") as f:
            for i in range(40):
                f.write(json.dumps({"text": txt.format(i, i) * 3}) + "\n")
    heldout.build(hd, os.path.join(hd, "heldout.pt"), 2, 1, ByteTokenizer(), tokens_per_sample=64)
    for arm in ("opt", "ref", "ref_s2", "opt_s2"):
        ck = sorted(os.path.join(V, arm, "ckpt", f) for f in os.listdir(os.path.join(V, arm, "ckpt")))
        assert eval_ckpt.main([os.path.join(hd, "heldout.pt"), os.path.join(V, arm, "eval.json"), *ck,
                               "--arch", "yoco_tiny", "--kernels", "torch"]) == 0
        ev = json.load(open(os.path.join(V, arm, "eval.json")))
        assert set(ev) == {"model_000002.pt", "model_000004.pt"}
        assert all(0 < r["mix_0.8_0.2_bits"] < 20 for r in ev.values())
    assert analyze.main([V]) == 0
    S = json.load(open(os.path.join(V, "summary.json")))["arms"]
    assert S["opt"]["updates"] == 4 and set(S["opt"]["heldout"]) == {"2", "4"}
    assert verdict.main([V]) == 0
    text = open(os.path.join(V, "verdict.md")).read()
    v = json.loads(text[text.index("{"):])
    assert v["mix"]["checkpoints"] == 2
    # same seed, same path: the opt and ref arms are the same run
    assert S["opt"]["heldout"]["4"]["mix_bits"] == S["ref"]["heldout"]["4"]["mix_bits"]
