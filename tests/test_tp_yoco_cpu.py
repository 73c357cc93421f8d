"""Tensor-parallel YOCO (the reference's Megatron column / row / vocabulary-parallel declarations) on 2 gloo ranks:
loading the TP slices of a full checkpoint reproduces the TP=1 logits and weight gradients."""
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.config import build_args
from faster_yoco_b200.utils.launch import run_ranks


def _args(mp, window=None):
    return build_args("yoco_tiny", n_layers=2, max_seq_len=64, max_batch_size=2, model_parallel_size=mp,
                      sliding_window=window)


def _worker(rank, world, full_sd, ids, ref_logits, ref_grads, window):
    from faster_yoco_b200.models.yoco import YOCO, shard_state_dict
    from faster_yoco_b200.parallel import tp
    ops.set_backend("torch")
    tp.init_model_parallel(world)
    torch.manual_seed(0)
    m = YOCO(_args(world, window))
    missing, unexpected = m.load_state_dict(shard_state_dict(full_sd, world, rank), strict=True)
    logits, _ = m(ids)
    torch.testing.assert_close(logits, ref_logits, atol=2e-4, rtol=2e-4)
    logits.pow(2).mean().backward()
    mix = m.self_decoder.layers[0].mixer
    merged = mix.qkvg_proj if window is None else mix.qkv_proj
    n = merged.parts[0]                                   # this rank's q rows
    torch.testing.assert_close(merged.weight.grad[:n], ref_grads["q"][rank * n:(rank + 1) * n], atol=1e-5, rtol=1e-3)
    g_out = mix.out_proj.weight.grad
    c = g_out.shape[1]
    torch.testing.assert_close(g_out, ref_grads["out"][:, rank * c:(rank + 1) * c], atol=1e-5, rtol=1e-3)
    g_emb = m.embed_tokens.weight.grad
    v = g_emb.shape[0]
    torch.testing.assert_close(g_emb, ref_grads["emb"][rank * v:(rank + 1) * v], atol=1e-5, rtol=1e-3)
    # the exported state dict is this rank's shard under the reference names
    sd = m.state_dict()
    assert sd["self_decoder.layers.0.mixer.q_proj.weight"].shape[0] == n
    tp.destroy_model_parallel()


def _run(window):
    from faster_yoco_b200.models.yoco import YOCO
    ops.set_backend("torch")
    torch.manual_seed(0)
    m = YOCO(_args(1, window))
    ids = torch.randint(0, 1024, (2, 32))
    logits, _ = m(ids)
    logits.pow(2).mean().backward()
    mix = m.self_decoder.layers[0].mixer
    merged = mix.qkvg_proj if window is None else mix.qkv_proj
    grads = {"q": merged.weight.grad[:merged.parts[0]].clone(), "out": mix.out_proj.weight.grad.clone(),
             "emb": m.embed_tokens.weight.grad.clone()}
    full = {k: v.detach().clone() for k, v in m.state_dict().items()}
    run_ranks(_worker, 2, full, ids, logits.detach(), grads, window)


def test_tp2_retention_yoco_matches_tp1():
    _run(None)


def test_tp2_sliding_window_yoco_matches_tp1():
    _run(16)


def _cli_tp_worker(rank, world, data, save, out, max_update):
    import contextlib
    import io
    from faster_yoco_b200.cli import train as T
    from faster_yoco_b200.parallel import tp
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                     "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead", "4",
                     "--log-interval", "2", "--warmup-updates", "1", "--max-update", str(max_update),
                     "--save-dir", save, "--cpu", "--kernels", "torch", "--model-parallel-size", "2", "--seed", "3"])
    assert rc == 0
    if rank == 0:
        open(out, "w").write(buf.getvalue())
    tp.destroy_model_parallel()


def test_cli_tensor_parallel_training_matches_single_rank(tmp_path):
    """The train CLI with --model-parallel-size 2 on 2 ranks: the same losses / gradient norms as one rank, one
    checkpoint part per TP rank holding that rank's slices of the single-rank weights, and resume from the parts."""
    import contextlib
    import io
    import json
    import os
    from faster_yoco_b200.cli import train as T
    from faster_yoco_b200.models.yoco import shard_state_dict
    data = str(tmp_path / "data")
    os.makedirs(os.path.join(data, "json"))
    os.makedirs(os.path.join(data, "shard", "w"))
    with open(os.path.join(data, "shard", "w", "00000.jsonl"), "w") as f:
        for d in range(40):
            f.write(json.dumps({"text": f"doc {d}: a few words to pack\n\nmore words"}) + "\n")
    json.dump(["shard/w/00000.jsonl"], open(os.path.join(data, "json", "w.json"), "w"))
    json.dump([{"name": "w", "weight": 1.0}], open(os.path.join(data, "json", "train.json"), "w"))
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        assert T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                       "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead",
                       "4", "--log-interval", "2", "--warmup-updates", "1", "--max-update", "2",
                       "--save-dir", str(tmp_path / "s1"), "--cpu", "--kernels", "torch", "--seed", "3"]) == 0
    single = [l for l in buf.getvalue().splitlines() if l.startswith("epoch")][-1]
    out = str(tmp_path / "tp.log")
    run_ranks(_cli_tp_worker, 2, data, str(tmp_path / "s2"), out, 2)
    tpline = [l for l in open(out).read().splitlines() if l.startswith("epoch")][-1]
    loss = lambda l: float(l.split("loss ")[1].split(" ")[0])
    gn = lambda l: float(l.split("gnorm ")[1].split(" ")[0])
    assert abs(loss(single) - loss(tpline)) < 2e-3 and abs(gn(single) - gn(tpline)) < 2e-3 * max(1.0, gn(single))
    s1 = torch.load(str(tmp_path / "s1" / "checkpoint_last.pt"), weights_only=False)["model"]
    full = {k[len("decoder.model."):]: v.float() for k, v in s1.items()}
    for r in range(2):
        part = torch.load(str(tmp_path / "s2" / f"checkpoint_last-model_part-{r}.pt"), weights_only=False)["model"]
        want = shard_state_dict(full, 2, r)
        for k in ("embed_tokens.weight", "self_decoder.layers.0.mixer.q_proj.weight",
                  "self_decoder.layers.0.mixer.out_proj.weight", "self_decoder.layers.0.mixer_layer_norm.weight"):
            torch.testing.assert_close(part["decoder.model." + k].float(), want[k], atol=1e-5, rtol=1e-4)
    # resume from the parts and take one more update
    run_ranks(_cli_tp_worker, 2, data, str(tmp_path / "s2"), out, 3)
    assert "loaded checkpoint" in open(out).read()


def _cli_validate_tp_worker(rank, world, data_dir, out, mp):
    import contextlib
    import io
    from faster_yoco_b200.cli import validate as V
    from faster_yoco_b200.parallel import tp
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        assert V.main(["--task", "harness_eval", "--criterion", "harness_eval", "--eval-data", "harness_boolq",
                       "--data-dir", data_dir, "--batch-size", "4", "--arch", "yoco_tiny", "--n-layers", "2",
                       "--tiktoken-model", "byte", "--tokens-per-sample", "128", "--cpu", "--kernels", "torch",
                       "--model-parallel-size", str(mp), "--seed", "5"]) == 0
    if rank == 0:
        open(out, "w").write(buf.getvalue())
    tp.destroy_model_parallel()


def test_cli_validate_tensor_parallel_matches_single_rank(tmp_path):
    """Harness evaluation with --model-parallel-size 2 on 2 ranks (both ranks on the same batches) reproduces the
    single-rank accuracy and loss."""
    import json
    import test_components_cpu as TC
    TC._write_boolq(str(tmp_path))
    one, two = str(tmp_path / "one.log"), str(tmp_path / "two.log")
    run_ranks(_cli_validate_tp_worker, 1, str(tmp_path), one, 1)
    run_ranks(_cli_validate_tp_worker, 2, str(tmp_path), two, 2)
    a = json.loads(open(one).read().strip().splitlines()[-1])
    b = json.loads(open(two).read().strip().splitlines()[-1])
    assert a["accuracy"] == b["accuracy"] and a["accuracy_norm"] == b["accuracy_norm"]
    assert abs(a["loss"] - b["loss"]) <= 2e-3, (a, b)            # per-option NLL: the same model outputs
