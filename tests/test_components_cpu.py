"""Tasks, criterions, generation, LLaMA baseline, tensor parallelism, CLI entry points (CPU)."""
import json
import math
import os

import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.config import OptimConfig, build_args
from faster_yoco_b200.data.tokenizers import ByteTokenizer
from faster_yoco_b200.ops import reference as R
from faster_yoco_b200.utils.launch import run_ranks


def test_hier_chunk_retention_matches_chunkwise():
    torch.manual_seed(0)
    B, H, L, D = 1, 2, 512, 16
    q, k, v = [torch.randn(B, H, L, D, dtype=torch.float64) for _ in range(3)]
    g = torch.nn.functional.logsigmoid(torch.randn(B, H, L, dtype=torch.float64)) / 16
    a = R.hier_chunk_gate_retention(q, k, v, g, 64, 128)
    b = R.chunk_gate_retention(q, k, v, g, 64)
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-6)


def test_neox_rope_oracle():
    torch.manual_seed(0)
    x = torch.randn(2, 5, 3, 16)
    ang = R.llama_rope_angles(16, 5, 10000.0)
    cos, sin = torch.cos(ang), torch.sin(ang)
    y = R.apply_rope(x, cos, sin, interleaved=False)
    z = torch.complex(x[..., :8], x[..., 8:]) * torch.polar(torch.ones_like(ang), ang)[None, :, None, :]
    torch.testing.assert_close(y, torch.cat([z.real, z.imag], -1), atol=1e-5, rtol=1e-5)
    back = R.apply_rope(y, cos, sin, conjugate=True, interleaved=False)
    torch.testing.assert_close(back, x, atol=1e-5, rtol=1e-5)


def _tiny_llama(window=None, mp=1, vocab=96):
    from faster_yoco_b200.models.transformer import LLaMA, Transformer, llama_args_from_cfg
    a = llama_args_from_cfg(64, 2, 4, 2, vocab, batch_size=2, tokens_per_sample=64, model_parallel_size=mp,
                            sliding_window=window)
    return LLaMA(Transformer(a))


@pytest.mark.parametrize("window", [None, 8])
def test_llama_incremental_decode_matches_full(window):
    ops.set_backend("torch")
    torch.manual_seed(0)
    m = _tiny_llama(window).eval()
    ids = torch.randint(0, 96, (2, 24))
    full, _ = m(ids)
    st = {}
    out = [m(ids[:, :10], start_pos=0, incremental_state=st)[0]]
    for t in range(10, 24):
        out.append(m(ids[:, t:t + 1], start_pos=t, incremental_state=st)[0])
    torch.testing.assert_close(torch.cat(out, 1), full, atol=2e-4, rtol=2e-4)


def test_llama_param_names_and_hidden_dim():
    m = _tiny_llama()
    names = set(m.model.state_dict())
    assert "layers.0.attention.wq.weight" in names and "layers.1.feed_forward.w3.weight" in names
    assert m.model.layers[0].feed_forward.w1.weight.shape == (int(64 * 8 / 3), 64)
    assert "tok_embeddings.weight" in names and "output.weight" in names and "norm.weight" in names


def _tp_worker(rank, world, full_sd, ids, ref_logits, ref_grads):
    from faster_yoco_b200.parallel import tp
    ops.set_backend("torch")
    tp.init_model_parallel(world)
    torch.manual_seed(0)
    m = _tiny_llama(mp=world)
    m.model.load_state_dict(full_sd)
    logits, _ = m(ids)
    # the output layer is column-parallel without gather: each rank holds its vocabulary slice
    n = ref_logits.shape[-1] // world
    torch.testing.assert_close(logits, ref_logits[..., rank * n:(rank + 1) * n], atol=1e-4, rtol=1e-4)
    full = tp.gather_from_tp(logits)
    full.float().pow(2).sum().backward()
    g = m.model.layers[0].attention.wq.weight.grad
    rows = g.shape[0]
    torch.testing.assert_close(g, ref_grads["wq"][rank * rows:(rank + 1) * rows], atol=1e-3, rtol=1e-3)
    g2 = m.model.layers[0].feed_forward.w2.weight.grad
    cols = g2.shape[1]
    torch.testing.assert_close(g2, ref_grads["w2"][:, rank * cols:(rank + 1) * cols], atol=1e-3, rtol=1e-3)
    ge = m.model.tok_embeddings.weight.grad
    torch.testing.assert_close(ge, ref_grads["emb"][rank * ge.shape[0]:(rank + 1) * ge.shape[0]], atol=1e-3,
                               rtol=1e-3)
    tp.destroy_model_parallel()


def test_tensor_parallel_llama_matches_dense():
    ops.set_backend("torch")
    torch.manual_seed(0)
    m = _tiny_llama()
    ids = torch.randint(0, 96, (2, 12))
    logits, _ = m(ids)
    logits.float().pow(2).sum().backward()
    grads = {"wq": m.model.layers[0].attention.wq.weight.grad.clone(),
             "w2": m.model.layers[0].feed_forward.w2.weight.grad.clone(),
             "emb": m.model.tok_embeddings.weight.grad.clone()}
    sd = {k: v.detach().clone() for k, v in m.model.state_dict().items()}
    run_ranks(_tp_worker, 2, sd, ids, logits.detach(), grads)


def _tiny_yoco(vocab=264, layers=2):
    from faster_yoco_b200.models.yoco import YOCO
    a = build_args("yoco_tiny", vocab_size=vocab, n_layers=layers, max_seq_len=512, max_batch_size=2)
    return YOCO(a)


def test_generate_matches_naive_greedy():
    from faster_yoco_b200.eval.generate import generate
    ops.set_backend("torch")
    torch.manual_seed(0)
    m = _tiny_yoco().eval()
    tok = ByteTokenizer()
    prompt = torch.tensor([tok.encode("hello world, the magic number is", bos=True)])
    out = generate(m, prompt, tok, generate_tokens=6, chunk_length=8)
    seq = prompt.clone()
    with torch.no_grad():
        for _ in range(6):
            lg, _ = m(seq)
            lg = lg[:, -1].float()
            lg[:, tok.bos_id] = -math.inf
            lg[:, tok.pad_id] = -math.inf
            nxt = lg.argmax(-1, keepdim=True)
            seq = torch.cat([seq, nxt], 1)
            if int(nxt) == tok.eos_id:
                break
    assert torch.equal(out[:, :seq.shape[1]], seq)


def _write_boolq(d):
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "boolq"), "w") as f:
        for i in range(6):
            f.write(json.dumps({"ctx": f"passage {i}\nQuestion: is it true?\nAnswer:", "label": i % 2}) + "\n")
    with open(os.path.join(d, "winogrande"), "w") as f:
        f.write(json.dumps({"sentence": "The cat sat because _ was tired.", "option1": "the cat",
                            "option2": "the mat", "answer": "1"}) + "\n")


def test_harness_tokenization_and_mask(tmp_path):
    from faster_yoco_b200.tasks.harness import HARNESS_TASKS, HarnessDataset
    assert len(HARNESS_TASKS) == 19 + 57
    _write_boolq(str(tmp_path))
    tok = ByteTokenizer()
    ds = HarnessDataset("harness_boolq", tok, str(tmp_path), tokens_per_sample=64)
    src, masks, label_len, labels = ds.get_data_for_evaluation()
    assert len(src) == 12 and list(labels[:2]) == [0, 0]
    assert tok.decode(src[0]).endswith("Answer: no") and tok.decode(src[1]).endswith("Answer: yes")
    assert src[0][0] == tok.bos_id and sum(masks[0]) == len(" no") and masks[0][-1]
    assert list(label_len[:2]) == [2, 3]
    short = HarnessDataset("harness_boolq", tok, str(tmp_path), tokens_per_sample=16)
    s2, m2, _, _ = short.get_data_for_evaluation()
    assert all(len(s) <= 16 for s in s2) and all(len(s) == len(m) for s, m in zip(s2, m2))
    w = HarnessDataset("harness_winogrande", tok, str(tmp_path), tokens_per_sample=64)
    ws, _, _, wl = w.get_data_for_evaluation()
    assert tok.decode(ws[0]).startswith("The cat sat because the cat") and int(wl[0]) == 0


def test_harness_criterion_argmin():
    from faster_yoco_b200.criterions.harness_eval import HarnessEvalCriterion
    from faster_yoco_b200.tasks.harness import collate_options

    class Task:
        class harness_task:
            class_num = 2

        class target_dictionary:
            @staticmethod
            def pad():
                return 1

    V = 8

    class Model(torch.nn.Module):
        def forward(self, ids):
            # next-token logits strongly prefer token 5 everywhere
            lg = torch.zeros(*ids.shape, V)
            lg[..., 5] = 10.0
            return lg, None

    src = [[0, 4, 5, 5], [0, 4, 6, 6], [0, 4, 6], [0, 4, 5]]
    masks = [[False, False, True, True], [False, False, True, True], [False, False, True], [False, False, True]]
    b = collate_options(src, masks, [2, 2, 1, 1], [0, 0, 1, 1], pad_id=1)
    _, _, log = HarnessEvalCriterion(Task)(Model(), b)
    assert log["ncorrect"] == 2 and log["ncorrect_norm"] == 2 and log["nsentences"] == 2


def test_needle_prompts(tmp_path):
    from faster_yoco_b200.criterions.needle import MultiNeedleCriterion, NeedleHaystackCriterion, random_partition
    import random
    essays = tmp_path / "essays"
    essays.mkdir()
    for i in range(3):
        (essays / f"e{i}.txt").write_text("\n".join(f"essay {i} line {j} about startups." for j in range(50)))

    class Task:
        tokenizer = ByteTokenizer()

    random.seed(3)
    parts = random_partition(100, 4)
    assert sum(parts) == 100 and all(p > 0 for p in parts)
    c = NeedleHaystackCriterion(Task, tokens_per_sample=600, interval=600, needle_file_path=str(essays))
    random.seed(0)
    text, ans = c.prompt(200, 200)
    assert f"number is {ans} ." in text and text.startswith("There is a special magic number")
    mc = MultiNeedleCriterion(Task, needle_num=3, tokens_per_sample=600, interval=600, needle_file_path=str(essays))
    random.seed(42)
    text, ans = mc.prompt(200, 200)
    assert text.count("The special magic") == 3 + 1 and f"number is: {ans}" in text


def test_needle_criterion_runs(tmp_path):
    from faster_yoco_b200.criterions.needle import NeedleHaystackCriterion
    ops.set_backend("torch")
    essays = tmp_path / "essays"
    essays.mkdir()
    (essays / "a.txt").write_text("\n".join(f"line {j}" for j in range(100)))

    class Task:
        tokenizer = ByteTokenizer()

    c = NeedleHaystackCriterion(Task, tokens_per_sample=300, interval=300, needle_file_path=str(essays),
                                generate_tokens=3)
    c.trials = 1
    torch.manual_seed(0)
    m = _tiny_yoco()
    _, _, log = c(m, device=torch.device("cpu"))
    assert list(log["retrieval"]) == [300] and len(log["retrieval"][300]) == 11


def test_pseudo_task_batches():
    from faster_yoco_b200.tasks.base import TaskConfig
    from faster_yoco_b200.tasks.pseudo import PseudoTask
    t = PseudoTask.setup_task(TaskConfig(tiktoken_model="byte", tokens_per_sample=16, batch_size=3))
    b = next(t.get_batch_iterator(None))
    assert b["src_tokens"].shape == (3, 16) and torch.equal(b["src_tokens"], b["target"])
    assert b["ntokens"] == 48 and int(b["src_tokens"].max()) < 9999


def test_update_freq_equals_concatenated_batch():
    from faster_yoco_b200.train.trainer import Trainer
    ops.set_backend("torch")

    def run(micro):
        torch.manual_seed(0)
        m = _tiny_yoco(vocab=128)
        tr = Trainer(m, OptimConfig(warmup_updates=0, lr=1e-3), device="cpu", graph_step=False)
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(2, 128, (2, 33), generator=g)
        if micro:
            batch = [{"src_tokens": ids[i:i + 1, :-1], "target": ids[i:i + 1, 1:], "ntokens": 33, "nsentences": 1}
                     for i in range(2)]
        else:
            batch = {"src_tokens": ids[:, :-1], "target": ids[:, 1:], "ntokens": 66, "nsentences": 2}
        loss = tr.train_step(batch)
        return float(loss), torch.cat([p.detach().reshape(-1) for p in m.parameters()])

    l1, p1 = run(True)
    l2, p2 = run(False)
    assert abs(l1 - l2) < 1e-3 * abs(l2)
    torch.testing.assert_close(p1, p2, atol=1e-5, rtol=1e-4)


def _corpus(root):
    os.makedirs(os.path.join(root, "json"), exist_ok=True)
    os.makedirs(os.path.join(root, "shard", "web"), exist_ok=True)
    files = []
    for i in range(4):
        rel = f"shard/web/{i:05d}.jsonl"
        with open(os.path.join(root, rel), "w") as f:
            for d in range(30):
                f.write(json.dumps({"text": f"document {i}.{d}: some words here\n\nand more words there"}) + "\n")
        files.append(rel)
    json.dump(files, open(os.path.join(root, "json", "web.json"), "w"))
    json.dump([{"name": "web", "weight": 1.0}], open(os.path.join(root, "json", "train.json"), "w"))


def test_cli_train_validation_pass(tmp_path, capsys):
    from faster_yoco_b200.cli import train as T
    data = str(tmp_path / "data")
    _corpus(data)
    json.dump([{"name": "web", "weight": 1.0}], open(os.path.join(data, "json", "valid.json"), "w"))
    assert T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                   "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead", "4",
                   "--log-interval", "2", "--validate-interval-updates", "2", "--max-valid-steps", "3",
                   "--max-update", "4", "--no-save", "--cpu", "--kernels", "torch"]) == 0
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("valid on 'valid' subset")]
    assert len(lines) == 2 and "num_updates 4" in lines[-1]


def test_cli_train_save_resume(tmp_path, capsys):
    from faster_yoco_b200.cli import train as T
    data = str(tmp_path / "data")
    _corpus(data)
    save = str(tmp_path / "ckpt")
    common = [data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
              "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead", "8",
              "--log-interval", "2", "--warmup-updates", "2", "--save-dir", save, "--cpu", "--kernels", "torch"]
    assert T.main(common + ["--max-update", "2", "--save-interval-updates", "2"]) == 0
    assert os.path.exists(os.path.join(save, "checkpoint_last.pt"))
    ck = torch.load(os.path.join(save, "checkpoint_last.pt"), weights_only=False)
    assert ck["optimizer_history"][-1]["num_updates"] == 2
    assert ck["extra_state"]["train_iterator"][0] is not None
    assert any(k.startswith("decoder.model.self_decoder.layers.0.mixer.q_proj") for k in ck["model"])
    assert T.main(common + ["--max-update", "4"]) == 0
    ck = torch.load(os.path.join(save, "checkpoint_last.pt"), weights_only=False)
    assert ck["optimizer_history"][-1]["num_updates"] == 4


def test_cli_validate_harness(tmp_path, capsys):
    from faster_yoco_b200.cli import validate as V
    _write_boolq(str(tmp_path))
    assert V.main(["--task", "harness_eval", "--criterion", "harness_eval", "--eval-data", "harness_boolq",
                   "--data-dir", str(tmp_path), "--batch-size", "4", "--arch", "yoco_tiny", "--n-layers", "2",
                   "--tiktoken-model", "byte", "--tokens-per-sample", "128", "--cpu", "--kernels", "torch"]) == 0
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert 0.0 <= res["accuracy"] <= 100.0 and "accuracy_norm" in res


def test_cli_llama_train_and_harness(tmp_path, capsys):
    from faster_yoco_b200.cli import train as T
    from faster_yoco_b200.cli import validate as V
    data = str(tmp_path / "data")
    _corpus(data)
    small = ["--arch", "llama_from_scratch", "--dim", "64", "--n-layers", "2", "--n-heads", "4", "--n-kv-heads", "2",
             "--tiktoken-model", "byte", "--cpu", "--kernels", "torch"]
    assert T.main([data, "--task", "gpt", "--tokens-per-sample", "32", "--batch-size", "2", "--pad-to-max-len",
                   "--batch-read-ahead", "4", "--log-interval", "2", "--warmup-updates", "1", "--max-update", "2",
                   "--save-dir", str(tmp_path / "ck"), *small]) == 0
    ck = torch.load(str(tmp_path / "ck" / "checkpoint_last.pt"), weights_only=False)
    assert "decoder.model.layers.0.attention.wq.weight" in ck["model"]       # the reference's key layout
    assert "layers.0.attention.wq.weight" in ck["last_optimizer_state"]["master"]
    # resume reads the same layout back
    assert T.main([data, "--task", "gpt", "--tokens-per-sample", "32", "--batch-size", "2", "--pad-to-max-len",
                   "--batch-read-ahead", "4", "--log-interval", "2", "--warmup-updates", "1", "--max-update", "3",
                   "--save-dir", str(tmp_path / "ck"), *small]) == 0
    assert torch.load(str(tmp_path / "ck" / "checkpoint_last.pt"),
                      weights_only=False)["optimizer_history"][-1]["num_updates"] == 3
    _write_boolq(str(tmp_path / "h"))
    capsys.readouterr()
    assert V.main(["--task", "harness_eval", "--criterion", "harness_eval", "--eval-data", "harness_boolq",
                   "--data-dir", str(tmp_path / "h"), "--batch-size", "2", "--tokens-per-sample", "128", *small]) == 0
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "accuracy" in res


def test_cli_validate_needle(tmp_path, capsys):
    from faster_yoco_b200.cli import validate as V
    essays = tmp_path / "essays"
    essays.mkdir()
    (essays / "a.txt").write_text("\n".join(f"line {j} of an essay" for j in range(60)))
    assert V.main(["--task", "pseudo", "--criterion", "needle_haystack", "--batch-size", "1", "--arch", "yoco_tiny",
                   "--n-layers", "2", "--tiktoken-model", "byte", "--tokens-per-sample", "256", "--interval", "256",
                   "--needle-file-path", str(essays), "--cpu", "--kernels", "torch"]) == 0
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    ret = res["retrieval"][0]
    assert list(ret) == ["256"] or list(ret) == [256]


def test_cli_validate_lm_perplexity(tmp_path, capsys):
    from faster_yoco_b200.cli import validate as V
    data = str(tmp_path / "data")
    _corpus(data)
    json.dump([{"name": "web", "weight": 1.0}], open(os.path.join(data, "json", "valid.json"), "w"))
    assert V.main([data, "--task", "gpt", "--criterion", "cross_entropy", "--valid-subset", "valid", "--arch",
                   "yoco_tiny", "--n-layers", "2", "--tiktoken-model", "byte", "--tokens-per-sample", "64",
                   "--batch-size", "2", "--pad-to-max-len", "--cpu", "--kernels", "torch"]) == 0
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert 0 < res["loss"] < 20 and res["ntokens"] > 0          # one finite pass over the valid split


def test_cli_keep_interval_updates(tmp_path, capsys):
    """--save-interval-updates 1 --keep-interval-updates 2: only the newest two interval checkpoints remain."""
    from faster_yoco_b200.cli import train as T
    data = str(tmp_path / "data")
    _corpus(data)
    save = str(tmp_path / "ckpt")
    assert T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                   "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead", "8",
                   "--log-interval", "2", "--warmup-updates", "2", "--save-dir", save, "--cpu", "--kernels", "torch",
                   "--max-update", "4", "--save-interval-updates", "1", "--keep-interval-updates", "2",
                   "--reset-meters"]) == 0
    kept = sorted(f for f in os.listdir(save) if f.startswith("checkpoint_1_"))
    assert kept == ["checkpoint_1_3.pt", "checkpoint_1_4.pt"], kept
    assert os.path.exists(os.path.join(save, "checkpoint_last.pt"))
