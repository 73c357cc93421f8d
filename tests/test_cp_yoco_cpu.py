"""Context-parallel YOCO on 2 gloo ranks: each rank holds half of every sequence; the summed loss and the summed
parameter gradients equal those of the whole sequence on one process (retention state carried across blocks,
shared K / V and sliding-window K / V gathered along the sequence)."""
import pytest
import torch
import torch.distributed as dist

from faster_yoco_b200 import ops
from faster_yoco_b200.config import build_args
from faster_yoco_b200.utils.launch import run_ranks

NAMES = ["self_decoder.layers.0.mixer", "cross_decoder.layers.0.mixer.q_proj.weight", "embed_tokens.weight",
         "cross_decoder.kv_proj.weight"]


def _args(window):
    return build_args("yoco_tiny", n_layers=2, max_seq_len=128, max_batch_size=2, sliding_window=window)


def _grads(m):
    out = {}
    for n, p in m.named_parameters():
        if any(n.startswith(k) for k in NAMES):
            out[n] = p.grad.detach().clone()
    return out


def _worker(rank, world, sd, ids, ref_loss, ref_grads, window):
    from faster_yoco_b200.models.yoco import YOCO
    from faster_yoco_b200.parallel import context as CP
    ops.set_backend("torch")
    CP.init_context_parallel(world)
    m = YOCO(_args(window))
    m.load_state_dict(sd)
    L = (ids.shape[1] - 1) // world
    src = ids[:, :-1][:, rank * L:(rank + 1) * L]
    tgt = ids[:, 1:][:, rank * L:(rank + 1) * L]
    logits, _ = m(src)
    loss = ops.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1), 1)
    loss.backward()
    tot = loss.detach().clone()
    dist.all_reduce(tot)
    assert abs(float(tot) - ref_loss) < 1e-5 * abs(ref_loss), (float(tot), ref_loss)
    g = _grads(m)
    for n, ref in ref_grads.items():
        t = g[n].clone()
        dist.all_reduce(t)
        torch.testing.assert_close(t, ref, atol=2e-5, rtol=2e-3, msg=n)
    CP.destroy_context_parallel()


@pytest.mark.parametrize("window", [None, 24])
def test_cp2_matches_full_sequence(window):
    from faster_yoco_b200.models.yoco import YOCO
    ops.set_backend("torch")
    torch.manual_seed(0)
    m = YOCO(_args(window))
    ids = torch.randint(2, 1024, (2, 65))
    logits, _ = m(ids[:, :-1])
    loss = ops.cross_entropy(logits.reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1), 1)
    loss.backward()
    sd = {k: v.detach().clone() for k, v in m.state_dict().items()}
    run_ranks(_worker, 2, sd, ids, float(loss), _grads(m), window)


def _cli_worker(rank, world, data, save, cp, out_dir):
    from faster_yoco_b200.cli import train as T
    import io, contextlib
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                     "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead", "4",
                     "--log-interval", "2", "--warmup-updates", "1", "--max-update", "2", "--save-dir", save,
                     "--cpu", "--kernels", "torch", "--context-parallel-size", str(cp), "--seed", "3"])
    assert rc == 0
    if rank == 0:
        open(out_dir, "w").write(buf.getvalue())
    from faster_yoco_b200.parallel import context as CP
    CP.destroy_context_parallel()


def test_cli_context_parallel_matches_single_rank(tmp_path):
    """The same 2 updates through the train CLI: one rank with whole sequences, and 2 context-parallel ranks."""
    import json, os
    from faster_yoco_b200.cli import train as T
    data = str(tmp_path / "data")
    os.makedirs(os.path.join(data, "json"))
    os.makedirs(os.path.join(data, "shard", "w"))
    with open(os.path.join(data, "shard", "w", "00000.jsonl"), "w") as f:
        for d in range(40):
            f.write(json.dumps({"text": f"doc {d}: a few words to pack\n\nmore words"}) + "\n")
    json.dump(["shard/w/00000.jsonl"], open(os.path.join(data, "json", "w.json"), "w"))
    json.dump([{"name": "w", "weight": 1.0}], open(os.path.join(data, "json", "train.json"), "w"))
    import io, contextlib
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        assert T.main([data, "--arch", "yoco_tiny", "--n-layers", "2", "--task", "gpt", "--tiktoken-model", "byte",
                       "--tokens-per-sample", "64", "--batch-size", "2", "--pad-to-max-len", "--batch-read-ahead",
                       "4", "--log-interval", "2", "--warmup-updates", "1", "--max-update", "2",
                       "--save-dir", str(tmp_path / "s1"), "--cpu", "--kernels", "torch", "--seed", "3"]) == 0
    single = [l for l in buf.getvalue().splitlines() if l.startswith("epoch")][-1]
    out = str(tmp_path / "cp.log")
    run_ranks(_cli_worker, 2, data, str(tmp_path / "s2"), 2, out)
    cpline = [l for l in open(out).read().splitlines() if l.startswith("epoch")][-1]
    loss = lambda l: float(l.split("loss ")[1].split(" ")[0])
    gn = lambda l: float(l.split("gnorm ")[1].split(" ")[0])
    assert abs(loss(single) - loss(cpline)) < 2e-3 and abs(gn(single) - gn(cpline)) < 2e-3 * max(1.0, gn(single))
    s1 = torch.load(str(tmp_path / "s1" / "checkpoint_last.pt"), weights_only=False)["model"]
    s2 = torch.load(str(tmp_path / "s2" / "checkpoint_last.pt"), weights_only=False)["model"]
    for k in ("decoder.model.embed_tokens.weight", "decoder.model.self_decoder.layers.0.mixer.q_proj.weight"):
        torch.testing.assert_close(s1[k], s2[k], atol=1e-5, rtol=1e-4)
