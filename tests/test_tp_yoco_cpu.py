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
