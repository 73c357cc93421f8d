"""The fused whole-layer autograd Functions (native training path) against the op-by-op module path on the same
weights: outputs and every parameter gradient."""
import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.config import build_args
from faster_yoco_b200.models.yoco import YOCO

pytestmark = pytest.mark.gpu


def rel(x, r):
    x, r = x.float(), r.float()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("gemm_fuse", [True, False])
@pytest.mark.parametrize("window", [None, 96])
def test_fused_layers_match_module_path(window, gemm_fuse, monkeypatch):
    """gemm_fuse: RoPE / SwiGLU in the GEMM epilogues (default) or as separate kernels."""
    old_fuse = ops.GEMM_FUSE
    ops.GEMM_FUSE = gemm_fuse
    try:
        _check_fused_layers(window, monkeypatch)
    finally:
        ops.GEMM_FUSE = old_fuse


def _check_fused_layers(window, monkeypatch):
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    args = build_args("yoco_small", max_seq_len=384, init_std=0.02, sliding_window=window)
    with torch.device(dev):
        model = YOCO(args)
    model = model.to(torch.bfloat16).train()
    x = torch.randint(0, args.vocab_size, (2, 384), device=dev)
    ops.set_backend("native")

    def run(fused):
        from faster_yoco_b200.models import fused as F
        if not fused:
            monkeypatch.setattr(F, "fused_path_ok", lambda *a, **k: False)
        else:
            monkeypatch.undo()
        model.zero_grad(set_to_none=True)
        logits, _ = model(x)
        loss = ops.cross_entropy(logits.view(-1, logits.shape[-1]), x.view(-1), 1)
        loss.backward()
        return logits.detach().clone(), {n: p.grad.detach().clone() for n, p in model.named_parameters()}

    l_mod, g_mod = run(False)
    l_fus, g_fus = run(True)
    assert rel(l_fus, l_mod) < 2e-2
    for n in g_mod:
        assert rel(g_fus[n], g_mod[n]) < 5e-2, n
