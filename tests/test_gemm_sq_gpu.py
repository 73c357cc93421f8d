"""Weight-gradient GEMM with the sum of squares of its stored bf16 output (the one-GPU gradient norm without a
second pass over the gradient buffer): against the plain GEMM and a PyTorch sum of squares, and one-GPU training
with and without it."""
import pytest
import torch

from faster_yoco_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,T", [(3072, 3072, 2048), (24, 3072, 2048), (12312, 3072, 2048), (200, 96, 256)])
@pytest.mark.parametrize("acc", [False, True])
def test_gemm_sq_output_and_partials(M, N, T, acc):
    C = ops._C()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + T)
    dy = torch.randn(T, M, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(T, N, generator=g, device=dev).to(torch.bfloat16)
    prev = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
    # the plain GEMM on the kernel the shape is routed to (gemm_sq takes the same route): identical stores
    want = ops.gemm(dy, x, a_mn_major=True, b_mn_major=True, residual=prev if acc else None)
    slots = C.gemm_sq_slots(M, N, T)
    part = torch.full((slots + 16,), 7.0, device=dev)
    for _ in range(2):
        out = prev.clone()
        n = C.gemm_sq(dy, x, out, acc, part)
        torch.cuda.synchronize()
        assert n == slots and int(C.status()[0].item()) == 0
        assert torch.equal(out, want)
        ref = want.float().pow(2).sum().item()
        assert abs(part[:n].sum().item() - ref) <= 1e-5 * ref
        assert bool((part[n:] == 7.0).all())                 # nothing written past the reported slots


@pytest.mark.parametrize("graph,tied", [(False, False), (True, False), (False, True)])
def test_one_gpu_training_norm_from_gemm_partials(graph, tied):
    """tied: the output projection shares the embedding weight, so one slot has two gradient producers (the
    output projection's GEMM, then the embedding backward); the GEMM's partials must then not be counted."""
    from faster_yoco_b200.utils import dist_checks
    ops.set_backend("native")
    dev = torch.device("cuda", 0)
    runs = {}
    for mode in ("pass", "gemm"):
        model, tr = dist_checks._tiny_trainer(dev, arch="yoco_small", dtype=torch.bfloat16, graph=graph,
                                              overlap=False, share_input_output_embed=tied)
        if mode == "gemm":
            tr.flat.enable_grad_sq()
        norms, losses = [], []
        for ids in dist_checks._batches(0, 1, 3, seq=256, vocab=8192):
            b = {"src_tokens": ids[0, :, :-1].contiguous(), "target": ids[0, :, 1:].contiguous(),
                 "ntokens": ids.shape[1] * (ids.shape[2] - 1), "nsentences": ids.shape[1]}
            losses.append(float(tr.train_step(b).item()))
            norms.append(float(tr.zero.last_grad_norm))
        tr.release_graph()
        runs[mode] = (losses, norms)
    for a, b in zip(runs["pass"][1], runs["gemm"][1]):
        assert abs(a - b) <= 1e-4 * abs(a), runs
    for a, b in zip(runs["pass"][0], runs["gemm"][0]):
        assert abs(a - b) <= 2e-4 * abs(a), runs


def test_adam_eight_wide_matches_adam():
    """The 8-wide Adam (the Adam + push kernel with no peers; default for contiguous owner maps) gives the same
    parameters as the 4-wide kernel."""
    from faster_yoco_b200.utils import dist_checks
    ops.set_backend("native")
    dev = torch.device("cuda", 0)
    out = {}
    for wide in (False, True):
        model, tr = dist_checks._tiny_trainer(dev, arch="yoco_small", dtype=torch.bfloat16, overlap=False)
        tr.zero.adam8 = wide
        for ids in dist_checks._batches(0, 1, 2, seq=256, vocab=8192):
            b = {"src_tokens": ids[0, :, :-1].contiguous(), "target": ids[0, :, 1:].contiguous(),
                 "ntokens": ids.shape[1] * (ids.shape[2] - 1), "nsentences": ids.shape[1]}
            tr.train_step(b)
        torch.cuda.synchronize()
        out[wide] = (tr.zero.master.clone(), tr.flat.flat.clone())
    # identical expression per element; only the attention dQ atomics' order differs between runs
    assert torch.allclose(out[False][0], out[True][0], rtol=1e-3, atol=1e-5)
