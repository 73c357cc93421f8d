"""GEMM-fused ZeRO reduce-scatter on the GPU: the weight-gradient GEMM whose epilogue stores every element at its
owner, against the plain GEMM + the host-side oracle of where each element goes (one GPU, four ranks' staging
buffers emulated in local memory: the kernel only sees addresses), and 2-GPU training against the serial exchange.

Marked ``gpu_pending``: this path has not yet run on a GPU, so ``-m gpu`` does not select it; run it with
``-m gpu_pending``."""
import math
import os

import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.ops import reference as ref

pytestmark = pytest.mark.gpu_pending


@pytest.mark.parametrize("M,N,T,acc", [(200, 96, 256, False), (200, 96, 256, True), (128, 128, 8192, False),
                                       (128, 128, 8192, True), (1024, 3072, 2048, False), (24, 3072, 2048, True)])
def test_gemm_scatter_stores_at_owners(M, N, T, acc):
    ops.set_backend("native")
    C = ops._C()
    dev = torch.device("cuda", 0)
    world, rank, x0 = 4, 1, 3000
    numel = M * N
    seg = int(math.ceil((x0 + numel) / 3 / 1024)) * 1024          # the slot spans owners 0, 1 and 2
    g = torch.Generator(device=dev).manual_seed(M + N + T)
    grad_flat = torch.randn(world * seg, generator=g, device=dev).to(torch.bfloat16)
    staging = [torch.zeros(world * seg, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    bases = torch.tensor([t.data_ptr() for t in staging], dtype=torch.int64, device=dev)
    dy = torch.randn(T, M, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(T, N, generator=g, device=dev).to(torch.bfloat16)
    slot = grad_flat[x0:x0 + numel].view(M, N)
    prev = slot.clone()
    want = ops.gemm(dy, x, a_mn_major=True, b_mn_major=True, out=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
                    residual=prev if acc else None)
    own_exp = grad_flat.clone()
    stag_exp = [t.clone() for t in staging]
    ref.owner_scatter(want, x0, seg, rank, own_exp, stag_exp)
    for _ in range(2):                                             # a second call stores the same values
        if acc:
            slot.copy_(prev)
        C.gemm_scatter(dy, x, slot, acc, grad_flat, bases, seg, rank)
        torch.cuda.synchronize()
        # this rank's buffer changes only where it owns the slot (elsewhere the slot keeps its earlier contents,
        # which with accumulation are the earlier micro-batches' sums)
        assert torch.equal(grad_flat, own_exp)
        for q in range(world):
            assert torch.equal(staging[q], stag_exp[q]), q
    assert int(C.status()[0].item()) == 0
    # and the GEMM itself against fp32
    r = dy.float().t() @ x.float() + (prev.float() if acc else 0)
    assert ((want.float() - r).abs().max() / r.abs().max()).item() < 2e-2


@pytest.mark.multigpu
def test_gemm_scatter_training_matches_serial_exchange(tmp_path):
    from faster_yoco_b200.utils import dist_checks
    from faster_yoco_b200.utils.launch import run_ranks
    run_ranks(dist_checks.gemm_scatter_vs_serial_gpu, 2, str(tmp_path), 4, backend="nccl", timeout_s=300)
    r = torch.load(os.path.join(tmp_path, "gemm_scatter.pt"))
    for name, base in (("gemm", "serial"), ("gemm_graph", "serial"), ("gemm_uf2", "serial_uf2")):
        assert r[name]["status"] == 0 and r[base]["status"] == 0
        for a, b in zip(r[name]["losses"], r[base]["losses"]):
            assert abs(a - b) / abs(b) < 2e-4, (name, r[name]["losses"], r[base]["losses"])
        pf, ps = r[name]["params"], r[base]["params"]
        assert ((pf - ps).abs().max() / ps.abs().max()).item() < 1e-2, name
