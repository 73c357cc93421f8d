"""The CTA-pair GEMM (tcgen05.mma.cta_group::2, 256 x 256 tiles over two CTAs, gemm2.cu) against the one-CTA GEMM
and an fp32 PyTorch oracle: every operand layout (forward, input gradient, weight gradient), M / N / K tails, the
residual epilogue and fp32 output, 256-, 192- and 128-wide tiles, whole-K and two-way split-K (the later half's epilogue
adds the earlier half's partial), two calls in a row."""
import pytest
import torch

from faster_yoco_b200 import ops

pytestmark = pytest.mark.gpu


def _operands(M, N, K, a_mn, b_mn, g):
    dev = torch.device("cuda", 0)
    a = torch.randn((K, M) if a_mn else (M, K), generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), generator=g, device=dev).to(torch.bfloat16)
    return a, b


def _close_in_ulps(x, y, ulps, acc_mag=None):
    """|x - y| within `ulps` bf16 units in the last place of the larger magnitude (plus a small absolute floor).
    acc_mag: magnitude of the product before a residual was added (the residual epilogue rounds the product to
    bf16 first, so a one-unit flip there is measured in units of the product, not of the smaller sum)."""
    mag = torch.maximum(x.abs(), y.abs())
    if acc_mag is not None:
        mag = torch.maximum(mag, acc_mag)
    mag = mag.clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)        # bf16: 8 significant bits
    tol = ulps * ulp + 2e-2 if ulps else 1e-2 + 1e-3 * mag
    bad = (x - y).abs() > tol
    assert not bool(bad.any()), (int(bad.sum()), float((x - y).abs().max()))


@pytest.mark.parametrize("M,N,K,a_mn,b_mn", [
    (2048, 12312, 3072, False, False),     # q/k/v/g projection forward
    (2048, 3072, 16384, False, True),      # FFN input gradient
    (12312, 3072, 2048, True, True),       # q/k/v/g weight gradient
    (300, 520, 200, False, False),         # tails in M, N and K
    (520, 300, 136, True, False),
])
@pytest.mark.parametrize("epi", ["bf16", "res", "f32"])
@pytest.mark.parametrize("bn,splits", [(256, 1), (192, 1), (128, 1), (256, 2), (192, 2), (256, 3), (256, 4), (256, 0),
                                       (192, 0)])
def test_gemm_pair_matches_one_cta_and_fp32(M, N, K, a_mn, b_mn, epi, bn, splits):
    nk = (K + 63) // 64
    if splits and (splits - 1) * ((nk + splits - 1) // splits) >= nk:
        pytest.skip("a K part would be empty")
    C = ops._C()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a, b = _operands(M, N, K, a_mn, b_mn, g)
    dev = a.device
    dt = torch.float32 if epi == "f32" else torch.bfloat16
    res = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16) if epi == "res" else None
    one = torch.empty(M, N, dtype=dt, device=dev)
    C.gemm(a, b, one, a_mn, b_mn, res)
    A32 = (a.float().t() if a_mn else a.float())
    B32 = (b.float() if b_mn else b.float().t())
    prod = A32 @ B32
    first = None
    for _ in range(2):
        pair = torch.full((M, N), float("nan"), dtype=dt, device=dev)
        C.gemm_pair(a, b, pair, a_mn, b_mn, res, bn, splits)
        torch.cuda.synchronize()
        assert int(C.status()[0].item()) == 0
        assert not bool(torch.isnan(pair.float()).any()), "unwritten output"
        # same per-element K order in both kernels: equal up to the tensor cores' accumulation rounding, which can
        # move a bf16 output by one unit in the last place (two with the residual epilogue's second rounding)
        _close_in_ulps(pair.float(), one.float(), 2 if dt == torch.bfloat16 else 0, prod.abs())
        # split-K parts are summed in part order whatever order they finish in: runs are bitwise identical
        if first is not None:
            assert torch.equal(pair, first)
        first = pair
    ref = prod
    if res is not None:
        ref = ref + res.float()
    err = ((pair.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-2, err
