"""Per-kernel microbenchmarks: the sm_100a kernels against the library baselines (cuBLAS, flash-attn) on the
YOCO-3B shapes, timed with CUDA events after warm-up, inputs rotated through a pool larger than L2.

    python -m faster_yoco_b200.utils.kernel_bench [--only gemm|splits|fused|adam|staged|attn|ret] [--pair 1]
"""
from __future__ import annotations

import argparse
import json
import math

import torch

L2_BYTES = 126 * 1024 * 1024


def _time(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _pool(make, bytes_each):
    n = max(2, int(math.ceil(2 * L2_BYTES / max(bytes_each, 1))))
    n = min(n, 16)
    return [make() for _ in range(n)]


def gemm_shapes():
    T, d, f, V = 2048, 3072, 8192, 100288
    # (name, M, N, K, a_mn, b_mn): forward (x W^T), dgrad (dy W), wgrad (dy^T x)
    out = []
    for name, n_out, n_in in [("qkvg", 4 * d + 24, d), ("out_proj", d, d), ("fc1_gate", 2 * f, d), ("fc2", d, f),
                              ("kv_proj", 2048, d), ("output_proj", V, d)]:
        out.append((name + ".fwd", T, n_out, n_in, False, False))
        out.append((name + ".dgrad", T, n_in, n_out, False, True))
        out.append((name + ".wgrad", n_out, n_in, T, True, True))
    return out


def bench_gemm(results, pair_too: bool = False):
    """pair_too: also time the CTA-pair kernel (gemm2.cu) on every shape."""
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    for name, M, N, K, a_mn, b_mn in gemm_shapes():
        a_shape = (K, M) if a_mn else (M, K)
        b_shape = (K, N) if b_mn else (N, K)
        bytes_each = 2 * (M * K + N * K)
        pool = _pool(lambda: (torch.randn(a_shape, device=dev, dtype=torch.bfloat16),
                              torch.randn(b_shape, device=dev, dtype=torch.bfloat16)), bytes_each)
        c = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        it = [0]

        def ours():
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            ops._C().gemm(a, b, c, a_mn, b_mn, None)

        def pair(bn=256, splits=1):
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            ops._C().gemm_pair(a, b, c, a_mn, b_mn, None, bn, splits)

        def routed():
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            ops.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, out=c)

        def cublas():
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            A = a.T if a_mn else a
            B = b if b_mn else b.T
            torch.matmul(A, B, out=c)

        t_ours, t_cub = _time(ours), _time(cublas)
        fl = 2.0 * M * N * K
        r = {"kernel": "gemm", "shape": name, "M": M, "N": N, "K": K, "ours_ms": t_ours, "cublas_ms": t_cub,
             "ours_tflops": fl / t_ours / 1e9, "cublas_tflops": fl / t_cub / 1e9}
        if pair_too:
            t_pair = _time(pair)
            t_pair192 = _time(lambda: pair(192))
            r.update(pair_ms=t_pair, pair_tflops=fl / t_pair / 1e9, pair192_ms=t_pair192,
                     pair192_tflops=fl / t_pair192 / 1e9)
        t_routed = _time(routed)
        r.update(routed_ms=t_routed, routed_tflops=fl / t_routed / 1e9,
                 route=list(ops._gemm_route(M, N, K)))
        results.append(r)


def bench_gemm_splits(results):
    """The CTA-pair kernel's in-kernel split-K (1 .. 4 K parts per 256 x 256 tile, 0 = stream-K) on every YOCO-3B
    shape, next to the routed GEMM: the data behind the routing rule for shapes whose tiles fill the last round
    poorly."""
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    for name, M, N, K, a_mn, b_mn in gemm_shapes():
        a_shape = (K, M) if a_mn else (M, K)
        b_shape = (K, N) if b_mn else (N, K)
        pool = _pool(lambda: (torch.randn(a_shape, device=dev, dtype=torch.bfloat16),
                              torch.randn(b_shape, device=dev, dtype=torch.bfloat16)), 2 * (M * K + N * K))
        c = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        it = [0]

        def pair(splits):
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            ops._C().gemm_pair(a, b, c, a_mn, b_mn, None, 256, splits)

        def routed():
            a, b = pool[it[0] % len(pool)]
            it[0] += 1
            ops.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, out=c)

        nk = (K + 63) // 64
        r = {"kernel": "gemm_splits", "shape": name, "M": M, "N": N, "K": K, "routed_ms": _time(routed),
             "route": list(ops._gemm_route(M, N, K))}
        for sp in (0, 1, 2, 3, 4):         # 0: stream-K
            if sp == 0 or (sp - 1) * ((nk + sp - 1) // sp) < nk:
                r[f"pair_s{sp}_ms"] = _time(lambda: pair(sp))
        results.append(r)


def bench_gemm_fused(results):
    """The fused elementwise epilogues against the routed GEMM followed by the separate kernel, YOCO-3B shapes:
    RoPE on q / k in the retention layer's QKVG projection and on q in a cross layer's q projection, SwiGLU in the
    fc1 | gate projection, the SwiGLU backward in the fc2 input gradient."""
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    C = ops._C()
    T, L, d, f, H = 2048, 2048, 3072, 8192, 24
    ang = torch.rand(L, 64, device=dev) * 6.283
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    bf = dict(device=dev, dtype=torch.bfloat16)
    # training-scale operands: activations ~ N(0, 1), weights ~ N(0, 0.02), output gradients ~ 1e-3 (the
    # activation's cost depends on the value range, e.g. a sigmoid of |x| > 88 takes a slow reciprocal path)

    def wt(*shape):
        return (torch.randn(*shape, device=dev) * 0.02).to(torch.bfloat16)

    for name, N, rot in [("qkvg.fwd+rope", 4 * d + H, 2 * d), ("q_proj.fwd+rope", d, d)]:
        pool = _pool(lambda: (torch.randn(T, d, **bf), wt(N, d)), 2 * (T * d + N * d))
        y = torch.empty(T, N, **bf)
        it = [0]

        def fused():
            a, w = pool[it[0] % len(pool)]
            it[0] += 1
            ops.gemm_rope(a, w, cos, sin, L, rot, out=y)

        def separate():
            a, w = pool[it[0] % len(pool)]
            it[0] += 1
            ops.gemm(a, w, out=y)
            for c0 in range(0, rot, d):
                C.rope_fwd(y[:, c0:c0 + d].view(1, L, H, 128), cos, sin, False)

        tf, ts = _time(fused), _time(separate)
        results.append({"kernel": "gemm_fused", "shape": name, "fused_ms": tf, "separate_ms": ts,
                        "fused_tflops": 2.0 * T * N * d / tf / 1e9})
    # SwiGLU forward
    pool = _pool(lambda: (torch.randn(T, d, **bf), wt(2 * f, d)), 2 * (T * d + 2 * f * d))
    it = [0]

    def sw_fused():
        a, w = pool[it[0] % len(pool)]
        it[0] += 1
        ops.gemm_swiglu(a, w)

    def sw_separate():
        a, w = pool[it[0] % len(pool)]
        it[0] += 1
        u = ops.gemm(a, w)
        C.swiglu_fwd(u[:, :f], u[:, f:])

    tf, ts = _time(sw_fused), _time(sw_separate)
    results.append({"kernel": "gemm_fused", "shape": "fc1_gate.fwd+swiglu", "fused_ms": tf, "separate_ms": ts,
                    "fused_tflops": 2.0 * T * 2 * f * d / tf / 1e9})
    # SwiGLU backward in the fc2 input gradient
    pool = _pool(lambda: ((torch.randn(T, d, device=dev) * 1e-3).to(torch.bfloat16), wt(d, f),
                          torch.randn(T, 2 * f, **bf)),
                 2 * (T * d + d * f + 2 * T * f))
    du = torch.empty(T, 2 * f, **bf)

    def sb_fused():
        g, w2, u = pool[it[0] % len(pool)]
        it[0] += 1
        ops.gemm_swiglu_bwd(g, w2, u, du)

    def sb_separate():
        g, w2, u = pool[it[0] % len(pool)]
        it[0] += 1
        dh = ops.gemm(g, w2, b_mn_major=True)
        C.swiglu_bwd(u[:, :f], u[:, f:], dh, du[:, :f], du[:, f:])

    tf, ts = _time(sb_fused), _time(sb_separate)
    results.append({"kernel": "gemm_fused", "shape": "fc2.dgrad+swiglu_bwd", "fused_ms": tf, "separate_ms": ts,
                    "fused_tflops": 2.0 * T * f * d / tf / 1e9})


def bench_adam(results, n=1 << 30):
    """Adam (apex expression) + bf16 parameter copy over n elements (28 bytes each: fp32 master, m, v read + write,
    bf16 gradient read, bf16 parameter write), the 4-per-thread kernel and the 8-per-thread form (the Adam + push
    kernel with no peers); achieved bandwidth = algorithmic bytes / CUDA-event time."""
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    C = ops._C()
    p32 = torch.randn(n, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    g16 = torch.randn(n, device=dev, dtype=torch.bfloat16)
    p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
    hyper = torch.tensor([1e-4, 0.1, 0.05, 1.0], device=dev)
    factor = torch.tensor([1.0], device=dev)
    t4 = _time(lambda: C.adam_step(p32, g16, m, v, p16, hyper, factor, 0.9, 0.95, 1e-6, 0.05, True), iters=10,
               warmup=3)
    t8 = _time(lambda: C.adam_push(p32, g16, m, v, p16, hyper, factor, 0.9, 0.95, 1e-6, 0.05, True,
                                   [p16.data_ptr()], 0, 0, 0), iters=10, warmup=3)
    gb = 28.0 * n / 1e9
    results.append({"kernel": "adam", "n": n, "adam_ms": t4, "adam_tbs": gb / t4, "adam8_ms": t8,
                    "adam8_tbs": gb / t8})


def bench_staged(results, seg=1 << 25):
    """The owner's staged sum (ZeRO exchange with copy-engine gradient pushes): one owner's segment of `seg` bf16
    elements summed over its own gradient buffer and world - 1 staging slots in rank order, bf16 result written back,
    over a table of 26 bucket pieces; world ranks emulated in local memory. Achieved bandwidth = (world reads + one
    write) x 2 bytes x seg / CUDA-event time; inputs (>= 256 MB) exceed L2."""
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    C = ops._C()
    for world in (2, 4, 8):
        rank = 1
        grad = torch.randn(world * seg, device=dev).to(torch.bfloat16)
        staging = torch.randn(world * seg, device=dev).to(torch.bfloat16)
        cuts = [rank * seg + (seg * k // 26) // 64 * 64 for k in range(26)] + [(rank + 1) * seg]
        ranges = torch.tensor([[a, b - a] for a, b in zip(cuts, cuts[1:])], dtype=torch.int64, device=dev)
        gb = (world + 1) * 2.0 * seg / 1e9
        row = {"kernel": "reduce_staged", "world": world, "seg": seg}
        for ctas in (296, 444, 592):
            part = torch.zeros(ctas, device=dev)
            t = _time(lambda: C.reduce_staged(grad, staging, ranges, world, rank, seg, part, ctas, 0), iters=10,
                      warmup=3)
            row[f"ctas{ctas}_ms"] = t
            row[f"ctas{ctas}_tbs"] = gb / t
        results.append(row)
        del grad, staging


def bench_attention(results, L=2048, Hq=24, Hk=8, B=1):
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    ops.set_backend("native")
    q = torch.randn(B, L, Hq, 128, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, L, Hk, 128, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, L, Hk, 128, device=dev, dtype=torch.bfloat16)
    do = torch.randn_like(q)
    C = ops._C()
    sc = 128 ** -0.5
    o, lse = C.attention_fwd(q, k, v, True, 0, sc)
    t_f = _time(lambda: C.attention_fwd(q, k, v, True, 0, sc))
    t_b = _time(lambda: C.attention_bwd(do, q, k, v, o, lse, True, 0, sc))
    fl = 4.0 * B * Hq * L * L * 128 / 2
    r = {"kernel": "attention_causal_gqa", "L": L, "Hq": Hq, "Hk": Hk, "fwd_ms": t_f, "bwd_ms": t_b,
         "fwd_tflops": fl / t_f / 1e9, "bwd_tflops": 2.5 * fl / t_b / 1e9}
    try:
        from flash_attn import flash_attn_func
        qq, kk, vv = q.clone().requires_grad_(), k.clone().requires_grad_(), v.clone().requires_grad_()
        r["flash_attn_fwd_ms"] = _time(lambda: flash_attn_func(q, k, v, causal=True))
        oo = flash_attn_func(qq, kk, vv, causal=True)
        r["flash_attn_fwdbwd_ms"] = _time(lambda: torch.autograd.grad(flash_attn_func(qq, kk, vv, causal=True),
                                                                      (qq, kk, vv), do))
    except Exception as e:  # pragma: no cover
        r["flash_attn"] = repr(e)[:100]
    results.append(r)


def bench_retention(results, L=2048, H=24, B=1):
    from faster_yoco_b200 import ops
    dev = torch.device("cuda")
    q = torch.randn(B, L, H, 128, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, L, H, 128, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, L, H, 128, device=dev, dtype=torch.bfloat16)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, H, L, device=dev)) / 16).cumsum(-1).contiguous()
    do = torch.randn_like(q)
    C = ops._C()
    o = C.retention_fwd(q, k, v, g)
    t_f = _time(lambda: C.retention_fwd(q, k, v, g))
    t_b = _time(lambda: C.retention_bwd(do, q, k, v, g, o))
    fl = 4.0 * B * H * L * L * 128 / 2
    results.append({"kernel": "retention_parallel", "L": L, "H": H, "fwd_ms": t_f, "bwd_ms": t_b,
                    "fwd_tflops": fl / t_f / 1e9, "bwd_tflops": 2.5 * fl / t_b / 1e9})
    # chunkwise kernels (chunk 128): forward = the state outer products, the scan and the per-chunk outputs
    # (4 MMAs of 128^3 per chunk: K^T V, Q K^T, Q S, P V); backward = Q^T dO, the reverse scan and the per-chunk
    # gradients (8 MMAs per chunk) plus the gate row dots
    gl = C.retention_chunk_cumsum((torch.nn.functional.logsigmoid(torch.randn(B, H, L, device=dev)) / 16)
                                  .contiguous())
    o, states, _ = C.retention_chunk_fwd(q, k, v, gl)
    t_cf = _time(lambda: C.retention_chunk_fwd(q, k, v, gl))
    t_cb = _time(lambda: C.retention_chunk_bwd(do, q, k, v, gl, states, want_dgate=True))
    nc = (L + 127) // 128
    fl_f = 4 * 2.0 * 128 ** 3 * B * H * nc
    results.append({"kernel": "retention_chunk", "L": L, "H": H, "fwd_ms": t_cf, "bwd_ms": t_cb,
                    "fwd_tflops": fl_f / t_cf / 1e9, "bwd_tflops": 2 * fl_f / t_cb / 1e9,
                    "speedup_vs_parallel": (t_f + t_b) / (t_cf + t_cb)})


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--only", default=None)
    p.add_argument("--pair", type=int, default=0, help="GEMMs: also time the CTA-pair kernel")
    a = p.parse_args()
    res = []
    if a.only in (None, "gemm"):
        bench_gemm(res, pair_too=bool(a.pair))
    if a.only == "splits":
        bench_gemm_splits(res)
    if a.only == "adam":
        bench_adam(res)
    if a.only == "staged":
        bench_staged(res)
    if a.only in (None, "gemm", "fused"):
        bench_gemm_fused(res)
    if a.only in (None, "attn"):
        bench_attention(res)
    if a.only in (None, "ret"):
        bench_retention(res)
    for r in res:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
