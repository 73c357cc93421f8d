"""Small, self-terminating launches of the hot kernels for `ncu` captures (a few MB on the device, a handful of
launches each). Used as:  ncu --set full --clock-control none -k regex:<kernel> -s <n> -c <m> \\
    python -m faster_yoco_b200.utils.profile_kernels --what <case>

cases: attn, attn_bwd, swa, swa_bwd (sliding window 1024), ret, ret_bwd (parallel form), ret_chunk,
ret_chunk_bwd (chunkwise kernels), gemm, gemm_dgrad, gemm_scatter (weight
gradient stored at 4 emulated owners, block-cyclic map), adam, ce, ce_bwd, rms, rms_bwd, subln, subln_bwd, swiglu,
swiglu_bwd, rope, embed, embed_bwd, reduce_compact, reduce_owner, adam_push (eight ranks emulated in local memory),
reduce_staged (four ranks emulated),
gate_cumsum (chunk-local), gemm_pair, gemm_pair128, gemm_swiglu, gemm_swiglu_bwd (fused epilogues), gemm_pair_sk / gemm_pair_s1 (stream-K vs one part).
"""
import argparse

import torch


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--what", default="attn")
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--L", type=int, default=2048)
    a = p.parse_args()
    from faster_yoco_b200 import ops
    C = ops._C()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    L = a.L
    if a.what in ("swa", "swa_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        o, lse = C.attention_fwd(q, k, v, True, 1024, 128 ** -0.5)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "swa":
                C.attention_fwd(q, k, v, True, 1024, 128 ** -0.5)
            else:
                C.attention_bwd(do, q, k, v, o, lse, True, 1024, 128 ** -0.5)
    elif a.what in ("attn", "attn_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 8, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 8, 128, device=dev, dtype=torch.bfloat16)
        o, lse = C.attention_fwd(q, k, v, True, 0, 128 ** -0.5)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "attn":
                C.attention_fwd(q, k, v, True, 0, 128 ** -0.5)
            else:
                C.attention_bwd(do, q, k, v, o, lse, True, 0, 128 ** -0.5)
    elif a.what in ("ret", "ret_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        g = (torch.nn.functional.logsigmoid(torch.randn(1, 24, L, device=dev)) / 16).cumsum(-1).contiguous()
        o = C.retention_fwd(q, k, v, g)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "ret":
                C.retention_fwd(q, k, v, g)
            else:
                C.retention_bwd(do, q, k, v, g, o)
    elif a.what in ("ret_chunk", "ret_chunk_bwd"):
        q = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        gl = C.retention_chunk_cumsum((torch.nn.functional.logsigmoid(torch.randn(1, 24, L, device=dev)) / 16)
                                      .contiguous())
        o, states, _ = C.retention_chunk_fwd(q, k, v, gl)
        do = torch.randn_like(o)
        for _ in range(a.reps):
            if a.what == "ret_chunk":
                C.retention_chunk_fwd(q, k, v, gl)
            else:
                C.retention_chunk_bwd(do, q, k, v, gl, states, want_dgate=True)
    elif a.what == "gemm":
        x = torch.randn(2048, 3072, device=dev, dtype=torch.bfloat16)
        w = torch.randn(12312, 3072, device=dev, dtype=torch.bfloat16)
        y = torch.empty(2048, 12312, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gemm(x, w, y, False, False, None)
    elif a.what == "gemm_dgrad":
        dy = torch.randn(2048, 16384, device=dev, dtype=torch.bfloat16)
        w = torch.randn(16384, 3072, device=dev, dtype=torch.bfloat16)
        y = torch.empty(2048, 3072, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gemm(dy, w, y, False, True, None)
    elif a.what == "adam":
        # a quarter of one rank's ZeRO segment at 8 GPUs (1.7 GB in total, well above L2)
        n = 107_665_728
        p32 = torch.randn(n, device=dev)
        m = torch.zeros(n, device=dev)
        v = torch.zeros(n, device=dev)
        g16 = torch.randn(n, device=dev, dtype=torch.bfloat16)
        p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
        hyper = torch.tensor([1e-4, 0.1, 0.05, 0.0], device=dev)
        factor = torch.tensor([1.0], device=dev)
        for _ in range(a.reps):
            C.adam_step(p32, g16, m, v, p16, hyper, factor, 0.9, 0.95, 1e-6, 0.05, True)
    elif a.what in ("ce", "ce_bwd"):
        x = (torch.randn(L, 100288, device=dev) * 2).to(torch.bfloat16)
        t = torch.randint(0, 100288, (L,), device=dev)
        loss, lse = C.ce_fwd(x, t, 1)
        g = torch.ones(1, device=dev)
        out = torch.empty_like(x)
        for _ in range(a.reps):
            if a.what == "ce":
                C.ce_fwd(x, t, 1)
            else:
                C.ce_bwd(x, t, lse, g, 1, out)
    elif a.what in ("rms", "rms_bwd"):
        x = torch.randn(L, 3072, device=dev, dtype=torch.bfloat16)
        w = torch.ones(3072, device=dev, dtype=torch.bfloat16)
        y, rstd = C.rms_norm_fwd(x, w, 1e-5)
        for _ in range(a.reps):
            if a.what == "rms":
                C.rms_norm_fwd(x, w, 1e-5)
            else:
                C.rms_norm_bwd(y, x, w, rstd)
    elif a.what in ("subln", "subln_bwd"):
        o = torch.randn(L, 3072, device=dev, dtype=torch.bfloat16)
        g = torch.randn(L, 3072, device=dev, dtype=torch.bfloat16)
        out, rstd = C.subln_swiglu_fwd(o, g, 1e-6, 128)
        dout = torch.randn_like(out)
        for _ in range(a.reps):
            if a.what == "subln":
                C.subln_swiglu_fwd(o, g, 1e-6, 128)
            else:
                C.subln_swiglu_bwd(dout, o, g, rstd, 128)
    elif a.what in ("swiglu", "swiglu_bwd"):
        u = torch.randn(L, 16384, device=dev, dtype=torch.bfloat16)
        x, y = u[:, :8192], u[:, 8192:]
        da = torch.randn(L, 8192, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            if a.what == "swiglu":
                C.swiglu_fwd(x, y)
            else:
                C.swiglu_bwd(x, y, da)
    elif a.what == "rope":
        from faster_yoco_b200.ops import reference as ref
        x = torch.randn(1, L, 24, 128, device=dev, dtype=torch.bfloat16)
        cos, sin = ref.rope_tables(128, 0, L, 1e4, torch.bfloat16, dev)
        for _ in range(a.reps):
            C.rope_fwd(x, cos, sin, False)
    elif a.what in ("embed", "embed_bwd"):
        w = torch.randn(100288, 3072, device=dev, dtype=torch.bfloat16)
        tok = torch.randint(0, 100288, (L,), device=dev)
        dy = torch.randn(L, 3072, device=dev, dtype=torch.bfloat16)
        dw = torch.empty_like(w)
        for _ in range(a.reps):
            if a.what == "embed":
                C.embedding_fwd(tok, w, 3072 ** 0.5)
            else:
                C.embedding_bwd(tok, dy, 100288, 3072 ** 0.5, dw)
    elif a.what in ("gemm_scatter", "reduce_compact"):
        # four owners emulated in this GPU's memory (the kernels only see addresses); block-cyclic map
        world, rank, chunk = 4, 1, 1 << 18
        M, N, T = 12312, 3072, 2048
        seg = -(-(M * N) // (world * chunk)) * chunk
        grad = torch.zeros(world * seg, device=dev, dtype=torch.bfloat16)
        staging = [torch.zeros(world * seg, device=dev, dtype=torch.bfloat16) for _ in range(world)]
        bases = torch.tensor([t.data_ptr() for t in staging], dtype=torch.int64, device=dev)
        dy = torch.randn(T, M, device=dev, dtype=torch.bfloat16)
        x = torch.randn(T, N, device=dev, dtype=torch.bfloat16)
        slot = grad[:M * N].view(M, N)
        part = torch.zeros(296, device=dev)
        for _ in range(a.reps):
            if a.what == "gemm_scatter":
                C.gemm_scatter(dy, x, slot, False, grad, bases, seg, rank, chunk)
            else:
                C.reduce_compact(grad, staging[rank], seg, world, rank, seg, chunk, part, 296)
    elif a.what in ("reduce_owner", "adam_push"):
        # eight ranks emulated in this GPU's memory (the kernels only see addresses), contiguous owner segments:
        # rank 2's reduce-to-owner of a 16 Mi-element segment over 8 gradient buffers (fp32 rank-order sum), and
        # its Adam step fused with the push of the new bf16 values into the 8 parameter buffers
        world, rank, seg = 8, 2, 1 << 24
        n = world * seg
        if a.what == "reduce_owner":
            grads = [torch.randn(n, device=dev).to(torch.bfloat16) for _ in range(world)]
            ptrs = [t.data_ptr() for t in grads]
            part = torch.zeros(296, device=dev)
            sq = torch.zeros(1, device=dev)
            for _ in range(a.reps):
                C.reduce_owner(ptrs, grads[rank], rank * seg, seg, part, sq, 0, rank)
        else:
            p32 = torch.randn(seg, device=dev)
            m = torch.zeros(seg, device=dev)
            v = torch.zeros(seg, device=dev)
            g16 = torch.randn(seg, device=dev).to(torch.bfloat16)
            pb = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for _ in range(world)]
            hyper = torch.tensor([1e-4, 0.1, 0.001, 1.0], device=dev)
            factor = torch.tensor([1.0], device=dev)
            for _ in range(a.reps):
                C.adam_push(p32, g16, m, v, pb[rank][rank * seg:(rank + 1) * seg], hyper, factor, 0.9, 0.95, 1e-6,
                            0.05, True, [t.data_ptr() for t in pb], rank * seg, rank, 0)
    elif a.what == "reduce_staged":
        # four ranks emulated in this GPU's memory: rank 1's owner-side sum after the copy engines delivered the
        # other ranks' gradient pieces into its staging slots (the 4-GPU default exchange), over a 32 Mi-element
        # segment cut into 26 bucket pieces as in the training step
        world, rank, seg = 4, 1, 1 << 25
        grad = torch.randn(world * seg, device=dev).to(torch.bfloat16)
        staging = torch.randn(world * seg, device=dev).to(torch.bfloat16)
        cuts = [rank * seg + (seg * k // 26) // 64 * 64 for k in range(26)] + [(rank + 1) * seg]
        ranges = torch.tensor([[a0, b0 - a0] for a0, b0 in zip(cuts, cuts[1:])], dtype=torch.int64, device=dev)
        part = torch.zeros(444, device=dev)
        for _ in range(a.reps):
            C.reduce_staged(grad, staging, ranges, world, rank, seg, part, 444, 0)
    elif a.what == "gate_cumsum":
        y = torch.randn(2048, 12312, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gate_cumsum_fwd(y[:, 4 * 3072:4 * 3072 + 24], 1, 2048, 16.0, True)
    elif a.what in ("gemm_pair", "gemm_pair128", "gemm_swiglu"):
        # the fc1 | gate projection at training scale (activations ~ N(0, 1), weights ~ N(0, 0.02))
        x = torch.randn(2048, 3072, device=dev, dtype=torch.bfloat16)
        w = (torch.randn(16384, 3072, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(2048, 16384, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            if a.what == "gemm_swiglu":
                C.gemm_swiglu(x, w)
            else:
                C.gemm_pair(x, w, y, False, False, None, 128 if a.what == "gemm_pair128" else 256)
    elif a.what in ("gemm_pair_sk", "gemm_pair_s1"):
        # a 3,072-wide output (96 pair tiles on 74 CTA pairs): stream-K vs one K part per tile
        x = torch.randn(2048, 3072, device=dev, dtype=torch.bfloat16)
        w = (torch.randn(3072, 3072, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(2048, 3072, device=dev, dtype=torch.bfloat16)
        for _ in range(a.reps):
            C.gemm_pair(x, w, y, False, False, None, 256, 0 if a.what == "gemm_pair_sk" else 1)
    elif a.what == "gemm_swiglu_bwd":
        g = (torch.randn(2048, 3072, device=dev) * 1e-3).to(torch.bfloat16)
        w2 = (torch.randn(3072, 8192, device=dev) * 0.02).to(torch.bfloat16)
        u = torch.randn(2048, 16384, device=dev, dtype=torch.bfloat16)
        du = torch.empty_like(u)
        for _ in range(a.reps):
            C.gemm_swiglu_bwd(g, w2, True, u, du)
    else:
        raise SystemExit(f"unknown --what {a.what}")
    torch.cuda.synchronize()
    st = int(C.status()[0].item())
    if st != 0:
        raise SystemExit(f"device status {st:#x}")


if __name__ == "__main__":
    main()
