"""Fused-path microbenchmark (one rank per GPU, launched with torch.distributed.run):

* parameter all-gather: NCCL all_gather_into_tensor vs the peer-memory pull (gather_segments) and push
  (push_range) kernels, per-rank message sizes 1 MB .. 1 GB;
* copy-engine push all-gather (one cudaMemcpyAsync per peer on per-peer streams), and how much a GEMM chain slows
  down while the copy engines push (the question for overlapping the exchange with compute);
* gradient reduce-scatter: NCCL reduce_scatter_tensor (AVG, bf16) vs the owner-side FP32 rank-order reduction over
  NVLink (reduce_owner, with the grad-norm partial);
* ``--fused-gemm 1``: the GEMM fused with the reduce-scatter -- the q/k/v/g weight gradient dW = dy^T x
  ([2048 x 12312]^T [2048 x 3072]) stored by the GEMM's epilogue at each element's owner (block-cyclic owner map)
  and summed by the owner from local memory -- against GEMM + NCCL reduce-scatter and GEMM + P2P reduce-to-owner;
  roofline = max(FLOPs / measured bf16 peak, bytes this rank sends over NVLink / 770 GB/s);
* ``--fused-gather 1``: all-gather -> GEMM of a forward weight (1 MB .. 1 GB): the all-gather fused into the
  consumer GEMM (gemm_gather) against NCCL all_gather_into_tensor + GEMM;
* ``--fused-adam 1``: reduce-scatter + sharded Adam + parameter all-gather over per-rank segments of 1 MB .. 1 GB
  (gradients N(0, 1e-3)): P2P reduce-to-owner + Adam fused with the push all-gather, against NCCL reduce-scatter +
  Adam + NCCL all-gather; roofline = max(inbound NVLink bytes / 770 GB/s, Adam's HBM bytes / measured HBM bandwidth).

Each point is timed with CUDA events on the launching stream after warm-up, max over ranks; bandwidth is the bytes
this rank receives ((world-1)/world of the gathered / reduced buffer) per second, and `frac` is that over the
measured 770 GB/s per-direction NVLink peer-copy bandwidth of this pool.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

LINK_GBS = 770.0
BF16_TFLOPS = 1661.4      # measured cuBLAS bf16 burst throughput of this pool's B200s
HBM_GBS = 6529.1          # measured copy bandwidth of this pool's B200s


def _time(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,8,64,256,1024")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--ctas", default="64,148,296")
    ap.add_argument("--interference", type=int, default=1)
    ap.add_argument("--fused-gemm", type=int, default=0)
    ap.add_argument("--fused-adam", type=int, default=0)
    ap.add_argument("--fused-gather", type=int, default=0)
    ap.add_argument("--skip-sweep", type=int, default=0, help="only the --fused-* sections")
    a = ap.parse_args()
    from faster_yoco_b200.parallel import dist as D
    from faster_yoco_b200.parallel.p2p import PeerComm
    D.init()
    rank, world = dist.get_rank(), dist.get_world_size()
    comm = PeerComm()
    maxmb = max(int(x) for x in a.sizes_mb.split(","))
    seg_max = maxmb * 1024 * 1024 // 2
    flat = comm.alloc("param", world * seg_max, torch.bfloat16)
    grad = comm.alloc("grad", world * seg_max, torch.bfloat16)
    flat.normal_()
    grad.normal_()
    C = comm.C
    if a.fused_gemm:
        fused_gemm_bench(comm, a.iters)
    if a.fused_adam:
        fused_adam_bench(comm, [int(x) for x in a.sizes_mb.split(",")], a.iters)
    if a.fused_gather:
        fused_gather_bench(comm, [int(x) for x in a.sizes_mb.split(",")], a.iters)
    if a.skip_sweep:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        return
    for mb in (int(x) for x in a.sizes_mb.split(",")):
        seg = mb * 1024 * 1024 // 2
        recv_gb = (world - 1) * seg * 2 / 1e9
        f = flat[: world * seg]
        res = {"size_mb_per_rank": mb, "world": world}
        res["nccl_allgather_ms"] = _time(lambda: dist.all_gather_into_tensor(f, f[rank * seg:(rank + 1) * seg]),
                                         a.iters)
        segs = torch.tensor([[q * seg, seg, q] for q in range(world) if q != rank], dtype=torch.int64,
                            device="cuda").view(-1, 3)
        for ctas in (int(x) for x in a.ctas.split(",")):
            res[f"pull_allgather_ms_c{ctas}"] = _time(
                lambda: (comm.barrier(), C.gather_segments(comm.peers["param"], f, segs, rank, ctas)), a.iters)
            res[f"push_allgather_ms_c{ctas}"] = _time(
                lambda: (C.push_range(f, comm.peers["param"], rank * seg, seg, rank, ctas), comm.barrier()), a.iters)
        # copy-engine push: one cudaMemcpyAsync per peer, each on its own stream
        streams = [torch.cuda.Stream() for _ in range(world)]
        esz = 2

        def ce_push(chunks=1):
            cur = torch.cuda.current_stream()
            ev = torch.cuda.Event()
            ev.record(cur)
            step = (seg + chunks - 1) // chunks
            for q in range(world):
                if q == rank:
                    continue
                with torch.cuda.stream(streams[q]):
                    streams[q].wait_event(ev)
                    for c0 in range(0, seg, step):
                        n = min(step, seg - c0)
                        off = (rank * seg + c0) * esz
                        C.peer_copy(comm.peers["param"][q] + off, f.data_ptr() + off, n * esz)
            for q in range(world):
                if q != rank:
                    cur.wait_stream(streams[q])
            comm.barrier()

        res["ce_push_allgather_ms"] = _time(lambda: ce_push(1), a.iters)
        res["ce_push4_allgather_ms"] = _time(lambda: ce_push(4), a.iters)
        g = grad[: world * seg]
        out = torch.empty(seg, dtype=torch.bfloat16, device="cuda")
        res["nccl_reducescatter_ms"] = _time(
            lambda: dist.reduce_scatter_tensor(out, g, op=dist.ReduceOp.AVG), a.iters)
        part = torch.zeros(1024, device="cuda")
        sq = torch.zeros(1, device="cuda")
        res["p2p_reduce_owner_ms"] = _time(
            lambda: comm.reduce_to_owner(g, seg), a.iters)
        for k in list(res):
            if k.endswith("_ms") or "_ms_c" in k:
                res[k.replace("_ms", "_gbs")] = recv_gb / (res[k] / 1e3)
                res[k.replace("_ms", "_frac")] = res[k.replace("_ms", "_gbs")] / LINK_GBS
        if rank == 0:
            print(json.dumps(res), flush=True)
    # interference: a GEMM chain alone vs while the copy engines push 1 GB to every peer
    if a.interference:
        x = torch.randn(2048, 3072, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(16384, 3072, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(2048, 16384, device="cuda", dtype=torch.bfloat16)

        def gemms():
            for _ in range(40):
                C.gemm(x, w, y, False, False, None)
        seg = min(seg_max, 512 * 1024 * 1024)
        f = flat[: world * seg]
        side = [torch.cuda.Stream() for _ in range(world)]

        def pushes():
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
            for q in range(world):
                if q != rank:
                    with torch.cuda.stream(side[q]):
                        side[q].wait_event(ev)
                        off = rank * seg * 2
                        C.peer_copy(comm.peers["param"][q] + off, f.data_ptr() + off, seg * 2)

        def join():
            for q in range(world):
                if q != rank:
                    torch.cuda.current_stream().wait_stream(side[q])

        alone = _time(gemms, 3)
        both = _time(lambda: (pushes(), gemms(), join()), 3)
        push_only = _time(lambda: (pushes(), join()), 3)
        if rank == 0:
            print(json.dumps({"interference": True, "gemm_chain_ms": alone, "gemm_chain_with_ce_push_ms": both,
                              "ce_push_only_ms": push_only, "push_gb_per_rank": (world - 1) * seg * 2 / 1e9}),
                  flush=True)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


def fused_gemm_bench(comm, iters, T=2048, M=12312, N=3072, chunk=1 << 18):
    """GEMM -> reduce-scatter of the q/k/v/g weight gradient: fused (owner-scatter epilogue + local owner sum) vs
    GEMM then NCCL reduce-scatter vs GEMM then the P2P reduce-to-owner."""
    C = comm.C
    rank, world = comm.rank, comm.world
    numel = M * N
    span = chunk * world
    seg = -(-numel // span) * chunk                         # whole chunks per owner
    grad = comm.alloc("fg_grad", world * seg, torch.bfloat16)
    staging = comm.alloc("fg_staging", world * seg, torch.bfloat16)
    bases = torch.tensor(comm.peers["fg_staging"], dtype=torch.int64, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(rank)
    dy = torch.randn(T, M, generator=g, device="cuda").to(torch.bfloat16)
    x = torch.randn(T, N, generator=g, device="cuda").to(torch.bfloat16)
    slot = grad[:numel].view(M, N)
    part = torch.zeros(296, device="cuda")
    sq = torch.zeros(1, device="cuda")
    out = torch.empty(seg, dtype=torch.bfloat16, device="cuda")
    res = {"fused_gemm": "qkvg wgrad", "world": world, "T": T, "M": M, "N": N, "chunk": chunk}
    res["gemm_only_ms"] = _time(lambda: C.gemm(dy, x, slot, True, True, None), iters)
    res["gemm_scatter_only_ms"] = _time(
        lambda: (C.gemm_scatter(dy, x, slot, False, grad, bases, seg, rank, chunk), comm.barrier()), iters)
    res["fused_gemm_reduce_scatter_ms"] = _time(
        lambda: (C.gemm_scatter(dy, x, slot, False, grad, bases, seg, rank, chunk), comm.barrier(),
                 C.reduce_compact(grad, staging, seg, world, rank, seg, chunk, part, 296), C.sum_partials(part, sq)),
        iters)
    res["gemm_then_nccl_reduce_scatter_ms"] = _time(
        lambda: (C.gemm(dy, x, slot, True, True, None),
                 dist.reduce_scatter_tensor(out, grad, op=dist.ReduceOp.AVG)), iters)
    res["gemm_then_p2p_reduce_owner_ms"] = _time(
        lambda: (C.gemm(dy, x, slot, True, True, None), comm.barrier(),
                 C.reduce_owner(comm.peers["fg_grad"], grad, rank * seg, seg, part, sq, 0, rank)), iters)
    t_compute = 2.0 * T * M * N / (BF16_TFLOPS * 1e12) * 1e3
    t_link = (world - 1) / world * numel * 2 / (LINK_GBS * 1e9) * 1e3
    res["roofline_ms"] = max(t_compute, t_link)
    res["roofline_compute_ms"], res["roofline_link_ms"] = t_compute, t_link
    for k in [k for k in res if k.endswith("_ms") and not k.startswith("roofline")]:
        res[k.replace("_ms", "_frac_of_roofline")] = res["roofline_ms"] / res[k]
    if rank == 0:
        print(json.dumps(res), flush=True)


def fused_gather_bench(comm, sizes_mb, iters, T=2048, K=3072, chunk=1 << 18):
    """All-gather -> GEMM of a forward weight ([N, 3072] bf16, N from the weight size; x [2048, 3072]): the
    all-gather fused into the consumer GEMM (gemm_gather: the GEMM's gather warps pull the rows other ranks own
    from their replicas ahead of the tiles, block-cyclic owner map) against NCCL all_gather_into_tensor + the GEMM.
    Sizes are the whole weight (1 MB .. 1 GB); roofline = max(FLOPs / measured bf16 peak, bytes this rank receives
    ((world - 1) / world of the weight) / 770 GB/s)."""
    from .. import ops
    C = comm.C
    rank, world = comm.rank, comm.world
    g = torch.Generator(device="cuda").manual_seed(rank)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    nmax = max(sizes_mb) * 1024 * 1024 // (2 * K) // 8 * 8
    span = chunk * world
    seg_max = -(-nmax * K // span) * chunk
    flat = comm.alloc("gg_param", world * seg_max, torch.bfloat16)
    flat.normal_(0, 0.02)
    peers = torch.tensor(comm.peers["gg_param"], dtype=torch.int64, device="cuda")
    for mb in sizes_mb:
        N = max(8, mb * 1024 * 1024 // (2 * K) // 8 * 8)
        numel = N * K
        seg_n = -(-numel // (world * 8)) * 8                  # NCCL: contiguous shards of the weight
        w = flat[:numel].view(N, K)
        y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        full = torch.empty(world * seg_n, dtype=torch.bfloat16, device="cuda")
        shard = flat[rank * seg_n:(rank + 1) * seg_n] if (rank + 1) * seg_n <= flat.numel() else full[:seg_n]
        res = {"fused_gather": "all-gather + GEMM", "world": world, "weight_mb": mb, "T": T, "N": N, "K": K,
               "chunk": chunk}
        res["gemm_only_ms"] = _time(lambda: ops.gemm(x, w, out=y), iters)
        res["fused_gather_gemm_ms"] = _time(
            lambda: (comm.barrier(), ops.gemm_gather(x, w, flat, peers, seg_max, chunk, rank, out=y)), iters)
        res["nccl_allgather_then_gemm_ms"] = _time(
            lambda: (dist.all_gather_into_tensor(full, shard),
                     ops.gemm(x, full[:numel].view(N, K), out=y)), iters)
        t_compute = 2.0 * T * N * K / (BF16_TFLOPS * 1e12) * 1e3
        t_link = (world - 1) / world * numel * 2 / (LINK_GBS * 1e9) * 1e3
        res["roofline_ms"] = max(t_compute, t_link)
        res["roofline_compute_ms"], res["roofline_link_ms"] = t_compute, t_link
        for k in [k for k in res if k.endswith("_ms") and not k.startswith("roofline")]:
            res[k.replace("_ms", "_frac_of_roofline")] = res["roofline_ms"] / res[k]
        if rank == 0:
            print(json.dumps(res), flush=True)


def fused_adam_bench(comm, sizes_mb, iters):
    """Reduce-scatter + Adam + all-gather over per-rank segments: ours (P2P FP32 rank-order reduce-to-owner with
    the norm partial, then Adam fused with the push all-gather, one barrier) vs NCCL reduce-scatter + Adam + NCCL
    all-gather."""
    C = comm.C
    rank, world = comm.rank, comm.world
    seg_max = max(sizes_mb) * 1024 * 1024 // 2
    grad = comm.alloc("fa_grad", world * seg_max, torch.bfloat16)
    param = comm.alloc("fa_param", world * seg_max, torch.bfloat16)
    grad.normal_(0.0, 1e-3)
    param.normal_(0.0, 0.02)
    hyper = torch.tensor([1.5e-4, 0.1, 0.05, 1.0], device="cuda")
    factor = torch.ones(1, device="cuda")
    part = torch.zeros(296, device="cuda")
    sq = torch.zeros(1, device="cuda")
    for mb in sizes_mb:
        seg = mb * 1024 * 1024 // 2
        g, p = grad[: world * seg], param[: world * seg]
        p32 = p[rank * seg:(rank + 1) * seg].float()
        m = torch.zeros_like(p32)
        v = torch.zeros_like(p32)
        out = torch.empty(seg, dtype=torch.bfloat16, device="cuda")

        def ours():
            comm.barrier()
            C.reduce_owner(comm.peers["fa_grad"], g, rank * seg, seg, part, sq, 0, rank)
            C.adam_push(p32, g[rank * seg:(rank + 1) * seg], m, v, p[rank * seg:(rank + 1) * seg], hyper, factor,
                        0.9, 0.95, 1e-6, 0.05, True, comm.peers["fa_param"], rank * seg, rank, 0)
            comm.barrier()

        def nccl():
            dist.reduce_scatter_tensor(out, g, op=dist.ReduceOp.AVG)
            C.adam_step(p32, out, m, v, p[rank * seg:(rank + 1) * seg], hyper, factor, 0.9, 0.95, 1e-6, 0.05, True)
            dist.all_gather_into_tensor(p, p[rank * seg:(rank + 1) * seg])

        res = {"fused_adam": True, "size_mb_per_rank": mb, "world": world}
        res["p2p_reduce_adam_push_ms"] = _time(ours, iters)
        res["nccl_reduce_scatter_adam_allgather_ms"] = _time(nccl, iters)
        t_link = 2 * (world - 1) * seg * 2 / (LINK_GBS * 1e9) * 1e3     # reduce in + all-gather in, per rank
        t_hbm = seg * 28 / (HBM_GBS * 1e9) * 1e3                        # Adam: fp32 p/m/v r+w, bf16 g r, bf16 p w
        res["roofline_ms"] = max(t_link, t_hbm)
        res["roofline_link_ms"], res["roofline_hbm_ms"] = t_link, t_hbm
        for k in ("p2p_reduce_adam_push_ms", "nccl_reduce_scatter_adam_allgather_ms"):
            res[k.replace("_ms", "_frac_of_roofline")] = res["roofline_ms"] / res[k]
        if rank == 0:
            print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
