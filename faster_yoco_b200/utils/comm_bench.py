"""Fused-path microbenchmark (one rank per GPU, launched with torch.distributed.run):

* parameter all-gather: NCCL all_gather_into_tensor vs the peer-memory pull (gather_segments) and push
  (push_range) kernels, per-rank message sizes 1 MB .. 1 GB;
* copy-engine push all-gather (one cudaMemcpyAsync per peer on per-peer streams), and how much a GEMM chain slows
  down while the copy engines push (the question for overlapping the exchange with compute);
* gradient reduce-scatter: NCCL reduce_scatter_tensor (AVG, bf16) vs the owner-side FP32 rank-order reduction over
  NVLink (reduce_owner, with the grad-norm partial).

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


if __name__ == "__main__":
    main()
