"""Rank functions used by the multi-process tests (importable by spawned children)."""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def _tiny_trainer(device, comm="nccl", seed=0, graph=False, arch="yoco_tiny", dtype=torch.float32, overlap=True,
                  transport="sm", partition="even", chunk=None, zero_sharding="os", **arch_overrides):
    from ..config import OptimConfig, build_args
    from ..models.yoco import YOCO
    from ..train.trainer import Trainer
    torch.manual_seed(seed)
    args = build_args(arch, max_seq_len=256, init_std=0.02, **arch_overrides)
    model = YOCO(args).to(device=device, dtype=dtype)
    cfg = OptimConfig(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, warmup_updates=0, total_num_update=20)
    return model, Trainer(model, cfg, device=device, comm=comm, graph_step=graph, overlap=overlap,
                          transport=transport, partition=partition, chunk=chunk, zero_sharding=zero_sharding)


def _batches(rank, world, n, seed=1, batch=2, seq=256, vocab=1024):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, vocab, (world, batch, seq + 1), generator=g)
        out.append(ids)
    return out


def zero_matches_single(rank, world, outdir, steps, partition="even", chunk=None, zero_sharding="os"):
    """World-size-N ZeRO training on N shards of each global batch; rank 0 saves the final flat params."""
    model, tr = _tiny_trainer(torch.device("cpu"), partition=partition, chunk=chunk, zero_sharding=zero_sharding)
    for ids in _batches(rank, world, steps):
        mine = ids[rank]
        b = {"src_tokens": mine[:, :-1].contiguous(), "target": mine[:, 1:].contiguous(),
             "ntokens": mine.shape[0] * mine.shape[1], "nsentences": mine.shape[0]}
        tr.train_step(b)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    if rank == 0:
        torch.save({"sd": sd, "num_updates": tr.num_updates()},
                   os.path.join(outdir, f"ws{world}_{partition}_{zero_sharding}.pt"))


def single_reference(outdir, world, steps, with_norm=False):
    """Single process, batch = all shards concatenated (the same global batch)."""
    model, tr = _tiny_trainer(torch.device("cpu"))
    for ids in _batches(0, world, steps):
        allb = ids.reshape(-1, ids.shape[-1])
        b = {"src_tokens": allb[:, :-1].contiguous(), "target": allb[:, 1:].contiguous(),
             "ntokens": allb.shape[0] * allb.shape[1], "nsentences": allb.shape[0]}
        tr.train_step(b)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    return (sd, float(tr.zero.last_grad_norm)) if with_norm else sd


def checkpoint_resume(rank, world, outdir, steps, split, partition="even", chunk=None, resume_partition=None):
    """Train `steps`, or train `split`, checkpoint, rebuild everything (optionally with another owner map: the
    checkpoint holds per-parameter optimizer state), load, train the rest."""
    from ..train.checkpoint import load_checkpoint, save_checkpoint
    batches = _batches(rank, world, steps)

    def run(tr, bs):
        for ids in bs:
            mine = ids[rank]
            tr.train_step({"src_tokens": mine[:, :-1].contiguous(), "target": mine[:, 1:].contiguous(),
                           "ntokens": mine.shape[0] * mine.shape[1], "nsentences": mine.shape[0]})

    model, tr = _tiny_trainer(torch.device("cpu"), partition=partition, chunk=chunk)
    run(tr, batches[:split])
    path = os.path.join(outdir, "ckpt.pt")
    save_checkpoint(path, model, tr)
    dist.barrier()
    rp = resume_partition or partition
    model2, tr2 = _tiny_trainer(torch.device("cpu"), seed=123, partition=rp,  # different init: must be overwritten
                                chunk=chunk)
    load_checkpoint(path, model2, tr2)
    run(tr2, batches[split:])
    model3, tr3 = _tiny_trainer(torch.device("cpu"), partition=partition, chunk=chunk)
    run(tr3, batches)
    if rank == 0:
        torch.save({"resumed": model2.state_dict(), "straight": model3.state_dict(),
                    "n2": tr2.num_updates(), "n3": tr3.num_updates()}, os.path.join(outdir, "resume.pt"))


def rank_fails_before_collective(rank, world, outdir):
    """Host-injected failure: rank 1 raises before the collective; rank 0 must see a timeout/error, not hang."""
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    t = torch.ones(1)
    dist.all_reduce(t)


def fused_vs_nccl_gpu(rank, world, outdir, steps):
    """GPU: the same training with the NVLink peer-memory collectives and with NCCL; rank 0 saves both."""
    from .. import ops
    ops.set_backend("native")
    dev = torch.device("cuda", rank)
    res = {}
    # overlap "grads": gradients per bucket during backward, parameters by the fused Adam + push after the update
    # (copy-engine pushes eager; kernel pushes inside the captured update)
    for name, comm, overlap, transport, graph in (
            ("nccl", "nccl", False, "sm", False), ("fused", "fused", True, "sm", False),
            ("fused_serial", "fused", False, "sm", False), ("fused_ce", "fused", True, "ce", False),
            ("fused_ce_graph", "fused", True, "ce", True), ("fused_serial_two_pass", "fused", False, "sm", False),
            ("fused_grads_ce", "fused", "grads", "ce", False), ("fused_grads_sm_graph", "fused", "grads", "sm", True)):
        model, tr = _tiny_trainer(dev, comm=comm, arch="yoco_small", dtype=torch.bfloat16, overlap=overlap,
                                  transport=transport, graph=graph)
        # the serial variants differ only in Adam + all-gather: one fused kernel, or Adam then the push kernel
        tr.zero.fuse_adam_push = name != "fused_serial_two_pass"
        losses = []
        for ids in _batches(rank, world, steps, seq=256, vocab=8192):
            mine = ids[rank]
            b = {"src_tokens": mine[:, :-1].contiguous(), "target": mine[:, 1:].contiguous(),
                 "ntokens": mine.shape[0] * mine.shape[1], "nsentences": mine.shape[0]}
            losses.append(float(tr.train_step(b).item()))
        tr.sync_params()
        tr.release_graph()
        torch.cuda.synchronize()
        status = int(ops._C().status()[0].item())
        # parameters in model order (the padding of the flat buffer differs between owner maps)
        params = torch.cat([p.detach().float().reshape(-1) for p in model.parameters()]).cpu()
        res[name] = {"losses": losses, "params": params, "status": status}
        if tr.zero.p2p is not None:
            tr.zero.p2p.close()
    if rank == 0:
        torch.save(res, os.path.join(outdir, "fused_vs_nccl.pt"))


def gemm_scatter_vs_serial_gpu(rank, world, outdir, steps):
    """GPU: serial P2P exchange against the GEMM-fused reduce-scatter (weight-gradient GEMMs store at the owners),
    eager and graphed, and with two micro-batches per update; rank 0 saves every variant's losses and parameters."""
    from .. import ops
    ops.set_backend("native")
    dev = torch.device("cuda", rank)
    res = {}
    for name, transport, graph, uf, part in (
            ("serial", "sm", False, 1, "even"), ("gemm", "gemm", False, 1, "even"),
            ("gemm_graph", "gemm", True, 1, "even"), ("serial_uf2", "sm", False, 2, "even"),
            ("gemm_uf2", "gemm", False, 2, "even"), ("serial_cyclic", "sm", False, 1, "cyclic"),
            ("gemm_cyclic", "gemm", False, 1, "cyclic"), ("gemm_cyclic_graph", "gemm", True, 1, "cyclic"),
            ("gemm_overlap_cyclic", "gemm+overlap", True, 1, "cyclic"), ("sm_overlap_cyclic", "sm+overlap", False,
                                                                          1, "cyclic"),
            ("pull_cyclic", "pull", False, 1, "cyclic"), ("pull_cyclic_graph", "pull", True, 1, "cyclic"),
            ("pull_even", "pull", False, 1, "even")):
        overlap = transport.endswith("+overlap")
        model, tr = _tiny_trainer(dev, comm="fused", arch="yoco_small", dtype=torch.bfloat16, overlap=overlap,
                                  transport=transport.split("+")[0], graph=graph, partition=part, chunk=1 << 14)
        losses = []
        for ids in _batches(rank, world, steps, seq=256, vocab=8192, batch=2 * uf):
            mine = ids[rank]
            micro = []
            for m in mine.chunk(uf, 0):
                micro.append({"src_tokens": m[:, :-1].contiguous(), "target": m[:, 1:].contiguous(),
                              "ntokens": m.shape[0] * (m.shape[1] - 1), "nsentences": m.shape[0]})
            losses.append(float(tr.train_step(micro if uf > 1 else micro[0]).item()))
        tr.sync_params()
        tr.release_graph()
        torch.cuda.synchronize()
        status = int(ops._C().status()[0].item())
        # parameters in model order (the padding of the flat buffer differs between owner maps)
        params = torch.cat([p.detach().float().reshape(-1) for p in model.parameters()]).cpu()
        res[name] = {"losses": losses, "params": params, "status": status}
        tr.zero.p2p.close()
    if rank == 0:
        torch.save(res, os.path.join(outdir, "gemm_scatter.pt"))


def gemm_gather_gpu(rank, world, outdir, chunk):
    """GPU, one rank per GPU over CUDA-IPC peer replicas: the ZeRO all-gather fused into the consumer GEMM
    (gemm_gather). Every rank writes only the elements it owns (block-cyclic map of `chunk`, or contiguous segments
    for chunk 0) and garbage elsewhere; after a barrier each rank's gather-GEMM must leave the weight current in its
    replica and produce a @ w_true^T. Twice, so the second call also reads rows that the first one pulled."""
    from .. import ops
    from ..parallel.p2p import PeerComm
    ops.set_backend("native")
    dev = torch.device("cuda", rank)
    comm = PeerComm()
    K, N, M = 512, 1544, 512
    span = (chunk or 1024) * world
    seg = ((N * K + 65536 + span - 1) // span) * span // world
    flat = comm.alloc("param", world * seg, torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(7)
    truth = (torch.randn(world * seg, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.arange(world * seg, device=dev)
    own = (x // chunk) % world if chunk else x // seg
    flat.copy_(torch.where(own == rank, truth, torch.full_like(truth, 7.0)))
    torch.cuda.synchronize()
    comm.barrier()
    peers = torch.tensor(comm.peers["param"], dtype=torch.int64, device=dev)
    a = (torch.randn(M, K, device=dev, generator=g)).to(torch.bfloat16)
    w_off = 40960 + 16
    w = flat[w_off:w_off + N * K].view(N, K)
    ok = True
    for _ in range(2):
        y = ops.gemm_gather(a, w, flat, peers, seg, chunk, rank)
        torch.cuda.synchronize()
        ok = ok and torch.equal(flat[w_off:w_off + N * K], truth[w_off:w_off + N * K])
    y0 = ops.gemm(a, truth[w_off:w_off + N * K].view(N, K).contiguous())
    err = float(((y.float() - y0.float()).abs().max() / y0.float().abs().max()).item())
    status = int(ops._C().status()[0].item())
    comm.barrier()
    torch.cuda.synchronize()
    comm.close()
    torch.save({"ok": ok, "err": err, "status": status}, os.path.join(outdir, f"gemm_gather_{rank}.pt"))


def exchange_free_steps(rank, world, outdir, steps):
    """Updates without any cross-rank exchange (the measurement mode behind exposed-communication timing): they run
    without collectives, so ranks diverge; normal updates work again afterwards."""
    model, tr = _tiny_trainer(torch.device("cpu"))
    bs = _batches(rank, world, 2 * steps + 1)

    def one(ids):
        mine = ids[rank]
        return tr.train_step({"src_tokens": mine[:, :-1].contiguous(), "target": mine[:, 1:].contiguous(),
                              "ntokens": mine.shape[0] * mine.shape[1], "nsentences": mine.shape[0]})

    for ids in bs[:steps]:
        one(ids)
    same_before = tr.flat.flat.clone()
    tr.measure_without_exchange(True)
    for ids in bs[steps:2 * steps]:
        one(ids)
    tr.measure_without_exchange(False)
    mine = tr.flat.flat.clone()
    allp = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allp, mine)
    loss = float(one(bs[-1]))
    if rank == 0:
        torch.save({"diverged": not torch.equal(allp[0], allp[1]), "loss": loss,
                    "changed": not torch.equal(same_before, mine)}, os.path.join(outdir, "noexchange.pt"))


def tp_dp_matches_single(rank, world, outdir, steps, full_sd):
    """Tensor x data parallel training (TP 2 x DP world/2) of the tiny YOCO started from the slices of `full_sd`;
    data-parallel rank 0 of every TP slice saves its final weights (reference names, this slice's shapes)."""
    from ..config import OptimConfig, build_args
    from ..models.yoco import YOCO, shard_state_dict
    from ..parallel import tp as TP
    from ..train.trainer import Trainer
    tps = 2
    TP.init_model_parallel(tps)
    dp, dpr = world // tps, rank // tps
    torch.manual_seed(0)
    args = build_args("yoco_tiny", max_seq_len=256, init_std=0.02, model_parallel_size=tps)
    model = YOCO(args).to(torch.float32)
    model.load_state_dict(shard_state_dict(full_sd, tps, TP.tp_rank()), strict=True)
    cfg = OptimConfig(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, warmup_updates=0, total_num_update=20)
    tr = Trainer(model, cfg, device=torch.device("cpu"), comm="nccl")
    assert tr.world == dp and tr.rank == dpr
    for ids in _batches(dpr, dp, steps):
        mine = ids[dpr]
        tr.train_step({"src_tokens": mine[:, :-1].contiguous(), "target": mine[:, 1:].contiguous(),
                       "ntokens": mine.shape[0] * mine.shape[1], "nsentences": mine.shape[0]})
    gn = float(tr.zero.last_grad_norm)
    if dpr == 0:
        torch.save({"sd": {k: v.detach().clone() for k, v in model.state_dict().items()}, "gnorm": gn},
                   os.path.join(outdir, f"tp{TP.tp_rank()}.pt"))
    TP.destroy_model_parallel()
