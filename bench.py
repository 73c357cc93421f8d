"""Headline benchmark: YOCO-3B pretraining updates, 2,048 tokens per GPU, ZeRO-1, BF16 + FP32 master / Adam.

    python bench.py --gpus N --steps K --warmup W            (N > 1: under torch.distributed.run, one rank per GPU)
    python bench.py --impl reference ...                      (the unmodified reference; see `reference_arm`)

Prints ONE JSON line on rank 0. ``value`` is the whole-job throughput (tokens/s over all N GPUs) from CUDA events
on each rank's launching stream around exactly K updates (barrier + synchronize on both sides), max over ranks.
``e2e`` is the same metric through the public training API with, every update, the host->device copy of that
update's token ids from pinned memory and a device->host read of its loss.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TOKS = 138983.0          # published Faster-YOCO throughput, 8 x H100, tokens/s over all GPUs
METRIC = "ms/update & tokens/sec, YOCO-3B 2048 tok/GPU, 1/2/4/8 B200, max over ranks"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--arch", default="yoco_3b")
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--batch", type=int, default=1, help="sequences per GPU")
    p.add_argument("--kernels", default="native", choices=["native", "torch"])
    p.add_argument("--comm", default="fused", choices=["nccl", "fused"],
                   help="fused: NVLink peer-memory collectives overlapped with compute; nccl: the baseline path")
    p.add_argument("--graph", type=int, default=1, help="capture the whole update as one CUDA graph")
    p.add_argument("--overlap", default="auto", choices=["auto", "0", "1", "grads"],
                   help="fused comm: 1 = gradients and parameters pushed per layer bucket, overlapped with "
                        "backward / forward; grads = only the gradients per bucket during backward, the parameters "
                        "by the fused Adam + push after it; 0 = the serial exchange (P2P reduce + fused Adam + push "
                        "after backward); auto = the measured schedule of this GPU count "
                        "(faster_yoco_b200.parallel.zero.AUTO_SCHEDULE)")
    p.add_argument("--transport", default="auto", choices=["auto", "sm", "ce", "gemm", "pull"],
                   help="overlapped exchange: pushes by kernels (sm) or by the copy engines (ce); gemm: the "
                        "weight-gradient GEMMs store every element at its ZeRO owner over NVLink (GEMM fused with the "
                        "reduce-scatter), parameters pushed after the update (--overlap 0) or per layer ahead of "
                        "the next forward (--overlap 1); pull: the parameter all-gather fused into the consuming "
                        "forward GEMMs (gather warps pull each weight's rows from their owners ahead of the tiles; "
                        "use with --partition cyclic), gradients by the serial P2P reduce")
    p.add_argument("--partition", default="even", choices=["even", "greedy", "cyclic"],
                   help="ZeRO owner map: even contiguous segments, the OSS greedy per-parameter rule, or block-cyclic "
                        "chunks (every weight spread over all owners)")
    p.add_argument("--zero-chunk", type=int, default=None, help="chunk size (elements) of --partition cyclic")
    p.add_argument("--sliding-window", type=int, default=None)
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--count-launches", type=int, default=1)
    p.add_argument("--exposed-comm", type=int, default=0,
                   help="after the measurements, time the same updates without any cross-rank exchange and report "
                        "exposed_comm_ms = ms_per_step - that (N > 1)")
    return p.parse_args()


def reference_arm(args):
    """The reference (a fairseq plug-in) cannot be installed or run on this image: the reference tree has no
    setup.py / pyproject.toml (pip: 'not installable'), and it needs the fairseq fork, fairscale, infinibatch and
    apex, none of which exist here or in the offline wheelhouse."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    why = ("reference is not pip-installable (no setup.py/pyproject.toml) and its runtime deps "
           "(fairseq fork, fairscale, infinibatch, apex) are absent offline")
    if os.path.isdir(ref_dir) and os.path.exists(os.path.join(ref_dir, "yoco")):
        why = "reference tree present but fairseq/fairscale/infinibatch/apex are not installed"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
    return 0


def nvml_handle(nv, props, index: int):
    """NVML handle of the CUDA device with properties ``props``. NVML numbers every GPU of the machine and ignores
    CUDA_VISIBLE_DEVICES, so the device is found by its UUID (then its PCI address); the CUDA index is used only
    when neither is available and no device is hidden."""
    def norm(u):
        u = (u.decode() if isinstance(u, bytes) else str(u)).lower()
        return u[4:] if u.startswith("gpu-") else u

    uuid = getattr(props, "uuid", None)
    pci = tuple(getattr(props, k, None) for k in ("pci_domain_id", "pci_bus_id", "pci_device_id"))
    try:                                    # enumerate: independent of how either side formats the ids
        for i in range(nv.nvmlDeviceGetCount()):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            if uuid is not None and norm(nv.nvmlDeviceGetUUID(h)) == norm(uuid):
                return h
            info = nv.nvmlDeviceGetPciInfo(h)
            if None not in pci and (info.domain, info.bus, info.device) == pci:
                return h
    except Exception:
        pass
    if uuid is not None:
        text = str(uuid)
        try:
            return nv.nvmlDeviceGetHandleByUUID(text if text.startswith("GPU-") else "GPU-" + text)
        except Exception:
            pass
    if getattr(props, "pci_bus_id", None) is not None:
        bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
        try:
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            pass
    if os.environ.get("CUDA_VISIBLE_DEVICES") is None:
        return nv.nvmlDeviceGetHandleByIndex(index)
    raise RuntimeError("cannot map CUDA device %d to an NVML device" % index)


class ClockSampler:
    """Samples SM clock / max clock / throttle reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = nvml_handle(pynvml, torch.cuda.get_device_properties(index), index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.1)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def merge_clocks(per_rank):
    """One clock record for the job from every rank's samples: the median SM clock over ranks, each rank's median,
    and the union of the throttle reasons any rank saw."""
    meds = [c["sm_mhz"] for c in per_rank if c.get("sm_mhz") is not None]
    reasons = sorted(set(r for c in per_rank for r in c.get("reasons", [])))
    maxes = [c["sm_max_mhz"] for c in per_rank if c.get("sm_max_mhz") is not None]
    out = {"sm_mhz": statistics.median(meds) if meds else None, "sm_max_mhz": max(maxes) if maxes else None,
           "reasons": reasons, "samples": sum(c.get("samples", 0) for c in per_rank)}
    if len(per_rank) > 1:
        out["per_rank_sm_mhz"] = [c.get("sm_mhz") for c in per_rank]
    return out


def result_line(args, world: int, ms: float, clocks, e2e, launches, exposed=None) -> dict:
    """The one JSON line of the benchmark contract (rank 0 prints it)."""
    tokens_per_update = args.batch * args.seq_len * world
    value = tokens_per_update / (ms / 1000.0)
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        # like with like under weak scaling: this run's tokens/s per GPU against the published 8-GPU run's per GPU
        # (138,983 / 8); at N = 8 this equals value / 138,983
        "vs_baseline": (value / world) / (BASELINE_TOKS / 8.0), "dtype": "bf16",
        "data": "synthetic uniform-random token ids, N(0,0.02) random-init weights",
        "config": {"model": args.arch + ("-swa%d" % args.sliding_window if args.sliding_window else ""),
                   "global_batch": args.batch * world, "seq_len": args.seq_len,
                   "tokens_per_update": tokens_per_update, "parallelism": f"dp{world}-zero1",
                   "kernels": args.kernels, "comm": args.comm if world > 1 else "none",
                   "vs_baseline_basis": "tokens/s per GPU vs 138983/8 (8xH100 published)",
                   "cuda_graph": bool(args.graph),
                   "comm_overlap": args.overlap if args.overlap == "grads" else bool(int(args.overlap)),
                   "zero_partition": args.partition,
                   "transport": (args.transport if (args.overlap or args.transport in ("gemm", "pull")) else "serial")
                   if world > 1 else None,
                   "l2": "working set (>=55 GB of params/grads/Adam state per update) >> 126 MB L2"},
        "clocks": clocks, "e2e": e2e, "gpu_launches": launches,
    }
    if exposed is not None:
        out["exposed_comm"] = exposed
    return out


def count_our_launches(step_fn) -> int:
    """Kernels from this repository's extension launched by one update (profiled separately, not timed)."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and "fyb::" in ev.name:
            n += 1
    return n


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)

    from faster_yoco_b200 import ops
    from faster_yoco_b200.config import OptimConfig, build_args
    from faster_yoco_b200.data.synthetic import SyntheticLM
    from faster_yoco_b200.models.yoco import YOCO
    from faster_yoco_b200.parallel import dist as D
    from faster_yoco_b200.parallel.zero import exchange_schedule
    from faster_yoco_b200.train.trainer import Trainer

    dev_index = D.init(timeout_s=300)
    rank, world = D.rank(), D.world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", dev_index)
    ops.set_backend(args.kernels)
    args.overlap, args.transport = exchange_schedule(world, args.comm, args.overlap, args.transport)
    torch.manual_seed(1234)

    margs = build_args(args.arch, max_seq_len=args.seq_len, max_batch_size=args.batch, init_std=0.02,
                       sliding_window=args.sliding_window)
    with torch.device(dev):
        model = YOCO(margs)
    model = model.to(torch.bfloat16)
    optim = OptimConfig()
    trainer = Trainer(model, optim, device=dev, comm=args.comm, graph_step=bool(args.graph),
                      overlap=args.overlap, transport=args.transport, partition=args.partition, chunk=args.zero_chunk)
    data = SyntheticLM(margs.vocab_size, args.seq_len, args.batch, seed=1, rank=rank, pin=True)
    batches = [next(data) for _ in range(4)]

    def step(i):
        return trainer.train_step(batches[i % len(batches)])

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    D.barrier()

    sampler = ClockSampler(dev_index)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        step(i)
    end.record()
    torch.cuda.synchronize()
    D.barrier()
    clocks = merge_clocks(D.all_gather_object(sampler.stop()))
    ms = start.elapsed_time(end) / args.steps
    ms = D.all_reduce_max(ms, dev)
    tokens_per_update = args.batch * args.seq_len * world
    value = tokens_per_update / (ms / 1000.0)

    # end to end through the public API: pinned H2D of each update's ids + D2H read of its loss
    e2e = None
    if not args.no_e2e:
        k = args.e2e_steps or args.steps
        D.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(k):
            loss = step(i)
            float(loss.item())
        torch.cuda.synchronize()
        dt = (time.perf_counter() - t0) / k
        dt = D.all_reduce_max(dt, dev)
        b = batches[0]
        e2e = {"value": tokens_per_update / dt, "unit": "tokens/s", "ms_per_step": dt * 1000.0,
               "h2d_bytes_per_step": int(b["src_tokens"].numel() * 8 + b["target"].numel() * 8),
               "d2h_bytes_per_step": 4}

    if os.environ.get("FYB_TIMELINE") == "1" and not args.graph:
        step(0)
        tl = trainer.timeline()
        if rank == 0:
            print(json.dumps({"timeline_ms": [(n, round(t, 3)) for n, t in tl]}), flush=True)

    launches = None
    if args.count_launches:
        try:
            launches = count_our_launches(lambda: step(0)) * args.steps
        except Exception:
            launches = None

    exposed = None
    if args.exposed_comm and world > 1:
        trainer.measure_without_exchange(True)
        for i in range(max(args.warmup, 3)):
            step(i)
        D.barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for i in range(args.steps):
            step(i)
        s1.record()
        torch.cuda.synchronize()
        D.barrier()
        ms_local = D.all_reduce_max(s0.elapsed_time(s1) / args.steps, dev)
        exposed = {"compute_only_ms_per_step": ms_local, "exposed_comm_ms": ms - ms_local}

    if rank == 0:
        out = result_line(args, world, ms, clocks, e2e, launches, exposed)
        print(json.dumps(out), flush=True)
    trainer.release_graph()
    D.barrier()
    D.destroy()
    return 0


if __name__ == "__main__":
    sys.exit(main())
