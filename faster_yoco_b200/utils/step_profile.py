"""Kernel-time breakdown of one training update (torch.profiler / CUPTI), grouped by kernel name.

    python -m faster_yoco_b200.utils.step_profile [--arch yoco_3b] [--seq-len 2048] [--top 40]

Prints one JSON line per kernel group (name, launches, total ms, share) for the profiled update; the numbers are
for attribution only (the profiler serialises nothing but adds overhead), not benchmark values.
"""
import argparse
import json
from collections import defaultdict

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--arch", default="yoco_3b")
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--top", type=int, default=40)
    ap.add_argument("--kernels", default="native")
    a = ap.parse_args()
    from faster_yoco_b200 import ops
    from faster_yoco_b200.config import OptimConfig, build_args
    from faster_yoco_b200.data.synthetic import SyntheticLM
    from faster_yoco_b200.models.yoco import YOCO
    from faster_yoco_b200.train.trainer import Trainer
    ops.set_backend(a.kernels)
    dev = torch.device("cuda", 0)
    args = build_args(a.arch, max_seq_len=a.seq_len, init_std=0.02)
    with torch.device(dev):
        model = YOCO(args)
    model = model.to(torch.bfloat16)
    tr = Trainer(model, OptimConfig(), device=dev)
    data = SyntheticLM(args.vocab_size, a.seq_len, 1, pin=True)
    for _ in range(3):
        tr.train_step(next(data))
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        tr.train_step(next(data))
        torch.cuda.synchronize()
    groups = defaultdict(lambda: [0, 0.0])
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            name = ev.name.replace("(anonymous namespace)::", "").replace("void ", "")
            name = name.split("(")[0][:140]
            g = groups[name]
            g[0] += 1
            g[1] += ev.device_time_total / 1000.0
    total = sum(v[1] for v in groups.values())
    print(json.dumps({"total_kernel_ms": total, "groups": len(groups)}))
    for name, (n, ms) in sorted(groups.items(), key=lambda kv: -kv[1][1])[:a.top]:
        print(json.dumps({"kernel": name, "launches": n, "ms": round(ms, 3), "share": round(ms / total, 4)}))


if __name__ == "__main__":
    main()
