"""Summary of the validation arms (scripts/validate/analyze.py of the reference): training-loss means per 100
updates, held-out losses per checkpoint, time per update (train_wall of the log lines, excluding the model saves),
peak memory, non-finite values. Reads ``<val dir>/<arm>/{train.log, eval.json}``; writes ``summary.json`` and
``tables.md``.

    python -m faster_yoco_b200.validation.analyze VAL_DIR [arms...]     (default arms: opt ref ref_s2 opt_s2)
"""
from __future__ import annotations

import json
import math
import os
import re
import sys

LOG = re.compile(r"epoch \d+: (.*)$")
KV = re.compile(r"(\w+) ([^|]+)")
ARMS = ("opt", "ref", "ref_s2", "opt_s2")


def parse_train_log(path: str):
    rows, saves, mem, nonfinite = [], [], {}, []
    with open(path, errors="replace") as f:
        for line in f:
            m = LOG.search(line)
            if m:
                kv = {k: v.strip() for k, v in KV.findall(m.group(1))}
                try:
                    n, loss = int(kv["num_updates"]), float(kv["loss"])
                    gn, wall = float(kv.get("gnorm", "nan")), float(kv.get("train_wall", "nan"))
                except (KeyError, ValueError):
                    continue
                rows.append((n, loss, gn, wall))
                if not (math.isfinite(loss) and math.isfinite(gn)):
                    nonfinite.append(n)
            if "VALIDATION_MEM" in line:
                for js in re.findall(r"\{[^{}]*\}", line):
                    try:
                        r = json.loads(js)
                    except ValueError:
                        continue
                    if "rank" in r and "max_allocated_gib" in r:
                        mem[r["rank"]] = max(mem.get(r["rank"], 0.0), r["max_allocated_gib"])
            for m2 in re.finditer(r"VALIDATION_CKPT \S+ ([0-9.]+)s", line):
                saves.append(float(m2.group(1)))
    return rows, saves, mem, nonfinite


def summarize_arm(d: str):
    rows, saves, mem, nonfinite = parse_train_log(os.path.join(d, "train.log"))
    if not rows:
        return None
    bins = {}
    for n, loss, _, _ in rows:
        bins.setdefault((n - 1) // 100, []).append(loss)
    per = {str((k + 1) * 100): sum(v) / len(v) for k, v in sorted(bins.items())}
    a = next((r for r in rows if r[0] >= 1000), rows[0])
    b = rows[-1]
    spu = ((b[3] - a[3]) - sum(saves)) / (b[0] - a[0]) if b[0] > a[0] else None
    ev_path = os.path.join(d, "eval.json")
    held = {}
    if os.path.exists(ev_path):
        for v in json.load(open(ev_path)).values():
            if "mix_0.8_0.2_bits" in v:
                held[str(v["num_updates"])] = {"mix_bits": v["mix_0.8_0.2_bits"],
                                               "fineweb_bits": v["fineweb_edu"]["loss_bits"],
                                               "code_bits": v["codeparrot"]["loss_bits"]}
    last = [r[1] for r in rows if r[0] > rows[-1][0] - 1000]
    return {"updates": rows[-1][0], "final_train_loss_bits_last1000": sum(last) / len(last),
            "train_curve_per100": per, "heldout": held, "s_per_update_excl_saves": spu,
            "save_s_total": sum(saves), "peak_alloc_gib_max_rank": max(mem.values()) if mem else None,
            "nonfinite": nonfinite[:5]}


def train_window(arm: dict, k: int, w: int = 1000):
    c = arm["train_curve_per100"]
    vals = [c[str(j)] for j in range(k - w + 100, k + 1, 100) if str(j) in c]
    return sum(vals) / len(vals) if len(vals) == w // 100 else None


def tables(out: dict, checkpoints) -> str:
    cols = [a for a in ("opt", "ref", "ref_s2", "opt_s2") if a in out]
    fmt = lambda x: "-" if x is None else f"{x:.4f}"
    lines = ["| update | " + " | ".join(f"train {a}" for a in cols) + " | " +
             " | ".join(f"held-out mix {a}" for a in cols) + " |", "|" + "---|" * (1 + 2 * len(cols))]
    for k in checkpoints:
        tr = [train_window(out[a], k) for a in cols]
        hm = [out[a]["heldout"].get(str(k), {}).get("mix_bits") for a in cols]
        lines.append(f"| {k} | " + " | ".join(map(fmt, tr)) + " | " + " | ".join(map(fmt, hm)) + " |")
    return "\n".join(lines) + "\n"


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    V = os.path.abspath(argv[0])
    arms = argv[1:] or list(ARMS)
    out = {}
    for arm in arms:
        d = os.path.join(V, arm)
        if os.path.exists(os.path.join(d, "train.log")):
            s = summarize_arm(d)
            if s is not None:
                out[arm] = s
    every = sorted({int(k) for a in out.values() for k in a["heldout"]}) or \
        list(range(1000, max((a["updates"] for a in out.values()), default=0) + 1, 1000))
    with open(os.path.join(V, "summary.json"), "w") as f:
        json.dump({"arms": out}, f, indent=1)
    text = tables(out, every)
    with open(os.path.join(V, "tables.md"), "w") as f:
        f.write(text)
    print(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
