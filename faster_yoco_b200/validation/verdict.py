"""The paired-validation criterion (scripts/validate/verdict.py of the reference): with the seed yardstick
``Y = ref_s2 - ref`` and the effects ``E1 = opt - ref``, ``E2 = opt_s2 - ref_s2``, ``S = opt_s2 - opt``, the optimised
arm is consistent with the reference arm at a checkpoint when ``|E1|, |E2|, |S| <= |Y|``; reported for the held-out mix,
each held-out source and the training loss (mean of the 1000 updates up to the checkpoint). Writes ``verdict.md``.

    python -m faster_yoco_b200.validation.verdict VAL_DIR
"""
from __future__ import annotations

import json
import os
import sys

from .analyze import train_window

NEED = ("opt", "ref", "ref_s2", "opt_s2")
KEYS = {"mix": "mix_bits", "fineweb": "fineweb_bits", "code": "code_bits"}


def metric(arm: dict, k: int, m: str):
    if m == "train":
        return train_window(arm, k)
    h = arm["heldout"].get(str(k))
    return None if h is None else h[KEYS[m]]


def apply_criterion(S: dict, checkpoints):
    rows, verdict = [], {}
    for m in ("mix", "fineweb", "code", "train"):
        rows += [f"\n### {m} (bits)\n", "| update | opt | ref | ref_s2 | opt_s2 | Y | E1 | E2 | S | within |Y| |",
                 "|---|---|---|---|---|---|---|---|---|---|"]
        res = []
        for k in checkpoints:
            v = {a: metric(S[a], k, m) for a in NEED}
            if any(x is None for x in v.values()):
                continue
            Y = v["ref_s2"] - v["ref"]
            E1, E2, Sd = v["opt"] - v["ref"], v["opt_s2"] - v["ref_s2"], v["opt_s2"] - v["opt"]
            flags = [abs(x) <= abs(Y) for x in (E1, E2, Sd)]
            res.append((k, all(flags), *flags))
            bad = ",".join(n for n, f in zip(("E1", "E2", "S"), flags) if not f)
            rows.append(f"| {k} | {v['opt']:.4f} | {v['ref']:.4f} | {v['ref_s2']:.4f} | {v['opt_s2']:.4f} | "
                        f"{Y:+.4f} | {E1:+.4f} | {E2:+.4f} | {Sd:+.4f} | {'yes' if all(flags) else 'no (' + bad + ')'} |")
        verdict[m] = {"checkpoints_within": sum(r[1] for r in res), "checkpoints": len(res),
                      "final_within": res[-1][1] if res else None, "E1_within": sum(r[2] for r in res),
                      "E2_within": sum(r[3] for r in res), "S_within": sum(r[4] for r in res)}
    return "\n".join(rows), verdict


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    V = os.path.abspath(argv[0])
    S = json.load(open(os.path.join(V, "summary.json")))["arms"]
    missing = [a for a in NEED if a not in S]
    if missing:
        raise SystemExit(f"missing arms {missing}")
    cps = sorted({int(k) for a in S.values() for k in a["heldout"]})
    text, verdict = apply_criterion(S, cps)
    with open(os.path.join(V, "verdict.md"), "w") as f:
        f.write(text + "\n\n" + json.dumps(verdict, indent=1) + "\n")
    print(text)
    print(json.dumps(verdict, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
