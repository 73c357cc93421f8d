"""Loss parity of the sm_100a path against the PyTorch path (the same model, optimizer and data; only the kernels
differ), in the spirit of the reference's statistical gate: several seeds per path, the per-window mean training
loss, and the criterion that the cross-path differences stay within the seed-to-seed spread of the PyTorch path
(|E1|, |E2|, |S| <= |Y| per window, with Y = torch_s2 - torch_s1, E1 = native_s1 - torch_s1,
E2 = native_s2 - torch_s2, S = native_s2 - native_s1) plus the mean absolute difference in units of 2 sigma of the
seeds.

The data is a learnable synthetic corpus (token sequences from a fixed random first-order Markov chain over the
vocabulary, seeded independently of the model seed), so the curves fall from ln(V) towards the chain's entropy and
differences between paths are visible, unlike with uniform-random ids.

    python -m faster_yoco_b200.validation.parity --arch yoco_small --updates 200 --seeds 1,2 --out parity.json
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from typing import Dict, List

import torch


class MarkovLM:
    """Batches of sequences from a fixed sparse random Markov chain (each token has `fanout` successors)."""

    def __init__(self, vocab: int, seq_len: int, batch: int, chain_seed: int = 1234, data_seed: int = 0,
                 fanout: int = 4):
        g = torch.Generator().manual_seed(chain_seed)
        self.next = torch.randint(2, vocab, (vocab, fanout), generator=g)        # ids 0/1 (bos/pad) never emitted
        logits = torch.randn(vocab, fanout, generator=g) * 1.5
        self.probs = torch.softmax(logits, -1)
        self.vocab, self.seq_len, self.batch = vocab, seq_len, batch
        self.gen = torch.Generator().manual_seed(data_seed)

    def entropy_nats(self) -> float:
        p = self.probs
        return float(-(p * p.clamp_min(1e-30).log()).sum(-1).mean())

    def __next__(self):
        B, L = self.batch, self.seq_len + 1
        ids = torch.empty(B, L, dtype=torch.int64)
        ids[:, 0] = torch.randint(2, self.vocab, (B,), generator=self.gen)
        for t in range(1, L):
            choice = torch.multinomial(self.probs[ids[:, t - 1]], 1, generator=self.gen).squeeze(1)
            ids[:, t] = self.next[ids[:, t - 1], choice]
        return {"src_tokens": ids[:, :-1].contiguous(), "target": ids[:, 1:].contiguous(),
                "ntokens": B * L, "nsentences": B}


def run(arch: str, backend: str, seed: int, updates: int, seq_len: int, batch: int, device, lr: float = 1e-3,
        data_seed: int = 0) -> List[float]:
    from .. import ops
    from ..config import OptimConfig, build_args
    from ..models.yoco import YOCO
    from ..train.trainer import Trainer
    ops.set_backend(backend)
    torch.manual_seed(seed)
    args = build_args(arch, max_seq_len=seq_len, init_std=0.02)
    with torch.device(device):
        model = YOCO(args)
    if device.type == "cuda":
        model = model.to(torch.bfloat16)
    cfg = OptimConfig(lr=lr, warmup_updates=20, total_num_update=max(updates, 100))
    tr = Trainer(model, cfg, device=device, graph_step=False)
    data = MarkovLM(args.vocab_size, seq_len, batch, data_seed=data_seed)
    losses = []
    for _ in range(updates):
        b = next(data)
        loss = tr.train_step(b)
        losses.append(float(loss) / (b["ntokens"]))
    return losses


def windows(xs: List[float], edges: List[int]) -> List[float]:
    return [sum(xs[a:b]) / max(1, len(xs[a:b])) for a, b in zip(edges[:-1], edges[1:])]


def criterion(curves: Dict[str, List[float]], edges: List[int]) -> dict:
    w = {k: windows(v, edges) for k, v in curves.items()}
    rows = []
    for i in range(len(edges) - 1):
        Y = w["torch_s2"][i] - w["torch_s1"][i]
        E1 = w["native_s1"][i] - w["torch_s1"][i]
        E2 = w["native_s2"][i] - w["torch_s2"][i]
        S = w["native_s2"][i] - w["native_s1"][i]
        sigma = abs(Y) / math.sqrt(2.0)              # two-seed estimate of the per-run standard deviation
        rows.append({"window": [edges[i], edges[i + 1]], "Y": Y, "E1": E1, "E2": E2, "S": S,
                     "within_Y": all(abs(x) <= abs(Y) for x in (E1, E2, S)),
                     "mean_native_minus_torch": (E1 + E2) / 2, "two_sigma": 2 * sigma,
                     "within_2sigma": abs((E1 + E2) / 2) <= 2 * sigma})
    return {"windows": rows, "within_2sigma_all": all(r["within_2sigma"] for r in rows)}


def main(argv=None):
    p = argparse.ArgumentParser("parity")
    p.add_argument("--arch", default="yoco_small")
    p.add_argument("--updates", type=int, default=200)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    curves = {}
    for backend in (("native", "torch") if dev.type == "cuda" else ("torch",)):
        for s in (1, 2):
            curves[f"{backend}_s{s}"] = run(a.arch, backend, s, a.updates, a.seq_len, a.batch, dev, a.lr,
                                            data_seed=s)
    n = a.updates
    edges = [0, 5, 15, 25, 35, 50, 100, 200]
    edges = [e for e in edges if e < n] + [n]
    out = {"arch": a.arch, "updates": n, "edges": edges, "curves": curves}
    if "native_s1" in curves:
        out["criterion"] = criterion(curves, edges)
    text = json.dumps(out)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    summary = {k: v for k, v in out.items() if k != "curves"}
    summary["final_loss"] = {k: sum(v[-10:]) / 10 for k, v in curves.items()}
    print(json.dumps(summary), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
