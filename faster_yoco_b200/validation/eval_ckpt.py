"""Held-out loss of model-only checkpoints (scripts/validate/eval_ckpt.py of the reference), identical code for
every arm: rank 0 reads each checkpoint and broadcasts every tensor; samples are split across ranks; the loss is the
fp32 log-softmax cross-entropy of the next token averaged over non-pad targets, sums all-reduced in float64; the mix
is 0.8 fineweb + 0.2 code (bits).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m faster_yoco_b200.validation.eval_ckpt \\
        heldout.pt eval.json ckpt/model_*.pt [--arch yoco_3b]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import torch
import torch.nn.functional as F

from .. import ops
from ..config import build_args
from ..models.yoco import YOCO
from ..parallel import dist as D

PREFIX = "decoder.model."


def evaluate(model, samples: torch.Tensor, pad_id: int, device, rank: int, world: int):
    tot = torch.zeros(2, dtype=torch.float64, device=device)
    with torch.no_grad():
        for i in range(rank, samples.shape[0], world):
            s = samples[i].to(device)
            logits, _ = model(s[None, :-1])
            lp = F.log_softmax(logits.float(), dim=-1)
            nll = F.nll_loss(lp.view(-1, lp.shape[-1]), s[1:], ignore_index=pad_id, reduction="sum")
            tot += torch.stack([nll.double(), (s[1:] != pad_id).sum().double()])
    if D.is_dist():
        torch.distributed.all_reduce(tot)
    return {"loss_nats": float(tot[0] / tot[1]), "loss_bits": float(tot[0] / tot[1] / math.log(2)),
            "tokens": int(tot[1])}


def main(argv=None):
    p = argparse.ArgumentParser("eval_ckpt")
    p.add_argument("heldout"), p.add_argument("out"), p.add_argument("ckpts", nargs="+")
    p.add_argument("--arch", default="yoco_3b")
    p.add_argument("--kernels", default="native", choices=["native", "torch"])
    a = p.parse_args(argv)
    dev_index = D.init()
    rank, world = D.rank(), D.world()
    device = torch.device("cuda", dev_index) if dev_index >= 0 else torch.device("cpu")
    ops.set_backend(a.kernels if device.type == "cuda" else "torch")
    H = torch.load(a.heldout)
    args = build_args(a.arch, vocab_size=H["n_words"], max_batch_size=1, max_seq_len=H["tokens_per_sample"])
    with torch.device(device):
        model = YOCO(args)
    model = model.to(torch.bfloat16 if device.type == "cuda" else torch.float32).eval()
    results = json.load(open(a.out)) if os.path.exists(a.out) else {}
    for ck in a.ckpts:
        name = os.path.basename(ck)
        if name in results:
            continue
        t0 = time.time()
        meta = [None]
        st = None
        if rank == 0:
            sd = torch.load(ck, map_location="cpu")
            st = {k[len(PREFIX):] if k.startswith(PREFIX) else k: v for k, v in sd["model"].items()}
            model.load_state_dict(st)
            meta = [sd.get("num_updates")]
        if D.is_dist():
            torch.distributed.broadcast_object_list(meta, src=0)
            with torch.no_grad():
                for t in list(model.parameters()) + list(model.buffers()):
                    torch.distributed.broadcast(t.data, src=0)
        r = {"num_updates": meta[0], "load_s": time.time() - t0}
        for src, data in H["samples"].items():
            r[src] = evaluate(model, data, H["pad_id"], device, rank, world)
        if "fineweb_edu" in r and "codeparrot" in r:
            r["mix_0.8_0.2_bits"] = 0.8 * r["fineweb_edu"]["loss_bits"] + 0.2 * r["codeparrot"]["loss_bits"]
        r["eval_s"] = time.time() - t0
        results[name] = r
        if rank == 0:
            print("EVAL", name, json.dumps(r), flush=True)
            with open(a.out, "w") as f:
                json.dump(results, f, indent=1)
    D.destroy()
    return 0


if __name__ == "__main__":
    sys.exit(main())
