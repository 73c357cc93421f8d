"""Checkpoints in the fairseq layout the reference's tooling reads.

File content (one ``torch.save`` dict, written by rank 0):

* ``model``: the BF16 model state dict with the reference's parameter names under the ``decoder.model.`` prefix
  (``LanguageModel.decoder = YOCOModel``, ``YOCOModel.model = YOCO``; the merged projections of this framework are
  split back into ``q_proj`` / ``k_proj`` / ... by the model's state-dict hook);
* ``optimizer_history``: ``[{criterion_name, optimizer_name, lr_scheduler_state, num_updates}]``;
* ``extra_state``: ``{train_iterator, previous_training_time, metrics}``;
* ``last_optimizer_state``: the CONSOLIDATED FP32 Adam state per reference parameter name
  (``{"master": {name: fp32}, "exp_avg": {...}, "exp_avg_sq": {...}, "step": n}``), gathered from the ZeRO owners.

Because the optimizer state is stored per parameter, a checkpoint written with one world size resumes with another
(the owners re-slice it through the partition of the resuming run). The reference never saved or resumed full
checkpoints with its switches on (docs/training.md:88-90); fairseq's own layout is kept so that model-only
consumers (yoco/models/yoco.py:106-121, scripts/validate/eval_ckpt.py:35) load these files.
"""
from __future__ import annotations

import os
import time
from typing import Dict, Optional

import torch
import torch.distributed as dist

PREFIX = "decoder.model."


def _core(model):
    """(module whose state dict goes under ``decoder.model.``, prefix of its parameter names inside `model`):
    the LLaMA task wrapper holds the Transformer as ``.model`` (reference: LanguageModel.decoder = LLaMA,
    LLaMA.model = Transformer, so its keys are ``decoder.model.layers...``)."""
    from ..models.transformer import LLaMA
    if isinstance(model, LLaMA):
        return model.model, "model."
    return model, ""


def _split_for_export(model, name: str, t: torch.Tensor) -> Dict[str, torch.Tensor]:
    """Internal parameter name -> {reference name: slice} (identity for unmerged parameters)."""
    from ..models.layers import MergedLinear
    mod_name, _, leaf = name.rpartition(".")
    mod = model.get_submodule(mod_name) if mod_name else model
    if isinstance(mod, MergedLinear) and leaf == "weight":
        parent = mod_name.rpartition(".")[0]
        out = {}
        for (off, n), sub in zip(mod.offsets(), mod.names):
            out[(parent + "." if parent else "") + sub + ".weight"] = t[off:off + n]
        return out
    return {name: t}


def _join_for_import(model, name: str, entries: Dict[str, torch.Tensor]) -> Optional[torch.Tensor]:
    """Inverse of _split_for_export for one internal parameter; None if a piece is missing."""
    from ..models.layers import MergedLinear
    mod_name, _, leaf = name.rpartition(".")
    mod = model.get_submodule(mod_name) if mod_name else model
    if isinstance(mod, MergedLinear) and leaf == "weight":
        parent = mod_name.rpartition(".")[0]
        keys = [(parent + "." if parent else "") + sub + ".weight" for sub in mod.names]
        if not all(k in entries for k in keys):
            return None
        w = torch.cat([entries[k] for k in keys], 0)
        if w.shape[0] < mod.rows:
            w = torch.cat([w, w.new_zeros(mod.rows - w.shape[0], *w.shape[1:])], 0)
        return w
    return entries.get(name)


def part_path(path: str) -> str:
    """Tensor parallelism: each TP rank's slice goes to its own file, fairseq's `<name>-model_part-<tp_rank>.pt`."""
    from ..parallel import tp as TP
    if TP.tp_size() <= 1:
        return path
    base, ext = os.path.splitext(path)
    return f"{base}-model_part-{TP.tp_rank()}{ext or '.pt'}"


def save_checkpoint(path: str, model, trainer, *, extra_state: Optional[dict] = None, cfg: Optional[dict] = None,
                    rank: Optional[int] = None):
    """Collective (every rank must call): gathers the optimizer state, rank 0 of the data-parallel group writes
    `path` (with tensor parallelism: one part file per TP rank, see part_path)."""
    rank = trainer.rank if rank is None else rank
    path = part_path(path)
    # the overlapped and the pull exchanges gather parameters lazily (at the next forward): make them current first
    if hasattr(trainer, "sync_params"):
        trainer.sync_params()
    opt = trainer.zero.consolidated_state()            # {internal name: {master, exp_avg, exp_avg_sq}}
    if rank != 0:
        return None
    core, strip = _core(model)
    state = {"master": {}, "exp_avg": {}, "exp_avg_sq": {}, "step": trainer.zero.num_updates}
    for name, st in opt.items():
        for key in ("master", "exp_avg", "exp_avg_sq"):
            for ref_name, t in _split_for_export(model, name, st[key]).items():
                state[key][ref_name[len(strip):] if strip and ref_name.startswith(strip) else ref_name] = t.clone()
    msd = {PREFIX + k: v.detach().cpu() for k, v in core.state_dict().items()}
    ckpt = {
        "args": None,
        "cfg": cfg or {},
        "model": msd,
        "optimizer_history": [{
            "criterion_name": "CrossEntropyCriterion",
            "optimizer_name": "FP16Optimizer",
            "lr_scheduler_state": trainer.sched.state_dict(),
            "num_updates": trainer.zero.num_updates,
        }],
        "extra_state": dict({"previous_training_time": 0.0, "train_iterator": None, "saved_at": time.time()},
                            **(extra_state or {})),
        "last_optimizer_state": state,
    }
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    torch.save(ckpt, tmp)
    os.replace(tmp, path)
    return path


def load_model_weights(model, path_or_ckpt, strict: bool = True):
    """Model-only load (accepts a full checkpoint or a bare reference-named state dict, with/without prefix)."""
    ck = torch.load(path_or_ckpt, map_location="cpu", mmap=True) if isinstance(path_or_ckpt, str) else path_or_ckpt
    sd = ck.get("model", ck) if isinstance(ck, dict) else ck
    sd = {(k[len(PREFIX):] if k.startswith(PREFIX) else k): v for k, v in sd.items()}
    core, _ = _core(model)
    with torch.no_grad():
        missing, unexpected = core.load_state_dict(sd, strict=strict)
    return ck


def load_checkpoint(path: str, model, trainer, reset_lr_scheduler: bool = False) -> dict:
    """Restore model weights, this rank's optimizer shard, the update count and (unless reset_lr_scheduler) the LR
    schedule."""
    ck = load_model_weights(model, part_path(path))
    _, strip = _core(model)
    st = ck.get("last_optimizer_state") or {}
    zero = trainer.zero
    fp = trainer.flat
    with torch.no_grad():
        for e in fp.entries:
            for off, cnt, owner in fp.owner_ranges(e):
                if owner != fp.rank:
                    continue
                lo = fp.local_of(off)           # position in this rank's shard (a piece is contiguous there)
                pe = off - e.offset             # position inside the parameter
                for key, dst in (("master", zero.master), ("exp_avg", zero.exp_avg),
                                 ("exp_avg_sq", zero.exp_avg_sq)):
                    entries = st.get(key, {})
                    if strip:
                        entries = {strip + k: v for k, v in entries.items()}
                    t = _join_for_import(model, e.name, entries)
                    if t is None:
                        if key == "master":
                            dst[lo:lo + cnt].copy_(e.param.detach().reshape(-1)[pe:pe + cnt].float())
                        continue
                    dst[lo:lo + cnt].copy_(t.reshape(-1)[pe:pe + cnt].to(dst.device, torch.float32))
    zero.num_updates = int(st.get("step", ck["optimizer_history"][-1]["num_updates"] if ck.get("optimizer_history")
                                      else 0))
    hist = ck.get("optimizer_history") or []
    if hist and "lr_scheduler_state" in hist[-1] and not reset_lr_scheduler:
        trainer.sched.load_state_dict(hist[-1]["lr_scheduler_state"])
    if dist.is_initialized():
        dist.barrier()
    return ck


def prune_interval_checkpoints(save_dir: str, keep: int) -> list:
    """fairseq's --keep-interval-updates: delete all but the newest `keep` checkpoint_1_<update>.pt files (and their
    tensor-parallel part files). Returns the removed paths."""
    import re
    if keep < 0 or not os.path.isdir(save_dir):
        return []
    pat = re.compile(r"^checkpoint_1_(\d+)(-model_part-\d+)?\.pt$")
    found = {}
    for f in os.listdir(save_dir):
        m = pat.match(f)
        if m:
            found.setdefault(int(m.group(1)), []).append(os.path.join(save_dir, f))
    removed = []
    for nu in sorted(found)[:max(0, len(found) - keep)]:
        for p in found[nu]:
            os.remove(p)
            removed.append(p)
    return removed
