"""Command-line options with the reference's fairseq flag names (scripts/train.sh, scripts/train_faster_yoco_3b.sh,
scripts/eval_task.sh, scripts/eval_needle.sh), plus this framework's own switches (``--comm``, ``--kernels``,
``--cuda-graph``, ``--overlap``, ``--partition``) in place of the reference's ``YOCO_*`` environment switches."""
from __future__ import annotations

import argparse
import ast


def _betas(s: str):
    v = ast.literal_eval(s)
    return tuple(float(x) for x in v)


def _bool_int(s: str) -> bool:
    return str(s).lower() in ("1", "true", "yes", "on")


def add_common(p: argparse.ArgumentParser):
    g = p.add_argument_group("task / model")
    g.add_argument("--task", default="gpt")
    g.add_argument("--criterion", default="cross_entropy")
    g.add_argument("--arch", default="yoco_3b")
    g.add_argument("--tokens-per-sample", type=int, default=2048)
    g.add_argument("--max-target-positions", type=int, default=None)
    g.add_argument("--tokenizer-pad-to-multiple", type=int, default=8)
    g.add_argument("--tiktoken-model", default=None, help="encoding name, .tiktoken file, or 'byte'")
    g.add_argument("--llama-model", default=None)
    g.add_argument("--yoco-model", default=None, help="directory holding params.json")
    g.add_argument("--load-ckpt", default=None)
    g.add_argument("--batch-size", type=int, default=1)
    g.add_argument("--model-parallel-size", type=int, default=1)
    g.add_argument("--context-parallel-size", type=int, default=1,
                   help="split every sequence into this many contiguous blocks, one per rank (YOCO)")
    g.add_argument("--seed", type=int, default=1)
    g.add_argument("--bf16", action="store_true")
    g.add_argument("--fp16", action="store_true")
    g.add_argument("--cpu", action="store_true")
    g.add_argument("--sliding-window", type=int, default=None)
    g.add_argument("--checkpoint-activations", action="store_true")
    g.add_argument("--share-input-output-embed", action="store_true")
    g.add_argument("--rope-theta", type=float, default=None)
    for k in ("dim", "hidden-dim", "n-layers", "n-self-heads", "n-attn-heads", "n-attn-kv-heads", "n-heads",
              "n-kv-heads"):
        g.add_argument(f"--{k}", type=int, default=None)
    g.add_argument("--init-std", type=float, default=None, help="N(0, std) for every weight (benchmark init)")
    g.add_argument("--log-format", default="simple", choices=["simple", "json", "tqdm", "none"])
    g.add_argument("--log-interval", type=int, default=10)
    g.add_argument("--kernels", default="native", choices=["native", "torch"])
    # data
    g.add_argument("--batch-read-ahead", type=int, default=10000)
    g.add_argument("--pad-to-max-len", action="store_true")
    g.add_argument("--absolute-path", action="store_true")
    # harness / needle evaluation
    g.add_argument("--data-dir", default=None)
    g.add_argument("--eval-data", default="")
    g.add_argument("--needle-num", type=int, default=4)
    g.add_argument("--interval", type=int, default=1024)
    g.add_argument("--needle-file-path", default=None)
    g.add_argument("--max-len-b", type=int, default=5,
                   help="accepted as in the reference's needle criterion config, which never reads it either: the "
                        "needle criterions generate 20 tokens")
    return p


def load_preset(name: str) -> dict:
    """A named switch set (``faster_yoco_b200/presets/<name>.json``, or a path): {"args": {dest: value}}."""
    import json
    import os
    path = name if os.path.exists(name) else os.path.join(os.path.dirname(os.path.dirname(__file__)), "presets",
                                                           name + ".json")
    with open(path) as f:
        return json.load(f).get("args", {})


def parse_with_preset(parser: argparse.ArgumentParser, argv=None):
    """--preset NAME supplies defaults; flags given on the command line still win."""
    pre = argparse.ArgumentParser(add_help=False)
    pre.add_argument("--preset", default=None)
    known, _ = pre.parse_known_args(argv)
    if known.preset:
        parser.set_defaults(**load_preset(known.preset))
    return parser.parse_args(argv)


def train_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser("faster_yoco_b200 train")
    p.add_argument("--preset", default=None, help="named switch set (presets/*.json)")
    p.add_argument("data", nargs="?", default=None)
    add_common(p)
    g = p.add_argument_group("optimization")
    g.add_argument("--optimizer", default="adam", choices=["adam"])
    g.add_argument("--adam-betas", type=_betas, default=(0.9, 0.95))
    g.add_argument("--adam-eps", type=float, default=1e-6)
    g.add_argument("--weight-decay", type=float, default=0.05)
    g.add_argument("--clip-norm", type=float, default=2.0)
    g.add_argument("--lr", type=float, nargs="+", default=[1.5e-4])
    g.add_argument("--lr-scheduler", default="polynomial_decay", choices=["polynomial_decay"])
    g.add_argument("--warmup-updates", type=int, default=50)
    g.add_argument("--total-num-update", type=int, default=300000)
    g.add_argument("--end-learning-rate", type=float, default=0.0)
    g.add_argument("--power", type=float, default=1.0)
    g.add_argument("--max-update", type=int, default=0)
    g.add_argument("--update-freq", type=int, default=1)
    g.add_argument("--zero-sharding", default="os", choices=["none", "os"])
    g = p.add_argument_group("checkpointing")
    g.add_argument("--save-dir", default="checkpoints")
    g.add_argument("--save-interval-updates", type=int, default=0)
    g.add_argument("--no-save", action="store_true")
    g.add_argument("--no-epoch-checkpoints", action="store_true")
    g.add_argument("--restore-file", default="checkpoint_last.pt")
    g.add_argument("--reset-optimizer", action="store_true")
    g.add_argument("--reset-dataloader", action="store_true")
    g.add_argument("--reset-lr-scheduler", action="store_true",
                   help="resume without the checkpoint's learning-rate schedule state")
    g.add_argument("--reset-meters", action="store_true",
                   help="fairseq compatibility: meters are never restored from a checkpoint here")
    g.add_argument("--keep-interval-updates", type=int, default=-1,
                   help="keep only the last N checkpoint_1_<update>.pt files (-1: keep all)")
    g.add_argument("--disable-validation", action="store_true")
    g.add_argument("--validate-interval-updates", type=int, default=0,
                   help="evaluate the valid subset every N updates (0: only after the last update)")
    g.add_argument("--valid-subset", default="valid")
    g.add_argument("--max-valid-steps", type=int, default=100)
    g.add_argument("--save-model-only", action="store_true",
                   help="paired-validation saves: bf16 model state dict model_<update>.pt on rank 0 (no optimizer "
                        "state) at every save point, plus each rank's peak memory as a VALIDATION_MEM line")
    g = p.add_argument_group("B200 execution")
    g.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                   help="fused: NVLink peer-memory reduce/all-gather kernels; nccl: the NCCL baseline path")
    g.add_argument("--cuda-graph", type=_bool_int, default=True, help="capture each update as one CUDA graph")
    g.add_argument("--overlap", default="auto",
                   help="overlap the ZeRO exchange with forward/backward: auto (the measured schedule of the GPU "
                        "count), 1 (gradients and parameters per layer bucket), grads (gradients per bucket during "
                        "backward, parameters by the fused Adam + push) or 0 (serial)")
    g.add_argument("--transport", default="auto", choices=["auto", "sm", "ce", "gemm", "pull"],
                   help="overlapped pushes by kernels (sm) or by the copy engines (ce); gemm: serial schedule whose "
                        "weight-gradient GEMMs store each element at its ZeRO owner (GEMM fused with the "
                        "reduce-scatter); pull: the parameter all-gather fused into the consuming forward GEMMs "
                        "(use with --partition cyclic)")
    g.add_argument("--partition", default="even", choices=["even", "greedy", "cyclic"],
                   help="ZeRO owner map: even contiguous split, the fairscale OSS greedy per-parameter split, or "
                        "block-cyclic chunks (every weight spread over all owners)")
    g.add_argument("--zero-chunk", type=int, default=None, help="chunk size (elements) of --partition cyclic")
    return p


def validate_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser("faster_yoco_b200 validate")
    p.add_argument("data", nargs="?", default=None)
    add_common(p)
    p.add_argument("--valid-subset", default="valid")
    p.add_argument("--max-epoch", type=int, default=1)
    p.add_argument("--no-save", action="store_true")
    p.add_argument("--profile", action="store_true", help="emit NVTX ranges for an external profiler")
    p.add_argument("--max-valid-steps", type=int, default=None)
    return p
