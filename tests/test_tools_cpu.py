"""Data builder, held-out pipeline, validation summary / verdict, performance views, presets (CPU)."""
import gzip
import json
import os

import pytest
import torch

from faster_yoco_b200.data.tokenizers import ByteTokenizer


def _sources(tmp):
    import pyarrow as pa
    import pyarrow.parquet as pq
    fw = os.path.join(tmp, "fw.parquet")
    pq.write_table(pa.table({"text": [f"web document {i} " * 20 if i % 7 else "" for i in range(60)]}), fw)
    cp = os.path.join(tmp, "cp.json.gz")
    with gzip.open(cp, "wt") as f:
        for i in range(30):
            f.write(json.dumps({"content": f"def f{i}():\n    return {i}\n" * 10}) + "\n")
    return fw, cp


def test_build_data_layout(tmp_path):
    from faster_yoco_b200.data import build_data as B
    fw, cp = _sources(str(tmp_path))
    out = str(tmp_path / "out")
    assert B.main(["--source", f"fineweb_edu:{fw}:text:0.8", "--source", f"codeparrot:{cp}:content:0.2",
                   "--lines-per-shard", "20", out]) == 0
    root = os.path.join(out, "Data")
    train = json.load(open(os.path.join(root, "json", "train.json")))
    assert train == [{"name": "fineweb_edu", "weight": 0.8}, {"name": "codeparrot", "weight": 0.2}]
    shards = json.load(open(os.path.join(root, "json", "fineweb_edu.json")))
    assert len(shards) == 3 and all(os.path.isabs(p) for p in shards)     # 51 non-empty docs / 20 per shard
    m = json.load(open(os.path.join(out, "data_manifest.json")))
    assert m["sources"]["fineweb_edu"]["docs"] == 51 and m["sources"]["fineweb_edu"]["skipped_empty"] == 9
    with pytest.raises(ValueError):
        B.build([B.Source("x", fw, "text", 1.0, sha256="0" * 64)], str(tmp_path / "out2"))
    # the GPT task reads it
    from faster_yoco_b200.data.lm_loader import LMLoader
    L = LMLoader(train, root, ByteTokenizer(), tokens_per_sample=32, batch_size=2, prefetch=0, batch_read_ahead=4)
    b = next(L)
    assert b["src_tokens"].shape == (2, 32)


def test_heldout_pipeline(tmp_path):
    from faster_yoco_b200.data import build_data as B
    from faster_yoco_b200.validation import heldout as H
    fw, cp = _sources(str(tmp_path))
    out = str(tmp_path / "out")
    B.build([B.Source("fineweb_edu", fw, "text", 0.8), B.Source("codeparrot", cp, "content", 0.2)], out)
    hd = str(tmp_path / "held")
    r = H.extract(fw, cp, hd, 10, 5)
    assert r["fineweb_edu"] == 10 and r["codeparrot"] == 5
    # every held-out document also occurs in training here -> dedup drops them all
    d = H.dedup(os.path.join(out, "Data"), hd)
    assert d["fineweb_edu"] == {"kept": 0, "dropped": 10}
    assert H.check(os.path.join(out, "Data"), hd)["exact_duplicates_in_training_shards"] == {}
    # restore the originals and pack them
    for n in H.SOURCES:
        os.replace(os.path.join(hd, f"heldout_{n}.jsonl.orig"), os.path.join(hd, f"heldout_{n}.jsonl"))
    res = H.build(hd, os.path.join(hd, "heldout.pt"), 2, 1, ByteTokenizer(), tokens_per_sample=64)
    t = torch.load(os.path.join(hd, "heldout.pt"))
    assert t["samples"]["fineweb_edu"].shape == (2, 65) and t["n_words"] == 264 and t["pad_id"] == 1
    assert int(t["samples"]["codeparrot"][0, 0]) == 0


def _fake_arm(d, offset, updates=4000, evals=(2000, 4000)):
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "train.log"), "w") as f:
        for n in range(10, updates + 1, 10):
            loss = 10.0 / (1 + n / 500) + offset
            f.write(f"epoch 001: loss {loss:.4f} | ppl 1.0 | gnorm 0.5 | num_updates {n} | lr 1e-4 | "
                    f"train_wall {n * 0.08:.1f}\n")
        f.write('VALIDATION_MEM {"rank": 0, "num_updates": 4000, "max_allocated_gib": 61.5}\n')
    ev = {f"model_{k:06d}.pt": {"num_updates": k, "fineweb_edu": {"loss_bits": 3.0 + offset - k / 1e4},
                                "codeparrot": {"loss_bits": 2.0 + offset - k / 1e4},
                                "mix_0.8_0.2_bits": 2.8 + offset - k / 1e4} for k in evals}
    json.dump(ev, open(os.path.join(d, "eval.json"), "w"))


def test_analyze_and_verdict(tmp_path):
    from faster_yoco_b200.validation import analyze, verdict
    V = str(tmp_path)
    for arm, off in (("opt", 0.001), ("ref", 0.0), ("ref_s2", 0.01), ("opt_s2", 0.008)):
        _fake_arm(os.path.join(V, arm), off)
    assert analyze.main([V]) == 0
    S = json.load(open(os.path.join(V, "summary.json")))["arms"]
    assert S["opt"]["updates"] == 4000 and S["opt"]["peak_alloc_gib_max_rank"] == 61.5
    assert abs(S["opt"]["s_per_update_excl_saves"] - 0.08) < 1e-3
    assert verdict.main([V]) == 0
    text = open(os.path.join(V, "verdict.md")).read()
    v = json.loads(text[text.index("{"):])
    assert v["mix"]["checkpoints"] == 2 and v["mix"]["final_within"] is True
    _fake_arm(os.path.join(V, "opt"), 0.05)                    # far off: no longer within the seed yardstick
    analyze.main([V])
    verdict.main([V])
    text = open(os.path.join(V, "verdict.md")).read()
    assert json.loads(text[text.index("{"):])["mix"]["final_within"] is False


def test_perf_views(tmp_path):
    from faster_yoco_b200.utils import perf_views as P
    json.dump([{"label": "a", "ms_per_update": 100.0}, {"label": "b", "ms_per_update": 50.0, "n_gpus": 8}],
              open(tmp_path / "history.json", "w"))
    json.dump({"phases": [["gemm", 30], ["adam", 10]]}, open(tmp_path / "time-budget.json", "w"))
    json.dump({"arms": {"opt": {"updates": [1, 2, 3], "loss": [3, 2, 1]}}}, open(tmp_path / "validation.json", "w"))
    out = P.render(str(tmp_path), str(tmp_path / "svg"))
    assert len(out) == 3
    for p in out:
        s = open(p).read()
        assert s.startswith("<svg") and s.rstrip().endswith("</svg>")
    assert "75.0%" in open(out[1]).read()


def test_presets_and_parse():
    from faster_yoco_b200.cli.options import load_preset, parse_with_preset, train_parser
    assert load_preset("b200_fused")["comm"] == "fused"
    a = parse_with_preset(train_parser(), ["--preset", "torch_baseline", "DATA"])
    assert a.kernels == "torch" and a.comm == "nccl" and a.cuda_graph is False and a.partition == "greedy"
    a = parse_with_preset(train_parser(), ["--preset", "torch_baseline", "--comm", "fused", "DATA"])
    assert a.comm == "fused"
    a = parse_with_preset(train_parser(), ["DATA", "--adam-betas", "(0.9, 0.98)", "--lr", "3e-4"])
    assert a.adam_betas == (0.9, 0.98) and a.lr == [3e-4]


def test_parity_markov_data_and_criterion():
    import math
    from faster_yoco_b200.validation.parity import MarkovLM, criterion
    d = MarkovLM(64, 16, 3, data_seed=5)
    b = next(d)
    assert b["src_tokens"].shape == (3, 16) and torch.equal(b["src_tokens"][:, 1:], b["target"][:, :-1])
    assert int(b["src_tokens"].min()) >= 2 and 0 < d.entropy_nats() < math.log(4) + 1e-6
    # every transition is one of the chain's successors
    src, tgt = b["src_tokens"].reshape(-1), b["target"].reshape(-1)
    assert all(int(t) in d.next[int(s)].tolist() for s, t in zip(src, tgt))
    curves = {"torch_s1": [3.0] * 10, "torch_s2": [3.2] * 10, "native_s1": [3.05] * 10, "native_s2": [3.22] * 10}
    r = criterion(curves, [0, 5, 10])
    assert r["windows"][0]["within_Y"] and r["within_2sigma_all"]
    curves["native_s1"] = [4.0] * 10
    assert not criterion(curves, [0, 5, 10])["windows"][0]["within_Y"]


def _bench():
    import importlib.util
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("fyb_bench", os.path.join(root, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _FakeNVML:
    """Two NVML devices; the one the CUDA process sees is NVML device 1."""

    def __init__(self, uuid_ok=True, pci_ok=True):
        self.uuid_ok, self.pci_ok = uuid_ok, pci_ok

    def nvmlDeviceGetHandleByUUID(self, u):
        if not self.uuid_ok or u != "GPU-1234abcd-0000-0000-0000-000000000001":
            raise RuntimeError("not found")
        return "dev1"

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        if not self.pci_ok or bus != "00000000:1b:00.0":
            raise RuntimeError("not found")
        return "dev1"

    def nvmlDeviceGetHandleByIndex(self, i):
        return "dev%d" % i


class _FakeNVMLEnum(_FakeNVML):
    """Direct lookups fail; enumeration finds the device by its UUID (bytes, upper case) or PCI address."""

    def __init__(self, by_uuid=True):
        super().__init__(uuid_ok=False, pci_ok=False)
        self.by_uuid = by_uuid

    def nvmlDeviceGetCount(self):
        return 2

    def nvmlDeviceGetUUID(self, h):
        return b"GPU-1234ABCD-0000-0000-0000-000000000001" if (h == "dev1" and self.by_uuid) else b"GPU-other"

    def nvmlDeviceGetPciInfo(self, h):
        class Info:
            domain, bus, device = (0, 0x1B, 0) if h == "dev1" else (0, 0x2C, 0)
        return Info()


class _Props:
    uuid = "1234abcd-0000-0000-0000-000000000001"
    pci_domain_id, pci_bus_id, pci_device_id = 0, 0x1B, 0


def test_bench_clock_sampler_maps_visible_device(monkeypatch):
    """The clock sampler must read the GPU that the process runs on, not NVML's device with the same index."""
    bench = _bench()
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "1")
    assert bench.nvml_handle(_FakeNVML(), _Props(), 0) == "dev1"
    assert bench.nvml_handle(_FakeNVML(uuid_ok=False), _Props(), 0) == "dev1"
    with pytest.raises(RuntimeError):
        bench.nvml_handle(_FakeNVML(uuid_ok=False, pci_ok=False), _Props(), 0)
    assert bench.nvml_handle(_FakeNVMLEnum(True), _Props(), 0) == "dev1"
    assert bench.nvml_handle(_FakeNVMLEnum(False), _Props(), 0) == "dev1"
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.nvml_handle(_FakeNVML(uuid_ok=False, pci_ok=False), _Props(), 0) == "dev0"


def test_bench_reference_arm_line(capsys, monkeypatch):
    bench = _bench()
    monkeypatch.setenv("RANK", "0")
    assert bench.reference_arm(None) == 0
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference" and line["unavailable"]


def test_bench_merge_clocks():
    bench = _bench()
    one = {"sm_mhz": 1900, "sm_max_mhz": 1965, "reasons": ["sw_power_cap"], "samples": 10}
    assert bench.merge_clocks([one])["sm_mhz"] == 1900 and "per_rank_sm_mhz" not in bench.merge_clocks([one])
    two = {"sm_mhz": 1500, "sm_max_mhz": 1965, "reasons": ["hw_slowdown"], "samples": 9}
    m = bench.merge_clocks([one, two, one])
    assert m["sm_mhz"] == 1900 and m["per_rank_sm_mhz"] == [1900, 1500, 1900]
    assert m["reasons"] == ["hw_slowdown", "sw_power_cap"] and m["samples"] == 29


def test_bench_result_line_contract(monkeypatch):
    """Every key of the benchmark line the driver reads, with the right types (no GPU needed to assemble it)."""
    import sys
    bench = _bench()
    monkeypatch.setattr(sys, "argv", ["bench.py", "--steps", "7", "--warmup", "2"])
    args = bench.parse()
    args.overlap = 0
    clocks = bench.merge_clocks([{"sm_mhz": 1900, "sm_max_mhz": 1965, "reasons": ["sw_power_cap"], "samples": 5}])
    e2e = {"value": 28000.0, "unit": "tokens/s", "ms_per_step": 73.0, "h2d_bytes_per_step": 32768,
           "d2h_bytes_per_step": 4}
    out = bench.result_line(args, 8, 70.0, clocks, e2e, 8000)
    line = json.loads(json.dumps(out))
    for k, t in (("metric", str), ("value", float), ("unit", str), ("n_gpus", int), ("steps", int),
                 ("warmup", int), ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str),
                 ("vs_baseline", float), ("dtype", str), ("data", str), ("config", dict), ("clocks", dict),
                 ("e2e", dict), ("gpu_launches", int)):
        assert isinstance(line[k], t), k
    assert line["warmup"] >= 3 and line["steps"] == 7 and line["n_gpus"] == 8 and line["scaling"] == "weak"
    assert abs(line["value"] - 8 * 2048 / 0.070) < 1e-6 * line["value"]
    assert abs(line["vs_baseline"] - line["value"] / 138983.0) < 1e-9      # N = 8: whole job vs whole job
    one = bench.result_line(args, 1, 70.0, clocks, e2e, 8000)             # N = 1: per GPU vs per GPU
    assert abs(one["vs_baseline"] - one["value"] / (138983.0 / 8)) < 1e-9
    assert one["config"]["comm"] == "none" and one["config"]["transport"] is None
    assert line["config"]["transport"] == "serial"                         # N = 8, no overlap: the serial exchange
    args.transport = "pull"
    assert bench.result_line(args, 8, 70.0, clocks, e2e, 8000)["config"]["transport"] == "pull"
    for k in ("model", "global_batch", "seq_len", "parallelism", "l2"):
        assert k in line["config"], k
    assert line["config"]["model"] == "yoco_3b" and line["config"]["global_batch"] == 8
    for k in ("sm_mhz", "sm_max_mhz", "reasons"):
        assert k in line["clocks"], k
    for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"):
        assert k in line["e2e"], k
    assert line["metric"] == json.load(open(os.path.join(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__))), "BASELINE.json")))["metric"]


def test_reference_recipe_command_lines_parse():
    """The reference's training and evaluation command lines (scripts/train.sh, eval_task.sh, eval_needle.sh) are
    accepted unchanged."""
    from faster_yoco_b200.cli.options import train_parser, validate_parser
    a = train_parser().parse_args([
        "DATA", "--save-interval-updates", "5000", "--no-epoch-checkpoints", "--arch", "yoco_base", "--criterion",
        "cross_entropy", "--task", "gpt", "--tokens-per-sample", "2048", "--tokenizer-pad-to-multiple", "8",
        "--pad-to-max-len", "--optimizer", "adam", "--adam-betas", "(0.9, 0.95)", "--adam-eps", "1e-06",
        "--clip-norm", "2.0", "--lr", "0.00015", "--lr-scheduler", "polynomial_decay", "--warmup-updates", "50",
        "--weight-decay", "0.05", "--batch-size", "1", "--model-parallel-size", "1", "--update-freq", "1",
        "--batch-read-ahead", "1000", "--total-num-update", "300000", "--log-format", "simple", "--log-interval", "10",
        "--disable-validation", "--tiktoken-model", "cl100k_base", "--no-save", "--bf16", "--zero-sharding", "os"])
    assert a.adam_betas == (0.9, 0.95) and a.clip_norm == 2.0 and a.total_num_update == 300000
    v = validate_parser()
    v.parse_args(["--data-dir", "hd/", "--criterion", "harness_eval", "--task", "harness_eval", "--batch-size", "4",
                  "--eval-data", "harness_boolq", "--log-format", "simple", "--log-interval", "10", "--bf16",
                  "--tokenizer-pad-to-multiple", "8", "--arch", "yoco_3b_new", "--tiktoken-model", "cl100k_base",
                  "--load-ckpt", "c/checkpoint.pth", "--yoco-model", "c", "--tokens-per-sample", "4096"])
    v.parse_args(["--arch", "llama_from_ckpt", "--llama-model", "l", "--load-ckpt", "l/consolidated.00.pth",
                  "--tokens-per-sample", "4096", "--task", "harness_eval", "--criterion", "harness_eval"])
    v.parse_args(["--task", "pseudo", "--criterion", "multi_needle", "--needle-num", "4", "--batch-size", "1",
                  "--max-epoch", "1", "--no-save", "--tiktoken-model", "cl100k_base", "--bf16", "--arch", "yoco_3b_new",
                  "--load-ckpt", "c/c.pth", "--yoco-model", "c", "--tokens-per-sample", "1048576", "--interval",
                  "1048576"])


def test_every_module_imports():
    """Every module of the package (tools that only run on GPU boxes included) imports on a CPU machine."""
    import importlib
    import pkgutil
    import faster_yoco_b200
    failed = []
    for m in pkgutil.walk_packages(faster_yoco_b200.__path__, "faster_yoco_b200."):
        try:
            importlib.import_module(m.name)
        except Exception as e:          # pragma: no cover - the assertion below reports it
            failed.append((m.name, repr(e)))
    assert not failed, failed


def test_log_formats():
    from faster_yoco_b200.train.metrics import format_log
    st = {"loss": 3.14159, "num_updates": 10}
    assert format_log(st).startswith("epoch 001: loss 3.14159 | num_updates 10")
    assert json.loads(format_log(st, fmt="json")) == {"epoch": 1, "loss": 3.1416, "num_updates": 10}
    assert format_log(st, fmt="none") == "" and format_log(st, fmt="tqdm") == format_log(st)


def test_every_preset_parses():
    """Each switch set in presets/ applies to the train parser with values its choices accept."""
    import glob
    from faster_yoco_b200.cli.options import parse_with_preset, train_parser
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    names = sorted(os.path.splitext(os.path.basename(f))[0]
                   for f in glob.glob(os.path.join(root, "faster_yoco_b200", "presets", "*.json")))
    assert "b200_gemm_scatter" in names and len(names) >= 5
    for n in names:
        a = parse_with_preset(train_parser(), ["--preset", n, "DATA"])
        assert a.comm in ("fused", "nccl") and a.partition in ("even", "greedy", "cyclic"), n
