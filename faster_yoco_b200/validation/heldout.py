"""Held-out set for the paired training validation (scripts/validate/extract_heldout.py, dedup_heldout.py,
check_disjoint.py, build_heldout.py of the reference).

    python -m faster_yoco_b200.validation.heldout extract FINEWEB.parquet CODEPARROT.json.gz OUT_DIR 3000 800
    python -m faster_yoco_b200.validation.heldout dedup DATA_ROOT OUT_DIR
    python -m faster_yoco_b200.validation.heldout check DATA_ROOT OUT_DIR
    python -m faster_yoco_b200.validation.heldout build OUT_DIR OUT_DIR/heldout.pt 800 200 [--tiktoken-model cl100k_base]

``extract`` keeps the first non-empty documents of two files the training corpus does not use; ``dedup`` drops
held-out documents whose exact text (sha1) occurs in a training shard (the original file is kept as ``.orig``);
``check`` reports the remaining exact duplicates (zero after dedup); ``build`` tokenises and packs the documents with
the training loader's own functions (``doc_to_ids`` + ``pack``) into ``tokens_per_sample + 1``-token samples and keeps
the first n per source.
"""
from __future__ import annotations

import argparse
import glob
import gzip
import hashlib
import json
import os
import sys
from typing import Dict, Iterator

SOURCES = ("fineweb_edu", "codeparrot")


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def _text_sha1(text: str) -> str:
    return hashlib.sha1(text.encode()).hexdigest()


def parquet_texts(path: str, column: str = "text") -> Iterator[str]:
    import pyarrow.parquet as pq
    for batch in pq.ParquetFile(path).iter_batches(batch_size=1024, columns=[column]):
        yield from batch.column(0).to_pylist()


def jsonl_gz_texts(path: str, field: str = "content") -> Iterator[str]:
    opener = gzip.open if path.endswith(".gz") else open
    with opener(path, "rt", encoding="utf-8") as f:
        for line in f:
            yield json.loads(line)[field]


def _write_first(texts: Iterator[str], path: str, n: int) -> int:
    k = 0
    with open(path, "w") as f:
        for t in texts:
            if k >= n:
                break
            if t:
                f.write(json.dumps({"text": t}) + "\n")
                k += 1
    return k


def extract(fineweb: str, codeparrot: str, out_dir: str, n_fw: int, n_cp: int) -> Dict:
    os.makedirs(out_dir, exist_ok=True)
    res = {}
    p_fw = os.path.join(out_dir, "heldout_fineweb_edu.jsonl")
    p_cp = os.path.join(out_dir, "heldout_codeparrot.jsonl")
    res["fineweb_edu"] = _write_first(parquet_texts(fineweb), p_fw, n_fw)
    res["codeparrot"] = _write_first(jsonl_gz_texts(codeparrot), p_cp, n_cp)
    for p in (fineweb, codeparrot, p_fw, p_cp):
        res[os.path.basename(p)] = _sha256(p)
    return res


def _training_hashes(data_root: str):
    seen = set()
    for f in sorted(glob.glob(os.path.join(data_root, "shard", "*", "*.jsonl"))):
        with open(f) as fh:
            for line in fh:
                seen.add(_text_sha1(json.loads(line)["text"]))
    return seen


def dedup(data_root: str, heldout_dir: str) -> Dict:
    train = _training_hashes(data_root)
    res = {}
    for name in SOURCES:
        p = os.path.join(heldout_dir, f"heldout_{name}.jsonl")
        if not os.path.exists(p + ".orig"):
            os.rename(p, p + ".orig")
        kept = dropped = 0
        with open(p + ".orig") as src, open(p, "w") as out:
            for line in src:
                if _text_sha1(json.loads(line)["text"]) in train:
                    dropped += 1
                else:
                    out.write(line)
                    kept += 1
        res[name] = {"kept": kept, "dropped": dropped}
    return res


def check(data_root: str, heldout_dir: str) -> Dict:
    held = {}
    for name in SOURCES:
        with open(os.path.join(heldout_dir, f"heldout_{name}.jsonl")) as f:
            for line in f:
                held[_text_sha1(json.loads(line)["text"])] = name
    hits: Dict[str, int] = {}
    for h in _training_hashes(data_root):
        if h in held:
            hits[held[h]] = hits.get(held[h], 0) + 1
    return {"heldout_docs": len(held), "exact_duplicates_in_training_shards": hits}


def build(heldout_dir: str, out_path: str, n_fw: int, n_cp: int, tokenizer, tokens_per_sample: int = 2048) -> Dict:
    import torch
    from ..data.lm_loader import doc_to_ids, pack
    res, samples = {}, {}
    for name, want in (("fineweb_edu", n_fw), ("codeparrot", n_cp)):
        pieces = []
        with open(os.path.join(heldout_dir, f"heldout_{name}.jsonl")) as f:
            for line in f:
                text = json.loads(line)["text"]
                if text:
                    pieces.extend(doc_to_ids(text, tokenizer))
        data = pack(pieces, tokenizer.bos_id, tokens_per_sample)
        if len(data) < want:
            raise SystemExit(f"{name}: only {len(data)} samples, need {want}")
        samples[name] = torch.tensor(data[:want], dtype=torch.int64)
        res[name] = {"samples": len(data), "kept": want}
    torch.save({"samples": samples, "tokens_per_sample": tokens_per_sample, "n_words": tokenizer.n_words,
                "pad_id": tokenizer.pad_id}, out_path)
    return res


def main(argv=None):
    p = argparse.ArgumentParser("heldout")
    sub = p.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("extract")
    e.add_argument("fineweb"), e.add_argument("codeparrot"), e.add_argument("out_dir")
    e.add_argument("n_fw", type=int), e.add_argument("n_cp", type=int)
    for name in ("dedup", "check"):
        s = sub.add_parser(name)
        s.add_argument("data_root"), s.add_argument("heldout_dir")
    b = sub.add_parser("build")
    b.add_argument("heldout_dir"), b.add_argument("out"), b.add_argument("n_fw", type=int)
    b.add_argument("n_cp", type=int)
    b.add_argument("--tiktoken-model", default="cl100k_base")
    b.add_argument("--tokens-per-sample", type=int, default=2048)
    a = p.parse_args(argv)
    if a.cmd == "extract":
        r = extract(a.fineweb, a.codeparrot, a.out_dir, a.n_fw, a.n_cp)
    elif a.cmd == "dedup":
        r = dedup(a.data_root, a.heldout_dir)
    elif a.cmd == "check":
        r = check(a.data_root, a.heldout_dir)
    else:
        from ..tasks.base import TaskConfig, build_task_tokenizer
        tok = build_task_tokenizer(TaskConfig(tiktoken_model=a.tiktoken_model))
        r = build(a.heldout_dir, a.out, a.n_fw, a.n_cp, tok, a.tokens_per_sample)
    print(json.dumps(r, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
