"""Build a pretraining corpus in the layout the GPT task reads (scripts/data/build_data.py of the reference):

    <out>/Data/json/train.json          [{"name": <source>, "weight": w}, ...]
    <out>/Data/json/valid.json          []
    <out>/Data/json/<source>.json       absolute paths of that source's shards
    <out>/Data/shard/<source>/NNNNN.jsonl   <= 10,000 lines of {"text": ...} in source order, empty documents skipped
    <out>/data_manifest.json            per-source document / character counts and the sha256 of every shard

The default sources are the reference's two pinned public files (their sha256 is checked unless ``--no-verify``):
fineweb-edu ``sample/10BT/000_00000.parquet`` (column ``text``, weight 0.8) and codeparrot-clean
``file-000000000001.json.gz`` (field ``content``, weight 0.2). Any parquet / jsonl(.gz) file works with ``--source``.

    python -m faster_yoco_b200.data.build_data 000_00000.parquet file-000000000001.json.gz OUT
    python -m faster_yoco_b200.data.build_data --source web:a.parquet:text:0.7 --source code:b.jsonl.gz:content:0.3 OUT
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from dataclasses import dataclass
from typing import Iterator, List, Optional

LINES_PER_SHARD = 10000


@dataclass
class Source:
    name: str
    path: str
    field: str
    weight: float
    sha256: Optional[str] = None


PINNED = [
    ("fineweb_edu", "text", 0.8, "b1ba7b2ce4cb5ea6ef42dca40263eabb85f37700d01693a68e9b30a31d78e871"),
    ("codeparrot", "content", 0.2, "3726a0239b5cb7d0ef3ea36886c533d0becc7404217763015559edb546d53c94"),
]


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def iter_texts(src: Source) -> Iterator[str]:
    if src.path.endswith(".parquet"):
        import pyarrow.parquet as pq
        for batch in pq.ParquetFile(src.path).iter_batches(batch_size=8192, columns=[src.field]):
            yield from batch.column(0).to_pylist()
    else:
        import gzip
        opener = gzip.open if src.path.endswith(".gz") else open
        with opener(src.path, "rt", encoding="utf-8") as f:
            for line in f:
                yield json.loads(line)[src.field]


def build(sources: List[Source], out: str, verify: bool = True, lines_per_shard: int = LINES_PER_SHARD) -> dict:
    out = os.path.abspath(out)
    root = os.path.join(out, "Data")
    if os.path.exists(root):
        raise FileExistsError(root)
    os.makedirs(os.path.join(root, "json"))
    manifest = {"sources": {}}
    for src in sources:
        got = sha256_file(src.path)
        if verify and src.sha256 is not None and got != src.sha256:
            raise ValueError(f"{src.path}: sha256 {got} != pinned {src.sha256}")
        sdir = os.path.join(root, "shard", src.name)
        os.makedirs(sdir)
        paths: List[str] = []
        buf: List[str] = []
        n_docs = n_chars = n_empty = 0

        def flush():
            p = os.path.join(sdir, "%05d.jsonl" % len(paths))
            with open(p, "w", encoding="utf-8") as f:
                f.write("".join(buf))
            paths.append(p)
            buf.clear()

        for text in iter_texts(src):
            if not text:
                n_empty += 1
                continue
            buf.append(json.dumps({"text": text}, ensure_ascii=False) + "\n")
            n_docs += 1
            n_chars += len(text)
            if len(buf) == lines_per_shard:
                flush()
        if buf:
            flush()
        with open(os.path.join(root, "json", src.name + ".json"), "w") as f:
            json.dump(paths, f, indent=1)
        manifest["sources"][src.name] = {
            "file": os.path.basename(src.path), "sha256": got, "weight": src.weight, "docs": n_docs,
            "skipped_empty": n_empty, "chars": n_chars, "shards": len(paths),
            "shard_sha256": {os.path.basename(p): sha256_file(p) for p in paths}}
    with open(os.path.join(root, "json", "train.json"), "w") as f:
        json.dump([{"name": s.name, "weight": s.weight} for s in sources], f, indent=1)
    with open(os.path.join(root, "json", "valid.json"), "w") as f:
        json.dump([], f)
    with open(os.path.join(out, "data_manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    return manifest


def main(argv=None):
    p = argparse.ArgumentParser("build_data")
    p.add_argument("files", nargs="*", help="fineweb-edu parquet and codeparrot json.gz (pinned sources)")
    p.add_argument("out")
    p.add_argument("--source", action="append", default=[], help="name:path:field:weight (repeatable)")
    p.add_argument("--no-verify", action="store_true")
    p.add_argument("--lines-per-shard", type=int, default=LINES_PER_SHARD)
    a = p.parse_args(argv)
    if a.source:
        sources = []
        for spec in a.source:
            name, path, field, weight = spec.rsplit(":", 3)
            sources.append(Source(name, path, field, float(weight)))
    else:
        if len(a.files) != 2:
            raise SystemExit("give the two pinned files (fineweb parquet, codeparrot json.gz) or --source specs")
        sources = [Source(n, f, fld, w, h) for (n, fld, w, h), f in zip(PINNED, a.files)]
    m = build(sources, a.out, verify=not a.no_verify, lines_per_shard=a.lines_per_shard)
    for name, s in m["sources"].items():
        print(name, "docs", s["docs"], "shards", s["shards"], "chars", s["chars"], flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
