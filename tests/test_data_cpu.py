"""Tokenizers, packing and the checkpointable LM loader (CPU)."""
import json
import os

import torch

from faster_yoco_b200.data import iterators as it
from faster_yoco_b200.data.lm_loader import LMLoader, doc_to_ids, pack
from faster_yoco_b200.data.tokenizers import ByteTokenizer, build_tokenizer


def _make_corpus(root, n_files=6, docs=40):
    os.makedirs(os.path.join(root, "json"), exist_ok=True)
    for src in ("a", "b"):
        files = []
        for i in range(n_files):
            rel = f"shard/{src}/{i:05d}.jsonl"
            os.makedirs(os.path.dirname(os.path.join(root, rel)), exist_ok=True)
            with open(os.path.join(root, rel), "w") as f:
                for d in range(docs):
                    f.write(json.dumps({"text": f"{src} doc {i}-{d}\n\nline two of {d}\nthird " * 3}) + "\n")
            files.append(rel)
        with open(os.path.join(root, "json", f"{src}.json"), "w") as f:
            json.dump(files, f)


def test_byte_tokenizer_ids_and_specials():
    t = ByteTokenizer()
    assert (t.bos_id, t.pad_id, t.eos_id, t.unk_id) == (0, 1, 2, 3)
    assert t.n_words == 264
    ids = t.encode("hi", bos=True, eos=True)
    assert ids == [0, ord("h") + 4, ord("i") + 4, 2]
    assert t.decode(ids) == "hi"


def test_build_tokenizer_falls_back_offline():
    tok = build_tokenizer(tiktoken_model="cl100k_base")
    assert tok.encode("a")[0] >= 4


def test_doc_to_ids_and_pack_semantics():
    t = ByteTokenizer()
    pieces = doc_to_ids("ab\ncd\n\nef", t)
    assert [t.decode(p) for p in pieces] == ["ab\n", "cd\n\n", "ef"]
    assert pieces[-1][-1] == t.eos_id
    samples = pack([[10] * 5, [11] * 5, [12] * 5], bos=0, tokens_per_sample=8)
    assert samples == [[0] + [10] * 5 + [11] * 3]


def test_loader_batches_and_resume(tmp_path):
    _make_corpus(str(tmp_path))
    data = [{"name": "a", "weight": 0.8}, {"name": "b", "weight": 0.2}]
    tok = ByteTokenizer()
    mk = lambda: LMLoader(data, str(tmp_path), tok, tokens_per_sample=64, batch_size=2, seed=1, num_shards=2,
                          shard_id=1, batch_read_ahead=5, prefetch=3)
    L = mk()
    first = [next(L) for _ in range(4)]
    b = first[0]
    assert b["src_tokens"].shape == (2, 64) and b["ntokens"] == 2 * 65
    assert torch.equal(b["src_tokens"][:, 1:], b["target"][:, :-1])
    assert (b["src_tokens"][:, 0] == tok.bos_id).all()
    state = L.state_dict()
    nxt = [next(L) for _ in range(3)]
    L.close()
    L2 = mk()
    L2.load_state_dict(state)
    again = [next(L2) for _ in range(3)]
    L2.close()
    for x, y in zip(nxt, again):
        assert torch.equal(x["src_tokens"], y["src_tokens"])
    L3 = mk()
    assert torch.equal(next(L3)["src_tokens"], first[0]["src_tokens"])      # deterministic
    L3.close()


def test_weight_iterator_is_stateless_per_position():
    w = it.WeightNoRandomStateIterator([0.5, 0.5], 3)
    seq = [next(w) for _ in range(10)]
    w.setstate({"n": 4})
    assert [next(w) for _ in range(6)] == seq[4:]


def test_weight_and_index_iterators_resume():
    w = it.WeightIterator([0.2, 0.8], 7)
    seq = [next(w) for _ in range(12)]
    w2 = it.WeightIterator([0.2, 0.8], 7)
    for _ in range(5):
        next(w2)
    st = w2.getstate()
    w3 = it.WeightIterator([0.2, 0.8], 7)
    w3.setstate(st)
    assert [next(w3) for _ in range(7)] == seq[5:]
    ix = it.IndexIterator(3)
    assert [next(ix) for _ in range(5)] == [0, 1, 2, 0, 1]
    ix.setstate({"n": 4})
    assert next(ix) == 1


def test_loader_single_pass_for_evaluation(tmp_path):
    _make_corpus(str(tmp_path), n_files=2, docs=10)
    data = [{"name": "a", "weight": 0.5}, {"name": "b", "weight": 0.5}]
    L = LMLoader(data, str(tmp_path), ByteTokenizer(), tokens_per_sample=64, batch_size=2, batch_read_ahead=0,
                 prefetch=0, endless=False)
    n = sum(1 for _ in L)
    L2 = LMLoader(data, str(tmp_path), ByteTokenizer(), tokens_per_sample=64, batch_size=2, batch_read_ahead=0,
                  prefetch=2, endless=False)
    assert n > 0 and sum(1 for _ in L2) == n          # finite, and the same count with prefetching
    L2.close()
