"""Tokenizers with the reference's id conventions.

* :class:`TiktokenTokenizer` -- cl100k_base with the FIM / code special tokens 100264-100281, four prepended
  symbols ``<s>=0, <pad>=1, </s>=2, <unk>=3``, BPE ids shifted by +4, vocabulary rounded up to a multiple of 8
  (100,288 for cl100k_base) (yoco/tasks/data/tiktoken_tokenizer.py:5-81). The BPE ranks come from tiktoken's cache
  or from a local ``.tiktoken`` file (``tiktoken_model`` may be a path) since this machine has no network.
* :class:`LLaMATokenizer` -- sentencepiece model file (yoco/tasks/data/llama_tokenizer.py:6-38).
* :class:`ByteTokenizer` -- offline fallback with the same four symbols: UTF-8 bytes shifted by +4 (vocab 264 -> 264).
"""
from __future__ import annotations

import os
from typing import List

SYMBOLS = ["<s>", "<pad>", "</s>", "<unk>"]
FIM_SPECIALS = ["<fim_prefix>", "<fim_middle>", "<fim_suffix>", "<fim_pad>", "<reponame>", "<filename>", "<gh_stars>",
                "<issue_start>", "<issue_comment>", "<issue_closed>", "<jupyter_start>", "<jupyter_text>",
                "<jupyter_code>", "<jupyter_output>", "<empty_output>", "<commit_before>", "<commit_msg>",
                "<commit_after>"]


class _Base:
    symbols = SYMBOLS

    @property
    def bos_id(self) -> int:
        return 0

    @property
    def pad_id(self) -> int:
        return 1

    @property
    def eos_id(self) -> int:
        return 2

    @property
    def unk_id(self) -> int:
        return 3

    def _wrap(self, t: List[int], bos: bool, eos: bool) -> List[int]:
        if bos:
            t = [self.bos_id] + t
        if eos:
            t = t + [self.eos_id]
        return t


class TiktokenTokenizer(_Base):
    def __init__(self, tiktoken_model: str = "cl100k_base", tokenizer_pad_to_multiple: int = 8):
        import tiktoken
        if os.path.exists(tiktoken_model):
            from tiktoken.load import load_tiktoken_bpe
            ranks = load_tiktoken_bpe(tiktoken_model)
            pat = r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"""
            base_special = {"<|endoftext|>": 100257, "<|fim_prefix|>": 100258, "<|fim_middle|>": 100259,
                            "<|fim_suffix|>": 100260, "<|endofprompt|>": 100276}
        else:
            base = tiktoken.get_encoding(tiktoken_model)
            ranks, pat, base_special = base._mergeable_ranks, base._pat_str, base._special_tokens
        special = dict(base_special)
        special.update({name: 100264 + i for i, name in enumerate(FIM_SPECIALS)})
        self._model = tiktoken.Encoding(name="cl100k_im", pat_str=pat, mergeable_ranks=ranks, special_tokens=special)
        self.pad_multiple = tokenizer_pad_to_multiple

    @property
    def n_words(self) -> int:
        n = self._model.n_vocab + len(self.symbols)
        return (n + self.pad_multiple - 1) // self.pad_multiple * self.pad_multiple

    def encode(self, s: str, bos: bool = False, eos: bool = False) -> List[int]:
        t = [i + len(self.symbols) for i in self._model.encode(s, allowed_special="all")]
        return self._wrap(t, bos, eos)

    def decode(self, t: List[int]) -> str:
        return self._model.decode([i - len(self.symbols) for i in t if i >= len(self.symbols)])


class LLaMATokenizer:
    def __init__(self, model_path: str):
        from sentencepiece import SentencePieceProcessor
        if not os.path.exists(model_path):
            raise FileNotFoundError(model_path)
        self._model = SentencePieceProcessor(model_file=model_path)

    @property
    def n_words(self) -> int:
        return self._model.vocab_size()

    @property
    def bos_id(self) -> int:
        return self._model.bos_id()

    @property
    def eos_id(self) -> int:
        return self._model.eos_id()

    @property
    def pad_id(self) -> int:
        return self._model.pad_id()

    def encode(self, s: str, bos: bool = False, eos: bool = False) -> List[int]:
        t = self._model.encode(s)
        if bos:
            t = [self.bos_id] + t
        if eos:
            t = t + [self.eos_id]
        return t

    def decode(self, t: List[int]) -> str:
        return self._model.decode(t)


class ByteTokenizer(_Base):
    """UTF-8 bytes + 4; n_words = 264 rounded to the pad multiple."""

    def __init__(self, tokenizer_pad_to_multiple: int = 8):
        self.pad_multiple = tokenizer_pad_to_multiple

    @property
    def n_words(self) -> int:
        n = 256 + len(self.symbols)
        return (n + self.pad_multiple - 1) // self.pad_multiple * self.pad_multiple

    def encode(self, s: str, bos: bool = False, eos: bool = False) -> List[int]:
        return self._wrap([b + len(self.symbols) for b in s.encode("utf-8")], bos, eos)

    def decode(self, t: List[int]) -> str:
        return bytes([i - len(self.symbols) for i in t if 4 <= i < 260]).decode("utf-8", errors="replace")


def build_tokenizer(tiktoken_model=None, llama_model=None, pad_to_multiple: int = 8, fallback: bool = True):
    if llama_model:
        return LLaMATokenizer(llama_model)
    if tiktoken_model:
        try:
            return TiktokenTokenizer(tiktoken_model, pad_to_multiple)
        except Exception:
            if not fallback:
                raise
    return ByteTokenizer(pad_to_multiple)
