"""Greedy generation with chunked prefill (yoco/criterions/needle_haystack.py:135-160).

The prompt except its last token is prefilled in chunks of ``chunk_length`` tokens with ``skip_cross_decoder=True``
(YOCO fills the self-decoder states and the single shared K/V cache only; the cross-decoder layers do not run over
the prompt), then each step feeds the previous token, masks BOS and PAD out of the logits, takes the argmax, and
stops once every row produced EOS. Works for any model with the ``model(ids, start_pos=, incremental_state=,
is_prefilling=, skip_cross_decoder=)`` signature (YOCO, and LLaMA which ignores the YOCO-only flags).
"""
from __future__ import annotations

import math

import torch


@torch.no_grad()
def generate(model, prompt: torch.Tensor, tokenizer, generate_tokens: int = 20, chunk_length: int = 32768,
             yoco: bool = True) -> torch.Tensor:
    """prompt: [B, P] ids on the model's device -> [B, P + generate_tokens] (pad where nothing was produced)."""
    B, P = prompt.shape
    dev = prompt.device
    out = torch.cat([prompt, torch.full((B, generate_tokens), tokenizer.pad_id, dtype=torch.long, device=dev)], 1)
    begin = P
    state = {}
    eos = torch.zeros(B, dtype=torch.bool, device=dev)
    extra = {"skip_cross_decoder": True} if yoco else {}
    for s in range(0, begin - 1, chunk_length):
        e = min(s + chunk_length, begin - 1)
        model(out[:, s:e], incremental_state=state, start_pos=s, is_prefilling=True, **extra)
    extra = {"skip_cross_decoder": False} if yoco else {}
    for idx in range(begin, out.shape[1]):
        logits, _ = model(out[:, idx - 1:idx], incremental_state=state, start_pos=idx - 1, is_prefilling=False,
                          **extra)
        logits = logits[:, -1, :].float()
        logits[:, tokenizer.bos_id] = -math.inf
        logits[:, tokenizer.pad_id] = -math.inf
        nxt = logits.argmax(-1)
        cur = out[:, idx]
        nxt = torch.where((cur == tokenizer.pad_id) & ~eos, nxt, cur)
        out[:, idx] = nxt
        eos |= nxt == tokenizer.eos_id
        if bool(eos.all()):
            break
    return out
