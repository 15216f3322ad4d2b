"""Incremental decoding with per-layer caches (the reference recomputes the
padded context for every token, generate.py:151-200; this is the optional
KV / recurrent-state cache).

* full / sliding-window attention layers keep their RoPE'd keys and values;
  a step's queries attend to the cached keys with ``q_offset`` = tokens seen;
* KDA layers keep the recurrent state ``S [B, H, K, V]`` (fp32) and the last
  three projected rows of q / k / v for the causal conv (ShortConv1D.step,
  model/kda.py:138-146), and advance with the token-by-token delta rule.

Greedy decoding with the cache produces the same tokens as the reference's
full recomputation (tests/test_train_cpu.py).
"""
from __future__ import annotations

import numpy as np
import torch

from .models.transformer import Transformer


class KVCache:
    def __init__(self):
        self.k = None
        self.v = None

    @property
    def length(self) -> int:
        return 0 if self.k is None else self.k.shape[1]

    def update(self, k, v):
        q_offset = self.length
        self.k = k if self.k is None else torch.cat([self.k, k], dim=1)
        self.v = v if self.v is None else torch.cat([self.v, v], dim=1)
        return self.k, self.v, q_offset


class DecodeCache:
    """Per-layer decoding state for one batch of sequences."""

    def __init__(self, model: Transformer):
        self.kvs, self.states = {}, {}
        for i, blk in enumerate(model.blocks):
            if blk.attention_type == "kda":
                self.states[i] = {}
            else:
                self.kvs[i] = KVCache()
        self.pos = 0

    def kv(self, layer: int) -> KVCache:
        return self.kvs[layer]

    def kda_state(self, layer: int) -> dict:
        return self.states[layer]


@torch.no_grad()
def step(model: Transformer, tokens: torch.Tensor, cache: DecodeCache) -> torch.Tensor:
    """Feed ``tokens [B, S]`` after everything already in ``cache``; returns the
    logits of the last position ``[B, V]``."""
    B, S = tokens.shape
    positions = torch.arange(cache.pos, cache.pos + S, device=tokens.device)[None].expand(B, S)
    h, _ = model(tokens, positions=positions, cache=cache)
    cache.pos += S
    return model.logits(h[:, -1])


@torch.no_grad()
def generate_cached(model: Transformer, tokenizer, prompt: str, max_tokens: int = 100,
                    temperature: float = 1.0, top_k: int = 0, seed: int = 0):
    """Prefill the prompt once, then one token per step through the caches."""
    from .generate import sample_next
    rng = np.random.default_rng(seed)
    ids = tokenizer.encode(prompt) or [0]
    dev = model.wte.device
    cache = DecodeCache(model)
    logits = step(model, torch.tensor([ids], device=dev), cache)
    generated = list(ids)
    eos = getattr(tokenizer, "eos_id", None)
    for _ in range(max_tokens):
        nxt = sample_next(logits[0].float().cpu().numpy(), temperature, top_k, rng)
        generated.append(nxt)
        if eos is not None and nxt == eos:
            break
        logits = step(model, torch.tensor([[nxt]], device=dev), cache)
    return tokenizer.decode(generated), generated
