"""Text generation (generate.py of the reference).

Same semantics as the reference: the context is right-padded to a fixed
``seq_len`` and the whole forward is recomputed for every new token (no KV
cache, generate.py:151-200), logits are read at the last real position, and
sampling is temperature + top-k on the host (generate.py:71-85).  YaRN is
enabled by building the model with ``yarn_factor > 1``.
"""
from __future__ import annotations

import numpy as np
import torch

from .checkpoint import latest_checkpoint, load_params
from .config import Config
from .data import get_tokenizer
from .models.transformer import Transformer


def sample_next(logits: np.ndarray, temperature: float = 1.0, top_k: int = 0, rng=None) -> int:
    if temperature <= 0:
        return int(np.argmax(logits))
    logits = logits.astype(np.float64) / temperature
    if top_k > 0:
        k = min(top_k, logits.shape[-1])
        thresh = np.sort(logits)[-k]
        logits = np.where(logits < thresh, -1e30, logits)
    p = np.exp(logits - logits.max())
    p /= p.sum()
    rng = rng or np.random.default_rng()
    return int(rng.choice(len(p), p=p))


@torch.no_grad()
def generate_from_model(model: Transformer, config: Config, tokenizer, prompt: str,
                        max_tokens: int = 100, temperature: float = 1.0, top_k: int = 0,
                        seed: int = 0, seq_len: int = None):
    rng = np.random.default_rng(seed)
    ids = tokenizer.encode(prompt) or [0]
    seq_len = seq_len or config.seq_len
    dev = model.wte.device
    generated = list(ids)
    eos = getattr(tokenizer, "eos_id", None)
    for _ in range(max_tokens):
        ctx = generated[-seq_len:]
        n_real = len(ctx)
        row = np.zeros((1, seq_len), dtype=np.int64)
        row[0, :n_real] = ctx
        h, _ = model(torch.from_numpy(row).to(dev))
        logits = model.logits(h[:, n_real - 1])
        nxt = sample_next(logits[0].float().cpu().numpy(), temperature, top_k, rng)
        generated.append(nxt)
        if eos is not None and nxt == eos:
            break
    return tokenizer.decode(generated), generated


def load_for_generate(config: Config, prompt: str, max_tokens: int = 100,
                      temperature: float = 1.0, top_k: int = 0, seed: int = 0,
                      device: str = None, cached: bool = False):
    """Latest checkpoint of ``config`` -> text (generate.py:20-68)."""
    path = latest_checkpoint(config)
    if path is None:
        raise FileNotFoundError(f"No checkpoint under {config.checkpoint_dir}/{config.name}. Train first.")
    print(f"[generate] Loading checkpoint {path}")
    model = Transformer(config)
    params = load_params(path)
    named = dict(model.named_parameters())
    if len(params) != len(named):
        raise AssertionError(f"Leaf count mismatch: fresh={len(named)} saved={len(params)}")
    for n, p in named.items():
        p.data.copy_(params[n].to(p.dtype).view(p.shape))
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    model.to(dev)
    if dev != "cpu":
        from .engine import Engine
        Engine(model, config, torch.device(dev))   # attaches compute-dtype working copies
    if cached:
        from .decode import generate_cached
        return generate_cached(model, get_tokenizer(config), prompt, max_tokens, temperature, top_k, seed)
    return generate_from_model(model, config, get_tokenizer(config), prompt, max_tokens,
                               temperature, top_k, seed)
