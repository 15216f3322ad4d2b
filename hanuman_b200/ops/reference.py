"""Pure-PyTorch restatement of the reference model's math.

Every function here is the oracle for one CUDA kernel in ``csrc/`` and is also
the CPU execution path (the tiny fp32 benchmark configuration runs on it).  The
semantics follow the reference file:line cited on each function; where the
reference's JAX code and a B200 kernel legitimately differ (rounding points in
bf16), the kernel tests compare against these functions evaluated in fp32.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


# ---------------------------------------------------------------------------
# Norms
# ---------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
             out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """RMSNorm in fp32, scaled by ``w`` and cast (model/transformer.py:20-24)."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps) * w.float()
    return y.to(out_dtype or x.dtype)


def l2_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(sum(x^2) + eps) over the last axis (model/kda.py:78-81)."""
    return x / torch.sqrt((x * x).sum(-1, keepdim=True) + eps)


# ---------------------------------------------------------------------------
# RoPE / YaRN (model/rope.py:13-103)
# ---------------------------------------------------------------------------
def _yarn_correction_dim(num_rot: float, dim: int, base: float, max_pos: int) -> float:
    return (dim * math.log(max_pos / (2 * math.pi))) / (2 * num_rot * math.log(base))


def compute_inv_freqs(head_dim: int, base: float, yarn_factor: float, max_seq_len: int,
                      beta_fast: float = 32.0, beta_slow: float = 1.0) -> torch.Tensor:
    """Inverse frequencies with the YaRN ramp blend (model/rope.py:36-56)."""
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if yarn_factor != 1.0:
        hi = _yarn_correction_dim(beta_fast, head_dim, base, max_seq_len)
        lo = _yarn_correction_dim(beta_slow, head_dim, base, max_seq_len)
        dim = head_dim // 2
        lo_, hi_ = lo, hi
        if lo_ == hi_:
            hi_ += 0.001
        ramp = ((torch.arange(dim, dtype=torch.float64) / dim) - lo_) / (hi_ - lo_)
        ramp = ramp.clamp(0.0, 1.0)
        factor = 1.0 - (1.0 - 1.0 / yarn_factor) * ramp
        inv = inv / factor
    return inv.float()


def precompute_rope(head_dim: int, max_seq_len: int, base: float = 10000.0,
                    yarn_factor: float = 1.0, beta_fast: float = 32.0,
                    beta_slow: float = 1.0):
    """cos/sin tables ``[max_seq_len, head_dim]`` in the rotate-half layout."""
    inv = compute_inv_freqs(head_dim, base, yarn_factor, max_seq_len, beta_fast, beta_slow)
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               positions: Optional[torch.Tensor] = None):
    """q,k ``[B,S,N,H]``; cos/sin ``[S_max,H]`` (model/rope.py:84-103)."""
    if positions is not None:
        c = cos[positions][..., None, :]
        s = sin[positions][..., None, :]
    else:
        S = q.shape[-3]
        c = cos[:S][None, :, None, :]
        s = sin[:S][None, :, None, :]
    c = c.to(q.dtype)
    s = s.to(q.dtype)
    return q * c + rotate_half(q) * s, k * c + rotate_half(k) * s


# ---------------------------------------------------------------------------
# Attention (model/attention.py:136-224)
# ---------------------------------------------------------------------------
def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     window: int = 0, scale: Optional[float] = None,
                     q_offset: int = 0) -> torch.Tensor:
    """Causal GQA attention with an optional left window (incl. self).

    q ``[B,Sq,Nq,H]``, k/v ``[B,Sk,Nkv,H]``; query i (absolute position
    ``q_offset + i``) sees key j iff ``j <= pos`` and ``pos - j < window``
    when ``window > 0``.  Softmax in fp32.
    """
    B, Sq, Nq, H = q.shape
    Sk, Nkv = k.shape[1], k.shape[2]
    rep = Nq // Nkv
    scale = (1.0 / math.sqrt(H)) if scale is None else scale
    qf = q.float().transpose(1, 2)                            # B,Nq,Sq,H
    kf = k.float().repeat_interleave(rep, dim=2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, dim=2).transpose(1, 2)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale        # B,Nq,Sq,Sk
    qi = torch.arange(Sq, device=q.device)[:, None] + q_offset
    kj = torch.arange(Sk, device=q.device)[None, :]
    mask = kj <= qi
    if window and window > 0:
        mask = mask & (qi - kj < window)
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vf)
    return o.transpose(1, 2).to(q.dtype)


# ---------------------------------------------------------------------------
# KDA (model/kda.py)
# ---------------------------------------------------------------------------
def short_conv(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Causal depthwise conv, taps ``w [D, 1, 4]`` (model/kda.py:122-136).

    ``out[t] = sum_i w[:, i] * x[t - (Kc-1-i)]`` with zero fill; fp32 math,
    result cast back to ``x.dtype``.
    """
    Kc = w.shape[-1]
    xf = x.float()
    wf = w[:, 0, :].float()
    y = torch.zeros_like(xf)
    S = x.shape[1]
    for i in range(Kc):
        shift = Kc - 1 - i
        if shift == 0:
            xs = xf
        elif shift >= S:
            continue
        else:
            xs = F.pad(xf[:, :-shift], (0, 0, shift, 0))
        y = y + xs * wf[:, i]
    return y.to(x.dtype)


def kda_gate(f: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
             mode: str = "kimi") -> torch.Tensor:
    """Log-space per-channel decay ``g <= 0`` from the gate pre-activation.

    ``f [B,S,H,K]``; ``a_log [H]``; ``dt_bias [H*K]``.
    kimi:    g = -exp(A_log) * softplus(f + dt_bias)  (model/kda.py:272-281)
    sigmoid: g = logsigmoid(f + dt_bias)
    """
    H, K = f.shape[-2], f.shape[-1]
    z = f + dt_bias.reshape(H, K)
    if mode == "kimi":
        return -torch.exp(a_log)[:, None] * F.softplus(z)
    if mode == "sigmoid":
        return F.logsigmoid(z)
    raise ValueError(mode)


def kda_recurrent(q, k, v, g, beta, scale: Optional[float] = None,
                  initial_state: Optional[torch.Tensor] = None):
    """Token-by-token delta rule, the reference's ``step_fn`` (model/kda.py:305-323).

    Shapes: q,k,g ``[B,S,H,K]``; v ``[B,S,H,V]``; beta ``[B,S,H]``.  Per token:
    ``S *= exp(g)`` (along K); ``v' = v - beta * S^T k``;
    ``S += beta * k v'^T``; ``o = (S^T q) * scale`` (readout after update).
    Returns ``(o [B,S,H,V] fp32, final state [B,H,K,V] fp32)``.
    """
    B, S, H, K = q.shape
    V = v.shape[-1]
    scale = (1.0 / math.sqrt(K)) if scale is None else scale
    st = (torch.zeros(B, H, K, V, dtype=torch.float32, device=q.device)
          if initial_state is None else initial_state.float().clone())
    qf, kf, vf, gf, bf = q.float(), k.float(), v.float(), g.float(), beta.float()
    outs = []
    for t in range(S):
        st = st * torch.exp(gf[:, t])[..., None]
        sk = torch.einsum("bhkv,bhk->bhv", st, kf[:, t])
        vn = vf[:, t] - bf[:, t][..., None] * sk
        st = st + bf[:, t][..., None, None] * torch.einsum("bhv,bhk->bhkv", vn, kf[:, t])
        outs.append(torch.einsum("bhkv,bhk->bhv", st, qf[:, t]) * scale)
    return torch.stack(outs, dim=1), st


def kda_chunked(q, k, v, g, beta, scale: Optional[float] = None, chunk: int = 64,
                initial_state: Optional[torch.Tensor] = None):
    """Chunk-parallel form of :func:`kda_recurrent` (same outputs).

    Within a chunk with state ``S0`` and cumulative log-decay ``G_t`` the
    recurrence ``S_t = D_t S_{t-1} + k_t u_t^T`` with
    ``u_t = beta_t v_t - beta_t^2 (D_t S_{t-1})^T k_t`` solves to
    ``U = T (beta V - beta^2 (K*e^G) S0)`` where ``T = (I + diag(beta^2) A)^-1``
    and ``A_ts = sum_c k_t k_s e^{G_t-G_s}`` (s < t); the output is
    ``scale * ((Q*e^G) S0 + P U)`` with ``P_ts = sum_c q_t k_s e^{G_t-G_s}``
    (s <= t) and the carried state ``e^{G_C} S0 + (K*e^{G_C-G})^T U``.
    Pairwise decays are formed in log space, so nothing under- or overflows.
    """
    B, S, H, K = q.shape
    V = v.shape[-1]
    scale = (1.0 / math.sqrt(K)) if scale is None else scale
    st = (torch.zeros(B, H, K, V, dtype=torch.float64 if q.dtype == torch.float64 else torch.float32,
                      device=q.device) if initial_state is None else initial_state.clone())
    dt = st.dtype
    qf, kf, vf, gf, bf = (t.to(dt) for t in (q, k, v, g, beta))
    outs = []
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        C = c1 - c0
        qc = qf[:, c0:c1].transpose(1, 2)        # B,H,C,K
        kc = kf[:, c0:c1].transpose(1, 2)
        vc = vf[:, c0:c1].transpose(1, 2)        # B,H,C,V
        gc = gf[:, c0:c1].transpose(1, 2)
        bc = bf[:, c0:c1].transpose(1, 2)        # B,H,C
        G = gc.cumsum(dim=2)                     # B,H,C,K
        diff = G[:, :, :, None, :] - G[:, :, None, :, :]      # t,s
        tri_strict = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device), -1)
        tri_incl = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device), 0)
        e = torch.exp(torch.where(tri_incl[..., None], diff, torch.zeros_like(diff)))
        A = torch.einsum("bhtc,bhsc,bhtsc->bhts", kc, kc, e) * tri_strict
        P = torch.einsum("bhtc,bhsc,bhtsc->bhts", qc, kc, e) * tri_incl
        L = torch.eye(C, dtype=dt, device=q.device) + (bc ** 2)[..., None] * A
        eG = torch.exp(G)
        rhs = bc[..., None] * vc - (bc ** 2)[..., None] * torch.einsum(
            "bhck,bhkv->bhcv", kc * eG, st)
        U = torch.linalg.solve_triangular(L, rhs, upper=False, unitriangular=True)
        o = torch.einsum("bhck,bhkv->bhcv", qc * eG, st) + torch.einsum("bhts,bhsv->bhtv", P, U)
        outs.append((o * scale).transpose(1, 2))
        GC = G[:, :, -1:, :]
        st = torch.exp(GC[:, :, 0, :])[..., None] * st + torch.einsum(
            "bhck,bhcv->bhkv", kc * torch.exp(GC - G), U)
    return torch.cat(outs, dim=1), st


# ---------------------------------------------------------------------------
# MoE (model/moe.py)
# ---------------------------------------------------------------------------
def swiglu(x, w_gate, w_up, w_down):
    """down(silu(x @ gate) * (x @ up)) (model/moe.py:23-29)."""
    return (F.silu(x @ w_gate) * (x @ w_up)) @ w_down


def route(logits: torch.Tensor, bias: Optional[torch.Tensor], k: int,
          router_type: str = "sigmoid_bias", scaling: float = 2.5):
    """Top-k routing from fp32 router logits ``[T, N]``.

    sigmoid_bias (model/moe.py:177-192): select on ``sigmoid(l) + bias``, weight
    the selected experts by their renormalised sigmoid score times ``scaling``.
    softmax: select on softmax probabilities, renormalise over the top-k.
    Returns ``(scores [T,N], top_idx [T,k] int64, weights [T,k])``.
    """
    if router_type == "sigmoid_bias":
        scores = torch.sigmoid(logits)
        eff = scores + (bias.float()[None, :] if bias is not None else 0.0)
        _, idx = torch.topk(eff, k, dim=-1)
        sel = torch.gather(scores, -1, idx)
        w = sel / (sel.sum(-1, keepdim=True) + 1e-9) * scaling
        return scores, idx, w
    if router_type == "softmax":
        scores = torch.softmax(logits, dim=-1)
        sel, idx = torch.topk(scores, k, dim=-1)
        w = sel / (sel.sum(-1, keepdim=True) + 1e-9)
        return scores, idx, w
    raise ValueError(router_type)


def router_aux(logits: torch.Tensor, scores: torch.Tensor, top_idx: torch.Tensor,
               B: int, S: int, n_experts: int, router_type: str = "sigmoid_bias"):
    """Aux terms of model/moe.py:253-293 for one MoE layer.

    Returns a dict with ``router_z_loss``, ``balance_loss``, ``mean_entropy``,
    ``expert_counts [N]`` and (softmax router) ``switch_loss``.
    """
    K = top_idx.shape[-1]
    N = n_experts
    lse = torch.logsumexp(logits, dim=-1)
    z = (lse ** 2).mean()
    idx = top_idx.reshape(B, S * K)
    counts = torch.zeros(B, N, dtype=torch.float32, device=logits.device)
    counts.scatter_add_(1, idx, torch.ones_like(idx, dtype=torch.float32))
    fractions = counts / (S * K)
    sc = scores.reshape(B, S, N)
    probs = sc / (sc.sum(-1, keepdim=True) + 1e-9)
    mean_probs = probs.mean(1)
    balance = (N * (fractions * mean_probs).sum(-1)).mean()
    ent = -(probs * torch.log(probs + 1e-9)).sum(-1).mean()
    out = {"router_z_loss": z, "balance_loss": balance, "mean_entropy": ent,
           "expert_counts": counts.sum(0)}
    return out


def moe_dispatch_dense(x, top_idx, weights, w_gate, w_up, w_down):
    """Dropless routed-expert output by looping over experts (oracle for the
    grouped path; model/moe.py:37-85).  ``x [T,D]``; returns fp32 ``[T,D]``."""
    T, D = x.shape
    out = torch.zeros(T, D, dtype=torch.float32, device=x.device)
    N = w_gate.shape[0]
    for e in range(N):
        tok, slot = (top_idx == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        y = swiglu(x[tok], w_gate[e], w_up[e], w_down[e])
        out.index_add_(0, tok, y.float() * weights[tok, slot].float()[:, None])
    return out


# ---------------------------------------------------------------------------
# Loss (train.py:180-217)
# ---------------------------------------------------------------------------
def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean integer-label softmax cross-entropy in fp32."""
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1))
