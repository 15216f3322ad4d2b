"""Model building blocks: RMSNorm, GQA attention, KDA, dense SwiGLU, MoE.

Parameter names and shapes follow the reference tree (weights stored
``[in, out]``, used as ``x @ W``) so checkpoints map one-to-one:
RMSNorm ``weight`` (model/transformer.py:14-24); attention ``wq wk wv wo``
(model/attention.py:258-261); KDA (model/kda.py:202-235); MoE
(model/moe.py:138-159); DenseFFN (model/moe.py:88-99).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref


_META = False  # set by checkpoint.param_shapes: build shapes without storage


def _normal(shape, std, gen):
    if _META:
        return torch.empty(shape, device="meta")
    return torch.randn(shape, generator=gen, dtype=torch.float32) * std


def _expert_normal(n, lo, shape, std, base, which):
    """Experts lo .. lo+n-1 of one expert weight: expert e's matrix comes from
    a generator seeded ``base + 3 e + which`` (which: 0 gate, 1 up, 2 down)."""
    if _META:
        return torch.empty((n,) + tuple(shape), device="meta")
    out = torch.empty((n,) + tuple(shape), dtype=torch.float32)
    for i in range(n):
        g = torch.Generator().manual_seed(base + 3 * (lo + i) + which)
        out[i] = torch.randn(shape, generator=g, dtype=torch.float32) * std
    return out


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x, out_dtype):
        return ops.rms_norm(x, self.weight, self.eps, out_dtype)


class Attention(nn.Module):
    """GQA with RoPE; causal or sliding-window (model/attention.py:227-285)."""

    def __init__(self, d_model, n_q, n_kv, head_dim, gen, window: int = 0):
        super().__init__()
        self.n_q, self.n_kv, self.head_dim = n_q, n_kv, head_dim
        self.window = window
        std = d_model ** -0.5
        self.wq = nn.Parameter(_normal((d_model, n_q * head_dim), std, gen))
        self.wk = nn.Parameter(_normal((d_model, n_kv * head_dim), std, gen))
        self.wv = nn.Parameter(_normal((d_model, n_kv * head_dim), std, gen))
        self.wo = nn.Parameter(_normal((n_q * head_dim, d_model), std, gen))

    def forward(self, h, cos, sin, dtype, positions=None, cache=None):
        B, S, D = h.shape
        H = self.head_dim
        if h.is_cuda and cache is None:
            from ..ops.flash import attention_layer_cuda
            return attention_layer_cuda(self, h, cos, sin, dtype, positions)
        x2 = h.reshape(B * S, D)
        q = ops.linear(x2, self.wq, compute_dtype=dtype).view(B, S, self.n_q, H)
        k = ops.linear(x2, self.wk, compute_dtype=dtype).view(B, S, self.n_kv, H)
        v = ops.linear(x2, self.wv, compute_dtype=dtype).view(B, S, self.n_kv, H)
        q, k = ops.apply_rope(q, k, cos.to(dtype), sin.to(dtype), positions)
        q_offset = 0
        if cache is not None:
            k, v, q_offset = cache.update(k, v)
        o = ops.attention(q, k, v, self.window, q_offset)
        o = o.reshape(B * S, self.n_q * H)
        return ops.linear(o, self.wo, out_dtype=torch.float32, compute_dtype=dtype).view(B, S, D)


class ShortConv1D(nn.Module):
    """Depthwise causal conv, kernel 4 (model/kda.py:85-136)."""

    def __init__(self, dim, gen, kernel_size: int = 4):
        super().__init__()
        w = _normal((dim, 1, kernel_size), 0.01, gen)
        w[:, :, -1] += 1.0
        self.weight = nn.Parameter(w)


def _init_dt_bias(shape, gen):
    log_min, log_max = math.log(0.001), math.log(0.1)
    rand = torch.rand(shape, generator=gen)
    dt = torch.exp(rand * (log_max - log_min) + log_min).clamp(min=1e-4)
    return dt + torch.log(-torch.expm1(-dt))


class KDA(nn.Module):
    """Kimi Delta Attention layer (model/kda.py:170-376).

    Forward: q/k/v projections -> ShortConv4 + SiLU -> L2-norm(q, k); decay
    g (log space) and beta; gated delta rule (chunk-parallel kernel, readout
    after update); RMSNorm over V (eps 1e-5) x o_norm x sigmoid(low-rank
    gate); output projection.
    """

    def __init__(self, d_model, n_heads, head_dim, gen, chunk: int = 64, gate: str = "kimi"):
        super().__init__()
        H, K, V, D = n_heads, head_dim, head_dim, d_model
        self.n_heads, self.head_dim, self.chunk, self.gate = H, K, chunk, gate
        std = D ** -0.5
        self.wq = nn.Parameter(_normal((D, H * K), std, gen))
        self.wk = nn.Parameter(_normal((D, H * K), std, gen))
        self.wv = nn.Parameter(_normal((D, H * V), std, gen))
        self.q_conv = ShortConv1D(H * K, gen)
        self.k_conv = ShortConv1D(H * K, gen)
        self.v_conv = ShortConv1D(H * V, gen)
        self.f_proj0 = nn.Parameter(_normal((D, K), std, gen))
        self.f_proj1 = nn.Parameter(_normal((K, H * K), std, gen))
        self.wb = nn.Parameter(_normal((D, H), std, gen))
        a = torch.rand(H, generator=gen) * 15.0 + 1.0
        self.a_log = nn.Parameter(torch.log(a))
        if gate == "sigmoid":
            # sigmoid(dt_bias) spread over [0.9, 0.999]: slow initial forgetting
            keep = 0.9 + 0.099 * torch.rand(H * K, generator=gen)
            self.dt_bias = nn.Parameter(torch.log(keep / (1 - keep)))
        else:
            self.dt_bias = nn.Parameter(_init_dt_bias((H * K,), gen))
        self.g_proj0 = nn.Parameter(_normal((D, K), std, gen))
        self.g_proj1 = nn.Parameter(_normal((K, H * V), std, gen))
        self.g_proj1_bias = nn.Parameter(torch.zeros(H * V))
        self.wo = nn.Parameter(_normal((H * V, D), std, gen))
        self.o_norm = nn.Parameter(torch.ones(V))

    def _conv_with_history(self, state, name, x):
        """Causal conv of ``x [B, S, C]`` continuing the rows kept in ``state``;
        returns (conv output [B, S, C], ) and stores the new history."""
        w = getattr(self, f"{name}_conv").weight
        taps = w.shape[-1]
        hist = state.get(f"conv_{name}")
        if hist is None:
            hist = torch.zeros(x.shape[0], taps - 1, x.shape[2], dtype=x.dtype, device=x.device)
        full = torch.cat([hist.to(x.dtype), x], dim=1)
        out = ref.short_conv(full, w)[:, taps - 1:]
        state[f"conv_{name}"] = full[:, -(taps - 1):].detach()
        return (out,)

    def forward(self, h, dtype, state=None):
        B, S, D = h.shape
        H, K = self.n_heads, self.head_dim
        V = K
        if h.is_cuda and state is None:
            from ..ops.kda import kda_layer_cuda
            return kda_layer_cuda(self, h, dtype)
        x = h.reshape(B * S, D)
        xf = x.float()
        # fp32 projections rounded to the compute dtype before the conv
        # (model/kda.py:248-261)
        qr = (xf @ self.wq.float()).to(dtype).view(B, S, H * K)
        kr = (xf @ self.wk.float()).to(dtype).view(B, S, H * K)
        vr = (xf @ self.wv.float()).to(dtype).view(B, S, H * V)
        if state is not None:
            # incremental decoding: the conv sees the last (taps - 1) projected
            # rows of earlier calls (ShortConv1D.step of the reference, model/kda.py:138-146)
            qr, kr, vr = (self._conv_with_history(state, name, x_)
                          for name, x_ in (("q", qr), ("k", kr), ("v", vr)))
            q = F.silu(qr[0].float()).view(B, S, H, K)
            k = F.silu(kr[0].float()).view(B, S, H, K)
            v = F.silu(vr[0].float()).view(B, S, H, V)
        else:
            q = F.silu(ref.short_conv(qr, self.q_conv.weight).float()).view(B, S, H, K)
            k = F.silu(ref.short_conv(kr, self.k_conv.weight).float()).view(B, S, H, K)
            v = F.silu(ref.short_conv(vr, self.v_conv.weight).float()).view(B, S, H, V)
        q = ref.l2_norm(q, 1e-6)
        k = ref.l2_norm(k, 1e-6)
        f = ((xf @ self.f_proj0.float()) @ self.f_proj1.float()).view(B, S, H, K)
        g = ref.kda_gate(f, self.a_log, self.dt_bias, self.gate)
        beta = torch.sigmoid(xf @ self.wb.float()).view(B, S, H)
        scale = 1.0 / math.sqrt(K)
        if state is not None:
            o, new_state = ref.kda_recurrent(q, k, v, g, beta, scale, state.get("S"))
            state["S"] = new_state
        else:
            o = ops.kda_core(q, k, v, g, beta, scale, self.chunk,
                             getattr(self, "recompute_core", False))
        o = o.float()
        var = (o * o).mean(-1, keepdim=True)
        o = o * torch.rsqrt(var + 1e-5) * self.o_norm
        gate = torch.sigmoid((xf @ self.g_proj0.float()) @ self.g_proj1.float()
                             + self.g_proj1_bias).view(B, S, H, V)
        o = (o * gate).reshape(B * S, H * V)
        return (o @ self.wo.float()).view(B, S, D)


class DenseFFN(nn.Module):
    """SwiGLU FFN of the first ``dense_layers`` layers (model/moe.py:88-99)."""

    def __init__(self, d_model, d_ff, gen):
        super().__init__()
        std = d_model ** -0.5
        self.w_gate = nn.Parameter(_normal((d_model, d_ff), std, gen))
        self.w_up = nn.Parameter(_normal((d_model, d_ff), std, gen))
        self.w_down = nn.Parameter(_normal((d_ff, d_model), std, gen))

    def forward(self, h, dtype):
        B, S, D = h.shape
        x = h.reshape(B * S, D)
        if h.is_cuda:
            from ..ops.moe import swiglu_ffn_cuda
            return swiglu_ffn_cuda(x, self.w_gate, self.w_up, self.w_down, dtype).view(B, S, D)
        y = ref.swiglu(x.to(dtype), self.w_gate.to(dtype), self.w_up.to(dtype), self.w_down.to(dtype))
        return y.float().view(B, S, D)


class MoE(nn.Module):
    """Routed SwiGLU experts + shared expert (model/moe.py:116-294)."""

    def __init__(self, d_model, d_ff, n_experts, n_active, n_shared, router_std,
                 scaling, gen, d_ff_shared=None, router_type="sigmoid_bias", ep=None):
        super().__init__()
        self.n_experts, self.n_active, self.n_shared = n_experts, n_active, n_shared
        self.scaling = scaling
        self.router_type = router_type
        std = d_model ** -0.5
        self.router = nn.Parameter(_normal((d_model, n_experts), router_std, gen))
        self.bias = nn.Parameter(torch.zeros(n_experts), requires_grad=False)
        # Every expert matrix is drawn from its own generator, seeded from the
        # layer's stream, so an expert-parallel rank draws only its own experts
        # (1/world of the work) and still gets exactly the unsliced values.
        base = 0 if _META else int(torch.randint(0, 2 ** 48, (1,), generator=gen))
        if ep is not None and n_experts % ep[1]:
            raise ValueError(f"{n_experts} experts do not split over {ep[1]} ranks")
        nl = n_experts if ep is None else n_experts // ep[1]
        lo = 0 if ep is None else ep[0] * nl
        shapes = {"expert_w_gate": (d_model, d_ff), "expert_w_up": (d_model, d_ff),
                  "expert_w_down": (d_ff, d_model)}
        for which, (name, shp) in enumerate(shapes.items()):
            setattr(self, name, nn.Parameter(_expert_normal(nl, lo, shp, std, base, which)))
        if ep is not None:
            self._mark_expert_parallel(*ep)
        dfs = d_ff if d_ff_shared is None else d_ff_shared
        if n_shared == 1:
            shp_in, shp_out = (d_model, dfs), (dfs, d_model)
        else:
            shp_in, shp_out = (n_shared, d_model, dfs), (n_shared, dfs, d_model)
        self.shared_w_gate = nn.Parameter(_normal(shp_in, std, gen))
        self.shared_w_up = nn.Parameter(_normal(shp_in, std, gen))
        self.shared_w_down = nn.Parameter(_normal(shp_out, std, gen))

    def shared_ffn(self, x, dtype):
        if self.n_shared == 1:
            return ref.swiglu(x.to(dtype), self.shared_w_gate.to(dtype),
                              self.shared_w_up.to(dtype), self.shared_w_down.to(dtype)).float()
        out = 0.0
        for i in range(self.n_shared):
            out = out + ref.swiglu(x.to(dtype), self.shared_w_gate[i].to(dtype),
                                   self.shared_w_up[i].to(dtype),
                                   self.shared_w_down[i].to(dtype)).float()
        return out / self.n_shared

    def make_expert_parallel(self, rank: int, world: int):
        """Keep only this rank's experts (global ids rank*N/E .. (rank+1)*N/E - 1)."""
        if self.n_experts % world:
            raise ValueError(f"{self.n_experts} experts do not split over {world} ranks")
        nl = self.n_experts // world
        for name in ("expert_w_gate", "expert_w_up", "expert_w_down"):
            p = getattr(self, name)
            p.data = p.data[rank * nl:(rank + 1) * nl].clone()
        self._mark_expert_parallel(rank, world)

    def _mark_expert_parallel(self, rank: int, world: int):
        for name in ("expert_w_gate", "expert_w_up", "expert_w_down"):
            getattr(self, name)._ep_local = True
        self.ep_rank, self.ep_world = rank, world
        self.ep_ctx = None

    def forward(self, h, dtype):
        """h ``[B,S,D]`` (compute dtype) -> (fp32 output, aux dict)."""
        if h.is_cuda and getattr(self, "ep_world", 1) > 1:
            from ..ops.moe_ep import moe_ep_layer_cuda, shared_ep_context
            T = h.shape[0] * h.shape[1]
            if self.ep_ctx is None or self.ep_ctx.T != T:
                self.ep_ctx = shared_ep_context(self, T, h.shape[2], self.expert_w_gate.shape[2],
                                                self.ep_dist, self.capacity_factor)
            return moe_ep_layer_cuda(self, h, dtype)
        if h.is_cuda:
            from ..ops.moe import moe_layer_cuda
            return moe_layer_cuda(self, h, dtype)
        B, S, D = h.shape
        x = h.reshape(B * S, D)
        logits = x.float() @ self.router.float()
        scores, idx, w = ref.route(logits, self.bias, self.n_active, self.router_type,
                                   self.scaling)
        routed = ref.moe_dispatch_dense(
            x.to(dtype), idx, w.to(dtype), self.expert_w_gate.to(dtype),
            self.expert_w_up.to(dtype), self.expert_w_down.to(dtype))
        out = routed + self.shared_ffn(x, dtype)
        aux = ref.router_aux(logits, scores, idx, B, S, self.n_experts, self.router_type)
        return out.view(B, S, D), aux
