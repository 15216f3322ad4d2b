"""Context parallelism for the token mixers: KDA state passing along the
sequence, and attention over all-gathered keys and values.

The reference has no sequence or context parallelism (attention keeps heads
and sequence whole per device, model/attention.py:217-224); its long-context
levers are the chunked KDA scan, SWA and remat.  This module is the optional
extension for sequences that do not fit one GPU: a sequence is split into
``world`` contiguous segments, one per rank of ``group``, and the linear
recurrence carries across the segment boundaries as its state.

Forward: rank r waits for the state ``S_in`` [B, H, K, V] (fp32) that rank r-1
ended with (zeros on rank 0), runs the chunked delta rule on its segment from
that state, and hands its final state to rank r+1.  Backward: the chain runs
in reverse; rank r receives d(S_out) from rank r+1, back-propagates through
its segment (which also yields d(S_in)) and hands d(S_in) to rank r-1.  Only
the [B, H, K, V] state crosses a boundary, in each direction once per step.

The ranks run one after the other along the chain (the state-passing form);
a parallel prefix over the per-segment affine maps S_out = M S_in + N would let
them overlap but needs the K x K transition M of every segment.  This is the
PyTorch chunked form (ops/reference.py:kda_chunked), so it runs on CPU (gloo)
and on GPU tensors (NCCL) alike; the sm_100a KDA kernels do not take a
gradient for the initial state, so they are not used here.

Attention (``attention_context_parallel``): every rank gathers the keys and
values of all segments (a differentiable all-gather: the backward sums the
key / value gradients of every rank's queries into the owner) and attends its
own queries at their global positions, causal and with the sliding window,
over the keys up to the end of its segment.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..ops import reference as ref


class _RecvState(torch.autograd.Function):
    """Forward: the incoming state from ``src`` (zeros when src < 0).
    Backward: its gradient goes back to ``src``.  ``anchor`` (a scalar that
    requires grad) only records the node in the graph."""

    @staticmethod
    def forward(ctx, anchor, shape, dtype, src, group):
        st = torch.zeros(shape, dtype=dtype, device=anchor.device)
        if src >= 0:
            dist.recv(st, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
        ctx.src, ctx.group = src, group
        return st

    @staticmethod
    def backward(ctx, grad):
        if ctx.src >= 0:
            g = grad.contiguous()
            dst = dist.get_global_rank(ctx.group, ctx.src) if ctx.group is not None else ctx.src
            dist.send(g, dst=dst, group=ctx.group)
        return None, None, None, None, None


class _SendState(torch.autograd.Function):
    """Forward: the outgoing state goes to ``dst``; returns a zero scalar that
    the caller adds to its output so that the backward reaches this node.
    Backward: the state's gradient is received from ``dst``."""

    @staticmethod
    def forward(ctx, st, dst, group):
        peer = dist.get_global_rank(group, dst) if group is not None else dst
        dist.send(st.detach().contiguous(), dst=peer, group=group)
        ctx.peer, ctx.group = peer, group
        ctx.shape, ctx.dtype = st.shape, st.dtype
        return torch.zeros((), dtype=st.dtype, device=st.device)

    @staticmethod
    def backward(ctx, grad):
        g = torch.empty(ctx.shape, dtype=ctx.dtype, device=grad.device)
        dist.recv(g, src=ctx.peer, group=ctx.group)
        return g, None, None


def kda_context_parallel(q, k, v, g, beta, scale: Optional[float] = None, chunk: int = 64,
                         group=None):
    """Delta rule over a sequence split across the ranks of ``group``.

    Each rank passes its own segment: q, k, g ``[B, S_r, H, K]``, v ``[B, S_r,
    H, V]``, beta ``[B, S_r, H]`` (rank r holds tokens r*S_r .. (r+1)*S_r - 1).
    Returns this rank's output ``[B, S_r, H, V]``; its gradients (and those of
    the other ranks' segments through the passed states) come out of the
    ordinary ``backward``.  Every rank must call this, in rank order of the
    sequence, once per forward; the backward must run on every rank too.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    B, _, H, K = q.shape
    V = v.shape[-1]
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    anchor = torch.zeros((), device=q.device, requires_grad=True)
    s_in = _RecvState.apply(anchor, (B, H, K, V), dt, rank - 1 if rank > 0 else -1, group)
    o, s_out = ref.kda_chunked(q, k, v, g, beta, scale, chunk, initial_state=s_in)
    if rank < world - 1:
        o = o + _SendState.apply(s_out, rank + 1, group).to(o.dtype)
    return o


class _GatherSeq(torch.autograd.Function):
    """All-gather along dim 1 (the sequence); the backward sums every rank's
    gradient of the gathered tensor and keeps this rank's slice (reduce-scatter
    on NCCL, all-reduce and slice on backends without it)."""

    @staticmethod
    def forward(ctx, x, group):
        world = dist.get_world_size(group)
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        ctx.group, ctx.rank, ctx.world, ctx.n = group, dist.get_rank(group), world, x.shape[1]
        return torch.cat(parts, dim=1)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        if dist.get_backend(ctx.group) == dist.Backend.NCCL:
            parts = [p.contiguous() for p in grad.split(ctx.n, dim=1)]
            out = torch.empty_like(parts[ctx.rank])
            dist.reduce_scatter(out, parts, group=ctx.group)
            return out, None
        dist.all_reduce(grad, group=ctx.group)
        return grad[:, ctx.rank * ctx.n:(ctx.rank + 1) * ctx.n].contiguous(), None


def attention_context_parallel(q, k, v, window: int = 0, scale: Optional[float] = None, group=None):
    """Causal GQA attention over a sequence split across the ranks of ``group``.

    Each rank passes its segment: q ``[B, S_r, Nq, H]``, k / v ``[B, S_r, Nkv,
    H]`` (rank r holds tokens r*S_r .. (r+1)*S_r - 1, equal S_r on every rank).
    Returns this rank's output ``[B, S_r, Nq, H]``; query i of rank r sits at
    global position r*S_r + i and sees the keys at or before it (within the
    window when ``window > 0``), whichever rank holds them."""
    rank = dist.get_rank(group)
    n, H = q.shape[1], k.shape[-1]
    # keys and values in ONE gather: the backward is then one collective too
    # (two would run in whatever order autograd reaches them on each rank)
    kv_all = _GatherSeq.apply(torch.cat([k, v], dim=-1), group)
    k_all, v_all = kv_all[..., :H], kv_all[..., H:]
    end = (rank + 1) * n          # causal: no key past this segment's last query
    return ref.causal_attention(q, k_all[:, :end], v_all[:, :end], window, scale, q_offset=rank * n)


class _Halo(torch.autograd.Function):
    """Prepends the last ``n`` rows (dim 1) of the previous rank's ``x`` (zeros
    on rank 0) and hands this rank's last ``n`` rows to the next rank; the
    backward returns the halo's gradient to its owner and adds the gradient
    the next rank sends for this rank's last rows.  One exchange per call, so
    callers concatenate what they need (e.g. the q | k | v projections)."""

    @staticmethod
    def forward(ctx, x, n, group):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        glob = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
        halo = torch.zeros(x.shape[0], n, *x.shape[2:], dtype=x.dtype, device=x.device)
        reqs = []
        if rank > 0:
            reqs.append(dist.irecv(halo, src=glob(rank - 1), group=group))
        if rank < world - 1:
            reqs.append(dist.isend(x[:, -n:].contiguous(), dst=glob(rank + 1), group=group))
        for r in reqs:
            r.wait()
        ctx.n, ctx.group, ctx.rank, ctx.world, ctx.glob = n, group, rank, world, glob
        return torch.cat([halo, x], dim=1)

    @staticmethod
    def backward(ctx, grad):
        n = ctx.n
        gx = grad[:, n:].contiguous()
        tail = torch.zeros_like(gx[:, -n:])
        reqs = []
        if ctx.rank < ctx.world - 1:
            reqs.append(dist.irecv(tail, src=ctx.glob(ctx.rank + 1), group=ctx.group))
        if ctx.rank > 0:
            reqs.append(dist.isend(grad[:, :n].contiguous(), dst=ctx.glob(ctx.rank - 1), group=ctx.group))
        for r in reqs:
            r.wait()
        if ctx.rank < ctx.world - 1:
            gx[:, -n:] += tail
        return gx, None, None


def kda_layer_context_parallel(mod, h, dtype, group=None):
    """A KDA layer (models/layers.py:KDA, its CPU math) over a sequence split
    across the ranks of ``group``: the 4-tap conv reads the previous rank's
    last 3 projected rows (one halo exchange for q | k | v), the delta rule
    passes its state along the chain; everything else is per token.  Each
    rank passes its segment ``h [B, S_r, D]`` and gets its output; parameter
    gradients are this rank's share (sum them over the ranks)."""
    import math
    import torch.nn.functional as F
    B, S, D = h.shape
    H, K = mod.n_heads, mod.head_dim
    V = K
    xf = h.reshape(B * S, D).float()
    proj = torch.cat([(xf @ mod.wq.float()).to(dtype), (xf @ mod.wk.float()).to(dtype),
                      (xf @ mod.wv.float()).to(dtype)], dim=-1).view(B, S, -1)
    taps = mod.q_conv.weight.shape[-1]
    full = _Halo.apply(proj, taps - 1, group)
    HK = H * K
    convs = []
    for i, conv in enumerate((mod.q_conv, mod.k_conv, mod.v_conv)):
        c = ref.short_conv(full[..., i * HK:(i + 1) * HK], conv.weight)[:, taps - 1:]
        convs.append(F.silu(c.float()))
    q, k, v = (c.view(B, S, H, K) for c in convs)
    q = ref.l2_norm(q, 1e-6)
    k = ref.l2_norm(k, 1e-6)
    f = ((xf @ mod.f_proj0.float()) @ mod.f_proj1.float()).view(B, S, H, K)
    g = ref.kda_gate(f, mod.a_log, mod.dt_bias, mod.gate)
    beta = torch.sigmoid(xf @ mod.wb.float()).view(B, S, H)
    o = kda_context_parallel(q, k, v, g, beta, 1.0 / math.sqrt(K), mod.chunk, group).float()
    var = (o * o).mean(-1, keepdim=True)
    o = o * torch.rsqrt(var + 1e-5) * mod.o_norm
    gate = torch.sigmoid((xf @ mod.g_proj0.float()) @ mod.g_proj1.float()
                         + mod.g_proj1_bias).view(B, S, H, V)
    o = (o * gate).reshape(B * S, H * V)
    return (o @ mod.wo.float()).view(B, S, D)


def _attention_layer_cp(mod, h, cos, sin, dtype, pos0, group):
    """models/layers.py:Attention (CPU math) for this rank's segment: RoPE at
    the global positions, attention over the all-gathered keys / values."""
    from .. import ops
    B, S, D = h.shape
    H = mod.head_dim
    x2 = h.reshape(B * S, D)
    q = ops.linear(x2, mod.wq, compute_dtype=dtype).view(B, S, mod.n_q, H)
    k = ops.linear(x2, mod.wk, compute_dtype=dtype).view(B, S, mod.n_kv, H)
    v = ops.linear(x2, mod.wv, compute_dtype=dtype).view(B, S, mod.n_kv, H)
    positions = torch.arange(pos0, pos0 + S, device=h.device)
    q, k = ops.apply_rope(q, k, cos.to(dtype), sin.to(dtype), positions)
    o = attention_context_parallel(q, k, v, mod.window, None, group).reshape(B * S, mod.n_q * H)
    return ops.linear(o, mod.wo, out_dtype=torch.float32, compute_dtype=dtype).view(B, S, D)


def _moe_cp(mod, h, dtype, world, group):
    """models/layers.py:MoE (CPU math) for this rank's segment; the router
    statistics of the aux losses (ops/reference.py:router_aux) are sums over
    the whole sequence, so they are summed over the ranks (differentiable:
    the backward sums every rank's gradient of the global statistics)."""
    import torch.distributed.nn.functional as dnn
    B, S, D = h.shape
    N, K = mod.n_experts, mod.n_active
    x = h.reshape(B * S, D)
    logits = x.float() @ mod.router.float()
    scores, idx, w = ref.route(logits, mod.bias, K, mod.router_type, mod.scaling)
    routed = ref.moe_dispatch_dense(x.to(dtype), idx, w.to(dtype), mod.expert_w_gate.to(dtype),
                                    mod.expert_w_up.to(dtype), mod.expert_w_down.to(dtype))
    out = routed + mod.shared_ffn(x, dtype)
    lse = torch.logsumexp(logits, dim=-1)
    counts = torch.zeros(B, N, dtype=torch.float32, device=h.device)
    counts.scatter_add_(1, idx.reshape(B, S * K), torch.ones(B, S * K, device=h.device))
    sc = scores.reshape(B, S, N)
    probs = sc / (sc.sum(-1, keepdim=True) + 1e-9)
    stats = torch.cat([(lse ** 2).sum().reshape(1), probs.sum(1).reshape(-1),
                       (-(probs * torch.log(probs + 1e-9)).sum(-1)).sum().reshape(1)])
    stats = dnn.all_reduce(stats, group=group)
    dist.all_reduce(counts, group=group)
    s_tot = S * world
    aux = {"router_z_loss": stats[0] / (B * s_tot),
           "balance_loss": (N * (counts / (s_tot * K) * stats[1:1 + B * N].view(B, N) / s_tot)
                            .sum(-1)).mean(),
           "mean_entropy": stats[-1] / (B * s_tot),
           "expert_counts": counts.sum(0)}
    return out.view(B, S, D), aux


def transformer_loss_context_parallel(model, tokens, next_first, group=None):
    """This rank's share of the training loss of ``models/transformer.py:
    Transformer.loss`` (CPU math) for a batch whose sequences are split across
    the ranks of ``group`` in equal contiguous segments.

    ``tokens [B, S_r]`` is this rank's segment; ``next_first [B]`` the first
    token of the next rank's segment (the target of this segment's last
    position; unused on the last rank).  The shares of all ranks sum to the
    single-process loss: CE summed over this rank's positions / all positions,
    plus the router z and balance losses (computed from statistics summed over
    the ranks) / world.  The parameter gradients of the shares sum (over the
    ranks) to the single-process gradients."""
    from ..models.transformer import merge_aux
    from .. import ops
    cfg = model.cfg
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, S = tokens.shape
    dtype = model.dtype
    x = model.embed(tokens)
    aux_list = []
    for blk in model.blocks:
        h = blk.norm1(x, dtype)
        if blk.attention_type == "kda":
            a = kda_layer_context_parallel(blk.attn, h, dtype, group)
        else:
            a = _attention_layer_cp(blk.attn, h, model.rope_cos, model.rope_sin, dtype, rank * S, group)
        x = x + blk.residual_scale.float() * a
        h = blk.norm2(x, dtype)
        if blk.use_moe:
            f, aux = _moe_cp(blk.ffn, h, dtype, world, group)
            aux_list.append(aux)
        else:
            f = blk.ffn(h, dtype)
        x = x + blk.residual_scale.float() * f
    hN = model.norm_f(x, dtype)
    if rank < world - 1:
        tgt = torch.cat([tokens[:, 1:], next_first[:, None]], dim=1)
        hs = hN
    else:
        tgt = tokens[:, 1:]
        hs = hN[:, :-1]
    n_local = hs.shape[0] * hs.shape[1]
    n_all = B * (S * world - 1)
    ce = ops.head_cross_entropy(hs.reshape(n_local, -1), model.wte, tgt.reshape(-1),
                                compute_dtype=dtype) * (n_local / n_all)
    aux = merge_aux(aux_list, cfg.n_experts, model.n_moe, x.device)
    return ce + (cfg.z_loss_weight * aux["router_z_loss"]
                 + cfg.balance_loss_weight * aux["balance_loss"]) / world
