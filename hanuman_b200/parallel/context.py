"""Context parallelism for the KDA delta rule: state passing along the sequence.

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
