"""Flash attention (causal / sliding window, GQA) on the native kernels, and the
GPU forward of a full attention layer (fused q/k/v projection, RoPE,
attention, output projection)."""
from __future__ import annotations

import torch

from ._ext import ext


class FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, window):
        q, k, v = (t.contiguous() for t in (q, k, v))
        B, S, Nq, H = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(B, Nq, S, dtype=torch.float32, device=q.device)
        ext().flash_fwd(q, k, v, out, lse, int(window))
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.window = int(window)
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        do = do.to(torch.bfloat16).contiguous()
        B, S, Nq, H = q.shape
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        delta = torch.empty(B, Nq, S, dtype=torch.float32, device=q.device)
        ext().flash_bwd(q, k, v, out, do, lse, delta, dq, dk, dv, ctx.window)
        return dq, dk, dv, None


def flash_attention(q, k, v, window=0, q_offset=0):
    if q_offset or q.shape[1] != k.shape[1]:
        # incremental decoding (queries at the end of a longer key range): a few
        # query rows, computed with the reference formula on the device
        from . import reference as ref
        return ref.causal_attention(q.float(), k.float(), v.float(), window,
                                    q_offset=q_offset).to(q.dtype)
    return FlashAttnFn.apply(q, k, v, window)


def attention_layer_cuda(mod, h, cos, sin, dtype, positions=None):
    """``wo(attn(rope(h wq), rope(h wk), h wv))`` with one fp32 input gradient."""
    from .dense import linear_multi
    from .norm import rope_cuda
    B, S, D = h.shape
    H = mod.head_dim
    x2 = h.reshape(B * S, D)
    q, k, v = linear_multi(x2, [mod.wq, mod.wk, mod.wv], torch.bfloat16)
    q = q.view(B, S, mod.n_q, H)
    k = k.view(B, S, mod.n_kv, H)
    v = v.view(B, S, mod.n_kv, H)
    q, k = rope_cuda(q, k, cos.to(torch.bfloat16), sin.to(torch.bfloat16), positions)
    o = FlashAttnFn.apply(q, k, v, mod.window)
    (y,) = linear_multi(o.view(B * S, mod.n_q * H), [mod.wo], torch.float32)
    return y.view(B, S, D)
