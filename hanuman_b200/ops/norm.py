"""RMSNorm, RoPE, SwiGLU activation and embedding on the native kernels."""
from __future__ import annotations

import torch

from ._ext import ext


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, out_dtype):
        xf = x.float().contiguous()
        D = xf.shape[-1]
        y = torch.empty(xf.shape, dtype=out_dtype, device=x.device)
        rstd = torch.empty(xf.numel() // D, dtype=torch.float32, device=x.device)
        ext().rmsnorm_fwd(xf, w.float().contiguous(), y, rstd, eps)
        ctx.save_for_backward(xf, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        xf, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        if dy.dtype not in (torch.float32, torch.bfloat16):
            dy = dy.float()
        dx = torch.empty(xf.shape, dtype=torch.float32, device=xf.device)
        dw = torch.zeros(xf.shape[-1], dtype=torch.float32, device=xf.device)
        ext().rmsnorm_bwd(dy, xf, w.float().contiguous(), rstd, dx, dw, False)
        return dx, dw.to(w.dtype), None, None


def rms_norm_cuda(x, w, eps, out_dtype):
    return RMSNormFn.apply(x, w, eps, out_dtype)


class AddNormFn(torch.autograd.Function):
    """``x_new = x + rs * a`` and ``h = RMSNorm(x_new) * w`` (bf16) in one kernel
    each way; ``rs`` is the block's residual-scale parameter (read on the
    device, no host synchronisation)."""

    @staticmethod
    def forward(ctx, x, a, rs, w, eps):
        shape = x.shape
        D = shape[-1]
        x2 = x.float().reshape(-1, D).contiguous()
        a2 = a.float().reshape(-1, D).contiguous()
        T = x2.shape[0]
        xn = torch.empty_like(x2)
        h = torch.empty(T, D, dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty(T, dtype=torch.float32, device=x.device)
        rsf = rs.detach().float().reshape(1).contiguous()
        wf = w.detach().float().contiguous()
        ext().add_norm_fwd(x2, a2, rsf, wf, eps, xn, h, rstd)
        ctx.save_for_backward(xn, a2, rsf, wf, rstd)
        ctx.meta = (shape, rs.dtype, w.dtype)
        return xn.view(shape), h.view(shape)

    @staticmethod
    def backward(ctx, g, dh):
        xn, a2, rsf, wf, rstd = ctx.saved_tensors
        shape, rs_dtype, w_dtype = ctx.meta
        D = shape[-1]
        dh = (torch.zeros(xn.shape, dtype=torch.bfloat16, device=xn.device) if dh is None
              else dh.reshape(-1, D).to(torch.bfloat16).contiguous())
        g = None if g is None else g.reshape(-1, D).float().contiguous()
        dx = torch.empty_like(xn)
        da = torch.empty_like(xn)
        buf = torch.zeros(D + 4, dtype=torch.float32, device=xn.device)   # dw | drs, one fill
        dw, drs = buf[:D], buf[D:D + 1]
        ext().add_norm_bwd(g, dh, xn, a2, rsf, wf, rstd, dx, da, drs, dw)
        return dx.view(shape), da.view(shape), drs.reshape(()).to(rs_dtype), dw.to(w_dtype), None


def add_rms_norm_cuda(x, a, rs, w, eps):
    return AddNormFn.apply(x, a, rs, w, eps)


class RopeFn(torch.autograd.Function):
    """In-place rotary embedding of ``x [B, S, N, H]`` (bf16)."""

    @staticmethod
    def forward(ctx, x, cos, sin, positions):
        B, S, N, H = x.shape
        x3 = x.view(B * S, N, H)
        ext().rope_apply(x3, cos.contiguous(), sin.contiguous(), S,
                         None if positions is None else positions.reshape(-1).long().contiguous(),
                         False)
        ctx.mark_dirty(x)
        ctx.save_for_backward(cos, sin)
        ctx.positions = positions
        return x

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        B, S, N, H = dy.shape
        d = dy.to(torch.bfloat16).contiguous().clone()
        pos = ctx.positions
        ext().rope_apply(d.view(B * S, N, H), cos.contiguous(), sin.contiguous(), S,
                         None if pos is None else pos.reshape(-1).long().contiguous(), True)
        return d, None, None, None


def rope_cuda(q, k, cos, sin, positions=None):
    q = RopeFn.apply(q.contiguous(), cos, sin, positions)
    k = RopeFn.apply(k.contiguous(), cos, sin, positions)
    return q, k


class SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        R, F2 = gu.shape
        h = torch.empty(R, F2 // 2, dtype=torch.bfloat16, device=gu.device)
        ext().swiglu_fwd(gu, h)
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dh.to(torch.bfloat16).contiguous(), gu, dgu)
        return dgu


def swiglu_cuda(gu):
    shp = gu.shape
    return SwiGLUFn.apply(gu.reshape(-1, shp[-1])).view(*shp[:-1], shp[-1] // 2)


class EmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, w):
        tok = tokens.reshape(-1).long().contiguous()
        D = w.shape[1]
        x = torch.empty(tok.numel(), D, dtype=torch.float32, device=w.device)
        ext().embed_fwd(tok, w.detach(), x)
        ctx.save_for_backward(tok)
        ctx.param = w
        ctx.shape = tokens.shape
        return x.view(*tokens.shape, D)

    @staticmethod
    def backward(ctx, dx):
        (tok,) = ctx.saved_tensors
        from .dense import main_grad
        ext().embed_bwd(tok, dx.float().contiguous().view(tok.numel(), -1), main_grad(ctx.param))
        return None, None


def embedding_cuda(tokens, w):
    return EmbedFn.apply(tokens, w)
