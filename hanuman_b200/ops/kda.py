"""KDA layer on the native kernels (model/kda.py:240-376 semantics).

    [q|k|v|f0|g0] = h @ [wq|wk|wv|f_proj0|g_proj0]     one bf16 buffer
    braw = h @ wb;  f = f0 @ f_proj1;  gl = g0 @ g_proj1  (fp32 outputs)
    q, k, v, g, beta = prep(...)   conv4 + SiLU (+ L2 norm for q, k), decay, sigmoid
      (the projections and the prep are one autograd node, KdaFrontFn)
    o = chunked gated delta rule (fp32)
    y = RMSNorm_V(o) * o_norm * sigmoid(gl + bias) @ wo   (norm and gate in one kernel)
"""
from __future__ import annotations

import math
import os

import torch

from ._ext import ext
from .dense import _bf16, _gemm_or_narrow, _work, linear_fused, main_grad


def chunk_size(dk: int) -> int:
    return int(ext().kda_chunk_size(dk))


def use_chunk64(dk: int) -> bool:
    """Head dim 64 runs the chunk-64 sub-block kernels (csrc/kda/kda64.cu);
    HB_KDA_CHUNK64=0 selects the chunk-32 kernels (csrc/kda/kda.cu) instead."""
    return dk == 64 and os.environ.get("HB_KDA_CHUNK64", "1") != "0"


class KdaCoreFn(torch.autograd.Function):
    """Chunk-parallel gated delta rule; q,k,v,g ``[B,S,H,K]`` fp32, beta ``[B,S,H]``.

    With ``recompute`` the forward keeps only its inputs and the backward
    re-runs the forward kernels for the chunk intermediates (Wt, Ut, Kh, Qg,
    P, states, ...: about 9 fp32 values per token, head and channel), which
    are the largest activations of the model (the ``dots`` remat policies)."""

    @staticmethod
    def _run_fwd(q, k, v, g, beta, scale):
        B, S, H, K = q.shape
        c64 = use_chunk64(K)
        C = 64 if c64 else chunk_size(K)
        NC = (S + C - 1) // C
        f32 = dict(dtype=torch.float32, device=q.device)
        o = torch.empty_like(v)
        Wt, Ut, Kh, Qg = (torch.empty(B, H, NC, C, K, **f32) for _ in range(4))
        Pm = torch.empty(B, H, NC, C, C, **f32)
        gC = torch.empty(B, H, NC, K, **f32)
        states = torch.empty(B, H, NC, K, K, **f32)
        if c64:
            Linv = torch.empty(B, H, NC, C, C, **f32)
            Am = torch.empty(B, H, NC, C, C, **f32)
            U = torch.empty(B, H, NC, C, K, **f32)
            ext().kda_fwd64(q, k, v, g, beta, float(scale), o, Wt, Ut, Kh, Qg, Pm, gC, states, Linv, Am, U)
            return o, (Wt, Ut, Kh, Qg, Pm, gC, states, Linv, Am, U)
        ext().kda_fwd(q, k, v, g, beta, float(scale), o, Wt, Ut, Kh, Qg, Pm, gC, states, None, None)
        return o, (Wt, Kh, Qg, Pm, gC, states)

    @staticmethod
    def forward(ctx, q, k, v, g, beta, scale, recompute=False):
        q, k, v, g, beta = (t.float().contiguous() for t in (q, k, v, g, beta))
        ctx.scale = float(scale)
        ctx.c64 = use_chunk64(q.shape[-1])
        ctx.recompute = bool(recompute)
        o, inter = KdaCoreFn._run_fwd(q, k, v, g, beta, scale)
        if recompute:
            del inter
            ctx.save_for_backward(q, k, v, g, beta)
        else:
            ctx.save_for_backward(q, k, v, g, beta, *inter)
        return o

    @staticmethod
    def backward(ctx, do):
        do = do.float().contiguous()
        q, k, v, g, beta = ctx.saved_tensors[:5]
        inter = ctx.saved_tensors[5:] if not ctx.recompute else \
            KdaCoreFn._run_fwd(q, k, v, g, beta, ctx.scale)[1]
        dq, dk, dv, dg = (torch.empty_like(q) for _ in range(4))
        dbeta = torch.empty_like(beta)
        if ctx.c64:
            Wt, Ut, Kh, Qg, Pm, gC, states, Linv, Am, U = inter
            dstates, dSq = torch.empty_like(states), torch.empty_like(states)
            dU, dUp, dQg, dKh, dWt, dP = (torch.empty_like(Wt) for _ in range(6))
            dgC = torch.empty_like(gC)
            ext().kda_bwd64(q, k, v, g, beta, ctx.scale, do, Wt, Ut, Kh, Qg, Pm, gC, states, Linv, Am, U,
                            dstates, dU, dUp, dSq, dQg, dKh, dWt, dP, dgC, dq, dk, dv, dg, dbeta)
            return dq, dk, dv, dg, dbeta, None, None
        Wt, Kh, Qg, Pm, gC, states = inter
        dstates = torch.empty_like(states)
        ext().kda_bwd(q, k, v, g, beta, ctx.scale, do, Wt, Kh, Qg, Pm, gC, states, dstates,
                      dq, dk, dv, dg, dbeta)
        return dq, dk, dv, dg, dbeta, None, None


def kda_chunked_cuda(q, k, v, g, beta, scale, chunk=None):
    return KdaCoreFn.apply(q, k, v, g, beta, scale)


class KdaFrontFn(torch.autograd.Function):
    """Everything between the block's normed input and the delta rule, as ONE
    autograd node (model/kda.py:248-284):

        [q|k|v|f0|g0] = x @ [wq|wk|wv|f_proj0|g_proj0]   (one bf16 buffer)
        braw = x @ wb;  f = f0 @ f_proj1;  gl = g0 @ g_proj1   (fp32)
        q, k, v, g, beta = ShortConv4 + SiLU (+ L2 norm), decay gate, sigmoid

    Returns q, k, v, g, beta and gl (the output gate's logits).  The backward
    writes d[q|k|v|f0|g0] into one buffer (the prep kernel fills the q|k|v
    columns, the low-rank GEMMs the f0|g0 columns) and accumulates a single
    fp32 input gradient, so autograd never zero-fills, slices or sums
    per-consumer gradients of x or of the projection buffer."""

    @staticmethod
    def forward(ctx, x, wq, wk, wv, f0, g0, wb, f1, g1, cq, ck, cv, a_log, dt_bias,
                gate_mode, S, H, K):
        xb = _bf16(x)
        T = xb.shape[0]
        HK = H * K
        dev = xb.device
        pw = [_work(w) for w in (wq, wk, wv, f0, g0)]
        wbw, f1w, g1w = _work(wb), _work(f1), _work(g1)
        W = 3 * HK + 2 * K
        big = torch.empty(T, W, dtype=torch.bfloat16, device=dev)
        off = 0
        for w in pw:
            _gemm_or_narrow(xb, w, big[:, off:off + w.shape[1]], False, False, False)
            off += w.shape[1]
        f32 = dict(dtype=torch.float32, device=dev)
        braw = torch.empty(T, H, **f32)
        _gemm_or_narrow(xb, wbw, braw, False, False, False)
        f = torch.empty(T, HK, **f32)
        _gemm_or_narrow(big[:, 3 * HK:3 * HK + K], f1w, f, False, False, False)
        gl = torch.empty(T, HK, **f32)
        _gemm_or_narrow(big[:, 3 * HK + K:], g1w, gl, False, False, False)
        q = torch.empty(T, H, K, **f32)
        k, v, g = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
        beta = torch.empty(T, H, **f32)
        conv = [c.float().contiguous() for c in (cq, ck, cv)]
        al, dtb = a_log.float().contiguous(), dt_bias.float().contiguous()
        ext().kda_prep_fwd(big[:, :3 * HK], *conv, f, al, dtb, braw, gate_mode, S, q, k, v, g, beta)
        ctx.save_for_backward(xb, big, f, beta, *pw, wbw, f1w, g1w, *conv, al, dtb)
        ctx.params = (wq, wk, wv, f0, g0, wb, f1, g1)
        ctx.meta = (gate_mode, S, H, K, x.dtype)
        return q, k, v, g, beta, gl

    @staticmethod
    def backward(ctx, dq, dk, dv, dg, dbeta, dgl):
        (xb, big, f, beta, wq, wk, wv, wf0, wg0, wbw, f1w, g1w,
         cq, ck, cv, al, dtb) = ctx.saved_tensors
        gate_mode, S, H, K, x_dtype = ctx.meta
        T = xb.shape[0]
        HK = H * K
        W = big.shape[1]
        dev = xb.device
        z = lambda t: torch.zeros_like(f) if t is None else t.float().contiguous()
        dq, dk, dv, dg = z(dq), z(dk), z(dv), z(dg)
        dbeta = torch.zeros(T, H, device=dev) if dbeta is None else dbeta.float().contiguous()
        df = torch.empty(T, HK, dtype=torch.bfloat16, device=dev)
        dbraw = torch.empty(T, H, dtype=torch.float32, device=dev)
        # the five small parameter gradients share one zero-filled buffer (one fill launch)
        small = torch.zeros(HK + H + 3 * HK * 4, dtype=torch.float32, device=dev)
        d_dtb, d_alog = small[:HK], small[HK:HK + H]
        dcq, dck, dcv = (small[HK + H + i * HK * 4:HK + H + (i + 1) * HK * 4].view(HK, 1, 4)
                         for i in range(3))
        dbig = torch.empty(T, W, dtype=torch.bfloat16, device=dev)
        ext().kda_prep_bwd(big[:, :3 * HK], cq, ck, cv, f, al, dtb, beta, gate_mode, S,
                           dq, dk, dv, dg, dbeta, df, dbraw, d_alog, d_dtb,
                           dbig[:, :3 * HK], dcq, dck, dcv)
        p_wq, p_wk, p_wv, p_f0, p_g0, p_wb, p_f1, p_g1 = ctx.params
        # low-rank second stage: d f0 / d g0 straight into their dbig columns
        f0s, g0s = big[:, 3 * HK:3 * HK + K], big[:, 3 * HK + K:]
        dfb = df
        _gemm_or_narrow(dfb, f1w, dbig[:, 3 * HK:3 * HK + K], False, True, False)
        _gemm_or_narrow(f0s, dfb, main_grad(p_f1), True, False, True)
        if dgl is None:
            dbig[:, 3 * HK + K:].zero_()
        else:
            dglb = dgl.to(torch.bfloat16)
            _gemm_or_narrow(dglb, g1w, dbig[:, 3 * HK + K:], False, True, False)
            _gemm_or_narrow(g0s, dglb, main_grad(p_g1), True, False, True)
        # first stage: one fp32 input gradient over all six projections
        dx = torch.empty(xb.shape, dtype=torch.float32, device=dev) \
            if ctx.needs_input_grad[0] else None
        first = (wq, wk, wv, wf0, wg0)
        kseg = dx is not None and all(w.shape[1] % 64 == 0 for w in first)
        if kseg:
            # dx = dbig @ [wq|wk|wv|f_proj0|g_proj0]^T: one GEMM, K split by weight
            ext().gemm_kseg(dbig, list(first), dx, False)
        off = 0
        for i, (w, p) in enumerate(zip(first, (p_wq, p_wk, p_wv, p_f0, p_g0))):
            sl = dbig[:, off:off + w.shape[1]]
            if dx is not None and not kseg:
                _gemm_or_narrow(sl, w, dx, False, True, i > 0)
            _gemm_or_narrow(xb, sl, main_grad(p), True, False, True)
            off += w.shape[1]
        dbb = dbraw.to(torch.bfloat16)
        if dx is not None:
            _gemm_or_narrow(dbb, wbw, dx, False, True, True)
        _gemm_or_narrow(xb, dbb, main_grad(p_wb), True, False, True)
        if dx is not None and x_dtype != torch.float32:
            dx = dx.to(x_dtype)
        return (dx,) + (None,) * 8 + (dcq, dck, dcv, d_alog, d_dtb, None, None, None, None)


class KdaOutGateFn(torch.autograd.Function):
    """y = RMSNorm_K(o) * o_norm * sigmoid(gl + g_bias) as bf16 (one fused kernel each way)."""

    @staticmethod
    def forward(ctx, o, gl, w, gb):
        T, H, K = o.shape
        o = o.contiguous()
        gl = gl.float().contiguous()
        y = torch.empty(T, H * K, dtype=torch.bfloat16, device=o.device)
        rstd = torch.empty(T * H, dtype=torch.float32, device=o.device)
        wf, gbf = w.float().contiguous(), gb.float().contiguous()
        ext().kda_out_gate_fwd(o, gl, wf, gbf, 1e-5, y, rstd)
        ctx.save_for_backward(o, gl, wf, gbf, rstd)
        ctx.dtypes = (w.dtype, gb.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        o, gl, wf, gbf, rstd = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        do = torch.empty_like(o)
        dgl = torch.empty_like(gl)
        buf = torch.zeros(wf.numel() + gbf.numel(), dtype=torch.float32, device=o.device)
        dw, dgb = buf[:wf.numel()].view_as(wf), buf[wf.numel():].view_as(gbf)
        ext().kda_out_gate_bwd(dy, o, gl, wf, gbf, rstd, do, dgl, dw, dgb)
        return do, dgl, dw.to(ctx.dtypes[0]), dgb.to(ctx.dtypes[1])


def kda_layer_cuda(mod, h, dtype):
    B, S, D = h.shape
    T = B * S
    H, K = mod.n_heads, mod.head_dim
    HK = H * K
    x2 = h.reshape(T, D)
    gate_mode = 0 if mod.gate == "kimi" else 1
    q, k, v, g, beta, gl = KdaFrontFn.apply(
        x2, mod.wq, mod.wk, mod.wv, mod.f_proj0, mod.g_proj0, mod.wb, mod.f_proj1, mod.g_proj1,
        mod.q_conv.weight, mod.k_conv.weight, mod.v_conv.weight, mod.a_log, mod.dt_bias,
        gate_mode, S, H, K)
    o = KdaCoreFn.apply(q.view(B, S, H, K), k.view(B, S, H, K), v.view(B, S, H, K),
                        g.view(B, S, H, K), beta.view(B, S, H), 1.0 / math.sqrt(K),
                        getattr(mod, "recompute_core", False))
    if K in (32, 64, 128):
        y = KdaOutGateFn.apply(o.view(T, H, K), gl, mod.o_norm, mod.g_proj1_bias)
    else:
        var = (o * o).mean(-1, keepdim=True)
        on = o * torch.rsqrt(var + 1e-5) * mod.o_norm
        gate = torch.sigmoid(gl + mod.g_proj1_bias).view(B, S, H, K)
        y = (on * gate).reshape(T, HK).to(torch.bfloat16)
    out = linear_fused(y, [mod.wo], torch.float32)
    return out.view(B, S, D)
