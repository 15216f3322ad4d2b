"""KDA layer on the native kernels (model/kda.py:240-376 semantics).

    [q|k|v|f0|g0] = h @ [wq|wk|wv|f_proj0|g_proj0]     one fused bf16 GEMM
    braw = h @ wb;  f = f0 @ f_proj1;  gl = g0 @ g_proj1  (fp32 outputs)
    q, k, v, g, beta = prep(...)   conv4 + SiLU (+ L2 norm for q, k), decay, sigmoid
    o = chunked gated delta rule (fp32)
    y = RMSNorm_V(o) * o_norm * sigmoid(gl + bias) @ wo   (norm and gate in one kernel)
"""
from __future__ import annotations

import math

import torch

from ._ext import ext
from .dense import linear_fused


def chunk_size(dk: int) -> int:
    return int(ext().kda_chunk_size(dk))


class KdaCoreFn(torch.autograd.Function):
    """Chunk-parallel gated delta rule; q,k,v,g ``[B,S,H,K]`` fp32, beta ``[B,S,H]``."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, scale):
        q, k, v, g, beta = (t.float().contiguous() for t in (q, k, v, g, beta))
        B, S, H, K = q.shape
        C = chunk_size(K)
        NC = (S + C - 1) // C
        dev = q.device
        o = torch.empty_like(v)
        f32 = dict(dtype=torch.float32, device=dev)
        Wt = torch.empty(B, H, NC, C, K, **f32)
        Ut = torch.empty(B, H, NC, C, K, **f32)
        Kh = torch.empty(B, H, NC, C, K, **f32)
        Qg = torch.empty(B, H, NC, C, K, **f32)
        Pm = torch.empty(B, H, NC, C, C, **f32)
        gC = torch.empty(B, H, NC, K, **f32)
        states = torch.empty(B, H, NC, K, K, **f32)
        ext().kda_fwd(q, k, v, g, beta, float(scale), o, Wt, Ut, Kh, Qg, Pm, gC, states, None, None)
        del Ut
        ctx.save_for_backward(q, k, v, g, beta, Wt, Kh, Qg, Pm, gC, states)
        ctx.scale = float(scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, g, beta, Wt, Kh, Qg, Pm, gC, states = ctx.saved_tensors
        do = do.float().contiguous()
        dstates = torch.empty_like(states)
        dq, dk, dv, dg = (torch.empty_like(q) for _ in range(4))
        dbeta = torch.empty_like(beta)
        ext().kda_bwd(q, k, v, g, beta, ctx.scale, do, Wt, Kh, Qg, Pm, gC, states, dstates,
                      dq, dk, dv, dg, dbeta)
        return dq, dk, dv, dg, dbeta, None


def kda_chunked_cuda(q, k, v, g, beta, scale, chunk=None):
    return KdaCoreFn.apply(q, k, v, g, beta, scale)


class KdaPrepFn(torch.autograd.Function):
    """ShortConv4 + SiLU (+ L2 norm) for q/k/v, decay gate and beta."""

    @staticmethod
    def forward(ctx, raw, f, braw, wq, wk, wv, a_log, dt_bias, gate_mode, S, H, K):
        T = raw.shape[0]
        dev = raw.device
        q = torch.empty(T, H, K, dtype=torch.float32, device=dev)
        k, v, g = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
        beta = torch.empty(T, H, dtype=torch.float32, device=dev)
        args = (raw, wq.float().contiguous(), wk.float().contiguous(), wv.float().contiguous(),
                f.float().contiguous(), a_log.float().contiguous(), dt_bias.float().contiguous())
        ext().kda_prep_fwd(*args, braw.float().contiguous(), gate_mode, S, q, k, v, g, beta)
        ctx.save_for_backward(raw, f, wq, wk, wv, a_log, dt_bias, beta)
        ctx.meta = (gate_mode, S, H, K)
        return q, k, v, g, beta

    @staticmethod
    def backward(ctx, dq, dk, dv, dg, dbeta):
        raw, f, wq, wk, wv, a_log, dt_bias, beta = ctx.saved_tensors
        gate_mode, S, H, K = ctx.meta
        T = raw.shape[0]
        HK = H * K
        dev = raw.device
        z = lambda t: torch.zeros_like(t) if t is None else t.float().contiguous()
        dq, dk, dv, dg = z(dq), z(dk), z(dv), z(dg)
        dbeta = torch.zeros(T, H, device=dev) if dbeta is None else dbeta.float().contiguous()
        dconv = torch.empty(T, 3 * HK, dtype=torch.float32, device=dev)
        df = torch.empty(T, HK, dtype=torch.float32, device=dev)
        dbraw = torch.empty(T, H, dtype=torch.float32, device=dev)
        d_alog = torch.zeros(H, dtype=torch.float32, device=dev)
        d_dtb = torch.zeros(HK, dtype=torch.float32, device=dev)
        ld = raw.stride(0)
        draw_full = torch.empty(T, ld, dtype=torch.bfloat16, device=dev)
        draw = draw_full[:, :3 * HK]
        dwq = torch.zeros(HK, 1, 4, dtype=torch.float32, device=dev)
        dwk, dwv = torch.zeros_like(dwq), torch.zeros_like(dwq)
        ext().kda_prep_bwd(raw, wq.float().contiguous(), wk.float().contiguous(),
                           wv.float().contiguous(), f.float().contiguous(),
                           a_log.float().contiguous(), dt_bias.float().contiguous(), beta,
                           gate_mode, S, dq, dk, dv, dg, dbeta, dconv, df, dbraw, d_alog, d_dtb,
                           draw, dwq, dwk, dwv)
        return (draw, df, dbraw, dwq, dwk, dwv, d_alog, d_dtb, None, None, None, None)


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
        dw = torch.zeros_like(wf)
        dgb = torch.zeros_like(gbf)
        ext().kda_out_gate_bwd(dy, o, gl, wf, gbf, rstd, do, dgl, dw, dgb)
        return do, dgl, dw.to(ctx.dtypes[0]), dgb.to(ctx.dtypes[1])


def kda_layer_cuda(mod, h, dtype):
    B, S, D = h.shape
    T = B * S
    H, K = mod.n_heads, mod.head_dim
    HK = H * K
    x2 = h.reshape(T, D)
    big = linear_fused(x2, [mod.wq, mod.wk, mod.wv, mod.f_proj0, mod.g_proj0], torch.bfloat16)
    braw = linear_fused(x2, [mod.wb], torch.float32)
    raw = big[:, :3 * HK]
    f = linear_fused(big[:, 3 * HK:3 * HK + K], [mod.f_proj1], torch.float32)
    gl = linear_fused(big[:, 3 * HK + K:3 * HK + 2 * K], [mod.g_proj1], torch.float32)
    gate_mode = 0 if mod.gate == "kimi" else 1
    q, k, v, g, beta = KdaPrepFn.apply(raw, f, braw, mod.q_conv.weight, mod.k_conv.weight,
                                       mod.v_conv.weight, mod.a_log, mod.dt_bias, gate_mode, S, H, K)
    o = KdaCoreFn.apply(q.view(B, S, H, K), k.view(B, S, H, K), v.view(B, S, H, K),
                        g.view(B, S, H, K), beta.view(B, S, H), 1.0 / math.sqrt(K))
    if K in (32, 64, 128):
        y = KdaOutGateFn.apply(o.view(T, H, K), gl, mod.o_norm, mod.g_proj1_bias)
    else:
        var = (o * o).mean(-1, keepdim=True)
        on = o * torch.rsqrt(var + 1e-5) * mod.o_norm
        gate = torch.sigmoid(gl + mod.g_proj1_bias).view(B, S, H, K)
        y = (on * gate).reshape(T, HK).to(torch.bfloat16)
    out = linear_fused(y, [mod.wo], torch.float32)
    return out.view(B, S, D)
