"""MoE layer and dense SwiGLU FFN on the native kernels (model/moe.py).

Forward of one MoE layer (dropless, the reference's ragged dispatch):
  router kernel   fp32 logits, sigmoid(+bias)/softmax scores, top-k, weights,
                  per-sequence counts / probability sums / z and entropy sums
  plan kernels    stable counting sort of (token, slot) by expert into a row
                  buffer whose expert segments start at multiples of 128
  gather          Xp[row] = h[token(row)]           (pad rows zero)
  grouped GEMMs   GU = Xp @ [W_gate | W_up] (per expert), H = silu(G) * U,
                  Y = H @ W_down                     (tcgen05, grouped over rows)
  shared expert   dense GEMMs + SwiGLU, fp32 output
  combine         out[t] += sum_k bf16(w_tk) * Y[row(t, k)]
Backward mirrors it; expert weight gradients use the grouped-K GEMM (the
contraction runs over each expert's row segment) accumulating into the
parameters' fp32 main_grad; the router backward covers the combine weights,
the z-loss and the sequence-wise balance loss.  No host synchronisation: the
row buffer is sized for the worst case and the grouped GEMMs read their tile
counts from device memory.
"""
from __future__ import annotations

import os

import torch

from ._ext import ext
from .dense import _bf16, _work, main_grad
from .norm import SwiGLUFn

# The expert backward runs dh = dY W_down^T with the SwiGLU backward in the
# GEMM's epilogue (one kernel, dh never stored); HB_MOE_FUSED_SWIGLU=0 selects
# the grouped GEMM followed by the standalone SwiGLU backward kernel.
FUSED_SWIGLU_BWD = os.environ.get("HB_MOE_FUSED_SWIGLU", "1") != "0"


def _bn(n: int) -> int:
    return 256 if n >= 256 else 128


class SwiGLUFFNFn(torch.autograd.Function):
    """down(silu(x @ gate) * (x @ up)) -> fp32."""

    @staticmethod
    def forward(ctx, x, wg, wu, wd):
        xb = _bf16(x)
        g, u, d = _work(wg), _work(wu), _work(wd)
        T = xb.shape[0]
        F = g.shape[1]
        gu = torch.empty(T, 2 * F, dtype=torch.bfloat16, device=x.device)
        ext().gemm(xb, g, gu[:, :F], False, False, False, 1.0)
        ext().gemm(xb, u, gu[:, F:], False, False, False, 1.0)
        hh = torch.empty(T, F, dtype=torch.bfloat16, device=x.device)
        ext().swiglu_fwd(gu, hh)
        out = torch.empty(T, d.shape[1], dtype=torch.float32, device=x.device)
        ext().gemm(hh, d, out, False, False, False, 1.0)
        ctx.save_for_backward(xb, g, u, d, gu, hh)
        ctx.params = (wg, wu, wd)
        ctx.x_dtype = x.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        xb, g, u, d, gu, hh = ctx.saved_tensors
        wg, wu, wd = ctx.params
        F = g.shape[1]
        db = _bf16(dout)
        dh = torch.empty_like(hh)
        ext().gemm(db, d, dh, False, True, False, 1.0)
        ext().gemm(hh, db, main_grad(wd), True, False, True, 1.0)
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dh, gu, dgu)
        dx = torch.empty(xb.shape, dtype=torch.float32, device=xb.device)
        ext().gemm(dgu[:, :F], g, dx, False, True, False, 1.0)
        ext().gemm(dgu[:, F:], u, dx, False, True, True, 1.0)
        ext().gemm(xb, dgu[:, :F], main_grad(wg), True, False, True, 1.0)
        ext().gemm(xb, dgu[:, F:], main_grad(wu), True, False, True, 1.0)
        return dx.to(ctx.x_dtype), None, None, None


def swiglu_ffn_cuda(x, wg, wu, wd, dtype=torch.bfloat16):
    return SwiGLUFFNFn.apply(x, wg, wu, wd)


class ExpertGather:
    """Per-MoE-layer state of the fused expert-weight all-gather: every rank's
    shard address of each expert tensor, the local gathered copies and the
    tile flags shared by the three GEMMs (they run one after another)."""

    def __init__(self, ptrs: dict, rank: int, groups_per_rank: int, shapes: dict, device):
        self.ptrs, self.rank, self.gpr = ptrs, rank, groups_per_rank
        self.bufs = {k: torch.empty(s, dtype=torch.bfloat16, device=device) for k, s in shapes.items()}
        n = 0
        for s in shapes.values():
            G, Kd, Nd = s
            n = max(n, G * ((Kd + 63) // 64) * ((Nd + _bn(Nd) - 1) // _bn(Nd)))
        self.flags = torch.zeros(n, dtype=torch.int32, device=device)

    def gemm(self, a, name, c, starts, counts, tprefix):
        ext().grouped_gemm_m_gather(a, self.ptrs[name], self.rank, self.gpr, self.bufs[name],
                                    self.flags, c, starts, counts, tprefix)


_ONE_GROUP: dict = {}


def _one_group(T: int, tiles_n: int, dev) -> tuple:
    """Group arrays of a grouped GEMM over ONE group of T rows (the shared
    expert on the expert kernels), cached per shape: start 0, count T, tile
    prefix [0, T / 128 * tiles_n]."""
    key = (T, tiles_n, str(dev))
    if key not in _ONE_GROUP:
        i32 = dict(dtype=torch.int32, device=dev)
        _ONE_GROUP[key] = (torch.zeros(1, **i32), torch.full((1,), T, **i32),
                           torch.tensor([0, T // 128 * tiles_n], **i32))
    return _ONE_GROUP[key]


def _shared_fused(T: int, Fs: int) -> bool:
    """The fused SwiGLU kernels write whole 128-row tiles (pad rows zeroed), so
    the shared expert uses them when T fills whole tiles."""
    return T % 128 == 0 and Fs % 128 == 0


class MoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, mod, B, S):
        dev = h.device
        xb = _bf16(h)
        T, D = xb.shape
        N, K = mod.n_experts, mod.n_active
        softmax = mod.router_type == "softmax"
        Wr = mod.router.detach().float().contiguous()
        bias = mod.bias.detach().float().contiguous()
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        logits = torch.empty(T, N, **f32)
        topi = torch.empty(T, K, **i32)
        topw = torch.empty(T, K, **f32)
        stats = torch.zeros(2 * B * N + 2, **f32)   # counts | probs | sums, one fill
        seq_counts = stats[:B * N].view(B, N)
        seq_probs = stats[B * N:2 * B * N].view(B, N)
        sums = stats[2 * B * N:]
        ext().router_fwd(xb, Wr, bias, S, K, softmax, float(mod.scaling), logits, topi, topw,
                         seq_counts, seq_probs, sums)
        # dispatch plan
        wg, wu, wd = _work(mod.expert_w_gate), _work(mod.expert_w_up), _work(mod.expert_w_down)
        F = wg.shape[2]
        R = T * K + N * 127
        R = (R + 127) // 128 * 128
        counts = torch.empty(N, **i32)
        starts = torch.empty(N, **i32)
        tprefix_f = torch.empty(N + 1, **i32)
        padded = torch.empty(N, **i32)
        total = torch.empty(1, **i32)
        pos = torch.empty(T, K, **i32)
        row_src = torch.full((R,), -1, **i32)
        ext().moe_plan(topi, N, (F + _bn(F) - 1) // _bn(F), counts, starts, tprefix_f, padded,
                       total, pos, row_src)
        # tile prefix for the D-wide down projection (tiles_n differs)
        tn_f, tn_d = (F + _bn(F) - 1) // _bn(F), (D + _bn(D) - 1) // _bn(D)
        tprefix_d = (tprefix_f // tn_f * tn_d).to(torch.int32)
        xp = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
        ext().moe_gather(xb, row_src, xp, K)
        gu = torch.empty(R, 2 * F, dtype=torch.bfloat16, device=dev)
        gat = getattr(mod, "_gather", None)
        if gat is not None:
            # FSDP expert weights: the all-gather runs inside these GEMMs (peer
            # tiles land in gat.bufs, which the backward then reads)
            wg, wu, wd = (gat.bufs[k] for k in ("expert_w_gate", "expert_w_up", "expert_w_down"))
            gat.gemm(xp, "expert_w_gate", gu[:, :F], starts, counts, tprefix_f)
            gat.gemm(xp, "expert_w_up", gu[:, F:], starts, counts, tprefix_f)
        hh = torch.empty(R, F, dtype=torch.bfloat16, device=dev)
        if gat is None and F % 128 == 0:
            # gate and up in one GEMM (tile j: 128 columns of each), the SwiGLU
            # in its epilogue; pad rows of h -> 0 (grouped-K reads them)
            tprefix_v = (tprefix_f // tn_f * (2 * F // 256)).to(torch.int32)
            ext().grouped_gemm_m_swiglu_fwd(xp, wg, wu, hh, gu, starts, counts, tprefix_v)
        else:
            if gat is None:
                ext().grouped_gemm_m(xp, wg, gu[:, :F], starts, counts, tprefix_f, False)
                ext().grouped_gemm_m(xp, wu, gu[:, F:], starts, counts, tprefix_f, False)
            ext().swiglu_fwd(gu, hh, row_src)  # pad rows -> 0 (grouped-K reads them)
        y = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
        if gat is not None:
            gat.gemm(hh, "expert_w_down", y, starts, counts, tprefix_d)
        else:
            ext().grouped_gemm_m(hh, wd, y, starts, counts, tprefix_d, False)
        # shared expert (fp32 out) + combine
        if mod.n_shared != 1:
            raise NotImplementedError("GPU MoE supports one shared expert")
        sg, su, sd = _work(mod.shared_w_gate), _work(mod.shared_w_up), _work(mod.shared_w_down)
        Fs = sg.shape[1]
        sgu = torch.empty(T, 2 * Fs, dtype=torch.bfloat16, device=dev)
        shh = torch.empty(T, Fs, dtype=torch.bfloat16, device=dev)
        if _shared_fused(T, Fs):
            # the fused expert kernels with one group of T rows
            gs1, gc1, gt1 = _one_group(T, 2 * Fs // 256, dev)
            ext().grouped_gemm_m_swiglu_fwd(xb, sg.unsqueeze(0), su.unsqueeze(0), shh, sgu,
                                            gs1, gc1, gt1)
        else:
            ext().gemm(xb, sg, sgu[:, :Fs], False, False, False, 1.0)
            ext().gemm(xb, su, sgu[:, Fs:], False, False, False, 1.0)
            ext().swiglu_fwd(sgu, shh)
        out = torch.empty(T, D, **f32)
        ext().gemm(shh, sd, out, False, False, False, 1.0)
        ext().moe_combine(y, pos, topw, out)
        # aux (model/moe.py:253-293)
        z = sums[0] / T
        ent = sums[1] / T
        frac = seq_counts / (S * K)
        mean_probs = seq_probs / S
        bal = (N * (frac * mean_probs).sum(-1)).mean()
        expert_counts = seq_counts.sum(0)
        ctx.save_for_backward(xb, logits, topi, topw, pos, row_src, starts, counts, padded,
                              tprefix_f, tprefix_d, xp, gu, hh, y, sgu, shh, frac)
        ctx.mod = mod
        ctx.expert_w = (wg, wu, wd)
        ctx.meta = (B, S, T, D, N, K, F, Fs, R, softmax)
        ctx.mark_non_differentiable(ent, expert_counts)
        return out, z, bal, ent, expert_counts

    @staticmethod
    def backward(ctx, dout, dz, dbal, dent, dcounts):
        (xb, logits, topi, topw, pos, row_src, starts, counts, padded, tprefix_f, tprefix_d, xp,
         gu, hh, y, sgu, shh, frac) = ctx.saved_tensors
        mod = ctx.mod
        B, S, T, D, N, K, F, Fs, R, softmax = ctx.meta
        dev = xb.device
        dout = dout.float().contiguous()
        db = dout.to(torch.bfloat16)
        dy = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
        dtopw = torch.empty(T, K, dtype=torch.float32, device=dev)
        ext().moe_combine_bwd(dout, y, pos, topw, row_src, dy, dtopw)
        # shared expert
        sg, su, sd = _work(mod.shared_w_gate), _work(mod.shared_w_up), _work(mod.shared_w_down)
        dsgu = torch.empty_like(sgu)
        dx = torch.empty(T, D, dtype=torch.float32, device=dev)
        if _shared_fused(T, Fs):
            gs1, gc1, gtf = _one_group(T, (Fs + _bn(Fs) - 1) // _bn(Fs), dev)
            ext().grouped_gemm_m_swiglu_bwd(db, sd.unsqueeze(0), sgu, dsgu, gs1, gc1, gtf)
            gtd = _one_group(T, (D + _bn(D) - 1) // _bn(D), dev)[2]
            ext().grouped_gemm_m_cat2(dsgu, sg.unsqueeze(0), su.unsqueeze(0), dx, gs1, gc1, gtd)
        else:
            dsh = torch.empty_like(shh)
            ext().gemm(db, sd, dsh, False, True, False, 1.0)
            ext().swiglu_bwd(dsh, sgu, dsgu)
            ext().gemm(dsgu[:, :Fs], sg, dx, False, True, False, 1.0)
            ext().gemm(dsgu[:, Fs:], su, dx, False, True, True, 1.0)
        ext().gemm(shh, db, main_grad(mod.shared_w_down), True, False, True, 1.0)
        ext().gemm(xb, dsgu[:, :Fs], main_grad(mod.shared_w_gate), True, False, True, 1.0)
        ext().gemm(xb, dsgu[:, Fs:], main_grad(mod.shared_w_up), True, False, True, 1.0)
        wg, wu, wd = ctx.expert_w
        dgu = torch.empty_like(gu)
        if FUSED_SWIGLU_BWD:
            # dh = dy W_down^T stays in TMEM; the epilogue writes dgu (pad rows 0)
            ext().grouped_gemm_m_swiglu_bwd(dy, wd, gu, dgu, starts, counts, tprefix_f)
        else:
            dhh = torch.empty(R, F, dtype=torch.bfloat16, device=dev)
            ext().grouped_gemm_m(dy, wd, dhh, starts, counts, tprefix_f, True)
            ext().swiglu_bwd(dhh, gu, dgu, row_src)  # pad rows -> 0 for the grouped-K GEMMs
        ext().grouped_gemm_k(hh, dy, main_grad(mod.expert_w_down), starts, padded, True)
        tn_d = (D + _bn(D) - 1) // _bn(D)
        tn_f = (F + _bn(F) - 1) // _bn(F)
        tprefix_dx = (tprefix_f // tn_f * tn_d).to(torch.int32)
        if F % 64 == 0:
            # one GEMM over K = 2F: [dg | du] @ [W_gate | W_up]^T, rows in bf16
            # (the reference's ragged_dot input cotangent is bf16 as well)
            dxp = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
            ext().grouped_gemm_m_cat2(dgu, wg, wu, dxp, starts, counts, tprefix_dx)
        else:
            dxp = torch.empty(R, D, dtype=torch.float32, device=dev)
            ext().grouped_gemm_m(dgu[:, :F], wg, dxp, starts, counts, tprefix_dx, True, False)
            ext().grouped_gemm_m(dgu[:, F:], wu, dxp, starts, counts, tprefix_dx, True, True)
        ext().grouped_gemm_k(xp, dgu[:, :F], main_grad(mod.expert_w_gate), starts, padded, True)
        ext().grouped_gemm_k(xp, dgu[:, F:], main_grad(mod.expert_w_up), starts, padded, True)
        # router backward (z-loss, balance loss, combine weights)
        dz = torch.zeros((), device=dev) if dz is None else dz
        dbal = torch.zeros((), device=dev) if dbal is None else dbal
        coef_z = (dz.float() * 2.0 / T).reshape(1).contiguous()
        bal_coef = (dbal.float() * N / (B * S) * frac).contiguous()
        dlogits = torch.empty(T, N, dtype=torch.float32, device=dev)
        ext().router_bwd(logits, topi, dtopw, bal_coef, S, softmax, float(mod.scaling), coef_z,
                         dlogits)
        ext().router_grads(xb, mod.router.detach().float().contiguous(), dlogits, dx,
                           main_grad(mod.router))
        # the routed rows last: their sum with dx goes out in bf16 (no separate cast)
        dxb = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        ext().moe_scatter_add(dxp, pos, dx, dxb)
        return dxb, None, None, None


def moe_layer_cuda(mod, h, dtype):
    B, S, D = h.shape
    out, z, bal, ent, counts = MoEFn.apply(h.reshape(B * S, D), mod, B, S)
    aux = {"router_z_loss": z, "balance_loss": bal, "mean_entropy": ent,
           "expert_counts": counts}
    return out.view(B, S, D), aux
