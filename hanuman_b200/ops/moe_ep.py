"""Expert-parallel MoE layer (BASELINE configs 3 and 5) on the fused peer-memory
transport of ``csrc/moe/ep.cu``.

Every rank routes its own tokens, plans them per global expert (stable,
token-ordered), and keeps at most ``cap = ceil(capacity_factor * T * K / N)``
(rounded up to 128) rows per (source rank, expert).  The forward then runs

    ep_scatter   kept rows -> owner's recv[le][me][i]        (peer stores)
    ep_zero_pads rows [kept, cap) of the owner's blocks := 0; kept -> owner
    barrier
    grouped GEMMs on recv (gate|up -> SwiGLU -> down)         (tcgen05)
    ep_return    recv-order outputs -> source's ret[e][i]      (peer stores)
    barrier
    ep_combine   out[t] += sum_k w_tk * ret[e][i]  (+ shared expert, local)

and the backward sends ``w_tk * dout[t]`` to the owners the same way, runs the
grouped backward GEMMs (dW accumulates into the rank's own experts) and returns
the input gradient rows.  Dropped slots contribute nothing, as in a capacity-
factor dispatch.  ``transport='nccl'`` performs the same exchange with
``all_to_all_single`` on packed buffers (the baseline).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ._ext import ext
from .dense import _bf16, _work, main_grad


def _bn(n):
    return 256 if n >= 256 else 128


class EPContext:
    """Per-layer symmetric buffers and peer address tables for one MoE layer."""

    def __init__(self, layer, T: int, D: int, F: int, ctx, capacity_factor: float,
                 transport: str = "p2p"):
        import torch.distributed._symmetric_memory as symm
        self.E, self.me = ctx.world, ctx.rank
        self.N = layer.n_experts
        self.Nl = self.N // self.E
        self.K = layer.n_active
        self.D, self.F = D, F
        cf = capacity_factor if capacity_factor > 0 else 1.25
        self.cap = int(math.ceil(cf * T * self.K / self.N / 128.0)) * 128
        self.T = T
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.transport = transport
        rows_recv = self.Nl * self.E * self.cap
        rows_ret = self.N * self.cap
        group = dist.group.WORLD
        bf = torch.bfloat16

        def sym(n, dtype):
            t = symm.empty(n, dtype=dtype, device=dev)
            t.zero_()
            h = symm.rendezvous(t, group)
            ptrs = torch.tensor([int(p) for p in h.buffer_ptrs], dtype=torch.int64, device=dev)
            return t, h, ptrs

        self.recv, self._h1, self.recv_peers = sym(rows_recv * D, bf)
        self.ret, self._h2, self.ret_peers = sym(rows_ret * D, bf)
        self.drecv, self._h3, self.drecv_peers = sym(rows_recv * D, bf)
        self.dret, self._h4, self.dret_peers = sym(rows_ret * D, bf)
        self.cnt, self._h5, self.cnt_peers = sym(self.Nl * self.E, torch.int32)
        self.flags, self._h6, self.pads = sym(max(32, self.E), torch.int32)
        self.epoch = 0
        Ec = self.E * self.cap
        i32 = dict(dtype=torch.int32, device=dev)
        self.g_starts = torch.arange(self.Nl, **i32) * Ec
        self.g_counts = torch.full((self.Nl,), Ec, **i32)
        tn_f = (F + _bn(F) - 1) // _bn(F)
        tn_d = (D + _bn(D) - 1) // _bn(D)
        tiles_m = (Ec + 127) // 128
        self.tp_f = torch.arange(self.Nl + 1, **i32) * (tiles_m * tn_f)
        self.tp_d = torch.arange(self.Nl + 1, **i32) * (tiles_m * tn_d)
        torch.cuda.synchronize(dev)
        dist.barrier()

    def barrier(self):
        self.epoch += 1
        ext().p2p_barrier(self.pads, self.me, self.E, self.epoch)

    def views(self):
        rr = self.Nl * self.E * self.cap
        return (self.recv.view(rr, self.D), self.ret.view(self.N * self.cap, self.D),
                self.drecv.view(rr, self.D), self.dret.view(self.N * self.cap, self.D))


def _plan(topi, N):
    T, K = topi.shape
    dev = topi.device
    i32 = dict(dtype=torch.int32, device=dev)
    counts = torch.empty(N, **i32)
    starts = torch.empty(N, **i32)
    tp = torch.empty(N + 1, **i32)
    padded = torch.empty(N, **i32)
    total = torch.empty(1, **i32)
    pos = torch.empty(T, K, **i32)
    R = ((T * K + N * 127 + 127) // 128) * 128
    row_src = torch.full((R,), -1, **i32)
    ext().moe_plan(topi, N, 1, counts, starts, tp, padded, total, pos, row_src)
    return counts, starts, pos


class MoEEPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, mod, ep, B, S):
        dev = h.device
        xb = _bf16(h)
        T, D = xb.shape
        N, K, Nl, E, cap = mod.n_experts, mod.n_active, ep.Nl, ep.E, ep.cap
        softmax = mod.router_type == "softmax"
        f32 = dict(dtype=torch.float32, device=dev)
        logits = torch.empty(T, N, **f32)
        topi = torch.empty(T, K, dtype=torch.int32, device=dev)
        topw = torch.empty(T, K, **f32)
        stats = torch.zeros(2 * B * N + 2, **f32)   # counts | probs | sums, one fill
        seq_counts = stats[:B * N].view(B, N)
        seq_probs = stats[B * N:2 * B * N].view(B, N)
        sums = stats[2 * B * N:]
        ext().router_fwd(xb, mod.router.detach().float().contiguous(),
                         mod.bias.detach().float().contiguous(), S, K, softmax, float(mod.scaling),
                         logits, topi, topw, seq_counts, seq_probs, sums)
        counts, starts, pos = _plan(topi, N)
        recv, ret, drecv, dret = ep.views()
        # dispatch
        ep.barrier()  # owners no longer read recv from the previous use
        ext().ep_scatter(xb, None, None, None, None, topi, pos, starts, ep.recv_peers, ep.me, E, Nl,
                         cap, False)
        ext().ep_zero_pads(counts, ep.recv_peers, ep.cnt_peers, D, ep.me, E, Nl, cap)
        ep.barrier()
        # expert compute on the receive buffer
        wg, wu, wd = _work(mod.expert_w_gate), _work(mod.expert_w_up), _work(mod.expert_w_down)
        F = wg.shape[2]
        Rr = recv.shape[0]
        xr = recv.clone()  # saved for the weight gradients (recv is reused next layer step)
        gu = torch.empty(Rr, 2 * F, dtype=torch.bfloat16, device=dev)
        ext().grouped_gemm_m(xr, wg, gu[:, :F], ep.g_starts, ep.g_counts, ep.tp_f, False)
        ext().grouped_gemm_m(xr, wu, gu[:, F:], ep.g_starts, ep.g_counts, ep.tp_f, False)
        hh = torch.empty(Rr, F, dtype=torch.bfloat16, device=dev)
        ext().swiglu_fwd(gu, hh)
        y = torch.empty(Rr, D, dtype=torch.bfloat16, device=dev)
        ext().grouped_gemm_m(hh, wd, y, ep.g_starts, ep.g_counts, ep.tp_d, False)
        cnt = ep.cnt.clone()
        ext().ep_return(y, cnt, ep.ret_peers, ep.me, E, Nl, cap)
        ep.barrier()
        # shared expert + combine (local)
        sg, su, sd = _work(mod.shared_w_gate), _work(mod.shared_w_up), _work(mod.shared_w_down)
        Fs = sg.shape[1]
        sgu = torch.empty(T, 2 * Fs, dtype=torch.bfloat16, device=dev)
        ext().gemm(xb, sg, sgu[:, :Fs], False, False, False, 1.0)
        ext().gemm(xb, su, sgu[:, Fs:], False, False, False, 1.0)
        shh = torch.empty(T, Fs, dtype=torch.bfloat16, device=dev)
        ext().swiglu_fwd(sgu, shh)
        out = torch.empty(T, D, **f32)
        ext().gemm(shh, sd, out, False, False, False, 1.0)
        ret_saved = ret.clone()
        ext().ep_combine(ret_saved, topw, topi, pos, starts, out, cap)
        z = sums[0] / T
        ent = sums[1] / T
        frac = seq_counts / (S * K)
        bal = (N * (frac * (seq_probs / S)).sum(-1)).mean()
        expert_counts = seq_counts.sum(0)
        ctx.save_for_backward(xb, logits, topi, topw, pos, starts, counts, xr, gu, hh, cnt,
                              ret_saved, sgu, shh, frac)
        ctx.mod, ctx.ep = mod, ep
        ctx.meta = (B, S, T, D, N, K, F, Fs, softmax)
        ctx.mark_non_differentiable(ent, expert_counts)
        return out, z, bal, ent, expert_counts

    @staticmethod
    def backward(ctx, dout, dz, dbal, dent, dcounts):
        (xb, logits, topi, topw, pos, starts, counts, xr, gu, hh, cnt, ret_saved, sgu, shh,
         frac) = ctx.saved_tensors
        mod, ep = ctx.mod, ctx.ep
        B, S, T, D, N, K, F, Fs, softmax = ctx.meta
        E, Nl, cap = ep.E, ep.Nl, ep.cap
        dev = xb.device
        dout = dout.float().contiguous()
        db = dout.to(torch.bfloat16)
        # shared expert
        sg, su, sd = _work(mod.shared_w_gate), _work(mod.shared_w_up), _work(mod.shared_w_down)
        dsh = torch.empty_like(shh)
        ext().gemm(db, sd, dsh, False, True, False, 1.0)
        ext().gemm(shh, db, main_grad(mod.shared_w_down), True, False, True, 1.0)
        dsgu = torch.empty_like(sgu)
        ext().swiglu_bwd(dsh, sgu, dsgu)
        dx = torch.empty(T, D, dtype=torch.float32, device=dev)
        ext().gemm(dsgu[:, :Fs], sg, dx, False, True, False, 1.0)
        ext().gemm(dsgu[:, Fs:], su, dx, False, True, True, 1.0)
        ext().gemm(xb, dsgu[:, :Fs], main_grad(mod.shared_w_gate), True, False, True, 1.0)
        ext().gemm(xb, dsgu[:, Fs:], main_grad(mod.shared_w_up), True, False, True, 1.0)
        # send w * dout to the expert owners; dw from the returned outputs
        recv, ret, drecv, dret = ep.views()
        dtopw = torch.empty(T, K, dtype=torch.float32, device=dev)
        ep.barrier()
        ext().ep_scatter(xb, dout, topw, ret_saved, dtopw, topi, pos, starts, ep.drecv_peers, ep.me,
                         E, Nl, cap, True)
        ext().ep_zero_pads(counts, ep.drecv_peers, None, D, ep.me, E, Nl, cap)
        ep.barrier()
        dy = drecv.clone()
        wg, wu, wd = _work(mod.expert_w_gate), _work(mod.expert_w_up), _work(mod.expert_w_down)
        Rr = dy.shape[0]
        dhh = torch.empty(Rr, F, dtype=torch.bfloat16, device=dev)
        ext().grouped_gemm_m(dy, wd, dhh, ep.g_starts, ep.g_counts, ep.tp_f, True)
        ext().grouped_gemm_k(hh, dy, main_grad(mod.expert_w_down), ep.g_starts, ep.g_counts, True)
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dhh, gu, dgu)
        dxr = torch.empty(Rr, D, dtype=torch.float32, device=dev)
        ext().grouped_gemm_m(dgu[:, :F], wg, dxr, ep.g_starts, ep.g_counts, ep.tp_d, True, False)
        ext().grouped_gemm_m(dgu[:, F:], wu, dxr, ep.g_starts, ep.g_counts, ep.tp_d, True, True)
        ext().grouped_gemm_k(xr, dgu[:, :F], main_grad(mod.expert_w_gate), ep.g_starts, ep.g_counts, True)
        ext().grouped_gemm_k(xr, dgu[:, F:], main_grad(mod.expert_w_up), ep.g_starts, ep.g_counts, True)
        ext().ep_return(dxr.to(torch.bfloat16), cnt, ep.dret_peers, ep.me, E, Nl, cap)
        ep.barrier()
        ext().ep_combine(dret, None, topi, pos, starts, dx, cap)
        # router
        dz = torch.zeros((), device=dev) if dz is None else dz
        dbal = torch.zeros((), device=dev) if dbal is None else dbal
        coef_z = (dz.float() * 2.0 / T).reshape(1).contiguous()
        bal_coef = (dbal.float() * N / (B * S) * frac).contiguous()
        dlogits = torch.empty(T, N, dtype=torch.float32, device=dev)
        ext().router_bwd(logits, topi, dtopw, bal_coef, S, softmax, float(mod.scaling), coef_z, dlogits)
        ext().router_grads(xb, mod.router.detach().float().contiguous(), dlogits, dx,
                           main_grad(mod.router))
        return dx.to(torch.bfloat16), None, None, None, None


_SHARED_CTX: dict = {}


def shared_ep_context(layer, T: int, D: int, F: int, ctx, capacity_factor: float) -> EPContext:
    """One set of symmetric dispatch / return buffers per layer shape, shared by
    every MoE layer: each use is fenced by device barriers and everything the
    backward needs is copied out of the buffers, so layers never hold them."""
    key = (T, D, F, layer.n_experts, layer.n_active, float(capacity_factor), ctx.world, ctx.rank,
           torch.cuda.current_device())
    ep = _SHARED_CTX.get(key)
    if ep is None:
        ep = EPContext(layer, T, D, F, ctx, capacity_factor)
        _SHARED_CTX[key] = ep
    return ep


def release_shared_contexts():
    """Drop the shared buffers (before the process group is destroyed)."""
    _SHARED_CTX.clear()


def moe_ep_layer_cuda(mod, h, dtype):
    B, S, D = h.shape
    ep = mod.ep_ctx
    out, z, bal, ent, counts = MoEEPFn.apply(h.reshape(B * S, D), mod, ep, B, S)
    return out.view(B, S, D), {"router_z_loss": z, "balance_loss": bal, "mean_entropy": ent,
                               "expert_counts": counts}
