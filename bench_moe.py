"""MoE dispatch microbenchmark (the reference's bench_dispatch.py; BASELINE
config 5): one MoE layer, forward and forward+backward, per GPU

    8192 tokens x d_model 2048 (bf16, N(0,1)), router logits over 64 experts,
    top-8, SwiGLU hidden 1408, capacity factor 1.25

    python bench_moe.py                                   # 1 GPU: local dropless path
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29512 bench_moe.py --ep 8           # expert parallel

Arms (EP > 1):
  fused   peer-memory dispatch/return kernels + tcgen05 grouped GEMMs (this repo)
  nccl    all_to_all_single on packed buffers + the same grouped GEMMs (baseline)
The roofline is the slower of the layer's GEMM FLOPs at the measured bf16 peak
and the bytes that must cross NVLink at 770 GB/s per direction; times are CUDA
events after warm-up, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch
import torch.distributed as dist


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ep", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--d", type=int, default=2048)
    ap.add_argument("--f", type=int, default=1408)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--cf", type=float, default=1.25)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    return ap.parse_args()


def time_it(fn, iters, warmup, ctx):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if ctx:
        ctx.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    return ctx.max_scalar(ms) if ctx else ms


def main():
    args = parse()
    from hanuman_b200.flops import peak_flops_per_device
    from hanuman_b200.models.layers import MoE
    from hanuman_b200.parallel.mesh import init_distributed
    ctx = init_distributed(timeout_s=300)
    world = ctx.world if ctx else 1
    rank = ctx.rank if ctx else 0
    local = ctx.local_rank if ctx else 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    assert args.ep == world, "--ep must equal the number of ranks"
    T, D, F, N, K = args.tokens, args.d, args.f, args.experts, args.topk
    gen = torch.Generator().manual_seed(0)
    mod = MoE(D, F, N, K, 1, 1.0, 2.5, gen, d_ff_shared=F)
    if world > 1:
        mod.make_expert_parallel(rank, world)
        mod.ep_dist = ctx
        mod.capacity_factor = args.cf
    mod = mod.to(dev)
    for p in mod.parameters():
        if p.dim() >= 2 and p is not mod.router:
            p.data = p.data.bfloat16()
    h = torch.randn(1, T, D, generator=torch.Generator().manual_seed(1 + rank)).to(dev).bfloat16()
    hg = h.clone().requires_grad_()

    def fwd():
        with torch.no_grad():
            mod(h, torch.bfloat16)

    def fwd_bwd():
        out, aux = mod(hg, torch.bfloat16)
        (out.sum() * 1e-6 + aux["balance_loss"] + aux["router_z_loss"]).backward()

    res = {"T": T, "D": D, "F": F, "N": N, "K": K, "ep": world, "cf": args.cf}
    res["fused_fwd_ms"] = time_it(fwd, args.iters, args.warmup, ctx)
    res["fused_fwd_bwd_ms"] = time_it(fwd_bwd, args.iters, args.warmup, ctx)
    # roofline (routed experts + shared expert GEMMs; NVLink bytes of dispatch + return)
    flop_fwd = 2 * 3 * T * K * D * F + 2 * 3 * T * D * F
    bytes_link = 2 * T * K * (world - 1) / world * D * 2 if world > 1 else 0
    peak = peak_flops_per_device()
    t_roof = max(flop_fwd / peak, bytes_link / 770e9) * 1e3
    res["roofline_fwd_ms"] = t_roof
    res["fused_fwd_frac_of_roofline"] = t_roof / res["fused_fwd_ms"]
    res["fwd_tflops"] = flop_fwd / (res["fused_fwd_ms"] / 1e3) / 1e12
    if world > 1:
        res["nccl_fwd_ms"] = time_it(lambda: nccl_baseline_fwd(mod, h, ctx), args.iters,
                                     args.warmup, ctx)
        res["fused_speedup_vs_nccl"] = res["nccl_fwd_ms"] / res["fused_fwd_ms"]
    if rank == 0:
        print(json.dumps(res))
    if ctx:
        ctx.barrier()
        ctx.shutdown()


@torch.no_grad()
def nccl_baseline_fwd(mod, h, ctx):
    """Baseline EP forward: packed all_to_all_single in both directions around the
    same grouped GEMMs (the capacity layout and routing of the fused path)."""
    from hanuman_b200.ops._ext import ext
    from hanuman_b200.ops.dense import _work
    from hanuman_b200.ops.moe_ep import _plan
    ep = mod.ep_ctx
    E, Nl, cap, N, K = ep.E, ep.Nl, ep.cap, ep.N, ep.K
    xb = h.reshape(-1, h.shape[-1]).contiguous()
    T, D = xb.shape
    dev = xb.device
    logits = torch.empty(T, N, device=dev)
    topi = torch.empty(T, K, dtype=torch.int32, device=dev)
    topw = torch.empty(T, K, device=dev)
    sc = torch.zeros(1, N, device=dev)
    sp = torch.zeros(1, N, device=dev)
    sums = torch.zeros(2, device=dev)
    ext().router_fwd(xb, mod.router.float().contiguous(), mod.bias.float().contiguous(), T, K,
                     False, 2.5, logits, topi, topw, sc, sp, sums)
    counts, starts, pos = _plan(topi, N)
    # pack: send[dest][le][i]  (row index e * cap + i), dropped slots skipped
    e = topi.long()
    i = (pos - starts[e.clamp_min(0)].to(pos.dtype)).long()
    keep = i < cap
    send = torch.zeros(N * cap, D, dtype=torch.bfloat16, device=dev)
    tok = torch.arange(T, device=dev)[:, None].expand(T, K)
    send.index_copy_(0, (e * cap + i)[keep], xb[tok[keep]])
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)          # recv[src][le][i]
    xr = recv.view(E, Nl, cap, D).transpose(0, 1).contiguous().view(-1, D)
    wg, wu, wd = _work(mod.expert_w_gate), _work(mod.expert_w_up), _work(mod.expert_w_down)
    F = wg.shape[2]
    gu = torch.empty(xr.shape[0], 2 * F, dtype=torch.bfloat16, device=dev)
    ext().grouped_gemm_m(xr, wg, gu[:, :F], ep.g_starts, ep.g_counts, ep.tp_f, False)
    ext().grouped_gemm_m(xr, wu, gu[:, F:], ep.g_starts, ep.g_counts, ep.tp_f, False)
    hh = torch.empty(xr.shape[0], F, dtype=torch.bfloat16, device=dev)
    ext().swiglu_fwd(gu, hh)
    y = torch.empty(xr.shape[0], D, dtype=torch.bfloat16, device=dev)
    ext().grouped_gemm_m(hh, wd, y, ep.g_starts, ep.g_counts, ep.tp_d, False)
    back = y.view(Nl, E, cap, D).transpose(0, 1).contiguous().view(-1, D)
    ret = torch.empty_like(back)
    dist.all_to_all_single(ret, back)           # ret[e][i]
    out = torch.zeros(T, D, device=dev)
    ext().ep_combine(ret, topw, topi, pos, starts, out, cap)
    return out


if __name__ == "__main__":
    main()
