"""Small, self-contained kernel cases for device profiling (ncu) and timing.

    python -m hanuman_b200.profile_cases <case> [--time]

Each case builds inputs on the current GPU (a few GB at most; operands larger
than the 126 MB L2 where the kernel is memory-bound), runs the kernel a few
times and exits.  With ``--time`` it prints the CUDA-event time of one launch
and the achieved TFLOP/s or GB/s.  Cases: gemm_fwd, gemm_dw, grouped_fwd,
grouped_swiglu_fwd, grouped_swiglu_bwd, grouped_cat2, gather_gemm_emulated, kda_layer, kda_fwd, kda_bwd, kda128_fwd, kda128_bwd, flash_fwd, flash_bwd, router_fwd, p2p_rs_emulated,
ep_dispatch_emulated, flash128_fwd, flash128_bwd.
"""
from __future__ import annotations

import math
import sys

import torch

from .ops._ext import ext


def _time(fn, n=5):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def case_gemm_fwd():
    x = torch.randn(32768, 1024, device="cuda").bfloat16()
    w = torch.randn(1024, 3200, device="cuda").bfloat16()
    y = torch.empty(32768, 3200, device="cuda", dtype=torch.bfloat16)
    return (lambda: ext().gemm(x, w, y, False, False, False, 1.0)), 2 * 32768 * 1024 * 3200, "flop"


def case_gemm_dw():
    x = torch.randn(32768, 1024, device="cuda").bfloat16()
    dy = torch.randn(32768, 1024, device="cuda").bfloat16()
    g = torch.zeros(1024, 1024, device="cuda")
    return (lambda: ext().gemm(x, dy, g, True, False, True, 1.0)), 2 * 32768 * 1024 * 1024, "flop"


def case_grouped_fwd():
    T, K, N, D, F = 32768, 4, 32, 1024, 768
    counts = [T * K // N] * N
    starts = [i * ((T * K // N + 127) // 128 * 128) for i in range(N)]
    R = starts[-1] + counts[-1]
    xp = torch.randn(R, D, device="cuda").bfloat16()
    w = torch.randn(N, D, F, device="cuda").bfloat16()
    y = torch.empty(R, F, device="cuda", dtype=torch.bfloat16)
    tiles_n = (F + 255) // 256
    tp = [0]
    for c in counts:
        tp.append(tp[-1] + (c + 127) // 128 * tiles_n)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    gs, gc, gt = i32(starts), i32(counts), i32(tp)
    return (lambda: ext().grouped_gemm_m(xp, w, y, gs, gc, gt, False)), 2 * T * K * D * F, "flop"


def _expert_plan(tiles_n, T=32768, K=4, N=32):
    """Balanced expert segments of the flagship MoE (T tokens x top-K over N
    experts, 128-row aligned) and the grouped GEMM tile prefix."""
    counts = [T * K // N] * N
    starts = [i * ((T * K // N + 127) // 128 * 128) for i in range(N)]
    R = starts[-1] + counts[-1]
    tp = [0]
    for c in counts:
        tp.append(tp[-1] + (c + 127) // 128 * tiles_n)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    return R, i32(starts), i32(counts), i32(tp)


def case_grouped_swiglu_fwd():
    """Expert gate + up GEMMs with the SwiGLU in the epilogue (one launch)."""
    T, K, N, D, F = 32768, 4, 32, 1024, 768
    R, gs, gc, gt = _expert_plan(2 * F // 256)
    xp = torch.randn(R, D, device="cuda").bfloat16()
    wg = (torch.randn(N, D, F, device="cuda") * 0.03).bfloat16()
    wu = (torch.randn(N, D, F, device="cuda") * 0.03).bfloat16()
    h = torch.empty(R, F, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(R, 2 * F, device="cuda", dtype=torch.bfloat16)
    return (lambda: ext().grouped_gemm_m_swiglu_fwd(xp, wg, wu, h, gu, gs, gc, gt)), \
        2 * 2 * T * K * D * F, "flop"


def case_grouped_swiglu_bwd():
    """dh = dY W_down^T with the SwiGLU backward in the epilogue (one launch)."""
    T, K, N, D, F = 32768, 4, 32, 1024, 768
    R, gs, gc, gt = _expert_plan((F + 255) // 256)
    dy = torch.randn(R, D, device="cuda").bfloat16()
    wd = (torch.randn(N, F, D, device="cuda") * 0.03).bfloat16()
    gu = torch.randn(R, 2 * F, device="cuda").bfloat16()
    dgu = torch.empty(R, 2 * F, device="cuda", dtype=torch.bfloat16)
    return (lambda: ext().grouped_gemm_m_swiglu_bwd(dy, wd, gu, dgu, gs, gc, gt)), \
        2 * T * K * D * F, "flop"


def case_grouped_cat2():
    """Expert input gradient [dg | du] @ [W_gate | W_up]^T in one launch (K = 2F)."""
    T, K, N, D, F = 32768, 4, 32, 1024, 768
    R, gs, gc, gt = _expert_plan((D + 255) // 256)
    dgu = torch.randn(R, 2 * F, device="cuda").bfloat16()
    wg = (torch.randn(N, D, F, device="cuda") * 0.03).bfloat16()
    wu = (torch.randn(N, D, F, device="cuda") * 0.03).bfloat16()
    dxp = torch.empty(R, D, device="cuda", dtype=torch.bfloat16)
    return (lambda: ext().grouped_gemm_m_cat2(dgu, wg, wu, dxp, gs, gc, gt)), \
        2 * T * K * 2 * F * D, "flop"


def case_gather_gemm_emulated():
    """Fused expert-weight all-gather + grouped GEMM on one GPU: the 8 "ranks'"
    expert shards are local buffers (the kernel's tile claiming, copy-out and
    waiting, without NVLink).  Flagship MoE shape: 32 experts, D 1024, F 768."""
    T, K, N, D, F, W = 32768, 4, 32, 1024, 768, 8
    counts = [T * K // N] * N
    starts = [i * ((T * K // N + 127) // 128 * 128) for i in range(N)]
    R = starts[-1] + counts[-1]
    xp = torch.randn(R, D, device="cuda").bfloat16()
    w = torch.randn(N, D, F, device="cuda").bfloat16()
    shards = [w[r * (N // W):(r + 1) * (N // W)].clone() for r in range(W)]
    y = torch.empty(R, F, device="cuda", dtype=torch.bfloat16)
    gathered = torch.empty_like(w)
    tiles_n = (F + 255) // 256
    flags = torch.zeros(N * (D // 64) * tiles_n, dtype=torch.int32, device="cuda")
    tp = [0]
    for c in counts:
        tp.append(tp[-1] + (c + 127) // 128 * tiles_n)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    gs, gc, gt = i32(starts), i32(counts), i32(tp)
    ptrs = [s.data_ptr() for s in shards]
    return (lambda: ext().grouped_gemm_m_gather(xp, ptrs, 0, N // W, gathered, flags, y, gs, gc, gt)), \
        2 * T * K * D * F, "flop"


def _kda_inputs(B=8, S=4096, H=16, K=64):
    g = torch.Generator(device="cuda").manual_seed(0)
    n = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    q = n(torch.randn(B, S, H, K, device="cuda", generator=g))
    k = n(torch.randn(B, S, H, K, device="cuda", generator=g))
    v = torch.randn(B, S, H, K, device="cuda", generator=g)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, S, H, K, device="cuda", generator=g))
    beta = torch.sigmoid(torch.randn(B, S, H, device="cuda", generator=g))
    return q, k, v, gg, beta


def case_kda_fwd():
    from .ops.kda import KdaCoreFn
    ins = _kda_inputs()
    B, S, H, K = ins[0].shape
    flops = 8 * H * K * K * B * S   # reference FLOP model of the recurrence
    return (lambda: KdaCoreFn.apply(*ins, 1 / math.sqrt(K))), flops, "flop"


def case_kda_bwd():
    from .ops.kda import KdaCoreFn
    ins = [t.requires_grad_() for t in _kda_inputs()]
    B, S, H, K = ins[0].shape
    def run():
        o = KdaCoreFn.apply(*ins, 1 / math.sqrt(K))
        o.backward(torch.ones_like(o))
    return run, 3 * 8 * H * K * K * B * S, "flop"


def case_kda_layer():
    """Whole KDA layer (projections, conv/gate front-end, chunked core, output
    gate, wo) forward + backward at the flagship shape: 8 x 4096 tokens, d 1024,
    16 heads of 64."""
    from .models.layers import KDA
    m = KDA(1024, 16, 64, torch.Generator().manual_seed(0)).cuda()
    h = torch.randn(8, 4096, 1024, device="cuda").bfloat16().requires_grad_()
    def run():
        y = m(h, torch.bfloat16)
        y.backward(torch.ones_like(y))
    return run, 3 * 2 * 8 * 4096 * (1024 * 16 * 64 * 4 + 8 * 16 * 64 * 64), "flop"


def case_kda128_fwd():
    """KDA-layer microbench shape: 16 heads of head dim 128, 2 x 32768 tokens."""
    from .ops.kda import KdaCoreFn
    ins = _kda_inputs(B=2, S=32768, H=16, K=128)
    B, S, H, K = ins[0].shape
    return (lambda: KdaCoreFn.apply(*ins, 1 / math.sqrt(K))), 8 * H * K * K * B * S, "flop"


def case_kda128_bwd():
    from .ops.kda import KdaCoreFn
    ins = [t.requires_grad_() for t in _kda_inputs(B=2, S=32768, H=16, K=128)]
    B, S, H, K = ins[0].shape
    def run():
        o = KdaCoreFn.apply(*ins, 1 / math.sqrt(K))
        o.backward(torch.ones_like(o))
    return run, 3 * 8 * H * K * K * B * S, "flop"


def _attn_inputs(B=8, S=4096, Nq=16, Nkv=4, H=64):
    q = torch.randn(B, S, Nq, H, device="cuda").bfloat16()
    k = torch.randn(B, S, Nkv, H, device="cuda").bfloat16()
    v = torch.randn(B, S, Nkv, H, device="cuda").bfloat16()
    return q, k, v


def case_flash_fwd():
    q, k, v = _attn_inputs()
    B, S, Nq, H = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Nq, S, device="cuda")
    return (lambda: ext().flash_fwd(q, k, v, out, lse, 0)), 4 * B * Nq * H * S * (S + 1) / 2, "flop"


def case_flash_bwd():
    q, k, v = _attn_inputs()
    B, S, Nq, H = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Nq, S, device="cuda")
    ext().flash_fwd(q, k, v, out, lse, 0)
    do = torch.randn_like(q)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B, Nq, S, device="cuda")
    return (lambda: ext().flash_bwd(q, k, v, out, do, lse, delta, dq, dk, dv, 0)), \
        2.5 * 4 * B * Nq * H * S * (S + 1) / 2, "flop"


def case_flash128_fwd():
    """Head dim 128 (16 query heads, 4 KV heads, 4 x 4096 tokens)."""
    q, k, v = _attn_inputs(B=4, H=128)
    B, S, Nq, H = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Nq, S, device="cuda")
    return (lambda: ext().flash_fwd(q, k, v, out, lse, 0)), 4 * B * Nq * H * S * (S + 1) / 2, "flop"


def case_flash128_bwd():
    q, k, v = _attn_inputs(B=4, H=128)
    B, S, Nq, H = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Nq, S, device="cuda")
    ext().flash_fwd(q, k, v, out, lse, 0)
    do = torch.randn_like(q)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B, Nq, S, device="cuda")
    return (lambda: ext().flash_bwd(q, k, v, out, do, lse, delta, dq, dk, dv, 0)), \
        2.5 * 4 * B * Nq * H * S * (S + 1) / 2, "flop"


def case_router_fwd():
    T, D, N, K = 32768, 1024, 32, 4
    x = torch.randn(T, D, device="cuda").bfloat16()
    W = torch.randn(D, N, device="cuda") * 0.01
    bias = torch.zeros(N, device="cuda")
    lg = torch.empty(T, N, device="cuda")
    ti = torch.empty(T, K, dtype=torch.int32, device="cuda")
    tw = torch.empty(T, K, device="cuda")
    sc, sp = torch.zeros(8, N, device="cuda"), torch.zeros(8, N, device="cuda")
    su = torch.zeros(2, device="cuda")
    return (lambda: ext().router_fwd(x, W, bias, 4096, K, False, 2.5, lg, ti, tw, sc, sp, su)), \
        T * D * 2 + D * N * 4, "byte"


def case_p2p_rs_emulated():
    """The fused reduce-scatter kernel on one GPU: both 'peers' are local
    buffers (the kernel and its memory traffic without NVLink)."""
    n = 64 * 1024 * 1024
    a = torch.randn(2 * n, device="cuda")
    out = torch.empty(n // 2, device="cuda")
    s = torch.zeros(1, device="cuda")
    peers = torch.tensor([a.data_ptr(), a.data_ptr() + n * 4], dtype=torch.int64, device="cuda")
    return (lambda: ext().p2p_reduce_scatter(peers, 2, 0, n // 2, out, 0.5, s)), \
        3 * (n // 2) * 4, "byte"


def case_ep_dispatch_emulated():
    """Expert-parallel dispatch of one rank on one GPU: the token scatter to the
    experts' owners, the return of the expert rows and the weighted combine, with
    the 8 "ranks'" receive / return buffers as local buffers (the kernels and
    their memory traffic without NVLink).  BASELINE config 5 per GPU: 64
    experts top-8 over 8 ranks, D 2048, capacity factor 1.25; 4096 tokens."""
    T, K, N, E, D = 4096, 8, 64, 8, 2048
    Nl = N // E
    cap = int(math.ceil(T * K / N * 1.25))
    dev = "cuda"
    x = torch.randn(T, D, device=dev).bfloat16()
    topi = torch.rand(T, N, device=dev).topk(K, dim=-1).indices.int().contiguous()
    topw = torch.rand(T, K, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    counts, starts, tp = torch.empty(N, **i32), torch.empty(N, **i32), torch.empty(N + 1, **i32)
    padded, total, pos = torch.empty(N, **i32), torch.empty(1, **i32), torch.empty(T, K, **i32)
    row_src = torch.full((((T * K + N * 127 + 127) // 128) * 128,), -1, **i32)
    ext().moe_plan(topi, N, 1, counts, starts, tp, padded, total, pos, row_src)
    recv = [torch.zeros(Nl * E * cap, D, device=dev, dtype=torch.bfloat16) for _ in range(E)]
    ret = [torch.zeros(N * cap, D, device=dev, dtype=torch.bfloat16) for _ in range(E)]
    recv_peers = torch.tensor([t.data_ptr() for t in recv], dtype=torch.int64, device=dev)
    ret_peers = torch.tensor([t.data_ptr() for t in ret], dtype=torch.int64, device=dev)
    # rank 0's own tokens stand in for every source rank's block
    cnt = torch.clamp(counts[:Nl], max=cap).repeat_interleave(E).int().contiguous()
    out = torch.zeros(T, D, device=dev)

    def run():
        ext().ep_scatter(x, None, None, None, None, topi, pos, starts, recv_peers, 0, E, Nl, cap, False)
        ext().ep_return(recv[0], cnt, ret_peers, 0, E, Nl, cap)
        ext().ep_combine(ret[0], topw, topi, pos, starts, out, cap)
    return run, 3 * T * K * D * 2 + 2 * T * D * 4, "byte"


CASES = {k[5:]: v for k, v in globals().items() if k.startswith("case_")}

# phase slots of the chunk-64 KDA intra kernels (csrc/kda/kda64.cu PhaseClock marks)
KDA64_PHASES = {
    0: "fwd load", 1: "fwd cumsum", 2: "fwd Kh/Qg + off-diagonal A,P", 3: "fwd diagonal pairs",
    4: "fwd store P,A / N", 5: "fwd block inverse", 6: "fwd Linv store, bV, b2Ke^G",
    7: "fwd Ut/Wt products",
    10: "bwd load", 11: "bwd X,Y", 12: "bwd dN", 13: "bwd dbeta,dv", 14: "bwd init accumulators",
    15: "bwd j0 staging", 16: "bwd j0 products", 17: "bwd j0 epilogue",
    18: "bwd j1 staging", 19: "bwd j1 products", 20: "bwd j1 epilogue",
    21: "bwd j2 staging", 22: "bwd j2 products", 23: "bwd j2 epilogue",
    24: "bwd diagonal pairs", 25: "bwd cumsum", 26: "bwd stores"}


def kda64_phases(fn):
    """Run ``fn`` once with the chunk-64 KDA phase counters on; print each
    phase's share of its kernel's summed CTA cycles."""
    import torch
    cnt = torch.zeros(64, dtype=torch.int64, device="cuda")
    ext().kda64_set_profile(cnt)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext().kda64_set_profile(None)
    c = cnt.cpu().tolist()
    for lo, hi, name in ((0, 8, "intra_fwd64"), (10, 27, "intra_bwd64")):
        tot = sum(c[lo:hi])
        if tot == 0:
            continue
        print(f"{name}: {tot / 1e9:.3f} G CTA-cycles")
        for i in range(lo, hi):
            print(f"  {KDA64_PHASES[i]:34s} {100 * c[i] / tot:5.1f} %")


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    name = argv[0]
    fn, work, unit = CASES[name]()
    ms = _time(fn)
    if "--time" in argv:
        rate = work / (ms / 1e3)
        print(f"{name}: {ms:.3f} ms  " + (f"{rate/1e12:.1f} TFLOP/s" if unit == "flop"
                                          else f"{rate/1e9:.0f} GB/s"))
    if "--phases" in argv:
        kda64_phases(fn)
    assert ext().read_status() == 0


if __name__ == "__main__":
    main()
