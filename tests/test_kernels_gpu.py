"""Native kernels against the fp32 PyTorch oracle (ops/reference.py), forward
and backward.  Every test here needs a B200 and the built extension."""
import math

import pytest
import torch
import torch.nn.functional as F

from hanuman_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def test_extension_is_native():
    from hanuman_b200.ops._ext import ext, available
    assert available()
    assert ext().num_sms() > 0


def test_rmsnorm_fwd_bwd():
    from hanuman_b200.ops.norm import rms_norm_cuda
    torch.manual_seed(0)
    x = torch.randn(300, 1024, device=DEV, requires_grad=True)
    w = (1 + 0.1 * torch.randn(1024, device=DEV)).requires_grad_()
    y = rms_norm_cuda(x, w, 1e-6, torch.float32)
    x2, w2 = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    y2 = ref.rms_norm(x2, w2, 1e-6, torch.float32)
    assert rel(y, y2) < 1e-5
    g = torch.randn_like(y)
    (y * g).sum().backward()
    (y2 * g).sum().backward()
    assert rel(x.grad, x2.grad) < 1e-4 and rel(w.grad, w2.grad) < 1e-4


def test_rope_fwd_bwd():
    from hanuman_b200.ops.norm import rope_cuda
    torch.manual_seed(1)
    B, S, N, H = 2, 70, 3, 64
    cos, sin = ref.precompute_rope(H, 128)
    cos, sin = cos.to(DEV, torch.bfloat16), sin.to(DEV, torch.bfloat16)
    q = torch.randn(B, S, N, H, device=DEV).bfloat16().requires_grad_()
    k = torch.randn(B, S, 1, H, device=DEV).bfloat16().requires_grad_()
    q1, k1 = rope_cuda(q.clone(), k.clone(), cos, sin)
    qr, kr = ref.apply_rope(q.float(), k.float(), cos.float(), sin.float())
    assert rel(q1, qr) < 1e-2 and rel(k1, kr) < 1e-2
    qq = q.detach().float().requires_grad_()
    qr2, _ = ref.apply_rope(qq, k.detach().float(), cos.float(), sin.float())
    g = torch.randn_like(qr2)
    (qr2 * g).sum().backward()
    qa = q.detach().clone().requires_grad_()
    qa1, _ = rope_cuda(qa * 1, k.detach().clone(), cos, sin)
    (qa1.float() * g).sum().backward()
    assert rel(qa.grad, qq.grad) < 2e-2


def test_swiglu_fwd_bwd():
    from hanuman_b200.ops.norm import swiglu_cuda
    torch.manual_seed(2)
    gu = torch.randn(257, 2 * 96, device=DEV).bfloat16().requires_grad_()
    h = swiglu_cuda(gu)
    gf = gu.detach().float().requires_grad_()
    hr = F.silu(gf[:, :96]) * gf[:, 96:]
    assert rel(h, hr) < 1e-2
    g = torch.randn_like(hr)
    (h.float() * g).sum().backward()
    (hr * g).sum().backward()
    assert rel(gu.grad, gf.grad) < 2e-2


def test_embedding_fwd_bwd():
    from hanuman_b200.ops.norm import embedding_cuda
    w = torch.randn(100, 256, device=DEV).bfloat16()
    tok = torch.randint(0, 100, (4, 33), device=DEV)
    x = embedding_cuda(tok, w)
    assert torch.equal(x, w.float()[tok])
    w.main_grad = torch.zeros(100, 256, device=DEV)
    xx = embedding_cuda(tok, w.requires_grad_())
    g = torch.randn_like(xx)
    (xx * g).sum().backward()
    exp = torch.zeros(100, 256, device=DEV).index_add_(0, tok.reshape(-1), g.reshape(-1, 256))
    assert rel(w.main_grad, exp) < 1e-5


def test_head_cross_entropy_fwd_bwd():
    from hanuman_b200.ops.ce import head_ce_cuda
    torch.manual_seed(3)
    T, D, V = 9000, 256, 2048  # more than one token chunk
    x = (torch.randn(T, D, device=DEV) * 0.5).bfloat16().requires_grad_()
    w = (torch.randn(V, D, device=DEV) * 0.05).bfloat16()
    w.main_grad = torch.zeros(V, D, device=DEV)
    tgt = torch.randint(0, V, (T,), device=DEV)
    loss = head_ce_cuda(x, w.requires_grad_(), tgt)
    xf = x.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    lr = F.cross_entropy(xf @ wf.t(), tgt)
    assert abs(loss.item() - lr.item()) < 1e-3
    (2.0 * loss).backward()
    (2.0 * lr).backward()
    assert rel(x.grad, xf.grad) < 2e-2
    assert rel(w.main_grad, wf.grad) < 2e-2


def test_head_ce_full_vocab_against_fp32_head_and_memory():
    """The tied head at the flagship shape (D 1024, V 32768) with bf16 operands
    against an fp32 head over the fp32 master weights (the reference's
    ``x @ wte.T``), and no [T, V] buffer: peak extra memory stays under half of
    one bf16 [T, V] array."""
    from hanuman_b200.ops.ce import head_ce_cuda
    torch.manual_seed(21)
    T, D, V = 65536, 1024, 32768
    x = torch.randn(T, D, device=DEV).bfloat16().requires_grad_()
    w32 = torch.randn(V, D, device=DEV) * D ** -0.5
    w = w32.bfloat16()
    w.main_grad = torch.zeros(V, D, device=DEV)
    tgt = torch.randint(0, V, (T,), device=DEV)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    loss = head_ce_cuda(x, w.requires_grad_(), tgt)
    loss.backward()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    assert peak < 0.5 * T * V * 2, peak
    xf = x.detach().float().requires_grad_()
    wf = w32.clone().requires_grad_()
    torch.backends.cuda.matmul.allow_tf32 = False
    lr_ = F.cross_entropy(xf @ wf.t(), tgt)
    lr_.backward()
    assert abs(loss.item() - lr_.item()) / lr_.item() < 1e-4
    assert rel(x.grad, xf.grad) < 1e-2
    assert rel(w.main_grad, wf.grad) < 1e-2


@pytest.mark.parametrize("H,window,S,Nq,Nkv", [(64, 0, 256, 4, 2), (64, 0, 200, 4, 4),
                                               (32, 0, 128, 2, 1), (32, 64, 128, 2, 1),
                                               (64, 96, 300, 4, 1), (128, 0, 192, 2, 2),
                                               (128, 64, 130, 4, 2), (128, 0, 777, 4, 1)])
def test_flash_attention_fwd_bwd(H, window, S, Nq, Nkv):
    from hanuman_b200.ops.flash import flash_attention
    torch.manual_seed(4)
    B = 2
    q = torch.randn(B, S, Nq, H, device=DEV).bfloat16().requires_grad_()
    k = torch.randn(B, S, Nkv, H, device=DEV).bfloat16().requires_grad_()
    v = torch.randn(B, S, Nkv, H, device=DEV).bfloat16().requires_grad_()
    o = flash_attention(q, k, v, window)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = ref.causal_attention(qf, kf, vf, window)
    assert rel(o, orf) < 1e-2
    g = torch.randn_like(orf)
    (o.float() * g).sum().backward()
    (orf * g).sum().backward()
    assert rel(q.grad, qf.grad) < 2e-2
    assert rel(k.grad, kf.grad) < 2e-2
    assert rel(v.grad, vf.grad) < 2e-2


def _kda_inputs(B, S, H, K, gscale, seed=5, dtype=torch.float32):
    g_ = torch.Generator(device="cpu").manual_seed(seed)
    q = ref.l2_norm(torch.randn(B, S, H, K, generator=g_)).to(DEV)
    k = ref.l2_norm(torch.randn(B, S, H, K, generator=g_)).to(DEV)
    v = torch.randn(B, S, H, K, generator=g_).to(DEV)
    g = (F.logsigmoid(torch.randn(B, S, H, K, generator=g_)) * gscale).to(DEV)
    beta = torch.sigmoid(torch.randn(B, S, H, generator=g_)).to(DEV)
    return q, k, v, g, beta


@pytest.mark.parametrize("K,S,gscale", [(64, 100, 1.0), (64, 64, 20.0), (32, 77, 1.0), (16, 40, 5.0),
                                         (128, 70, 1.0), (128, 96, 8.0)])
def test_kda_core_fwd_bwd(K, S, gscale):
    from hanuman_b200.ops.kda import kda_chunked_cuda
    B, H = 2, 3
    ins = _kda_inputs(B, S, H, K, gscale)
    scale = 1.0 / math.sqrt(K)
    xs = [t.clone().requires_grad_() for t in ins]
    o = kda_chunked_cuda(*xs, scale)
    xr = [t.double().clone().requires_grad_() for t in ins]
    orf, _ = ref.kda_chunked(*xr, scale=scale, chunk=16)
    assert rel(o, orf) < 1e-4
    gout = torch.randn_like(orf)
    (o.double() * gout).sum().backward()
    (orf * gout).sum().backward()
    for a, b, name in zip(xs, xr, "q k v g beta".split()):
        assert rel(a.grad, b.grad) < 1e-3, name


def test_kda_layer_matches_cpu_reference():
    """Full KDA layer on the GPU (bf16 projections) vs the CPU path (fp32)."""
    from hanuman_b200.models.layers import KDA
    torch.manual_seed(6)
    gen = torch.Generator().manual_seed(0)
    for gate in ("kimi", "sigmoid"):
        m = KDA(128, 2, 64, gen, gate=gate)
        h = torch.randn(2, 70, 128).bfloat16()
        ycpu = m(h, torch.bfloat16)
        mg = KDA(128, 2, 64, torch.Generator().manual_seed(0), gate=gate)
        mg.load_state_dict(m.state_dict())
        mg = mg.to(DEV)
        ygpu = mg(h.to(DEV), torch.bfloat16)
        assert rel(ygpu.cpu(), ycpu) < 3e-2, gate


def test_kda_layer_grads_match_cpu():
    from hanuman_b200.models.layers import KDA
    torch.manual_seed(7)
    m = KDA(128, 2, 32, torch.Generator().manual_seed(1))
    h = torch.randn(2, 50, 128)
    hc = h.clone().requires_grad_()
    y = m(hc, torch.float32)
    g = torch.randn_like(y)
    (y * g).sum().backward()
    mg = KDA(128, 2, 32, torch.Generator().manual_seed(1)).to(DEV)
    hg = h.to(DEV).bfloat16().requires_grad_()
    yg = mg(hg, torch.bfloat16)
    (yg * g.to(DEV)).sum().backward()
    assert rel(hg.grad.cpu(), hc.grad) < 5e-2
    # small (fp32) parameters receive autograd grads; matrices accumulate main_grad
    for name in ("a_log", "dt_bias", "o_norm", "g_proj1_bias"):
        assert rel(getattr(mg, name).grad.cpu(), getattr(m, name).grad) < 5e-2, name
    for conv in ("q_conv", "k_conv", "v_conv"):
        assert rel(getattr(mg, conv).weight.grad.cpu(), getattr(m, conv).weight.grad) < 5e-2, conv
    for name in ("wq", "wk", "wv", "wo", "f_proj0", "f_proj1", "g_proj0", "g_proj1", "wb"):
        assert rel(getattr(mg, name).main_grad.cpu(), getattr(m, name).grad) < 5e-2, name


@pytest.mark.parametrize("S", [96, 128])   # 128: whole-tile shared expert (fused kernels)
@pytest.mark.parametrize("router_type", ["sigmoid_bias", "softmax"])
def test_moe_layer_fwd_bwd(router_type, S):
    from hanuman_b200.models.layers import MoE
    torch.manual_seed(8)
    D, Fh, N, K = 256, 128, 8, 2
    m = MoE(D, Fh, N, K, 1, 0.5, 2.5, torch.Generator().manual_seed(2), router_type=router_type)
    with torch.no_grad():
        m.bias.copy_(torch.randn(N) * 0.1)
    B = 2
    h = torch.randn(B, S, D).bfloat16()
    hc = h.float().requires_grad_()
    yc, auxc = m(hc, torch.float32)
    mg = MoE(D, Fh, N, K, 1, 0.5, 2.5, torch.Generator().manual_seed(2), router_type=router_type)
    mg.load_state_dict(m.state_dict())
    mg = mg.to(DEV)
    hg = h.to(DEV).requires_grad_()
    yg, auxg = mg(hg, torch.bfloat16)
    assert rel(yg.cpu(), yc) < 3e-2
    assert torch.equal(auxg["expert_counts"].cpu(), auxc["expert_counts"])
    for k_ in ("router_z_loss", "balance_loss", "mean_entropy"):
        assert abs(auxg[k_].item() - auxc[k_].item()) < 1e-3 * max(1, abs(auxc[k_].item())), k_
    g = torch.randn_like(yc)
    loss_c = (yc * g).sum() + 3.0 * auxc["router_z_loss"] + 5.0 * auxc["balance_loss"]
    loss_g = (yg * g.to(DEV)).sum() + 3.0 * auxg["router_z_loss"] + 5.0 * auxg["balance_loss"]
    loss_c.backward()
    loss_g.backward()
    assert rel(hg.grad.cpu(), hc.grad) < 5e-2
    for name in ("expert_w_gate", "expert_w_up", "expert_w_down", "shared_w_gate",
                 "shared_w_up", "shared_w_down", "router"):
        assert rel(getattr(mg, name).main_grad.cpu(), getattr(m, name).grad) < 5e-2, name


@pytest.mark.parametrize("opt", ["adamw", "lion"])
def test_fused_optimizer_matches_reference(opt):
    from hanuman_b200 import optimizer as optim
    from hanuman_b200.config import get_config
    from hanuman_b200.engine import FlatGroup
    from hanuman_b200.ops.optim import fused_update_cuda
    cfg = get_config("smoke").replace(optimizer=opt, weight_decay=0.1)
    n = 10000
    torch.manual_seed(9)
    p = torch.randn(n, device=DEV)
    gr = torch.randn(n, device=DEV)
    decay = (torch.rand(n, device=DEV) > 0.5).float()
    mdt = torch.bfloat16 if opt == "lion" else torch.float32
    g = FlatGroup([], [], [], n, torch.bfloat16)
    g.master, g.grad, g.decay = p.clone(), gr.clone(), decay
    g.m = torch.zeros(n, device=DEV, dtype=mdt)
    g.v = torch.zeros(n, device=DEV) if opt == "adamw" else None
    g.work = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    g.lo, g.hi = 0, n
    coef = torch.tensor(0.5, device=DEV)
    pr, mr = p.clone(), torch.zeros(n, device=DEV, dtype=mdt)
    vr = torch.zeros(n, device=DEV)
    for step in (1, 2):
        fused_update_cuda(g, cfg, 1e-3, step, coef)
        if opt == "lion":
            optim.lion_update_(pr, gr, mr, decay, 1e-3, 0.1, cfg.lion_b1, cfg.lion_b2, 0.5)
        else:
            optim.adamw_update_(pr, gr, mr, vr, decay, 1e-3, 0.1, cfg.adam_b1, cfg.adam_b2,
                                cfg.adam_eps, step, 0.5)
    assert (g.master - pr).abs().max() < 1e-5
    assert torch.equal(g.work, g.master.bfloat16())


def test_gemm_device_alpha_and_strided_slices():
    from hanuman_b200.ops._ext import ext
    torch.manual_seed(10)
    a = torch.randn(256, 192, device=DEV).bfloat16()
    big = torch.randn(192, 512, device=DEV).bfloat16()
    b = big[:, 128:384]  # column slice, row stride 512
    c = torch.zeros(256, 1024, device=DEV)
    cs = c[:, 256:512]
    alpha = torch.tensor([0.25], device=DEV)
    ext().gemm(a, b, cs, False, False, True, 1.0, alpha)
    assert rel(cs, 0.25 * (a.float() @ b.float())) < 1e-5
    assert c[:, :256].abs().max() == 0 and c[:, 512:].abs().max() == 0


def test_no_kernel_reported_errors():
    from hanuman_b200.ops._ext import ext
    torch.cuda.synchronize()
    assert ext().read_status() == 0


@pytest.mark.parametrize("N", [32, 12])
def test_router_logits_and_grads_match_fp32(N):
    """N=32 runs the split-bf16 tensor-core GEMM route, N=12 the SIMT route."""
    from hanuman_b200.ops._ext import ext
    torch.manual_seed(11)
    T, D, S, K = 1024, 512, 256, 4
    x = torch.randn(T, D, device=DEV).bfloat16()
    W = torch.randn(D, N, device=DEV) * 0.02
    bias = torch.zeros(N, device=DEV)
    lg = torch.empty(T, N, device=DEV)
    ti = torch.empty(T, K, dtype=torch.int32, device=DEV)
    tw = torch.empty(T, K, device=DEV)
    sc, sp = torch.zeros(T // S, N, device=DEV), torch.zeros(T // S, N, device=DEV)
    su = torch.zeros(2, device=DEV)
    ext().router_fwd(x, W, bias, S, K, False, 2.5, lg, ti, tw, sc, sp, su)
    ref_lg = x.double() @ W.double()
    assert (lg.double() - ref_lg).abs().max().item() < 1e-5
    want = torch.topk(torch.sigmoid(ref_lg), K, dim=-1).indices
    assert torch.equal(ti.long().sort(-1)[0], want.sort(-1)[0])
    assert torch.equal(sc.sum(0), torch.bincount(ti.flatten().long(), minlength=N).float())
    dl = torch.randn(T, N, device=DEV)
    dx = torch.randn(T, D, device=DEV)
    dx0 = dx.clone()
    dW = torch.zeros(D, N, device=DEV)
    ext().router_grads(x, W, dl, dx, dW)
    assert rel(dx - dx0, dl @ W.t()) < 1e-4
    assert rel(dW, x.float().t() @ dl) < 1e-4


@pytest.mark.parametrize("N", [32, 12])
def test_router_ids_stay_in_range_on_nan_logits(N):
    """NaN activations (a diverged step) must not produce out-of-range expert
    ids: those index shared memory and the dispatch.  Every token gets K
    distinct ids in [0, N), NaN rows included."""
    from hanuman_b200.ops._ext import ext
    torch.manual_seed(13)
    T, D, S, K = 512, 256, 128, 4
    x = torch.randn(T, D, device=DEV).bfloat16()
    x[::3] = float("nan")
    W = torch.randn(D, N, device=DEV) * 0.02
    bias = torch.zeros(N, device=DEV)
    lg = torch.empty(T, N, device=DEV)
    ti = torch.full((T, K), -7, dtype=torch.int32, device=DEV)
    tw = torch.empty(T, K, device=DEV)
    sc, sp = torch.zeros(T // S, N, device=DEV), torch.zeros(T // S, N, device=DEV)
    su = torch.zeros(2, device=DEV)
    ext().router_fwd(x, W, bias, S, K, False, 2.5, lg, ti, tw, sc, sp, su)
    torch.cuda.synchronize()
    tl = ti.long()
    assert tl.min().item() >= 0 and tl.max().item() < N
    assert (tl.sort(-1)[0].diff(dim=-1) > 0).all()
    assert sc.sum().item() == T * K
    clean = torch.ones(T, dtype=torch.bool, device=DEV)
    clean[::3] = False
    want = torch.topk(torch.sigmoid(x[clean].double() @ W.double()), K, dim=-1).indices
    assert torch.equal(tl[clean].sort(-1)[0], want.sort(-1)[0])


@pytest.mark.parametrize("T,K,N", [(32768, 4, 32), (1000, 8, 64), (37, 2, 5)])
def test_moe_plan_is_a_stable_counting_sort(T, K, N):
    """Slots grouped by expert in slot order, each expert's segment starting
    at a multiple of 128; the same rows as a CPU stable sort."""
    from hanuman_b200.ops._ext import ext
    g = torch.Generator().manual_seed(T)
    topi_c = torch.randint(0, N, (T, K), generator=g, dtype=torch.int32)
    topi = topi_c.to(DEV)
    counts = torch.zeros(N, dtype=torch.int32, device=DEV)
    starts = torch.empty(N, dtype=torch.int32, device=DEV)
    tp = torch.empty(N + 1, dtype=torch.int32, device=DEV)
    padded = torch.empty(N, dtype=torch.int32, device=DEV)
    total = torch.empty(1, dtype=torch.int32, device=DEV)
    rmax = T * K + 128 * N
    pos = torch.full((T * K,), -1, dtype=torch.int32, device=DEV)
    row_src = torch.full((rmax,), -1, dtype=torch.int32, device=DEV)
    ext().moe_plan(topi, N, 1, counts, starts, tp, padded, total, pos, row_src)
    torch.cuda.synchronize()
    flat = topi_c.flatten().long()
    cnt = torch.bincount(flat, minlength=N)
    assert torch.equal(counts.cpu().long(), cnt)
    pc = (cnt + 127) // 128 * 128
    st = torch.cumsum(pc, 0) - pc
    assert torch.equal(starts.cpu().long(), st)
    want_pos = torch.empty(T * K, dtype=torch.long)
    for e in range(N):
        idx = (flat == e).nonzero().flatten()          # slot order
        want_pos[idx] = st[e] + torch.arange(idx.numel())
    assert torch.equal(pos.cpu().long(), want_pos)
    rs = row_src.cpu().long()
    assert torch.equal(rs[want_pos], torch.arange(T * K))
    assert ext().read_status() == 0


@pytest.mark.parametrize("K,cap", [(4, 40), (8, 1000), (12, 30)])
def test_ep_combine_matches_torch(K, cap):
    """Expert-parallel combine: out[t] += sum over kept slots of bf16(w) *
    ret[e * cap + rank]; slots ranked at or past the capacity are dropped."""
    from hanuman_b200.ops._ext import ext
    torch.manual_seed(K)
    T, N, D = 300, 16, 256
    i32 = dict(dtype=torch.int32, device=DEV)
    topi = torch.rand(T, N, device=DEV).topk(K, dim=-1).indices.int().contiguous()
    counts, starts, tp = torch.empty(N, **i32), torch.empty(N, **i32), torch.empty(N + 1, **i32)
    padded, total, pos = torch.empty(N, **i32), torch.empty(1, **i32), torch.empty(T, K, **i32)
    row_src = torch.full((T * K + 128 * N,), -1, **i32)
    ext().moe_plan(topi, N, 1, counts, starts, tp, padded, total, pos, row_src)
    ret = torch.randn(N * cap, D, device=DEV).bfloat16()
    w = torch.rand(T, K, device=DEV)
    out = torch.randn(T, D, device=DEV)
    want = out.clone().double()
    rank = (pos - starts[topi.long()]).long()
    kept = rank < cap
    wb = w.bfloat16().double()
    for k in range(K):
        rows = (topi[:, k].long() * cap + rank[:, k].clamp(max=cap - 1))
        want += torch.where(kept[:, k:k + 1], wb[:, k:k + 1] * ret[rows].double(), 0.0)
    ext().ep_combine(ret, w, topi, pos, starts, out, cap)
    torch.cuda.synchronize()
    assert (out.double() - want).abs().max().item() < 1e-4
    assert ext().read_status() == 0


def test_out_of_range_indices_are_skipped_and_reported():
    """A label outside the vocabulary and a MoE row position outside the row
    buffer are skipped (no read or write outside the tensors) and recorded as
    kErrBounds (5) in the device status word; the in-range entries are
    computed as usual."""
    from hanuman_b200.ops._ext import ext
    e = ext()
    e.clear_status()
    torch.manual_seed(21)
    T, V = 6, 64
    logits = torch.randn(T, V, device=DEV)
    tgt = torch.tensor([3, V, 10, -1, 63, 0], dtype=torch.int64, device=DEV)
    loss = torch.zeros(1, device=DEV)
    dl = torch.full((T, V), 7.0, device=DEV).bfloat16()
    e.ce_fwd_bwd(logits, tgt, None, loss, dl, 1.0)
    torch.cuda.synchronize()
    assert e.read_status() == 5
    ok = torch.tensor([1, 0, 1, 0, 1, 1], dtype=torch.bool, device=DEV)
    lse = torch.logsumexp(logits, -1)
    want = (lse - logits.gather(1, tgt.clamp(0, V - 1)[:, None])[:, 0])[ok].sum()
    assert abs(loss.item() - want.item()) < 1e-4 * abs(want.item()) + 1e-4
    assert (dl[~ok].float() == 0).all()
    e.clear_status()
    R, D, K = 16, 8, 2
    dxp = torch.randn(R, D, device=DEV)
    pos = torch.tensor([[0, 5], [R, 3], [7, 15]], dtype=torch.int32, device=DEV)
    dx = torch.zeros(3, D, device=DEV)
    e.moe_scatter_add(dxp, pos, dx)
    torch.cuda.synchronize()
    assert e.read_status() == 5
    want = torch.stack([dxp[0] + dxp[5], dxp[3], dxp[7] + dxp[15]])
    assert torch.allclose(dx, want, atol=1e-6)
    e.clear_status()
    assert e.read_status() == 0


def test_add_norm_fwd_bwd():
    from hanuman_b200.ops.norm import add_rms_norm_cuda
    torch.manual_seed(12)
    B, S, D = 2, 100, 1024
    x = torch.randn(B, S, D, device=DEV, requires_grad=True)
    a = torch.randn(B, S, D, device=DEV, requires_grad=True)
    rs = torch.tensor(0.7, device=DEV, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_()
    xn, h = add_rms_norm_cuda(x, a, rs, w, 1e-6)
    xr = [t.detach().clone().requires_grad_() for t in (x, a, rs, w)]
    xnr = xr[0] + xr[2] * xr[1]
    hr = xnr * torch.rsqrt((xnr * xnr).mean(-1, keepdim=True) + 1e-6) * xr[3]
    assert rel(xn, xnr) < 1e-6 and rel(h, hr) < 1e-2
    g1, g2 = torch.randn_like(xnr), torch.randn_like(hr)
    ((xn * g1).sum() + (h.float() * g2).sum()).backward()
    ((xnr * g1).sum() + (hr * g2.bfloat16().float()).sum()).backward()
    for got, want, name in zip((x, a, rs, w), xr, "x a rs w".split()):
        assert rel(got.grad, want.grad) < 1e-3, name


def test_kda_out_gate_fwd_bwd():
    from hanuman_b200.ops.kda import KdaOutGateFn
    torch.manual_seed(13)
    T, H, K = 300, 4, 64
    o = torch.randn(T, H, K, device=DEV, requires_grad=True)
    gl = torch.randn(T, H * K, device=DEV, requires_grad=True)
    w = (1 + 0.1 * torch.randn(K, device=DEV)).requires_grad_()
    gb = (0.1 * torch.randn(H * K, device=DEV)).requires_grad_()
    y = KdaOutGateFn.apply(o, gl, w, gb)
    r = [t.detach().clone().requires_grad_() for t in (o, gl, w, gb)]
    on = r[0] * torch.rsqrt((r[0] * r[0]).mean(-1, keepdim=True) + 1e-5) * r[2]
    yr = (on * torch.sigmoid(r[1] + r[3]).view(T, H, K)).reshape(T, H * K)
    assert rel(y, yr) < 1e-2
    g = torch.randn_like(yr)
    (y.float() * g).sum().backward()
    (yr * g.bfloat16().float()).sum().backward()
    for got, want, name in zip((o, gl, w, gb), r, "o gl w gb".split()):
        assert rel(got.grad, want.grad) < 1e-3, name
