"""tcgen05 GEMM numerics against an fp32 PyTorch matmul of the same bf16 inputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    from hanuman_b200.ops._ext import ext
    return ext()


def _rel_err(x, ref):
    return ((x.float() - ref).norm() / ref.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 200, 136), (304, 200, 136), (1024, 1024, 1024),
                                   (4096, 768, 1024), (77, 64, 520), (2048, 3072, 512),
                                   (256, 256, 8192), (1024, 64, 20000)])
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
def test_dense_gemm(M, N, K, ta, tb):
    # TMA needs 16-byte row strides: the contiguous dimension of each operand
    # must be a multiple of 8 bf16 elements.
    if (ta and M % 8) or (not ta and K % 8) or (tb and K % 8) or (not tb and N % 8):
        pytest.skip("operand row stride not 16-byte aligned")
    torch.manual_seed(0)
    dev = "cuda"
    a = torch.randn(K, M, device=dev) if ta else torch.randn(M, K, device=dev)
    b = torch.randn(N, K, device=dev) if tb else torch.randn(K, N, device=dev)
    a, b = a.bfloat16(), b.bfloat16()
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    ref = A @ B
    c = torch.empty(M, N, device=dev, dtype=torch.float32)
    _ext().gemm(a, b, c, ta, tb, False, 1.0)
    torch.cuda.synchronize()
    assert _rel_err(c, ref) < 1e-5
    c16 = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    _ext().gemm(a, b, c16, ta, tb, False, 1.0)
    assert _rel_err(c16, ref) < 1e-2
    acc = torch.randn(M, N, device=dev)
    ref2 = acc + 0.5 * ref
    _ext().gemm(a, b, acc, ta, tb, True, 0.5)
    assert _rel_err(acc, ref2) < 1e-5


def _groups(counts, align=128):
    starts, s = [], 0
    for c in counts:
        starts.append(s)
        s += (c + align - 1) // align * align
    return starts, s


@pytest.mark.parametrize("trans_b", [False, True])
def test_grouped_m(trans_b):
    torch.manual_seed(1)
    dev = "cuda"
    G, K, N = 6, 512, 384
    counts = [0, 130, 7, 256, 1000, 64]
    starts, R = _groups(counts)
    a = torch.randn(R, K, device=dev).bfloat16()
    b = (torch.randn(G, N, K, device=dev) if trans_b else torch.randn(G, K, N, device=dev)).bfloat16()
    c = torch.full((R, N), float("nan"), device=dev)
    BN = 256 if N >= 256 else 128
    tiles_n = (N + BN - 1) // BN
    tstart = [0]
    for cnt in counts:
        tstart.append(tstart[-1] + (cnt + 127) // 128 * tiles_n)
    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    gt = torch.tensor(tstart, dtype=torch.int32, device=dev)
    _ext().grouped_gemm_m(a, b, c, gs, gc, gt, trans_b)
    torch.cuda.synchronize()
    for g in range(G):
        if counts[g] == 0:
            continue
        s, n = starts[g], counts[g]
        W = b[g].float().t() if trans_b else b[g].float()
        ref = a[s:s + n].float() @ W
        assert _rel_err(c[s:s + n], ref) < 1e-5


@pytest.mark.parametrize("acc", [False, True])
def test_grouped_k(acc):
    torch.manual_seed(2)
    dev = "cuda"
    G, M, N = 5, 256, 384
    counts = [128, 0, 384, 128, 1024]
    starts, R = _groups(counts)
    a = torch.randn(R, M, device=dev).bfloat16()
    b = torch.randn(R, N, device=dev).bfloat16()
    c = torch.randn(G, M, N, device=dev)
    c0 = c.clone()
    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    _ext().grouped_gemm_k(a, b, c, gs, gc, acc)
    torch.cuda.synchronize()
    for g in range(G):
        s, n = starts[g], counts[g]
        ref = a[s:s + n].float().t() @ b[s:s + n].float()
        if acc:
            ref = ref + c0[g]
        assert _rel_err(c[g], ref) < 1e-5 or (n == 0 and torch.equal(c[g], ref))


@pytest.mark.parametrize("world", [2, 4])
def test_grouped_gemm_fused_gather_emulated(world):
    """The fused all-gather GEMM on one GPU: each "rank's" expert shard is a
    separate local buffer; the output must equal the plain grouped GEMM on the
    full weight, and the gathered copy must hold every expert that has rows."""
    torch.manual_seed(3)
    dev = "cuda"
    G, K, N = 8, 512, 768
    counts = [130, 0, 7, 256, 300, 64, 1, 200]
    starts, R = _groups(counts)
    a = torch.randn(R, K, device=dev).bfloat16()
    b = torch.randn(G, K, N, device=dev).bfloat16()
    gpr = G // world
    shards = [b[r * gpr:(r + 1) * gpr].clone() for r in range(world)]
    BN = 256 if N >= 256 else 128
    tiles_n = (N + BN - 1) // BN
    tstart = [0]
    for cnt in counts:
        tstart.append(tstart[-1] + (cnt + 127) // 128 * tiles_n)
    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    gt = torch.tensor(tstart, dtype=torch.int32, device=dev)
    ref = torch.full((R, N), float("nan"), device=dev).bfloat16()
    _ext().grouped_gemm_m(a, b, ref, gs, gc, gt, False)
    for rank in range(world):
        gathered = torch.zeros(G, K, N, device=dev).bfloat16()
        flags = torch.zeros(G * (K // 64) * tiles_n, dtype=torch.int32, device=dev)
        for _ in range(2):   # the flags are re-armed on every call
            c = torch.full((R, N), float("nan"), device=dev).bfloat16()
            _ext().grouped_gemm_m_gather(a, [s.data_ptr() for s in shards], rank, gpr, gathered,
                                         flags, c, gs, gc, gt)
            torch.cuda.synchronize()
            for g in range(G):
                s, n = starts[g], counts[g]
                if n:
                    assert torch.equal(c[s:s + n], ref[s:s + n]), (rank, g)
                    assert torch.equal(gathered[g], b[g]), (rank, g)
        assert _ext().read_status() == 0


_PAIR_SCRIPT = r"""
import torch
from hanuman_b200.ops._ext import ext
def rel(x, r):
    return ((x.float() - r).norm() / r.norm().clamp_min(1e-12)).item()
torch.manual_seed(0)
for (M, N, K, ta, tb) in [(4096, 768, 1024, False, False), (300, 512, 136, False, True), (1024, 3072, 512, False, False),
                          (768, 1024, 4096, True, False), (2048, 256, 64, False, True), (520, 1000, 200, True, False)]:
    a = (torch.randn(K, M, device="cuda") if ta else torch.randn(M, K, device="cuda")).bfloat16()
    b = (torch.randn(N, K, device="cuda") if tb else torch.randn(K, N, device="cuda")).bfloat16()
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    ref = A @ B
    for dt, acc in ((torch.float32, False), (torch.bfloat16, False), (torch.float32, True)):
        c = torch.randn(M, N, device="cuda").to(dt)
        c0 = c.float().clone()
        ext().gemm(a, b, c, ta, tb, acc, 0.5)
        torch.cuda.synchronize()
        want = 0.5 * ref + (c0 if acc else 0)
        e = rel(c, want)
        assert e < (1e-2 if dt == torch.bfloat16 else 1e-5), (M, N, K, ta, tb, dt, acc, e)
# grouped over K
G, M, N = 5, 512, 768
counts = [128, 0, 384, 128, 1024]
starts, s = [], 0
for c_ in counts:
    starts.append(s); s += c_
a = torch.randn(s, M, device="cuda").bfloat16()
b = torch.randn(s, N, device="cuda").bfloat16()
c = torch.randn(G, M, N, device="cuda")
c0 = c.clone()
gs = torch.tensor(starts, dtype=torch.int32, device="cuda")
gc = torch.tensor(counts, dtype=torch.int32, device="cuda")
ext().grouped_gemm_k(a, b, c, gs, gc, True)
torch.cuda.synchronize()
for g in range(G):
    st, n = starts[g], counts[g]
    r = a[st:st + n].float().t() @ b[st:st + n].float() + c0[g]
    assert rel(c[g], r) < 1e-5, g
assert ext().read_status() == 0
print("PAIR_OK")
"""


def test_pair_gemm_forced():
    """The CTA-pair (cta_group::2) kernel on every supported shape, forced on
    (it normally runs only when the pair tiles fill a wave)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, HB_GEMM_PAIR="force", PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT], env=env, capture_output=True, text=True,
                       timeout=600)
    assert "PAIR_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_grouped_m_swiglu_bwd_matches_separate_kernels():
    """dh = dy W_down^T with the SwiGLU backward in the epilogue equals the
    grouped GEMM followed by the standalone SwiGLU backward (pad rows zero)."""
    torch.manual_seed(4)
    dev = "cuda"
    G, D, F = 5, 512, 384
    counts = [130, 0, 7, 256, 300]
    starts, R = _groups(counts)
    dy = torch.randn(R, D, device=dev).bfloat16()
    wd = torch.randn(G, F, D, device=dev).bfloat16() * 0.05
    gu = torch.randn(R, 2 * F, device=dev).bfloat16()
    row_src = torch.full((R,), -1, dtype=torch.int32, device=dev)
    for s, n in zip(starts, counts):
        row_src[s:s + n] = 0
    BN = 256 if F >= 256 else 128
    tiles_n = (F + BN - 1) // BN
    tstart = [0]
    for cnt in counts:
        tstart.append(tstart[-1] + (cnt + 127) // 128 * tiles_n)
    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    gt = torch.tensor(tstart, dtype=torch.int32, device=dev)
    dh = torch.zeros(R, F, device=dev).bfloat16()
    _ext().grouped_gemm_m(dy, wd, dh, gs, gc, gt, True)
    ref = torch.empty_like(gu)
    _ext().swiglu_bwd(dh, gu, ref, row_src)
    got = torch.full_like(gu, float("nan"))
    _ext().grouped_gemm_m_swiglu_bwd(dy, wd, gu, got, gs, gc, gt)
    torch.cuda.synchronize()
    for s, n in zip(starts, counts):
        if n == 0:
            continue
        seg = slice(s, s + (n + 127) // 128 * 128)
        assert torch.equal(got[seg], ref[seg]), s


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_grouped_m_cat2_matches_fp32_reference(out_dtype):
    """c = a[:, :K1] b1[g]^T + a[:, K1:] b2[g]^T in one GEMM (second B operand
    for the K blocks past K1), against an fp32 PyTorch reference."""
    torch.manual_seed(5)
    dev = "cuda"
    G, N, K1 = 4, 384, 192
    counts = [70, 0, 129, 256]
    starts, R = _groups(counts)
    a = torch.randn(R, 2 * K1, device=dev).bfloat16()
    b1 = (torch.randn(G, N, K1, device=dev) * 0.1).bfloat16()
    b2 = (torch.randn(G, N, K1, device=dev) * 0.1).bfloat16()
    BN = 256 if N >= 256 else 128
    tiles_n = (N + BN - 1) // BN
    tstart = [0]
    for cnt in counts:
        tstart.append(tstart[-1] + (cnt + 127) // 128 * tiles_n)
    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    gt = torch.tensor(tstart, dtype=torch.int32, device=dev)
    c = torch.zeros(R, N, device=dev, dtype=out_dtype)
    _ext().grouped_gemm_m_cat2(a, b1, b2, c, gs, gc, gt)
    torch.cuda.synchronize()
    for g, (s, n) in enumerate(zip(starts, counts)):
        if n == 0:
            continue
        ref = a[s:s + n, :K1].float() @ b1[g].float().t() + a[s:s + n, K1:].float() @ b2[g].float().t()
        got = c[s:s + n].float()
        assert (got - ref).norm() / ref.norm() < (1e-5 if out_dtype == torch.float32 else 1e-2), g


def test_grouped_m_swiglu_fwd_matches_separate_kernels():
    """Gate and up in one GEMM with the SwiGLU in the epilogue equals two
    grouped GEMMs followed by the standalone SwiGLU kernel, bit for bit
    (g | u and h; pad rows of h zero)."""
    torch.manual_seed(6)
    dev = "cuda"
    G, D, F = 5, 512, 384
    counts = [130, 0, 7, 256, 300]
    starts, R = _groups(counts)
    x = torch.randn(R, D, device=dev).bfloat16()
    wg = (torch.randn(G, D, F, device=dev) * 0.05).bfloat16()
    wu = (torch.randn(G, D, F, device=dev) * 0.05).bfloat16()
    row_src = torch.full((R,), -1, dtype=torch.int32, device=dev)
    for s, n in zip(starts, counts):
        row_src[s:s + n] = 0

    def prefix(tiles_n):
        t = [0]
        for cnt in counts:
            t.append(t[-1] + (cnt + 127) // 128 * tiles_n)
        return torch.tensor(t, dtype=torch.int32, device=dev)

    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(counts, dtype=torch.int32, device=dev)
    BN = 256 if F >= 256 else 128
    gu_ref = torch.zeros(R, 2 * F, device=dev).bfloat16()
    _ext().grouped_gemm_m(x, wg, gu_ref[:, :F], gs, gc, prefix((F + BN - 1) // BN), False)
    _ext().grouped_gemm_m(x, wu, gu_ref[:, F:], gs, gc, prefix((F + BN - 1) // BN), False)
    h_ref = torch.empty(R, F, device=dev).bfloat16()
    _ext().swiglu_fwd(gu_ref, h_ref, row_src)
    gu = torch.zeros(R, 2 * F, device=dev).bfloat16()
    h = torch.full((R, F), float("nan"), device=dev).bfloat16()
    _ext().grouped_gemm_m_swiglu_fwd(x, wg, wu, h, gu, gs, gc, prefix(2 * F // 256))
    torch.cuda.synchronize()
    for s, n in zip(starts, counts):
        if n == 0:
            continue
        assert torch.equal(gu[s:s + n], gu_ref[s:s + n]), s
        seg = slice(s, s + (n + 127) // 128 * 128)
        assert torch.equal(h[seg], h_ref[seg]), s


@pytest.mark.parametrize("M", [32768, 200])   # pair path (>= 74 pair tiles) / per-segment fallback
def test_gemm_kseg_matches_fp32_reference(M):
    """c = sum_s a[:, k_s:k_s+K_s] @ b_s^T (K-segmented B) against fp32 PyTorch."""
    torch.manual_seed(10)
    dev = "cuda"
    N = 512
    ks = [256, 128, 64, 64]
    a = torch.randn(M, sum(ks), device=dev).bfloat16()
    bs = [(torch.randn(N, k, device=dev) * 0.1).bfloat16() for k in ks]
    c = torch.full((M, N), float("nan"), device=dev)
    _ext().gemm_kseg(a, bs, c, False)
    ref = a.float() @ torch.cat([b.float() for b in bs], 1).t()
    torch.cuda.synchronize()
    assert (c - ref).norm() / ref.norm() < 1e-5
    c2 = torch.ones(M, N, device=dev)
    _ext().gemm_kseg(a, bs, c2, True)
    assert (c2 - 1.0 - ref).norm() / ref.norm() < 1e-5


def _swiglu_case(seed, G=5, D=512, F=384, counts=(130, 0, 7, 256, 300)):
    torch.manual_seed(seed)
    dev = "cuda"
    starts, R = _groups(list(counts))
    BN = 256 if F >= 256 else 128

    def prefix(tiles_n):
        t = [0]
        for cnt in counts:
            t.append(t[-1] + (cnt + 127) // 128 * tiles_n)
        return torch.tensor(t, dtype=torch.int32, device=dev)

    gs = torch.tensor(starts, dtype=torch.int32, device=dev)
    gc = torch.tensor(list(counts), dtype=torch.int32, device=dev)
    return dev, starts, R, BN, prefix, gs, gc


def test_grouped_m_swiglu_fwd_matches_fp32_product():
    """The fused gate|up GEMM with the SwiGLU epilogue against an fp32 PyTorch
    product of the same bf16 operands: g | u and h = silu(g) u per expert."""
    import torch.nn.functional as F_
    G, D, F = 5, 512, 384
    dev, starts, R, BN, prefix, gs, gc = _swiglu_case(16, G, D, F)
    counts = (130, 0, 7, 256, 300)
    x = torch.randn(R, D, device=dev).bfloat16()
    wg = (torch.randn(G, D, F, device=dev) * 0.05).bfloat16()
    wu = (torch.randn(G, D, F, device=dev) * 0.05).bfloat16()
    gu = torch.zeros(R, 2 * F, device=dev).bfloat16()
    h = torch.zeros(R, F, device=dev).bfloat16()
    _ext().grouped_gemm_m_swiglu_fwd(x, wg, wu, h, gu, gs, gc, prefix(2 * F // 256))
    torch.cuda.synchronize()
    for g, (s, n) in enumerate(zip(starts, counts)):
        if n == 0:
            continue
        xf = x[s:s + n].float()
        gr, ur = xf @ wg[g].float(), xf @ wu[g].float()
        hr = F_.silu(gr) * ur
        assert _rel_err(gu[s:s + n, :F].float(), gr) < 5e-3, g
        assert _rel_err(gu[s:s + n, F:].float(), ur) < 5e-3, g
        assert _rel_err(h[s:s + n].float(), hr) < 1e-2, g


def test_grouped_m_swiglu_bwd_matches_fp32_product():
    """dh = dy W_down^T with the SwiGLU backward in the epilogue against fp32
    PyTorch: dg = dh u silu'(g), du = dh silu(g)."""
    G, D, F = 5, 512, 384
    dev, starts, R, BN, prefix, gs, gc = _swiglu_case(17, G, D, F)
    counts = (130, 0, 7, 256, 300)
    dy = torch.randn(R, D, device=dev).bfloat16()
    wd = (torch.randn(G, F, D, device=dev) * 0.05).bfloat16()
    gu = torch.randn(R, 2 * F, device=dev).bfloat16()
    got = torch.zeros_like(gu)
    _ext().grouped_gemm_m_swiglu_bwd(dy, wd, gu, got, gs, gc, prefix((F + BN - 1) // BN))
    torch.cuda.synchronize()
    for g, (s, n) in enumerate(zip(starts, counts)):
        if n == 0:
            continue
        dh = dy[s:s + n].float() @ wd[g].float().t()
        gg, uu = gu[s:s + n, :F].float(), gu[s:s + n, F:].float()
        sg = torch.sigmoid(gg)
        dg = dh * uu * sg * (1 + gg * (1 - sg))
        du = dh * gg * sg
        assert _rel_err(got[s:s + n, :F].float(), dg) < 1e-2, g
        assert _rel_err(got[s:s + n, F:].float(), du) < 1e-2, g
