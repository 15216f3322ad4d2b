"""CPU tests of the oracle math (ops/reference.py) against independent restatements."""
import math

import pytest
import torch
import torch.nn.functional as F

from hanuman_b200.ops import reference as ref


def test_kda_chunked_matches_recurrent_fp64():
    torch.manual_seed(0)
    B, S, H, K = 2, 90, 2, 16
    q = ref.l2_norm(torch.randn(B, S, H, K, dtype=torch.float64))
    k = ref.l2_norm(torch.randn(B, S, H, K, dtype=torch.float64))
    v = torch.randn(B, S, H, K, dtype=torch.float64)
    beta = torch.sigmoid(torch.randn(B, S, H, dtype=torch.float64))
    for gs in (1.0, 50.0):  # 50: strongly negative decay, per-step e^-35
        g = F.logsigmoid(torch.randn(B, S, H, K, dtype=torch.float64)) * gs
        o1, s1 = ref.kda_recurrent(q, k, v, g, beta)
        for chunk in (16, 64):
            o2, s2 = ref.kda_chunked(q, k, v, g, beta, chunk=chunk)
            assert (o1.double() - o2).abs().max() < 1e-5
            assert (s1.double() - s2).abs().max() < 1e-5


def test_kda_recurrent_is_reference_step():
    """One token by hand: S*=e^g; v'=v-b S^T k; S+=b k v'^T; o=S^T q/sqrt(K)."""
    torch.manual_seed(1)
    K = 4
    S0 = torch.randn(1, 1, K, K)
    q, k, v, g = (torch.randn(1, 1, 1, K) for _ in range(4))
    g = -g.abs()
    b = torch.rand(1, 1, 1)
    o, S1 = ref.kda_recurrent(q, k, v, g, b, initial_state=S0)
    Sd = S0[0, 0] * torch.exp(g[0, 0, 0])[:, None]
    vn = v[0, 0, 0] - b[0, 0, 0] * (Sd.t() @ k[0, 0, 0])
    Se = Sd + b[0, 0, 0] * torch.outer(k[0, 0, 0], vn)
    assert torch.allclose(S1[0, 0], Se, atol=1e-6)
    assert torch.allclose(o[0, 0, 0], Se.t() @ q[0, 0, 0] / math.sqrt(K), atol=1e-6)


def test_short_conv_is_causal_depthwise():
    torch.manual_seed(2)
    x = torch.randn(2, 10, 6)
    w = torch.randn(6, 1, 4)
    y = ref.short_conv(x, w)
    y2 = F.conv1d(F.pad(x.transpose(1, 2), (3, 0)), w, groups=6).transpose(1, 2)
    assert torch.allclose(y, y2, atol=1e-5)


@pytest.mark.parametrize("window", [0, 5])
def test_attention_window_semantics(window):
    torch.manual_seed(3)
    B, S, Nq, Nkv, H = 1, 12, 4, 2, 8
    q, k, v = torch.randn(B, S, Nq, H), torch.randn(B, S, Nkv, H), torch.randn(B, S, Nkv, H)
    o = ref.causal_attention(q, k, v, window)
    for i in range(S):
        for h in range(Nq):
            kv = h // (Nq // Nkv)
            lo = max(0, i - window + 1) if window else 0
            s = (k[0, lo:i + 1, kv] @ q[0, i, h]) / math.sqrt(H)
            exp = torch.softmax(s, 0) @ v[0, lo:i + 1, kv]
            assert torch.allclose(o[0, i, h], exp, atol=1e-5)


def test_rope_rotate_half_and_positions():
    cos, sin = ref.precompute_rope(8, 16)
    q = torch.randn(1, 16, 2, 8)
    k = torch.randn(1, 16, 1, 8)
    q1, k1 = ref.apply_rope(q, k, cos, sin)
    pos = torch.arange(16)[None]
    q2, k2 = ref.apply_rope(q, k, cos, sin, pos)
    assert torch.allclose(q1, q2) and torch.allclose(k1, k2)
    # rotation preserves the norm of each pair (d, d + H/2)
    assert torch.allclose(q1.norm(dim=-1), q.norm(dim=-1), atol=1e-5)


def test_yarn_ramp_blend_matches_reference_formula():
    """model/rope.py:24-56: correction dims use dim*log(L/2pi)/(2*rot*log base);
    ramp(lo=corr(beta_slow), hi=corr(beta_fast)); inv /= 1 - (1 - 1/s) * ramp."""
    base = ref.compute_inv_freqs(64, 10000.0, 1.0, 4096)
    y = ref.compute_inv_freqs(64, 10000.0, 8.0, 4096)
    lo = 64 * math.log(4096 / (2 * math.pi)) / (2 * 1.0 * math.log(10000.0))
    hi = 64 * math.log(4096 / (2 * math.pi)) / (2 * 32.0 * math.log(10000.0))
    ramp = ((torch.arange(32) / 32 - lo) / (hi - lo)).clamp(0, 1)
    exp = base / (1 - (1 - 1 / 8.0) * ramp)
    assert torch.allclose(y, exp.float(), rtol=1e-6)


def test_sigmoid_router_selection_and_weights():
    torch.manual_seed(4)
    logits = torch.randn(5, 8)
    bias = torch.zeros(8)
    bias[3] = 10.0  # always selected
    scores, idx, w = ref.route(logits, bias, 2, "sigmoid_bias", 2.5)
    assert (idx == 3).any(-1).all()
    sel = torch.gather(torch.sigmoid(logits), -1, idx)
    assert torch.allclose(w, sel / (sel.sum(-1, keepdim=True) + 1e-9) * 2.5)
    assert torch.allclose(w.sum(-1), torch.full((5,), 2.5), atol=1e-5)


def test_router_aux_balance_is_one_at_uniform():
    T, N, K, B = 8, 4, 2, 1
    logits = torch.zeros(T, N)
    scores = torch.sigmoid(logits)
    idx = torch.tensor([[i % N, (i + 1) % N] for i in range(T)])
    aux = ref.router_aux(logits, scores, idx, B, T, N)
    assert abs(aux["balance_loss"].item() - 1.0) < 1e-5
    assert torch.equal(aux["expert_counts"], torch.full((N,), T * K / N))


def test_moe_dispatch_dense_matches_per_token_loop():
    torch.manual_seed(5)
    T, D, Fh, N, K = 7, 6, 5, 3, 2
    x = torch.randn(T, D)
    wg, wu, wd = torch.randn(N, D, Fh), torch.randn(N, D, Fh), torch.randn(N, Fh, D)
    idx = torch.randint(0, N, (T, K))
    idx[:, 1] = (idx[:, 0] + 1) % N
    w = torch.rand(T, K)
    out = ref.moe_dispatch_dense(x, idx, w, wg, wu, wd)
    for t in range(T):
        e = sum(w[t, j] * ref.swiglu(x[t:t + 1], wg[idx[t, j]], wu[idx[t, j]], wd[idx[t, j]])[0]
                for j in range(K))
        assert torch.allclose(out[t], e, atol=1e-4)
