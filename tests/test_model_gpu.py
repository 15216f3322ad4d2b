"""Whole model on the GPU: native path loaded, loss parity with the CPU oracle,
training descent, micro-batching."""
import math

import pytest
import torch

from hanuman_b200.config import get_config
from hanuman_b200.train import Trainer

pytestmark = pytest.mark.gpu


def _tokens(c, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=g)


def _tiny():
    c = get_config("tiny_hybrid")
    c.batch_size, c.seq_len = 2, 128
    return c


def test_tiny_hybrid_gpu_matches_cpu_first_loss():
    c = _tiny()
    toks = _tokens(c)
    cpu = Trainer(c, device="cpu")
    l_cpu = float(cpu.step(toks))
    g = Trainer(c.replace(dtype="bf16"), device="cuda")
    l_gpu = float(g.step(toks))
    assert abs(l_gpu - l_cpu) < 2e-2 * l_cpu, (l_gpu, l_cpu)
    # same update direction: second-step losses stay close (bf16 vs fp32)
    l_cpu2 = float(cpu.step(toks))
    l_gpu2 = float(g.step(toks))
    assert abs(l_gpu2 - l_cpu2) < 5e-2 * l_cpu2, (l_gpu2, l_cpu2)


@pytest.mark.parametrize("name", ["smoke", "smoke_kda", "tiny_hybrid"])
def test_presets_train_on_gpu(name):
    c = get_config(name) if name != "tiny_hybrid" else _tiny()
    c = c.replace(dtype="bf16")
    tr = Trainer(c, device="cuda")
    toks = _tokens(c)
    losses = [float(tr.step(toks)) for _ in range(8)]
    assert all(math.isfinite(x) for x in losses)
    assert losses[-1] < losses[0] - 0.3, losses


def test_gpu_micro_batching_equivalence():
    c = _tiny().replace(dtype="bf16", batch_size=4)
    toks = _tokens(c)
    a = Trainer(c, device="cuda")
    b = Trainer(c.replace(micro_batch=2), device="cuda")
    la, lb = float(a.step(toks)), float(b.step(toks))
    assert abs(la - lb) < 1e-2 * la


def test_status_word_clean_after_training():
    from hanuman_b200.ops._ext import ext
    torch.cuda.synchronize()
    assert ext().read_status() == 0


def test_cached_decoding_on_gpu_matches_recompute():
    """KV / KDA-state caches on the device: teacher-forced step logits equal the
    full recomputation's logits at every position (bf16 projections: 5e-2)."""
    from hanuman_b200.decode import DecodeCache, step
    # A top-k router is discontinuous: two nearly tied experts can swap under
    # bf16-level input differences between the two paths.  Fixed, well
    # separated biases pin the routing so the comparison measures the caches.
    c = _tiny().replace(dtype="bf16", router_type="sigmoid_bias")
    tr = Trainer(c, device="cuda")
    tr.step(_tokens(c))
    model = tr.model
    for m in model.moe_layers():
        b = torch.zeros_like(m.bias)
        b[1], b[5] = 20.0, 19.0
        m.bias.data.copy_(b)
    g = torch.Generator().manual_seed(3)
    seq = torch.randint(0, c.vocab_size, (1, 40), generator=g).cuda()
    with torch.no_grad():
        h, _ = model(seq)
        full = model.logits(h[0]).float()
        cache = DecodeCache(model)
        got = [step(model, seq[:, :8], cache).float()]
        for t in range(8, 40):
            got.append(step(model, seq[:, t:t + 1], cache).float())
    ref = torch.stack([full[7]] + [full[t] for t in range(8, 40)])
    got = torch.cat(got)
    err = ((got - ref).norm(dim=-1) / ref.norm(dim=-1)).max().item()
    assert err < 5e-2, err


def test_tiny_hybrid_gpu_tracks_cpu_oracle_for_ten_steps():
    """Config 1 trained 10 steps on the GPU (bf16 kernels) and on the CPU fp32
    oracle from the same weights and tokens: every step's loss within the
    bf16-versus-fp32 gap, and both descend."""
    c = _tiny()
    cpu = Trainer(c, device="cpu")
    gpu = Trainer(c.replace(dtype="bf16"), device="cuda")
    lc, lg = [], []
    for step in range(10):
        toks = _tokens(c, seed=step % 3)
        lc.append(float(cpu.step(toks)))
        lg.append(float(gpu.step(toks)))
    for a, b in zip(lg, lc):
        assert abs(a - b) < 3e-2 * b, (lg, lc)
    assert lg[-1] < lg[0] - 0.2 and lc[-1] < lc[0] - 0.2, (lg, lc)
