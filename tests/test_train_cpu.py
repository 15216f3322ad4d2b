"""End-to-end CPU tests: presets train, checkpoint/resume, generation, CLI."""
import math
import os

import pytest
import torch

from hanuman_b200 import flops
from hanuman_b200.checkpoint import (export_reference_tree, latest_checkpoint, load_checkpoint,
                                     param_shapes, save_checkpoint)
from hanuman_b200.config import PRESETS, get_config
from hanuman_b200.optimizer import wsd_lr
from hanuman_b200.train import Trainer


def _tokens(c, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=g)


@pytest.mark.parametrize("name", ["smoke", "smoke_kda"])
def test_smoke_presets_train(name):
    c = get_config(name)
    tr = Trainer(c, device="cpu")
    toks = _tokens(c)
    losses = [float(tr.step(toks)) for _ in range(6)]
    assert losses[-1] < losses[0] - 0.5
    assert abs(losses[0] - math.log(c.vocab_size)) < 1.0


def test_tiny_hybrid_first_loss_and_descent():
    c = get_config("tiny_hybrid")
    c.batch_size, c.seq_len = 2, 64
    tr = Trainer(c, device="cpu")
    toks = _tokens(c)
    l0 = float(tr.step(toks))
    assert abs(l0 - math.log(c.vocab_size)) < 1.0
    l1 = float(tr.step(toks))
    assert l1 < l0


def test_micro_batching_matches_full_batch():
    c = get_config("smoke_kda")
    c.batch_size = 4
    c.dtype = "fp32"  # exact comparison needs no bf16 rounding points
    toks = _tokens(c)
    a = Trainer(c, device="cpu")
    b = Trainer(c.replace(micro_batch=2), device="cpu")
    la, lb = float(a.step(toks)), float(b.step(toks))
    assert abs(la - lb) < 1e-5
    for ga, gb in zip(a.engine.groups, b.engine.groups):
        assert torch.allclose(ga.grad, gb.grad, atol=1e-5)
        assert torch.allclose(ga.master, gb.master, atol=1e-6)


def test_router_bias_update_is_per_layer_sign_rule():
    c = get_config("smoke")
    c.dense_layers = 0
    tr = Trainer(c, device="cpu")
    toks = _tokens(c)
    before = [m.bias.detach().clone() for m in tr.model.moe_layers()]
    tr.step(toks)
    counts = tr.last_metrics["expert_counts"]
    for i, m in enumerate(tr.model.moe_layers()):
        exp = before[i] - c.bias_update_rate * torch.sign(counts[i] - counts[i].mean())
        assert torch.allclose(m.bias.detach(), exp)


def test_checkpoint_resume_gives_identical_next_loss(tmp_path):
    c = get_config("smoke_kda")
    c.checkpoint_dir = str(tmp_path)
    c.optimizer = "adamw"
    toks = [_tokens(c, s) for s in range(3)]
    a = Trainer(c, device="cpu")
    a.step(toks[0])
    a.step(toks[1])
    path = save_checkpoint(a, c, 2)
    assert latest_checkpoint(c) == path
    la = float(a.step(toks[2]))
    b = Trainer(c.replace(seed=123), device="cpu")
    load_checkpoint(b, path)
    lb = float(b.step(toks[2]))
    assert abs(la - lb) < 1e-6


def test_checkpoint_names_and_shapes_follow_reference_tree():
    c = get_config("smoke")
    shapes = param_shapes(c)
    assert shapes["wte"] == (c.vocab_size, c.d_model)
    assert shapes["blocks.1.ffn.expert_w_gate"] == (c.n_experts, c.d_model, c.d_ff)
    assert shapes["blocks.0.attn.wq"] == (c.d_model, c.n_q_heads * c.head_dim)
    assert shapes["blocks.0.residual_scale"] == ()
    k = get_config("smoke_kda")
    ks = param_shapes(k)
    H, K, D = k.kda_heads, k.kda_head_dim, k.d_model
    assert ks["blocks.0.attn.q_conv.weight"] == (H * K, 1, 4)
    assert ks["blocks.0.attn.f_proj1"] == (K, H * K)
    assert ks["blocks.0.attn.a_log"] == (H,)
    # scan-path export stacks blocks on a leading layer axis
    tr = Trainer(c, device="cpu")
    tree = export_reference_tree(tr.engine.master_state(), c)
    assert tree["moe_stack/blocks/attn/wq"].shape == (c.layers - c.dense_layers, D_ := c.d_model,
                                                      c.n_q_heads * c.head_dim)
    assert "dense_stack/blocks/ffn/w_gate" in tree


def test_generate_roundtrip(tmp_path):
    from hanuman_b200.generate import load_for_generate
    c = get_config("smoke")
    c.checkpoint_dir = str(tmp_path)
    tr = Trainer(c, device="cpu")
    tr.step(_tokens(c))
    save_checkpoint(tr, c, 1)
    text, ids = load_for_generate(c, "hi", max_tokens=5, temperature=0.0, device="cpu")
    assert len(ids) == 2 + 5 or ids[-1] == 255
    # greedy decoding is deterministic
    text2, ids2 = load_for_generate(c, "hi", max_tokens=5, temperature=0.0, device="cpu")
    assert ids == ids2


def test_wsd_schedule():
    lr = lambda s: wsd_lr(s, 1.0, 0.1, 10, 100, 0.2)
    assert lr(0) == 0.0 and abs(lr(5) - 0.5) < 1e-12 and lr(10) == 1.0
    assert lr(79) == 1.0 and abs(lr(80) - 1.0) < 1e-12 and abs(lr(100) - 0.1) < 1e-12
    assert wsd_lr(0, 3e-4, 3e-4, 0, 10, 0.0) == 3e-4


def test_step_flops_matches_reference_figure():
    # BENCHMARKS.md:6 quotes 203.1 T model FLOPs for `full` at seq 4096.
    c = get_config("full")
    c.seq_len = 4096
    m, _ = flops.step_flops(c)
    assert abs(m / 1e12 - 203.1) < 0.5


def test_presets_exist_and_count():
    for name in PRESETS:
        c = get_config(name)
        assert flops.count_total_params(c) >= flops.count_active_params(c)
    assert abs(flops.count_total_params(get_config("full")) / 1e9 - 6.23) < 0.01


def test_cli_count_and_report(capsys):
    from hanuman_b200.main import main
    main(["count", "--config", "smoke"])
    main(["report", "--config", "smoke"])
    out = capsys.readouterr().out
    assert "Total params" in out and "step FLOPs" in out


@pytest.mark.parametrize("name", ["smoke", "smoke_kda"])
def test_cached_decoding_matches_full_recompute(name):
    """KV / KDA-state caches: greedy tokens equal the reference's padded
    full-recompute decoding (attention with a window in `smoke`, KDA + full
    attention in `smoke_kda`)."""
    from hanuman_b200.data import get_tokenizer
    from hanuman_b200.decode import generate_cached
    from hanuman_b200.generate import generate_from_model
    c = get_config(name).replace(dtype="fp32")
    tr = Trainer(c, device="cpu")
    for s in range(3):
        tr.step(_tokens(c, s))
    model = tr.model
    tok = get_tokenizer(c)
    _, ref_ids = generate_from_model(model, c, tok, "hello world", max_tokens=12, temperature=0.0,
                                     seq_len=64)
    _, ids = generate_cached(model, tok, "hello world", max_tokens=12, temperature=0.0)
    assert ids == ref_ids


def test_train_loop_writes_jsonl_metrics(tmp_path, monkeypatch):
    """The training loop's metrics sink: one JSON record per logged step with
    the log line's fields."""
    import json
    from hanuman_b200.train import train
    monkeypatch.chdir(tmp_path)
    c = get_config("smoke").replace(train_steps=4, log_every=1, batch_size=2, seq_len=32,
                                    metrics_jsonl=str(tmp_path / "m.jsonl"))
    _, losses = train(c, save=False, log=lambda *a, **k: None)
    recs = [json.loads(line) for line in open(tmp_path / "m.jsonl")]
    assert [r["step"] for r in recs] == [1, 2, 3]
    for r in recs:
        for key in ("loss", "ce", "z_loss", "bal_loss", "lr", "ms_per_step", "tokens_per_s", "grad_norm"):
            assert math.isfinite(r[key]), key
    assert recs[-1]["loss"] == pytest.approx(losses[-1])


def test_memory_report_labels_the_replicated_working_copy():
    from hanuman_b200.train import memory_report
    rep = memory_report(get_config("hybrid_1p3b"))
    assert "bf16 working copy and the fp32 gradient buffers are full on every rank" in rep
    assert "state shard/8" in rep


@pytest.mark.parametrize("policy", ["full", "experts", "dots"])
def test_remat_recomputes_and_gradients_are_bitwise_equal(policy, monkeypatch):
    """Activation recompute re-runs the forward in the backward and gives the
    same gradients, bit for bit, as keeping every activation."""
    from hanuman_b200 import ops
    from hanuman_b200.models.layers import KDA

    def grads(pol):
        c = get_config("smoke_kda").replace(remat=pol != "none", remat_policy=pol)
        tr = Trainer(c, device="cpu")
        toks = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len),
                             generator=torch.Generator().manual_seed(1))
        calls = {"kda": 0, "core": 0}
        f0, c0 = KDA.forward, ops.kda_core

        def kda_fwd(self, *a, **k):
            calls["kda"] += 1
            return f0(self, *a, **k)

        def core(*a, **k):
            calls["core"] += 1
            return c0(*a, **k)
        monkeypatch.setattr(KDA, "forward", kda_fwd)
        monkeypatch.setattr(ops, "kda_core", core)
        tr.engine.zero_grad()
        loss, _ = tr.forward_backward(toks)
        monkeypatch.setattr(KDA, "forward", f0)
        monkeypatch.setattr(ops, "kda_core", c0)
        g = [p.grad.clone() for p in tr.model.parameters() if p.grad is not None]
        return float(loss), g, calls

    l0, g0, c_none = grads("none")
    l1, g1, c_pol = grads(policy)
    assert l0 == l1
    assert len(g0) == len(g1) and all(torch.equal(a, b) for a, b in zip(g0, g1))
    n_kda = c_none["kda"]
    if policy in ("full", "experts"):
        assert c_pol["kda"] == 2 * n_kda          # every KDA layer ran again in the backward
    else:
        assert c_pol["kda"] == n_kda


def test_expert_parallel_construction_slices_the_full_models_experts():
    """Each rank of an expert-parallel model builds only its experts, and they
    are exactly the rank's slice of the unsliced model (same random stream)."""
    from hanuman_b200.models.transformer import Transformer
    c = get_config("tiny_hybrid")
    full = Transformer(c, seed=3)
    world = 2
    for rank in range(world):
        part = Transformer(c, seed=3, ep=(rank, world))
        fm, pm = full.moe_layers(), part.moe_layers()
        assert len(fm) == len(pm) > 0
        for a, b in zip(fm, pm):
            nl = a.n_experts // world
            for name in ("expert_w_gate", "expert_w_up", "expert_w_down"):
                assert torch.equal(getattr(a, name)[rank * nl:(rank + 1) * nl],
                                   getattr(b, name))
            assert torch.equal(a.router, b.router)
        for (na, pa), (nb, pb) in zip(full.named_parameters(), part.named_parameters()):
            assert na == nb
            if "expert_w" not in na:
                assert torch.equal(pa, pb), na


@pytest.mark.parametrize("name", sorted(PRESETS))
def test_flop_breakdown_sums_to_the_step_flops(name):
    """The per-component split (breakdown.py of the reference) adds up to the
    model FLOPs of the step accounting for every preset."""
    from hanuman_b200.breakdown import analytical_breakdown
    c = get_config(name)
    parts = analytical_breakdown(c)
    model, hw = flops.step_flops(c)
    assert all(v >= 0 for v in parts.values())
    assert abs(sum(parts.values()) - model) <= 1e-9 * model
    assert hw >= model
