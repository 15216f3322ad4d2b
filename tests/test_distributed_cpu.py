"""Data-parallel engine on CPU ranks (gloo): sharded master/optimizer state,
reduce-scatter of gradients and all-gather of the working copy must reproduce
single-process full-batch training."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from hanuman_b200.config import get_config


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    c = get_config("smoke_kda")
    c.batch_size = 4
    c.dtype = "fp32"
    c.optimizer = "adamw"
    c.weight_decay = 0.1
    c.dense_layers = 0
    return c


def _tokens(c, step):
    g = torch.Generator().manual_seed(100 + step)
    return torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=g)


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from hanuman_b200.parallel.mesh import init_distributed
    from hanuman_b200.train import Trainer
    ctx = init_distributed(timeout_s=60)
    try:
        c = _cfg()
        tr = Trainer(c, device="cpu", dist_ctx=ctx)
        per = c.batch_size // world
        losses = []
        for step in range(3):
            toks = _tokens(c, step)[rank * per:(rank + 1) * per]
            losses.append(float(tr.step(toks)))
        eng = tr.engine
        # FSDP: every block's and the embedding's matrix group keeps only its
        # shard between steps (no storage behind the full working tensor)
        assert len(eng.sharded_units) == len(tr.model.blocks) + 1
        for gs in eng.sharded_units.values():
            for g in gs:
                assert g.work.untyped_storage().nbytes() == 0
                assert g.shard.numel() * world == g.numel
        st = tr.engine.master_state()
        if rank == 0:
            torch.save((losses, {k: v.clone() for k, v in st.items()},
                        [m.bias.detach().clone() for m in tr.model.moe_layers()]), out_path)
    finally:
        ctx.shutdown()


def test_fsdp_gloo_matches_single_process(tmp_path):
    from hanuman_b200.train import Trainer
    c = _cfg()
    single = Trainer(c, device="cpu")
    ref_losses = [float(single.step(_tokens(c, s))) for s in range(3)]
    ref_state = single.engine.master_state()
    ctx = mp.get_context("spawn")
    port = _port()
    out = str(tmp_path / "rank0.pt")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    losses, state, biases = torch.load(out)
    for a, b in zip(losses, ref_losses):
        assert abs(a - b) < 1e-4, (losses, ref_losses)
    for k, v in ref_state.items():
        assert torch.allclose(state[k], v, atol=2e-5, rtol=1e-4), k
    for b, m in zip(biases, single.model.moe_layers()):
        assert torch.allclose(b, m.bias.detach())


def test_unit_hooks_fire_in_backward_order():
    """The block-boundary autograd nodes call pre_backward(i) before block i's
    backward and post_backward(i) once its gradients are final, last block first:
    the order in which the engine starts the per-block gradient reduce-scatter."""
    from hanuman_b200.models.transformer import Transformer
    c = _cfg()
    m = Transformer(c)
    events = []

    class Rec:
        def pre_forward(self, u):
            events.append(("fwd", u))

        def post_forward(self, u):
            events.append(("fwd_done", u))

        def pre_backward(self, u):
            events.append(("pre", u))

        def post_backward(self, u):
            grads_final = all(p.grad is not None for p in m.blocks[u - 1].parameters() if p.requires_grad
                              and p is not m.blocks[u - 1].ffn.bias if hasattr(m.blocks[u - 1].ffn, "bias"))
            events.append(("post", u, grads_final))

    m.unit_hooks = Rec()
    loss, _ = m.loss(_tokens(c, 0))
    loss.backward()
    L = len(m.blocks)
    want = [("fwd", 0)]
    for u in range(1, L + 1):
        want += [("fwd", u), ("fwd_done", u)]
    for u in range(L, 0, -1):
        want += [("pre", u), ("post", u, True)]
    assert events == want, events
