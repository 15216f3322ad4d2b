"""Context parallelism on CPU ranks (gloo): a sequence split across ranks
(KDA: the recurrent state handed along the chain; attention: keys and values
all-gathered) must give the single-process output and gradients of the whole
sequence."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(B=2, S=96, H=2, K=16, V=16):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, S, H, K, generator=g, dtype=torch.float64)
    k = torch.nn.functional.normalize(torch.randn(B, S, H, K, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(B, S, H, V, generator=g, dtype=torch.float64)
    gate = -torch.rand(B, S, H, K, generator=g, dtype=torch.float64) * 0.5
    beta = torch.rand(B, S, H, generator=g, dtype=torch.float64)
    w = torch.randn(B, S, H, V, generator=g, dtype=torch.float64)   # loss weights
    return q, k, v, gate, beta, w


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from hanuman_b200.parallel.context import kda_context_parallel
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, gate, beta, w = _inputs()
        S = q.shape[1]
        seg = slice(rank * S // world, (rank + 1) * S // world)
        xs = [t[:, seg].clone().requires_grad_() for t in (q, k, v, gate, beta)]
        o = kda_context_parallel(*xs, chunk=16)
        (o * w[:, seg]).sum().backward()
        torch.save((o.detach(), [x.grad for x in xs]), os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run(tmp_path, world):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    return [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]


def test_kda_context_parallel_matches_one_process(tmp_path):
    from hanuman_b200.ops import reference as ref
    q, k, v, gate, beta, w = _inputs()
    xs = [t.clone().requires_grad_() for t in (q, k, v, gate, beta)]
    o, _ = ref.kda_chunked(*xs, chunk=16)
    (o * w).sum().backward()
    for world in (2, 3):
        res = _run(tmp_path, world)
        S = q.shape[1]
        for r, (o_r, grads_r) in enumerate(res):
            seg = slice(r * S // world, (r + 1) * S // world)
            assert torch.allclose(o_r, o[:, seg].detach(), atol=1e-10), (world, r)
            for name, gr, x in zip("q k v g beta".split(), grads_r, xs):
                assert torch.allclose(gr, x.grad[:, seg], atol=1e-9), (world, r, name)


def _attn_worker(rank, world, port, out_dir, window):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from hanuman_b200.parallel.context import attention_context_parallel
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, w = _attn_inputs()
        S = q.shape[1]
        seg = slice(rank * S // world, (rank + 1) * S // world)
        xs = [t[:, seg].clone().requires_grad_() for t in (q, k, v)]
        o = attention_context_parallel(*xs, window=window)
        (o * w[:, seg]).sum().backward()
        torch.save((o.detach(), [x.grad for x in xs]), os.path.join(out_dir, f"a{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _attn_inputs(B=2, S=60, Nq=4, Nkv=2, H=8):
    g = torch.Generator().manual_seed(6)
    q, k, v = (torch.randn(B, S, n, H, generator=g, dtype=torch.float64) for n in (Nq, Nkv, Nkv))
    w = torch.randn(B, S, Nq, H, generator=g, dtype=torch.float64)
    return q, k, v, w


def test_attention_context_parallel_matches_one_process(tmp_path):
    from hanuman_b200.ops import reference as ref
    q, k, v, w = _attn_inputs()
    S = q.shape[1]
    for window in (0, 17):
        xs = [t.clone().requires_grad_() for t in (q, k, v)]
        o = ref.causal_attention(*xs, window=window)
        (o * w).sum().backward()
        for world in (2, 3):
            ctx = mp.get_context("spawn")
            port = _port()
            procs = [ctx.Process(target=_attn_worker, args=(r, world, port, str(tmp_path), window))
                     for r in range(world)]
            for p in procs:
                p.start()
            for p in procs:
                p.join(timeout=300)
                assert p.exitcode == 0
            for r in range(world):
                o_r, grads_r = torch.load(tmp_path / f"a{r}.pt")
                seg = slice(r * S // world, (r + 1) * S // world)
                # the attention math runs in fp32 (softmax included), and the key /
                # value gradients of the ranks' queries are summed in another order
                assert torch.allclose(o_r, o[:, seg].detach(), atol=1e-6), (window, world, r)
                for name, gr, x in zip("q k v".split(), grads_r, xs):
                    assert torch.allclose(gr, x.grad[:, seg], atol=1e-5), (window, world, r, name)


def _layer_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from hanuman_b200.models.layers import KDA
    from hanuman_b200.parallel.context import kda_layer_context_parallel
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = KDA(32, 2, 16, torch.Generator().manual_seed(8), chunk=16)
        h, w = _layer_inputs()
        S = h.shape[1]
        seg = slice(rank * S // world, (rank + 1) * S // world)
        hs = h[:, seg].clone().requires_grad_()
        y = kda_layer_context_parallel(m, hs, torch.float32)
        (y * w[:, seg]).sum().backward()
        grads = {n: p.grad.clone() for n, p in m.named_parameters()}
        for t in grads.values():
            dist.all_reduce(t)
        torch.save((y.detach(), hs.grad, grads), os.path.join(out_dir, f"l{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _layer_inputs(B=2, S=64, D=32):
    g = torch.Generator().manual_seed(9)
    return torch.randn(B, S, D, generator=g), torch.randn(B, S, D, generator=g)


def test_kda_layer_context_parallel_matches_one_process(tmp_path):
    """The whole KDA layer (conv halo + state passing) on 2 and 3 ranks gives
    the single-process output, input gradient and summed parameter gradients."""
    from hanuman_b200.models.layers import KDA
    m = KDA(32, 2, 16, torch.Generator().manual_seed(8), chunk=16)
    h, w = _layer_inputs()
    hr = h.clone().requires_grad_()
    y = m(hr, torch.float32)
    (y * w).sum().backward()
    S = h.shape[1]
    for world in (2, 3):
        ctx = mp.get_context("spawn")
        port = _port()
        procs = [ctx.Process(target=_layer_worker, args=(r, world, port, str(tmp_path)))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        for r in range(world):
            y_r, gh_r, grads = torch.load(tmp_path / f"l{r}.pt")
            seg = slice(r * S // world, (r + 1) * S // world)
            assert torch.allclose(y_r, y[:, seg].detach(), atol=2e-5, rtol=1e-4), (world, r)
            assert torch.allclose(gh_r, hr.grad[:, seg], atol=2e-5, rtol=1e-4), (world, r)
            for n, p in m.named_parameters():
                assert torch.allclose(grads[n], p.grad, atol=2e-4, rtol=1e-3), (world, r, n)


def _model_cfg():
    from hanuman_b200.config import get_config
    c = get_config("tiny_hybrid")
    c.seq_len = 48
    c.batch_size = 2
    c.vocab_size = 512
    c.d_model = 64
    c.n_experts = 4
    c.d_ff = 64
    c.kda_heads = 2
    c.kda_head_dim = 16
    c.kda_chunk_size = 16
    c.n_q_heads, c.n_kv_heads, c.head_dim = 2, 1, 16
    return c


def _model_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from hanuman_b200.models.transformer import Transformer
    from hanuman_b200.parallel.context import transformer_loss_context_parallel
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _model_cfg()
        m = Transformer(c, seed=1)
        toks = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=torch.Generator().manual_seed(2))
        S = c.seq_len // world
        seg = toks[:, rank * S:(rank + 1) * S]
        nxt = toks[:, (rank + 1) * S] if rank < world - 1 else toks[:, -1]
        loss = transformer_loss_context_parallel(m, seg, nxt)
        loss.backward()
        total = loss.detach().clone()
        dist.all_reduce(total)
        grads = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
        for t in grads.values():
            dist.all_reduce(t)
        torch.save((total, grads), os.path.join(out_dir, f"m{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_transformer_loss_context_parallel_matches_one_process(tmp_path):
    """The hybrid model (3 KDA layers + 1 attention layer, MoE blocks) with
    its sequences split across 2 and 3 ranks: the ranks' loss shares sum to
    the single-process loss and their summed parameter gradients match."""
    from hanuman_b200.models.transformer import Transformer
    c = _model_cfg()
    m = Transformer(c, seed=1)
    toks = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=torch.Generator().manual_seed(2))
    loss, _ = m.loss(toks)
    loss.backward()
    for world in (2, 3):
        ctx = mp.get_context("spawn")
        port = _port()
        procs = [ctx.Process(target=_model_worker, args=(r, world, port, str(tmp_path)))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        total, grads = torch.load(tmp_path / "m0.pt")
        assert abs(total.item() - loss.item()) < 1e-4 * abs(loss.item()), (world, total, loss)
        for n, p in m.named_parameters():
            if p.grad is None:
                continue
            assert torch.allclose(grads[n], p.grad, atol=2e-5, rtol=2e-3), (world, n)
