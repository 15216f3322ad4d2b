"""Data parallel on 2 GPUs: the fused peer-memory transport (reduce-scatter in a
kernel reading peers over NVLink, optimizer storing the new weights into every
peer) must match the NCCL baseline, and so must the fused expert-weight
all-gather inside the grouped GEMMs.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _losses_match(la, lb):
    """Step 1 sees identical weights and the same forward kernels, so its loss
    agrees to rounding.  Later steps inherit run-to-run differences of the
    gradients that are summed with atomics (the split-K weight-gradient GEMMs,
    the embedding scatter-add, the decay-bias sums); AdamW's first updates are
    sign-like, so a near-zero gradient element can move by 2 lr either way and
    the loss drifts by up to about 1e-3 relative between any two runs, the NCCL
    arm against itself included (measured: 2.3e-4 and 2.5e-4 at steps 2 and 3
    of two identical NCCL runs).  The transports themselves are checked
    exactly by test_p2p_transport_kernels_are_exact_and_replayable."""
    assert abs(la[0] - lb[0]) < 1e-4 * abs(la[0]), (la, lb)
    for a, b in zip(la[1:], lb[1:]):
        assert abs(a - b) < 3e-3 * abs(a), (la, lb)


def _state_bound(name):
    """Largest difference of one state element that two correct runs of 3 steps
    can show.  AdamW parameters: the first updates are sign-like, so an element
    can move by up to 2 lr per step between runs (lr = 3e-4).  The MoE router
    bias (`ffn.bias`) is not an AdamW parameter: each step moves it by
    +-bias_update_rate or 0 by the sign of the expert's load against the mean
    (reference train.py:259), so one token routed differently between the runs
    flips that sign and the runs can differ by 2 * rate per step (rate = 1e-3)."""
    if name.endswith("ffn.bias"):
        return 3 * 2 * 1e-3 + 1e-6
    return 6 * 3e-4 + 1e-5


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from hanuman_b200.config import get_config
    from hanuman_b200.ops._ext import ext
    from hanuman_b200.parallel.mesh import init_distributed
    from hanuman_b200.train import Trainer
    ctx = init_distributed(timeout_s=120)
    try:
        res = {}
        for fused in (False, True, "gather"):
            c = get_config("tiny_hybrid").replace(dtype="bf16", batch_size=4, seq_len=128,
                                                  fused_comm=fused in (True, "gather"))
            if fused == "gather":
                c = c.replace(expert_weights="fused_gather")
            tr = Trainer(c, dist_ctx=ctx)
            assert tr.engine.transport == ("p2p" if fused in (True, "gather") else "nccl")
            if fused == "gather":
                assert all(getattr(m, "_gather", None) is not None for m in tr.model.moe_layers())
            per = c.batch_size // world
            losses = []
            for step in range(3):
                g = torch.Generator().manual_seed(step)
                toks = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=g)
                losses.append(float(tr.step(toks[rank * per:(rank + 1) * per])))
            st = tr.engine.master_state()
            res[fused] = (losses, {k: v.float().cpu() for k, v in st.items()})
            del tr
        torch.cuda.synchronize()
        assert ext().read_status() == 0
        if rank == 0:
            torch.save(res, out_path)
    finally:
        ctx.shutdown()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_transport_matches_nccl(tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    out = str(tmp_path / "res.pt")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    res = torch.load(out)
    # the fused expert-weight gather (P1) computes what the replicated weights
    # compute: the same products (the replicated arm's SwiGLU-epilogue GEMM
    # matches the separate GEMMs + SwiGLU bit for bit), only the source of B differs
    (lg, sg), (lp, sp) = res["gather"], res[True]
    _losses_match(lg, lp)
    for k in sp:
        diff = (sg[k] - sp[k]).abs()
        assert diff.max().item() <= _state_bound(k), (k, diff.max().item())
    (l0, s0), (l1, s1) = res[False], res[True]
    _losses_match(l0, l1)
    # The embedding gradient is summed with atomics, so the two runs differ in the
    # last bits, and the state may drift by _state_bound per element.
    for k in s0:
        diff = (s0[k] - s1[k]).abs()
        assert diff.max().item() <= _state_bound(k), (k, diff.max().item())
        if diff.numel() > 1000:
            assert diff.mean().item() < 1e-4, (k, diff.mean().item())


def _ep_worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from hanuman_b200.config import get_config
    from hanuman_b200.ops._ext import ext
    from hanuman_b200.parallel.mesh import init_distributed
    from hanuman_b200.train import Trainer
    ctx = init_distributed(timeout_s=120)
    try:
        res = {}
        for ep in (1, 2):
            # capacity 4x the mean load: no (source, expert) block overflows at T = 256
            c = get_config("tiny_hybrid").replace(dtype="bf16", batch_size=4, seq_len=128,
                                                  mesh_expert_axis=ep, capacity_factor=4.0)
            tr = Trainer(c, dist_ctx=ctx)
            per = c.batch_size // world
            losses = []
            for step in range(3):
                g = torch.Generator().manual_seed(step)
                toks = torch.randint(0, c.vocab_size, (c.batch_size, c.seq_len), generator=g)
                losses.append(float(tr.step(toks[rank * per:(rank + 1) * per])))
            st = tr.engine.master_state()
            res[ep] = (losses, {k: v.float().cpu() for k, v in st.items()})
            del tr
        torch.cuda.synchronize()
        assert ext().read_status() == 0
        if rank == 0:
            torch.save(res, out_path)
    finally:
        ctx.shutdown()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_matches_data_parallel(tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    out = str(tmp_path / "ep.pt")
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    res = torch.load(out)
    (l0, s0), (l1, s1) = res[1], res[2]
    for a, b in zip(l0, l1):
        assert abs(a - b) < 2e-3 * abs(a), (l0, l1)
    assert set(s0) == set(s1)
    for k in s0:
        assert s0[k].shape == s1[k].shape, k
        diff = (s0[k] - s1[k]).abs()
        assert diff.max().item() <= _state_bound(k), (k, diff.max().item())


def _replay_worker(rank, world, port, out_path):
    """The peer-memory reduce-scatter run twice on the same symmetric buffers:
    bitwise-equal outputs, the NCCL all-reduce's values, and every signal-pad
    slot at the last barrier epoch; the FSDP copy-engine gather of every rank's
    symmetric shard equals NCCL's all-gather bit for bit."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm
    from hanuman_b200.ops._ext import ext
    from hanuman_b200.parallel.mesh import init_distributed
    ctx = init_distributed(timeout_s=120)
    try:
        dev = torch.device("cuda", rank)
        n = (1 << 20) + 12          # not a multiple of the block stride: exercises the tail
        buf = symm.empty(n, dtype=torch.float32, device=dev)
        hdl = symm.rendezvous(buf, dist.group.WORLD)
        flags = symm.empty(32, dtype=torch.int32, device=dev)
        flags.zero_()
        fh = symm.rendezvous(flags, dist.group.WORLD)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        buf.copy_(torch.randn(n, generator=g, device=dev))
        torch.cuda.synchronize(dev)
        dist.barrier()
        peers = torch.tensor([int(hdl.buffer_ptrs[r]) for r in range(world)], dtype=torch.int64, device=dev)
        pads = torch.tensor([int(p) for p in fh.buffer_ptrs], dtype=torch.int64, device=dev)
        per = (n // world) // 4 * 4
        lo = rank * per
        cnt = per if rank < world - 1 else n - lo
        outs, epoch = [], 0
        for _ in range(2):
            epoch += 1
            ext().p2p_barrier(pads, rank, world, epoch)
            out = torch.empty(cnt, device=dev)
            ss = torch.zeros(1, device=dev)
            ext().p2p_reduce_scatter(peers, world, lo, cnt, out, 0.5, ss)
            epoch += 1
            ext().p2p_barrier(pads, rank, world, epoch)
            outs.append((out.clone(), ss.clone()))
        torch.cuda.synchronize(dev)
        ref = buf.clone()
        dist.all_reduce(ref)
        ref = ref[lo:lo + cnt] * 0.5
        # FSDP gather: copy engines from the peers' symmetric shards vs NCCL
        shard = symm.empty(4096, dtype=torch.bfloat16, device=dev)
        shard.copy_(torch.randn(4096, generator=g, device=dev).bfloat16())
        sh = symm.rendezvous(shard, dist.group.WORLD)
        torch.cuda.synchronize(dev)
        dist.barrier()
        full = torch.empty(4096 * world, dtype=torch.bfloat16, device=dev)
        ext().copy_engine_gather([int(sh.buffer_ptrs[r]) for r in range(world)], 4096 * 2, full)
        ref_full = torch.empty_like(full)
        dist.all_gather_into_tensor(ref_full, shard)
        torch.cuda.synchronize(dev)
        res = {"bitwise": torch.equal(outs[0][0], outs[1][0]),
               "gather_exact": torch.equal(full, ref_full),
               "err": ((outs[0][0] - ref).abs().max() / ref.abs().max()).item(),
               "ss_rel": abs(outs[0][1].item() - (ref * ref).sum().item()) / (ref * ref).sum().item(),
               "flags": flags[:world].cpu().tolist(), "epoch": epoch,
               "status": int(ext().read_status())}
        torch.save(res, f"{out_path}.{rank}")
        dist.barrier()
    finally:
        ctx.shutdown()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_transport_kernels_are_exact_and_replayable(tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    out = str(tmp_path / "replay.pt")
    procs = [ctx.Process(target=_replay_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        res = torch.load(f"{out}.{r}")
        assert res["bitwise"], res
        assert res["gather_exact"], res
        assert res["err"] < 1e-6, res
        assert res["ss_rel"] < 1e-5, res
        assert res["flags"] == [res["epoch"]] * 2, res
        assert res["status"] == 0, res
