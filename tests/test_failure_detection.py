"""Failure detection without faulting a GPU.

* CPU (gloo) ranks: a rank that stops heart-beating is reported to the others
  by the watchdog; a rank that never joins a collective makes the others'
  collective end with an error after the process-group timeout (no hang).
* GPU: the device barrier waits on a flag that nothing sets; the bounded wait
  runs out, the kernel records kErrTimeoutPeer in the status word and returns,
  and the context stays usable.
"""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _wd_worker(rank, world, port, out_path):
    import datetime
    import torch.distributed as dist
    from hanuman_b200.parallel.watchdog import PeerFailure, Watchdog
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    wd = Watchdog(store, rank, world, timeout_s=2.0, interval_s=0.2)
    if rank == 1:
        wd.close()          # rank 1 dies between steps: it stops beating and exits
        return
    result = "no-failure"
    for step in range(100):
        wd.tick(step)
        try:
            wd.check()
        except PeerFailure as e:
            result = f"detected:{e}"
            break
        time.sleep(0.1)
    wd.close()
    with open(out_path, "w") as f:
        f.write(result)
    os._exit(0)  # do not wait for the departed peer in destroy_process_group


def test_watchdog_reports_silent_rank(tmp_path):
    ctx = mp.get_context("spawn")
    out = str(tmp_path / "wd.txt")
    port = _port()
    ps = [ctx.Process(target=_wd_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    assert open(out).read().startswith("detected:")
    assert "[1]" in open(out).read()


def _timeout_worker(rank, world, port, out_path):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        time.sleep(8)       # never joins the collective below in time
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        res = "completed"
    except Exception as e:  # gloo raises once the timeout expires
        res = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"
    with open(out_path, "w") as f:
        f.write(res)
    os._exit(0)


def test_collective_with_missing_rank_errors_instead_of_hanging(tmp_path):
    ctx = mp.get_context("spawn")
    out = str(tmp_path / "to.txt")
    port = _port()
    ps = [ctx.Process(target=_timeout_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    assert open(out).read().startswith("error after")


@pytest.mark.gpu
def test_device_barrier_times_out_with_error_status():
    from hanuman_b200.ops._ext import ext
    e = ext()
    e.clear_status()
    # two "ranks" whose signal pads are both this GPU's buffer: slot 1 is never set
    pad = torch.zeros(32, dtype=torch.int32, device="cuda")
    pads = torch.tensor([pad.data_ptr(), pad.data_ptr()], dtype=torch.int64, device="cuda")
    e.set_peer_wait_budget_ns(200_000_000)      # 0.2 s
    try:
        t0 = time.time()
        e.p2p_barrier(pads, 0, 2, 1)
        torch.cuda.synchronize()
        assert time.time() - t0 < 10
        assert e.read_status() == 4             # kErrTimeoutPeer
    finally:
        e.set_peer_wait_budget_ns(120_000_000_000)
        e.clear_status()
    # the context is still usable
    x = torch.randn(64, 64, device="cuda")
    assert torch.isfinite((x @ x).sum())


@pytest.mark.gpu
def test_trainer_step_raises_after_device_wait_timeout():
    """A bounded device wait that runs out (a peer flag nothing sets, 0.2 s)
    makes the next Trainer steps raise KernelStatusError instead of training on."""
    from hanuman_b200.config import get_config
    from hanuman_b200.ops._ext import KernelStatusError, ext
    from hanuman_b200.train import Trainer
    e = ext()
    e.clear_status()
    cfg = get_config("tiny_hybrid").replace(seq_len=128, batch_size=2, micro_batch=0)
    tr = Trainer(cfg, device="cuda:0")
    toks = torch.randint(0, cfg.vocab_size, (2, 128), generator=torch.Generator().manual_seed(0))
    tr.step(toks)
    tr.check_device_status()                    # a clean step raises nothing
    pad = torch.zeros(32, dtype=torch.int32, device="cuda")
    pads = torch.tensor([pad.data_ptr(), pad.data_ptr()], dtype=torch.int64, device="cuda")
    e.set_peer_wait_budget_ns(200_000_000)
    try:
        e.p2p_barrier(pads, 0, 2, 1)            # slot 1 is never signalled
        with pytest.raises(KernelStatusError) as ei:
            for _ in range(3):
                tr.step(toks)
        assert ei.value.code == 4
    finally:
        torch.cuda.synchronize()
        e.set_peer_wait_budget_ns(120_000_000_000)
        e.clear_status()
    x = torch.randn(64, 64, device="cuda")
    assert torch.isfinite((x @ x).sum())


def test_watchdog_peer_without_any_heartbeat_is_reported_after_timeout():
    """A peer that dies before its first heartbeat is reported after timeout_s
    (counted from the watchdog's start), neither at once nor after the store's
    own blocking timeout."""
    import torch.distributed as dist
    from hanuman_b200.parallel.watchdog import Watchdog
    store = dist.HashStore()
    wd = Watchdog(store, 0, 2, timeout_s=1.0, interval_s=0.1)
    try:
        time.sleep(0.4)
        assert wd.dead == []
        t0 = time.time()
        while not wd.dead and time.time() - t0 < 5:
            time.sleep(0.05)
        assert wd.dead == [1]
        assert time.time() - t0 < 3
    finally:
        wd.close()
