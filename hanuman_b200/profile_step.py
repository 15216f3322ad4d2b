"""Per-kernel device-time breakdown of one training step or one profile case.

    python -m hanuman_b200.profile_step                      # flagship step, 8 x 4096 tokens
    python -m hanuman_b200.profile_step --seqs 32 --micro 8  # the bench's per-GPU batch
    python -m hanuman_b200.profile_step --case kda_bwd        # a profile_cases case

The step (or case) runs a few times untimed, then once under the CUDA
activity profiler (CUPTI); every kernel's device time is summed by name and
the top entries are printed with their launch counts.  The total is the sum
of kernel times (serialised), so compare shares, not the absolute total with
a CUDA-event timing.  The same method the reference documents for its TPU
traces: fold every device op back to a name and charge it its device time
(BENCHMARKS.md:91-99 of theorionic/hanuman).
"""
from __future__ import annotations

import argparse

import torch
from torch.profiler import ProfilerActivity, profile


def kernel_table(fn, warmup: int = 3):
    """Run ``fn`` ``warmup`` times, then once under CUPTI; returns
    ``[(name, total_us, launches)]`` sorted by time."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    agg: dict[str, list] = {}
    for ev in prof.events():
        if ev.device_type is None or "cuda" not in str(ev.device_type).lower():
            continue
        a = agg.setdefault(ev.name[:160], [0.0, 0])
        a[0] += ev.device_time_total
        a[1] += 1
    return sorted(((n, t, c) for n, (t, c) in agg.items()), key=lambda x: -x[1])


def _step_fn(seqs: int, micro: int, seq_len: int, config: str):
    from .config import get_config
    from .train import Trainer
    cfg = get_config(config).replace(seq_len=seq_len, batch_size=seqs, micro_batch=micro,
                                     train_steps=10 ** 6, warmup_steps=0)
    tr = Trainer(cfg, device="cuda:0")
    tok = torch.randint(0, cfg.vocab_size, (seqs, seq_len), device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(0))
    return lambda: tr.step(tok)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", default="hybrid_1p3b")
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--micro", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--case", default=None, help="a hanuman_b200.profile_cases case instead of the step")
    ap.add_argument("--top", type=int, default=40)
    a = ap.parse_args(argv)
    if a.case:
        from .profile_cases import CASES
        fn = CASES[a.case]()[0]
    else:
        fn = _step_fn(a.seqs, a.micro, a.seq_len, a.config)
    rows = kernel_table(fn)
    tot = sum(r[1] for r in rows)
    print(f"TOTAL {tot / 1e3:.2f} ms of kernel time ({sum(r[2] for r in rows)} launches)")
    for name, t, c in rows[:a.top]:
        print(f"{t / 1e3:9.3f} ms {100 * t / tot:5.1f} % {c:6d}  {name}")


if __name__ == "__main__":
    main()
