"""The allocation-free KDA forward, called through its exported C symbol.

``hb_kda_fwd_noalloc`` serves callers that cannot allocate device memory
(code under CUDA-graph capture, runtimes with their own fixed pools, plugins in
a process whose allocator they do not own): its scratch is a fixed 64 MiB
device array inside the library.  This test loads the built library with
ctypes, calls the symbol twice in a row with different inputs, and checks each
output against the regular (allocating) entry point within the tolerance the
KDA kernel tests use.  It is collected last so that a failure here never hides
the other tests.
"""
import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    from hanuman_b200 import _build
    from hanuman_b200.ops._ext import ext
    ext()  # loads libtorch-linked dependencies into the process first
    lib = ctypes.CDLL(_build.so_path())
    fn = lib.hb_kda_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def _inputs(B, S, H, K, seed):
    g_ = torch.Generator().manual_seed(seed)
    n = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    q = n(torch.randn(B, S, H, K, generator=g_)).cuda()
    k = n(torch.randn(B, S, H, K, generator=g_)).cuda()
    v = torch.randn(B, S, H, K, generator=g_).cuda()
    g = (F.logsigmoid(torch.randn(B, S, H, K, generator=g_)) * 3.0).cuda()
    beta = torch.sigmoid(torch.randn(B, S, H, generator=g_)).cuda()
    return q, k, v, g, beta


def _reference_entry(q, k, v, g, beta, scale):
    from hanuman_b200.ops.kda import KdaCoreFn
    with torch.no_grad():
        return KdaCoreFn.apply(q, k, v, g, beta, scale)


def _rel(a, b):
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("K", [16, 32, 64])
@pytest.mark.parametrize("S", [200, 256])   # 256: a whole number of 32-token chunks
def test_noalloc_matches_allocating_entry_point_twice(K, S):
    fn = _lib()
    B, H = 2, 4
    scale = 1.0 / math.sqrt(K)
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (0, 1):  # two calls in a row share the static scratch
        q, k, v, g, beta = _inputs(B, S, H, K, seed)
        o = torch.empty_like(v)
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
                o.data_ptr(), B, S, H, K, scale, stream)
        assert rc == 0
        ref = _reference_entry(q, k, v, g, beta, scale)
        torch.cuda.synchronize()
        assert _rel(o, ref) < 1e-4


def test_noalloc_rejects_oversize_input():
    fn = _lib()
    B, S, H, K = 64, 8192, 16, 64  # far beyond the 64 MiB scratch
    dummy = torch.empty(1, device="cuda")
    p = dummy.data_ptr()
    rc = fn(p, p, p, p, p, p, B, S, H, K, 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == 3  # HB_NOALLOC_TOO_LARGE, nothing launched
    rc = fn(p, p, p, p, p, p, 1, 16, 1, 48, 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # unsupported head dim
