"""GPU test of iw_linear8_noalloc, the allocation-free Linear8 entry point.

Callers that cannot allocate device memory while they run (captured CUDA
graphs with a pool they do not own, servers that pre-plan all device memory,
foreign runtimes that only pass raw pointers) use iw_linear8_noalloc, which
keeps the zero-point row sums in a fixed device array instead of a scratch
allocation. This file checks, through the C ABI, that it returns exactly what
iw_linear8 returns on calls in a row -- a larger call first, then a smaller
one that runs over the rows the first call left in the shared array, then
one without a weight zero point -- that it takes nothing from the device's
stream-ordered memory pool (where iw_linear8 takes its scratch), and that
sizes beyond its array are rejected. It is named so that pytest collects it
after every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(rng, M, K, N):
    x = rng.integers(-128, 128, (M, K), dtype=np.int8)
    w = rng.integers(-128, 128, (N, K), dtype=np.int8)
    b = rng.integers(-(2 ** 20), 2 ** 20, N, dtype=np.int32)
    wz = rng.integers(-128, 128, N, dtype=np.int8)
    m = rng.integers(0, 2 ** 32, N, dtype=np.uint32)
    s = rng.integers(-2, 34, N).astype(np.int8)
    return [torch.from_numpy(a).cuda() for a in (x, w, b, wz, m, s)]


def _call(name, t, M, K, N, zero_point=True):
    from i_whisper_b200 import _lib
    x, w, b, wz, m, s = t
    y = torch.empty(M, N, dtype=torch.int8, device="cuda")
    rc = getattr(_lib.LIB, name)(x.data_ptr(), w.data_ptr(), b.data_ptr(), wz.data_ptr() if zero_point else None,
                                 m.data_ptr(), s.data_ptr(), y.data_ptr(), M, K, N,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return y


class _PoolWatch:
    """Used-memory high-water mark of the current device's stream-ordered
    memory pool (the one cudaMallocAsync draws from), through the CUDA
    runtime the library itself loads."""
    USED_MEM_HIGH = 8  # cudaMemPoolAttrUsedMemHigh

    def __init__(self):
        self.rt = ctypes.CDLL("libcudart.so.12")
        self.pool = ctypes.c_void_p()
        assert self.rt.cudaDeviceGetMemPool(ctypes.byref(self.pool), torch.cuda.current_device()) == 0

    def reset(self):
        zero = ctypes.c_uint64(0)
        assert self.rt.cudaMemPoolSetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(zero)) == 0

    def high(self) -> int:
        v = ctypes.c_uint64(0)
        assert self.rt.cudaMemPoolGetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(v)) == 0
        return v.value


def test_noalloc_matches_linear8_twice():
    rng = np.random.default_rng(2024)
    # larger then smaller: the second call's rows are a prefix of what the
    # first left in the shared array, so a read of stale rows would show
    shapes = [(4096, 384, 1536), (1500, 1024, 1024)]
    for M, K, N in shapes:
        t = _case(rng, M, K, N)
        ref = _call("iw_linear8", t, M, K, N)
        got = _call("iw_linear8_noalloc", t, M, K, N)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (M, K, N)
    # without a weight zero point the array is not used at all
    M, K, N = 777, 512, 256
    t = _case(rng, M, K, N)
    ref = _call("iw_linear8", t, M, K, N, zero_point=False)
    got = _call("iw_linear8_noalloc", t, M, K, N, zero_point=False)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


def test_noalloc_takes_nothing_from_the_memory_pool():
    rng = np.random.default_rng(11)
    M, K, N = 2000, 1024, 512
    t = _case(rng, M, K, N)
    _call("iw_linear8_noalloc", t, M, K, N)  # first call on this device: symbol lookup
    torch.cuda.synchronize()
    watch = _PoolWatch()
    watch.reset()
    _call("iw_linear8_noalloc", t, M, K, N)
    torch.cuda.synchronize()
    assert watch.high() == 0
    # the check can see an allocation: iw_linear8 takes its row sums from the pool
    _call("iw_linear8", t, M, K, N)
    torch.cuda.synchronize()
    assert watch.high() >= M * 4


def test_noalloc_rejects_oversize_and_unpadded():
    from i_whisper_b200 import _lib
    rng = np.random.default_rng(7)
    M = _lib.NOALLOC_MAX_ROWS + 1
    t = _case(rng, M, 16, 32)
    with pytest.raises(_lib.IWhisperError, match="exceeds"):
        _call("iw_linear8_noalloc", t, M, 16, 32)
    t = _case(rng, 8, 24, 32)
    with pytest.raises(_lib.IWhisperError, match="multiple of 16"):
        _call("iw_linear8_noalloc", t, 8, 24, 32)
