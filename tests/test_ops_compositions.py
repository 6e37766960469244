"""Host-side plumbing of the accumulator-only operator mirrors, on the CPU.

``qk_cuda``, ``pv_cuda``, ``conv1d_accum_cuda``, ``classifier_accum_cuda``
and ``linear32_accum_cuda_debug`` are built from two C-ABI entry points
(``iw_linear8_accum`` and ``iw_im2col``) plus pointer arithmetic, views and
the uint8 split of P. This test runs those functions on CPU tensors with
the two entry points served by a numpy stand-in that reads and writes the
same raw pointers, and compares the results with the oracle's restatement
of the reference accumulators. The GPU tests check the real entry points."""
import ctypes

import numpy as np
import pytest
import torch

from i_whisper_b200 import ops
from oracle import oracle as O


def _view(ptr, n, dtype):
    dt = np.dtype(dtype)
    buf = (ctypes.c_char * (n * dt.itemsize)).from_address(ptr)
    return np.frombuffer(buf, dtype=dt, count=n)


def _fake_call(name, *a):
    if name == "iw_linear8_accum":
        x, w, bias, wz, y, M, K, N, _ = a
        X = _view(x, M * K, np.int8).reshape(M, K).astype(np.int64)
        W = _view(w, N * K, np.int8).reshape(N, K).astype(np.int64)
        acc = X @ W.T
        if bias is not None:
            acc += _view(bias, N, np.int32)
        if wz is not None:
            acc -= _view(wz, N, np.int8).astype(np.int64) * X.sum(1, keepdims=True)
        _view(y, M * N, np.int32)[:] = acc.astype(np.uint64).astype(np.uint32).view(np.int32).reshape(-1)
    elif name == "iw_im2col":
        x, out, B, Cin, Tin, K, stride, pad, Tout, ldo, cl, _ = a
        assert cl == 0 and ldo >= Cin * K
        X = _view(x, B * Cin * Tin, np.int8).reshape(B, Cin, Tin)
        O_ = _view(out, B * Tout * ldo, np.int8).reshape(B, Tout, ldo)
        O_[:] = 0
        for t in range(Tout):
            for k in range(K):
                pos = t * stride - pad + k
                if 0 <= pos < Tin:
                    O_[:, t, k:Cin * K:K] = X[:, :, pos]
    else:
        raise AssertionError(f"unexpected entry point {name}")


def _chk_any_device(t, name, dtype):
    if not isinstance(t, torch.Tensor) or t.dtype != ops._DT[dtype] or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous {dtype} tensor")


@pytest.fixture
def cpu_ops(monkeypatch):
    monkeypatch.setattr(ops, "_chk", _chk_any_device)
    monkeypatch.setattr(ops, "_stream", lambda: None)
    monkeypatch.setattr(ops._lib, "call", _fake_call)
    return ops


@pytest.fixture(scope="module")
def L():
    return O.lib()


T = torch.from_numpy


@pytest.mark.parametrize("B,H,Tq,Tk,D", [(2, 3, 5, 17, 64), (1, 2, 1, 9, 7), (1, 1, 4, 0, 8), (1, 2, 3, 5, 0)])
def test_qk_composition(cpu_ops, L, B, H, Tq, Tk, D):
    rng = np.random.default_rng(B * 100 + Tk + D)
    q = rng.integers(-128, 128, (B, H, Tq, D), dtype=np.int8)
    k = rng.integers(-128, 128, (B, H, Tk, D), dtype=np.int8)
    got = cpu_ops.qk_cuda(T(q), T(k)).numpy()
    assert got.shape == (B, H, Tq, Tk)
    if got.size:
        assert np.array_equal(got, L.qk(q, k))


@pytest.mark.parametrize("B,H,Tq,Tk,D", [(2, 3, 4, 33, 64), (1, 1, 1, 1500, 64), (1, 2, 3, 7, 5)])
def test_pv_composition_full_uint8_range(cpu_ops, L, B, H, Tq, Tk, D):
    rng = np.random.default_rng(Tk + D)
    p = rng.integers(0, 256, (B, H, Tq, Tk), dtype=np.uint8)
    p.reshape(-1)[:4] = [255, 128, 127, 0]
    vt = rng.integers(-128, 128, (B, H, D, Tk), dtype=np.int8)
    got = cpu_ops.pv_cuda(T(p), T(vt)).numpy()
    assert np.array_equal(got, L.pv(p, vt))


@pytest.mark.parametrize("B,Cin,Tin,Cout,K,stride,pad,bias", [
    (2, 5, 20, 7, 3, 1, 1, True), (1, 8, 31, 4, 3, 2, 1, True), (2, 3, 10, 6, 4, 3, 0, False),
    (1, 2, 4, 3, 5, 1, 2, True)])
def test_conv1d_accum_composition(cpu_ops, L, B, Cin, Tin, Cout, K, stride, pad, bias):
    rng = np.random.default_rng(Cin * Tin + K)
    x = rng.integers(-128, 128, (B, Cin, Tin), dtype=np.int8)
    w = rng.integers(-128, 128, (Cout, Cin * K), dtype=np.int8)
    b = rng.integers(-(2 ** 20), 2 ** 20, Cout, dtype=np.int32) if bias else None
    got = cpu_ops.conv1d_accum_cuda(T(x), T(w), None if b is None else T(b), stride, pad).numpy()
    assert np.array_equal(got, L.conv1d_accum(x, w, b, stride, pad))


def test_conv1d_accum_checks(cpu_ops):
    x = torch.zeros(1, 4, 3, dtype=torch.int8)
    with pytest.raises(RuntimeError, match="output length would be non-positive"):
        cpu_ops.conv1d_accum_cuda(x, torch.zeros(2, 4 * 5, dtype=torch.int8), None, 1, 0)
    with pytest.raises(RuntimeError, match="divisible"):
        cpu_ops.conv1d_accum_cuda(x, torch.zeros(2, 7, dtype=torch.int8), None, 1, 0)
    with pytest.raises(RuntimeError, match="bias.numel"):
        cpu_ops.conv1d_accum_cuda(x, torch.zeros(2, 12, dtype=torch.int8), torch.zeros(3, dtype=torch.int32), 1, 1)


@pytest.mark.parametrize("B,Tt,K,N", [(2, 3, 48, 101), (1, 1, 7, 5)])
def test_classifier_accum_composition(cpu_ops, L, B, Tt, K, N):
    rng = np.random.default_rng(K * N)
    x = rng.integers(-128, 128, (B, Tt, K), dtype=np.int8)
    e = rng.integers(-128, 128, (N, K), dtype=np.int8)
    got = cpu_ops.classifier_accum_cuda(T(x), T(e)).numpy()
    assert np.array_equal(got, L.classifier_accum(x, e))
    with pytest.raises(RuntimeError, match="hidden size must match"):
        cpu_ops.classifier_accum_cuda(T(x), T(e[:, :-1].copy()))


def test_linear32_accum_is_linear8_accum(cpu_ops, L):
    rng = np.random.default_rng(9)
    x = rng.integers(-128, 128, (6, 40), dtype=np.int8)
    w = rng.integers(-128, 128, (12, 40), dtype=np.int8)
    b = rng.integers(-(2 ** 30), 2 ** 30, 12, dtype=np.int32)
    wz = rng.integers(-128, 128, 12, dtype=np.int8)
    got = cpu_ops.linear32_accum_cuda_debug(T(x), T(w), T(b), T(wz)).numpy()
    assert np.array_equal(got, L.linear8_accum(x, w, b, wz))
