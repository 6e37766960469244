"""Index arithmetic of the conv stem's windowed GEMM, checked on the CPU.

The model runs conv1 and conv2 as GEMMs whose X rows overlap (row stride
ldx smaller than K) over zero-padded channels-last buffers, with the weights
reordered from the checkpoint's [cout, cin*3] (tap fastest) to [cout, 3*cin].
This test builds exactly those buffers, strides and reorderings in numpy
(an as_strided view plays the GPU tensor map) and compares the int32
accumulators with the oracle's conv1d accumulation (conv1d_scalar.cpp)."""
import numpy as np
import pytest
from numpy.lib.stride_tricks import as_strided

from oracle import oracle as O


def taps_first(w):
    """[cout, cin*3] (tap fastest) -> [cout, 3*cin] (channel fastest)."""
    return np.ascontiguousarray(w.reshape(w.shape[0], -1, 3).transpose(0, 2, 1).reshape(w.shape[0], -1))


def channels_last_pad(x, front, back):
    """[B, C, T] -> [B, T + front + back, C] with zero rows (iw_channels_last_pad)."""
    B, C, T = x.shape
    out = np.zeros((B, T + front + back, C), x.dtype)
    out[:, front:front + T] = x.transpose(0, 2, 1)
    return out


def windowed_rows(buf, rows, ldx, K):
    """The GEMM's X: per window `rows` rows of K bytes, ldx bytes apart."""
    B = buf.shape[0]
    flat = np.ascontiguousarray(buf).reshape(-1)
    return as_strided(flat, shape=(B, rows, K), strides=(buf.shape[1] * buf.shape[2], ldx, 1))


@pytest.mark.parametrize("B,Cin,Tin,Cout", [(2, 80, 40, 16), (1, 128, 34, 8)])
def test_conv1_layout(B, Cin, Tin, Cout):
    rng = np.random.default_rng(Cin + Tin)
    x = rng.integers(-127, 128, (B, Cin, Tin), dtype=np.int8)
    w = rng.integers(-127, 128, (Cout, Cin * 3), dtype=np.int8)
    b = rng.integers(-5000, 5000, Cout, dtype=np.int32)
    ref = O.lib().conv1d_accum(x, w, b, 1, 1)                      # [B, Cout, Tin]
    buf = channels_last_pad(x, 2, 1)                                # [B, Tin + 3, Cin]
    X = windowed_rows(buf, Tin + 1, Cin, 3 * Cin).astype(np.int64)  # row t' = t + 1
    acc = X @ taps_first(w).astype(np.int64).T + b                  # [B, Tin + 1, Cout]
    assert np.array_equal(acc[:, 1:].transpose(0, 2, 1), ref)


@pytest.mark.parametrize("B,Cin,Tin,Cout", [(2, 64, 40, 16), (1, 48, 30, 8)])
def test_conv2_layout(B, Cin, Tin, Cout):
    rng = np.random.default_rng(Cin * Tin)
    x = rng.integers(-127, 128, (B, Cin, Tin), dtype=np.int8)
    w = rng.integers(-127, 128, (Cout, Cin * 3), dtype=np.int8)
    b = rng.integers(-5000, 5000, Cout, dtype=np.int32)
    ref = O.lib().conv1d_accum(x, w, b, 2, 1)                       # [B, Cout, Tin / 2]
    Tout = ref.shape[2]
    # conv1's output as the model leaves it: one zeroed row before each window
    buf = channels_last_pad(x, 1, 0)                                 # [B, Tin + 1, Cin]
    X = windowed_rows(buf, Tout, 2 * Cin, 3 * Cin).astype(np.int64)  # row t reads rows 2t..2t+2
    acc = X @ taps_first(w).astype(np.int64).T + b
    assert np.array_equal(acc.transpose(0, 2, 1), ref)
