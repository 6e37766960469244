"""Lane arithmetic of the channel-major GEMM's int8 row stores, checked on the CPU.

In the channel-major kernel, lane L of an epilogue warp owns output channel
n0 + 32*quad + L and holds 16 consecutive rows of it (v[0..15]). For the
fc1 path (GeLU table, row-major int8 output) the kernel turns that into
32-bit row stores with a 4x4 byte transpose inside each group of four
lanes: two byte permutes pack four rows' low bytes into one word, then two
`shfl.xor` steps (distances 2 and 1) with selector pairs chosen by the lane's
index inside its group. This test restates `prmt.b32` (default mode) and
`shfl.xor` from the PTX ISA in numpy, runs the exact selector constants of
gemm_cm.cu on random accumulators, and checks that every word lands at the
row and column the plain byte stores would have written."""
import numpy as np
import pytest


def prmt(a, b, sel):
    """PTX prmt.b32 default mode: result byte k = byte (sel >> 4k) & 7 of the
    8-byte value {b:a}, replicated sign when bit 3 of that nibble is set."""
    a = np.asarray(a, dtype=np.uint64)
    b = np.asarray(b, dtype=np.uint64)
    sel = np.asarray(sel, dtype=np.uint64)
    src = (b << np.uint64(32)) | a
    out = np.zeros(np.broadcast(a, b, sel).shape, dtype=np.uint64)
    for k in range(4):
        nib = (sel >> np.uint64(4 * k)) & np.uint64(0xF)
        byte = (src >> ((nib & np.uint64(7)) * np.uint64(8))) & np.uint64(0xFF)
        sign = (byte >> np.uint64(7)) * np.uint64(0xFF)
        byte = np.where(nib & np.uint64(8), sign, byte)
        out |= byte << np.uint64(8 * k)
    return out.astype(np.uint32)


def shfl_xor(vals, d):
    """shfl.sync.bfly over a full warp: lane L reads lane L ^ d."""
    return vals[np.arange(32) ^ d]


def quad_row_words(v):
    """v: [32 lanes, 16 rows] int32 results after the clamp to [-127, 127].
    Returns [32 lanes, 4] uint32 words exactly as the kernel computes them."""
    lane = np.arange(32)
    gi = lane & 3
    sel1 = np.where(gi & 2, 0x3276, 0x5410)
    sel2 = np.where(gi & 1, 0x3715, 0x6240)
    u = v.astype(np.int64).astype(np.uint32)  # the registers' bit patterns
    words = []
    for q in range(4):
        w = prmt(prmt(u[:, 4 * q], u[:, 4 * q + 1], 0x0040), prmt(u[:, 4 * q + 2], u[:, 4 * q + 3], 0x0040), 0x5410)
        x = prmt(w, shfl_xor(w, 2), sel1)
        t = prmt(x, shfl_xor(x, 1), sel2)
        words.append(t)
    return np.stack(words, axis=1)


@pytest.mark.parametrize("seed", range(4))
def test_quad_transpose_matches_byte_stores(seed):
    rng = np.random.default_rng(seed)
    N, ldo, n_base = 64, 96, 8          # channels n_base + lane; ldo > N exercises the row pitch
    r0 = 0
    v = rng.integers(-127, 128, (32, 16)).astype(np.int32)
    # reference: the plain path's byte stores out[r0 + j, n] = (int8) v[lane, j]
    ref = np.zeros((16, ldo), dtype=np.int8)
    for L in range(32):
        if n_base + L < N:
            ref[:, n_base + L] = v[L].astype(np.int8)
    # kernel: lane 4g+i stores word q at row r0 + i + 4q, columns cn .. cn+3
    got = np.zeros((16, ldo), dtype=np.int8)
    words = quad_row_words(v)
    for L in range(32):
        gi, cn = L & 3, n_base + (L & ~3)
        if cn >= N:
            continue
        for q in range(4):
            row = r0 + gi + 4 * q
            got[row, cn:cn + 4] = np.frombuffer(np.uint32(words[L, q]).tobytes(), dtype=np.int8)
    assert np.array_equal(got, ref)


def test_prmt_restatement_known_answers():
    a, b = 0x33221100, 0x77665544
    assert prmt(a, b, 0x3210) == 0x33221100
    assert prmt(a, b, 0x7654) == 0x77665544
    assert prmt(a, b, 0x0040) == 0x00004400
    assert prmt(0x80, 0, 0x0008) == 0x808080FF  # byte 0 = sign of byte 0; bytes 1-3 = byte 0
    assert prmt(0x80, 0, 0x8880) == 0xFFFFFF80
