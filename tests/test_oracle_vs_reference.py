"""The C restatement (oracle/iw_oracle.c) against the reference's own scalar
C++ kernels (oracle/_ref, compiled from vcsd-lab/I-Whisper's sources), on
seeded random and edge-case inputs. Skipped where the reference library
could not be built (no reference checkout at build time)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.skipif(not os.path.exists(O.REF_PATH), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def P():
    return O.lib("port")


@pytest.fixture(scope="module")
def R():
    return O.lib("ref")


def eq(a, b):
    if isinstance(a, tuple):
        return all(np.array_equal(x, y) for x, y in zip(a, b))
    return np.array_equal(a, b)


@pytest.mark.parametrize("seed", [0, 1, 1234])
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (7, 100, 29), (33, 384, 70), (5, 4096, 9)])
def test_linear(P, R, seed, M, K, N):
    rng = np.random.default_rng(seed)
    x = rng.integers(-128, 128, (M, K), dtype=np.int8)
    w = rng.integers(-128, 128, (N, K), dtype=np.int8)
    b = rng.integers(-(2 ** 24), 2 ** 24, N, dtype=np.int32)
    wz = rng.integers(-128, 128, N, dtype=np.int8)
    m = rng.integers(0, 2 ** 32, N, dtype=np.uint32)
    m[0] = 0xFFFFFFFF
    s8 = rng.integers(-3, 36, N).astype(np.int8)
    s32 = rng.integers(0, 40, N).astype(np.int8)  # the reference scalar Linear32 shift is defined for s >= 0
    for bb, zz in [(b, wz), (None, None), (b, None), (None, wz)]:
        assert eq(P.linear8(x, w, bb, zz, m, s8), R.linear8(x, w, bb, zz, m, s8))
        assert eq(P.linear8_accum(x, w, bb, zz), R.linear8_accum(x, w, bb, zz))
        assert eq(P.linear32(x, w, bb, zz, m, s32), R.linear32(x, w, bb, zz, m, s32))


def test_residual15(P, R):
    rng = np.random.default_rng(3)
    br = rng.integers(-(2 ** 31), 2 ** 31, 5000, dtype=np.int32)
    r = rng.integers(-32768, 32768, 5000, dtype=np.int16)
    for m in (0, 1, 255, 32768, 65535):
        assert eq(P.residual15(br, r, m), R.residual15(br, r, m))


@pytest.mark.parametrize("d", [384, 512, 768, 1024, 1280])
def test_layernorm(P, R, d):
    rng = np.random.default_rng(d)
    x = rng.integers(-16383, 16384, (9, d), dtype=np.int16)
    x[1] = 0
    x[2] = x[2] // 256
    x[3, ::2] = 16383
    x[3, 1::2] = -16383
    g = rng.integers(-127, 128, d, dtype=np.int8)
    be = rng.integers(-(2 ** 20), 2 ** 20, d, dtype=np.int32)
    for lm, ls, om, os_ in [(200, 5, 2 ** 31 + 12345, 7), (255, 0, 0xFFFFFFFF, 0), (1, 20, 123456789, 31),
                            (37, -2, 2 ** 30, -1), (128, 7, 2 ** 31, 40)]:
        assert eq(P.layernorm32(x, g, be, lm, ls, om, os_), R.layernorm32(x, g, be, lm, ls, om, os_))
        assert eq(P.layernorm32(x, g, None, lm, ls, om, os_), R.layernorm32(x, g, None, lm, ls, om, os_))
    assert eq(P.layernorm32_stats(x), R.layernorm32_stats(x))


@pytest.mark.parametrize("d", [384, 512, 768, 1024, 1280])
def test_layernorm_full_int16_range(P, R, d):
    """Rows beyond INT15: the reference squares the centred values in int32
    (wrapping past 46340) before the renorm shift."""
    rng = np.random.default_rng(100 + d)
    x = rng.integers(-32768, 32768, (6, d), dtype=np.int16)
    x[1, : d // 2], x[1, d // 2:] = 32767, -32768
    x[2, :3], x[2, 3:] = 32767, -32768
    g = rng.integers(-127, 128, d, dtype=np.int8)
    be = rng.integers(-(2 ** 20), 2 ** 20, d, dtype=np.int32)
    assert eq(P.layernorm32(x, g, be, 200, 5, 2 ** 30, 12), R.layernorm32(x, g, be, 200, 5, 2 ** 30, 12))
    assert eq(P.layernorm32_stats(x), R.layernorm32_stats(x))


@pytest.mark.parametrize("d", [384, 512, 768, 1024, 1280])
def test_layernorm64(P, R, d):
    """The LayerNorm64 research variant (layernorm_scalar.cpp:230-297,
    626-825) with the torch wrapper's rsqrt offset 15 and offset 2."""
    rng = np.random.default_rng(200 + d)
    x = rng.integers(-32768, 32768, (9, d), dtype=np.int16)
    x[1] = 0
    x[2] = x[2] // 256
    x[3, : d // 2], x[3, d // 2:] = 32767, -32768
    x[4] = rng.integers(-16383, 16384, d)
    g = rng.integers(-127, 128, d, dtype=np.int8)
    be = rng.integers(-(2 ** 20), 2 ** 20, d, dtype=np.int32)
    for lm, ls, om, os_ in [(200, 5, 2 ** 31 + 12345, 7), (255, 0, 0xFFFFFFFF, 0), (1, 20, 123456789, 31),
                            (37, -2, 2 ** 30, -1), (128, 7, 2 ** 31, 40)]:
        assert eq(P.layernorm64(x, g, be, lm, ls, om, os_), R.layernorm64(x, g, be, lm, ls, om, os_))
        assert eq(P.layernorm64(x, g, None, lm, ls, om, os_), R.layernorm64(x, g, None, lm, ls, om, os_))
    assert eq(P.layernorm64_stats(x), R.layernorm64_stats(x))


def test_layernorm_bad_width(P):
    with pytest.raises(ValueError):
        P.layernorm32(np.zeros((1, 100), np.int16), np.zeros(100, np.int8), None, 1, 0, 1, 0)


def test_fisr(P, R):
    vals = {0}
    for bit in range(31):
        for dlt in (-1, 0, 1):
            v = (1 << bit) + dlt
            if 0 <= v < 2 ** 31:
                vals.add(v)
    rng = np.random.default_rng(17)
    v = np.array(sorted(vals) + list(rng.integers(0, 2 ** 31, 2000)), np.int32)
    for off in (13, 16, 0, 29):
        assert eq(P.fisr(v, off), R.fisr(v, off))


@pytest.mark.parametrize("C,ni,no", [(64, 64, 64), (64, 1, 64), (3000, 1, 1), (7, 7, 1)])
def test_gelu(P, R, C, ni, no):
    rng = np.random.default_rng(C)
    x = rng.integers(-128, 128, (6, C), dtype=np.int8)
    lut = rng.integers(0, 256, 16, dtype=np.uint8)
    mi = rng.integers(0, 256, ni, dtype=np.uint8); si = rng.integers(-3, 36, ni).astype(np.int8)
    mo = rng.integers(0, 256, no, dtype=np.uint8); so = rng.integers(-3, 36, no).astype(np.int8)
    assert eq(P.gelu(x, lut, mi, si, mo, so), R.gelu(x, lut, mi, si, mo, so))


@pytest.mark.parametrize("D", [1, 7, 15, 16, 17, 31, 64])
@pytest.mark.parametrize("Tq,Tk", [(1, 1), (3, 3), (4, 65), (1, 448)])
def test_attention(P, R, D, Tq, Tk):
    rng = np.random.default_rng(D * 1000 + Tq * 100 + Tk)
    B, H = 2, 3
    q = rng.integers(-128, 128, (B, H, Tq, D), dtype=np.int8)
    k = rng.integers(-128, 128, (B, H, Tk, D), dtype=np.int8)
    vt = rng.integers(-128, 128, (B, H, D, Tk), dtype=np.int8)
    for mask in (None, (rng.random((Tq, Tk)) < 0.3).astype(np.uint8), np.ones((Tq, Tk), np.uint8)):
        assert eq(P.qk(q, k), R.qk(q, k))
        for sh in (-3, 0, 1, 7, 31, 32):
            for mult in (0, 1, 77, 255):
                assert eq(P.qk_requant_rowmax(q, k, mask, mult, sh), R.qk_requant_rowmax(q, k, mask, mult, sh))
        s, rm = P.qk_requant_rowmax(q, k, mask, 77, 9)
        for fb in (1, 6, 7, 8, 13):
            assert eq(P.shift_exp(s, rm, mask, fb), R.shift_exp(s, rm, mask, fb))
        p, rs = P.shift_exp(s, rm, mask, 7)
        assert eq(P.pv(p, vt), R.pv(p, vt))
        for av_m, av_s, off in [(150, 9, 16), (255, -2, 16), (1, 33, 13), (200, 0, 0)]:
            assert eq(P.pv_norm_requant(p, vt, rs, av_m, av_s, off), R.pv_norm_requant(p, vt, rs, av_m, av_s, off))


def test_shift_exp_int16_wrap(P, R):
    # row max + 1 wraps at 32767, and extreme differences wrap in int16
    s = np.array([[[[32767, -32768, 0, 32000, -32000]]]], np.int16)
    for rm in (-32768, 32767, 0, 1):
        r = np.array([[[[rm]]]], np.int16)
        for fb in (1, 7, 13):
            assert eq(P.shift_exp(s, r, None, fb), R.shift_exp(s, r, None, fb))


def test_pv_norm_negative_rowsum(P, R):
    p = np.zeros((1, 1, 2, 4), np.uint8)
    vt = np.zeros((1, 1, 8, 4), np.int8)
    rs = np.array([0, -1], np.int32).reshape(1, 1, 2, 1)
    with pytest.raises(ValueError):
        P.pv_norm_requant(p, vt, rs, 1, 0, 16)
    with pytest.raises(ValueError):
        R.pv_norm_requant(p, vt, rs, 1, 0, 16)


@pytest.mark.parametrize("B,Cin,Tin,Cout,K,stride,pad", [(1, 3, 10, 4, 3, 1, 1), (2, 8, 31, 5, 3, 2, 1),
                                                         (1, 4, 5, 2, 5, 1, 0), (1, 80, 300, 16, 3, 1, 1)])
def test_conv1d(P, R, B, Cin, Tin, Cout, K, stride, pad):
    rng = np.random.default_rng(Cin + Tin)
    x = rng.integers(-128, 128, (B, Cin, Tin), dtype=np.int8)
    w = rng.integers(-128, 128, (Cout, Cin * K), dtype=np.int8)
    b = rng.integers(-5000, 5000, Cout, dtype=np.int32)
    assert eq(P.conv1d_accum(x, w, b, stride, pad), R.conv1d_accum(x, w, b, stride, pad))
    for m, s in [(2 ** 30 + 5, 6), (0xFFFFFFFF, 0), (123456, -2), (1, 40)]:
        for bb in (b, None):
            assert eq(P.conv1d(x, w, bb, m, s, stride, pad), R.conv1d(x, w, bb, m, s, stride, pad))


@pytest.mark.parametrize("nm,ns", [(1, 1), (16, 16), (1, 16), (16, 1)])
def test_add_requant15(P, R, nm, ns):
    rng = np.random.default_rng(nm * 10 + ns)
    x = rng.integers(-128, 128, (2, 9, 16), dtype=np.int8)
    pe = rng.integers(-128, 128, (9, 16), dtype=np.int8)
    mu = rng.integers(0, 65536, nm, dtype=np.uint16)
    su = rng.integers(-3, 36, ns).astype(np.int8)
    assert eq(P.add_requant15(x, pe, mu, su), R.add_requant15(x, pe, mu, su))


def test_classifier(P, R):
    rng = np.random.default_rng(8)
    x = rng.integers(-128, 128, (3, 100), dtype=np.int8)
    w = rng.integers(-128, 128, (517, 100), dtype=np.int8)
    assert eq(P.classifier_accum(x, w), R.classifier_accum(x, w))
    for m, s in [(3 * 2 ** 30, 3), (2 ** 31, 9), (12345, -1), (0xFFFFFFFF, 40)]:
        assert eq(P.classifier(x, w, m, s), R.classifier(x, w, m, s))
