"""Argument validation of the C ABI, without a GPU: every call below is
rejected before it touches the device, with the status code and the Python
exception class the torch-facing layer maps it to (a reference TORCH_CHECK
failure is a RuntimeError). Pointers are never dereferenced on these paths,
so placeholders stand in for device buffers."""
import ctypes as C

import pytest

from i_whisper_b200.build import build

build()  # the library is compiled in-tree (a no-op when up to date)
from i_whisper_b200 import _lib  # noqa: E402

FAKE = 0x1000  # a 16-byte aligned placeholder address


def _gemm_desc(**kw):
    d = _lib.GemmDesc()
    d.x, d.ldx, d.w, d.ldw, d.M, d.N, d.K = FAKE, 64, FAKE, 64, 32, 64, 64
    d.mode, d.out, d.ldo = _lib.IW_GEMM_INT8, FAKE, 64
    d.multiplier, d.shift = FAKE, FAKE
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _gemm_rc(**kw):
    return _lib.LIB.iw_gemm_i8(C.byref(_gemm_desc(**kw)), None)


@pytest.mark.parametrize("kw,needle", [
    (dict(M=-1), "invalid shape"),
    (dict(N=0), "invalid shape"),
    (dict(K=24, ldx=32, ldw=32), "multiples of 16"),
    (dict(ldx=40), "multiples of 16"),
    (dict(weight_zero=FAKE), "x_rowsum"),
    (dict(mode=7), "bad mode"),
    (dict(mode=_lib.IW_GEMM_LINEAR32_RES), "residual"),
    (dict(x_window_rows=5), "windowed X"),
    (dict(x_window_rows=16, x_window_stride=24), "windowed X"),
    (dict(x_window_rows=16, x_window_stride=1024, headmajor_T=16, headmajor_B=2), "windowed X"),
    (dict(gelu_table=FAKE, gelu_table_tiled=FAKE + 8), "gelu_table_tiled"),
    (dict(gelu_table_tiled=FAKE), "gelu_table_tiled"),
])
def test_gemm_descriptor_rejected(kw, needle):
    rc = _gemm_rc(**kw)
    assert rc == _lib.IW_EINVAL
    assert needle in _lib.last_error()
    with pytest.raises(RuntimeError):
        _lib.check(rc)


def test_gemm_empty_rows_is_a_no_op():
    assert _gemm_rc(M=0) == _lib.IW_OK


def test_layernorm_hidden_size():
    with pytest.raises(RuntimeError, match="hidden size"):
        _lib.call("iw_layernorm32", FAKE, FAKE, FAKE, 100, 9, 1 << 30, 18, FAKE, 4, 100, None)
    with pytest.raises(RuntimeError, match="row count"):
        _lib.call("iw_layernorm32", FAKE, FAKE, FAKE, 100, 9, 1 << 30, 18, FAKE, -1, 1024, None)


def test_greedy_step_descriptor():
    g = _lib.GreedyDesc()
    g.V, g.ld, g.alpha = 100, 64, 1.0
    assert _lib.LIB.iw_greedy_step(C.byref(g), 1, None) == _lib.IW_EINVAL
    assert "V <= ld" in _lib.last_error()
    g.ld, g.alpha = 128, 0.0
    assert _lib.LIB.iw_greedy_step(C.byref(g), 1, None) == _lib.IW_EINVAL
    assert "alpha" in _lib.last_error()


@pytest.mark.parametrize("field,value,needle", [
    ("B", -1, "invalid shape"), ("frac_bits", 0, "frac_bits"), ("rsqrt_offset", 30, "rsqrt_offset"),
    ("mask_mode", 2, "mask"),
])
def test_attention_descriptor_rejected(field, value, needle):
    a = _lib.AttnDesc()
    a.B, a.H, a.Tq, a.Tk, a.frac_bits, a.rsqrt_offset = 1, 1, 1, 8, 7, 16
    setattr(a, field, value)
    assert _lib.LIB.iw_attention_ex(C.byref(a), None) == _lib.IW_EINVAL
    assert needle in _lib.last_error()


def test_gelu_table_tiled_arguments():
    with pytest.raises(RuntimeError, match="invalid N"):
        _lib.call("iw_gelu_table_tiled", FAKE, 0, FAKE, None)
    with pytest.raises(RuntimeError, match="16-byte"):
        _lib.call("iw_gelu_table_tiled", FAKE, 128, FAKE + 4, None)


def test_conv_stem_helpers_arguments():
    with pytest.raises(RuntimeError, match="invalid shape"):
        _lib.call("iw_channels_last_pad", FAKE, 2, -1, 3000, 2, 1, FAKE, None)
    with pytest.raises(RuntimeError, match="invalid shape"):
        _lib.call("iw_zero_rows", FAKE, 4, 1024, 512, None)
    assert _lib.LIB.iw_zero_rows(FAKE, 0, 1024, 2048, None) == _lib.IW_OK
