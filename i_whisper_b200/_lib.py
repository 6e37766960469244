"""ctypes binding of ``libiwhisper_b200.so`` (the C ABI in
``include/iwhisper_b200.h``).

The shared library is the product: there is no CPU fallback. Loading
fails with an ImportError naming the missing file when the library has not
been built (``python -m i_whisper_b200.build``).
"""
from __future__ import annotations

import ctypes as C
import os

from .build import LIB_PATH

IW_OK = 0
IW_EINVAL = -1
IW_EVALUE = -2
IW_ECUDA = -3
IW_EDEVICE = -4
IW_EOVERFLOW = -5

_P = C.c_void_p
_I64 = C.c_int64
_U8, _I8, _U16, _U32, _I32 = C.c_uint8, C.c_int8, C.c_uint16, C.c_uint32, C.c_int32

# name -> argtypes (restype is always c_int)
SIGNATURES = {
    "iw_linear8": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear8_accum": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear8_requant": [_P, _P, _P, _P, _I64, _I64, _P],
    "iw_rounding_rshift": [_P, C.c_uint32, _P, _I64, _P],
    "iw_linear32": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear32_residual15": [_P, _P, _P, _P, _P, _P, _P, _U16, _P, _I64, _I64, _I64, _P],
    "iw_residual15": [_P, _P, _U16, _P, _I64, _P],
    "iw_layernorm32": [_P, _P, _P, _U8, _I8, _U32, _I8, _P, _I64, _I64, _P],
    "iw_layernorm32_stats": [_P, _P, _P, _P, _I64, _I64, _P],
    "iw_layernorm64": [_P, _P, _P, _U8, _I8, _U32, _I8, _P, _I64, _I64, _P],
    "iw_layernorm64_stats": [_P, _P, _P, _I64, _I64, _P],
    "iw_layernorm64_ex": [_P, _I64, _P, _P, _U8, _I8, _U32, _I8, _P, _I64, _I64, _I64, _P, _P, _P],
    "iw_layernorm32_rsqrt": [_P, _P, _I64, _P],
    "iw_gelu": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P],
    "iw_qk_requant_rowmax": [_P, _P, _P, _U8, _I8, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_shift_exp": [_P, _P, _P, _I32, _P, _P, _I64, _I64, _I64, _I64, _P],
    "iw_pv_norm_requant": [_P, _P, _P, _U8, _I8, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_attention": [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                     C.c_int, _P, _U8, _I8, _I32, _U8, _I8, _I64, _P],
    "iw_conv1d": [_P, _P, _P, _U32, _I8, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_add_requant15": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_embed_add_requant15": [_P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_classifier": [_P, _P, _U32, _I8, _P, _I64, _I64, _I64, _P],
    "iw_rowsum_i8": [_P, _I64, _I64, _I64, _P, _P],
    "iw_device_status": [C.POINTER(C.c_uint32), C.c_int],
    "iw_abi_version": [],
    "iw_gemm_i8": [_P, _P],
    "iw_attention_ex": [_P, _P],
    "iw_layernorm32_ex": [_P, _I64, _P, _P, _U8, _I8, _U32, _I8, _P, _I64, _I64, _I64, _P, _P, _P],
    "iw_im2col": [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, C.c_int, _P],
    "iw_channels_last_pad": [_P, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "iw_zero_rows": [_P, _I64, _I64, _I64, _P],
    "iw_set_wait_timeout_ns": [C.c_uint64],
    "iw_selftest_wait_timeout": [_P, _P],
    "iw_embed_add_requant15_dev": [_P, _P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "iw_kv_append": [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P],
    "iw_greedy_step": [_P, _I64, _P],
    "iw_add_i32": [_P, _I32, _P],
    "iw_log_mel_int8": [_P, _I64, _I64, _I64, _P, _I64, C.c_float, _P, _P],
    "iw_gelu_table": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P],
    "iw_gelu_table_tiled": [_P, _I64, _P, _P],
    "iw_shift_exp_table": [_I32, _P, _P],
    "iw_linear8_noalloc": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
}

IW_GEMM_ACC32, IW_GEMM_INT8, IW_GEMM_LINEAR32, IW_GEMM_LINEAR32_RES = 0, 1, 2, 3
NOALLOC_MAX_ROWS = 65536  # IW_NOALLOC_MAX_ROWS


class GemmDesc(C.Structure):
    """``iw_gemm_desc`` (include/iwhisper_b200.h)."""
    _fields_ = [
        ("x", _P), ("ldx", _I64), ("w", _P), ("ldw", _I64), ("M", _I64), ("N", _I64), ("K", _I64),
        ("mode", C.c_int), ("out", _P), ("ldo", _I64),
        ("bias", _P), ("weight_zero", _P), ("x_rowsum", _P), ("multiplier", _P), ("shift", _P),
        ("scalar_multiplier", _U32), ("scalar_shift", _I32),
        ("lut", _P), ("luti_multiplier", _P), ("luti_shift", _P), ("luto_multiplier", _P), ("luto_shift", _P),
        ("luti_per_channel", C.c_int), ("luto_per_channel", C.c_int),
        ("residual", _P), ("ldr", _I64), ("residual_multiplier", _U32),
        ("pos", _P), ("pos_T", _I64), ("pos_multiplier", _P), ("pos_shift", _P), ("pos_per_channel", C.c_int),
        ("transpose_T", _I64), ("headmajor_T", _I64), ("headmajor_B", _I64),
        ("out_rowsum", _P), ("tile_n", C.c_int), ("gelu_table", _P),
        ("vt_out", _P), ("vt_ld", _I64), ("vt_col0", _I64), ("vt_T", _I64),
        ("kv_cache_k", _P), ("kv_cache_v", _P), ("kv_col0", _I64), ("kv_heads", _I64), ("kv_T", _I64),
        ("kv_Tcap", _I64), ("kv_pos", _I64), ("kv_pos_dev", _P), ("gelu_table_tiled", _P),
        ("x_window_rows", _I64), ("x_window_stride", _I64), ("weight_sign", _P),
    ]


class AttnDesc(C.Structure):
    """``iw_attn_desc`` (include/iwhisper_b200.h)."""
    _fields_ = [
        ("q", _P), ("ldq", _I64), ("q_bs", _I64), ("q_hs", _I64),
        ("k", _P), ("ldk", _I64), ("k_bs", _I64), ("k_hs", _I64),
        ("v", _P), ("ldv", _I64), ("v_bs", _I64), ("v_hs", _I64),
        ("y", _P), ("ldy", _I64), ("y_bs", _I64), ("y_hs", _I64),
        ("B", _I64), ("H", _I64), ("Tq", _I64), ("Tk", _I64),
        ("Tk_dev", _P), ("Tk_cap", _I64), ("mask_mode", C.c_int), ("mask", _P),
        ("qk_multiplier", _U8), ("qk_shift", _I8), ("frac_bits", _I32),
        ("av_multiplier", _U8), ("av_shift", _I8), ("rsqrt_offset", _I32),
        ("exp_table", _P), ("vt", _P), ("vt_ld", _I64), ("vt_ready", C.c_int), ("row_sum_out", _P),
    ]


class GreedyDesc(C.Structure):
    """``iw_greedy_desc`` (include/iwhisper_b200.h)."""
    _fields_ = [
        ("logits", _P), ("ld", _I64), ("V", _I64), ("alpha", C.c_float),
        ("suppress_bits", _P), ("blank", _P), ("n_blank", _I64),
        ("eot", _I64), ("timestamp_begin", _I64), ("no_timestamps", _I64), ("max_initial_timestamp_index", _I64),
        ("state", _P), ("tokens", _P), ("ld_tok", _I64), ("step_dev", _P), ("next", _P),
    ]


class IWhisperError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"i_whisper_b200: CUDA library {LIB_PATH} is not built; run `python -m i_whisper_b200.build`")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = C.c_int
    lib.iw_last_error.argtypes = []
    lib.iw_last_error.restype = C.c_char_p
    return lib


LIB = _load()


def last_error() -> str:
    return LIB.iw_last_error().decode("utf-8", "replace")


def check(rc: int):
    if rc == IW_OK:
        return
    msg = last_error()
    if rc == IW_EVALUE:
        raise ValueError(msg)
    if rc == IW_EOVERFLOW:
        raise OverflowError(msg)
    raise IWhisperError(msg)


def call(name: str, *args):
    check(getattr(LIB, name)(*args))


def device_status(clear: bool = True) -> int:
    v = C.c_uint32(0)
    check(LIB.iw_device_status(C.byref(v), 1 if clear else 0))
    return int(v.value)
