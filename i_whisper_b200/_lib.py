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

_P = C.c_void_p
_I64 = C.c_int64
_U8, _I8, _U16, _U32, _I32 = C.c_uint8, C.c_int8, C.c_uint16, C.c_uint32, C.c_int32

# name -> argtypes (restype is always c_int)
SIGNATURES = {
    "iw_linear8": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear8_accum": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear32": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "iw_linear32_residual15": [_P, _P, _P, _P, _P, _P, _P, _U16, _P, _I64, _I64, _I64, _P],
    "iw_residual15": [_P, _P, _U16, _P, _I64, _P],
    "iw_layernorm32": [_P, _P, _P, _U8, _I8, _U32, _I8, _P, _I64, _I64, _P],
    "iw_layernorm32_stats": [_P, _P, _P, _P, _I64, _I64, _P],
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
}


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
    raise IWhisperError(msg)


def call(name: str, *args):
    check(getattr(LIB, name)(*args))


def device_status(clear: bool = True) -> int:
    v = C.c_uint32(0)
    check(LIB.iw_device_status(C.byref(v), 1 if clear else 0))
    return int(v.value)
