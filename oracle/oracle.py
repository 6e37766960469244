"""CPU oracle for the I-Whisper integer hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker that the CUDA path is compared against. It is
imported only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / ``--impl reference`` legs, never by the product package.

Two interchangeable kernel libraries sit under it, both loaded with ctypes:

* ``port`` -- ``oracle/libiw_oracle.so``, the C restatement in ``iw_oracle.c``
  (each function cites the reference kernel it restates);
* ``ref``  -- ``oracle/_ref/libiw_ref.so``, the reference's own scalar C++
  kernels (``i_whisper/kernels/csrc/*/*_scalar.cpp``) compiled in place by
  ``oracle/Makefile`` with ``ref_shim.cpp``; present only where the reference
  checkout was available at build time.

On top of the kernels, :func:`encoder_forward`, :func:`decoder_forward` and
:func:`greedy_decode` restate the module dataflow of
``i_whisper/model_int.py`` (AudioEncoder_int.forward :1260-1316,
ResidualAttentionBlock_int.forward :1112-1177, MultiHeadAttention_int
:713-1042, TextDecoder_int.forward :1398-1484) and the greedy loop of
``i_whisper/decoding.py`` (:684-712, filters :426-510, GreedyDecoder :280-296)
over a state dict keyed exactly like ``Whisper_int.state_dict()``.

Parity is pinned: the kernels against the reference's compiled scalar
kernels and its own kernel test suite, the dataflow and greedy loop against
golden digests and tokens that the reference's Whisper_int and DecodingTask
produced (tests/golden), and the filter chain against the reference
DecodingTask's own logit filters.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(_HERE, "libiw_oracle.so")
REF_PATH = os.path.join(_HERE, "_ref", "libiw_ref.so")

_P = C.c_void_p
_I64 = C.c_int64

_SIGS = {
    "linear8_accum": ([_P, _P, _P, _P, _P, _I64, _I64, _I64], None),
    "linear8": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64], None),
    "linear32": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64], None),
    "residual15": ([_P, _P, C.c_uint16, _P, _I64], None),
    "layernorm32": ([_P, _P, _P, C.c_uint8, C.c_int8, C.c_uint32, C.c_int8, C.c_uint32, _P, _I64, _I64], C.c_int),
    "layernorm32_stats": ([_P, _P, _P, _P, _I64, _I64], C.c_int),
    "layernorm64": ([_P, _P, _P, C.c_uint8, C.c_int8, C.c_uint32, C.c_int8, C.c_uint32, C.c_int32, _P, _I64, _I64],
                    C.c_int),
    "layernorm64_stats": ([_P, _P, _P, _I64, _I64], C.c_int),
    "fisr_vec": ([_P, _P, _I64, C.c_uint32], None),
    "gelu": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64], None),
    "qk": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64], None),
    "qk_requant_rowmax": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, C.c_uint8, C.c_int32], None),
    "shift_exp": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, C.c_int32], None),
    "pv": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64], None),
    "pv_norm_requant": ([_P, _P, _P, C.c_uint8, C.c_int8, C.c_uint32, _P, _I64, _I64, _I64, _I64, _I64], C.c_int),
    "conv1d_accum": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64], None),
    "conv1d": ([_P, _P, _P, C.c_uint32, C.c_int8, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64], None),
    "add_requant15": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64], None),
    "classifier_accum": ([_P, _P, _P, _I64, _I64, _I64], None),
    "classifier": ([_P, _P, C.c_uint32, C.c_int8, _P, _I64, _I64, _I64], None),
}


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(np.asarray(a), dtype=dtype)


class OracleLib:
    """numpy-level wrapper with the reference ``_C`` op semantics."""

    def __init__(self, kind: str = "port"):
        path = PORT_PATH if kind == "port" else REF_PATH
        if not os.path.exists(path):
            raise FileNotFoundError(f"oracle library {path} is not built (make -C oracle {'' if kind == 'port' else 'ref'})")
        self.kind = kind
        self.path = path
        self.lib = C.CDLL(path)
        prefix = "iwo_" if kind == "port" else "iwr_"
        self.fn = {}
        for name, (args, res) in _SIGS.items():
            f = getattr(self.lib, prefix + name)
            f.argtypes = args
            f.restype = res
            self.fn[name] = f
        if kind == "port":
            self.lib.iwo_set_threads.argtypes = [C.c_int]

    def set_threads(self, n: int):
        if self.kind == "port":
            self.lib.iwo_set_threads(int(n))

    # ---- linear ---------------------------------------------------------
    def linear8_accum(self, x, w, bias=None, wz=None):
        x = _c(x, np.int8); w = _c(w, np.int8)
        K = x.shape[-1]; N = w.shape[0]; M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.int32)
        self.fn["linear8_accum"](_ptr(x), _ptr(w), _ptr(_c(bias, np.int32)), _ptr(_c(wz, np.int8)), _ptr(y), M, K, N)
        return y

    def linear8(self, x, w, bias, wz, mult, shift):
        x = _c(x, np.int8); w = _c(w, np.int8)
        K = x.shape[-1]; N = w.shape[0]; M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.int8)
        self.fn["linear8"](_ptr(x), _ptr(w), _ptr(_c(bias, np.int32)), _ptr(_c(wz, np.int8)),
                           _ptr(_c(mult, np.uint32)), _ptr(_c(shift, np.int8)), _ptr(y), M, K, N)
        return y

    def linear32(self, x, w, bias, wz, mult, shift):
        x = _c(x, np.int8); w = _c(w, np.int8)
        K = x.shape[-1]; N = w.shape[0]; M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.int32)
        self.fn["linear32"](_ptr(x), _ptr(w), _ptr(_c(bias, np.int32)), _ptr(_c(wz, np.int8)),
                            _ptr(_c(mult, np.uint32)), _ptr(_c(shift, np.int8)), _ptr(y), M, K, N)
        return y

    def linear8_requant(self, acc, mult, shift):
        """linear8_requant_scalar (linear8_scalar.cpp:130-150): int32
        rrs(mulh(acc, m[n]), (u32)s[n]), no clamp. Port library only."""
        acc = _c(acc, np.int32)
        N = acc.shape[-1]
        y = np.empty(acc.shape, np.int32)
        f = self.lib.iwo_linear8_requant
        f.argtypes, f.restype = [_P, _P, _P, _P, _I64, _I64], None
        f(_ptr(acc), _ptr(_c(mult, np.uint32)), _ptr(_c(shift, np.int8)), _ptr(y), acc.size // N, N)
        return y

    def rounding_rshift(self, x, shift):
        """fixedpoint::rounding_rshift (common/fixedpoint.h:47-87) elementwise.
        Port library only."""
        x = _c(x, np.int32)
        f = self.lib.iwo_rounding_rshift
        f.argtypes, f.restype = [C.c_int32, C.c_uint32], C.c_int32
        return np.array([f(int(v), int(shift)) for v in x.reshape(-1)], np.int32).reshape(x.shape)

    def residual15(self, branch, residual, mult):
        b = _c(branch, np.int32); r = _c(residual, np.int16)
        y = np.empty(r.shape, np.int16)
        self.fn["residual15"](_ptr(b), _ptr(r), int(np.asarray(mult).reshape(-1)[0]), _ptr(y), r.size)
        return y

    def layernorm32(self, x, gamma, beta, ln_m, ln_s, out_m, out_s, rsqrt_offset=13):
        x = _c(x, np.int16); d = x.shape[-1]
        y = np.empty(x.shape, np.int8)
        rc = self.fn["layernorm32"](_ptr(x), _ptr(_c(gamma, np.int8)), _ptr(_c(beta, np.int32)),
                                    int(np.asarray(ln_m).reshape(-1)[0]), int(np.asarray(ln_s).reshape(-1)[0]),
                                    int(np.asarray(out_m).reshape(-1)[0]), int(np.asarray(out_s).reshape(-1)[0]),
                                    rsqrt_offset, _ptr(y), x.size // d, d)
        if rc != 0:
            raise ValueError(f"unsupported LayerNorm hidden size: {d}")
        return y

    def layernorm64(self, x, gamma, beta, ln_m, ln_s, out_m, out_s, rsqrt_offset=15, additional_offset=2):
        """LayerNorm64 (layernorm_torch.cpp:446-460 fixes rsqrt_offset 15 and
        additional_offset 2); OverflowError when a row's variance does not
        fit INT32, as the reference."""
        x = _c(x, np.int16); d = x.shape[-1]
        y = np.empty(x.shape, np.int8)
        rc = self.fn["layernorm64"](_ptr(x), _ptr(_c(gamma, np.int8)), _ptr(_c(beta, np.int32)),
                                    int(np.asarray(ln_m).reshape(-1)[0]), int(np.asarray(ln_s).reshape(-1)[0]),
                                    int(np.asarray(out_m).reshape(-1)[0]), int(np.asarray(out_s).reshape(-1)[0]),
                                    rsqrt_offset, additional_offset, _ptr(y), x.size // d, d)
        if rc == -2:
            raise OverflowError("LayerNorm64 variance does not fit INT32")
        if rc != 0:
            raise ValueError(f"unsupported LayerNorm hidden size: {d}")
        return y

    def layernorm64_stats(self, x):
        x = _c(x, np.int16); d = x.shape[-1]; rows = x.size // d
        mean = np.empty(rows, np.int32); var = np.empty(rows, np.int64)
        rc = self.fn["layernorm64_stats"](_ptr(x), _ptr(mean), _ptr(var), rows, d)
        if rc != 0:
            raise ValueError(f"unsupported LayerNorm hidden size: {d}")
        return mean, var

    def with_layernorm(self, variant: str) -> "OracleLib":
        """A view of this library whose model dataflow uses LayerNorm32 ("32",
        the reference default) or the LayerNorm64 research variant ("64",
        backend "scalar64" of LayerNorm_int, model_int.py:252-287)."""
        import copy
        v = copy.copy(self)
        v.ln_variant = variant
        return v

    def layernorm32_stats(self, x):
        x = _c(x, np.int16); d = x.shape[-1]; rows = x.size // d
        mean = np.empty(rows, np.int32); var = np.empty(rows, np.int32); rs = np.empty(rows, np.int32)
        rc = self.fn["layernorm32_stats"](_ptr(x), _ptr(mean), _ptr(var), _ptr(rs), rows, d)
        if rc != 0:
            raise ValueError(f"unsupported LayerNorm hidden size: {d}")
        return mean, var, rs

    def fisr(self, x, offset):
        x = _c(x, np.int32)
        y = np.empty(x.shape, np.int32)
        self.fn["fisr_vec"](_ptr(x), _ptr(y), x.size, offset)
        return y

    def gelu(self, x, lut, mi, si, mo, so):
        x = _c(x, np.int8)
        mi = _c(mi, np.uint8).reshape(-1); mo = _c(mo, np.uint8).reshape(-1)
        y = np.empty(x.shape, np.int8)
        self.fn["gelu"](_ptr(x), _ptr(_c(lut, np.uint8)), _ptr(mi), _ptr(_c(si, np.int8)), _ptr(mo),
                        _ptr(_c(so, np.int8)), _ptr(y), x.size, x.shape[-1], mi.size, mo.size)
        return y

    # ---- attention ------------------------------------------------------
    def qk(self, q, k):
        q = _c(q, np.int8); k = _c(k, np.int8)
        B, H, Tq, D = q.shape; Tk = k.shape[2]
        y = np.empty((B, H, Tq, Tk), np.int32)
        self.fn["qk"](_ptr(q), _ptr(k), _ptr(y), B, H, Tq, Tk, D)
        return y

    def qk_requant_rowmax(self, q, k, mask, mult, shift):
        q = _c(q, np.int8); k = _c(k, np.int8)
        B, H, Tq, D = q.shape; Tk = k.shape[2]
        qk = np.empty((B, H, Tq, Tk), np.int16); rm = np.empty((B, H, Tq, 1), np.int16)
        self.fn["qk_requant_rowmax"](_ptr(q), _ptr(k), _ptr(_c(mask, np.uint8)), _ptr(qk), _ptr(rm),
                                     B, H, Tq, Tk, D, int(np.asarray(mult).reshape(-1)[0]),
                                     int(np.asarray(shift).reshape(-1)[0]))
        return qk, rm

    def shift_exp(self, x, rmax1, mask, frac_bits):
        x = _c(x, np.int16); B, H, Tq, Tk = x.shape
        p = np.empty(x.shape, np.uint8); rs = np.empty((B, H, Tq, 1), np.int32)
        self.fn["shift_exp"](_ptr(x), _ptr(_c(rmax1, np.int16)), _ptr(_c(mask, np.uint8)), _ptr(p), _ptr(rs),
                             B, H, Tq, Tk, int(np.asarray(frac_bits).reshape(-1)[0]))
        return p, rs

    def pv(self, p, vt):
        p = _c(p, np.uint8); vt = _c(vt, np.int8)
        B, H, Tq, Tk = p.shape; D = vt.shape[2]
        y = np.empty((B, H, Tq, D), np.int32)
        self.fn["pv"](_ptr(p), _ptr(vt), _ptr(y), B, H, Tq, Tk, D)
        return y

    def pv_norm_requant(self, p, vt, rowsum, av_m, av_s, rsqrt_offset=16):
        p = _c(p, np.uint8); vt = _c(vt, np.int8)
        B, H, Tq, Tk = p.shape; D = vt.shape[2]
        y = np.empty((B, Tq, H * D), np.int8)
        rc = self.fn["pv_norm_requant"](_ptr(p), _ptr(vt), _ptr(_c(rowsum, np.int32)),
                                        int(np.asarray(av_m).reshape(-1)[0]), int(np.asarray(av_s).reshape(-1)[0]),
                                        rsqrt_offset, _ptr(y), B, H, Tq, Tk, D)
        if rc != 0:
            raise ValueError("row_sum must be non-negative")
        return y

    # ---- conv / add / classifier ------------------------------------------
    def conv1d_accum(self, x, w, bias, stride, pad):
        x = _c(x, np.int8); w = _c(w, np.int8)
        B, Cin, Tin = x.shape; Cout = w.shape[0]; K = w.shape[1] // Cin
        Tout = (Tin + 2 * pad - K) // stride + 1
        y = np.empty((B, Cout, Tout), np.int32)
        self.fn["conv1d_accum"](_ptr(x), _ptr(w), _ptr(_c(bias, np.int32)), _ptr(y), B, Cin, Tin, Cout, K, stride, pad)
        return y

    def conv1d(self, x, w, bias, mult, shift, stride, pad):
        x = _c(x, np.int8); w = _c(w, np.int8)
        B, Cin, Tin = x.shape; Cout = w.shape[0]; K = w.shape[1] // Cin
        Tout = (Tin + 2 * pad - K) // stride + 1
        y = np.empty((B, Cout, Tout), np.int8)
        self.fn["conv1d"](_ptr(x), _ptr(w), _ptr(_c(bias, np.int32)), int(np.asarray(mult).reshape(-1)[0]),
                          int(np.asarray(shift).reshape(-1)[0]), _ptr(y), B, Cin, Tin, Cout, K, stride, pad)
        return y

    def add_requant15(self, x, addend, mult, shift):
        x = _c(x, np.int8); B, T, Cc = x.shape
        m = _c(mult, np.uint16).reshape(-1); s = _c(shift, np.int8).reshape(-1)
        y = np.empty(x.shape, np.int16)
        self.fn["add_requant15"](_ptr(x), _ptr(_c(addend, np.int8)), _ptr(m), _ptr(s), _ptr(y), B, T, Cc, m.size, s.size)
        return y

    def classifier_accum(self, x, w):
        x = _c(x, np.int8); w = _c(w, np.int8)
        K = x.shape[-1]; N = w.shape[0]; M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.int32)
        self.fn["classifier_accum"](_ptr(x), _ptr(w), _ptr(y), M, K, N)
        return y

    def classifier(self, x, w, mult, shift):
        x = _c(x, np.int8); w = _c(w, np.int8)
        K = x.shape[-1]; N = w.shape[0]; M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.int8)
        self.fn["classifier"](_ptr(x), _ptr(w), int(np.asarray(mult).reshape(-1)[0]),
                              int(np.asarray(shift).reshape(-1)[0]), _ptr(y), M, K, N)
        return y


_LIBS: Dict[str, OracleLib] = {}


def lib(kind: str = "port") -> OracleLib:
    if kind not in _LIBS:
        _LIBS[kind] = OracleLib(kind)
    return _LIBS[kind]


# ---------------------------------------------------------------------------
# Model-level dataflow (model_int.py), over a Whisper_int-style state dict.
# ---------------------------------------------------------------------------

@dataclass
class Dims:
    n_mels: int
    n_audio_ctx: int
    n_audio_state: int
    n_audio_head: int
    n_audio_layer: int
    n_vocab: int
    n_text_ctx: int
    n_text_state: int
    n_text_head: int
    n_text_layer: int


def _lin8(L, P, pre, x):
    return L.linear8(x, P[pre + ".weight"], P.get(pre + ".bias"), P.get(pre + ".wgt_zeros"),
                     P[pre + ".req_multiplier"], P[pre + ".req_shiftmount"])


def _lin32(L, P, pre, x):
    return L.linear32(x, P[pre + ".weight"], P.get(pre + ".bias"), P.get(pre + ".wgt_zeros"),
                      P[pre + ".req_multiplier"], P[pre + ".req_shiftmount"])


def _ln(L, P, pre, x):
    if getattr(L, "ln_variant", "32") == "64":
        return L.layernorm64(x, P[pre + ".weight"], P.get(pre + ".bias"), P[pre + ".ln_req_multiplier"],
                             P[pre + ".ln_req_shiftmount"], P[pre + ".out_req_multiplier"],
                             P[pre + ".out_req_shiftmount"])
    return L.layernorm32(x, P[pre + ".weight"], P.get(pre + ".bias"), P[pre + ".ln_req_multiplier"],
                         P[pre + ".ln_req_shiftmount"], P[pre + ".out_req_multiplier"],
                         P[pre + ".out_req_shiftmount"], 13)


def _gelu(L, P, pre, x):
    return L.gelu(x, P[pre + ".lut"], P[pre + ".luti_req_multiplier"], P[pre + ".luti_req_shiftmount"],
                  P[pre + ".luto_req_multiplier"], P[pre + ".luto_req_shiftmount"])


def attention_core(L, P, pre, q, k, v, n_head, mask=None):
    """MultiHeadAttention_int.qkv_attention (model_int.py:774-1042):
    q [B,Tq,d], k/v [B,Tk,d] INT8 -> INT8 [B,Tq,d]."""
    B, Tq, d = q.shape
    Tk = k.shape[1]
    D = d // n_head
    q4 = q.reshape(B, Tq, n_head, D).transpose(0, 2, 1, 3)
    k4 = k.reshape(B, Tk, n_head, D).transpose(0, 2, 1, 3)
    vt = v.reshape(B, Tk, n_head, D).transpose(0, 2, 3, 1)
    am = None
    if mask is not None:
        off = Tk - Tq
        am = np.ascontiguousarray(mask[off:off + Tq, :Tk])
    qk, rm = L.qk_requant_rowmax(q4, k4, am, P[pre + ".qk_req_multiplier"], P[pre + ".qk_req_shiftmount"])
    p, rs = L.shift_exp(qk, rm, am, P[pre + ".qk_frac_bits"])
    return L.pv_norm_requant(p, vt, rs, P[pre + ".av_req_multiplier"], P[pre + ".av_req_shiftmount"], 16)


def block_forward(L, P, pre, x, n_head, xa=None, mask=None, cache=None, trace=None):
    """ResidualAttentionBlock_int.forward (model_int.py:1112-1177). ``cache``
    is a dict holding this block's self K/V and cross K/V (decoder)."""
    h = _ln(L, P, pre + ".attn_ln", x)
    q = _lin8(L, P, pre + ".attn.query", h)
    k = _lin8(L, P, pre + ".attn.key", h)
    v = _lin8(L, P, pre + ".attn.value", h)
    if cache is not None:
        if "k" in cache:
            k = np.concatenate([cache["k"], k], axis=1)
            v = np.concatenate([cache["v"], v], axis=1)
        cache["k"], cache["v"] = k, v
    a = attention_core(L, P, pre + ".attn", q, k, v, n_head, mask)
    if trace is not None:
        trace[pre + ".attn.wv"] = a
    br = _lin32(L, P, pre + ".attn.out", a)
    x = L.residual15(br, x, P[pre + ".attn_res_req_multiplier"])
    if xa is not None:
        h = _ln(L, P, pre + ".cross_attn_ln", x)
        q = _lin8(L, P, pre + ".cross_attn.query", h)
        if cache is not None and "ck" in cache:
            ck, cv = cache["ck"], cache["cv"]
        else:
            ck = _lin8(L, P, pre + ".cross_attn.key", xa)
            cv = _lin8(L, P, pre + ".cross_attn.value", xa)
            if cache is not None:
                cache["ck"], cache["cv"] = ck, cv
        a = attention_core(L, P, pre + ".cross_attn", q, ck, cv, n_head, None)
        br = _lin32(L, P, pre + ".cross_attn.out", a)
        x = L.residual15(br, x, P[pre + ".cross_attn_res_req_multiplier"])
    h = _ln(L, P, pre + ".mlp_ln", x)
    h = _lin8(L, P, pre + ".mlp.0", h)
    h = _gelu(L, P, pre + ".mlp.1", h)
    br = _lin32(L, P, pre + ".mlp.2", h)
    x = L.residual15(br, x, P[pre + ".mlp_res_req_multiplier"])
    if trace is not None:
        trace[pre] = x
    return x


def encoder_forward(P, dims: Dims, mel_i8: np.ndarray, kind="port", trace=None, layernorm="32") -> np.ndarray:
    """AudioEncoder_int.forward (model_int.py:1260-1316) on an INT8 mel
    [B,n_mels,2*n_audio_ctx] -> INT8 [B,n_audio_ctx,d]; layernorm "64" puts
    every LayerNorm_int on its LayerNorm64 backend."""
    L = lib(kind).with_layernorm(layernorm)
    e = "encoder"
    x = L.conv1d(mel_i8, P[e + ".conv1.weight"], P.get(e + ".conv1.bias"), P[e + ".conv1.req_multiplier"],
                 P[e + ".conv1.req_shiftmount"], 1, 1)
    x = _gelu(L, P, e + ".gelu1", x)
    x = L.conv1d(x, P[e + ".conv2.weight"], P.get(e + ".conv2.bias"), P[e + ".conv2.req_multiplier"],
                 P[e + ".conv2.req_shiftmount"], 2, 1)
    x = np.ascontiguousarray(x.transpose(0, 2, 1))
    x = _gelu(L, P, e + ".gelu2", x)
    if trace is not None:
        trace["encoder.stem"] = x
    x = L.add_requant15(x, P[e + ".positional_embedding"], P[e + ".req_multiplier"], P[e + ".req_shiftmount"])
    if trace is not None:
        trace["encoder.pos"] = x
    for i in range(dims.n_audio_layer):
        x = block_forward(L, P, f"{e}.blocks.{i}", x, dims.n_audio_head, trace=trace)
    return _ln(L, P, e + ".ln_post", x)


def decoder_forward(P, dims: Dims, tokens: np.ndarray, xa: np.ndarray, caches: List[dict], offset: int,
                    kind="port", layernorm="32") -> np.ndarray:
    """TextDecoder_int.forward (model_int.py:1398-1484) with the KV cache
    hooks of Whisper_int.install_kv_cache_hooks (:1587-1618): INT8 logits
    [B,T,V] (before the float dequantisation)."""
    L = lib(kind).with_layernorm(layernorm)
    d = "decoder"
    emb = P[d + ".token_embedding.weight"][tokens]
    pe = P[d + ".positional_embedding"][offset:offset + tokens.shape[-1]]
    x = L.add_requant15(emb, pe, P[d + ".req_multiplier"].astype(np.uint16), P[d + ".req_shiftmount"])
    mask = np.triu(np.ones((dims.n_text_ctx, dims.n_text_ctx), np.uint8), 1)
    for i in range(dims.n_text_layer):
        x = block_forward(L, P, f"{d}.blocks.{i}", x, dims.n_text_head, xa=xa, mask=mask, cache=caches[i])
    x = _ln(L, P, d + ".ln", x)
    return L.classifier(x, P[d + ".token_embedding.weight"], P[d + ".clf_req_multiplier"], P[d + ".clf_req_shiftmount"])


@dataclass
class DecodeTokens:
    """Special-token ids used by the greedy loop (tokenizer.py constants)."""
    sot: int
    eot: int
    sot_sequence: Sequence[int]
    no_timestamps: int
    timestamp_begin: int
    blank: Sequence[int]
    suppress: Sequence[int]
    max_initial_timestamp_index: Optional[int] = 50


def apply_filters_torch(logits, tokens, tk: DecodeTokens, sample_begin: int):
    """SuppressBlank, SuppressTokens and ApplyTimestampRules of
    decoding.py:426-510, applied in place to float32 torch logits [B,V]."""
    import torch
    import torch.nn.functional as F
    if tokens.shape[1] == sample_begin:
        logits[:, list(tk.blank) + [tk.eot]] = -np.inf
    logits[:, list(tk.suppress)] = -np.inf
    logits[:, tk.no_timestamps] = -np.inf
    tb = tk.timestamp_begin
    for k in range(tokens.shape[0]):
        sampled = tokens[k, sample_begin:]
        seq = sampled.tolist()
        last_ts = len(seq) >= 1 and seq[-1] >= tb
        pen_ts = len(seq) < 2 or seq[-2] >= tb
        if last_ts:
            if pen_ts:
                logits[k, tb:] = -np.inf
            else:
                logits[k, :tk.eot] = -np.inf
        ts = sampled[sampled.ge(tb)]
        if ts.numel() > 0:
            last = ts[-1] if (last_ts and not pen_ts) else ts[-1] + 1
            logits[k, tb:last] = -np.inf
    if tokens.shape[1] == sample_begin:
        logits[:, :tb] = -np.inf
        if tk.max_initial_timestamp_index is not None:
            logits[:, tb + tk.max_initial_timestamp_index + 1:] = -np.inf
    logprobs = F.log_softmax(logits.float(), dim=-1)
    for k in range(tokens.shape[0]):
        ts_lp = logprobs[k, tb:].logsumexp(dim=-1)
        max_text = logprobs[k, :tb].max()
        if ts_lp > max_text:
            logits[k, :tb] = -np.inf


def greedy_decode(P, dims: Dims, xa: np.ndarray, tk: DecodeTokens, sample_len: int, kind="port",
                  stop_when_done=True, layernorm="32") -> np.ndarray:
    """DecodingTask._main_loop with GreedyDecoder (decoding.py:684-712,
    280-296): returns the token matrix [B, len(sot_sequence)+steps]."""
    import torch
    B = xa.shape[0]
    tokens = torch.tensor([list(tk.sot_sequence)] * B, dtype=torch.int64)
    sample_begin = tokens.shape[1]
    caches = [dict() for _ in range(dims.n_text_layer)]
    alpha = float(np.asarray(P["decoder.act_logits_alpha"]).reshape(-1)[0])
    offset = 0
    for i in range(sample_len):
        inp = tokens.numpy() if i == 0 else tokens[:, -1:].numpy()
        logits8 = decoder_forward(P, dims, inp, xa, caches, offset, kind, layernorm)
        offset += inp.shape[1]
        logits = torch.from_numpy(logits8[:, -1].astype(np.float32)).div(torch.tensor([alpha], dtype=torch.float32))
        apply_filters_torch(logits, tokens, tk, sample_begin)
        nxt = logits.argmax(dim=-1)
        nxt[tokens[:, -1] == tk.eot] = tk.eot
        tokens = torch.cat([tokens, nxt[:, None]], dim=-1)
        if stop_when_done and bool((tokens[:, -1] == tk.eot).all()):
            break
        if tokens.shape[-1] > dims.n_text_ctx:
            break
    return tokens.numpy()
