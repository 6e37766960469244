"""A CPU stand-in for the per-op C ABI of libiwhisper_b200.so (test helper).

Each entry below has the name and the argument list of an ``iw_*`` function
of include/iwhisper_b200.h, applies the same argument checks as
i_whisper_b200/csrc/capi.cu (same status codes and messages), and computes
its result with the oracle's C restatement (oracle/iw_oracle.c) on the same
raw host pointers. With ``install(monkeypatch)`` the torch-facing mirror
``i_whisper_b200.ops`` runs on CPU tensors end to end: its own argument
checks, output allocation and pointer plumbing, with the oracle in place of
the GPU kernels. This lets the host layer be tested without a GPU, including
by the reference's own kernel tests. It is never part of the product path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from i_whisper_b200 import _lib
from oracle import oracle as O

LN_WIDTHS = (384, 512, 768, 1024, 1280)


class EmulatedError(Exception):
    def __init__(self, rc, msg):
        super().__init__(msg)
        self.rc = rc


def _fail(rc, msg):
    raise EmulatedError(rc, msg)


def _view(ptr, n, dtype):
    dt = np.dtype(dtype)
    if n == 0:
        return np.zeros(0, dt)
    return np.frombuffer((C.c_char * (n * dt.itemsize)).from_address(ptr), dtype=dt, count=n)


class CapiEmulator:
    def __init__(self):
        self.L = O.lib("port")
        self.f = dict(self.L.fn)
        lib = self.L.lib
        lib.iwo_linear8_requant.argtypes = [C.c_void_p] * 4 + [C.c_int64] * 2
        lib.iwo_linear8_requant.restype = None
        lib.iwo_rounding_rshift.argtypes = [C.c_int32, C.c_uint32]
        lib.iwo_rounding_rshift.restype = C.c_int32
        self.f["linear8_requant"] = lib.iwo_linear8_requant
        self.rrs = lib.iwo_rounding_rshift

    # -- linear ---------------------------------------------------------------
    @staticmethod
    def _linear_shape(name, M, K, N):
        if M < 0 or N <= 0:
            _fail(_lib.IW_EINVAL, f"{name}: invalid shape M={M} N={N}")
        if K <= 0:
            _fail(_lib.IW_EINVAL, f"{name}: x.size(-1) must be greater than 0")
        return M > 0

    def iw_linear8(self, x, w, b, wz, m, s, y, M, K, N, st):
        if self._linear_shape("iw_linear8", M, K, N):
            self.f["linear8"](x, w, b, wz, m, s, y, M, K, N)

    def iw_linear8_accum(self, x, w, b, wz, y, M, K, N, st):
        if self._linear_shape("iw_linear8_accum", M, K, N):
            self.f["linear8_accum"](x, w, b, wz, y, M, K, N)

    def iw_linear8_requant(self, acc, m, s, y, M, N, st):
        if M < 0 or N <= 0:
            _fail(_lib.IW_EINVAL, f"iw_linear8_requant: invalid shape M={M} N={N}")
        if not m or not s:
            _fail(_lib.IW_EINVAL, "iw_linear8_requant: multiplier and shift are required")
        self.f["linear8_requant"](acc, m, s, y, M, N)

    def iw_rounding_rshift(self, x, shift, y, n, st):
        if n < 0:
            _fail(_lib.IW_EINVAL, "iw_rounding_rshift: invalid numel")
        X, Y = _view(x, n, np.int32), _view(y, n, np.int32)
        Y[:] = [self.rrs(int(v), shift) for v in X]

    def iw_linear32(self, x, w, b, wz, m, s, y, M, K, N, st):
        if self._linear_shape("iw_linear32", M, K, N):
            self.f["linear32"](x, w, b, wz, m, s, y, M, K, N)

    def iw_linear32_residual15(self, x, w, b, wz, m, s, res, res_m, y, M, K, N, st):
        if not res:
            _fail(_lib.IW_EINVAL, "iw_linear32_residual15: residual is required")
        if self._linear_shape("iw_linear32_residual15", M, K, N):
            br = np.empty(M * N, np.int32)
            self.f["linear32"](x, w, b, wz, m, s, br.ctypes.data, M, K, N)
            self.f["residual15"](br.ctypes.data, res, res_m, y, M * N)

    def iw_residual15(self, br, res, m, y, n, st):
        if n < 0:
            _fail(_lib.IW_EINVAL, "iw_residual15: invalid numel")
        self.f["residual15"](br, res, m, y, n)

    # -- layernorm --------------------------------------------------------------
    @staticmethod
    def _ln_width(d):
        if d not in LN_WIDTHS:
            _fail(_lib.IW_EINVAL, f"unsupported LayerNorm hidden size: {d}")

    def iw_layernorm32(self, x, g, b, lm, ls, om, os_, y, rows, d, st):
        self._ln_width(d)
        if rows < 0 or rows > 2 ** 31 - 1:
            _fail(_lib.IW_EINVAL, "iw_layernorm32: invalid row count")
        self.f["layernorm32"](x, g, b, lm, ls, om, os_, 13, y, rows, d)

    def iw_layernorm64(self, x, g, b, lm, ls, om, os_, y, rows, d, st):
        self._ln_width(d)
        if rows < 0 or rows > 2 ** 31 - 1:
            _fail(_lib.IW_EINVAL, "iw_layernorm64: invalid row count")
        if self.f["layernorm64"](x, g, b, lm, ls, om, os_, 15, 2, y, rows, d) == -2:
            _fail(_lib.IW_EOVERFLOW, "LayerNorm64 variance does not fit INT32")

    def iw_layernorm32_stats(self, x, mean, var, rsh, rows, d, st):
        self._ln_width(d)
        self.f["layernorm32_stats"](x, mean, var, rsh, rows, d)

    def iw_layernorm64_stats(self, x, mean, var, rows, d, st):
        self._ln_width(d)
        if rows < 0 or rows > 2 ** 31 - 1:
            _fail(_lib.IW_EINVAL, "iw_layernorm64_stats: invalid row count")
        self.f["layernorm64_stats"](x, mean, var, rows, d)

    def iw_layernorm32_rsqrt(self, var, inv, n, st):
        if n > 0 and (_view(var, n, np.int32) < 0).any():
            _fail(_lib.IW_EINVAL, "input must be non-negative")
        self.f["fisr_vec"](var, inv, n, 13)

    # -- gelu -------------------------------------------------------------------
    def iw_gelu(self, x, lut, mi, si, mo, so, y, numel, channels, ni, no, st):
        if channels <= 0 and numel > 0:
            _fail(_lib.IW_EINVAL, "iw_gelu: input must have at least one dimension")
        if not (ni == 1 or ni == channels):
            _fail(_lib.IW_EINVAL, "luti parameters must be scalar or match input.size(-1)")
        if not (no == 1 or no == channels):
            _fail(_lib.IW_EINVAL, "luto parameters must be scalar or match input.size(-1)")
        self.f["gelu"](x, lut, mi, si, mo, so, y, numel, channels, ni, no)

    # -- attention stages -------------------------------------------------------
    def iw_qk_requant_rowmax(self, q, k, mask, m, s, qk, rm, B, H, Tq, Tk, D, st):
        if min(B, H, Tq, Tk, D) < 0:
            _fail(_lib.IW_EINVAL, "iw_qk_requant_rowmax: invalid shape")
        self.f["qk_requant_rowmax"](q, k, mask, qk, rm, B, H, Tq, Tk, D, m, s)

    def iw_shift_exp(self, x, rm, mask, fb, p, rs, B, H, Tq, Tk, st):
        if not (0 < fb < 14):
            _fail(_lib.IW_EINVAL, "frac_bits must be in [1, 14)")
        self.f["shift_exp"](x, rm, mask, p, rs, B, H, Tq, Tk, fb)

    def iw_pv_norm_requant(self, p, v, rs, am, as_, off, y, B, H, Tq, Tk, D, st):
        if not (0 <= off <= 29):
            _fail(_lib.IW_EINVAL, "rsqrt_offset must be in [0,29]")
        n = B * H * Tq
        if n > 0 and (_view(rs, n, np.int32) < 0).any():
            _fail(_lib.IW_EVALUE, "row_sum must be non-negative")
        self.f["pv_norm_requant"](p, v, rs, am, as_, off, y, B, H, Tq, Tk, D)

    # -- conv stem, add-requant, classifier ---------------------------------------
    def iw_conv1d(self, x, w, b, m, s, stride, pad, y, B, Cin, Tin, Cout, K, st):
        for cond, msg in ((stride <= 0, "stride must be positive"), (pad < 0, "padding must be non-negative"),
                          (Cin <= 0, "input channel count must be positive"),
                          (Tin <= 0, "input length must be positive"),
                          (Cout <= 0, "output channel count must be positive"), (K <= 0, "kernel size must be positive"),
                          (Tin + 2 * pad - K < 0, "invalid Conv1d geometry: output length would be non-positive")):
            if cond:
                _fail(_lib.IW_EINVAL, msg)
        if B > 0:
            self.f["conv1d"](x, w, b, m, s, y, B, Cin, Tin, Cout, K, stride, pad)

    def iw_im2col(self, x, out, B, Cin, Tin, K, stride, pad, Tout, ldo, channels_last, st):
        if ldo < Cin * K:
            _fail(_lib.IW_EINVAL, "iw_im2col: ldo < Cin*K")
        X = _view(x, B * Cin * Tin, np.int8)
        X = X.reshape(B, Tin, Cin).transpose(0, 2, 1) if channels_last else X.reshape(B, Cin, Tin)
        Y = _view(out, B * Tout * ldo, np.int8).reshape(B, Tout, ldo)
        Y[:] = 0
        for t in range(Tout):
            for k in range(K):
                pos = t * stride - pad + k
                if 0 <= pos < Tin:
                    Y[:, t, k:Cin * K:K] = X[:, :, pos]

    @staticmethod
    def _requant15_counts(Cc, nm, ns):
        if not (nm == 1 or nm == Cc):
            _fail(_lib.IW_EINVAL, "multiplier must contain 1 or C elements")
        if not (ns == 1 or ns == Cc):
            _fail(_lib.IW_EINVAL, "shift must contain 1 or C elements")

    def iw_add_requant15(self, x, a, m, s, y, B, T, Cc, nm, ns, st):
        self._requant15_counts(Cc, nm, ns)
        self.f["add_requant15"](x, a, m, s, y, B, T, Cc, nm, ns)

    def iw_embed_add_requant15(self, table, tokens, pe, offset, m, s, y, B, T, Cc, nm, ns, st):
        self._requant15_counts(Cc, nm, ns)
        tok = _view(tokens, B * T, np.int64)
        rows = np.ascontiguousarray(
            np.stack([_view(table + int(t) * Cc, Cc, np.int8) for t in tok]) if B * T else np.zeros((0, Cc), np.int8))
        self.f["add_requant15"](rows.ctypes.data, pe + offset * Cc, m, s, y, B, T, Cc, nm, ns)

    def iw_classifier(self, x, w, m, s, y, M, K, N, st):
        if M > 0:
            self.f["classifier"](x, w, m, s, y, M, K, N)

    # -- dispatch -----------------------------------------------------------------
    def call(self, name, *args):
        fn = getattr(self, name, None)
        if fn is None:
            raise NotImplementedError(f"{name} is not emulated")
        args = [a.value if isinstance(a, C.c_void_p) else a for a in args]
        try:
            fn(*args)
        except EmulatedError as e:
            if e.rc == _lib.IW_EVALUE:
                raise ValueError(str(e)) from None
            if e.rc == _lib.IW_EOVERFLOW:
                raise OverflowError(str(e)) from None
            raise _lib.IWhisperError(str(e)) from None


def _chk_host(t, name, dtype):
    """ops._chk without the device requirement (CPU tensors stand in for CUDA ones)."""
    from i_whisper_b200 import ops
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if t.dtype != ops._DT[dtype]:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def install(patch):
    """Route ``i_whisper_b200.ops`` through the emulator. ``patch(obj, name,
    value)`` is pytest's ``monkeypatch.setattr`` or any equivalent."""
    from i_whisper_b200 import ops
    emu = CapiEmulator()
    patch(ops, "_chk", _chk_host)
    patch(ops, "_stream", lambda: None)
    patch(ops._lib, "call", emu.call)
    return emu
