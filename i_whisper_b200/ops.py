"""Torch-tensor operators of the B200 integer path.

Each ``<op>_cuda`` function has the argument list, output shape/dtype and
error behaviour of the reference operator ``i_whisper.kernels._C.<op>_simd``
(vcsd-lab/I-Whisper, i_whisper/kernels/csrc/pybind.cpp:45-415), with CUDA
tensors instead of CPU tensors, and runs the sm_100a kernels of
``libiwhisper_b200.so`` through its C ABI on the current CUDA stream.
Checks follow ``common/checktensor.h``: exact dtype, contiguous, and here a
CUDA device; violations raise ``RuntimeError`` like ``TORCH_CHECK``.

Scalar quantisation parameters (the 1-element tensors of the reference)
are read with ``.item()``; the model runner caches them on the host instead.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_DT = {
    "int8": torch.int8, "uint8": torch.uint8, "int16": torch.int16, "uint16": torch.uint16,
    "int32": torch.int32, "uint32": torch.uint32, "bool": torch.bool, "int64": torch.int64,
}


def _chk(t, name: str, dtype: str):
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor, got device {t.device}")
    if t.dtype != _DT[dtype]:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _scalar(t, name: str) -> int:
    if isinstance(t, torch.Tensor):
        if t.numel() != 1:
            raise RuntimeError(f"{name} must be a scalar tensor")
        return int(t.reshape(-1)[0].item())
    return int(t)


# ---------------------------------------------------------------------------
# Linear8 / Linear32 (linear8_torch.cpp:14-152, linear32_torch.cpp)
# ---------------------------------------------------------------------------
def _linear_checks(x, weight, bias, weight_zero, multiplier, shift):
    _chk(x, "x", "int8"); _chk(weight, "weight", "int8")
    if multiplier is not None:
        _chk(multiplier, "multiplier", "uint32"); _chk(shift, "shift", "int8")
    if x.dim() < 1:
        raise RuntimeError("x must have at least 1 dimension")
    if weight.dim() != 2:
        raise RuntimeError(f"weight must have 2 dimensions, got {weight.dim()}")
    K = x.shape[-1]
    if K <= 0:
        raise RuntimeError("x.size(-1) must be greater than 0")
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise RuntimeError(f"weight.size(1) must equal x.size(-1), expected {K}, got {weight.shape[1]}")
    if multiplier is not None:
        if multiplier.dim() != 1 or shift.dim() != 1:
            raise RuntimeError("multiplier and shift should be 1D tensors")
        if multiplier.numel() != N:
            raise RuntimeError(f"weight.size(0) must equal multiplier's number of elements, expected {N}, got {multiplier.numel()}")
        if shift.numel() != multiplier.numel():
            raise RuntimeError("multiplier's number of elements must equal shift's number of elements")
    if bias is not None:
        _chk(bias, "bias", "int32")
        if bias.dim() != 1 or bias.shape[0] != N:
            raise RuntimeError(f"bias.size(0) must equal weight.size(0), expected {N}")
    if weight_zero is not None:
        _chk(weight_zero, "weight_zero", "int8")
        if weight_zero.dim() != 1 or weight_zero.shape[0] != N:
            raise RuntimeError(f"weight_zero.size(0) must equal weight.size(0), expected {N}")
    M = x.numel() // K
    return M, K, N


def linear8_cuda(x, weight, bias=None, weight_zero=None, multiplier=None, shift=None):
    """``_C.linear8_simd`` (linear8_scalar.cpp:30-84)."""
    M, K, N = _linear_checks(x, weight, bias, weight_zero, multiplier, shift)
    y = torch.empty(*x.shape[:-1], N, dtype=torch.int8, device=x.device)
    _lib.call("iw_linear8", x.data_ptr(), weight.data_ptr(), _p(bias), _p(weight_zero), multiplier.data_ptr(),
              shift.data_ptr(), y.data_ptr(), M, K, N, _stream())
    return y


def linear8_accum_cuda_debug(x, weight, bias=None, weight_zero=None):
    """``_C.linear8_accum_simd_debug`` (linear8_scalar.cpp:87-127)."""
    M, K, N = _linear_checks(x, weight, bias, weight_zero, None, None)
    y = torch.empty(*x.shape[:-1], N, dtype=torch.int32, device=x.device)
    _lib.call("iw_linear8_accum", x.data_ptr(), weight.data_ptr(), _p(bias), _p(weight_zero), y.data_ptr(), M, K, N,
              _stream())
    return y


def _requant_checks(input, multiplier, shift):
    """Argument checks of the requantise-only debug ops (linear8_torch.cpp:344-361,
    linear32_torch.cpp:334-351) -> (M, N)."""
    _chk(input, "input", "int32"); _chk(multiplier, "multiplier", "uint32"); _chk(shift, "shift", "int8")
    if input.dim() < 1:
        raise RuntimeError(f"input must have at least one dimension, got {input.dim()}")
    if multiplier.dim() != 1:
        raise RuntimeError(f"multiplier should be a 1D tensor, got {multiplier.dim()}")
    if shift.dim() != 1:
        raise RuntimeError(f"shift should be a 1D tensor, got {shift.dim()}")
    N = input.shape[-1]
    if N != multiplier.numel():
        raise RuntimeError(f"input.size(-1) must equal multiplier's number of elements, got {N} "
                           f"expected {multiplier.numel()}")
    if multiplier.numel() != shift.numel():
        raise RuntimeError(f"multiplier's number of elements must equal shift's number of elements, got "
                           f"{multiplier.numel()} expected {shift.numel()}")
    return (input.numel() // N if N else 0), N


def linear8_requant_cuda_debug(input, multiplier, shift):
    """``_C.linear8_requant_scalar_debug`` (linear8_torch.cpp:336-387): int32
    accumulators -> rrs(mulh(acc, m[n]), (u32)s[n]) as int32, without the
    final int8 clamp of Linear8."""
    M, N = _requant_checks(input, multiplier, shift)
    y = torch.empty(input.shape, dtype=torch.int32, device=input.device)
    if M > 0:
        _lib.call("iw_linear8_requant", input.data_ptr(), multiplier.data_ptr(), shift.data_ptr(), y.data_ptr(), M, N,
                  _stream())
    return y


def linear32_requant_cuda_debug(input, multiplier, shift):
    """``_C.linear32_requant_scalar_debug`` (linear32_torch.cpp:326-377): int32
    accumulators -> (int32)((u32)mulh(acc, m[n]) << s[n]), 0 for s >= 32.
    Each row m is the bias of a one-row Linear32 GEMM whose x and weight are
    zero, so the GEMM's requantisation epilogue sees acc = input[m, n]
    exactly; one launch per row (a debug path)."""
    M, N = _requant_checks(input, multiplier, shift)
    y = torch.empty(input.shape, dtype=torch.int32, device=input.device)
    if M == 0:
        return y
    rows, out = input.view(M, N), y.view(M, N)
    zx = torch.zeros(1, 16, dtype=torch.int8, device=input.device)
    zw = torch.zeros(N, 16, dtype=torch.int8, device=input.device)
    for m in range(M):
        _lib.call("iw_linear32", zx.data_ptr(), zw.data_ptr(), rows[m].data_ptr(), None, multiplier.data_ptr(),
                  shift.data_ptr(), out[m].data_ptr(), 1, 16, N, _stream())
    return y


def rounding_rshift_debug_cuda(x, shift):
    """``_C.rounding_rshift_debug`` (pybind.cpp:22-43): fixedpoint
    rounding_rshift of every int32 element by shift[0] (uint32). The shift is
    read on the host, so its tensor may live on either device."""
    _chk(x, "x", "int32")
    if not isinstance(shift, torch.Tensor) or shift.dtype != torch.uint32:
        raise RuntimeError("shift must be a uint32 tensor")
    if shift.numel() < 1:
        raise RuntimeError("shift must have at least one element")
    y = torch.empty_like(x)
    _lib.call("iw_rounding_rshift", x.data_ptr(), int(shift.reshape(-1)[0].item()), y.data_ptr(), x.numel(),
              _stream())
    return y


def linear32_cuda(x, weight, bias=None, weight_zero=None, multiplier=None, shift=None):
    """``_C.linear32_simd`` (linear32_scalar.cpp:96-129)."""
    M, K, N = _linear_checks(x, weight, bias, weight_zero, multiplier, shift)
    y = torch.empty(*x.shape[:-1], N, dtype=torch.int32, device=x.device)
    _lib.call("iw_linear32", x.data_ptr(), weight.data_ptr(), _p(bias), _p(weight_zero), multiplier.data_ptr(),
              shift.data_ptr(), y.data_ptr(), M, K, N, _stream())
    return y


def linear32_residual15_cuda(x, weight, bias, weight_zero, multiplier, shift, residual, residual_multiplier,
                             out: Optional[torch.Tensor] = None):
    """Linear32 followed by ``_C.residual15_simd`` in one kernel."""
    M, K, N = _linear_checks(x, weight, bias, weight_zero, multiplier, shift)
    _chk(residual, "residual", "int16")
    if residual.numel() != M * N:
        raise RuntimeError("branch and residual must have the same shape")
    y = torch.empty_like(residual) if out is None else out
    _lib.call("iw_linear32_residual15", x.data_ptr(), weight.data_ptr(), _p(bias), _p(weight_zero),
              multiplier.data_ptr(), shift.data_ptr(), residual.data_ptr(), _scalar(residual_multiplier, "multiplier"),
              y.data_ptr(), M, K, N, _stream())
    return y


def residual15_cuda(branch, residual, multiplier):
    """``_C.residual15_simd`` (residual15_scalar.cpp:9-27)."""
    _chk(branch, "branch", "int32"); _chk(residual, "residual", "int16")
    if isinstance(multiplier, torch.Tensor) and multiplier.dtype != torch.uint16:
        raise RuntimeError(f"multiplier must be uint16, got {multiplier.dtype}")
    if residual.shape != branch.shape:
        raise RuntimeError("branch and residual must have the same shape")
    y = torch.empty_like(residual)
    _lib.call("iw_residual15", branch.data_ptr(), residual.data_ptr(), _scalar(multiplier, "multiplier"), y.data_ptr(),
              branch.numel(), _stream())
    return y


# ---------------------------------------------------------------------------
# LayerNorm32 (layernorm_torch.cpp:200-305)
# ---------------------------------------------------------------------------
def _ln_width(x):
    d = x.shape[-1]
    if d not in (384, 512, 768, 1024, 1280):
        raise RuntimeError(f"unsupported LayerNorm hidden size: {d}")
    return d


def layernorm32_cuda(input, weight, bias, ln_multiplier, ln_shift, out_multiplier, out_shift, _entry="iw_layernorm32"):
    """``_C.layernorm32_simd`` (layernorm_scalar.cpp:464-624, offset 13)."""
    _chk(input, "input", "int16"); _chk(weight, "weight", "int8")
    if input.dim() < 1:
        raise RuntimeError("input must have at least one dimension")
    if weight.dim() != 1:
        raise RuntimeError("weight must be a 1D tensor")
    d = _ln_width(input)
    if weight.numel() != d:
        raise RuntimeError(f"weight.numel() must equal input.size(-1), got {weight.numel()} expected {d}")
    if bias is not None:
        _chk(bias, "bias", "int32")
        if bias.dim() != 1 or bias.numel() != d:
            raise RuntimeError(f"bias.numel() must equal input.size(-1), got {bias.numel()} expected {d}")
    y = torch.empty_like(input, dtype=torch.int8)
    _lib.call(_entry, input.data_ptr(), weight.data_ptr(), _p(bias), _scalar(ln_multiplier, "ln_multiplier"),
              _scalar(ln_shift, "ln_shift"), _scalar(out_multiplier, "out_multiplier"), _scalar(out_shift, "out_shift"),
              y.data_ptr(), input.numel() // d, d, _stream())
    return y


def layernorm32_stats_cuda(input) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``_C.layernorm32_stats_simd`` (layernorm_scalar.cpp:133-214)."""
    _chk(input, "input", "int16")
    d = _ln_width(input)
    rows = input.numel() // d
    mean = torch.empty(rows, dtype=torch.int32, device=input.device)
    var = torch.empty_like(mean); rs = torch.empty_like(mean)
    _lib.call("iw_layernorm32_stats", input.data_ptr(), mean.data_ptr(), var.data_ptr(), rs.data_ptr(), rows, d,
              _stream())
    return mean, var, rs


def layernorm64_cuda(input, weight, bias, ln_multiplier, ln_shift, out_multiplier, out_shift):
    """``_C.layernorm64_simd`` (layernorm_scalar.cpp:626-825; rsqrt offset 15,
    normalise-shift offset 2 as layernorm_torch.cpp:446-460). OverflowError
    when a row's variance does not fit INT32, as the reference."""
    return layernorm32_cuda(input, weight, bias, ln_multiplier, ln_shift, out_multiplier, out_shift,
                            _entry="iw_layernorm64")


def layernorm64_stats_cuda(input) -> Tuple[torch.Tensor, torch.Tensor]:
    """``_C.layernorm64_stats_simd`` (layernorm_scalar.cpp:230-297): mean
    int32 and variance int64 per row."""
    _chk(input, "input", "int16")
    d = _ln_width(input)
    rows = input.numel() // d
    mean = torch.empty(rows, dtype=torch.int32, device=input.device)
    var = torch.empty(rows, dtype=torch.int64, device=input.device)
    _lib.call("iw_layernorm64_stats", input.data_ptr(), mean.data_ptr(), var.data_ptr(), rows, d, _stream())
    return mean, var


def layernorm32_rsqrt_cuda(input):
    """``_C.layernorm32_rsqrt_scalar`` (layernorm_scalar.cpp:383-437)."""
    _chk(input, "input", "int32")
    y = torch.empty_like(input)
    _lib.call("iw_layernorm32_rsqrt", input.data_ptr(), y.data_ptr(), input.numel(), _stream())
    return y


# ---------------------------------------------------------------------------
# GeLU (gelu_torch.cpp:9-150)
# ---------------------------------------------------------------------------
def gelu_cuda(input, lut, luti_multiplier, luti_shift, luto_multiplier, luto_shift):
    """``_C.gelu_simd`` (gelu_scalar.cpp:10-181)."""
    _chk(input, "input", "int8"); _chk(lut, "lut", "uint8")
    _chk(luti_multiplier, "luti_multiplier", "uint8"); _chk(luti_shift, "luti_shift", "int8")
    _chk(luto_multiplier, "luto_multiplier", "uint8"); _chk(luto_shift, "luto_shift", "int8")
    if input.dim() < 1:
        raise RuntimeError("input must have at least one dimension")
    if lut.dim() != 1 or lut.numel() != 16:
        raise RuntimeError("lut must contain exactly 16 entries")
    for t, n in ((luti_multiplier, "luti_multiplier"), (luti_shift, "luti_shift"), (luto_multiplier, "luto_multiplier"),
                 (luto_shift, "luto_shift")):
        if t.dim() != 1:
            raise RuntimeError(f"{n} must be 1D")
    if luti_multiplier.numel() != luti_shift.numel():
        raise RuntimeError("luti multiplier/shift size mismatch")
    if luto_multiplier.numel() != luto_shift.numel():
        raise RuntimeError("luto multiplier/shift size mismatch")
    y = torch.empty_like(input)
    _lib.call("iw_gelu", input.data_ptr(), lut.data_ptr(), luti_multiplier.data_ptr(), luti_shift.data_ptr(),
              luto_multiplier.data_ptr(), luto_shift.data_ptr(), y.data_ptr(), input.numel(), input.shape[-1],
              luti_multiplier.numel(), luto_multiplier.numel(), _stream())
    return y


# ---------------------------------------------------------------------------
# Attention stages (attention_torch.cpp:116-700)
# ---------------------------------------------------------------------------
def _mask_arg(mask, Tq, Tk):
    if mask is None:
        return None
    _chk(mask, "mask", "bool")
    if mask.dim() != 2 or mask.shape[0] != Tq or mask.shape[1] != Tk:
        raise RuntimeError("mask must be [Tq,Tk]")
    return mask


def qk_requant_rowmax_cuda(q, k, mask, multiplier, shift):
    """``_C.qk_requant_rowmax_simd`` (attention_scalar.cpp:216-343)."""
    _chk(q, "q", "int8"); _chk(k, "k", "int8")
    if q.dim() != 4:
        raise RuntimeError("q must be [B,H,Tq,D]")
    if k.dim() != 4:
        raise RuntimeError("k must be [B,H,Tk,D]")
    if q.shape[0] != k.shape[0]:
        raise RuntimeError("batch mismatch")
    if q.shape[1] != k.shape[1]:
        raise RuntimeError("head count mismatch")
    if q.shape[3] != k.shape[3]:
        raise RuntimeError("head dimension mismatch")
    if isinstance(multiplier, torch.Tensor) and multiplier.dtype != torch.uint8:
        raise RuntimeError(f"multiplier must be uint8, got {multiplier.dtype}")
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    mask = _mask_arg(mask, Tq, Tk)
    qk = torch.empty(B, H, Tq, Tk, dtype=torch.int16, device=q.device)
    rm = torch.empty(B, H, Tq, 1, dtype=torch.int16, device=q.device)
    _lib.call("iw_qk_requant_rowmax", q.data_ptr(), k.data_ptr(), _p(mask), _scalar(multiplier, "multiplier"),
              _scalar(shift, "shift"), qk.data_ptr(), rm.data_ptr(), B, H, Tq, Tk, D, _stream())
    return qk, rm


def shift_exp_cuda(input, row_max_plus1, mask, frac_bits):
    """``_C.shift_exp_simd`` (attention_scalar.cpp:388-560)."""
    _chk(input, "input", "int16"); _chk(row_max_plus1, "row_max_plus1", "int16")
    if input.dim() != 4:
        raise RuntimeError("input must be [B,H,Tq,Tk]")
    if row_max_plus1.dim() != 4:
        raise RuntimeError("row_max_plus1 must be [B,H,Tq,1]")
    B, H, Tq, Tk = input.shape
    if tuple(row_max_plus1.shape) != (B, H, Tq, 1):
        raise RuntimeError("row_max_plus1.size(0) must equal input.size(0)")
    fb = _scalar(frac_bits, "frac_bits")
    mask = _mask_arg(mask, Tq, Tk)
    p = torch.empty(B, H, Tq, Tk, dtype=torch.uint8, device=input.device)
    rs = torch.empty(B, H, Tq, 1, dtype=torch.int32, device=input.device)
    _lib.call("iw_shift_exp", input.data_ptr(), row_max_plus1.data_ptr(), _p(mask), fb, p.data_ptr(), rs.data_ptr(),
              B, H, Tq, Tk, _stream())
    return p, rs


def pv_norm_requant_cuda(p, v, row_sum, av_multiplier, av_shift, rsqrt_offset: int):
    """``_C.pv_norm_requant_simd`` (attention_scalar.cpp:676-813)."""
    _chk(p, "p", "uint8"); _chk(v, "v", "int8"); _chk(row_sum, "row_sum", "int32")
    if p.dim() != 4:
        raise RuntimeError("p must be [B,H,Tq,Tk]")
    if v.dim() != 4:
        raise RuntimeError("v must be [B,H,D,Tk]")
    if row_sum.dim() != 4:
        raise RuntimeError("row_sum must be [B,H,Tq,1]")
    B, H, Tq, Tk = p.shape
    D = v.shape[2]
    if v.shape[0] != B or row_sum.shape[0] != B:
        raise RuntimeError("batch mismatch")
    if v.shape[1] != H or row_sum.shape[1] != H:
        raise RuntimeError("head count mismatch")
    if row_sum.shape[2] != Tq:
        raise RuntimeError("query length mismatch")
    if row_sum.shape[3] != 1:
        raise RuntimeError("row_sum must have last dimension 1")
    if v.shape[3] != Tk:
        raise RuntimeError("key length mismatch")
    y = torch.empty(B, Tq, H * D, dtype=torch.int8, device=p.device)
    _lib.call("iw_pv_norm_requant", p.data_ptr(), v.data_ptr(), row_sum.data_ptr(), _scalar(av_multiplier, "av_multiplier"),
              _scalar(av_shift, "av_shift"), int(rsqrt_offset), y.data_ptr(), B, H, Tq, Tk, D, _stream())
    return y


def _accum_i32(x2d, w2d, y2d):
    """y2d [M,N] int32 = x2d [M,K] @ w2d [N,K]^T with wrapping int32 sums,
    through the tensor-core accumulator GEMM (iw_linear8_accum). Views must be
    contiguous; K == 0 gives zeros, as the reference's empty sums do."""
    M, K = x2d.shape
    N = w2d.shape[0]
    if M == 0 or N == 0:
        return
    if K == 0:
        y2d.zero_()
        return
    _lib.call("iw_linear8_accum", x2d.data_ptr(), w2d.data_ptr(), None, None, y2d.data_ptr(), M, K, N, _stream())


def qk_cuda(q, k):
    """``_C.qk_simd`` (attention_torch.cpp:10-114, qk_scalar attention_scalar.cpp:130):
    q [B,H,Tq,D] int8, k [B,H,Tk,D] int8 -> int32 [B,H,Tq,Tk], the raw
    Q·Kᵀ sums. One accumulator GEMM per (batch, head)."""
    _chk(q, "q", "int8"); _chk(k, "k", "int8")
    if q.dim() != 4:
        raise RuntimeError("q must be [B,H,Tq,D]")
    if k.dim() != 4:
        raise RuntimeError("k must be [B,H,Tk,D]")
    if q.shape[0] != k.shape[0]:
        raise RuntimeError("batch mismatch")
    if q.shape[1] != k.shape[1]:
        raise RuntimeError("head count mismatch")
    if q.shape[3] != k.shape[3]:
        raise RuntimeError("head dimension mismatch")
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    y = torch.empty(B, H, Tq, Tk, dtype=torch.int32, device=q.device)
    qf, kf, yf = q.reshape(B * H, Tq, D), k.reshape(B * H, Tk, D), y.view(B * H, Tq, Tk)
    for i in range(B * H):
        _accum_i32(qf[i], kf[i], yf[i])
    return y


def pv_cuda(p, v):
    """``_C.pv_simd`` (attention_torch.cpp:401-521, pv_scalar attention_scalar.cpp:590):
    p [B,H,Tq,Tk] uint8, v [B,H,D,Tk] int8 (V transposed) -> int32
    [B,H,Tq,D], the raw P·V sums. The int8 GEMM takes signed operands, so
    p = lo + 128·hi with lo = p & 127 and hi = p >> 7 (both within int8), and
    the sum is Σ lo·v + 128·Σ hi·v; int32 wrapping sums make the split exact."""
    _chk(p, "p", "uint8"); _chk(v, "v", "int8")
    if p.dim() != 4:
        raise RuntimeError("p must be [B,H,Tq,Tk]")
    if v.dim() != 4:
        raise RuntimeError("v must be [B,H,D,Tk]")
    if p.shape[0] != v.shape[0]:
        raise RuntimeError("batch mismatch")
    if p.shape[1] != v.shape[1]:
        raise RuntimeError("head count mismatch")
    if p.shape[3] != v.shape[3]:
        raise RuntimeError("key length mismatch")
    B, H, Tq, Tk = p.shape
    D = v.shape[2]
    y = torch.empty(B, H, Tq, D, dtype=torch.int32, device=p.device)
    lo = torch.bitwise_and(p, 127).view(torch.int8).reshape(B * H, Tq, Tk)
    hi = torch.bitwise_right_shift(p, 7).view(torch.int8).reshape(B * H, Tq, Tk)
    vf, yf = v.reshape(B * H, D, Tk), y.view(B * H, Tq, D)
    y_hi = torch.empty(Tq, D, dtype=torch.int32, device=p.device)
    for i in range(B * H):
        _accum_i32(lo[i], vf[i], yf[i])
        _accum_i32(hi[i], vf[i], y_hi)
        yf[i].add_(y_hi, alpha=128)
    return y


def attention_cuda(q, k, v, n_head: int, qk_multiplier, qk_shift, frac_bits, av_multiplier, av_shift,
                   rsqrt_offset: int = 16, mask_mode: int = 0, mask=None, out=None):
    """Fused A1-A3 (MultiHeadAttention_int.qkv_attention, model_int.py:774-1042)
    on projection outputs q [B,Tq,H*64], k/v [B,Tk,H*64] (row strides may
    exceed H*64) -> [B,Tq,H*64] int8."""
    B, Tq, d = q.shape[0], q.shape[1], n_head * 64
    Tk = k.shape[1]
    y = torch.empty(B, Tq, d, dtype=torch.int8, device=q.device) if out is None else out
    _lib.call("iw_attention", q.data_ptr(), q.stride(1), q.stride(0), k.data_ptr(), k.stride(1), k.stride(0),
              v.data_ptr(), v.stride(1), v.stride(0), y.data_ptr(), y.stride(1), y.stride(0), B, n_head, Tq, Tk,
              mask_mode, _p(mask), _scalar(qk_multiplier, "qk_multiplier"), _scalar(qk_shift, "qk_shift"),
              _scalar(frac_bits, "frac_bits"), _scalar(av_multiplier, "av_multiplier"), _scalar(av_shift, "av_shift"),
              int(rsqrt_offset), _stream())
    return y


# ---------------------------------------------------------------------------
# Conv1d (conv1d_torch.cpp:136-360), Add+Requant15, classifier
# ---------------------------------------------------------------------------
def _conv1d_shape(input, weight, bias, stride, padding):
    """check_conv1d_common (conv1d_torch.cpp:26-133) -> (B, Cin, Tin, Cout, K, Tout)."""
    _chk(input, "input", "int8"); _chk(weight, "weight", "int8")
    if input.dim() != 3:
        raise RuntimeError("input must be [B,Cin,Tin]")
    if weight.dim() != 2:
        raise RuntimeError("weight must be flattened [Cout,Cin*K]")
    if stride <= 0:
        raise RuntimeError("stride must be positive")
    if padding < 0:
        raise RuntimeError("padding must be non-negative")
    B, Cin, Tin = input.shape
    Cout = weight.shape[0]
    if Cin <= 0:
        raise RuntimeError("input channel count must be positive")
    if Tin <= 0:
        raise RuntimeError("input length must be positive")
    if Cout <= 0:
        raise RuntimeError("output channel count must be positive")
    if weight.shape[1] % Cin != 0:
        raise RuntimeError("weight.size(1) must be divisible by input channels")
    K = weight.shape[1] // Cin
    if K <= 0:
        raise RuntimeError("kernel size must be positive")
    num = Tin + 2 * padding - K
    if num < 0:
        raise RuntimeError("invalid Conv1d geometry: output length would be non-positive")
    if bias is not None:
        _chk(bias, "bias", "int32")
        if bias.dim() != 1:
            raise RuntimeError("bias must be [Cout]")
        if bias.numel() != Cout:
            raise RuntimeError("bias.numel() must equal output channels")
    return B, Cin, Tin, Cout, K, num // stride + 1


def conv1d_cuda(input, weight, bias, multiplier, shift, stride: int, padding: int):
    """``_C.conv1d_simd`` (conv1d_scalar.cpp:186-288)."""
    B, Cin, Tin, Cout, K, Tout = _conv1d_shape(input, weight, bias, stride, padding)
    # scalar parameters are read on the host; they may live on either device
    if isinstance(multiplier, torch.Tensor):
        if multiplier.dtype != torch.uint32:
            raise RuntimeError(f"multiplier must be uint32, got {multiplier.dtype}")
        if multiplier.numel() != 1:
            raise RuntimeError("multiplier must contain exactly one element")
    if isinstance(shift, torch.Tensor):
        if shift.dtype != torch.int8:
            raise RuntimeError(f"shift must be int8, got {shift.dtype}")
        if shift.numel() != 1:
            raise RuntimeError("shift must contain exactly one element")
    y = torch.empty(B, Cout, Tout, dtype=torch.int8, device=input.device)
    _lib.call("iw_conv1d", input.data_ptr(), weight.data_ptr(), _p(bias), _scalar(multiplier, "multiplier"),
              _scalar(shift, "shift"), stride, padding, y.data_ptr(), B, Cin, Tin, Cout, K, _stream())
    return y


def conv1d_accum_cuda(input, weight, bias, stride: int, padding: int):
    """``_C.conv1d_accum_simd`` (conv1d_torch.cpp:136-209): the int32
    accumulators [B,Cout,Tout] before requantisation, bias included. im2col
    (column cin*K + k, the weight's flattened order) and one accumulator GEMM
    with the bias in its epilogue."""
    B, Cin, Tin, Cout, K, Tout = _conv1d_shape(input, weight, bias, stride, padding)
    y = torch.empty(B, Cout, Tout, dtype=torch.int32, device=input.device)
    if B == 0:
        return y
    cols = torch.empty(B * Tout, Cin * K, dtype=torch.int8, device=input.device)
    _lib.call("iw_im2col", input.data_ptr(), cols.data_ptr(), B, Cin, Tin, K, stride, padding, Tout, Cin * K, 0,
              _stream())
    acc = torch.empty(B * Tout, Cout, dtype=torch.int32, device=input.device)
    _lib.call("iw_linear8_accum", cols.data_ptr(), weight.data_ptr(), _p(bias), None, acc.data_ptr(), B * Tout,
              Cin * K, Cout, _stream())
    y.copy_(acc.view(B, Tout, Cout).permute(0, 2, 1))
    return y


def add_requant15_cuda(input, addend, multiplier, shift):
    """``_C.add_requant15_simd`` (add_requant15_scalar.cpp:29-80)."""
    _chk(input, "input", "int8"); _chk(addend, "addend", "int8")
    _chk(multiplier, "multiplier", "uint16"); _chk(shift, "shift", "int8")
    if input.dim() != 3:
        raise RuntimeError("input must be [B,T,C]")
    if addend.dim() != 2:
        raise RuntimeError("addend must be [T,C]")
    B, T, Cc = input.shape
    if addend.shape[0] != T or addend.shape[1] != Cc:
        raise RuntimeError("addend must match input [T,C]")
    if multiplier.dim() != 1 or shift.dim() != 1:
        raise RuntimeError("multiplier and shift must be 1D")
    y = torch.empty(B, T, Cc, dtype=torch.int16, device=input.device)
    _lib.call("iw_add_requant15", input.data_ptr(), addend.data_ptr(), multiplier.data_ptr(), shift.data_ptr(),
              y.data_ptr(), B, T, Cc, multiplier.numel(), shift.numel(), _stream())
    return y


def embed_add_requant15_cuda(table, tokens, pe, offset: int, multiplier, shift, out=None):
    """Token-embedding gather + add_requant15 (TextDecoder_int.forward,
    model_int.py:1411-1428): tokens [B,T] int64 -> [B,T,C] int16."""
    _chk(table, "table", "int8"); _chk(tokens, "tokens", "int64"); _chk(pe, "pe", "int8")
    _chk(multiplier, "multiplier", "uint16"); _chk(shift, "shift", "int8")
    B, T = tokens.shape
    Cc = table.shape[1]
    y = torch.empty(B, T, Cc, dtype=torch.int16, device=table.device) if out is None else out
    _lib.call("iw_embed_add_requant15", table.data_ptr(), tokens.data_ptr(), pe.data_ptr(), int(offset),
              multiplier.data_ptr(), shift.data_ptr(), y.data_ptr(), B, T, Cc, multiplier.numel(), shift.numel(),
              _stream())
    return y


def _classifier_shape(input, weight):
    """check_classifier_common (classifier_torch.cpp:23-75) -> (B, T, K, N)."""
    _chk(input, "input", "int8"); _chk(weight, "weight", "int8")
    if input.dim() != 3:
        raise RuntimeError("input must be [B,T,K]")
    if weight.dim() != 2:
        raise RuntimeError("weight must be [N,K]")
    B, T, K = input.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise RuntimeError("weight hidden size must match input")
    if K <= 0:
        raise RuntimeError("hidden size must be positive")
    if N <= 0:
        raise RuntimeError("vocabulary size must be positive")
    return B, T, K, N


def classifier_cuda(input, weight, multiplier, shift):
    """``_C.classifier_simd`` (classifier_scalar.cpp:91-140)."""
    B, T, K, N = _classifier_shape(input, weight)
    y = torch.empty(B, T, N, dtype=torch.int8, device=input.device)
    _lib.call("iw_classifier", input.data_ptr(), weight.data_ptr(), _scalar(multiplier, "multiplier"),
              _scalar(shift, "shift"), y.data_ptr(), B * T, K, N, _stream())
    return y


def classifier_accum_cuda(input, weight):
    """``_C.classifier_accum_simd`` (classifier_torch.cpp:78-143): the raw
    int32 sums x·Eᵀ [B,T,V] before requantisation."""
    B, T, K, N = _classifier_shape(input, weight)
    y = torch.empty(B, T, N, dtype=torch.int32, device=input.device)
    _accum_i32(input.view(B * T, K), weight, y.view(B * T, N))
    return y


def linear32_accum_cuda_debug(x, weight, bias=None, weight_zero=None):
    """``_C.linear32_accum_simd_debug`` (linear32_scalar.cpp:9-63): the same
    int32 accumulator as Linear8's (x·Wᵀ + bias − wz·Σx, wrapping), which the
    Linear8 accumulator entry point computes."""
    return linear8_accum_cuda_debug(x, weight, bias, weight_zero)
