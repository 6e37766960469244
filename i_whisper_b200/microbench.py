"""Kernel microbenchmark of the integer hot path (the seeded kernel shapes of
the reference's benchmark configuration: w8a8 GEMM at M = 1500*B, integer
LayerNorm over 1500 x 1024 rows, 16-head 1500 x 1500 integer attention) plus
the decode-shaped attention over a 1500-position cross-attention cache.

Every case runs through the C ABI on preallocated device buffers, is timed
with CUDA events on the launching stream after warm-up, and prints one JSON
line with its roofline fraction. It is also the command the committed ncu
summaries are taken with (small cases, one kernel per process).

    python -m i_whisper_b200.microbench gemm --M 12000 --K 1024 --N 4096
    python -m i_whisper_b200.microbench layernorm --rows 1500 --d 1024
    python -m i_whisper_b200.microbench attention --B 4 --H 16 --T 1500
    python -m i_whisper_b200.microbench cross_attention --B 256 --H 16 --T 1500
    python -m i_whisper_b200.microbench decode --B 256 --from-step 96

Input distributions follow the benchmark configuration: INT8 entries uniform
in [-127, 127]; per-channel scales uniform in [1e-3, 1e-2] turned into
(u32 multiplier, shift) by the frexp rule of the quantiser; attention Q/K/V
from clamp(round(N(0, 30)), +-127).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os

import numpy as np
import torch

from . import _lib
from .checkpoint import _frexp_u32

DATASHEET_INT8_TOPS = 4500.0


def hbm_peak():
    """(GB/s, source): the measured copy bandwidth of this GPU pool when the
    peaks file is present next to the package, else the earlier fallback."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def _time(fn, reps: int, warmup: int = 3, flush: torch.Tensor = None) -> float:
    """Mean ms per launch of fn on the current stream (CUDA events). With
    ``flush`` (a buffer larger than L2) each launch is timed alone, after a
    write of the buffer that evicts L2, so the inputs come from HBM."""
    for _ in range(warmup):
        fn()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if flush is None:
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps
    total = 0.0
    for _ in range(reps):
        flush.fill_(1)
        e0.record(st)
        fn()
        e1.record(st)
        e1.synchronize()
        total += e0.elapsed_time(e1)
    return total / reps


def _i8(g: torch.Generator, *shape) -> torch.Tensor:
    return torch.randint(-127, 128, shape, dtype=torch.int8, generator=g).cuda()


def _gauss_i8(g: torch.Generator, *shape, std: float = 30.0) -> torch.Tensor:
    return torch.clamp(torch.round(torch.randn(shape, generator=g) * std), -127, 127).to(torch.int8).cuda()


def bench_gemm(M: int, K: int, N: int, mode: str, tile_n: int, reps: int, seed: int, gelu: str = "none",
               rowsum_out: bool = False, flush: torch.Tensor = None, warmup: int = 3) -> dict:
    g = torch.Generator().manual_seed(seed)
    x, w = _i8(g, M, K), _i8(g, N, K)
    rng = np.random.default_rng(seed)
    m, s = _frexp_u32(rng.uniform(1e-3, 1e-2, N))
    mult = torch.from_numpy(m.astype(np.uint32)).cuda()
    shift = torch.from_numpy(s.astype(np.int8)).cuda()
    bias = torch.from_numpy(rng.integers(-2**20, 2**20, N).astype(np.int32)).cuda()
    wz = torch.from_numpy(rng.integers(-8, 8, N).astype(np.int8)).cuda()
    rs = torch.empty(M, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("iw_rowsum_i8", x.data_ptr(), K, M, K, rs.data_ptr(), stream)
    d = _lib.GemmDesc()
    d.x, d.ldx, d.w, d.ldw, d.M, d.N, d.K = x.data_ptr(), K, w.data_ptr(), K, M, N, K
    d.bias, d.weight_zero, d.x_rowsum, d.multiplier, d.shift = (bias.data_ptr(), wz.data_ptr(), rs.data_ptr(),
                                                               mult.data_ptr(), shift.data_ptr())
    d.tile_n = tile_n
    keep = [x, w, mult, shift, bias, wz, rs]
    if mode == "linear8":
        out = torch.empty(M, N, dtype=torch.int8, device="cuda")
        d.mode = _lib.IW_GEMM_INT8
        out_bytes = M * N
        if gelu != "none":  # fc1 form: per-channel GeLU on the int8 result
            gp = [torch.from_numpy(a).cuda() for a in (
                rng.integers(0, 256, 16).astype(np.uint8), rng.integers(0, 256, N).astype(np.uint8),
                rng.integers(0, 12, N).astype(np.int8), rng.integers(0, 256, N).astype(np.uint8),
                rng.integers(6, 14, N).astype(np.int8))]
            keep += gp
            if gelu == "table":
                tab = torch.empty(N, 256, dtype=torch.int8, device="cuda")
                keep.append(tab)
                _lib.call("iw_gelu_table", *[t.data_ptr() for t in gp], N, N, N, tab.data_ptr(), stream)
                tiled = torch.empty((N + 127) // 128, 32768, dtype=torch.int8, device="cuda")
                keep.append(tiled)
                _lib.call("iw_gelu_table_tiled", tab.data_ptr(), N, tiled.data_ptr(), stream)
                d.gelu_table, d.gelu_table_tiled = tab.data_ptr(), tiled.data_ptr()
            else:
                d.lut, d.luti_multiplier, d.luti_shift, d.luto_multiplier, d.luto_shift = [t.data_ptr() for t in gp]
                d.luti_per_channel = d.luto_per_channel = 1
        if rowsum_out:
            rso = torch.zeros(M, dtype=torch.int32, device="cuda")
            keep.append(rso)
            d.out_rowsum = rso.data_ptr()
    else:  # linear32 + residual15 (out-projection / fc2)
        out = torch.empty(M, N, dtype=torch.int16, device="cuda")
        res = torch.randint(-16383, 16384, (M, N), dtype=torch.int16, generator=g).cuda()
        keep.append(res)
        d.mode = _lib.IW_GEMM_LINEAR32_RES
        d.residual, d.ldr, d.residual_multiplier = res.data_ptr(), N, 23000
        out_bytes = 4 * M * N
    d.out, d.ldo = out.data_ptr(), N
    ms = _time(lambda: _lib.check(_lib.LIB.iw_gemm_i8(C.byref(d), stream)), reps, warmup, flush)
    tops = 2.0 * M * N * K / ms / 1e9
    return {"op": "gemm", "mode": mode, "gelu": gelu, "rowsum_out": rowsum_out, "M": M, "K": K, "N": N,
            "tile_n": tile_n, "ms": round(ms, 4),
            "tops": round(tops, 1), "frac_of_datasheet_4500": round(tops / DATASHEET_INT8_TOPS, 4),
            "algorithmic_bytes": M * K + N * K + out_bytes}


def bench_layernorm(rows: int, d: int, reps: int, seed: int, flush: torch.Tensor = None, warmup: int = 3) -> dict:
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-16383, 16384, (rows, d), dtype=torch.int16, generator=g).cuda()
    gamma = _i8(g, d)
    beta = torch.randint(-2**15, 2**15, (d,), dtype=torch.int32, generator=g).cuda()
    y = torch.empty(rows, d, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ms = _time(lambda: _lib.call("iw_layernorm32", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), 180, 9,
                                 1 << 30, 18, y.data_ptr(), rows, d, stream), reps, warmup, flush)
    hbm, src = hbm_peak()
    gbs = rows * d * 3 / ms / 1e6
    return {"op": "layernorm32", "rows": rows, "d": d, "ms": round(ms, 4), "gbs": round(gbs, 1),
            "frac": round(gbs / hbm, 4), "peak_gbs": hbm, "peak_source": src}


def _attn_desc(q, ldq, q_bs, q_hs, k, ldk, k_bs, k_hs, v, ldv, v_bs, v_hs, y, ldy, y_bs, B, H, Tq, Tk):
    a = _lib.AttnDesc()
    a.q, a.ldq, a.q_bs, a.q_hs = q, ldq, q_bs, q_hs
    a.k, a.ldk, a.k_bs, a.k_hs = k, ldk, k_bs, k_hs
    a.v, a.ldv, a.v_bs, a.v_hs = v, ldv, v_bs, v_hs
    a.y, a.ldy, a.y_bs, a.y_hs = y, ldy, y_bs, 64
    a.B, a.H, a.Tq, a.Tk = B, H, Tq, Tk
    a.qk_multiplier, a.qk_shift, a.frac_bits = 182, 12, 7
    a.av_multiplier, a.av_shift, a.rsqrt_offset = 192, 7, 16
    return a


def bench_attention(B: int, H: int, T: int, reps: int, seed: int, qk_m: int = 182, qk_s: int = 12, fb: int = 7,
                    std: float = 30.0, flush: torch.Tensor = None, warmup: int = 3) -> dict:
    """Encoder self-attention straight from a fused QKV projection buffer
    (Q/K/V clipped normal with standard deviation ``std``; the score
    requantisation and frac_bits of a layer: the calibrated whisper-medium
    checkpoint has qk multipliers 64-126, shifts 6-8, frac_bits 13-14)."""
    g = torch.Generator().manual_seed(seed)
    d = H * 64
    qkv = _gauss_i8(g, B * T, 3 * d, std=std)
    out = torch.empty(B * T, d, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    tab = torch.empty(32772, dtype=torch.uint8, device="cuda")
    _lib.call("iw_shift_exp_table", fb, tab.data_ptr(), stream)
    vt_ld = (T + 15) // 16 * 16
    vt = torch.empty(B * H * 64, vt_ld, dtype=torch.int8, device="cuda")
    base = qkv.data_ptr()
    a = _attn_desc(base, 3 * d, T * 3 * d, 64, base + d, 3 * d, T * 3 * d, 64, base + 2 * d, 3 * d, T * 3 * d, 64,
                   out.data_ptr(), d, T * d, B, H, T, T)
    a.exp_table, a.vt, a.vt_ld = tab.data_ptr(), vt.data_ptr(), vt_ld
    a.qk_multiplier, a.qk_shift, a.frac_bits = qk_m, qk_s, fb
    ms = _time(lambda: _lib.check(_lib.LIB.iw_attention_ex(C.byref(a), stream)), reps, warmup, flush)
    tops = 4.0 * B * H * T * T * 64 / ms / 1e9
    return {"op": "attention", "B": B, "H": H, "T": T, "qk_multiplier": qk_m, "qk_shift": qk_s, "frac_bits": fb,
            "std": std, "ms": round(ms, 4), "tops": round(tops, 1),
            "frac_of_datasheet_4500": round(tops / DATASHEET_INT8_TOPS, 4),
            "note": "ops count QK^T and P.V once (the kernel computes QK^T twice)"}


def bench_cross_attention(B: int, H: int, T: int, reps: int, seed: int) -> dict:
    """One decode step of cross-attention: one query row per utterance over
    a head-major [H, B, T, 64] INT8 key cache and value cache."""
    g = torch.Generator().manual_seed(seed)
    d = H * 64
    q = _gauss_i8(g, B, d)
    k = _gauss_i8(g, H, B, T, 64)
    v = _gauss_i8(g, H, B, T, 64)
    out = torch.empty(B, d, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    a = _attn_desc(q.data_ptr(), d, d, 64, k.data_ptr(), 64, T * 64, B * T * 64, v.data_ptr(), 64, T * 64,
                   B * T * 64, out.data_ptr(), d, d, B, H, 1, T)
    ms = _time(lambda: _lib.check(_lib.LIB.iw_attention_ex(C.byref(a), stream)), reps)
    hbm, src = hbm_peak()
    nbytes = 2 * B * H * T * 64
    gbs = nbytes / ms / 1e6
    return {"op": "cross_attention", "B": B, "H": H, "Tk": T, "ms": round(ms, 4), "gbs": round(gbs, 1),
            "frac": round(gbs / hbm, 4), "peak_gbs": hbm, "peak_source": src, "algorithmic_bytes": nbytes}


def bench_frontend(B: int, n_mels: int, reps: int, seed: int) -> dict:
    """GPU log-mel + INT8 quantisation of B windows of 30 s audio."""
    from .frontend import log_mel_int8_cuda
    g = torch.Generator().manual_seed(seed)
    audio = (torch.randn(B, 480000, generator=g) * 0.2).cuda()
    ms = _time(lambda: log_mel_int8_cuda(audio, n_mels, 100.0), reps)
    hbm, src = hbm_peak()
    nbytes = B * (480000 * 4 + n_mels * 3000)
    return {"op": "frontend", "B": B, "n_mels": n_mels, "ms": round(ms, 4), "windows_per_s": round(B / ms * 1e3, 1),
            "gbs": round(nbytes / ms / 1e6, 1), "frac": round(nbytes / ms / 1e6 / hbm, 4), "peak_gbs": hbm,
            "peak_source": src}


def bench_decode(B: int, n0: int, model: str = "medium", seed: int = 0) -> dict:
    """Greedy decode steps of the reference-calibrated checkpoint over B
    utterances (seeded random INT8 mel): the time of steps n0 .. n0+32 as
    t(decode of n0 + 32 steps) - t(decode of n0 steps), best of three, each
    step one CUDA-graph replay (self-attention over n0+3 .. n0+35 keys)."""
    from .checkpoint import load_calibrated
    from .model import WhisperIntB200
    dims, sd = load_calibrated(model)
    m = WhisperIntB200(dims, sd)
    del sd
    g = torch.Generator().manual_seed(seed)
    mel = torch.randint(-60, 60, (B, dims.n_mels, 2 * dims.n_audio_ctx), dtype=torch.int8, generator=g).cuda()
    xa = m.encoder(mel)
    rs = m._enc_ws[B]["rs_xa"]

    def run(n):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        m.decode(xa, rs, n, use_graph=True)
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1)

    n1 = n0 + 32
    run(n0), run(n1)  # graph capture
    ms = (min(run(n1) for _ in range(3)) - min(run(n0) for _ in range(3))) / 32
    return {"op": "decode", "model": model, "B": B, "steps": [n0, n1], "ms_per_step": round(ms, 4),
            "tok_per_s": round(B / ms * 1e3, 1)}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("op", choices=["gemm", "layernorm", "attention", "cross_attention", "frontend", "decode"])
    p.add_argument("--model", default="medium", help="decode: calibrated checkpoint size")
    p.add_argument("--from-step", type=int, default=16, help="decode: first timed step")
    p.add_argument("--n-mels", type=int, default=80)
    p.add_argument("--M", type=int, default=12000)
    p.add_argument("--K", type=int, default=1024)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--mode", choices=["linear8", "linear32_residual15"], default="linear8")
    p.add_argument("--tile-n", type=int, default=0, help="GEMM N tile (0: library choice)")
    p.add_argument("--gelu", choices=["none", "params", "table"], default="none",
                   help="Linear8 with per-channel GeLU from its parameters or from a lookup table")
    p.add_argument("--rowsum-out", action="store_true", help="also accumulate the output row sums")
    p.add_argument("--rows", type=int, default=1500)
    p.add_argument("--d", type=int, default=1024)
    p.add_argument("--B", type=int, default=4)
    p.add_argument("--H", type=int, default=16)
    p.add_argument("--T", type=int, default=1500)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--qk-mult", type=int, default=182, help="attention: qk requantisation multiplier")
    p.add_argument("--qk-shift", type=int, default=12, help="attention: qk requantisation shift")
    p.add_argument("--frac-bits", type=int, default=7, help="attention: shift-exp frac_bits")
    p.add_argument("--std", type=float, default=30.0, help="attention: standard deviation of Q/K/V")
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("microbench needs a CUDA device")
    torch.cuda.set_device(0)
    if a.op == "gemm":
        r = bench_gemm(a.M, a.K, a.N, a.mode, a.tile_n, a.reps, a.seed, a.gelu, a.rowsum_out)
    elif a.op == "layernorm":
        r = bench_layernorm(a.rows, a.d, a.reps, a.seed)
    elif a.op == "attention":
        r = bench_attention(a.B, a.H, a.T, a.reps, a.seed, a.qk_mult, a.qk_shift, a.frac_bits, a.std)
    elif a.op == "frontend":
        r = bench_frontend(a.B, a.n_mels, a.reps, a.seed)
    elif a.op == "decode":
        r = bench_decode(a.B, a.from_step, a.model, a.seed)
    else:
        r = bench_cross_attention(a.B, a.H, a.T, a.reps, a.seed)
    if _lib.device_status(clear=True) != 0:
        raise SystemExit("a device-side wait timed out")
    print(json.dumps(r))


if __name__ == "__main__":
    main()
