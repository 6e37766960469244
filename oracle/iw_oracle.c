/*
 * iw_oracle.c -- CPU restatement of the I-Whisper integer hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against.
 * Nothing in the product library links or loads this file.
 *
 * All arithmetic is restated from the reference kernels in
 * vcsd-lab/I-Whisper (paths relative to i_whisper/kernels/csrc/). Signed
 * 32-bit wrap-around, which the reference gets either from explicit
 * uint32 helpers or from two's-complement hardware, is written here with
 * explicit uint32 arithmetic so that the restatement has no undefined
 * behaviour. The outer loops are OpenMP-parallel so that model-sized
 * checks finish in seconds; every output element is computed by exactly one
 * thread with the same sequential inner loop, so threading cannot change a
 * result.
 *
 * Parity pinned: every function is compared with the reference's own scalar
 * kernels compiled from its sources (oracle/_ref), the reference's own
 * kernel test suite passes on it (hand-written known answers included), and
 * the model dataflow in oracle.py reproduces golden digests and greedy
 * tokens produced by the reference's Whisper_int and DecodingTask.
 */
#include "iw_oracle.h"

#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

void iwo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---- wrap helpers -------------------------------------------------------- */
static inline int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static inline int32_t wsub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
static inline int32_t wmul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }
static inline int16_t wadd16(int16_t a, int16_t b) { return (int16_t)(uint16_t)((uint16_t)a + (uint16_t)b); }
static inline int16_t wsub16(int16_t a, int16_t b) { return (int16_t)(uint16_t)((uint16_t)a - (uint16_t)b); }
static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* common/fixedpoint.h:35-44 -- high word of the signed x unsigned product */
int32_t iwo_mulh(int32_t x, uint32_t multiplier) {
    int64_t p = (int64_t)x * (int64_t)multiplier;
    return (int32_t)(p >> 32);
}

/* common/fixedpoint.h:47-87 -- shift 0 is identity, shift >= 32 gives 0,
 * otherwise add 2^(s-1) - signbit with uint32 wrap, then arithmetic shift. */
int32_t iwo_rounding_rshift(int32_t x, uint32_t shift) {
    if (shift == 0) return x;
    if (shift >= 32) return 0;
    uint32_t sign = (uint32_t)x >> 31;
    uint32_t rounding = (1u << (shift - 1)) - sign;
    int32_t v = (int32_t)((uint32_t)x + rounding);
    return v >> shift;
}

static inline int32_t requant(int32_t x, uint32_t m, uint32_t s) {
    return iwo_rounding_rshift(iwo_mulh(x, m), s);
}

static inline int32_t bit_length_nonneg(int32_t x) {
    if (x == 0) return 0;
    return 32 - __builtin_clz((uint32_t)x);
}

/* layernorm_scalar.cpp:309-343 -- int32 -> fp32 bit pattern, mantissa
 * truncated. Negative inputs follow the same formula on the unsigned bits. */
static int32_t int32_to_fp32_bits_trunc(int32_t x) {
    if (x == 0) return 0;
    int32_t e = bit_length_nonneg(x) - 1;
    uint64_t sig;
    if (e <= 23) sig = (uint64_t)(uint32_t)x << (23 - e);
    else sig = (uint64_t)(uint32_t)x >> (e - 23);
    uint32_t exponent = (uint32_t)(e + 127);
    uint32_t mant = (uint32_t)sig & 0x007FFFFFu;
    return (int32_t)((exponent << 23) | mant);
}

/* layernorm_scalar.cpp:345-381 -- fp32 bit pattern -> int32, truncating. */
static int32_t fp32_bits_to_int32_trunc(int32_t bits) {
    uint32_t raw = (uint32_t)bits;
    int32_t e = (int32_t)((raw >> 23) & 0xFFu) - 127;
    uint64_t sig = (uint64_t)((1u << 23) | (raw & 0x007FFFFFu));
    if (e < 0) return 0;
    uint64_t v;
    if (e >= 23) {
        int32_t sh = e - 23;
        /* reachable inputs give sh <= 56; larger shifts leave no low bits */
        v = sh >= 64 ? 0 : (sig << sh);
    } else {
        v = sig >> (23 - e);
    }
    return (int32_t)(uint32_t)v;
}

/* layernorm_scalar.cpp:383-437 -- integer fast inverse square root:
 * magic-constant seed in the fp32 bit domain, exponent offset, two Newton
 * steps in Q(offset) fixed point with wrapping products. */
int32_t iwo_fisr(int32_t x, uint32_t off) {
    int32_t i = int32_to_fp32_bits_trunc(x);
    i = (int32_t)0x5f3759dfu - (i >> 1);
    int32_t y = fp32_bits_to_int32_trunc((int32_t)((uint32_t)i + (off << 23)));
    int32_t three = (int32_t)(3u << off);
    for (int it = 0; it < 2; ++it) {
        int32_t xy = wmul(x, y);
        int32_t xys = iwo_rounding_rshift(xy, off);
        int32_t t = wmul(xys, y);
        int32_t corr = wsub(three, t);
        int32_t prod = wmul(y, corr);
        y = iwo_rounding_rshift(prod, off + 1);
    }
    return y;
}

void iwo_fisr_vec(const int32_t *x, int32_t *y, int64_t n, uint32_t off) {
    for (int64_t i = 0; i < n; ++i) y[i] = iwo_fisr(x[i], off);
}

/* ---- Linear8 / Linear32 -------------------------------------------------- */
static inline int32_t dot_i8(const int8_t *a, const int8_t *b, int64_t K) {
    int32_t acc = 0; /* |sum| < 2^31 for K < 2^17; wrap is implicit below */
    uint32_t accu = 0;
    int64_t k = 0;
    /* chunks of 4096 keep the int32 partial exact before folding */
    while (k < K) {
        int64_t e = K - k > 4096 ? k + 4096 : K;
        acc = 0;
        for (int64_t j = k; j < e; ++j) acc += (int32_t)a[j] * (int32_t)b[j];
        accu += (uint32_t)acc;
        k = e;
    }
    return (int32_t)accu;
}

static inline int32_t sum_i8(const int8_t *a, int64_t K) {
    uint32_t s = 0;
    for (int64_t k = 0; k < K; ++k) s += (uint32_t)(int32_t)a[k];
    return (int32_t)s;
}

/* linear8_scalar.cpp:87-127 (accum) and linear32_scalar.cpp:9-63: raw dot,
 * minus weight_zero[n] * sum(x row), plus bias[n], all in wrapping int32. */
void iwo_linear8_accum(const int8_t *x, const int8_t *w, const int32_t *bias,
                       const int8_t *wz, int32_t *y, int64_t M, int64_t K,
                       int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        const int8_t *xr = x + m * K;
        int32_t xs = wz ? sum_i8(xr, K) : 0;
        for (int64_t n = 0; n < N; ++n) {
            int32_t acc = dot_i8(xr, w + n * K, K);
            if (wz) acc = wsub(acc, wmul((int32_t)wz[n], xs));
            if (bias) acc = wadd(acc, bias[n]);
            y[m * N + n] = acc;
        }
    }
}

/* linear8_scalar.cpp:30-84 -- accum, then requant(acc, m[n], (uint32)s[n]),
 * clamp to [-127,127]. A negative int8 shift converts to a uint32 >= 32 and
 * therefore yields 0. */
void iwo_linear8(const int8_t *x, const int8_t *w, const int32_t *bias,
                 const int8_t *wz, const uint32_t *mult, const int8_t *shift,
                 int8_t *y, int64_t M, int64_t K, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        const int8_t *xr = x + m * K;
        int32_t xs = wz ? sum_i8(xr, K) : 0;
        for (int64_t n = 0; n < N; ++n) {
            int32_t acc = dot_i8(xr, w + n * K, K);
            if (wz) acc = wsub(acc, wmul((int32_t)wz[n], xs));
            if (bias) acc = wadd(acc, bias[n]);
            acc = requant(acc, mult[n], (uint32_t)(int32_t)shift[n]);
            y[m * N + n] = (int8_t)clampi(acc, -127, 127);
        }
    }
}

/* linear8_scalar.cpp:130-150 -- requant only, int32 result (no clamp). */
void iwo_linear8_requant(const int32_t *acc, const uint32_t *mult,
                         const int8_t *shift, int32_t *y, int64_t M, int64_t N) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            y[m * N + n] = requant(acc[m * N + n], mult[n], (uint32_t)(int32_t)shift[n]);
}

/* linear32_simd.cpp:231-255 (left_shift_wrap_s32 / requant32), equal to
 * linear32_scalar.cpp:65-94 for shifts in [0,63]: mulh, then a wrapping
 * left shift; a shift (as uint32) >= 32 gives 0. */
static inline int32_t requant32(int32_t acc, uint32_t m, int8_t s) {
    int32_t v = iwo_mulh(acc, m);
    uint32_t sh = (uint32_t)(int32_t)s;
    if (sh >= 32) return 0;
    return (int32_t)((uint32_t)v << sh);
}

void iwo_linear32_requant(const int32_t *acc, const uint32_t *mult,
                          const int8_t *shift, int32_t *y, int64_t M, int64_t N) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            y[m * N + n] = requant32(acc[m * N + n], mult[n], shift[n]);
}

/* linear32_scalar.cpp:96-129 */
void iwo_linear32(const int8_t *x, const int8_t *w, const int32_t *bias,
                  const int8_t *wz, const uint32_t *mult, const int8_t *shift,
                  int32_t *y, int64_t M, int64_t K, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        const int8_t *xr = x + m * K;
        int32_t xs = wz ? sum_i8(xr, K) : 0;
        for (int64_t n = 0; n < N; ++n) {
            int32_t acc = dot_i8(xr, w + n * K, K);
            if (bias) acc = wadd(acc, bias[n]);
            if (wz) acc = wsub(acc, wmul((int32_t)wz[n], xs));
            y[m * N + n] = requant32(acc, mult[n], shift[n]);
        }
    }
}

/* residual15_scalar.cpp:9-27 -- branch + residual*m (wrapping int32),
 * rounding shift by 15, clamp to +-16383. */
void iwo_residual15(const int32_t *branch, const int16_t *residual,
                    uint16_t mult, int16_t *y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        int32_t b = wadd(branch[i], wmul((int32_t)residual[i], (int32_t)mult));
        b = iwo_rounding_rshift(b, 15);
        y[i] = (int16_t)clampi(b, -16383, 16383);
    }
}

/* ---- LayerNorm32 ---------------------------------------------------------- */
/* layernorm_scalar.cpp:14-56 -- division by the width as add-of-shifts then
 * an arithmetic right shift. */
static inline int norm_reduce(int32_t x, int64_t d, int32_t *out) {
    switch (d) {
    case 384: *out = (x + (x >> 2) + (x >> 3)) >> 9; return 0;
    case 512: *out = x >> 9; return 0;
    case 768: *out = (x + (x >> 2) + (x >> 3)) >> 10; return 0;
    case 1024: *out = x >> 10; return 0;
    case 1280: *out = (x + (x >> 1)) >> 11; return 0;
    default: return -1;
    }
}

/* One row of layernorm_scalar.cpp:133-214 (stats). */
static int ln_row_stats(const int16_t *r, int64_t d, int32_t *mean_out,
                        int32_t *var_out, int32_t *rs_out) {
    uint32_t s = 0;
    for (int64_t c = 0; c < d; ++c) s += (uint32_t)(int32_t)r[c];
    int32_t mean;
    if (norm_reduce((int32_t)s, d, &mean)) return -1;
    int32_t mx = 0;
    for (int64_t c = 0; c < d; ++c) {
        int32_t ce = (int32_t)r[c] - mean;
        int32_t sq = wmul(ce, ce);
        if (sq > mx) mx = sq;
    }
    int32_t rs = bit_length_nonneg(mx) - 16;
    if (rs < 0) rs = 0;
    rs = (rs + 1) & ~1;
    uint32_t vs = 0;
    for (int64_t c = 0; c < d; ++c) {
        int32_t ce = (int32_t)r[c] - mean;
        vs += (uint32_t)iwo_rounding_rshift(wmul(ce, ce), (uint32_t)rs);
    }
    int32_t var;
    norm_reduce((int32_t)vs, d, &var);
    *mean_out = mean;
    *var_out = var;
    *rs_out = rs;
    return 0;
}

int iwo_layernorm32_stats(const int16_t *x, int32_t *mean, int32_t *var,
                          int32_t *renorm_shift, int64_t rows, int64_t d) {
    int32_t dummy;
    if (norm_reduce(0, d, &dummy)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        ln_row_stats(x + r * d, d, &mean[r], &var[r], &renorm_shift[r]);
    return 0;
}

/* layernorm_scalar.cpp:464-624 -- stats, FISR(var, offset), then per
 * element: (x-mean)*invstd*ln_m (wrapping), rounding shift by
 * ln_shift + renorm/2 (as uint32), clamp +-16383, *gamma + beta (wrapping),
 * mulh by out_m, rounding shift by out_shift (as uint32), clamp +-127. */
int iwo_layernorm32(const int16_t *x, const int8_t *gamma, const int32_t *beta,
                    uint8_t ln_mult, int8_t ln_shift, uint32_t out_mult,
                    int8_t out_shift, uint32_t rsqrt_offset, int8_t *y,
                    int64_t rows, int64_t d) {
    int32_t dummy;
    if (norm_reduce(0, d, &dummy)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int16_t *xr = x + r * d;
        int8_t *yr = y + r * d;
        int32_t mean, var, rs;
        ln_row_stats(xr, d, &mean, &var, &rs);
        int32_t inv = iwo_fisr(var, rsqrt_offset);
        int32_t nshift = (int32_t)ln_shift + (rs >> 1);
        for (int64_t c = 0; c < d; ++c) {
            int32_t v = wmul((int32_t)xr[c] - mean, inv);
            v = wmul(v, (int32_t)ln_mult);
            v = iwo_rounding_rshift(v, (uint32_t)nshift);
            v = clampi(v, -16383, 16383);
            v = wmul(v, (int32_t)gamma[c]);
            if (beta) v = wadd(v, beta[c]);
            v = iwo_mulh(v, out_mult);
            v = iwo_rounding_rshift(v, (uint32_t)(int32_t)out_shift);
            yr[c] = (int8_t)clampi(v, -127, 127);
        }
    }
    return 0;
}

/* ---- LayerNorm64 (research variant) ---------------------------------------- */
/* layernorm_scalar.cpp:58-90 -- the 64-bit width division of the unshifted
 * variance sum. */
static inline int norm_reduce64(int64_t x, int64_t d, int64_t *out) {
    switch (d) {
    case 384: *out = (x + (x >> 2) + (x >> 3)) >> 9; return 0;
    case 512: *out = x >> 9; return 0;
    case 768: *out = (x + (x >> 2) + (x >> 3)) >> 10; return 0;
    case 1024: *out = x >> 10; return 0;
    case 1280: *out = (x + (x >> 1)) >> 11; return 0;
    default: return -1;
    }
}

/* layernorm_scalar.cpp:230-297 -- the LayerNorm32 mean, then the full
 * int64 sum of centred squares (no renorm pre-shift), width-divided. */
static int ln64_row_stats(const int16_t *r, int64_t d, int32_t *mean_out, int64_t *var_out) {
    uint32_t s = 0;
    for (int64_t c = 0; c < d; ++c) s += (uint32_t)(int32_t)r[c];
    int32_t mean;
    if (norm_reduce((int32_t)s, d, &mean)) return -1;
    int64_t vs = 0;
    for (int64_t c = 0; c < d; ++c) {
        const int64_t ce = (int64_t)r[c] - (int64_t)mean;
        vs += ce * ce;
    }
    int64_t var;
    norm_reduce64(vs, d, &var);
    *mean_out = mean;
    *var_out = var;
    return 0;
}

int iwo_layernorm64_stats(const int16_t *x, int32_t *mean, int64_t *var,
                          int64_t rows, int64_t d) {
    int64_t dummy;
    if (norm_reduce64(0, d, &dummy)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) ln64_row_stats(x + r * d, d, &mean[r], &var[r]);
    return 0;
}

/* layernorm_scalar.cpp:626-825 -- FISR of the int64 variance (which must fit
 * INT32) with rsqrt_offset, normalise shift ln_shift + additional_offset
 * (no renorm term), otherwise the LayerNorm32 element chain. */
int iwo_layernorm64(const int16_t *x, const int8_t *gamma, const int32_t *beta,
                    uint8_t ln_mult, int8_t ln_shift, uint32_t out_mult,
                    int8_t out_shift, uint32_t rsqrt_offset,
                    int32_t additional_offset, int8_t *y, int64_t rows,
                    int64_t d) {
    int64_t dummy;
    if (norm_reduce64(0, d, &dummy)) return -1;
    for (int64_t r = 0; r < rows; ++r) {  /* rows in order: the first overflow stops, as in the reference */
        const int16_t *xr = x + r * d;
        int8_t *yr = y + r * d;
        int32_t mean;
        int64_t var64;
        ln64_row_stats(xr, d, &mean, &var64);
        if (var64 < 0 || var64 > (int64_t)INT32_MAX) return -2;
        const int32_t inv = iwo_fisr((int32_t)var64, rsqrt_offset);
        const int32_t nshift = (int32_t)ln_shift + additional_offset;
        for (int64_t c = 0; c < d; ++c) {
            int32_t v = wmul((int32_t)xr[c] - mean, inv);
            v = wmul(v, (int32_t)ln_mult);
            v = iwo_rounding_rshift(v, (uint32_t)nshift);
            v = clampi(v, -16383, 16383);
            v = wmul(v, (int32_t)gamma[c]);
            if (beta) v = wadd(v, beta[c]);
            v = iwo_mulh(v, out_mult);
            v = iwo_rounding_rshift(v, (uint32_t)(int32_t)out_shift);
            yr[c] = (int8_t)clampi(v, -127, 127);
        }
    }
    return 0;
}

/* ---- GeLU ----------------------------------------------------------------- */
/* gelu_scalar.cpp:10-181 -- LUT index = rrs(x*mi, clamp(si,0,32)) + 8,
 * clamped to [0,15]; y = rrs(x*lut[idx]*mo, clamp(so,0,32)), clamp +-127.
 * Parameters are per channel (last dim) or per tensor (count 1). */
void iwo_gelu(const int8_t *x, const uint8_t *lut, const uint8_t *mi,
              const int8_t *si, const uint8_t *mo, const int8_t *so,
              int8_t *y, int64_t numel, int64_t channels, int64_t n_in,
              int64_t n_out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < numel; ++i) {
        int64_t c = i % channels;
        int64_t a = n_in == 1 ? 0 : c;
        int64_t b = n_out == 1 ? 0 : c;
        int32_t idx = (int32_t)x[i] * (int32_t)mi[a];
        idx = iwo_rounding_rshift(idx, (uint32_t)clampi(si[a], 0, 32));
        idx = clampi(idx + 8, 0, 15);
        int32_t v = (int32_t)x[i] * (int32_t)lut[idx];
        v = v * (int32_t)mo[b];
        v = iwo_rounding_rshift(v, (uint32_t)clampi(so[b], 0, 32));
        y[i] = (int8_t)clampi(v, -127, 127);
    }
}

/* ---- Attention ------------------------------------------------------------ */
/* attention_scalar.cpp:130-176 -- raw QK^T, int32. */
void iwo_qk(const int8_t *q, const int8_t *k, int32_t *y, int64_t B,
            int64_t H, int64_t Tq, int64_t Tk, int64_t D) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bh = 0; bh < B * H; ++bh)
        for (int64_t i = 0; i < Tq; ++i)
            for (int64_t j = 0; j < Tk; ++j)
                y[(bh * Tq + i) * Tk + j] = dot_i8(q + (bh * Tq + i) * D, k + (bh * Tk + j) * D, D);
}

/* attention_scalar.cpp:216-343 -- requant by a u8 multiplier (wrapping
 * int32 product) and max(shift,0); clamp to int16; masked lanes are
 * INT16_MIN and are not evaluated; row max + 1 with int16 wrap. */
void iwo_qk_requant_rowmax(const int8_t *q, const int8_t *k,
                           const uint8_t *mask, int16_t *qk, int16_t *rmax1,
                           int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                           int64_t D, uint8_t mult, int32_t shift) {
    uint32_t sh = shift > 0 ? (uint32_t)shift : 0u;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bh = 0; bh < B * H; ++bh)
        for (int64_t i = 0; i < Tq; ++i) {
            const int8_t *qr = q + (bh * Tq + i) * D;
            int16_t *out = qk + (bh * Tq + i) * Tk;
            int16_t mx = -32768;
            for (int64_t j = 0; j < Tk; ++j) {
                if (mask && mask[i * Tk + j]) { out[j] = -32768; continue; }
                int32_t acc = dot_i8(qr, k + (bh * Tk + j) * D, D);
                int32_t v = wmul(acc, (int32_t)mult);
                v = iwo_rounding_rshift(v, sh);
                int16_t s = (int16_t)clampi(v, -32768, 32767);
                out[j] = s;
                if (s > mx) mx = s;
            }
            rmax1[bh * Tq + i] = wadd16(mx, 1);
        }
}

/* attention_scalar.cpp:388-560 -- shift-based exp2 of (x - rowmax1) in
 * int16 wrapping arithmetic; masked lanes and lanes with x_sub > 0 give 0.
 * The u8 results are summed per row into an int32. */
static inline uint8_t shift_exp_one(int16_t x, int16_t xm, int32_t fb) {
    int32_t scale = 1 << fb;
    int16_t xs = wsub16(x, xm);
    if (xs > 0) return 0;
    int16_t half = (int16_t)(xs >> 1);
    int16_t six = (int16_t)(xs >> 4);
    int16_t fix = wsub16(wadd16(xs, half), six);
    int16_t xi = (int16_t)(fix >> fb);
    int16_t ip = (int16_t)((int32_t)xi * scale);
    int16_t fr = (int16_t)(fix - ip);
    int16_t num = (int16_t)(scale + (int32_t)(fr >> 1));
    int16_t e;
    if (xi > 0) e = 0;
    else {
        int32_t es = -(int32_t)xi;
        e = es >= 16 ? 0 : (int16_t)(num >> es);
    }
    if (fb > 7) return (uint8_t)((int32_t)e >> (fb - 7));
    return (uint8_t)e;
}

void iwo_shift_exp(const int16_t *x, const int16_t *rmax1, const uint8_t *mask,
                   uint8_t *p, int32_t *rowsum, int64_t B, int64_t H,
                   int64_t Tq, int64_t Tk, int32_t fb) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bh = 0; bh < B * H; ++bh)
        for (int64_t i = 0; i < Tq; ++i) {
            int64_t base = (bh * Tq + i) * Tk;
            int16_t xm = rmax1[bh * Tq + i];
            int32_t s = 0;
            for (int64_t j = 0; j < Tk; ++j) {
                if (mask && mask[i * Tk + j]) { p[base + j] = 0; continue; }
                uint8_t e = shift_exp_one(x[base + j], xm, fb);
                p[base + j] = e;
                s += (int32_t)e;
            }
            rowsum[bh * Tq + i] = s;
        }
}

/* attention_scalar.cpp:590-644 -- P (u8) times V^T stored [B,H,D,Tk],
 * wrapping int32 accumulation; output [B,H,Tq,D]. */
void iwo_pv(const uint8_t *p, const int8_t *vt, int32_t *y, int64_t B,
            int64_t H, int64_t Tq, int64_t Tk, int64_t D) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bh = 0; bh < B * H; ++bh)
        for (int64_t i = 0; i < Tq; ++i)
            for (int64_t d = 0; d < D; ++d) {
                const uint8_t *pr = p + (bh * Tq + i) * Tk;
                const int8_t *vr = vt + (bh * D + d) * Tk;
                uint32_t acc = 0;
                for (int64_t j = 0; j < Tk; ++j) acc += (uint32_t)((int32_t)pr[j] * (int32_t)vr[j]);
                y[(bh * Tq + i) * D + d] = (int32_t)acc;
            }
}

/* attention_scalar.cpp:676-813 -- P.V, then two multiplies by
 * FISR(rowsum, offset) each followed by a rounding shift by offset, then the
 * AV requant (u8 multiplier, shift clamped to [0,32]), clamp +-127, written
 * in [B,Tq,H*D]. A negative row sum is an error (-1). */
int iwo_pv_norm_requant(const uint8_t *p, const int8_t *vt,
                        const int32_t *rowsum, uint8_t av_mult,
                        int8_t av_shift, uint32_t off, int8_t *y, int64_t B,
                        int64_t H, int64_t Tq, int64_t Tk, int64_t D) {
    for (int64_t i = 0; i < B * H * Tq; ++i)
        if (rowsum[i] < 0) return -1;
    uint32_t rsh = (uint32_t)clampi(av_shift, 0, 32);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bh = 0; bh < B * H; ++bh)
        for (int64_t i = 0; i < Tq; ++i) {
            int64_t b = bh / H, h = bh % H;
            int32_t inv = iwo_fisr(rowsum[bh * Tq + i], off);
            const uint8_t *pr = p + (bh * Tq + i) * Tk;
            for (int64_t d = 0; d < D; ++d) {
                const int8_t *vr = vt + (bh * D + d) * Tk;
                uint32_t acc = 0;
                for (int64_t j = 0; j < Tk; ++j) acc += (uint32_t)((int32_t)pr[j] * (int32_t)vr[j]);
                int32_t v = (int32_t)acc;
                v = iwo_rounding_rshift(wmul(v, inv), off);
                v = iwo_rounding_rshift(wmul(v, inv), off);
                v = iwo_rounding_rshift(wmul(v, (int32_t)av_mult), rsh);
                y[(b * Tq + i) * (H * D) + h * D + d] = (int8_t)clampi(v, -127, 127);
            }
        }
    return 0;
}

/* ---- Conv1d --------------------------------------------------------------- */
/* conv1d_scalar.cpp:42-104 -- bias + sum over (cin, k) of
 * x[cin, t*stride - pad + k] * w[cout, cin*K + k], zero padding, wrapping. */
static inline int32_t conv_one(const int8_t *xb, const int8_t *wr, int32_t bias,
                               int64_t Cin, int64_t Tin, int64_t K,
                               int64_t stride, int64_t pad, int64_t t) {
    uint32_t acc = (uint32_t)bias;
    int64_t o = t * stride - pad;
    for (int64_t c = 0; c < Cin; ++c)
        for (int64_t k = 0; k < K; ++k) {
            int64_t pos = o + k;
            if (pos < 0 || pos >= Tin) continue;
            acc += (uint32_t)((int32_t)xb[c * Tin + pos] * (int32_t)wr[c * K + k]);
        }
    return (int32_t)acc;
}

void iwo_conv1d_accum(const int8_t *x, const int8_t *w, const int32_t *bias,
                      int32_t *y, int64_t B, int64_t Cin, int64_t Tin,
                      int64_t Cout, int64_t K, int64_t stride, int64_t pad) {
    int64_t Tout = (Tin + 2 * pad - K) / stride + 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t oc = 0; oc < Cout; ++oc)
            for (int64_t t = 0; t < Tout; ++t)
                y[(b * Cout + oc) * Tout + t] = conv_one(x + b * Cin * Tin, w + oc * Cin * K,
                                                         bias ? bias[oc] : 0, Cin, Tin, K, stride, pad, t);
}

/* conv1d_scalar.cpp:186-288 -- accum, mulh by the layer multiplier, rounding
 * shift by max(shift,0), clamp +-127; output [B,Cout,Tout]. */
void iwo_conv1d(const int8_t *x, const int8_t *w, const int32_t *bias,
                uint32_t mult, int8_t shift, int8_t *y, int64_t B,
                int64_t Cin, int64_t Tin, int64_t Cout, int64_t K,
                int64_t stride, int64_t pad) {
    int64_t Tout = (Tin + 2 * pad - K) / stride + 1;
    uint32_t sh = shift > 0 ? (uint32_t)shift : 0u;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t oc = 0; oc < Cout; ++oc)
            for (int64_t t = 0; t < Tout; ++t) {
                int32_t v = conv_one(x + b * Cin * Tin, w + oc * Cin * K, bias ? bias[oc] : 0,
                                     Cin, Tin, K, stride, pad, t);
                v = requant(v, mult, sh);
                y[(b * Cout + oc) * Tout + t] = (int8_t)clampi(v, -127, 127);
            }
}

/* ---- Add + requant15 ------------------------------------------------------ */
/* add_requant15_scalar.cpp:29-80 -- (x + addend[t]) * m (u16, wrapping
 * int32), rounding shift by max(shift,0), clamp +-16383; per-channel or
 * per-tensor multiplier and shift. */
void iwo_add_requant15(const int8_t *x, const int8_t *addend,
                       const uint16_t *mult, const int8_t *shift, int16_t *y,
                       int64_t B, int64_t T, int64_t C, int64_t n_mult,
                       int64_t n_shift) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t t = 0; t < T; ++t)
            for (int64_t c = 0; c < C; ++c) {
                int64_t i = (b * T + t) * C + c;
                int32_t v = (int32_t)x[i] + (int32_t)addend[t * C + c];
                v = wmul(v, (int32_t)mult[n_mult == 1 ? 0 : c]);
                int32_t s = shift[n_shift == 1 ? 0 : c];
                v = iwo_rounding_rshift(v, (uint32_t)(s > 0 ? s : 0));
                y[i] = (int16_t)clampi(v, -16383, 16383);
            }
}

/* ---- Classifier ----------------------------------------------------------- */
/* classifier_scalar.cpp:56-88 */
void iwo_classifier_accum(const int8_t *x, const int8_t *w, int32_t *y,
                          int64_t M, int64_t K, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n)
        for (int64_t m = 0; m < M; ++m)
            y[m * N + n] = dot_i8(x + m * K, w + n * K, K);
}

/* classifier_scalar.cpp:91-140 -- dot, mulh, rounding shift by max(s,0),
 * clamp +-127. */
void iwo_classifier(const int8_t *x, const int8_t *w, uint32_t mult,
                    int8_t shift, int8_t *y, int64_t M, int64_t K, int64_t N) {
    uint32_t sh = shift > 0 ? (uint32_t)shift : 0u;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n)
        for (int64_t m = 0; m < M; ++m) {
            int32_t v = requant(dot_i8(x + m * K, w + n * K, K), mult, sh);
            y[m * N + n] = (int8_t)clampi(v, -127, 127);
        }
}
