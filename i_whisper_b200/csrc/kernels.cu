// kernels.cu -- bandwidth-bound kernels of the integer path: row sums,
// LayerNorm32, GeLU, Residual15, Add+Requant15 / embedding gather, im2col
// for the conv stem, the CUDA-core attention used for decode-shaped
// problems, and the reference-layout attention stages.
#include <cuda_runtime.h>

#include <cstdint>

#include "iw_common.cuh"
#include "kernels.cuh"

namespace iw {

// ---------------------------------------------------------------------------
// Row sums of an int8 matrix (zero-point term of Linear8/32, linear.py:89-91)
// ---------------------------------------------------------------------------
__global__ void rowsum_i8_kernel(const int8_t *__restrict__ x, int64_t ldx, int M, int K, int32_t *__restrict__ out) {
    pdl_wait();
    pdl_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const int8_t *r = x + (int64_t)warp * ldx;
    int32_t s = 0;
    if ((K & 3) == 0 && (reinterpret_cast<uintptr_t>(r) & 3) == 0) {
        const int32_t *r4 = reinterpret_cast<const int32_t *>(r);
        for (int i = lane; i < K / 4; i += 32) s += __dp4a(r4[i], 0x01010101, 0);
    } else {
        for (int i = lane; i < K; i += 32) s += r[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[warp] = s;
}

cudaError_t rowsum_i8(const int8_t *x, int64_t ldx, int M, int K, int32_t *out, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    const int threads = 256;
    const int blocks = (M * 32 + threads - 1) / threads;
    return launch_pdl(rowsum_i8_kernel, blocks, threads, 0, st, x, ldx, M, K, out);
}

// ---------------------------------------------------------------------------
// LayerNorm32 (layernorm_scalar.cpp:464-624). One warp per row; the row
// lives in registers (D/128 groups of 4 int16 per lane).
// ---------------------------------------------------------------------------
template <int D>
IW_DEV int32_t norm_reduce(int32_t x) {
    // layernorm_scalar.cpp:14-56
    if constexpr (D == 384) return (x + (x >> 2) + (x >> 3)) >> 9;
    else if constexpr (D == 512) return x >> 9;
    else if constexpr (D == 768) return (x + (x >> 2) + (x >> 3)) >> 10;
    else if constexpr (D == 1024) return x >> 10;
    else return (x + (x >> 1)) >> 11;  // 1280
}

template <int D>
IW_DEV int64_t norm_reduce64(int64_t x) {
    // layernorm_scalar.cpp:58-90 (LayerNorm64)
    if constexpr (D == 384) return (x + (x >> 2) + (x >> 3)) >> 9;
    else if constexpr (D == 512) return x >> 9;
    else if constexpr (D == 768) return (x + (x >> 2) + (x >> 3)) >> 10;
    else if constexpr (D == 1024) return x >> 10;
    else return (x + (x >> 1)) >> 11;  // 1280
}

IW_DEV int32_t warp_sum(int32_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
IW_DEV int32_t warp_max(int32_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// L64: the LayerNorm64 research variant (layernorm_scalar.cpp:626-825):
// int64 sum of the unshifted centred squares, FISR of that variance, and the
// normalise shift ln_shift + additional_offset; the element chain is shared.
// The kernel is issue-bound: registers are capped for seven 4-warp CTAs per
// SM (28 warps; 1.3% faster than 24 at d = 1024, 2% at 1280).
template <int D, bool L64>
__global__ void __launch_bounds__(128, 7) layernorm_kernel(const int16_t *__restrict__ x, int64_t ldx,
                                                           const int8_t *__restrict__ gamma,
                                                           const int32_t *__restrict__ beta, LnParams p,
                                                           int8_t *__restrict__ y, int64_t ldy, int rows,
                                                           int32_t *__restrict__ rowsum_out,
                                                           int32_t *__restrict__ rowsum_zero) {
    pdl_wait();
    pdl_launch();
    constexpr int G = D / 128;  // groups of 4 elements per lane
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int16_t *xr = x + (int64_t)row * ldx;
    int32_t v[G * 4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const uint2 u = *reinterpret_cast<const uint2 *>(xr + (g * 32 + lane) * 4);
        v[4 * g + 0] = (int16_t)(u.x & 0xFFFF);
        v[4 * g + 1] = (int16_t)(u.x >> 16);
        v[4 * g + 2] = (int16_t)(u.y & 0xFFFF);
        v[4 * g + 3] = (int16_t)(u.y >> 16);
    }
    int32_t s = 0;
#pragma unroll
    for (int i = 0; i < G * 4; ++i) s += v[i];
    s = warp_sum(s);
    const int32_t mean = norm_reduce<D>(s);
    int32_t inv;
    uint32_t nshift;
    if constexpr (!L64) {
        // The reference squares in int32 (centered_square, wrapping for
        // |x - mean| > 46340). For INT15 rows every square is exact and
        // non-negative and the rounding shift by the even renorm shift rs
        // (<= 16) needs no sign term; a row with a wrapped (negative) square
        // takes the signed form.
        // |x - mean| <= 65535, so every square is exact as uint32: their
        // unsigned max is the row's max square, and a row has a wrapped
        // (negative int32) square exactly when that max is >= 2^31
        uint32_t mxu = 0;
        int32_t sq[G * 4];
#pragma unroll
        for (int i = 0; i < G * 4; ++i) {
            v[i] -= mean;
            sq[i] = wmul(v[i], v[i]);
            mxu = max(mxu, (uint32_t)sq[i]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) mxu = max(mxu, __shfl_xor_sync(0xffffffffu, mxu, o));
        const bool wrapped = (mxu >> 31) != 0;
        int32_t mx = (int32_t)mxu;
        if (wrapped) {
            // the reference's max over the int32 (wrapped) squares
            mx = 0;
#pragma unroll
            for (int i = 0; i < G * 4; ++i) mx = max(mx, sq[i]);
            mx = warp_max(mx);
        }
        int32_t rs = bit_length_nonneg(mx) - 16;
        rs = rs < 0 ? 0 : rs;
        rs = (rs + 1) & ~1;
        const int32_t rs_rnd = rs ? (1 << (rs - 1)) : 0;
        int32_t vs = 0;
        if (!wrapped) {
#pragma unroll
            for (int i = 0; i < G * 4; ++i) vs = wadd(vs, (sq[i] + rs_rnd) >> rs);
        } else {
#pragma unroll
            for (int i = 0; i < G * 4; ++i) vs = wadd(vs, rrs(sq[i], (uint32_t)rs));
        }
        vs = warp_sum(vs);
        const int32_t var = norm_reduce<D>(vs);
        inv = fisr(var, p.rsqrt_offset);
        nshift = (uint32_t)(p.ln_shift + (rs >> 1));
    } else {
        // |x - mean| <= 65535, so each square fits uint32 exactly
        uint64_t vs = 0;
#pragma unroll
        for (int i = 0; i < G * 4; ++i) {
            v[i] -= mean;
            vs += (uint64_t)((uint32_t)v[i] * (uint32_t)v[i]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
        const int64_t var64 = norm_reduce64<D>((int64_t)vs);
        if (var64 > (int64_t)INT32_MAX && lane == 0) {
            if (p.overflow) atomicExch(p.overflow, 1);
            else atomicOr(&g_device_status, IW_DEVERR_LN64_OVERFLOW);
        }
        inv = fisr((int32_t)var64, p.rsqrt_offset);
        nshift = (uint32_t)(p.ln_shift + p.additional_offset);
    }
    // (v * inv) * ln_mult wraps mod 2^32 like v * (inv * ln_mult)
    const int32_t kmul = wmul(inv, p.ln_mult);
    const RrsK kn = rrs_k(nshift);
    const RrsK ko = rrs_k(p.out_shift);
    const bool fast = kn.sgn == -1 && ko.sgn == -1 && (p.out_mult >> 31) == 0;  // uniform per row
    int32_t osum = 0;
    int8_t *yr = y + (int64_t)row * ldy;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int c0 = (g * 32 + lane) * 4;
        const char4 gm = *reinterpret_cast<const char4 *>(gamma + c0);
        const int8_t gg[4] = {gm.x, gm.y, gm.z, gm.w};
        int4 bb = make_int4(0, 0, 0, 0);
        if (beta) bb = *reinterpret_cast<const int4 *>(beta + c0);
        const int32_t be[4] = {bb.x, bb.y, bb.z, bb.w};
        uint32_t packed = 0;
        if (fast) {
            // shifts in [1, 31], out multiplier below 2^31
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                int32_t t = wmul(v[4 * g + u], kmul);
                t = wadd(wadd(t, kn.rnd), t >> 31) >> kn.sh;
                t = clampi(t, -16383, 16383);
                t = wadd(wmul(t, (int32_t)gg[u]), be[u]);
                // rrs(mulh(t, m), sh) for m < 2^31: hi(t*m) has the sign of t,
                // so the rounding and its sign correction are multiply-adds
                int32_t hq;
                asm("mad.hi.s32 %0, %1, %2, %3;" : "=r"(hq) : "r"(t), "r"((int32_t)p.out_mult), "r"(ko.rnd));
                asm("mad.hi.s32 %0, %1, 1, %0;" : "+r"(hq) : "r"(t));
                t = clampi(hq >> ko.sh, -127, 127);
                osum += t;
                packed |= (uint32_t)(uint8_t)t << (8 * u);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                int32_t t = wmul(v[4 * g + u], kmul);
                t = rrs_apply(t, kn);
                t = clampi(t, -16383, 16383);
                t = wmul(t, (int32_t)gg[u]);
                t = wadd(t, be[u]);
                t = mulh(t, p.out_mult);
                t = rrs_apply(t, ko);
                t = clampi(t, -127, 127);
                osum += t;
                packed |= (uint32_t)(uint8_t)t << (8 * u);
            }
        }
        *reinterpret_cast<uint32_t *>(yr + c0) = packed;
    }
    if (rowsum_out) {
        osum = warp_sum(osum);
        if (lane == 0) rowsum_out[row] = osum;
    }
    if (rowsum_zero && lane == 0) rowsum_zero[row] = 0;
}

cudaError_t layernorm32(const int16_t *x, int64_t ldx, const int8_t *gamma, const int32_t *beta, const LnParams &p,
                        int8_t *y, int64_t ldy, int rows, int d, int32_t *rowsum_out, int32_t *rowsum_zero,
                        cudaStream_t st, bool l64) {
    if (rows <= 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(x) & 7) || (ldx & 3) || (reinterpret_cast<uintptr_t>(y) & 3) || (ldy & 3) ||
        (reinterpret_cast<uintptr_t>(gamma) & 3) || (beta && (reinterpret_cast<uintptr_t>(beta) & 15)))
        return cudaErrorMisalignedAddress;
    // one warp per row in 4-warp CTAs: decode-sized row counts spread over
    // more SMs with one warp per sub-partition, and encoder-sized ones
    // measured 2.6% faster than with 8-warp CTAs
    const int threads = 128;
    const int blocks = (rows * 32 + threads - 1) / threads;
#define IW_LN_CASE(DD)                                                                                        \
    case DD:                                                                                                  \
        if (l64)                                                                                              \
            return launch_pdl(layernorm_kernel<DD, true>, blocks, threads, 0, st, x, ldx, gamma, beta, p, y, ldy, \
                              rows, rowsum_out, rowsum_zero);                                                 \
        return launch_pdl(layernorm_kernel<DD, false>, blocks, threads, 0, st, x, ldx, gamma, beta, p, y, ldy,    \
                          rows, rowsum_out, rowsum_zero);
    switch (d) {
        IW_LN_CASE(384)
        IW_LN_CASE(512)
        IW_LN_CASE(768)
        IW_LN_CASE(1024)
        IW_LN_CASE(1280)
    default: return cudaErrorInvalidValue;
    }
#undef IW_LN_CASE
}

// LayerNorm statistics only (layernorm32_stats_scalar): mean, variance,
// renorm shift per row. Any width the reference accepts.
__global__ void ln_stats_kernel(const int16_t *__restrict__ x, int rows, int d, int32_t *mean_o, int32_t *var_o,
                                int32_t *rs_o) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int16_t *xr = x + (int64_t)row * d;
    int32_t s = 0;
    for (int c = lane; c < d; c += 32) s += xr[c];
    s = warp_sum(s);
    int32_t mean;
    switch (d) {
    case 384: mean = norm_reduce<384>(s); break;
    case 512: mean = norm_reduce<512>(s); break;
    case 768: mean = norm_reduce<768>(s); break;
    case 1024: mean = norm_reduce<1024>(s); break;
    default: mean = norm_reduce<1280>(s); break;
    }
    int32_t mx = 0;
    for (int c = lane; c < d; c += 32) {
        int32_t ce = (int32_t)xr[c] - mean;
        mx = max(mx, wmul(ce, ce));
    }
    mx = warp_max(mx);
    int32_t rs = bit_length_nonneg(mx) - 16;
    rs = rs < 0 ? 0 : rs;
    rs = (rs + 1) & ~1;
    int32_t vs = 0;
    for (int c = lane; c < d; c += 32) {
        int32_t ce = (int32_t)xr[c] - mean;
        vs = wadd(vs, rrs(wmul(ce, ce), (uint32_t)rs));
    }
    vs = warp_sum(vs);
    int32_t var;
    switch (d) {
    case 384: var = norm_reduce<384>(vs); break;
    case 512: var = norm_reduce<512>(vs); break;
    case 768: var = norm_reduce<768>(vs); break;
    case 1024: var = norm_reduce<1024>(vs); break;
    default: var = norm_reduce<1280>(vs); break;
    }
    if (lane == 0) {
        mean_o[row] = mean;
        var_o[row] = var;
        rs_o[row] = rs;
    }
}

cudaError_t layernorm32_stats(const int16_t *x, int rows, int d, int32_t *mean, int32_t *var, int32_t *rs,
                              cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    ln_stats_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(x, rows, d, mean, var, rs);
    return cudaGetLastError();
}

// LayerNorm64 statistics (layernorm_scalar.cpp:230-297): the LayerNorm32
// mean and the width-divided int64 sum of unshifted centred squares.
__global__ void ln64_stats_kernel(const int16_t *__restrict__ x, int rows, int d, int32_t *mean_o, int64_t *var_o) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int16_t *xr = x + (int64_t)row * d;
    int32_t s = 0;
    for (int c = lane; c < d; c += 32) s += xr[c];
    s = warp_sum(s);
    int32_t mean;
    switch (d) {
    case 384: mean = norm_reduce<384>(s); break;
    case 512: mean = norm_reduce<512>(s); break;
    case 768: mean = norm_reduce<768>(s); break;
    case 1024: mean = norm_reduce<1024>(s); break;
    default: mean = norm_reduce<1280>(s); break;
    }
    uint64_t vs = 0;
    for (int c = lane; c < d; c += 32) {
        const int32_t ce = (int32_t)xr[c] - mean;
        vs += (uint64_t)((uint32_t)ce * (uint32_t)ce);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
    int64_t var;
    switch (d) {
    case 384: var = norm_reduce64<384>((int64_t)vs); break;
    case 512: var = norm_reduce64<512>((int64_t)vs); break;
    case 768: var = norm_reduce64<768>((int64_t)vs); break;
    case 1024: var = norm_reduce64<1024>((int64_t)vs); break;
    default: var = norm_reduce64<1280>((int64_t)vs); break;
    }
    if (lane == 0) {
        mean_o[row] = mean;
        var_o[row] = var;
    }
}

cudaError_t layernorm64_stats(const int16_t *x, int rows, int d, int32_t *mean, int64_t *var, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    ln64_stats_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(x, rows, d, mean, var);
    return cudaGetLastError();
}

__global__ void fisr_kernel(const int32_t *x, int32_t *y, int64_t n, uint32_t off) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = fisr(x[i], off);
}

cudaError_t fisr_vec(const int32_t *x, int32_t *y, int64_t n, uint32_t off, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fisr_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n, off);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// GeLU (gelu_scalar.cpp:10-181), standalone.
// ---------------------------------------------------------------------------
__global__ void gelu_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, int64_t n, int channels,
                            GeluParams g) {
    __shared__ uint8_t lut[16];
    if (threadIdx.x < 16) lut[threadIdx.x] = g.lut[threadIdx.x];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % channels);
        const int a = g.n_in == 1 ? 0 : c;
        const int b = g.n_out == 1 ? 0 : c;
        y[i] = (int8_t)gelu_one(x[i], lut, g.mi[a], (uint32_t)clampi(g.si[a], 0, 32), g.mo[b],
                                (uint32_t)clampi(g.so[b], 0, 32));
    }
}

cudaError_t gelu(const int8_t *x, int8_t *y, int64_t n, int channels, const GeluParams &g, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    gelu_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, y, n, channels, g);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Residual15 (residual15_scalar.cpp:9-27), standalone.
// ---------------------------------------------------------------------------
__global__ void residual15_kernel(const int32_t *__restrict__ br, const int16_t *__restrict__ r, uint32_t m,
                                  int16_t *__restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int32_t b = wadd(br[i], wmul((int32_t)r[i], (int32_t)m));
        y[i] = (int16_t)clampi(rrs_pos(b, 15), -16383, 16383);
    }
}

cudaError_t residual15(const int32_t *br, const int16_t *r, uint16_t m, int16_t *y, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    residual15_kernel<<<(unsigned)blocks, 256, 0, st>>>(br, r, m, y, n);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Requantise-only debug paths (linear8_requant_scalar, linear8_scalar.cpp:130-150,
// via fixedpoint::requant; rounding_rshift_debug, pybind.cpp:22-43):
// with `mult` set, y[m,n] = rrs(mulh(x[m,n], mult[n]), (u32)shift[n]) with no
// clamp; without it, y = rrs(x, shamt) elementwise (M*N elements).
// ---------------------------------------------------------------------------
__global__ void requant_rows_kernel(const int32_t *__restrict__ x, const uint32_t *__restrict__ mult,
                                    const int8_t *__restrict__ shift, uint32_t shamt, int32_t *__restrict__ y,
                                    int64_t n, int64_t N) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (mult) {
            const int64_t c = i % N;
            y[i] = rrs(mulh(x[i], mult[c]), (uint32_t)(int32_t)shift[c]);
        } else {
            y[i] = rrs(x[i], shamt);
        }
    }
}

cudaError_t requant_rows(const int32_t *x, const uint32_t *mult, const int8_t *shift, uint32_t shamt, int32_t *y,
                         int64_t n, int64_t N, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    requant_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, mult, shift, shamt, y, n, N);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Add + requant to INT15 (add_requant15_scalar.cpp:29-80). With `tokens`
// set, the int8 input row is gathered from the embedding table
// (TextDecoder_int.forward, model_int.py:1411-1428) and the addend row is
// pe[offset + t]; `offset_dev` (optional) supplies the offset from device
// memory so the launch can be replayed by a CUDA graph.
// ---------------------------------------------------------------------------
__global__ void add_requant15_kernel(const int8_t *__restrict__ x, const int64_t *__restrict__ tokens,
                                     const int8_t *__restrict__ addend, const uint16_t *__restrict__ mult,
                                     const int8_t *__restrict__ shift, int16_t *__restrict__ y, int B, int T, int C,
                                     int n_mult, int n_shift, int offset, const int32_t *offset_dev) {
    pdl_wait();
    pdl_launch();
    const int64_t total = (int64_t)B * T * C;
    const int off = offset_dev ? *offset_dev : offset;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const int64_t bt = i / C;
        const int t = (int)(bt % T);
        int32_t xv;
        if (tokens) xv = x[tokens[bt] * C + c];
        else xv = x[i];
        int32_t v = xv + (int32_t)addend[(int64_t)(off + t) * C + c];
        v = wmul(v, (int32_t)mult[n_mult == 1 ? 0 : c]);
        const int32_t s = shift[n_shift == 1 ? 0 : c];
        v = rrs(v, (uint32_t)(s > 0 ? s : 0));
        y[i] = (int16_t)clampi(v, -16383, 16383);
    }
}

cudaError_t add_requant15(const int8_t *x, const int64_t *tokens, const int8_t *addend, const uint16_t *mult,
                          const int8_t *shift, int16_t *y, int B, int T, int C, int n_mult, int n_shift, int offset,
                          const int32_t *offset_dev, cudaStream_t st) {
    const int64_t total = (int64_t)B * T * C;
    if (total <= 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    return launch_pdl(add_requant15_kernel, (unsigned)blocks, 256, 0, st, x, tokens, addend, mult, shift, y, B, T, C, n_mult, n_shift,
                                                           offset, offset_dev);
}

// ---------------------------------------------------------------------------
// im2col for the conv stem (conv1d_scalar.cpp:42-104 ordering: column
// cin*K + k holds x[cin, t*stride - pad + k], zero outside [0, Tin)).
// `channels_last` selects an input stored [B, Tin, Cin] instead of
// [B, Cin, Tin]. The output row stride `ldo` may exceed Cin*K (zero pad).
// ---------------------------------------------------------------------------
__global__ void im2col_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ out, int B, int Cin, int Tin, int K,
                              int stride, int pad, int Tout, int64_t ldo, int channels_last) {
    pdl_wait();
    pdl_launch();
    const int64_t cols = ldo;
    const int64_t total = (int64_t)B * Tout * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t col = i % cols;
        const int64_t bt = i / cols;
        const int t = (int)(bt % Tout);
        const int b = (int)(bt / Tout);
        int8_t v = 0;
        if (col < (int64_t)Cin * K) {
            const int c = (int)(col / K), k = (int)(col % K);
            const int pos = t * stride - pad + k;
            if (pos >= 0 && pos < Tin)
                v = channels_last ? x[((int64_t)b * Tin + pos) * Cin + c] : x[((int64_t)b * Cin + c) * Tin + pos];
        }
        out[i] = v;
    }
}

cudaError_t im2col(const int8_t *x, int8_t *out, int B, int Cin, int Tin, int K, int stride, int pad, int Tout,
                   int64_t ldo, int channels_last, cudaStream_t st) {
    const int64_t total = (int64_t)B * Tout * ldo;
    if (total <= 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 16384) blocks = 16384;
    return launch_pdl(im2col_kernel, (unsigned)blocks, 256, 0, st, x, out, B, Cin, Tin, K, stride, pad, Tout, ldo, channels_last);
}

// Failure-path self-test: one thread waits, through the same bounded
// mbar_wait every tcgen05 kernel uses, on a barrier nothing arrives on. The
// wait gives up after the current bound, records IW_DEVERR_WAIT_TIMEOUT in
// the device status word and the kernel returns: no fault, no hang.
__global__ void selftest_wait_kernel(int *gave_up) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        *gave_up = mbar_wait(&bar, 0) ? 0 : 1;
    }
}

cudaError_t selftest_wait(int *gave_up, cudaStream_t st) {
    selftest_wait_kernel<<<1, 32, 0, st>>>(gave_up);
    return cudaGetLastError();
}

// Channel-first [B][C][T] -> channels-last [B][T + front + back][C] with
// `front` zero rows before and `back` after each window (the input of a
// convolution run as a windowed GEMM). A 32x32 tile per block through
// shared memory: coalesced reads along T, coalesced writes along C.
__global__ void channels_last_pad_kernel(const int8_t *__restrict__ x, int B, int C, int T, int front, int back,
                                         int8_t *__restrict__ out) {
    pdl_wait();
    pdl_launch();
    __shared__ int8_t tile[32][33];
    const int b = blockIdx.z;
    const int Tp = T + front + back;
    const int u0 = blockIdx.x * 32, c0 = blockIdx.y * 32;  // padded-row and channel origin
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, t = u0 + tx - front;
        tile[i][tx] = (c < C && t >= 0 && t < T) ? x[((int64_t)b * C + c) * T + t] : (int8_t)0;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int u = u0 + i, c = c0 + tx;
        if (u < Tp && c < C) out[((int64_t)b * Tp + u) * C + c] = tile[tx][i];
    }
}

cudaError_t channels_last_pad(const int8_t *x, int B, int C, int T, int front, int back, int8_t *out,
                              cudaStream_t st) {
    if (B <= 0 || C <= 0 || T <= 0) return cudaSuccess;
    dim3 grid((T + front + back + 31) / 32, (C + 31) / 32, B);
    return launch_pdl(channels_last_pad_kernel, grid, 256, 0, st, x, B, C, T, front, back, out);
}

// 2-D copy into a zero-padded buffer (row stride ldo >= cols).
__global__ void pad_rows_kernel(const int8_t *__restrict__ x, int64_t rows, int64_t cols, int8_t *__restrict__ out,
                                int64_t ldo) {
    const int64_t total = rows * ldo;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ldo, c = i % ldo;
        out[i] = c < cols ? x[r * cols + c] : (int8_t)0;
    }
}

cudaError_t pad_rows(const int8_t *x, int64_t rows, int64_t cols, int8_t *out, int64_t ldo, cudaStream_t st) {
    const int64_t total = rows * ldo;
    if (total <= 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 16384) blocks = 16384;
    pad_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, rows, cols, out, ldo);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Fused integer attention on CUDA cores (MultiHeadAttention_int.qkv_attention,
// model_int.py:774-1042; attention_scalar.cpp:216-813), head_dim 64.
// One CTA handles QB query rows of one (batch, head): QK^T + requant +
// row max (scores kept in shared memory), shift-exp + row sum, P.V,
// FISR^2 normalisation and the AV requant, written to [B, Tq, H*64].
// Used for decode-shaped problems (few query rows), where streaming K and V
// from HBM is the whole cost: four lanes share one 64-byte key or value row
// (one 16-byte load each, so a warp instruction reads eight whole rows),
// and kAttnU rows per lane are in flight before any arithmetic. A value row
// whose probabilities are all zero contributes nothing to P.V and is not
// read at all.
// ---------------------------------------------------------------------------
static constexpr int kAttnThreads = 256;
static constexpr int kAttnWarps = kAttnThreads / 32;
static constexpr int kAttnU = 4;                   // 64-key groups in flight per lane
static constexpr int kAttnKeysPerPass = kAttnThreads / 4;

// 16-byte asynchronous global -> shared copy (L2 only); a thread waits for
// its own copies with cp_async_wait<n> (all but the n most recent groups).
IW_DEV void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}
IW_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
IW_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kAttnRing = 3;  // K chunks of kAttnU*64 keys: one computed, two in flight

IW_DEV int4 ld_nc_v4(const int8_t *p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// c + sum over the four bytes of (unsigned a_i) * (signed b_i)
IW_DEV int32_t dp4a_us(uint32_t a, int32_t b, int32_t c) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// RING: K streams through a cp.async shared-memory ring (long key sequences,
// where the scores pass is bound by load latency); otherwise direct loads,
// which keep the shared-memory footprint (and so occupancy) of short ones.
template <int QB, bool RING>
__global__ void __launch_bounds__(kAttnThreads) attn_cc_kernel(AttnArgs a) {
    pdl_wait();
    pdl_launch();
    extern __shared__ uint8_t smem[];
    const int Tk = a.Tk_dev ? *a.Tk_dev : a.Tk;
    const int Tq = a.Tq;
    const int h = blockIdx.y, b = blockIdx.z;
    const int q0 = blockIdx.x * QB;
    const int nq = min(QB, Tq - q0);
    if (nq <= 0) return;
    constexpr int kChunk = kAttnU * kAttnKeysPerPass;        // keys per K chunk
    int8_t *kring = reinterpret_cast<int8_t *>(smem);        // [kAttnRing][kChunk][64] when RING
    int16_t *s = reinterpret_cast<int16_t *>(smem + (RING ? kAttnRing * kChunk * 64 : 0));  // [QB][Tk]
    uint8_t *pp = reinterpret_cast<uint8_t *>(s + QB * Tk);  // [QB][Tk]
    __shared__ int32_t red[QB][kAttnWarps];
    __shared__ int32_t rowv[QB][2];
    __shared__ int32_t pv_part[kAttnWarps][QB][64];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sub = lane & 3;                  // which 16 bytes of the 64-byte row
    const int slot = warp * 8 + (lane >> 2);   // key within a group of kAttnKeysPerPass

    int32_t qv[QB][4];
#pragma unroll
    for (int r = 0; r < QB; ++r) {
        int4 t = make_int4(0, 0, 0, 0);
        if (r < nq)
            t = *reinterpret_cast<const int4 *>(a.q + (int64_t)b * a.q_bs + (int64_t)(q0 + r) * a.ldq +
                                                (int64_t)h * a.q_hs + 16 * sub);
        qv[r][0] = t.x, qv[r][1] = t.y, qv[r][2] = t.z, qv[r][3] = t.w;
    }

    // pass 1: scores + row max
    int32_t lmax[QB];
#pragma unroll
    for (int r = 0; r < QB; ++r) lmax[r] = -32768;
    const uint32_t qsh = (uint32_t)(a.qk_shift > 0 ? a.qk_shift : 0);
    const int8_t *kb = a.k + (int64_t)b * a.k_bs + (int64_t)h * a.k_hs + 16 * sub;
    // With RING each thread copies exactly the 16-byte pieces it computes on,
    // so it only waits for its own copies (no block barrier) and the loads in
    // flight hold no registers.
    const int nchunks = (Tk + kChunk - 1) / kChunk;
    auto issue = [&](int c) {
        if (!RING) return;
        if (c < nchunks) {
#pragma unroll
            for (int u = 0; u < kAttnU; ++u) {
                const int jl = u * kAttnKeysPerPass + slot, j = c * kChunk + jl;
                if (j < Tk) cp_async16(kring + ((c % kAttnRing) * kChunk + jl) * 64 + 16 * sub, kb + (int64_t)j * a.ldk);
            }
        }
        cp_async_commit();  // possibly empty: keeps the group count uniform
    };
    for (int c = 0; c < kAttnRing - 1; ++c) issue(c);
    for (int c = 0; c < nchunks; ++c) {
        const int j0 = c * kChunk;
        int4 kk[kAttnU];
        if constexpr (RING) {
            cp_async_wait<kAttnRing - 2>();  // chunk c has landed
#pragma unroll
            for (int u = 0; u < kAttnU; ++u) {
                const int jl = u * kAttnKeysPerPass + slot;
                kk[u] = j0 + jl < Tk
                            ? *reinterpret_cast<const int4 *>(kring + ((c % kAttnRing) * kChunk + jl) * 64 + 16 * sub)
                            : make_int4(0, 0, 0, 0);
            }
        } else {
#pragma unroll
            for (int u = 0; u < kAttnU; ++u) {
                const int j = j0 + u * kAttnKeysPerPass + slot;
                kk[u] = j < Tk ? ld_nc_v4(kb + (int64_t)j * a.ldk) : make_int4(0, 0, 0, 0);
            }
        }
        issue(c + kAttnRing - 1);
#pragma unroll
        for (int u = 0; u < kAttnU; ++u) {
            const int j = j0 + u * kAttnKeysPerPass + slot;
#pragma unroll
            for (int r = 0; r < QB; ++r) {
                int32_t acc = __dp4a(kk[u].x, qv[r][0], 0);
                acc = __dp4a(kk[u].y, qv[r][1], acc);
                acc = __dp4a(kk[u].z, qv[r][2], acc);
                acc = __dp4a(kk[u].w, qv[r][3], acc);
                acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                acc += __shfl_xor_sync(0xffffffffu, acc, 2);
                if (r < nq && j < Tk) {
                    const int qi = Tk - Tq + q0 + r;  // absolute query position
                    bool masked = false;
                    if (a.mask_mode == 1) masked = j > qi;
                    else if (a.mask_mode == 2) masked = a.mask[(int64_t)(q0 + r) * Tk + j] != 0;
                    int16_t sv = -32768;
                    if (!masked) {
                        const int32_t t = rrs(wmul(acc, (int32_t)a.qk_mult), qsh);
                        sv = (int16_t)clampi(t, -32768, 32767);
                        lmax[r] = max(lmax[r], (int32_t)sv);
                    }
                    if (sub == (r & 3)) s[r * Tk + j] = sv;
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < QB; ++r) {
        const int32_t m = warp_max(lmax[r]);
        if (lane == 0) red[r][warp] = m;
    }
    __syncthreads();
    if (tid < QB) {
        int32_t m = -32768;
        for (int w = 0; w < kAttnWarps; ++w) m = max(m, red[tid][w]);
        rowv[tid][0] = (int16_t)(m + 1);  // int16 wrap of row max + 1
    }
    __syncthreads();
    // pass 2: shift-exp + row sum
    int32_t lsum[QB];
#pragma unroll
    for (int r = 0; r < QB; ++r) lsum[r] = 0;
    for (int j = tid; j < Tk; j += kAttnThreads) {
#pragma unroll
        for (int r = 0; r < QB; ++r) {
            if (r < nq) {
                const int qi = Tk - Tq + q0 + r;
                bool masked = false;
                if (a.mask_mode == 1) masked = j > qi;
                else if (a.mask_mode == 2) masked = a.mask[(int64_t)(q0 + r) * Tk + j] != 0;
                const int32_t e = masked ? 0 : shift_exp_one(s[r * Tk + j], rowv[r][0], a.frac_bits);
                pp[r * Tk + j] = (uint8_t)e;
                lsum[r] += e;
            }
        }
    }
#pragma unroll
    for (int r = 0; r < QB; ++r) {
        const int32_t v = warp_sum(lsum[r]);
        if (lane == 0) red[r][warp] = v;
    }
    __syncthreads();
    if (tid < QB) {
        int32_t v = 0;
        for (int w = 0; w < kAttnWarps; ++w) v += red[tid][w];
        rowv[tid][1] = v;
    }
    // pass 3: P.V, lane (slot, sub) accumulating dims 16*sub .. 16*sub+15.
    int32_t acc[QB][16];
#pragma unroll
    for (int r = 0; r < QB; ++r)
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[r][e] = 0;
    const int8_t *vb = a.v + (int64_t)b * a.v_bs + (int64_t)h * a.v_hs + 16 * sub;
    for (int j0 = 0; j0 < Tk; j0 += kAttnU * kAttnKeysPerPass) {
        int4 vv[kAttnU];
        uint32_t pw[kAttnU][QB];
#pragma unroll
        for (int u = 0; u < kAttnU; ++u) {
            const int j = j0 + u * kAttnKeysPerPass + slot;
            uint32_t any = 0;
#pragma unroll
            for (int r = 0; r < QB; ++r) {
                pw[u][r] = (j < Tk && r < nq) ? (uint32_t)pp[r * Tk + j] : 0u;
                any |= pw[u][r];
            }
            vv[u] = any ? ld_nc_v4(vb + (int64_t)j * a.ldv) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kAttnU; ++u) {
            const int32_t w4[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
            for (int r = 0; r < QB; ++r) {
#pragma unroll
                for (int w = 0; w < 4; ++w)
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        acc[r][4 * w + e] = dp4a_us(pw[u][r] << (8 * e), w4[w], acc[r][4 * w + e]);
            }
        }
    }
    // reduce over the eight key slots of the warp (lanes with equal sub)
#pragma unroll
    for (int r = 0; r < QB; ++r)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            int32_t v = acc[r][e];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            acc[r][e] = v;
        }
    if (lane < 4) {
#pragma unroll
        for (int r = 0; r < QB; ++r)
#pragma unroll
            for (int e = 0; e < 16; ++e) pv_part[warp][r][16 * sub + e] = acc[r][e];
    }
    __syncthreads();
    const uint32_t avs = (uint32_t)clampi(a.av_shift, 0, 32);
    static_assert(QB * 64 <= kAttnThreads, "one output value per thread");
    if (tid < QB * 64) {
        const int r = tid / 64, d = tid % 64;  // r is uniform within a warp
        int32_t o = 0;
        if (r < nq) {
            uint32_t sum = 0;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) sum += (uint32_t)pv_part[w][r][d];
            const int32_t inv = fisr(rowv[r][1], a.rsqrt_offset);
            int32_t v = rrs(wmul((int32_t)sum, inv), a.rsqrt_offset);
            v = rrs(wmul(v, inv), a.rsqrt_offset);
            v = rrs(wmul(v, (int32_t)a.av_mult), avs);
            o = clampi(v, -127, 127);
            a.out[(int64_t)b * a.o_bs + (int64_t)(q0 + r) * a.ldo + (int64_t)h * a.o_hs + d] = (int8_t)o;
        }
        if (a.rowsum_out) {
            // this head's share of the output row's sum (the next GEMM's
            // zero-point term), added to rowsum_out[b*Tq + q]
            const int32_t s = warp_sum(o);
            if (lane == 0 && r < nq) atomicAdd(a.rowsum_out + (int64_t)b * Tq + q0 + r, s);
        }
    }
}

template <int QB, bool RING>
static cudaError_t attention_cc_launch(const AttnArgs &a, int B, int H, cudaStream_t st) {
    const int tk_cap = a.Tk_cap > 0 ? a.Tk_cap : a.Tk;
    const size_t smem = (RING ? (size_t)kAttnRing * kAttnU * kAttnKeysPerPass * 64 : 0) + (size_t)QB * tk_cap * 3;
    static SmemLimit lim;
    cudaError_t e = raise_smem_limit(attn_cc_kernel<QB, RING>, smem, lim);
    if (e != cudaSuccess) return e;
    dim3 grid((a.Tq + QB - 1) / QB, H, B);
    return launch_pdl(attn_cc_kernel<QB, RING>, grid, kAttnThreads, smem, st, a);
}

// One decode query (Tq == 1) over at most 512 keys. A CTA of eight warps
// serves G = 1, 2, 4 or 8 warps per (batch, head), chosen on the device from
// the key count (the smallest G with Tk <= 32*G; 8 above 128 keys), so 8/G
// pairs per CTA. Warp s of a pair takes keys s*32 + lane (and 256 + s*32 +
// lane when Tk > 256) and issues its key rows (16-byte loads, lane = key)
// and the value rows of the same 32 keys (4-byte loads, half-warp = one
// 64-byte row) before any arithmetic, so a pair costs one memory round trip
// instead of one per group of keys. Row max and row sum combine across the
// pair's warps in shared memory, and so do the int32 P.V partials (integer
// sums: the order does not change them). Same integer steps as
// attn_cc_kernel (qk_requant_rowmax, shift_exp, pv_norm_requant).
constexpr int kAttnDecWarps = 8;
__global__ void __launch_bounds__(32 * kAttnDecWarps, 4) attn_dec_kernel(AttnArgs a, int B, int H) {
    pdl_wait();
    pdl_launch();
    __shared__ int32_t s_red[2][kAttnDecWarps];
    __shared__ int32_t s_pv[kAttnDecWarps][64];
    const int Tk = a.Tk_dev ? *a.Tk_dev : a.Tk;
    const int G = Tk <= 32 ? 1 : Tk <= 64 ? 2 : Tk <= 128 ? 4 : 8;  // warps per pair (CTA-uniform)
    const int per = kAttnDecWarps / G;                              // pairs per CTA
    if ((int)blockIdx.x * per >= B * H) return;  // the whole CTA, before any barrier
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int hw = lane >> 4, dl = lane & 15;
    const int pl = w / G, sub = w - pl * G;      // pair within the CTA, warp within the pair
    const int pair = (int)blockIdx.x * per + pl;
    const bool live = pair < B * H;              // warp-uniform
    const int b = live ? pair / H : 0, h = live ? pair - (pair / H) * H : 0;
    const int8_t *kb = a.k + (int64_t)b * a.k_bs + (int64_t)h * a.k_hs;
    const int8_t *vb = a.v + (int64_t)b * a.v_bs + (int64_t)h * a.v_hs + 4 * dl;
    const int8_t *qp = a.q + (int64_t)b * a.q_bs + (int64_t)h * a.q_hs;
    const int kt = live ? Tk : 0;                // keys this warp may read
    // round 0: this warp's keys and their value rows, all loads in flight
    const int j0 = sub * 32 + lane;
    int4 kk[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) kk[c] = j0 < kt ? ld_nc_v4(kb + (int64_t)j0 * a.ldk + 16 * c) : make_int4(0, 0, 0, 0);
    int32_t vw[16];
#pragma unroll
    for (int s2 = 0; s2 < 16; ++s2) {
        const int j = sub * 32 + 2 * s2 + hw;
        vw[s2] = j < kt ? __ldg(reinterpret_cast<const int32_t *>(vb + (int64_t)j * a.ldv)) : 0;
    }
    int4 qv[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) qv[c] = live ? *reinterpret_cast<const int4 *>(qp + 16 * c) : make_int4(0, 0, 0, 0);
    const uint32_t qsh = (uint32_t)(a.qk_shift > 0 ? a.qk_shift : 0);
    // score of key j (int16 after the requant; -32768 when masked or missing)
    auto score = [&](int j, const int4 (&k4)[4]) -> int32_t {
        if (j >= kt || (a.mask_mode == 2 && a.mask[j] != 0)) return -32768;
        int32_t acc = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            acc = __dp4a(k4[c].x, qv[c].x, acc);
            acc = __dp4a(k4[c].y, qv[c].y, acc);
            acc = __dp4a(k4[c].z, qv[c].z, acc);
            acc = __dp4a(k4[c].w, qv[c].w, acc);
        }
        // Tq == 1: the query sits at position Tk - 1, so a causal mask hides nothing
        return clampi(rrs(wmul(acc, (int32_t)a.qk_mult), qsh), -32768, 32767);
    };
    const int32_t sv0 = score(j0, kk);
    const bool two = Tk > 32 * kAttnDecWarps;  // CTA-uniform (G == 8)
    const int j1 = 32 * kAttnDecWarps + j0;
    int32_t sv1 = -32768;
    if (two) {
#pragma unroll
        for (int c = 0; c < 4; ++c) kk[c] = j1 < kt ? ld_nc_v4(kb + (int64_t)j1 * a.ldk + 16 * c) : make_int4(0, 0, 0, 0);
        sv1 = score(j1, kk);
    }
    // masked and missing keys hold -32768, which leaves the max of the
    // unmasked scores unchanged (-32768 for a row with none, as in the
    // reference's qk_requant_rowmax)
    int32_t m = warp_max(max(sv0, sv1));
    if (lane == 0) s_red[0][w] = m;
    __syncthreads();
    m = s_red[0][pl * G];
    for (int i = 1; i < G; ++i) m = max(m, s_red[0][pl * G + i]);
    const int32_t rmax1 = (int16_t)(m + 1);  // int16 wrap of row max + 1
    auto pexp = [&](int j, int32_t sv) -> int32_t {
        const bool masked = j >= kt || (a.mask_mode == 2 && a.mask[j] != 0);
        return masked ? 0 : shift_exp_one(sv, rmax1, a.frac_bits);
    };
    const int32_t e0 = pexp(j0, sv0);
    const int32_t e1 = two ? pexp(j1, sv1) : 0;
    const int32_t ls = warp_sum(e0 + e1);
    if (lane == 0) s_red[1][w] = ls;
    // P.V: half-warp hw takes keys of parity hw, lane accumulates dims 4*dl..4*dl+3
    int32_t acc4[4] = {0, 0, 0, 0};
#pragma unroll
    for (int s2 = 0; s2 < 16; ++s2) {
        const uint32_t pj = (uint32_t)__shfl_sync(0xffffffffu, e0, 2 * s2 + hw);
#pragma unroll
        for (int c = 0; c < 4; ++c) acc4[c] = dp4a_us(pj << (8 * c), vw[s2], acc4[c]);
    }
    if (two) {
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
            const int j = 32 * kAttnDecWarps + sub * 32 + 2 * s2 + hw;
            vw[s2] = j < kt ? __ldg(reinterpret_cast<const int32_t *>(vb + (int64_t)j * a.ldv)) : 0;
        }
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
            const uint32_t pj = (uint32_t)__shfl_sync(0xffffffffu, e1, 2 * s2 + hw);
#pragma unroll
            for (int c = 0; c < 4; ++c) acc4[c] = dp4a_us(pj << (8 * c), vw[s2], acc4[c]);
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) acc4[c] += __shfl_xor_sync(0xffffffffu, acc4[c], 16);
    if (hw == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) s_pv[w][4 * dl + c] = acc4[c];
    }
    __syncthreads();
    if (sub != 0 || !live) return;
    int32_t rowsum = 0;
    for (int i = 0; i < G; ++i) rowsum += s_red[1][pl * G + i];
    const int32_t inv = fisr(rowsum, a.rsqrt_offset);
    const uint32_t avs = (uint32_t)clampi(a.av_shift, 0, 32);
    uint32_t packed = 0;
    int32_t osum = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t sum = 0;
        for (int i = 0; i < G; ++i) sum += (uint32_t)s_pv[pl * G + i][4 * dl + c];
        int32_t v = rrs(wmul((int32_t)sum, inv), a.rsqrt_offset);
        v = rrs(wmul(v, inv), a.rsqrt_offset);
        v = rrs(wmul(v, (int32_t)a.av_mult), avs);
        v = clampi(v, -127, 127);
        osum += v;
        packed |= (uint32_t)(uint8_t)v << (8 * c);
    }
    if (hw == 0)
        *reinterpret_cast<uint32_t *>(a.out + (int64_t)b * a.o_bs + (int64_t)h * a.o_hs + 4 * dl) = packed;
    if (a.rowsum_out) {
        const int32_t s = warp_sum(hw == 0 ? osum : 0);
        if (lane == 0) atomicAdd(a.rowsum_out + b, s);
    }
}

cudaError_t attention_cc(const AttnArgs &a, int B, int H, cudaStream_t st) {
    if (B <= 0 || H <= 0 || a.Tq <= 0) return cudaSuccess;
    // single decode query over a short key sequence (decoder self-attention):
    // one to eight warps per (batch, head); 4-byte V loads need 4-byte
    // aligned rows, 16-byte K and Q loads 16-byte aligned ones
    const int cap = a.Tk_cap > 0 ? a.Tk_cap : a.Tk;
    const bool v_al = ((reinterpret_cast<uintptr_t>(a.v) | (uintptr_t)a.ldv | (uintptr_t)a.v_bs | (uintptr_t)a.v_hs) & 3) == 0;
    const bool o_al = ((reinterpret_cast<uintptr_t>(a.out) | (uintptr_t)a.o_bs | (uintptr_t)a.o_hs) & 3) == 0;
    const bool k_al = ((reinterpret_cast<uintptr_t>(a.k) | (uintptr_t)a.ldk | (uintptr_t)a.k_bs | (uintptr_t)a.k_hs) & 15) == 0 &&
                      ((reinterpret_cast<uintptr_t>(a.q) | (uintptr_t)a.q_bs | (uintptr_t)a.q_hs) & 15) == 0;
    if (a.Tq == 1 && cap <= 512 && v_al && o_al && k_al)
        return launch_pdl(attn_dec_kernel, B * H, 32 * kAttnDecWarps, 0, st, a, B, H);
    // one query row per CTA for decode steps; four otherwise (each CTA
    // re-reads K and V of its head, so wider query blocks save traffic)
    // (the K ring pays from ~1000 keys: measured on decode cross-attention
    // over 1500 encoder states, neutral-to-negative on short self-attention)
    const bool ring = (a.Tk_cap > 0 ? a.Tk_cap : a.Tk) >= 1024;
    if (a.Tq <= 2) return ring ? attention_cc_launch<1, true>(a, B, H, st) : attention_cc_launch<1, false>(a, B, H, st);
    return ring ? attention_cc_launch<4, true>(a, B, H, st) : attention_cc_launch<4, false>(a, B, H, st);
}

// ---------------------------------------------------------------------------
// KV-cache append (the torch.cat of Whisper_int.install_kv_cache_hooks,
// model_int.py:1604-1610, as an in-place write into a preallocated cache).
// ---------------------------------------------------------------------------
__global__ void kv_append_kernel(const int8_t *__restrict__ src, int64_t lds, int k_col, int v_col,
                                 int8_t *__restrict__ kc, int8_t *__restrict__ vc, int B, int H, int T, int Tcap,
                                 int pos, const int32_t *pos_dev) {
    pdl_wait();
    pdl_launch();
    const int p0 = pos_dev ? *pos_dev : pos;
    const int64_t total = (int64_t)B * T * H * 16;  // int32 words per K (and per V)
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int w = (int)(i % 16);
        const int64_t r = i / 16;
        const int h = (int)(r % H);
        const int64_t bt = r / H;
        const int t = (int)(bt % T);
        const int b = (int)(bt / T);
        const int8_t *row = src + bt * lds;
        const int64_t dst = (((int64_t)b * H + h) * Tcap + p0 + t) * 64 + 4 * w;
        reinterpret_cast<int32_t *>(kc + dst)[0] = reinterpret_cast<const int32_t *>(row + k_col + h * 64)[w];
        reinterpret_cast<int32_t *>(vc + dst)[0] = reinterpret_cast<const int32_t *>(row + v_col + h * 64)[w];
    }
}

cudaError_t kv_append(const int8_t *src, int64_t lds, int k_col, int v_col, int8_t *kc, int8_t *vc, int B, int H,
                      int T, int Tcap, int pos, const int32_t *pos_dev, cudaStream_t st) {
    const int64_t total = (int64_t)B * T * H * 16;
    if (total <= 0) return cudaSuccess;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    return launch_pdl(kv_append_kernel, (unsigned)blocks, 256, 0, st, src, lds, k_col, v_col, kc, vc, B, H, T, Tcap, pos, pos_dev);
}

// ---------------------------------------------------------------------------
// One greedy step on the device: the logit filters SuppressBlank,
// SuppressTokens and ApplyTimestampRules (decoding.py:426-510) on the
// dequantised logits q/alpha (model_int.py:1482-1483), then GreedyDecoder
// (decoding.py:280-296): first index of the maximum, EOT kept once emitted.
// One CTA per utterance.
// ---------------------------------------------------------------------------
static constexpr int kGreedyThreads = 512;

IW_DEV float block_reduce_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) r += red[w];
    return r;
}

// Best (largest int8 logit, then smallest index) of two candidates.
IW_DEV void best_merge(int &q, int &i, int oq, int oi) {
    if (oq > q || (oq == q && oi < i)) { q = oq; i = oi; }
}

IW_DEV void block_best(int &q, int &i, int *qred, int *ired) {
#pragma unroll
    for (int o = 16; o; o >>= 1) best_merge(q, i, __shfl_xor_sync(0xffffffffu, q, o), __shfl_xor_sync(0xffffffffu, i, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) { qred[threadIdx.x >> 5] = q; ired[threadIdx.x >> 5] = i; }
    __syncthreads();
    q = qred[0], i = ired[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best_merge(q, i, qred[w], ired[w]);
}

// One greedy step per utterance (GreedyDecoder.update after the logit
// filters SuppressBlank, SuppressTokens and ApplyTimestampRules,
// decoding.py:280-296 and 426-510). The logits are INT8 values q scaled by
// 1/alpha (alpha > 0), so the float logit is a monotone function of q and
// the log-softmax sums of ApplyTimestampRules need only a histogram of the
// 256 possible values: one pass over the row gathers, for the tokens no
// rule suppresses, the histogram of all of them and of the timestamp
// tokens, and the best text and best timestamp token (largest q, then
// smallest index, as torch.argmax). Every log-probability is then formed
// with the same float operations as the per-token formula.
__global__ void __launch_bounds__(kGreedyThreads) greedy_step_kernel(GreedyArgs g) {
    pdl_wait();
    pdl_launch();
    const int b = blockIdx.x;
    const int tid = threadIdx.x;
    __shared__ uint32_t hist[2][256];  // [0]: every allowed token, [1]: allowed timestamp tokens
    __shared__ float red[32];
    __shared__ int qred[32], ired[32];
    for (int i = tid; i < 512; i += kGreedyThreads) hist[i >> 8][i & 255] = 0;
    int32_t *st = g.state + 4 * b;
    const int n = st[0], last = st[1], pen = st[2], last_ts_val = st[3];
    const int tb = g.timestamp_begin;
    const bool at_begin = (n == 0);
    const bool last_ts = n >= 1 && last >= tb;
    const bool pen_ts = n < 2 || pen >= tb;
    int ts_hi = -1;  // timestamps in [tb, ts_hi) are forbidden
    if (last_ts_val >= 0) ts_hi = (last_ts && !pen_ts) ? last_ts_val : last_ts_val + 1;
    const int8_t *lg = g.logits + (int64_t)b * g.ld;
    auto allowed = [&](int i) -> bool {
        if (at_begin) {
            if (i == g.eot) return false;
            for (int u = 0; u < g.n_blank; ++u)
                if (g.blank[u] == i) return false;
        }
        if ((g.suppress_bits[i >> 5] >> (i & 31)) & 1u) return false;
        if (i == g.no_timestamps) return false;
        if (last_ts) {
            if (pen_ts) {
                if (i >= tb) return false;
            } else if (i < g.eot) {
                return false;
            }
        }
        if (i >= tb && i < ts_hi) return false;
        if (at_begin) {
            if (i < tb) return false;
            if (g.max_initial_timestamp_index >= 0 && i > tb + g.max_initial_timestamp_index) return false;
        }
        return true;
    };
    __syncthreads();
    int tq = -1000, ti = 0x7fffffff;  // best text token
    int sq = -1000, si = 0x7fffffff;  // best timestamp token
    for (int i = tid; i < g.V; i += kGreedyThreads) {
        if (!allowed(i)) continue;
        const int q = lg[i];
        atomicAdd(&hist[0][q + 128], 1u);
        if (i >= tb) {
            atomicAdd(&hist[1][q + 128], 1u);
            if (q > sq) sq = q, si = i;
        } else if (q > tq) {
            tq = q, ti = i;
        }
    }
    block_best(tq, ti, qred, ired);
    block_best(sq, si, qred, ired);
    const bool any_text = ti != 0x7fffffff, any_ts = si != 0x7fffffff;
    // log_softmax over the allowed logits
    const float mx = (!any_text && !any_ts) ? -INFINITY : (float)max(any_text ? tq : -1000, any_ts ? sq : -1000) / g.alpha;
    float se = 0.f;
    float vbin = 0.f;
    uint32_t c_all = 0, c_ts = 0;
    if (tid < 256) {
        vbin = (float)(tid - 128) / g.alpha;
        c_all = hist[0][tid];
        c_ts = hist[1][tid];
        if (c_all) se = (float)c_all * expf(vbin - mx);
    }
    se = block_reduce_sum(se, red);
    const float lse = logf(se);
    // timestamp mass against the best text token (decoding.py:500-510)
    const float m2 = any_ts ? (float)sq / g.alpha - mx - lse : -INFINITY;
    const float mt = any_text ? (float)tq / g.alpha - mx - lse : -INFINITY;
    float s2 = 0.f;
    if (tid < 256 && any_ts && c_ts) s2 = (float)c_ts * expf((vbin - mx - lse) - m2);
    s2 = block_reduce_sum(s2, red);
    const float ts_lp = any_ts ? m2 + logf(s2) : -INFINITY;
    const bool force_ts = ts_lp > mt;
    if (tid == 0) {
        int bq = -1000, bidx = 0x7fffffff;
        if (!force_ts) best_merge(bq, bidx, tq, ti);
        best_merge(bq, bidx, sq, si);
        if (bidx == 0x7fffffff) bidx = 0;
        const int col = *g.step_dev;
        const int64_t prev = g.tokens[(int64_t)b * g.ld_tok + col - 1];
        const int64_t nxt = (prev == g.eot) ? (int64_t)g.eot : (int64_t)bidx;
        g.tokens[(int64_t)b * g.ld_tok + col] = nxt;
        g.next[b] = nxt;
        st[0] = n + 1;
        st[2] = last;
        st[1] = (int32_t)nxt;
        if (nxt >= tb) st[3] = (int32_t)nxt;
    }
}

cudaError_t greedy_step(const GreedyArgs &g, int B, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    return launch_pdl(greedy_step_kernel, B, kGreedyThreads, 0, st, g);
}

__global__ void add_i32_kernel(int32_t *p, int32_t v) {
    pdl_wait();
    pdl_launch(); *p += v; }

cudaError_t add_i32(int32_t *p, int32_t v, cudaStream_t st) {
    return launch_pdl(add_i32_kernel, 1, 1, 0, st, p, v);
}

// ---------------------------------------------------------------------------
// Reference-layout attention stages (attention_torch.cpp), any head_dim.
// ---------------------------------------------------------------------------
// qk_requant_rowmax_scalar (attention_scalar.cpp:216-343)
__global__ void qk_rowmax_kernel(const int8_t *q, const int8_t *k, const uint8_t *mask, int16_t *qk, int16_t *rmax1,
                                 int H, int Tq, int Tk, int D, uint32_t mult, uint32_t sh) {
    const int64_t row = blockIdx.x;  // (b*H + h)*Tq + i
    const int i = (int)(row % Tq);
    const int64_t bh = row / Tq;
    const int8_t *qr = q + row * D;
    int32_t lm = -32768;
    for (int j = threadIdx.x; j < Tk; j += blockDim.x) {
        int16_t out;
        if (mask && mask[(int64_t)i * Tk + j]) {
            out = -32768;
        } else {
            const int8_t *kr = k + (bh * Tk + j) * D;
            int32_t acc = 0;
            for (int d = 0; d < D; ++d) acc += (int32_t)qr[d] * (int32_t)kr[d];
            out = (int16_t)clampi(rrs(wmul(acc, (int32_t)mult), sh), -32768, 32767);
            lm = max(lm, (int32_t)out);
        }
        qk[row * Tk + j] = out;
    }
    __shared__ int32_t red[32];
    lm = warp_max(lm);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = lm;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t m = -32768;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
        rmax1[row] = (int16_t)(m + 1);
    }
}

cudaError_t qk_requant_rowmax(const int8_t *q, const int8_t *k, const uint8_t *mask, int16_t *qk, int16_t *rmax1,
                              int B, int H, int Tq, int Tk, int D, uint8_t mult, int32_t shift, cudaStream_t st) {
    const int64_t rows = (int64_t)B * H * Tq;
    if (rows <= 0) return cudaSuccess;
    qk_rowmax_kernel<<<(unsigned)rows, 128, 0, st>>>(q, k, mask, qk, rmax1, H, Tq, Tk, D, mult,
                                                     (uint32_t)(shift > 0 ? shift : 0));
    return cudaGetLastError();
}

// shift_exp_scalar (attention_scalar.cpp:388-560)
__global__ void shift_exp_kernel(const int16_t *x, const int16_t *rmax1, const uint8_t *mask, uint8_t *p,
                                 int32_t *rowsum, int Tq, int Tk, int fb) {
    const int64_t row = blockIdx.x;
    const int i = (int)(row % Tq);
    const int32_t xm = rmax1[row];
    int32_t ls = 0;
    for (int j = threadIdx.x; j < Tk; j += blockDim.x) {
        int32_t e = 0;
        if (!(mask && mask[(int64_t)i * Tk + j])) e = shift_exp_one(x[row * Tk + j], xm, fb);
        p[row * Tk + j] = (uint8_t)e;
        ls += e;
    }
    __shared__ int32_t red[32];
    ls = warp_sum(ls);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ls;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t v = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[w];
        rowsum[row] = v;
    }
}

cudaError_t shift_exp(const int16_t *x, const int16_t *rmax1, const uint8_t *mask, uint8_t *p, int32_t *rowsum, int B,
                      int H, int Tq, int Tk, int fb, cudaStream_t st) {
    const int64_t rows = (int64_t)B * H * Tq;
    if (rows <= 0) return cudaSuccess;
    shift_exp_kernel<<<(unsigned)rows, 128, 0, st>>>(x, rmax1, mask, p, rowsum, Tq, Tk, fb);
    return cudaGetLastError();
}

// pv_norm_requant_scalar (attention_scalar.cpp:676-813); negative row sums
// are flagged in *bad (the reference throws).
__global__ void pv_norm_kernel(const uint8_t *p, const int8_t *vt, const int32_t *rowsum, uint32_t avm, uint32_t avs,
                               uint32_t off, int8_t *out, int H, int Tq, int Tk, int D, int *bad) {
    const int64_t row = blockIdx.x;  // (b*H + h)*Tq + i
    const int i = (int)(row % Tq);
    const int64_t bh = row / Tq;
    const int h = (int)(bh % H);
    const int64_t b = bh / H;
    const int32_t sum = rowsum[row];
    if (sum < 0) {
        if (threadIdx.x == 0) atomicExch(bad, 1);
        return;
    }
    const int32_t inv = fisr(sum, off);
    const uint8_t *pr = p + row * Tk;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const int8_t *vr = vt + (bh * D + d) * Tk;
        uint32_t acc = 0;
        for (int j = 0; j < Tk; ++j) acc += (uint32_t)((int32_t)pr[j] * (int32_t)vr[j]);
        int32_t v = rrs(wmul((int32_t)acc, inv), off);
        v = rrs(wmul(v, inv), off);
        v = rrs(wmul(v, (int32_t)avm), avs);
        out[((b * Tq + i) * H + h) * D + d] = (int8_t)clampi(v, -127, 127);
    }
}

cudaError_t pv_norm_requant(const uint8_t *p, const int8_t *vt, const int32_t *rowsum, uint8_t av_mult,
                            int8_t av_shift, uint32_t off, int8_t *out, int B, int H, int Tq, int Tk, int D, int *bad,
                            cudaStream_t st) {
    const int64_t rows = (int64_t)B * H * Tq;
    if (rows <= 0) return cudaSuccess;
    pv_norm_kernel<<<(unsigned)rows, 64, 0, st>>>(p, vt, rowsum, av_mult, (uint32_t)clampi(av_shift, 0, 32), off, out,
                                                  H, Tq, Tk, D, bad);
    return cudaGetLastError();
}

}  // namespace iw
