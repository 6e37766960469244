// gemm_i8.cu -- persistent tcgen05 (kind::i8) GEMM for sm_100a with the
// integer requantisation epilogues of the I-Whisper linears fused in.
//
// Work split per CTA (one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer. Loads a 128x128 X tile and a BNx128 W tile
//                 per k-block into a STAGES-deep shared-memory ring
//                 (128-byte swizzle, K-major), completion on `full[s]`.
//   warp 1      : allocates TMEM (2*BN columns: two accumulator buffers),
//                 one elected lane issues tcgen05.mma 128xBNx32 per 32-deep
//                 k-step and commits to `empty[s]` (stage free) and to
//                 `tfull[b]` (accumulator ready).
//   warps 2..9  : epilogue. Warp w reads TMEM lanes 32*(w%4)..+31 (its
//                 lane quadrant) and every 4th 32-column chunk, applies the
//                 requantisation of the layer (bias, zero point, MULH,
//                 rounding shift, clamp, optional GeLU / Residual15 /
//                 positional add) and stores straight to global memory,
//                 then releases the buffer on `tempty[b]`.
// The two TMEM buffers let the epilogue of tile i overlap the MMAs of
// tile i+1. All waits are bounded (iw_sm100.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "gemm_i8.cuh"
#include "iw_common.cuh"
#include "iw_sm100.cuh"
#include "iw_tmap.cuh"

namespace iw {

static constexpr int kBlockM = 128;
static constexpr int kBlockK = 128;  // bytes = int8 elements per k-block (one swizzle atom row)
static constexpr int kEpiWarps = 8;
static constexpr int kThreads = 64 + 32 * kEpiWarps;

// FLAVOR 0: general epilogue (any EpiParams); 1: fast per-channel epilogue
// with column parameters staged in shared memory; 2: fast + GeLU table.
template <int BN, int FLAVOR>
struct GemmCfg {
    static constexpr int A_BYTES = kBlockM * kBlockK;
    static constexpr int B_BYTES = BN * kBlockK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int PARAM_BYTES = FLAVOR ? BN * 32 : 0;
    static constexpr int GTAB_BYTES = FLAVOR == 2 ? BN * 256 : 0;
    static constexpr int FIXED = 1024 + 256 + PARAM_BYTES + GTAB_BYTES;
    static constexpr int STAGES_FIT = (232448 - FIXED) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
    static_assert(STAGES >= 2, "shared memory too small");
};

IW_DEV int32_t requant32(int32_t v, uint32_t m, int8_t s) {
    // linear32_simd.cpp:231-255: mulh, then a wrapping left shift; a shift
    // that is >= 32 as uint32 (including negative int8 shifts) gives 0.
    uint32_t sh = (uint32_t)(int32_t)s;
    int32_t h = mulh(v, m);
    return sh >= 32 ? 0 : (int32_t)((uint32_t)h << sh);
}

IW_DEV bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int MODE>
IW_DEV void epi_chunk(const EpiParams &p, int m, int n0, const uint32_t (&acc)[32], int M, int N) {
    if (m >= M) return;
    const bool full = (n0 + 32 <= N);
    const int32_t rs = p.wz ? __ldg(p.rowsum + m) : 0;
    int32_t v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        int32_t a = (int32_t)acc[j];
        if (full || n < N) {
            if (p.bias) a = wadd(a, __ldg(p.bias + n));
            if (p.wz) a = wsub(a, wmul((int32_t)__ldg(p.wz + n), rs));
        }
        v[j] = a;
    }

    if constexpr (MODE == EPI_ACC32 || MODE == EPI_L32) {
        int32_t *out = reinterpret_cast<int32_t *>(p.out) + (int64_t)m * p.ldo + n0;
        if constexpr (MODE == EPI_L32) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (full || n0 + j < N) v[j] = requant32(v[j], __ldg(p.mult + n0 + j), __ldg(p.shift + n0 + j));
        }
        if (full && (p.ldo & 3) == 0 && aligned16(out)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<int4 *>(out + j) = make_int4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
            for (int j = 0; j < 32; ++j)
                if (n0 + j < N) out[j] = v[j];
        }
        return;
    } else if constexpr (MODE == EPI_L32_RES) {
        // residual15_scalar.cpp:9-27 on top of the Linear32 requant.
        const int16_t *res = p.res + (int64_t)m * p.ldr + n0;
        int16_t *out = reinterpret_cast<int16_t *>(p.out) + (int64_t)m * p.ldo + n0;
        const bool vec = full && (p.ldo & 7) == 0 && (p.ldr & 7) == 0 && aligned16(out) && aligned16(res);
        int16_t r[32];
        if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                int4 t = *reinterpret_cast<const int4 *>(res + j);
                const int16_t *tt = reinterpret_cast<const int16_t *>(&t);
#pragma unroll
                for (int u = 0; u < 8; ++u) r[j + u] = tt[u];
            }
        } else {
            for (int j = 0; j < 32; ++j) r[j] = (n0 + j < N) ? res[j] : (int16_t)0;
        }
        int16_t o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            int32_t b = (full || n0 + j < N) ? requant32(v[j], __ldg(p.mult + n0 + j), __ldg(p.shift + n0 + j)) : 0;
            b = wadd(b, wmul((int32_t)r[j], (int32_t)p.res_mult));
            o[j] = (int16_t)clampi(rrs_pos(b, 15), -16383, 16383);
        }
        if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) *reinterpret_cast<int4 *>(out + j) = *reinterpret_cast<const int4 *>(o + j);
        } else {
            for (int j = 0; j < 32; ++j)
                if (n0 + j < N) out[j] = o[j];
        }
        return;
    } else {  // EPI_L8
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int n = n0 + j;
            int32_t a;
            if (p.per_channel) {
                a = (full || n < N) ? rrs(mulh(v[j], __ldg(p.mult + n)), (uint32_t)(int32_t)__ldg(p.shift + n)) : 0;
            } else {
                a = rrs(mulh(v[j], p.smult), p.sshift);
            }
            a = clampi(a, -127, 127);
            if (p.gelu && (full || n < N)) {
                const int ci = p.gelu_in_pc ? n : 0;
                const int co = p.gelu_out_pc ? n : 0;
                a = gelu_one(a, p.lut, __ldg(p.gmi + ci), (uint32_t)clampi(__ldg(p.gsi + ci), 0, 32),
                             __ldg(p.gmo + co), (uint32_t)clampi(__ldg(p.gso + co), 0, 32));
            }
            v[j] = a;
        }
        if (p.rowsum_out) {
            int32_t s = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (full || n0 + j < N) s += v[j];
            atomicAdd(p.rowsum_out + m, s);
        }
        if (p.posadd) {
            // add_requant15_scalar.cpp:29-80 on the GeLU output.
            const int t = m % p.pe_T;
            int16_t *out = reinterpret_cast<int16_t *>(p.out) + (int64_t)m * p.ldo + n0;
            int16_t o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = n0 + j;
                int32_t a = 0;
                if (full || n < N) {
                    const int pi = p.pos_pc ? n : 0;
                    a = v[j] + (int32_t)__ldg(p.pe + (int64_t)t * N + n);
                    a = wmul(a, (int32_t)__ldg(p.pm + pi));
                    const int32_t s = __ldg(p.ps + pi);
                    a = clampi(rrs(a, (uint32_t)(s > 0 ? s : 0)), -16383, 16383);
                }
                o[j] = (int16_t)a;
            }
            if (full && (p.ldo & 7) == 0 && aligned16(out)) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) *reinterpret_cast<int4 *>(out + j) = *reinterpret_cast<const int4 *>(o + j);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (n0 + j < N) out[j] = o[j];
            }
            return;
        }
        int8_t *base = reinterpret_cast<int8_t *>(p.out);
        if (p.transpose_T) {
            const int b = m / p.transpose_T, t = m % p.transpose_T;
            for (int j = 0; j < 32; ++j)
                if (n0 + j < N) base[((int64_t)b * N + n0 + j) * p.transpose_T + t] = (int8_t)v[j];
            return;
        }
        if (p.hm_T) {
            const int b = m / p.hm_T, t = m % p.hm_T;
            const int g = n0 >> 6;
            int8_t *out = base + (((int64_t)g * p.hm_B + b) * p.hm_T + t) * 64 + (n0 & 63);
            if (full) {
                uint32_t w[8];
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    w[q] = (uint32_t)(uint8_t)v[4 * q] | ((uint32_t)(uint8_t)v[4 * q + 1] << 8) |
                           ((uint32_t)(uint8_t)v[4 * q + 2] << 16) | ((uint32_t)(uint8_t)v[4 * q + 3] << 24);
                *reinterpret_cast<uint4 *>(out) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4 *>(out + 16) = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (n0 + j < N) out[j] = (int8_t)v[j];
            }
            return;
        }
        if (p.vt_T) {
            const int b = m / p.vt_T, t = m % p.vt_T;
            const int H = N / p.vt_D;
            for (int j = 0; j < 32; ++j) {
                const int n = n0 + j;
                if (n < N) {
                    const int h = n / p.vt_D, d = n % p.vt_D;
                    base[(((int64_t)b * H + h) * p.vt_D + d) * p.ldo + t] = (int8_t)v[j];
                }
            }
            return;
        }
        int8_t *out = base + (int64_t)m * p.ldo + n0;
        if (full && (p.ldo & 15) == 0 && aligned16(out)) {
            uint32_t w[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                w[q] = (uint32_t)(uint8_t)v[4 * q] | ((uint32_t)(uint8_t)v[4 * q + 1] << 8) |
                       ((uint32_t)(uint8_t)v[4 * q + 2] << 16) | ((uint32_t)(uint8_t)v[4 * q + 3] << 24);
            *reinterpret_cast<uint4 *>(out) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4 *>(out + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
            for (int j = 0; j < 32; ++j)
                if (n0 + j < N) out[j] = (int8_t)v[j];
        }
    }
}


// ---------------------------------------------------------------------------
// Fast epilogue: per-column constants precomputed once per tile into shared
// memory so that the per-element requantisation is branch-free:
//   A = {bias, -weight_zero, multiplier (as int32), multiplier >= 2^31 ? -1 : 0}
//   Linear8:  B = {2^(s-1) or 0, s in [1,31] ? -1 : 0, s (or 0), s < 32 ? -1 : 0}
//   Linear32: B = {s (or 0), s < 32 ? -1 : 0, 0, 0}
// with s the shift as uint32 (negative int8 shifts are >= 32).
// mulh(a, m) = mulhi_signed(a, (int32)m) + (m >= 2^31 ? a : 0).
// ---------------------------------------------------------------------------
template <int BN, int MODE, int FLAVOR>
IW_DEV void stage_columns(const EpiParams &p, int n0, int N, int4 *colA, int4 *colB, int8_t *gtab, int et) {
    for (int c = et; c < BN; c += kEpiWarps * 32) {
        const int n = n0 + c;
        int4 a = make_int4(0, 0, 0, 0), b = make_int4(0, 0, 0, 0);
        if (n < N) {
            const uint32_t m = p.mult[n];
            const uint32_t sh = (uint32_t)(int32_t)p.shift[n];
            a = make_int4(p.bias ? p.bias[n] : 0, p.wz ? -(int32_t)p.wz[n] : 0, (int32_t)m, (m >> 31) ? -1 : 0);
            if (MODE == EPI_L8) {
                if (sh == 0) b = make_int4(0, 0, 0, -1);
                else if (sh < 32) b = make_int4((int32_t)(1u << (sh - 1)), -1, (int32_t)sh, -1);
            } else {
                if (sh < 32) b = make_int4((int32_t)sh, -1, 0, 0);
            }
        }
        colA[c] = a;
        colB[c] = b;
    }
    if (FLAVOR == 2) {
        const int rows = min(BN, N - n0);
        const int4 *src = reinterpret_cast<const int4 *>(p.gelu_tab + (int64_t)n0 * 256);
        int4 *dst = reinterpret_cast<int4 *>(gtab);
        for (int i = et; i < rows * 16; i += kEpiWarps * 32) dst[i] = __ldg(src + i);
    }
}

IW_DEV void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

IW_DEV int32_t u_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
IW_DEV int32_t u_mad(int32_t a, int32_t b, int32_t c) { return (int32_t)((uint32_t)a * (uint32_t)b + (uint32_t)c); }

// One 32-column chunk of row m, fast path. Returns the sum of the int8
// outputs (Linear8) for the optional row-sum output.
template <int MODE, int FLAVOR>
IW_DEV int32_t epi_fast_chunk(const EpiParams &p, int m, int nc, int cl, int32_t rs, const uint32_t (&acc)[32],
                              const int4 *colA, const int4 *colB, const int8_t *gtab, int8_t *out8) {
    int32_t osum = 0;
    if constexpr (MODE == EPI_L8) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int4 A = colA[cl + j];
            const int4 Bv = colB[cl + j];
            int32_t a = u_mad(A.y, rs, u_add((int32_t)acc[j], A.x));
            const int32_t h = u_add(__mulhi(a, A.z), a & A.w);
            int32_t t = u_add(u_add(h, Bv.x), (h >> 31) & Bv.y);
            t = (t >> Bv.z) & Bv.w;
            t = clampi(t, -127, 127);
            if constexpr (FLAVOR == 2) t = gtab[(cl + j) * 256 + t + 128];
            osum += t;
            if ((j & 3) == 0) w[j >> 2] = 0;
            w[j >> 2] |= (uint32_t)(uint8_t)t << (8 * (j & 3));
        }
        *reinterpret_cast<uint4 *>(out8) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4 *>(out8 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
    } else {  // EPI_L32_RES
        int16_t *out = reinterpret_cast<int16_t *>(p.out) + (int64_t)m * p.ldo + nc;
        const int16_t *res = p.res + (int64_t)m * p.ldr + nc;
        uint32_t r[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 t = *reinterpret_cast<const uint4 *>(res + 8 * q);
            r[4 * q] = t.x; r[4 * q + 1] = t.y; r[4 * q + 2] = t.z; r[4 * q + 3] = t.w;
        }
        uint32_t o[16];
        const int32_t rm = (int32_t)p.res_mult;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int4 A = colA[cl + j];
            const int4 Bv = colB[cl + j];
            int32_t a = u_mad(A.y, rs, u_add((int32_t)acc[j], A.x));
            const int32_t h = u_add(__mulhi(a, A.z), a & A.w);
            const int32_t br = (int32_t)((uint32_t)h << Bv.x) & Bv.y;
            const int32_t rv = (int32_t)(int16_t)((r[j >> 1] >> (16 * (j & 1))) & 0xFFFF);
            int32_t v = u_mad(rv, rm, br);
            v = u_add(u_add(v, 1 << 14), v >> 31) >> 15;
            v = clampi(v, -16383, 16383);
            if ((j & 1) == 0) o[j >> 1] = 0;
            o[j >> 1] |= (uint32_t)(uint16_t)v << (16 * (j & 1));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4 *>(out + 8 * q) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
    }
    return osum;
}

template <int BN, int MODE, int FLAVOR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, const EpiParams p) {
    using Cfg = GemmCfg<BN, FLAVOR>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::STAGE_BYTES);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    int4 *colA = reinterpret_cast<int4 *>(smem + S * Cfg::STAGE_BYTES + 256);
    int4 *colB = colA + BN;
    int8_t *gtab = reinterpret_cast<int8_t *>(smem + S * Cfg::STAGE_BYTES + 256 + Cfg::PARAM_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (M + kBlockM - 1) / kBlockM;
    const int n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int kblocks = (K + kBlockK - 1) / kBlockK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // TMEM is held: let the next kernel be scheduled, then wait for the
    // previous one before touching global memory
    pdl_launch();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, last_parity = 0;  // per stage: issued at least once / parity of last issue
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * kBlockM;
                const int n0 = (tile % n_tiles) * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(&tmA, &full[stage], sA + stage * Cfg::A_BYTES, kb * kBlockK, m0);
                    tma_load_2d(&tmB, &full[stage], sB + stage * Cfg::B_BYTES, kb * kBlockK, n0);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                }
            }
            // Before the CTA may exit, every copy this thread issued must have
            // landed (bounded wait; already complete on the normal path).
            for (int s = 0; s < S; ++s)
                if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kBlockM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t bphase = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
                if (!mbar_wait(&tempty[buf], bphase ^ 1)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int ks = 0; ks < kBlockK / 32; ++ks) {
                        mma_i8(d, sdesc_kmajor_sw128(a0 + ks * 32), sdesc_kmajor_sw128(b0 + ks * 32), idesc,
                               (kb | ks) != 0);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                }
                if (!ok) { *abort_flag = 1; break; }
                mma_commit(&tfull[buf]);
                buf ^= 1;
                if (buf == 0) bphase ^= 1;
            }
            // All MMAs issued by this thread must be complete before TMEM is
            // released (bounded wait on a dedicated barrier).
            mma_commit(drain);
            mbar_wait(drain, 0);
        }
    } else {
        const int ew = warp - 2;
        const int quad = warp & 3;
        const int slice = ew >> 2;  // which of the kEpiWarps/4 column slices this warp takes
        const int row = quad * 32 + lane;
        int buf = 0;
        uint32_t bphase = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int m0 = (tile / n_tiles) * kBlockM;
            const int n0 = (tile % n_tiles) * BN;
            const int m = m0 + row;
            if constexpr (FLAVOR != 0) {
                // Barrier A: every epilogue warp is done with the previous
                // tile. The abort flag is only written after barrier B, so all
                // warps read the same value here and leave the loop together.
                epi_bar();
                const bool stop = *abort_flag != 0;
                if (!stop) stage_columns<BN, MODE, FLAVOR>(p, n0, N, colA, colB, gtab, ew * 32 + lane);
                epi_bar();
                if (stop) break;
            }
            bool ok = mbar_wait(&tfull[buf], bphase);  // every lane: the warp stays converged
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) *abort_flag = 1;
                if constexpr (FLAVOR == 0) break;
                else continue;  // keep meeting the named barriers until all warps see the flag
            }
            tc_fence_after();
            if constexpr (FLAVOR == 0) {
#pragma unroll 1
                for (int c = slice; c < BN / 32; c += kEpiWarps / 4) {
                    const int nc = n0 + c * 32;
                    if (nc >= N) break;  // warp-uniform
                    uint32_t acc[32];
                    tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + c * 32), acc);
                    tmem_ld_wait();
                    epi_chunk<MODE>(p, m, nc, acc, M, N);
                }
            } else {
                const bool live = m < M;
                const int32_t rs = (p.wz && live) ? __ldg(p.rowsum + m) : 0;
                int8_t *row8 = nullptr;
                if constexpr (MODE == EPI_L8) {
                    if (p.hm_T) {
                        const int b = m / p.hm_T, t = m - (m / p.hm_T) * p.hm_T;
                        row8 = reinterpret_cast<int8_t *>(p.out) + ((int64_t)b * p.hm_T + t) * 64;
                    } else {
                        row8 = reinterpret_cast<int8_t *>(p.out) + (int64_t)m * p.ldo;
                    }
                }
                int32_t osum = 0;
#pragma unroll 1
                for (int c = slice; c < BN / 32; c += kEpiWarps / 4) {
                    const int nc = n0 + c * 32;
                    if (nc >= N) break;  // warp-uniform
                    uint32_t acc[32];
                    tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + c * 32), acc);
                    tmem_ld_wait();
                    if (live) {
                        int8_t *o8 = nullptr;
                        if constexpr (MODE == EPI_L8)
                            o8 = p.hm_T ? row8 + (int64_t)(nc >> 6) * p.hm_B * p.hm_T * 64 + (nc & 63) : row8 + nc;
                        osum += epi_fast_chunk<MODE, FLAVOR>(p, m, nc, c * 32, rs, acc, colA, colB, gtab, o8);
                    }
                }
                if (MODE == EPI_L8 && p.rowsum_out && live) atomicAdd(p.rowsum_out + m, osum);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            buf ^= 1;
            if (buf == 0) bphase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

bool cm_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("IW_GEMM_ROWMAJOR");
        on = (e && e[0] == '1') ? 0 : 1;
    }
    return on == 1;
}

template <int BN, int MODE, int FLAVOR>
static cudaError_t launch_t(const GemmShape &g, const EpiParams &p, cudaStream_t stream) {
    using Cfg = GemmCfg<BN, FLAVOR>;
    CUtensorMap ta, tb;
    cudaError_t e = make_tmap_2d_u8(&ta, g.x, (uint64_t)g.K, (uint64_t)g.M, (uint64_t)g.ldx, kBlockK, kBlockM);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u8(&tb, g.w, (uint64_t)g.K, (uint64_t)g.N, (uint64_t)g.ldw, kBlockK, BN);
    if (e != cudaSuccess) return e;
    static SmemLimit lim;
    e = raise_smem_limit(gemm_i8_kernel<BN, MODE, FLAVOR>, Cfg::SMEM, lim);
    if (e != cudaSuccess) return e;
    const int tiles = ((g.M + kBlockM - 1) / kBlockM) * ((g.N + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    return launch_pdl(gemm_i8_kernel<BN, MODE, FLAVOR>, grid, kThreads, Cfg::SMEM, stream, ta, tb, g.M, g.N, g.K, p);
}

template <int MODE, int FLAVOR>
static cudaError_t launch_mode(const GemmShape &g, const EpiParams &p, cudaStream_t stream, int bn) {
    if (bn == 64) return launch_t<64, MODE, FLAVOR>(g, p, stream);
    if (bn == 128) return launch_t<128, MODE, FLAVOR>(g, p, stream);
    return launch_t<256, MODE, FLAVOR>(g, p, stream);
}

// The fast epilogue covers per-channel Linear8 (optionally with a GeLU
// table, row sums and the head-major layout) and Linear32+Residual15 with
// whole 32-column chunks and 16-byte aligned rows.
static bool fast_eligible(const GemmShape &g, EpiMode mode, const EpiParams &p) {
    if (!(mode == EPI_L8 || mode == EPI_L32_RES)) return false;
    if (!p.per_channel || p.gelu || p.posadd || p.transpose_T || p.vt_T) return false;
    if (g.N % 32) return false;
    if (reinterpret_cast<uintptr_t>(p.out) & 15) return false;
    if (mode == EPI_L8 && !p.hm_T && (p.ldo % 16)) return false;
    if (mode == EPI_L32_RES && ((p.ldo % 8) || (p.ldr % 8) || (reinterpret_cast<uintptr_t>(p.res) & 15))) return false;
    if (p.hm_T && (g.N % 64)) return false;
    return true;
}

cudaError_t gemm_i8_launch(const GemmShape &g, EpiMode mode, const EpiParams &p, cudaStream_t stream, int bn_hint) {
    if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaErrorInvalidValue;
    if ((g.ldx % 16) != 0 || (g.ldw % 16) != 0 || (g.K % 16) != 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(g.x) & 15) || (reinterpret_cast<uintptr_t>(g.w) & 15)) return cudaErrorMisalignedAddress;
    if (cm_enabled()) {
        EpiParams q = p;
        if (q.transpose_T && !q.tr_out) {
            q.tr_out = reinterpret_cast<int8_t *>(q.out);
            q.tr_c0 = 0;
            q.tr_N = g.N;
            q.tr_T = q.transpose_T;
            q.tr_ld = q.transpose_T;
            q.transpose_T = 0;
        }
        if (cm_eligible(g, mode, q))
            return gemm_cm_launch(g, mode, q, stream, (bn_hint == 64 || bn_hint == 128 || bn_hint == 256) ? bn_hint : 0);
    }
    // transposed and KV-cache outputs, windowed X and accumulator signs need
    // the channel-major kernel
    if (p.tr_out || p.kv_k || g.win_rows > 0 || p.wsign) return cudaErrorInvalidValue;
    int bn = bn_hint;
    if (bn == 0) {
        // Prefer wide tiles; fall back to narrower ones when the grid would
        // leave most SMs idle.
        const long m_tiles = (g.M + kBlockM - 1) / kBlockM;
        bn = 256;
        if (m_tiles * ((g.N + 255) / 256) < num_sms() / 2) bn = 128;
        if (m_tiles * ((g.N + 127) / 128) < num_sms() / 2) bn = 64;
    }
    if (p.gelu_tab && !fast_eligible(g, mode, p)) return cudaErrorInvalidValue;
    if (fast_eligible(g, mode, p)) {
        if (mode == EPI_L8) {
            if (p.gelu_tab) return launch_mode<EPI_L8, 2>(g, p, stream, bn == 256 ? 128 : bn);
            return launch_mode<EPI_L8, 1>(g, p, stream, bn);
        }
        return launch_mode<EPI_L32_RES, 1>(g, p, stream, bn);
    }
    switch (mode) {
    case EPI_ACC32: return launch_mode<EPI_ACC32, 0>(g, p, stream, bn);
    case EPI_L8: return launch_mode<EPI_L8, 0>(g, p, stream, bn);
    case EPI_L32: return launch_mode<EPI_L32, 0>(g, p, stream, bn);
    case EPI_L32_RES: return launch_mode<EPI_L32_RES, 0>(g, p, stream, bn);
    }
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// GeLU lookup table: tab[n][x+128] = gelu_one(x) with channel n's parameters.
// ---------------------------------------------------------------------------
__global__ void gelu_table_kernel(const uint8_t *lut, const uint8_t *mi, const int8_t *si, const uint8_t *mo,
                                  const int8_t *so, int n_in, int n_out, int N, int8_t *tab) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)N * 256) return;
    const int n = (int)(i >> 8);
    const int x = (int)(i & 255) - 128;
    const int a = n_in == 1 ? 0 : n, b = n_out == 1 ? 0 : n;
    tab[i] = (int8_t)gelu_one(x, lut, mi[a], (uint32_t)clampi(si[a], 0, 32), mo[b], (uint32_t)clampi(so[b], 0, 32));
}

cudaError_t gelu_table_build(const uint8_t *lut, const uint8_t *mi, const int8_t *si, const uint8_t *mo,
                             const int8_t *so, int n_in, int n_out, int N, int8_t *tab, cudaStream_t st) {
    const int64_t total = (int64_t)N * 256;
    if (total <= 0) return cudaSuccess;
    gelu_table_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(lut, mi, si, mo, so, n_in, n_out, N, tab);
    return cudaGetLastError();
}

__global__ void gelu_table_tile_kernel(const int8_t *tab, int N, int8_t *tiled, int64_t bytes) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= bytes) return;
    const int64_t tile = i >> 15;
    const int o = (int)(i & 32767), q = o >> 13, t = (o >> 5) & 255, l = o & 31;
    const int64_t n = tile * 128 + q * 32 + l;
    tiled[i] = n < N ? tab[n * 256 + t] : (int8_t)0;
}

cudaError_t gelu_table_tile(const int8_t *tab, int N, int8_t *tiled, cudaStream_t st) {
    const int64_t bytes = (int64_t)((N + 127) / 128) * 32768;
    if (bytes <= 0) return cudaSuccess;
    gelu_table_tile_kernel<<<(unsigned)((bytes + 255) / 256), 256, 0, st>>>(tab, N, tiled, bytes);
    return cudaGetLastError();
}

}  // namespace iw
