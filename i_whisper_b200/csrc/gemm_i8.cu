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
//                 lane quadrant) and half of the BN columns, applies the
//                 requantisation of the layer (bias, zero point, MULH,
//                 rounding shift, clamp, optional GeLU / Residual15 /
//                 positional add) and stores straight to global memory,
//                 then releases the buffer on `tempty[b]`.
// The two TMEM buffers let the epilogue of tile i overlap the MMAs of
// tile i+1. All waits are bounded (iw_sm100.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
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

template <int BN>
struct GemmCfg {
    static constexpr int STAGES = BN >= 256 ? 4 : 6;
    static constexpr int A_BYTES = kBlockM * kBlockK;
    static constexpr int B_BYTES = BN * kBlockK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
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

template <int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, const EpiParams p) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::STAGE_BYTES);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_slot + 1;

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
        const int half = ew >> 2;
        const int row = quad * 32 + lane;
        int buf = 0;
        uint32_t bphase = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&tfull[buf], bphase);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) { if (lane == 0) *abort_flag = 1; break; }
            tc_fence_after();
            const int m0 = (tile / n_tiles) * kBlockM;
            const int n0 = (tile % n_tiles) * BN;
            const int m = m0 + row;
#pragma unroll 1
            for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
                const int nc = n0 + c * 32;
                if (nc >= N) break;  // warp-uniform
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + c * 32), acc);
                tmem_ld_wait();
                epi_chunk<MODE>(p, m, nc, acc, M, N);
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

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int BN, int MODE>
static cudaError_t launch_t(const GemmShape &g, const EpiParams &p, cudaStream_t stream) {
    using Cfg = GemmCfg<BN>;
    CUtensorMap ta, tb;
    cudaError_t e = make_tmap_2d_u8(&ta, g.x, (uint64_t)g.K, (uint64_t)g.M, (uint64_t)g.ldx, kBlockK, kBlockM);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u8(&tb, g.w, (uint64_t)g.K, (uint64_t)g.N, (uint64_t)g.ldw, kBlockK, BN);
    if (e != cudaSuccess) return e;
    static bool attr_set = false;
    if (!attr_set) {
        e = cudaFuncSetAttribute(gemm_i8_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int tiles = ((g.M + kBlockM - 1) / kBlockM) * ((g.N + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gemm_i8_kernel<BN, MODE><<<grid, kThreads, Cfg::SMEM, stream>>>(ta, tb, g.M, g.N, g.K, p);
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_mode(const GemmShape &g, const EpiParams &p, cudaStream_t stream, int bn) {
    if (bn == 64) return launch_t<64, MODE>(g, p, stream);
    if (bn == 128) return launch_t<128, MODE>(g, p, stream);
    return launch_t<256, MODE>(g, p, stream);
}

cudaError_t gemm_i8_launch(const GemmShape &g, EpiMode mode, const EpiParams &p, cudaStream_t stream, int bn_hint) {
    if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaErrorInvalidValue;
    if ((g.ldx % 16) != 0 || (g.ldw % 16) != 0 || (g.K % 16) != 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(g.x) & 15) || (reinterpret_cast<uintptr_t>(g.w) & 15)) return cudaErrorMisalignedAddress;
    int bn = bn_hint;
    if (bn == 0) {
        // Prefer wide tiles; fall back to narrower ones when the grid would
        // leave most SMs idle.
        const long m_tiles = (g.M + kBlockM - 1) / kBlockM;
        bn = 256;
        if (m_tiles * ((g.N + 255) / 256) < num_sms() / 2) bn = 128;
        if (m_tiles * ((g.N + 127) / 128) < num_sms() / 2) bn = 64;
    }
    switch (mode) {
    case EPI_ACC32: return launch_mode<EPI_ACC32>(g, p, stream, bn);
    case EPI_L8: return launch_mode<EPI_L8>(g, p, stream, bn);
    case EPI_L32: return launch_mode<EPI_L32>(g, p, stream, bn);
    case EPI_L32_RES: return launch_mode<EPI_L32_RES>(g, p, stream, bn);
    }
    return cudaErrorInvalidValue;
}

}  // namespace iw
