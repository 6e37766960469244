// attn_tc.cu -- fused integer attention on the tcgen05 tensor cores (sm_100a)
// for encoder self-attention (MultiHeadAttention_int.qkv_attention,
// model_int.py:774-1042; attention_scalar.cpp:216-813), head_dim 64.
//
// One CTA computes 128 query rows of one (batch, head):
//   pass 1: S = Q K^T per 128-key block on the tensor cores; the softmax
//           warps keep the row maximum of the RAW int32 scores. The score
//           requantisation clamp16(rrs(acc * m_u8, s)) is monotonic and
//           cannot wrap for 64-wide int8 dot products (|acc*m| < 2^31), so
//           requant(max acc) == max requant(acc): one op per score.
//   pass 2: S is recomputed; each score is requantised, the int16
//           difference to rowmax+1 goes through the shift-exp as a lookup
//           table (built on the device with the same function, see
//           shift_exp_table), the u8 probabilities are summed per row and
//           written to shared memory in the tensor-core operand layout, and
//           O += P V^T runs on the tensor cores (u8 x s8 -> s32).
//   end:    O is normalised by FISR(rowsum)^2 and the AV requant, and written
//           as int8 rows [b*T + t, h*64 + d].
// The reference's online order (row max first, then exp and sum) is kept
// exactly; no rescaling of partial sums is needed.
//
// Warp roles: warp 0 TMA producer (Q once, K blocks twice, V^T blocks),
// warp 1 TMEM owner + MMA issuer, warps 2..9 softmax (thread = query row of
// its TMEM lane quadrant, two warps per quadrant split the 128 key columns).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "iw_common.cuh"
#include "iw_sm100.cuh"
#include "iw_tmap.cuh"
#include "kernels.cuh"

namespace iw {

namespace attn {

constexpr int BQ = 128;     // query rows per CTA
constexpr int BK = 128;     // keys per block
constexpr int KST = 4;      // K stages
constexpr int VST = 3;      // V^T stages
constexpr int SOFT_WARPS = 8;
constexpr int THREADS = 64 + 32 * SOFT_WARPS;
constexpr int TAB_MAX = 4096;  // entries of the shift-exp table kept in shared memory

constexpr int Q_BYTES = BQ * 64;
constexpr int K_BYTES = BK * 64;
constexpr int V_BYTES = 64 * BK;
constexpr int P_BYTES = BQ * BK;
// layout (offsets from the 1024-aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + KST * K_BYTES;
constexpr int OFF_P = OFF_V + VST * V_BYTES;
constexpr int OFF_TAB = OFF_P + 2 * P_BYTES;
constexpr int OFF_RED = OFF_TAB + TAB_MAX;  // [2][BQ] int32 cross-warp row reductions
constexpr int OFF_BAR = OFF_RED + 2 * BQ * 4;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr uint32_t TMEM_COLS = 256;  // S at columns [0,128), O at [128,192); two CTAs per SM
}  // namespace attn

struct AttnTcParams {
    int B, H, T;          // batch, heads, sequence length (queries == keys)
    int8_t *out;          // [B*T, ldo]
    int64_t ldo;
    uint32_t qk_mult;     // u8
    uint32_t qk_rnd, qk_sgn, qk_sh, qk_z;  // rrs(x, s) = (((x + rnd + ((x>>31)&sgn)) >> sh) & z)
    const uint8_t *tab;   // shift-exp table: [0] = last index T1 (zero entry), then T1+1 bytes
    uint32_t av_mult;     // u8
    uint32_t av_shift;    // clamp(av_s, 0, 32)
    uint32_t rsqrt_offset;
    int vt_ld;            // row stride (keys) of V^T
};

// K-major operand with 64-byte rows, 64-byte swizzle (8-row atoms of 512 B).
IW_DEV uint64_t sdesc_kmajor_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(512u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)4u << 61;  // SWIZZLE_64B
    return d;
}

IW_DEV void bar_soft() { asm volatile("bar.sync 1, %0;" ::"n"(attn::SOFT_WARPS * 32) : "memory"); }

IW_DEV int32_t rrs_masked(int32_t x, const AttnTcParams &p) {
    const uint32_t t = (uint32_t)x + p.qk_rnd + ((uint32_t)(x >> 31) & p.qk_sgn);
    return (int32_t)(((int32_t)t >> p.qk_sh) & (int32_t)p.qk_z);
}

__global__ void __launch_bounds__(attn::THREADS, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
    using namespace attn;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem + OFF_Q;
    uint8_t *sK = smem + OFF_K;
    uint8_t *sV = smem + OFF_V;
    uint8_t *sP = smem + OFF_P;
    uint8_t *sTab = smem + OFF_TAB;
    int32_t *sRed = reinterpret_cast<int32_t *>(smem + OFF_RED);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1;             // [KST]
    uint64_t *k_empty = k_full + KST;        // [KST]
    uint64_t *v_full = k_empty + KST;        // [VST]
    uint64_t *v_empty = v_full + VST;        // [VST]
    uint64_t *s_full = v_empty + VST;        // [1]
    uint64_t *s_empty = s_full + 1;          // [1]
    uint64_t *p_full = s_empty + 1;          // [2]
    uint64_t *p_empty = p_full + 2;          // [2]
    uint64_t *o_full = p_empty + 2;
    uint64_t *drain = o_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int T = p.T, H = p.H;
    const int nqb = (T + BQ - 1) / BQ;
    const int qb = blockIdx.x % nqb;
    const int bh = blockIdx.x / nqb;
    const int h = bh % H, b = bh / H;
    const int q0 = qb * BQ;
    const int nkb = (T + BK - 1) / BK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KST; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
        for (int s = 0; s < VST; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
        mbar_init(s_full, 1);
        mbar_init(s_empty, SOFT_WARPS);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&p_full[s], SOFT_WARPS);
            mbar_init(&p_empty[s], 1);
        }
        mbar_init(o_full, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // Q and K maps cover [B*T rows, H*64 columns]; V^T maps [B*H*64, vt_ld].
    const int row0 = b * T;

    if (warp == 0) {
        if (lane == 0) {
            // Q once
            mbar_arrive_expect_tx(q_full, Q_BYTES);
            tma_load_2d(&tmQ, q_full, sQ, h * 64, row0 + q0);
            int ks = 0;
            uint32_t kph = 0;
            int vs = 0;
            uint32_t vph = 0;
            bool ok = true;
            for (int pass = 0; pass < 2 && ok; ++pass) {
                for (int j = 0; j < nkb && ok; ++j) {
                    if (!mbar_wait(&k_empty[ks], kph ^ 1)) { ok = false; break; }
                    mbar_arrive_expect_tx(&k_full[ks], K_BYTES);
                    tma_load_2d(&tmK, &k_full[ks], sK + ks * K_BYTES, h * 64, row0 + j * BK);
                    if (++ks == KST) { ks = 0; kph ^= 1; }
                    if (pass == 1) {
                        if (!mbar_wait(&v_empty[vs], vph ^ 1)) { ok = false; break; }
                        mbar_arrive_expect_tx(&v_full[vs], V_BYTES);
                        tma_load_2d(&tmV, &v_full[vs], sV + vs * V_BYTES, j * BK, bh * 64);
                        if (++vs == VST) { vs = 0; vph ^= 1; }
                    }
                }
            }
            if (!ok) *abort_flag = 1;
            // all issued copies must land before exit (bounded)
            mbar_wait(q_full, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_i8(BQ, BK, true, true);
            constexpr uint32_t idesc_pv = idesc_i8(BQ, 64, false, true);
            const uint32_t tS = tmem_base, tO = tmem_base + 128;
            int ks = 0, sb = 0, pb = 0, vs = 0;
            uint32_t kph = 0, sph = 0, pph = 0, vph = 0;
            bool ok = mbar_wait(q_full, 0);
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ);
            auto issue_qk = [&](int j) -> bool {
                if (!mbar_wait(&s_empty[sb], sph ^ 1)) return false;
                if (!mbar_wait(&k_full[ks], kph)) return false;
                tc_fence_after();
                const uint32_t ka = smem_u32(sK + ks * K_BYTES);
                const uint32_t d = tS + (uint32_t)(sb * BK);
#pragma unroll
                for (int kk = 0; kk < 2; ++kk)
                    mma_i8(d, sdesc_kmajor_sw64(qa + kk * 32), sdesc_kmajor_sw64(ka + kk * 32), idesc_qk, kk);
                mma_commit(&k_empty[ks]);
                mma_commit(&s_full[sb]);
                if (++ks == KST) { ks = 0; kph ^= 1; }
                sph ^= 1;
                return true;
            };
            // pass 1
            for (int j = 0; j < nkb && ok; ++j) ok = issue_qk(j);
            // pass 2: QK of block j+1 is issued before PV of block j
            if (ok) ok = issue_qk(0);
            for (int j = 0; j < nkb && ok; ++j) {
                if (j + 1 < nkb) ok = issue_qk(j + 1);
                if (!ok) break;
                if (!mbar_wait(&p_full[pb], pph)) { ok = false; break; }
                if (!mbar_wait(&v_full[vs], vph)) { ok = false; break; }
                tc_fence_after();
                const uint32_t pa = smem_u32(sP + pb * P_BYTES);
                const uint32_t va = smem_u32(sV + vs * V_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 32; ++kk)
                    mma_i8(tO, sdesc_kmajor_sw128(pa + kk * 32), sdesc_kmajor_sw128(va + kk * 32), idesc_pv,
                           (j | kk) != 0);
                mma_commit(&v_empty[vs]);
                mma_commit(&p_empty[pb]);
                if (++vs == VST) { vs = 0; vph ^= 1; }
                if (++pb == 2) { pb = 0; pph ^= 1; }
            }
            if (ok) mma_commit(o_full);
            else *abort_flag = 1;
            mma_commit(drain);
            mbar_wait(drain, 0);
        }
    } else {
        // ------------------------------------------------------------------
        // softmax warps
        // ------------------------------------------------------------------
        const int sw = warp - 2;
        const int quad = warp & 3;
        const int half = sw >> 2;  // 0: key columns [0,64), 1: [64,128) of each block
        const int r = quad * 32 + lane;  // query row within the block
        const int et = sw * 32 + lane;
        // shift-exp table
        // index of the zero entry (bounded by the shared-memory table size)
        const uint32_t t1 = min((uint32_t)p.tab[0] | ((uint32_t)p.tab[1] << 8), (uint32_t)(TAB_MAX - 1));
        for (uint32_t i = et; i <= t1; i += SOFT_WARPS * 32) sTab[i] = p.tab[2 + i];
        bar_soft();
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        // ---- pass 1: raw row max ------------------------------------------
        int32_t mx = INT32_MIN;
        int sb = 0;
        uint32_t sph = 0;
        bool ok = true;
        for (int j = 0; j < nkb; ++j) {
            bool w = true;
            if (lane == 0) w = mbar_wait(&s_full[sb], sph);
            if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) { ok = false; break; }
            tc_fence_after();
            const int kbase = j * BK + half * 64;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + lane_base + (uint32_t)(sb * BK + half * 64 + c * 32), acc);
                tmem_ld_wait();
                const int valid = T - (kbase + c * 32);  // keys of this chunk that exist
                if (valid >= 32) {
#pragma unroll
                    for (int u = 0; u < 32; ++u) mx = max(mx, (int32_t)acc[u]);
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u)
                        if (u < valid) mx = max(mx, (int32_t)acc[u]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[sb]);
            sph ^= 1;
        }
        // combine the two column halves of each row
        if (half == 1) sRed[r] = mx;
        bar_soft();
        if (half == 0) sRed[r] = max(mx, sRed[r]);
        bar_soft();
        mx = sRed[r];
        // requantised row max + 1 (int16 wrap), qk_requant_rowmax_scalar
        int32_t smax = rrs_masked((int32_t)((uint32_t)mx * p.qk_mult), p);
        smax = clampi(smax, -32768, 32767);
        const int32_t rmax1 = (int32_t)(int16_t)(smax + 1);
        // ---- pass 2: exp, row sum, P to shared memory ----------------------
        int32_t rsum = 0;
        int pb = 0;
        uint32_t pph = 0;
        for (int j = 0; j < nkb && ok; ++j) {
            bool w = true;
            if (lane == 0) w = mbar_wait(&s_full[sb], sph) && mbar_wait(&p_empty[pb], pph ^ 1);
            if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) { ok = false; break; }
            tc_fence_after();
            const int kbase = j * BK + half * 64;
            uint8_t *prow = sP + pb * P_BYTES + r * 128;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + lane_base + (uint32_t)(sb * BK + half * 64 + c * 32), acc);
                tmem_ld_wait();
                const int valid = T - (kbase + c * 32);
                uint32_t w4[8];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    int32_t s = rrs_masked((int32_t)(acc[u] * p.qk_mult), p);
                    s = clampi(s, -32768, 32767);
                    const int32_t xs = (int32_t)(int16_t)(s - rmax1);
                    const uint32_t idx = min((uint32_t)(-xs), t1);
                    uint32_t e = sTab[idx];
                    if (valid < 32 && u >= valid) e = 0;
                    rsum += (int32_t)e;
                    if ((u & 3) == 0) w4[u >> 2] = 0;
                    w4[u >> 2] |= e << (8 * (u & 3));
                }
                // two 16-byte chunks of this row; 128-byte swizzle: chunk k of
                // row r lives at chunk (k ^ (r & 7))
                const int ch0 = half * 4 + c * 2;
                *reinterpret_cast<uint4 *>(prow + (((ch0) ^ (r & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                *reinterpret_cast<uint4 *>(prow + (((ch0 + 1) ^ (r & 7)) << 4)) = make_uint4(w4[4], w4[5], w4[6], w4[7]);
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_empty[sb]);
                mbar_arrive(&p_full[pb]);
            }
            sph ^= 1;
            if (++pb == 2) { pb = 0; pph ^= 1; }
        }
        // combine row sums
        if (half == 1) sRed[BQ + r] = rsum;
        bar_soft();
        if (half == 0) sRed[BQ + r] += rsum;
        bar_soft();
        rsum = sRed[BQ + r];
        // ---- epilogue: O / normalise / AV requant ---------------------------
        bool w = ok;
        if (ok && lane == 0) w = mbar_wait(o_full, 0);
        if (__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) {
            tc_fence_after();
            uint32_t acc[32];
            tmem_ld_32x32b_x32(tmem_base + lane_base + 128u + (uint32_t)(half * 32), acc);
            tmem_ld_wait();
            const int q = q0 + r;
            if (q < T) {
                const int32_t inv = fisr(rsum, p.rsqrt_offset);
                uint32_t w4[8];
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    int32_t v = rrs(wmul((int32_t)acc[u], inv), p.rsqrt_offset);
                    v = rrs(wmul(v, inv), p.rsqrt_offset);
                    v = rrs(wmul(v, (int32_t)p.av_mult), p.av_shift);
                    v = clampi(v, -127, 127);
                    if ((u & 3) == 0) w4[u >> 2] = 0;
                    w4[u >> 2] |= (uint32_t)(uint8_t)v << (8 * (u & 3));
                }
                int8_t *o = p.out + (int64_t)(row0 + q) * p.ldo + h * 64 + half * 32;
                *reinterpret_cast<uint4 *>(o) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                *reinterpret_cast<uint4 *>(o + 16) = make_uint4(w4[4], w4[5], w4[6], w4[7]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Table of the shift-exp of attention_scalar.cpp:388-560 as a function of
// the int16 difference xs = s - rowmax1 <= 0: tab[2 + i] = exp(xs = -i) for
// i in [0, t1), tab[2 + t1] = 0 (used for every xs > 0 and every xs below
// the last non-zero entry). tab[0..1] hold t1 (little endian).
__global__ void shift_exp_table_kernel(int32_t fb, uint8_t *tab, int *last_nz) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // i = -xs in [0, 32768]
    if (i > 32768) return;
    const int32_t e = shift_exp_one(-i, 0, fb);
    if (e != 0) atomicMax(last_nz, i);
}

__global__ void shift_exp_table_fill(int32_t fb, uint8_t *tab, const int *last_nz, int cap, int *status) {
    const int t1 = *last_nz + 1;
    if (t1 >= cap) {
        if (blockIdx.x == 0 && threadIdx.x == 0) *status = 1;
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i <= t1; i += gridDim.x * blockDim.x)
        tab[2 + i] = (uint8_t)(i < t1 ? shift_exp_one(-i, 0, fb) : 0);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        tab[0] = (uint8_t)(t1 & 0xFF);
        tab[1] = (uint8_t)(t1 >> 8);
        *status = 0;
    }
}

// V^T for the P.V operand: vt[(b*H + h)*64 + d][t] = V[b*T + t][h*64 + d]
// (V given with row stride ldv); keys are the contiguous dimension.
__global__ void transpose_v_kernel(const int8_t *__restrict__ v, int64_t ldv, int B, int T, int H,
                                   int8_t *__restrict__ vt, int vt_ld) {
    __shared__ int8_t tile[64][65];
    const int bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    const int t0 = blockIdx.x * 64;
    for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
        const int tt = i / 64, d = i % 64;
        const int t = t0 + tt;
        tile[tt][d] = t < T ? v[((int64_t)b * T + t) * ldv + h * 64 + d] : (int8_t)0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
        const int d = i / 64, tt = i % 64;
        const int t = t0 + tt;
        if (t < vt_ld) vt[((int64_t)bh * 64 + d) * vt_ld + t] = tile[tt][d];
    }
}

cudaError_t attention_tc(const AttnArgs &a, int B, int H, const uint8_t *tab, int8_t *vt, int vt_ld,
                         cudaStream_t st) {
    using namespace attn;
    const int T = a.Tk;
    // V^T
    dim3 tg((vt_ld + 63) / 64, B * H);
    transpose_v_kernel<<<tg, 256, 0, st>>>(a.v, a.ldv, B, T, H, vt, vt_ld);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap tq, tk, tv;
    e = make_tmap_2d_u8(&tq, a.q, (uint64_t)H * 64, (uint64_t)B * T, (uint64_t)a.ldq, 64, BQ, CU_TENSOR_MAP_SWIZZLE_64B);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u8(&tk, a.k, (uint64_t)H * 64, (uint64_t)B * T, (uint64_t)a.ldk, 64, BK,
                        CU_TENSOR_MAP_SWIZZLE_64B);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u8(&tv, vt, (uint64_t)vt_ld, (uint64_t)B * H * 64, (uint64_t)vt_ld, BK, 64);
    if (e != cudaSuccess) return e;
    AttnTcParams p;
    p.B = B; p.H = H; p.T = T;
    p.out = a.out; p.ldo = a.ldo;
    p.qk_mult = a.qk_mult;
    const uint32_t sh = (uint32_t)(a.qk_shift > 0 ? a.qk_shift : 0);
    if (sh == 0) { p.qk_rnd = 0; p.qk_sgn = 0; p.qk_sh = 0; p.qk_z = 0xFFFFFFFFu; }
    else if (sh < 32) { p.qk_rnd = 1u << (sh - 1); p.qk_sgn = 0xFFFFFFFFu; p.qk_sh = sh; p.qk_z = 0xFFFFFFFFu; }
    else { p.qk_rnd = 0; p.qk_sgn = 0; p.qk_sh = 0; p.qk_z = 0; }
    p.tab = tab;
    p.av_mult = a.av_mult;
    p.av_shift = (uint32_t)clampi(a.av_shift, 0, 32);
    p.rsqrt_offset = a.rsqrt_offset;
    p.vt_ld = vt_ld;
    static bool attr = false;
    if (!attr) {
        e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const int grid = B * H * ((T + BQ - 1) / BQ);
    attn_tc_kernel<<<grid, THREADS, SMEM, st>>>(tq, tk, tv, p);
    return cudaGetLastError();
}

cudaError_t shift_exp_table_build(int32_t fb, uint8_t *tab, int *scratch2, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(scratch2, 0xFF, sizeof(int), st);  // last_nz = -1
    if (e != cudaSuccess) return e;
    shift_exp_table_kernel<<<(32769 + 255) / 256, 256, 0, st>>>(fb, tab, scratch2);
    shift_exp_table_fill<<<32, 256, 0, st>>>(fb, tab, scratch2, attn::TAB_MAX, scratch2 + 1);
    return cudaGetLastError();
}

}  // namespace iw
