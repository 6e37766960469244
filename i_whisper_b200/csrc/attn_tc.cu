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
//           written to tensor memory (tcgen05.st) as the A operand of
//           O += P V^T, which runs on the tensor cores (u8 x s8 -> s32).
//   end:    O is normalised by FISR(rowsum)^2 and the AV requant, and written
//           as int8 rows [b*T + t, h*64 + d].
// The reference's online order (row max first, then exp and sum) is kept
// exactly; no rescaling of partial sums is needed.
//
// Each CTA walks its work items in phases: phase ph interleaves, block by
// block, pass 2 of its item ph-1 with pass 1 of its item ph. Producer, Q.K^T
// issuer and softmax warps follow that one order through the shared rings
// (K, S), the P.V issuer takes the pass-2 blocks in item order.
//
// Warp roles: warp 0 TMA producer (Q once, K blocks twice, V^T blocks),
// warp 1 TMEM owner + P.V issuer, warp 18 Q.K^T issuer, warps 2..17 softmax
// (thread = query row of its TMEM lane quadrant, four warps per quadrant
// split the 128 key columns).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "iw_common.cuh"
#include "iw_sm100.cuh"
#include "iw_tmap.cuh"
#include "kernels.cuh"

namespace iw {

namespace attn {

constexpr int BQ = 128;     // query rows per work item
constexpr int BK = 128;     // keys per block
constexpr int KST = 4;      // K stages
constexpr int VST = 3;      // V^T stages
constexpr int SBUF = 3;     // S accumulators in TMEM
// Softmax warps: SLICES per TMEM lane quadrant, each taking SC of a block's
// 128 keys (sixteen warps of 32 keys measured faster than eight of 64).
constexpr int SOFT_WARPS = 16;
constexpr int SLICES = SOFT_WARPS / 4;
constexpr int SC = BK / SLICES;       // keys per warp and block
constexpr int HALVES = SC / 32;       // 32-column TMEM loads per block
constexpr int OC = 64 / SLICES;       // output columns per warp
constexpr int QK_WARP = 2 + SOFT_WARPS;  // the Q.K^T issuer
constexpr int THREADS = 96 + 32 * SOFT_WARPS;
static_assert(SC % 32 == 0 && (OC == 16 || OC == 32), "softmax warp split");
// The whole shift-exp table lives in shared memory: its zero entry t1 is at
// most 32769 (frac_bits >= 15 keeps non-zero values down to xs = -32768), so
// the header (2 bytes) and t1 + 1 entries take at most 32772 bytes.
constexpr int TAB_MAX = 32770;                    // entries (indices 0..32769)
constexpr int TAB_SMEM = (2 + TAB_MAX + 15) / 16 * 16;  // header + entries, 16-byte chunks

constexpr int Q_BYTES = BQ * 64;
constexpr int K_BYTES = BK * 64;
constexpr int V_BYTES = 64 * BK;
constexpr int P_COLS = BK / 4;      // TMEM columns of one P buffer (four u8 keys per column)
// layout (offsets from the 1024-aligned base)
constexpr int OFF_Q = 0;                          // two Q buffers
constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + KST * K_BYTES;
constexpr int OFF_RED = OFF_V + VST * V_BYTES;    // 3 x [SLICES][BQ] int32 cross-warp row max / sum / output sum
constexpr int OFF_BAR = OFF_RED + 3 * SLICES * BQ * 4;
constexpr int SMEM = 1024 + OFF_BAR + 512;
// TMEM: S at 0/128/256, O at 384 (one buffer: a work item's epilogue reads
// O before the softmax warps write the next item's first P), P at 448/480.
// P lives in TMEM as the P.V MMA's A operand, written with tcgen05.st: no
// generic-to-async proxy fence per block (a shared-memory P needed one, 6%
// of the kernel's time).
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_O = 384;
constexpr uint32_t TMEM_P = 448;
static_assert(TMEM_O + 64 <= TMEM_P && TMEM_P + 2 * P_COLS <= TMEM_COLS && SBUF * BK <= (int)TMEM_O, "TMEM map");
static_assert(OFF_V % 1024 == 0, "swizzle-128 tiles need 1024-byte alignment");
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
    int32_t *rowsum_out;  // optional: += each output row's sum (the out-projection's zero-point term)
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

// Score requantisation for 1 <= m <= 255 and shift in [1,31]:
// rrs(acc*m, s) = (acc*m + 2^(s-1) - signbit(acc*m)) >> s, and since
// |acc*m| < 2^31 and m > 0, signbit(acc*m) == signbit(acc) == -mulhi(acc, 1).
IW_DEV int32_t score_fast(uint32_t acc, uint32_t m, uint32_t rnd, uint32_t sh) {
    int32_t x, y;
    asm("mad.lo.s32 %0, %1, %2, %3;" : "=r"(x) : "r"(acc), "r"(m), "r"(rnd));
    asm("mad.hi.s32 %0, %1, 1, %2;" : "=r"(y) : "r"(acc), "r"(x));
    return y >> sh;
}

// (C - acc*m + [acc < 0]) mod 2^32 for negm = -m: two multiply-adds, the
// second adding the sign bit of acc as the high word of acc * 2.
IW_DEV uint32_t exp_index(uint32_t acc, uint32_t negm, uint32_t c) {
    uint32_t t, u;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(t) : "r"(acc), "r"(negm), "r"(c));
    asm("mad.hi.u32 %0, %1, 2, %2;" : "=r"(u) : "r"(acc), "r"(t));
    return u;
}

IW_DEV int32_t rrs_masked(int32_t x, const AttnTcParams &p) {
    const uint32_t t = (uint32_t)x + p.qk_rnd + ((uint32_t)(x >> 31) & p.qk_sgn);
    return (int32_t)(((int32_t)t >> p.qk_sh) & (int32_t)p.qk_z);
}

template <bool FAST>
__global__ void __launch_bounds__(attn::THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
    using namespace attn;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sQ = smem + OFF_Q;
    uint8_t *sK = smem + OFF_K;
    uint8_t *sV = smem + OFF_V;
    // the shift-exp table lives in static shared memory: its address is a
    // compile-time constant, so a lookup is one load with an immediate offset
    __shared__ __align__(16) uint8_t sTabRaw[TAB_SMEM];
    uint8_t *const sTab = sTabRaw + 2;  // entry i at sTabRaw[2 + i], as in global memory
    int32_t *sRed = reinterpret_cast<int32_t *>(smem + OFF_RED);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;                 // [2]
    uint64_t *q_empty = q_full + 2;          // [2]
    uint64_t *k_full = q_empty + 2;          // [KST]
    uint64_t *k_empty = k_full + KST;        // [KST]
    uint64_t *v_full = k_empty + KST;        // [VST]
    uint64_t *v_empty = v_full + VST;        // [VST]
    uint64_t *s_full = v_empty + VST;        // [SBUF]
    uint64_t *s_empty = s_full + SBUF;       // [SBUF]
    uint64_t *p_full = s_empty + SBUF;       // [2]
    uint64_t *p_empty = p_full + 2;          // [2]
    uint64_t *o_full = p_empty + 2;          // [2]
    uint64_t *o_empty = o_full + 2;          // [2]
    uint64_t *drain = o_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int T = p.T, H = p.H;
    const int nqb = (T + BQ - 1) / BQ;
    const int nkb = (T + BK - 1) / BK;
    const int items = p.B * H * nqb;
    // work items of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ... (grid <= items)
    const int n_my = ((int)blockIdx.x < items) ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], 1);
            mbar_init(&p_full[s], SOFT_WARPS);
            mbar_init(&p_empty[s], 1);
            mbar_init(&o_full[s], 1);
            mbar_init(&o_empty[s], SOFT_WARPS);
        }
        for (int s = 0; s < KST; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
        for (int s = 0; s < VST; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
        for (int s = 0; s < SBUF; ++s) { mbar_init(&s_full[s], 1); mbar_init(&s_empty[s], SOFT_WARPS); }
        mbar_init(drain, 2);
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
    // TMEM is held: let the next kernel be scheduled, then wait for the
    // previous one before touching global memory
    pdl_launch();
    pdl_wait();

    // Q and K maps cover [B*T rows, H*64 columns]; V^T maps [B*H*64, vt_ld].
    if (warp == 0) {
        if (lane == 0) {
            int qs = 0, ks = 0, vs = 0;
            uint32_t qph = 0, kph = 0, vph = 0;
            bool ok = true;
            // Phase ph interleaves pass 2 of this CTA's item ph-1 with pass 1
            // of its item ph (block by block), the order every role follows.
            for (int ph = 0; ph <= n_my && ok && !*abort_flag; ++ph) {
                const bool has1 = ph < n_my, has2 = ph > 0;
                const int it1 = blockIdx.x + ph * gridDim.x, it2 = it1 - gridDim.x;
                const int bh1 = it1 / nqb, bh2 = it2 / nqb;
                const int h1 = bh1 % H, row1 = (bh1 / H) * T, h2 = bh2 % H, row2 = (bh2 / H) * T;
                if (has1) {
                    if (!mbar_wait(&q_empty[qs], qph ^ 1)) { ok = false; break; }
                    mbar_arrive_expect_tx(&q_full[qs], Q_BYTES);
                    tma_load_2d(&tmQ, &q_full[qs], sQ + qs * Q_BYTES, h1 * 64, row1 + (it1 % nqb) * BQ);
                    if (++qs == 2) { qs = 0; qph ^= 1; }
                }
                for (int j = 0; j < nkb && ok; ++j) {
                    if (has2) {
                        if (!mbar_wait(&k_empty[ks], kph ^ 1)) { ok = false; break; }
                        mbar_arrive_expect_tx(&k_full[ks], K_BYTES);
                        tma_load_2d(&tmK, &k_full[ks], sK + ks * K_BYTES, h2 * 64, row2 + j * BK);
                        if (++ks == KST) { ks = 0; kph ^= 1; }
                        if (!mbar_wait(&v_empty[vs], vph ^ 1)) { ok = false; break; }
                        mbar_arrive_expect_tx(&v_full[vs], V_BYTES);
                        tma_load_2d(&tmV, &v_full[vs], sV + vs * V_BYTES, j * BK, bh2 * 64);
                        if (++vs == VST) { vs = 0; vph ^= 1; }
                    }
                    if (has1) {
                        if (!mbar_wait(&k_empty[ks], kph ^ 1)) { ok = false; break; }
                        mbar_arrive_expect_tx(&k_full[ks], K_BYTES);
                        tma_load_2d(&tmK, &k_full[ks], sK + ks * K_BYTES, h1 * 64, row1 + j * BK);
                        if (++ks == KST) { ks = 0; kph ^= 1; }
                    }
                }
            }
            if (!ok) *abort_flag = 1;
        }
    } else if (warp == 1 || warp == QK_WARP) {
        // Two MMA issuers on different sub-partitions: QK_WARP issues every
        // Q.K^T (bounded by the free S buffers, so it runs ahead of the
        // softmax), warp 1 every P.V (after the softmax has written P).
        if (lane == 0) {
            bool ok = true;
            if (warp == QK_WARP) {
                constexpr uint32_t idesc_qk = idesc_i8(BQ, BK, true, true);
                int ks = 0, sb = 0;
                uint32_t kph = 0, sph = 0;
                // item k of this CTA uses Q buffer k & 1, q_full phase (k >> 1) & 1
                auto issue_qk = [&](int k) -> bool {
                    if (!mbar_wait(&s_empty[sb], sph ^ 1) || !mbar_wait(&k_full[ks], kph)) return false;
                    tc_fence_after();
                    const uint32_t qa = smem_u32(sQ + (k & 1) * Q_BYTES);
                    const uint32_t ka = smem_u32(sK + ks * K_BYTES);
                    const uint32_t d = tmem_base + (uint32_t)(sb * BK);
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk)
                        mma_i8(d, sdesc_kmajor_sw64(qa + kk * 32), sdesc_kmajor_sw64(ka + kk * 32), idesc_qk, kk);
                    mma_commit(&k_empty[ks]);
                    mma_commit(&s_full[sb]);
                    if (++ks == KST) { ks = 0; kph ^= 1; }
                    if (++sb == SBUF) { sb = 0; sph ^= 1; }
                    return true;
                };
                for (int ph = 0; ph <= n_my && ok && !*abort_flag; ++ph) {
                    const bool has1 = ph < n_my, has2 = ph > 0;
                    if (has1) {
                        if (!mbar_wait(&q_full[ph & 1], (uint32_t)(ph >> 1) & 1u)) { ok = false; break; }
                        tc_fence_after();
                    }
                    for (int j = 0; j < nkb && ok; ++j) {
                        if (has2) {
                            if (!issue_qk(ph - 1)) { ok = false; break; }
                            if (j + 1 == nkb) mma_commit(&q_empty[(ph - 1) & 1]);  // item ph-1's last QK issued
                        }
                        if (has1 && !issue_qk(ph)) { ok = false; break; }
                    }
                }
            } else {
                constexpr uint32_t idesc_pv = idesc_i8(BQ, 64, false, true);
                int pb = 0, vs = 0;
                constexpr int ob = 0;  // one O buffer
                uint32_t pph = 0, vph = 0, oph = 0;
                for (int it = blockIdx.x; it < items && ok && !*abort_flag; it += gridDim.x) {
                    for (int j = 0; j < nkb; ++j) {
                        if (!mbar_wait(&p_full[pb], pph) || !mbar_wait(&v_full[vs], vph)) { ok = false; break; }
                        if (j == 0 && !mbar_wait(&o_empty[ob], oph ^ 1)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t tp = tmem_base + TMEM_P + (uint32_t)(pb * P_COLS);
                        const uint32_t va = smem_u32(sV + vs * V_BYTES);
                        const uint32_t tO = tmem_base + TMEM_O;
#pragma unroll
                        for (int kk = 0; kk < BK / 32; ++kk)
                            mma_i8_ts(tO, tp + (uint32_t)(kk * 8), sdesc_kmajor_sw128(va + kk * 32), idesc_pv,
                                      (j | kk) != 0);
                        mma_commit(&v_empty[vs]);
                        mma_commit(&p_empty[pb]);
                        if (++vs == VST) { vs = 0; vph ^= 1; }
                        if (++pb == 2) { pb = 0; pph ^= 1; }
                    }
                    if (!ok) break;
                    mma_commit(&o_full[ob]);
                    oph ^= 1;  // one O buffer (ob stays 0)
                }
            }
            if (!ok) *abort_flag = 1;
            // every MMA this thread issued completes before TMEM is released
            // (the barrier counts both issuers' commits)
            mma_commit(drain);
            mbar_wait(drain, 0);
        }
    } else {
        // ------------------------------------------------------------------
        // softmax warps: thread = query row of the warp's TMEM lane quadrant,
        // the warp's slice = SC of the 128 key columns of every block, taken
        // as HALVES 32-column halves
        // ------------------------------------------------------------------
        const int sw = warp - 2;
        const int quad = warp & 3;
        const int slice = sw >> 2;
        const int r = quad * 32 + lane;  // query row within the work item
        const int et = sw * 32 + lane;
        // index of the zero entry (bounded by the shared-memory table size)
        const uint32_t t1 = min((uint32_t)p.tab[0] | ((uint32_t)p.tab[1] << 8), (uint32_t)(TAB_MAX - 1));
        {
            // header and entries 0..t1 (t1 + 3 bytes): whole 16-byte chunks
            // when the table is 16-byte aligned, then the tail bytes; never
            // past byte t1 + 2 of the caller's buffer
            const uint32_t nbytes = t1 + 3;
            uint32_t done = 0;
            if ((reinterpret_cast<uintptr_t>(p.tab) & 15u) == 0) {
                const uint32_t n16 = nbytes / 16;
                for (uint32_t i = et; i < n16; i += SOFT_WARPS * 32)
                    reinterpret_cast<uint4 *>(sTabRaw)[i] = __ldg(reinterpret_cast<const uint4 *>(p.tab) + i);
                done = n16 * 16;
            }
            for (uint32_t i = done + et; i < nbytes; i += SOFT_WARPS * 32) sTabRaw[i] = p.tab[i];
        }
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t col = (uint32_t)(slice * SC);
        const RrsK k_rsq = rrs_k(p.rsqrt_offset), k_av = rrs_k(p.av_shift);  // output normalisation shifts
        const bool epi_simple = k_rsq.sgn == -1 && k_av.sgn == -1;  // both shifts in [1, 31]
        int sb = 0, pb = 0;
        constexpr int ob = 0;  // one O buffer
        uint32_t sph = 0, pph = 0, oph = 0;
        // wait helper: every lane waits (the warp stays converged, which
        // measured faster than one lane waiting for the others), the warp
        // agrees; once a wait failed the warp stops waiting (and computing)
        // but keeps meeting the barriers
        bool ok = true;
        auto wait_all = [&](uint64_t *bar, uint32_t parity) {
            bool w = ok;
            if (ok) w = mbar_wait(bar, parity);
            w = __all_sync(0xffffffffu, w);
            if (!w && ok) {
                ok = false;
                if (lane == 0) *abort_flag = 1;
            }
            return ok;
        };
        auto ld_half = [&](int sbuf, int hf, uint32_t (&a)[32]) {
            tmem_ld_32x32b_x32(tmem_base + lane_base + (uint32_t)(sbuf * BK) + col + (uint32_t)(hf * 32), a);
        };
        // Pass-2 state of the item whose pass 1 ended in the previous phase.
        int32_t rmax1 = 0;
        bool warp_simple = false;
        uint32_t cidx = 0;
        const uint32_t negm = 0u - p.qk_mult;
        // exp of 32 scores of one half into eight packed words, adding to rs
        // fast-path exp of 32 scores into eight packed words; MASKED: keep
        // only the first `valid` (1..31) keys. Keys past T (a ragged last
        // block) hold the scores of whatever K rows follow (the next window's,
        // or the zero fill past the tensor): their index is clamped to the
        // table like any other and their bytes are masked off afterwards.
        // valid is the same for every lane, so the masks are warp-uniform.
        auto exp_fast = [&](const uint32_t (&a)[32], int valid, uint32_t (&w4)[8], int32_t &rs, auto masked) {
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
                uint32_t ww = 0;
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                    const uint32_t idx = min(exp_index(a[q4 * 4 + k4], negm, cidx) >> p.qk_sh, t1);
                    // ww += tab << 8*k4 as a multiply-add (keeps it off the ALU pipe)
                    asm("mad.lo.u32 %0, %1, %2, %0;" : "+r"(ww) : "r"((uint32_t)sTab[idx]), "r"(1u << (8 * k4)));
                }
                if constexpr (decltype(masked)::value) {
                    const int left = valid - 4 * q4;  // valid keys among this word's four
                    ww &= left >= 4 ? 0xFFFFFFFFu : (left <= 0 ? 0u : (1u << (8 * left)) - 1u);
                }
                // probabilities are unsigned bytes (up to 255 for frac_bits >= 15)
                rs = (int32_t)__dp4a(ww, 0x01010101u, (uint32_t)rs);
                w4[q4] = ww;
            }
        };
        // exp of 32 scores of one half into eight packed words, adding to rs
        auto exp_half = [&](const uint32_t (&a)[32], int valid, uint32_t (&w4)[8], int32_t &rs) {
            if (FAST && warp_simple && valid >= 32) {
                exp_fast(a, valid, w4, rs, std::false_type{});
            } else if (valid <= 0) {
                // keys past T only (warp-uniform): probabilities 0
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) w4[q4] = 0;
            } else if (FAST && warp_simple) {
                exp_fast(a, valid, w4, rs, std::true_type{});
            } else {
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    int32_t sc;
                    if constexpr (FAST) sc = score_fast(a[u], p.qk_mult, p.qk_rnd, p.qk_sh);
                    else sc = rrs_masked((int32_t)(a[u] * p.qk_mult), p);
                    sc = clampi(sc, -32768, 32767);
                    // int16 wrap of -(s - rowmax1), clamped to the zero entry
                    const uint32_t idx = min((uint32_t)(rmax1 - sc) & 0xFFFFu, t1);
                    const uint32_t e = u < valid ? (uint32_t)sTab[idx] : 0u;
                    rs += (int32_t)e;
                    if ((u & 3) == 0) w4[u >> 2] = e;
                    else w4[u >> 2] |= e << (8 * (u & 3));
                }
            }
        };
        int32_t *sRedMax = sRed, *sRedSum = sRed + SLICES * BQ, *sRedRow = sRed + 2 * SLICES * BQ;
        // Phase ph: pass 2 of this CTA's item ph-1 block by block interleaved
        // with pass 1 of its item ph, so that the light pass-1 blocks (a row
        // max) fill the Q.K^T round trip that the heavy pass-2 blocks hide.
        for (int ph = 0; ph <= n_my; ++ph) {
            // every softmax warp reads the abort flag between the same two
            // barriers (it is only written outside them) and leaves together
            bar_soft();
            const bool stop = *abort_flag != 0;
            bar_soft();
            if (stop) break;
            const bool has1 = ph < n_my, has2 = ph > 0;
            const int it2 = (int)blockIdx.x + (ph - 1) * (int)gridDim.x;
            int32_t mx = INT32_MIN, rsum = 0;
            for (int j = 0; j < nkb; ++j) {
                if (has2) {
                    // ---- pass 2 of item ph-1: exp, row sum, P to shared memory
                    if (!wait_all(&s_full[sb], sph)) break;
                    tc_fence_after();
                    uint32_t acc[HALVES][32];
                    uint32_t w4[HALVES][8];
                    // half 0 first; the other halves load while it is computed
                    ld_half(sb, 0, acc[0]);
                    tmem_ld_wait();
#pragma unroll
                    for (int hf = 1; hf < HALVES; ++hf) ld_half(sb, hf, acc[hf]);
                    exp_half(acc[0], T - (j * BK + slice * SC), w4[0], rsum);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_empty[sb]);
#pragma unroll
                    for (int hf = 1; hf < HALVES; ++hf)
                        exp_half(acc[hf], T - (j * BK + slice * SC + hf * 32), w4[hf], rsum);
                    // the P buffer must be free (P.V of block j-2 done)
                    if (!wait_all(&p_empty[pb], pph ^ 1)) break;
                    // this warp's 32 rows x SC keys of P: row = TMEM lane,
                    // keys 4c..4c+3 in column c (the A operand's K-major layout)
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf)
                        tmem_st_32x32b_x8(tmem_base + lane_base + TMEM_P +
                                              (uint32_t)(pb * P_COLS + (slice * SC + hf * 32) / 4),
                                          w4[hf]);
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[pb]);
                    if (++sb == SBUF) { sb = 0; sph ^= 1; }
                    if (++pb == 2) { pb = 0; pph ^= 1; }
                }
                if (has1) {
                    // ---- pass 1 of item ph: raw row max
                    if (!wait_all(&s_full[sb], sph)) break;
                    tc_fence_after();
                    uint32_t acc[HALVES][32];
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) ld_half(sb, hf, acc[hf]);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_empty[sb]);  // S is in registers: release it early
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) {
                        const int valid = T - (j * BK + slice * SC + hf * 32);
                        if (valid >= 32) {
#pragma unroll
                            for (int u = 0; u < 32; ++u) mx = max(mx, (int32_t)acc[hf][u]);
                        } else {
#pragma unroll
                            for (int u = 0; u < 32; ++u)
                                if (u < valid) mx = max(mx, (int32_t)acc[hf][u]);
                        }
                    }
                    if (++sb == SBUF) { sb = 0; sph ^= 1; }
                }
            }
            if (has2) {
                // combine row sums
                sRedSum[slice * BQ + r] = rsum;
                bar_soft();
                rsum = 0;
#pragma unroll
                for (int sl = 0; sl < SLICES; ++sl) rsum += sRedSum[sl * BQ + r];
                // ---- epilogue of item ph-1: O / normalise / AV requant ---------
                const int qb = it2 % nqb, bh = it2 / nqb;
                const int h = bh % H, row0 = (bh / H) * T;
                const int q0 = qb * BQ;
                if (wait_all(&o_full[ob], oph)) {
                    tc_fence_after();
                    uint32_t acc[OC];
                    if constexpr (OC == 32)
                        tmem_ld_32x32b_x32(tmem_base + lane_base + TMEM_O + (uint32_t)(slice * OC),
                                           *reinterpret_cast<uint32_t (*)[32]>(acc));
                    else
                        tmem_ld_32x32b_x16(tmem_base + lane_base + TMEM_O + (uint32_t)(slice * OC),
                                           *reinterpret_cast<uint32_t (*)[16]>(acc));
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_empty[ob]);
                    const int q = q0 + r;
                    if (q < T) {
                        const int32_t inv = fisr(rsum, p.rsqrt_offset);
                        uint32_t w4[OC / 4];
                        if (epi_simple) {
                            // both shifts in [1, 31]: three-op rounding shifts
#pragma unroll
                            for (int u = 0; u < OC; ++u) {
                                int32_t v = wmul((int32_t)acc[u], inv);
                                v = wmul(wadd(wadd(v, k_rsq.rnd), v >> 31) >> k_rsq.sh, inv);
                                v = wmul(wadd(wadd(v, k_rsq.rnd), v >> 31) >> k_rsq.sh, (int32_t)p.av_mult);
                                v = clampi(wadd(wadd(v, k_av.rnd), v >> 31) >> k_av.sh, -127, 127);
                                if ((u & 3) == 0) w4[u >> 2] = 0;
                                w4[u >> 2] |= (uint32_t)(uint8_t)v << (8 * (u & 3));
                            }
                        } else {
#pragma unroll
                            for (int u = 0; u < OC; ++u) {
                                int32_t v = rrs_apply(wmul((int32_t)acc[u], inv), k_rsq);
                                v = rrs_apply(wmul(v, inv), k_rsq);
                                v = rrs_apply(wmul(v, (int32_t)p.av_mult), k_av);
                                v = clampi(v, -127, 127);
                                if ((u & 3) == 0) w4[u >> 2] = 0;
                                w4[u >> 2] |= (uint32_t)(uint8_t)v << (8 * (u & 3));
                            }
                        }
                        int8_t *o = p.out + (int64_t)(row0 + q) * p.ldo + h * 64 + slice * OC;
#pragma unroll
                        for (int c4 = 0; c4 < OC / 16; ++c4)
                            *reinterpret_cast<uint4 *>(o + 16 * c4) =
                                make_uint4(w4[4 * c4], w4[4 * c4 + 1], w4[4 * c4 + 2], w4[4 * c4 + 3]);
                        if (p.rowsum_out) {
                            // this slice's share of the output row's sum (signed
                            // bytes, four per dp4a), combined across slices below
                            int32_t sum = 0;
#pragma unroll
                            for (int w = 0; w < OC / 4; ++w) sum = __dp4a((int32_t)w4[w], 0x01010101, sum);
                            sRedRow[slice * BQ + r] = sum;
                        }
                    }
                }
                oph ^= 1;  // one O buffer (ob stays 0)
                if (p.rowsum_out) {
                    // one atomic per row and head: slice-0 warps add the slices' sums
                    bar_soft();
                    const int q = q0 + r;
                    if (slice == 0 && q < T) {
                        int32_t sum = 0;
#pragma unroll
                        for (int sl = 0; sl < SLICES; ++sl) sum += sRedRow[sl * BQ + r];
                        atomicAdd(p.rowsum_out + row0 + q, sum);
                    }
                }
            }
            if (has1) {
                // combine the column slices of each row
                sRedMax[slice * BQ + r] = mx;
                bar_soft();
#pragma unroll
                for (int sl = 0; sl < SLICES; ++sl) mx = max(mx, sRedMax[sl * BQ + r]);
                // requantised row max + 1 (int16 wrap), qk_requant_rowmax_scalar
                const int32_t sraw = rrs_masked((int32_t)((uint32_t)mx * p.qk_mult), p);
                const int32_t smax = clampi(sraw, -32768, 32767);
                rmax1 = (int32_t)(int16_t)(smax + 1);
                // For a row whose requantised max is below 32767 (no int16 wrap
                // of rowmax+1) and whose rowmax1 + 32768 >= t1, neither the int16
                // clamp of a score nor the int16 wrap of its difference can
                // change the table index: idx = min(rowmax1 - s, t1) with s
                // unclamped. The warp uses that path only when all of its 32
                // rows qualify. On that path the index is computed from the raw
                // score in two multiply-adds: with y = acc*m + rnd - [acc < 0]
                // (the rounding shift's numerator, |acc*m| < 2^28) and the
                // row's unclamped requantised max rowmax1 - 1 = y_max >> sh,
                //   rowmax1 - (y >> sh) = (C - acc*m + [acc < 0]) >> sh,
                //   C = (rowmax1 + 1) * 2^sh - 1 - rnd,
                // where the numerator lies in [2^sh, 2^29 + 2^(sh+1)) and so is
                // exact in unsigned 32-bit arithmetic for sh <= 30.
                warp_simple =
                    __all_sync(0xffffffffu, sraw > -32768 && sraw < 32767 && rmax1 + 32768 >= (int32_t)t1) &&
                    p.qk_sh <= 30;
                cidx = ((uint32_t)(rmax1 + 1) << p.qk_sh) - 1u - p.qk_rnd;
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
    pdl_wait();
    pdl_launch();
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

cudaError_t transpose_v(const int8_t *v, int64_t ldv, int B, int T, int H, int8_t *vt, int vt_ld, cudaStream_t st) {
    if (B <= 0 || H <= 0 || T <= 0) return cudaSuccess;
    dim3 tg((vt_ld + 63) / 64, B * H);
    return launch_pdl(transpose_v_kernel, tg, 256, 0, st, v, ldv, B, T, H, vt, vt_ld);
}

cudaError_t attention_tc(const AttnArgs &a, int B, int H, const uint8_t *tab, int8_t *vt, int vt_ld, bool vt_ready,
                         cudaStream_t st) {
    using namespace attn;
    const int T = a.Tk;
    cudaError_t e = cudaSuccess;
    if (!vt_ready) {
        e = transpose_v(a.v, a.ldv, B, T, H, vt, vt_ld, st);
        if (e != cudaSuccess) return e;
    }
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
    p.rowsum_out = a.rowsum_out;
    static SmemLimit lim_fast, lim_gen;
    const int items = B * H * ((T + BQ - 1) / BQ);
    const int grid = items < num_sms() ? items : num_sms();
    const bool fast = a.qk_mult >= 1 && a.qk_mult <= 255 && sh >= 1 && sh <= 31;
    if (fast) {
        e = raise_smem_limit(attn_tc_kernel<true>, SMEM, lim_fast);
        if (e != cudaSuccess) return e;
        return launch_pdl(attn_tc_kernel<true>, grid, THREADS, SMEM, st, tq, tk, tv, p);
    }
    e = raise_smem_limit(attn_tc_kernel<false>, SMEM, lim_gen);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_tc_kernel<false>, grid, THREADS, SMEM, st, tq, tk, tv, p);
}

cudaError_t shift_exp_table_build(int32_t fb, uint8_t *tab, int *scratch2, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(scratch2, 0xFF, sizeof(int), st);  // last_nz = -1
    if (e != cudaSuccess) return e;
    shift_exp_table_kernel<<<(32769 + 255) / 256, 256, 0, st>>>(fb, tab, scratch2);
    shift_exp_table_fill<<<32, 256, 0, st>>>(fb, tab, scratch2, attn::TAB_MAX, scratch2 + 1);
    return cudaGetLastError();
}

}  // namespace iw
