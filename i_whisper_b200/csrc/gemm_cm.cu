// gemm_cm.cu -- channel-major variant of the persistent tcgen05 (kind::i8)
// GEMM: the weight tile is the MMA's 128-row operand and BR activation rows
// are its N operand, so TMEM lane i of the accumulator holds output channel
// n0 + i and column j holds row m0 + j.
//
// Why: the I-Whisper epilogues are per-output-channel (bias, weight zero
// point, u32 multiplier, shift, GeLU parameters). With one channel per
// epilogue thread those constants live in registers for the whole tile; the
// only per-row value, the zero-point row sum of X, is broadcast from shared
// memory once per four elements. The row-major kernel (gemm_i8.cu) instead
// re-reads two 16-byte column records from shared memory per element, and
// shared-memory bandwidth is what the tensor pipe also feeds on.
//
// Work split per CTA (one CTA per SM, persistent over tiles):
//   warp 0      : TMA producer: per 128-deep k-block a 128x128 W tile and a
//                 BRx128 X tile (128-byte swizzle, K-major) into a ring;
//                 per tile, by bulk copies into a second pair of buffers,
//                 the tile's input row sums and (pre-arranged) GeLU table.
//   warp 1      : TMEM allocation (2*BR columns) and the single-thread
//                 tcgen05.mma 128xBRx32 issue loop, committing stages and
//                 accumulator buffers.
//   warps 2..17 : epilogue; warp w reads TMEM lane quadrant w%4 (32
//                 channels) and every fourth 16-row chunk.
// Outputs: int8 row-major, int8 head-major (K/V caches), int8 transposed per
// batch (V^T for the attention's P.V operand, or [B, N, T]), int16 after
// Residual15, int16 after the positional add-requant; optional per-row sums
// of the int8 output for the next GEMM's zero point. All waits are bounded.
#include <type_traits>

#include "gemm_i8.cuh"
#include "iw_common.cuh"
#include "iw_sm100.cuh"
#include "iw_tmap.cuh"

namespace iw {

template <int BR, int GK>
struct CmCfg {
    static constexpr int A_BYTES = 128 * kBlockK;  // W tile
    static constexpr int B_BYTES = BR * kBlockK;   // X tile
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RS_BYTES = BR * 4;        // row sums of the tile's rows (two buffers)
    static constexpr int PART_BYTES = 4 * BR * 4;  // per-quadrant partial output row sums
    static constexpr int GTAB_BYTES = GK == 2 ? 128 * 256 : 0;  // the tile's GeLU table, lane-interleaved (two)
    static constexpr int FIXED = 1024 + 256 + 2 * RS_BYTES + PART_BYTES + 2 * GTAB_BYTES;
    static constexpr int STAGES_FIT = (232448 - FIXED) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int TMEM_COLS = 2 * BR;
    static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
    static_assert(STAGES >= 3, "shared memory too small");
};

// Epilogue shape of this kernel: 16 warps (four per TMEM lane quadrant, so
// four per SM sub-partition to hide latency) each taking 16-row chunks.
constexpr int kCmEpiWarps = 16;
constexpr int kCmCh = 16;
constexpr int kCmThreads = 64 + 32 * kCmEpiWarps;
IW_DEV void cm_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kCmEpiWarps * 32) : "memory"); }

// Everything the epilogue needs about its channel, loaded once per tile.
struct ChanK {
    int32_t bias, nwz, mul, hmask;  // sgn*acc + bias - wz*rowsum; mulh by u32 multiplier
    int32_t sgn;                     // +1, or -1 for a channel whose folded weights are negated
    RrsK q;                          // Linear8: rrs shift; Linear32: {sh, z} of the left shift
    int32_t gmi, gmo;                // GeLU multipliers (gelu_scalar.cpp)
    RrsK gi, go;                     // GeLU shifts (clamped to [0, 32])
    int32_t pm;                      // positional add-requant multiplier
    RrsK ps;
};

IW_DEV ChanK load_chan(const EpiParams &p, int n, bool cv, int mode) {
    ChanK c{};
    c.sgn = 1;
    c.q = {0, 0, 0, 0};
    c.gi = c.go = c.ps = {0, 0, 0, 0};
    if (!cv) return c;
    uint32_t m, sh;
    if (p.per_channel) {
        m = __ldg(p.mult + n);
        sh = (uint32_t)(int32_t)__ldg(p.shift + n);
    } else {
        m = p.smult;
        sh = p.sshift;
    }
    c.bias = p.bias ? __ldg(p.bias + n) : 0;
    c.nwz = p.wz ? -(int32_t)__ldg(p.wz + n) : 0;
    c.sgn = p.wsign ? (int32_t)__ldg(p.wsign + n) : 1;
    c.mul = (int32_t)m;
    c.hmask = (m >> 31) ? -1 : 0;
    if (mode == EPI_L8) {
        c.q = rrs_k(sh);
    } else {  // Linear32: wrapping left shift, 0 for shifts >= 32 (linear32_simd.cpp:231-255)
        c.q = sh < 32 ? RrsK{0, 0, (int32_t)sh, -1} : RrsK{0, 0, 0, 0};
    }
    if (p.gelu) {
        const int ci = p.gelu_in_pc ? n : 0, co = p.gelu_out_pc ? n : 0;
        c.gmi = __ldg(p.gmi + ci);
        c.gmo = __ldg(p.gmo + co);
        c.gi = rrs_k((uint32_t)clampi(__ldg(p.gsi + ci), 0, 32));
        c.go = rrs_k((uint32_t)clampi(__ldg(p.gso + co), 0, 32));
    }
    if (p.posadd) {
        const int pi = p.pos_pc ? n : 0;
        c.pm = (int32_t)__ldg(p.pm + pi);
        const int32_t s = __ldg(p.ps + pi);
        c.ps = rrs_k((uint32_t)(s > 0 ? s : 0));
    }
    return c;
}

// gelu_scalar.cpp:10-181 for one int8 value with the 16-entry LUT held in
// four registers.
IW_DEV int32_t gelu_k(int32_t x, const ChanK &c, const uint32_t (&lut)[4]) {
    int32_t i = rrs_apply(x * c.gmi, c.gi);
    i = clampi(i + 8, 0, 15);
    const uint32_t sel = (uint32_t)i & 7u;
    const uint32_t lo = __byte_perm(lut[0], lut[1], sel), hi = __byte_perm(lut[2], lut[3], sel);
    const int32_t l = (int32_t)(((i & 8) ? hi : lo) & 0xFFu);
    const int32_t v = rrs_apply(x * l * c.gmo, c.go);
    return clampi(v, -127, 127);
}

// GeLU through the tile's table in shared memory: the result for value x
// of channel (quadrant q, lane l) is byte q*8192 + (x + 128)*32 + l, so a
// lookup is one multiply-add and one byte load (the lanes of a 4-lane group
// share a bank word per value; other lanes never conflict). gb points at
// byte q*8192 + 128*32 + l. The result is the table byte zero-extended (the
// int8 bit pattern in bits 0..7): every consumer of this path stores bytes
// or uses (v ^ 0x80) & 0xFF.
IW_DEV int32_t gelu_tab_k(int32_t x, const uint8_t *gb) { return (int32_t)gb[x * 32]; }

// GK: GeLU flavour of a Linear8 epilogue: 0 none, 1 from its parameters
// (ALU), 2 from the per-channel lookup table.
template <int BR, int MODE, int GK>
__global__ void __launch_bounds__(kCmThreads, 1)
    gemm_cm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmR, int M, int N, int K, int WR, const EpiParams p,
                   bool res_prefetch) {
    using Cfg = CmCfg<BR, GK>;
    constexpr int S = Cfg::STAGES;
    constexpr bool GT = GK == 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + S * Cfg::A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::STAGE_BYTES);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + 2;
    uint64_t *aux_full = tempty + 2;   // [2] row sums / GeLU table of a tile landed
    uint64_t *aux_empty = aux_full + 2;  // [2] the epilogue is done with them
    uint64_t *drain = aux_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile uint32_t *stop_s = tmem_slot + 2;
    int32_t *rs_s = reinterpret_cast<int32_t *>(smem + S * Cfg::STAGE_BYTES + 256);  // [2][BR]
    int32_t *part = rs_s + 2 * BR;
    uint32_t *gtab_s = reinterpret_cast<uint32_t *>(part + 4 * BR);  // [2][8192]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ch_tiles = (N + 127) / 128;
    // WR > 0: X is M/WR windows of WR rows (a 3-D tensor map; rows may
    // overlap, which reads a channels-last activation as the im2col matrix
    // of a convolution); row tiles never straddle two windows
    const int tpw = WR > 0 ? (WR + BR - 1) / BR : 1;
    const int row_tiles = WR > 0 ? (M / WR) * tpw : (M + BR - 1) / BR;
    // first output row, row end, window and row within the window of row tile rt
    auto tile_rows = [&](int rt, int &m0, int &mend, int &wb, int &tw) {
        if (WR > 0) {
            wb = rt / tpw;
            tw = (rt - wb * tpw) * BR;
            m0 = wb * WR + tw;
            mend = wb * WR + WR;
        } else {
            wb = 0;
            tw = m0 = rt * BR;
            mend = M;
        }
    };
    const int tiles = ch_tiles * row_tiles;
    const int kblocks = (K + kBlockK - 1) / kBlockK;
    // Row sums of a full row tile come by one bulk copy when 16-byte aligned;
    // the GeLU table does when given in the pre-arranged layout.
    const bool rs_bulk = p.wz && (reinterpret_cast<uintptr_t>(p.rowsum) & 15) == 0;
    const bool gt_bulk = GT && p.gelu_tab_tiled && (reinterpret_cast<uintptr_t>(p.gelu_tab_tiled) & 15) == 0;
    // row-major int8 output stored as 32-bit words of four channels (per
    // warp: V^T, KV-cache and head-major channels take their own paths).
    // Measured on the GeLU-table path (fc1: 1739 vs 1650 TOPS); the plain
    // Linear8 epilogue keeps single-byte stores (QKV: 1939 vs 1878 TOPS).
    const bool quad_rows = MODE == EPI_L8 && GT && !p.posadd && (N & 3) == 0 && (p.ldo & 3) == 0 &&
                           (reinterpret_cast<uintptr_t>(p.out) & 3) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kCmEpiWarps);
            mbar_init(&aux_full[b], 1);
            mbar_init(&aux_empty[b], kCmEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *stop_s = 0;
        fence_mbar_init();
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmX);
        if (MODE == EPI_L32_RES && res_prefetch) prefetch_tmap(&tmR);
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
            uint32_t issued_mask = 0, last_parity = 0;
            int ab = 0;
            uint32_t aph = 0, aux_issued = 0, aux_parity = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
                int m0, mend, wb, tw;
                tile_rows(tile / ch_tiles, m0, mend, wb, tw);
                const int n0 = (tile % ch_tiles) * 128;
                {
                    // the tile's epilogue inputs (an empty transaction when
                    // the epilogue warps load them themselves)
                    if (!mbar_wait(&aux_empty[ab], aph ^ 1)) { *abort_flag = 1; break; }
                    const bool rs_t = rs_bulk && m0 + BR <= mend;
                    mbar_arrive_expect_tx(&aux_full[ab], (rs_t ? Cfg::RS_BYTES : 0) + (gt_bulk ? Cfg::GTAB_BYTES : 0));
                    if (rs_t) bulk_load(rs_s + ab * BR, p.rowsum + m0, Cfg::RS_BYTES, &aux_full[ab]);
                    if (gt_bulk)
                        bulk_load(gtab_s + ab * 8192, p.gelu_tab_tiled + (int64_t)(n0 >> 7) * Cfg::GTAB_BYTES,
                                  Cfg::GTAB_BYTES, &aux_full[ab]);
                    aux_issued |= 1u << ab;
                    aux_parity = (aux_parity & ~(1u << ab)) | (aph << ab);
                    if (++ab == 2) { ab = 0; aph ^= 1; }
                }
                // Linear32 + Residual15: the tile's residual block (BR rows x
                // 128 int16 channels) into L2 now, so that the epilogue's
                // residual loads, a main loop later, hit L2
                if (MODE == EPI_L32_RES && res_prefetch) tma_prefetch_l2_2d(&tmR, n0 * 2, m0);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(&tmW, &full[stage], sA + stage * Cfg::A_BYTES, kb * kBlockK, n0);
                    if (WR > 0)
                        tma_load_3d(&tmX, &full[stage], sB + stage * Cfg::B_BYTES, kb * kBlockK, tw, wb);
                    else
                        tma_load_2d(&tmX, &full[stage], sB + stage * Cfg::B_BYTES, kb * kBlockK, m0);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                }
            }
            // every copy this thread issued must land before the CTA exits
            for (int s = 0; s < S; ++s)
                if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u);
            for (int b = 0; b < 2; ++b)
                if (aux_issued & (1u << b)) mbar_wait(&aux_full[b], (aux_parity >> b) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(128, BR);
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t bphase = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
                if (!mbar_wait(&tempty[buf], bphase ^ 1)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * BR);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * Cfg::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int ks = 0; ks < kBlockK / 32; ++ks)
                        mma_i8(d, sdesc_kmajor_sw128(a0 + ks * 32), sdesc_kmajor_sw128(b0 + ks * 32), idesc,
                               (kb | ks) != 0);
                    mma_commit(&empty[stage]);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                }
                if (!ok) { *abort_flag = 1; break; }
                mma_commit(&tfull[buf]);
                buf ^= 1;
                if (buf == 0) bphase ^= 1;
            }
            mma_commit(drain);
            mbar_wait(drain, 0);
        }
    } else {
        const int ew = warp - 2;
        const int quad = warp & 3;  // TMEM lane quadrant this warp may read
        const int slice = ew >> 2;  // chunks slice, slice + 4, ...
        const int et = ew * 32 + lane;
        uint32_t lut[4] = {0, 0, 0, 0};
        if (GK == 1) {
#pragma unroll
            for (int w = 0; w < 4; ++w)
                lut[w] = (uint32_t)p.lut[4 * w] | ((uint32_t)p.lut[4 * w + 1] << 8) |
                         ((uint32_t)p.lut[4 * w + 2] << 16) | ((uint32_t)p.lut[4 * w + 3] << 24);
        }
        int buf = 0;
        uint32_t bphase = 0;
        int ab = 0;
        uint32_t aph = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            int m0, Mt, wb_, tw_;
            tile_rows(tile / ch_tiles, m0, Mt, wb_, tw_);  // rows [m0, min(m0 + BR, Mt))
            const int n0 = (tile % ch_tiles) * 128;
            int32_t *rs_t = rs_s + ab * BR;
            uint32_t *gt_t = gtab_s + ab * 8192;
            // Barrier A: every epilogue warp is done with the previous tile's
            // partial row sums. One thread samples the abort flag so that all
            // epilogue warps take the same decision.
            cm_bar();
            if (et == 0) *stop_s = *abort_flag;
            if (p.wz && !(rs_bulk && m0 + BR <= Mt))
                for (int i = et; i < BR; i += kCmEpiWarps * 32)
                    rs_t[i] = (p.wz && m0 + i < Mt) ? __ldg(p.rowsum + m0 + i) : 0;
            if (GT && !gt_bulk) {
                // 16 table bytes of one channel per thread, scattered into
                // the lookup layout (used only without the pre-arranged table)
                uint8_t *gb = reinterpret_cast<uint8_t *>(gt_t);
                for (int i = et; i < 128 * 16; i += kCmEpiWarps * 32) {
                    const int ch = i & 127, tq = i >> 7;
                    int4 t4 = make_int4(0, 0, 0, 0);
                    if (n0 + ch < N) t4 = __ldg(reinterpret_cast<const int4 *>(p.gelu_tab + (int64_t)(n0 + ch) * 256) + tq);
                    const uint32_t w[4] = {(uint32_t)t4.x, (uint32_t)t4.y, (uint32_t)t4.z, (uint32_t)t4.w};
                    uint8_t *dst = gb + (ch >> 5) * 8192 + tq * 16 * 32 + (ch & 31);
#pragma unroll
                    for (int k = 0; k < 16; ++k) dst[k * 32] = (uint8_t)(w[k >> 2] >> (8 * (k & 3)));
                }
            }
            cm_bar();
            if (*stop_s) break;

            const int n = n0 + quad * 32 + lane;
            const bool cv = n < N;
            const ChanK ck = load_chan(p, n, cv, MODE);
            const bool to_tr = p.tr_out && n >= p.tr_c0;
            const bool to_kv = p.kv_k && n >= p.kv_c0;
            int8_t *kv_base = nullptr;
            if (to_kv) {
                const int c = n - p.kv_c0, hd = p.kv_H * 64;
                const int pos = p.kv_pos_dev ? *p.kv_pos_dev : p.kv_pos;
                kv_base = (c < hd ? p.kv_k : p.kv_v) + ((int64_t)((c % hd) >> 6) * p.kv_Tcap + pos) * 64 + (c & 63);
            }
            // Checkpoints made by the quantiser's frexp rule have multipliers
            // below 2^31 and shifts in [1, 31]; for such a warp the MULH needs
            // no correction and the rounding shift is three instructions.
            // Linear32: multipliers below 2^31 and shifts below 32 make it a
            // plain high product and left shift.
            const bool simple = __all_sync(
                0xffffffffu, !cv || (ck.hmask == 0 && (MODE == EPI_L8 ? ck.q.sgn == -1 : ck.q.z == -1)));

            // Linear32 + Residual15: the residuals of a chunk are loaded one
            // chunk ahead (the first while the tile's MMAs run), so the epilogue
            // does not wait a memory round trip per chunk. Each thread reads
            // and writes only its own (row, channel) elements, so prefetching
            // from the in-place residual is safe.
            int32_t rv_next[kCmCh];
            auto load_res = [&](int c) {
                const int r0 = m0 + c * kCmCh;
                const int16_t *res = p.res + (int64_t)r0 * p.ldr + n;
                if (r0 + kCmCh <= Mt) {
                    // one pointer stepped by the row stride: measured cheaper
                    // than a 32-bit row offset per element (j * ld) added to
                    // a 64-bit base
#pragma unroll
                    for (int j = 0; j < kCmCh; ++j) {
                        rv_next[j] = cv ? (int32_t)*res : 0;
                        res += p.ldr;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kCmCh; ++j)
                        rv_next[j] = (cv && r0 + j < Mt) ? (int32_t)res[(int64_t)j * p.ldr] : 0;
                }
            };
            if constexpr (MODE == EPI_L32_RES) {
                if (m0 + slice * kCmCh < Mt) load_res(slice);
            }
            // every lane waits (the warp stays converged) for the bulk copies,
            // acquiring their data, and for the accumulator
            bool ok = mbar_wait(&aux_full[ab], aph) && mbar_wait(&tfull[buf], bphase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) *abort_flag = 1;
            } else {
                tc_fence_after();
#pragma unroll 1
                for (int c = slice; c < BR / kCmCh; c += kCmEpiWarps / 4) {
                    const int r0 = m0 + c * kCmCh;
                    if (r0 >= Mt) break;  // warp-uniform
                    uint32_t acc[kCmCh];
                    tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BR + c * kCmCh),
                                       acc);
                    tmem_ld_wait();
                    const int4 *rs4 = reinterpret_cast<const int4 *>(rs_t + c * kCmCh);
                    int32_t v[kCmCh];
                    // the simple epilogue's element chain from the zero-point-corrected
                    // accumulator a; ZP: a = acc + bias - wz*rowsum, else a = sgn*acc + bias
                    auto simple_chain = [&](auto zp) {
#pragma unroll
                        for (int q = 0; q < kCmCh / 4; ++q) {
                            int32_t rs[4] = {0, 0, 0, 0};
                            if constexpr (decltype(zp)::value) {
                                const int4 r4 = rs4[q];
                                rs[0] = r4.x; rs[1] = r4.y; rs[2] = r4.z; rs[3] = r4.w;
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int j = 4 * q + u;
                                int32_t a;
                                if constexpr (decltype(zp)::value)
                                    a = u_mad(ck.nwz, rs[u], u_add((int32_t)acc[j], ck.bias));
                                else
                                    a = u_mad((int32_t)acc[j], ck.sgn, ck.bias);
                                if constexpr (MODE != EPI_L8) {
                                    v[j] = (int32_t)((uint32_t)__mulhi(a, ck.mul) << ck.q.sh);
                                    continue;
                                }
                                // rrs(mulh(a, mul), sh) = (h + rnd - [h < 0]) >> sh with
                                // h = hi(a * mul); for 0 <= mul < 2^31 h has the sign of
                                // a, so both corrections are multiply-adds:
                                // t = hi(a * mul) + rnd, then t += hi(a * 1) (-1 or 0)
                                int32_t t;
                                asm("mad.hi.s32 %0, %1, %2, %3;" : "=r"(t) : "r"(a), "r"(ck.mul), "r"(ck.q.rnd));
                                asm("mad.hi.s32 %0, %1, 1, %0;" : "+r"(t) : "r"(a));
                                v[j] = clampi(t >> ck.q.sh, -127, 127);
                            }
                        }
                    };
                    if (simple) {
                        if (p.wz) simple_chain(std::true_type{});
                        else simple_chain(std::false_type{});
                    } else {
#pragma unroll
                        for (int q = 0; q < kCmCh / 4; ++q) {
                            const int4 r4 = rs4[q];
                            const int32_t rs[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int j = 4 * q + u;
                                const int32_t a = u_mad(ck.nwz, rs[u], u_mad((int32_t)acc[j], ck.sgn, ck.bias));
                                const int32_t h = u_add(__mulhi(a, ck.mul), a & ck.hmask);
                                if constexpr (MODE == EPI_L8) {
                                    v[j] = clampi(rrs_apply(h, ck.q), -127, 127);
                                } else {
                                    v[j] = (int32_t)((uint32_t)h << ck.q.sh) & ck.q.z;
                                }
                            }
                        }
                    }
                    if constexpr (MODE == EPI_L32_RES) {
                        // residual15_scalar.cpp:9-27 on the Linear32 output
                        int32_t rv[kCmCh];
#pragma unroll
                        for (int j = 0; j < kCmCh; ++j) rv[j] = rv_next[j];
                        const int cn = c + kCmEpiWarps / 4;  // this warp's next chunk
                        if (cn < BR / kCmCh && m0 + cn * kCmCh < Mt) load_res(cn);
                        if (cv) {
                            const int rm = (int32_t)p.res_mult;
                            int16_t *out = reinterpret_cast<int16_t *>(p.out);
                            int16_t *o16 = out + (int64_t)r0 * p.ldo + n;
                            if (r0 + kCmCh <= Mt) {
                                // whole chunk: the row pointer stepped by the stride
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    int32_t t = u_mad(rv[j], rm, v[j]);
                                    t = u_add(u_add(t, 1 << 14), t >> 31) >> 15;
                                    *o16 = (int16_t)clampi(t, -16383, 16383);
                                    o16 += p.ldo;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    if (r0 + j < Mt) {
                                        int32_t t = u_mad(rv[j], rm, v[j]);
                                        t = u_add(u_add(t, 1 << 14), t >> 31) >> 15;
                                        o16[(int64_t)j * p.ldo] = (int16_t)clampi(t, -16383, 16383);
                                    }
                                }
                            }
                        }
                    } else {
                        if constexpr (GT) {
                            const uint8_t *gb = reinterpret_cast<const uint8_t *>(gt_t) + quad * 8192 + 128 * 32 + lane;
#pragma unroll
                            for (int j = 0; j < kCmCh; ++j) v[j] = gelu_tab_k(v[j], gb);
                        } else if constexpr (GK == 1) {
#pragma unroll
                            for (int j = 0; j < kCmCh; ++j) v[j] = gelu_k(v[j], ck, lut);
                        }
                        // (lanes of channels past N hold v = 0: the tensor map
                        // zero-fills their weight rows and load_chan zeroes
                        // their constants, so acc, the requantised value and
                        // its GeLU are all 0)
                        if (!GT && p.posadd) {  // (never with a GeLU table: its bytes are zero-extended)
                            // add_requant15_scalar.cpp:29-80, int16 result
                            if (cv) {
                                int16_t *out = reinterpret_cast<int16_t *>(p.out);
                                int32_t pe[kCmCh];
                                int t = r0 % p.pe_T;
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    pe[j] = (r0 + j < Mt) ? (int32_t)__ldg(p.pe + (int64_t)t * N + n) : 0;
                                    if (++t == p.pe_T) t = 0;
                                }
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    if (r0 + j < Mt) {
                                        const int32_t a = clampi(rrs_apply(wmul(v[j] + pe[j], ck.pm), ck.ps), -16383, 16383);
                                        out[(int64_t)(r0 + j) * p.ldo + n] = (int16_t)a;
                                    }
                                }
                            }
                        } else if (to_tr) {
                            // per-batch transposed rows: tr_out[(b*tr_N + n - tr_c0)*tr_ld + t]
                            if (cv) {
                                int b = r0 / p.tr_T, t = r0 - (r0 / p.tr_T) * p.tr_T;
                                const bool vec = (p.tr_T & 3) == 0 && (p.tr_ld & 3) == 0 &&
                                                 (reinterpret_cast<uintptr_t>(p.tr_out) & 3) == 0;
                                // (with tr_T % 4 == 0 and r0 % 16 == 0 a group of four
                                // rows never straddles two batches; dst follows (b, t))
                                int8_t *dst = p.tr_out + ((int64_t)b * p.tr_N + (n - p.tr_c0)) * p.tr_ld + t;
                                const int64_t bstep = (int64_t)p.tr_N * p.tr_ld - p.tr_T;
#pragma unroll
                                for (int j = 0; j < kCmCh; j += 4) {
                                    const int m = r0 + j;
                                    if (vec && m + 3 < Mt) {
                                        *reinterpret_cast<uint32_t *>(dst) =
                                            (uint32_t)(uint8_t)v[j] | ((uint32_t)(uint8_t)v[j + 1] << 8) |
                                            ((uint32_t)(uint8_t)v[j + 2] << 16) | ((uint32_t)(uint8_t)v[j + 3] << 24);
                                        t += 4;
                                        dst += 4;
                                        if (t == p.tr_T) { t = 0; ++b; dst += bstep; }
                                    } else {
#pragma unroll
                                        for (int u = 0; u < 4; ++u) {
                                            if (m + u < Mt)
                                                p.tr_out[((int64_t)b * p.tr_N + (n - p.tr_c0)) * p.tr_ld + t] =
                                                    (int8_t)v[j + u];
                                            if (++t == p.tr_T) { t = 0; ++b; }
                                        }
                                        dst = p.tr_out + ((int64_t)b * p.tr_N + (n - p.tr_c0)) * p.tr_ld + t;
                                    }
                                }
                            }
                        } else if (to_kv) {
                            // self-attention K/V cache rows at the current position
                            if (cv) {
                                int b = r0 / p.kv_T, t = r0 - (r0 / p.kv_T) * p.kv_T;
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    if (r0 + j < Mt)
                                        kv_base[((int64_t)b * p.kv_H * p.kv_Tcap + t) * 64] = (int8_t)v[j];
                                    if (++t == p.kv_T) { t = 0; ++b; }
                                }
                            }
                        } else if (p.hm_T) {
                            // head-major K/V cache rows
                            if (cv) {
                                int8_t *base = reinterpret_cast<int8_t *>(p.out) + (int64_t)(n >> 6) * p.hm_B * p.hm_T * 64 +
                                               (n & 63);
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j)
                                    if (r0 + j < Mt) base[(int64_t)(r0 + j) * 64] = (int8_t)v[j];
                            }
                        } else if (quad_rows && r0 + kCmCh <= Mt) {
                            // Row-major int8 in 32-bit pieces: a 4x4 byte transpose
                            // across each group of four lanes (channels 4g..4g+3)
                            // gives lane 4g+i the four channels' bytes of row
                            // 4q+i, stored as one word (lanes of channels past N
                            // hold 0 and store only when their group is in range)
                            const int gi = lane & 3;
                            const uint32_t sel1 = (gi & 2) ? 0x3276u : 0x5410u;
                            const uint32_t sel2 = (gi & 1) ? 0x3715u : 0x6240u;
                            const int cn = n0 + quad * 32 + (lane & ~3);
                            int8_t *ob = reinterpret_cast<int8_t *>(p.out) + (int64_t)(r0 + gi) * p.ldo + cn;
                            const int64_t ld4 = 4 * p.ldo;
#pragma unroll
                            for (int q = 0; q < kCmCh / 4; ++q) {
                                const uint32_t w = __byte_perm(__byte_perm(v[4 * q], v[4 * q + 1], 0x0040u),
                                                               __byte_perm(v[4 * q + 2], v[4 * q + 3], 0x0040u), 0x5410u);
                                const uint32_t x = __byte_perm(w, __shfl_xor_sync(0xffffffffu, w, 2), sel1);
                                const uint32_t t = __byte_perm(x, __shfl_xor_sync(0xffffffffu, x, 1), sel2);
                                if (cn < N) *reinterpret_cast<uint32_t *>(ob) = t;
                                ob += ld4;
                            }
                        } else if (cv) {
                            int8_t *out = reinterpret_cast<int8_t *>(p.out) + (int64_t)r0 * p.ldo + n;
                            if (r0 + kCmCh <= Mt) {
                                // whole chunk: the row pointer stepped by the stride
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    *out = (int8_t)v[j];
                                    out += p.ldo;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < kCmCh; ++j) {
                                    if (r0 + j < Mt) *out = (int8_t)v[j];
                                    out += p.ldo;
                                }
                            }
                        }
                        if (p.rowsum_out) {
                            // Per row, the sum over this warp's 32 channels, two
                            // rows per reduction: each lane adds v + 128 (0..255,
                            // from the low byte whether v is sign- or
                            // zero-extended) into one 16-bit half, so a half
                            // totals at most 32 * 255 and the row sum is that
                            // total - 32 * 128 (lanes of channels past N hold 0).
                            uint32_t rsum[kCmCh / 2];
#pragma unroll
                            for (int j = 0; j < kCmCh / 2; ++j) {
                                uint32_t w;  // v0 + v1 * 2^16
                                asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(w) : "r"(v[2 * j + 1]), "r"(v[2 * j]));
                                // zero-extended bytes (GeLU table): flip the sign bits;
                                // sign-extended values: add 128 to each half
                                w = GT ? (w ^ 0x00800080u) : (w + 0x00800080u);
                                rsum[j] = __reduce_add_sync(0xffffffffu, w);
                            }
                            if (lane == 0) {
                                int4 *dst = reinterpret_cast<int4 *>(part + quad * BR + c * kCmCh);
#pragma unroll
                                for (int q4 = 0; q4 < kCmCh / 4; ++q4)
                                    dst[q4] = make_int4((int32_t)(rsum[2 * q4] & 0xFFFFu) - 4096,
                                                        (int32_t)(rsum[2 * q4] >> 16) - 4096,
                                                        (int32_t)(rsum[2 * q4 + 1] & 0xFFFFu) - 4096,
                                                        (int32_t)(rsum[2 * q4 + 1] >> 16) - 4096);
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            // this warp's shared-memory accesses to the tile's row sums and
            // table come before the next bulk copy into the buffer
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tempty[buf]);
                mbar_arrive(&aux_empty[ab]);
            }
            buf ^= 1;
            if (buf == 0) bphase ^= 1;
            if (++ab == 2) { ab = 0; aph ^= 1; }
            if (MODE == EPI_L8 && p.rowsum_out) {
                // Barrier C: all four quadrants' partial sums of each row are in.
                cm_bar();
                for (int i = et; i < BR; i += kCmEpiWarps * 32)
                    if (m0 + i < Mt)
                        atomicAdd(p.rowsum_out + m0 + i, part[i] + part[BR + i] + part[2 * BR + i] + part[3 * BR + i]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

template <int BR, int MODE, int GK>
static cudaError_t launch_cm_t(const GemmShape &g, const EpiParams &p, cudaStream_t stream) {
    using Cfg = CmCfg<BR, GK>;
    CUtensorMap tw, tx;
    cudaError_t e = make_tmap_2d_u8(&tw, g.w, (uint64_t)g.K, (uint64_t)g.N, (uint64_t)g.ldw, kBlockK, 128);
    if (e != cudaSuccess) return e;
    if (g.win_rows > 0)
        e = make_tmap_3d_windows_u8(&tx, g.x, (uint64_t)g.K, (uint64_t)g.win_rows, (uint64_t)(g.M / g.win_rows),
                                    (uint64_t)g.ldx, (uint64_t)g.win_stride, kBlockK, BR);
    else
        e = make_tmap_2d_u8(&tx, g.x, (uint64_t)g.K, (uint64_t)g.M, (uint64_t)g.ldx, kBlockK, BR);
    if (e != cudaSuccess) return e;
    // residual block prefetch map (bytes: 128 int16 channels x BR rows); off
    // when the residual is not 16-byte aligned for the tensor map
    CUtensorMap tr = tx;
    bool res_pf = false;
    if (MODE == EPI_L32_RES && p.res && (reinterpret_cast<uintptr_t>(p.res) & 15) == 0 && ((p.ldr * 2) & 15) == 0)
        res_pf = make_tmap_2d_u8(&tr, p.res, (uint64_t)g.N * 2, (uint64_t)g.M, (uint64_t)p.ldr * 2, 256, BR,
                                 CU_TENSOR_MAP_SWIZZLE_NONE) == cudaSuccess;
    static SmemLimit lim;
    e = raise_smem_limit(gemm_cm_kernel<BR, MODE, GK>, Cfg::SMEM, lim);
    if (e != cudaSuccess) return e;
    const long row_tiles = g.win_rows > 0 ? (long)(g.M / g.win_rows) * ((g.win_rows + BR - 1) / BR)
                                          : (long)((g.M + BR - 1) / BR);
    const long tiles = (long)((g.N + 127) / 128) * row_tiles;
    const int grid = tiles < num_sms() ? (int)tiles : num_sms();
    return launch_pdl(gemm_cm_kernel<BR, MODE, GK>, grid, kCmThreads, Cfg::SMEM, stream, tw, tx, tr, g.M, g.N, g.K,
                      g.win_rows, p, res_pf);
}

template <int MODE, int GK>
static cudaError_t launch_cm_mode(const GemmShape &g, const EpiParams &p, cudaStream_t stream, int br) {
    if (br == 64) return launch_cm_t<64, MODE, GK>(g, p, stream);
    if (br == 128) return launch_cm_t<128, MODE, GK>(g, p, stream);
    return launch_cm_t<256, MODE, GK>(g, p, stream);
}

// The channel-major path covers Linear8 (per-channel or scalar requant,
// optional GeLU from its parameters or a per-channel lookup table,
// positional add, row-major, head-major, KV-cache or per-batch transposed
// int8 output, optional output row sums) and Linear32 + Residual15.
bool cm_eligible(const GemmShape &g, EpiMode mode, const EpiParams &p) {
    // Linear8 and Linear32 + Residual15 (measured 1030 vs 864 TOPS at
    // K=1024 and 2241 vs 2157 at K=4096 against the row-major kernel).
    if (mode != EPI_L8 && mode != EPI_L32_RES) return false;
    if (p.vt_T) return false;
    if (p.gelu_tab && (p.gelu || !p.per_channel || p.posadd)) return false;
    if (mode == EPI_L32_RES && (!p.per_channel || p.gelu || p.posadd || p.hm_T || p.tr_out || p.rowsum_out))
        return false;
    if (mode == EPI_L32_RES && (reinterpret_cast<uintptr_t>(p.out) & 1)) return false;
    if (p.posadd && (p.hm_T || p.tr_out || p.rowsum_out)) return false;
    if (p.kv_k && (p.posadd || p.hm_T || p.tr_out || p.kv_T <= 0)) return false;
    if (p.tr_out && (p.tr_T <= 0 || p.tr_N <= 0)) return false;
    return true;
}

cudaError_t gemm_cm_launch(const GemmShape &g, EpiMode mode, const EpiParams &p, cudaStream_t stream, int br) {
    if (br == 0) {
        const long ch_tiles = (g.N + 127) / 128;
        br = 256;
        if (ch_tiles * ((g.M + 255) / 256) < num_sms() / 2) br = 128;
        if (ch_tiles * ((g.M + 127) / 128) < num_sms() / 2) br = 64;
    }
    if (mode == EPI_L8) {
        if (p.gelu_tab) return launch_cm_mode<EPI_L8, 2>(g, p, stream, br);
        if (p.gelu) return launch_cm_mode<EPI_L8, 1>(g, p, stream, br);
        return launch_cm_mode<EPI_L8, 0>(g, p, stream, br);
    }
    return launch_cm_mode<EPI_L32_RES, 0>(g, p, stream, br);
}

}  // namespace iw
