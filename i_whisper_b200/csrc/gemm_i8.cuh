// gemm_i8.cuh -- host-visible description of the tcgen05 w8a8 GEMM and its
// fused epilogues.
//
// Y[m, n] = epilogue( sum_k X[m, k] * W[n, k] )   X: [M, K] int8 row-major,
//                                                W: [N, K] int8 row-major.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace iw {

enum EpiMode : int {
    EPI_ACC32 = 0,    // int32 out: acc + bias - wz*rowsum            (linear8_accum)
    EPI_L8 = 1,       // int8 out: Linear8 / conv / classifier requant (+GeLU, +pos-add)
    EPI_L32 = 2,      // int32 out: Linear32 requant (mulh, wrapping left shift)
    EPI_L32_RES = 3,  // int16 out: Linear32 requant fused with Residual15
};

struct EpiParams {
    void *out = nullptr;
    int64_t ldo = 0;  // output row stride in elements
    // zero point / bias (Linear8/32, linear.py:50-97)
    const int32_t *bias = nullptr;    // [N]
    const int8_t *wz = nullptr;       // [N] weight zero points
    const int8_t *wsign = nullptr;    // [N] +1/-1 applied to the accumulator (folded zero points; no wz)
    const int32_t *rowsum = nullptr;  // [M] sum of each X row (needed with wz)
    // requant: per channel (Linear8/32) or one scalar (conv, classifier)
    const uint32_t *mult = nullptr;   // [N]
    const int8_t *shift = nullptr;    // [N]
    int per_channel = 1;
    uint32_t smult = 0;   // scalar multiplier
    uint32_t sshift = 0;  // scalar shift, already max(s,0)
    // fused GeLU on the int8 result (gelu_scalar.cpp)
    int gelu = 0;
    const uint8_t *lut = nullptr;
    const uint8_t *gmi = nullptr;
    const int8_t *gsi = nullptr;
    const uint8_t *gmo = nullptr;
    const int8_t *gso = nullptr;
    int gelu_in_pc = 0, gelu_out_pc = 0;  // per-channel (1) or per-tensor (0)
    // fused Residual15 (EPI_L32_RES)
    const int16_t *res = nullptr;
    int64_t ldr = 0;
    uint32_t res_mult = 0;
    // fused positional add + requant to INT15 (add_requant15_scalar.cpp)
    int posadd = 0;
    const int8_t *pe = nullptr;  // [T, N]
    int pe_T = 1;                // rows m map to position m % pe_T
    const uint16_t *pm = nullptr;
    const int8_t *ps = nullptr;
    int pos_pc = 1;
    // optional: int8 output written as [B, N, T] with m = b*T + t
    int transpose_T = 0;
    // optional: per-head transposed store for attention V^T:
    // out[(b*H + h)*D + d][t] with m = b*T + t, n = h*D + d, row stride ldo
    int vt_T = 0, vt_D = 0;
    // optional: head-major store for K/V caches: column n belongs to head
    // group g = n / 64; row m = b*hm_T + t goes to
    // out[((g*hm_B + b)*hm_T + t)*64 + n%64]
    int hm_T = 0, hm_B = 0;
    // optional: accumulate per-row sums of the int8 output (next GEMM's
    // zero-point term)
    int32_t *rowsum_out = nullptr;
    // optional: per-channel GeLU as a lookup table [N][256] of int8 results
    // indexed by (requantised value + 128); built by gelu_table_build from
    // the same GeLU parameters, so it is exact
    const int8_t *gelu_tab = nullptr;
    // optional (channel-major path): the same table in the layout of
    // gelu_table_tile (one 32 KB block per 128 channels, already in the
    // kernel's shared-memory order), staged by one bulk copy per tile
    const int8_t *gelu_tab_tiled = nullptr;
    // optional (channel-major path): int8 results of channels n >= tr_c0
    // are written per batch transposed, tr_out[(b*tr_N + n - tr_c0)*tr_ld + t]
    // with m = b*tr_T + t, instead of row-major (V^T for the attention)
    int8_t *tr_out = nullptr;
    int tr_c0 = 0, tr_N = 0, tr_T = 0;
    int64_t tr_ld = 0;
    // optional (channel-major path): channels n >= kv_c0 hold the keys then
    // the values of self-attention (2 * kv_H * 64 channels), written into the
    // head-major caches [B, kv_H, kv_Tcap, 64] at position (*kv_pos_dev, or
    // kv_pos) + t for row m = b * kv_T + t, instead of row-major
    int8_t *kv_k = nullptr, *kv_v = nullptr;
    int kv_c0 = 0, kv_H = 0, kv_T = 0, kv_Tcap = 0, kv_pos = 0;
    const int32_t *kv_pos_dev = nullptr;
};

// Builds tab[n][x+128] = GeLU_n(x) for x in [-128, 127] (gelu_scalar.cpp).
cudaError_t gelu_table_build(const uint8_t *lut, const uint8_t *mi, const int8_t *si, const uint8_t *mo,
                             const int8_t *so, int n_in, int n_out, int N, int8_t *tab, cudaStream_t st);

// Rearranges tab [N][256] into the channel-major GEMM's shared-memory order:
// for each tile of 128 channels, byte q*8192 + t*32 + l holds entry t of
// channel 128*tile + 32q + l (zero past N).
cudaError_t gelu_table_tile(const int8_t *tab, int N, int8_t *tiled, cudaStream_t st);

struct GemmShape {
    const int8_t *x;
    int64_t ldx;  // row stride of X in bytes (multiple of 16)
    const int8_t *w;
    int64_t ldw;  // row stride of W in bytes (multiple of 16)
    int M, N, K;
    // optional (channel-major kernel): X as M / win_rows windows of win_rows
    // rows, window w at x + w * win_stride; ldx may be smaller than K
    // (overlapping rows: the im2col matrix of a convolution over a
    // channels-last activation, read in place)
    int win_rows = 0;
    int64_t win_stride = 0;
};

// Launches the tcgen05 GEMM with the given epilogue on `stream`.
// Returns a cudaError_t (cudaSuccess when the launch was queued).
cudaError_t gemm_i8_launch(const GemmShape &g, EpiMode mode, const EpiParams &p, cudaStream_t stream,
                           int bn_hint = 0);

// Channel-major kernel (gemm_cm.cu): the weight tile is the MMA's 128-row
// operand, so each epilogue thread owns one output channel.
bool cm_eligible(const GemmShape &g, EpiMode mode, const EpiParams &p);
cudaError_t gemm_cm_launch(const GemmShape &g, EpiMode mode, const EpiParams &p, cudaStream_t stream, int br);
// False when IW_GEMM_ROWMAJOR=1 is set in the environment (selects the
// row-major kernel for every GEMM; used to compare the two).
bool cm_enabled();

}  // namespace iw
