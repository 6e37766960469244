// kernels.cuh -- launchers of the bandwidth-bound kernels (kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace iw {

struct LnParams {
    int32_t ln_mult;       // u8 value
    int32_t ln_shift;      // int8 value
    uint32_t out_mult;     // u32
    uint32_t out_shift;    // (uint32)(int32)int8: negative -> >= 32 -> 0
    uint32_t rsqrt_offset; // 13 (LayerNorm_int.offset); 15 for LayerNorm64
    int32_t additional_offset = 0;  // LayerNorm64 normalise-shift offset (2)
    int *overflow = nullptr;        // LayerNorm64: set to 1 when a variance does not fit INT32
};

struct GeluParams {
    const uint8_t *lut;
    const uint8_t *mi;
    const int8_t *si;
    const uint8_t *mo;
    const int8_t *so;
    int n_in, n_out;
};

struct AttnArgs {
    // element (b, t, h, d) of Q is q[b*q_bs + t*ldq + h*q_hs + d]; same for
    // K, V and the output with their own strides (head strides default 64)
    const int8_t *q;
    int64_t ldq, q_bs, q_hs = 64;
    const int8_t *k;
    int64_t ldk, k_bs, k_hs = 64;
    const int8_t *v;
    int64_t ldv, v_bs, v_hs = 64;
    int8_t *out;
    int64_t ldo, o_bs, o_hs = 64;
    int Tq, Tk;
    const int32_t *Tk_dev;  // optional: key count read on the device
    int Tk_cap;             // shared-memory capacity in keys (>= any Tk)
    int mask_mode;          // 0 none, 1 causal (key j > Tk-Tq+i masked), 2 explicit [Tq,Tk]
    const uint8_t *mask;
    uint32_t qk_mult;
    int32_t qk_shift;
    int32_t frac_bits;
    uint32_t av_mult;
    int32_t av_shift;
    uint32_t rsqrt_offset;
    int32_t *rowsum_out = nullptr;  // optional: += sum of each output row, index b*Tq + q
};

cudaError_t rowsum_i8(const int8_t *x, int64_t ldx, int M, int K, int32_t *out, cudaStream_t st);
// l64: the LayerNorm64 variant (p.rsqrt_offset / additional_offset / overflow)
cudaError_t layernorm32(const int16_t *x, int64_t ldx, const int8_t *gamma, const int32_t *beta, const LnParams &p,
                        int8_t *y, int64_t ldy, int rows, int d, int32_t *rowsum_out, int32_t *rowsum_zero,
                        cudaStream_t st, bool l64 = false);
// LayerNorm64 statistics (layernorm_scalar.cpp:230-297): mean int32, variance int64
cudaError_t layernorm64_stats(const int16_t *x, int rows, int d, int32_t *mean, int64_t *var, cudaStream_t st);
cudaError_t layernorm32_stats(const int16_t *x, int rows, int d, int32_t *mean, int32_t *var, int32_t *rs,
                              cudaStream_t st);
cudaError_t fisr_vec(const int32_t *x, int32_t *y, int64_t n, uint32_t off, cudaStream_t st);
cudaError_t gelu(const int8_t *x, int8_t *y, int64_t n, int channels, const GeluParams &g, cudaStream_t st);
cudaError_t residual15(const int32_t *br, const int16_t *r, uint16_t m, int16_t *y, int64_t n, cudaStream_t st);
cudaError_t requant_rows(const int32_t *x, const uint32_t *mult, const int8_t *shift, uint32_t shamt, int32_t *y,
                         int64_t n, int64_t N, cudaStream_t st);
cudaError_t add_requant15(const int8_t *x, const int64_t *tokens, const int8_t *addend, const uint16_t *mult,
                          const int8_t *shift, int16_t *y, int B, int T, int C, int n_mult, int n_shift, int offset,
                          const int32_t *offset_dev, cudaStream_t st);
// Bounded-wait self-test (see kernels.cu); *gave_up = 1 when the wait expired.
cudaError_t selftest_wait(int *gave_up, cudaStream_t st);
cudaError_t channels_last_pad(const int8_t *x, int B, int C, int T, int front, int back, int8_t *out,
                              cudaStream_t st);
cudaError_t im2col(const int8_t *x, int8_t *out, int B, int Cin, int Tin, int K, int stride, int pad, int Tout,
                   int64_t ldo, int channels_last, cudaStream_t st);
cudaError_t pad_rows(const int8_t *x, int64_t rows, int64_t cols, int8_t *out, int64_t ldo, cudaStream_t st);
cudaError_t attention_cc(const AttnArgs &a, int B, int H, cudaStream_t st);

// Tensor-core attention for unmasked self-attention with Tq == Tk (encoder):
// Q/K rows straight from the projection buffer (16-byte aligned, batch
// stride T*ld, head h at column h*64), V transposed into vt [B*H*64, vt_ld]
// (vt_ld >= T, multiple of 16). tab from shift_exp_table_build.
// vt_ready: vt already holds V^T (written by the QKV GEMM), skip the transpose.
cudaError_t attention_tc(const AttnArgs &a, int B, int H, const uint8_t *tab, int8_t *vt, int vt_ld, bool vt_ready,
                         cudaStream_t st);
// V^T of head-major V columns: vt[(b*H + h)*64 + d][t] = v[(b*T + t)*ldv + h*64 + d].
cudaError_t transpose_v(const int8_t *v, int64_t ldv, int B, int T, int H, int8_t *vt, int vt_ld, cudaStream_t st);
// Builds the shift-exp table for frac_bits fb into tab (>= 32772 bytes);
// scratch2 is two device ints, scratch2[1] == 1 afterwards when the table is
// too long for the tensor-core kernel.
cudaError_t shift_exp_table_build(int32_t fb, uint8_t *tab, int *scratch2, cudaStream_t st);

// Append one position of self-attention K and V (row b of src, columns
// [k_col, k_col+H*64) and [v_col, v_col+H*64)) to head-major caches
// [B, H, Tcap, 64] at position *pos_dev (or `pos` when pos_dev is null).
cudaError_t kv_append(const int8_t *src, int64_t lds, int k_col, int v_col, int8_t *kc, int8_t *vc, int B, int H,
                      int T, int Tcap, int pos, const int32_t *pos_dev, cudaStream_t st);

struct GreedyArgs {
    const int8_t *logits;      // [B, V] int8 logits of the current step
    int64_t ld;
    int V;
    float alpha;               // TextDecoder_int.act_logits_alpha
    const uint32_t *suppress_bits;  // bitmap [ceil(V/32)] of SuppressTokens ids
    const int32_t *blank;      // SuppressBlank ids (encode(" ")), eot added by the kernel
    int n_blank;
    int eot, timestamp_begin, no_timestamps;
    int max_initial_timestamp_index;  // < 0: none
    int32_t *state;            // [B, 4]: n_sampled, last, penultimate, last timestamp (-1)
    int64_t *tokens;           // [B, ld_tok] token history; next token written at column *step_dev
    int64_t ld_tok;
    int32_t *step_dev;         // column of the next token (advanced by the host loop)
    int64_t *next;             // [B] next token (also fed to the embedding gather)
};
cudaError_t greedy_step(const GreedyArgs &g, int B, cudaStream_t st);

// Log-mel + INT8 quantisation of B windows of n_samples float audio (row
// stride lda): out [B, n_mels, n_samples/160]; filters [n_mels, 257] on the
// device; work [B, n_mels, n_samples/160] floats and wmax [B] ints.
cudaError_t log_mel_int8(const float *audio, int B, int n_samples, int64_t lda, const float *filters, int n_mels,
                         float alpha, float *work, int32_t *wmax, int8_t *out, cudaStream_t st);
size_t logmel_smem_bytes(int n_mels);
cudaError_t add_i32(int32_t *p, int32_t v, cudaStream_t st);
cudaError_t qk_requant_rowmax(const int8_t *q, const int8_t *k, const uint8_t *mask, int16_t *qk, int16_t *rmax1,
                              int B, int H, int Tq, int Tk, int D, uint8_t mult, int32_t shift, cudaStream_t st);
cudaError_t shift_exp(const int16_t *x, const int16_t *rmax1, const uint8_t *mask, uint8_t *p, int32_t *rowsum, int B,
                      int H, int Tq, int Tk, int fb, cudaStream_t st);
cudaError_t pv_norm_requant(const uint8_t *p, const int8_t *vt, const int32_t *rowsum, uint8_t av_mult,
                            int8_t av_shift, uint32_t off, int8_t *out, int B, int H, int Tq, int Tk, int D, int *bad,
                            cudaStream_t st);

}  // namespace iw
