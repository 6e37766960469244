/*
 * iwhisper_b200.h -- C ABI of the B200 (sm_100a) integer Whisper hot path.
 *
 * Drop-in boundary for the operator library the reference binds as
 * `i_whisper.kernels._C` (vcsd-lab/I-Whisper,
 * i_whisper/kernels/csrc/pybind.cpp:45-415). Each entry point computes
 * exactly what the reference op of the same name computes (same integer
 * semantics, bit for bit) with these differences in form:
 *
 *   - all array arguments are DEVICE pointers to contiguous row-major data
 *     in the layouts of the reference op; outputs are caller-allocated;
 *   - per-tensor scalar parameters (the 1-element tensors of the reference)
 *     are passed by value;
 *   - work is queued on `stream` (a cudaStream_t, NULL = legacy default
 *     stream) and the call returns without synchronising, except where
 *     noted;
 *   - the return value is IW_OK (0) or a negative IW_E* code; the message
 *     of the last failure on the calling thread is given by iw_last_error().
 *     The reference raises RuntimeError/ValueError (TORCH_CHECK,
 *     std::invalid_argument) in the same situations.
 *
 * Optional arrays (bias, weight_zero, mask) may be NULL, like the
 * reference's std::optional<Tensor> arguments.
 */
#ifndef IWHISPER_B200_H
#define IWHISPER_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IW_OK 0
#define IW_EINVAL (-1)    /* bad shape / size / argument (TORCH_CHECK)      */
#define IW_EVALUE (-2)    /* value error (std::invalid_argument)            */
#define IW_ECUDA (-3)     /* CUDA runtime error                             */
#define IW_EDEVICE (-4)   /* device-side wait gave up (see iw_device_status) */
#define IW_EOVERFLOW (-5) /* overflow (std::overflow_error)                 */

/* Message of the last failed call on this thread ("" if none). */
const char *iw_last_error(void);
/* ABI version of this library. */
int iw_abi_version(void);
/* Synchronises the device, returns the device status word in *status
 * (bit 0: a bounded in-kernel wait timed out; bit 1: a LayerNorm64
 * variance did not fit INT32 in iw_layernorm64_ex) and clears it if `clear`. */
int iw_device_status(uint32_t *status, int clear);
/* Bound (ns) of every in-kernel mbarrier wait; default 2 s. */
int iw_set_wait_timeout_ns(uint64_t ns);
/* Failure-path self-test: a one-thread kernel waits, through the same
 * bounded wait the tcgen05 kernels use, on a barrier nothing completes;
 * when the bound expires it sets bit 0 of the device status word, writes
 * 1 to *gave_up (device int32) and returns. Nothing faults or hangs. */
int iw_selftest_wait_timeout(int32_t *gave_up, void *stream);

/* linear8_{scalar,simd} -- linear8_scalar.cpp:30-84; pybind.cpp:51-70.
 * x [M,K] int8, weight [N,K] int8, bias [N] int32?, weight_zero [N] int8?,
 * multiplier [N] uint32, shift [N] int8 -> y [M,N] int8. */
int iw_linear8(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
               const uint32_t *multiplier, const int8_t *shift, int8_t *y, int64_t M, int64_t K, int64_t N,
               void *stream);

/* linear8_accum_{scalar,simd}_debug -- linear8_scalar.cpp:87-127;
 * pybind.cpp:71-81. Same inputs, int32 accumulator out (no requant). */
int iw_linear8_accum(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                     int32_t *y, int64_t M, int64_t K, int64_t N, void *stream);

/* linear8_requant_scalar_debug -- linear8_scalar.cpp:130-150 (fixedpoint::requant,
 * common/fixedpoint.h); pybind.cpp:74-76. acc [M,N] int32 ->
 * y = rounding_rshift(mulh(acc, multiplier[n]), (uint32)shift[n]), int32, no clamp. */
int iw_linear8_requant(const int32_t *acc, const uint32_t *multiplier, const int8_t *shift, int32_t *y, int64_t M,
                       int64_t N, void *stream);

/* rounding_rshift_debug -- pybind.cpp:22-43 (fixedpoint.h:47-87):
 * y = rounding_rshift(x, shift) elementwise. */
int iw_rounding_rshift(const int32_t *x, uint32_t shift, int32_t *y, int64_t numel, void *stream);

/* linear32_{scalar,simd} -- linear32_scalar.cpp:96-129 (requant of
 * linear32_simd.cpp:231-255); pybind.cpp:82-101. -> y [M,N] int32. */
int iw_linear32(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                const uint32_t *multiplier, const int8_t *shift, int32_t *y, int64_t M, int64_t K, int64_t N,
                void *stream);

/* Fused Linear32 + residual15: y = residual15(linear32(x), residual, m).
 * Replaces the pair Linear32.forward (linear.py:118-187) ->
 * residual15_* (model_int.py:1126-1171; residual15_scalar.cpp:9-27).
 * residual/y [M,N] int16; y may alias residual (in-place update). */
int iw_linear32_residual15(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                           const uint32_t *multiplier, const int8_t *shift, const int16_t *residual,
                           uint16_t residual_multiplier, int16_t *y, int64_t M, int64_t K, int64_t N, void *stream);

/* residual15_{scalar,simd} -- residual15_scalar.cpp:9-27; pybind.cpp:115-128. */
int iw_residual15(const int32_t *branch, const int16_t *residual, uint16_t multiplier, int16_t *y, int64_t numel,
                  void *stream);

/* layernorm32_{scalar,simd} -- layernorm_scalar.cpp:464-624 with
 * rsqrt offset 13 (layernorm_torch.cpp:265); pybind.cpp:130-151.
 * x [rows,d] int16, d in {384,512,768,1024,1280} -> y [rows,d] int8. */
int iw_layernorm32(const int16_t *x, const int8_t *weight, const int32_t *bias, uint8_t ln_multiplier,
                   int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y, int64_t rows, int64_t d,
                   void *stream);

/* layernorm32_stats_{scalar,simd} -- layernorm_scalar.cpp:133-214;
 * pybind.cpp:185-194. mean/variance/renorm_shift [rows] int32. */
int iw_layernorm32_stats(const int16_t *x, int32_t *mean, int32_t *variance, int32_t *renorm_shift, int64_t rows,
                         int64_t d, void *stream);

/* layernorm64_{scalar,simd} -- layernorm_scalar.cpp:626-825;
 * pybind.cpp:163-178 (LayerNorm_int backend "scalar64"/"simd64",
 * model_int.py:252-287). Arguments as iw_layernorm32; rsqrt offset 15 and
 * normalise-shift offset 2 as fixed by layernorm_torch.cpp:446-460.
 * Synchronises; IW_EOVERFLOW when a row's int64 variance does not fit INT32
 * (std::overflow_error in the reference), the output then undefined. */
int iw_layernorm64(const int16_t *x, const int8_t *weight, const int32_t *bias, uint8_t ln_multiplier,
                   int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y, int64_t rows, int64_t d,
                   void *stream);

/* layernorm64_stats_{scalar,simd} -- layernorm_scalar.cpp:230-297;
 * pybind.cpp:153-162. mean [rows] int32, variance [rows] int64. */
int iw_layernorm64_stats(const int16_t *x, int32_t *mean, int64_t *variance, int64_t rows, int64_t d, void *stream);

/* layernorm32_rsqrt_scalar -- layernorm_scalar.cpp:383-437 (offset 13);
 * pybind.cpp:195-200. Synchronises to check that every input is >= 0. */
int iw_layernorm32_rsqrt(const int32_t *variance, int32_t *invstd, int64_t numel, void *stream);

/* gelu_{scalar,simd} -- gelu_scalar.cpp:10-181; pybind.cpp:216-235.
 * Parameters per channel (count == channels) or per tensor (count 1). */
int iw_gelu(const int8_t *x, const uint8_t *lut, const uint8_t *luti_multiplier, const int8_t *luti_shift,
            const uint8_t *luto_multiplier, const int8_t *luto_shift, int8_t *y, int64_t numel, int64_t channels,
            int64_t luti_count, int64_t luto_count, void *stream);

/* qk_requant_rowmax_{scalar,simd} -- attention_scalar.cpp:216-343;
 * pybind.cpp:251-269. q [B,H,Tq,D], k [B,H,Tk,D] int8, mask [Tq,Tk]
 * bool? -> qk [B,H,Tq,Tk] int16, row_max_plus1 [B,H,Tq] int16. */
int iw_qk_requant_rowmax(const int8_t *q, const int8_t *k, const uint8_t *mask, uint8_t multiplier, int8_t shift,
                         int16_t *qk, int16_t *row_max_plus1, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                         int64_t D, void *stream);

/* shift_exp_{scalar,simd} -- attention_scalar.cpp:388-560;
 * pybind.cpp:271-287. frac_bits in [1,14). -> p uint8, row_sum int32. */
int iw_shift_exp(const int16_t *x, const int16_t *row_max_plus1, const uint8_t *mask, int32_t frac_bits, uint8_t *p,
                 int32_t *row_sum, int64_t B, int64_t H, int64_t Tq, int64_t Tk, void *stream);

/* pv_norm_requant_{scalar,simd} -- attention_scalar.cpp:676-813;
 * pybind.cpp:303-323. p [B,H,Tq,Tk] uint8, v [B,H,D,Tk] int8, row_sum
 * [B,H,Tq] int32 -> y [B,Tq,H*D] int8. rsqrt_offset in [0,29].
 * Synchronises; a negative row sum gives IW_EVALUE. */
int iw_pv_norm_requant(const uint8_t *p, const int8_t *v, const int32_t *row_sum, uint8_t av_multiplier,
                       int8_t av_shift, int64_t rsqrt_offset, int8_t *y, int64_t B, int64_t H, int64_t Tq,
                       int64_t Tk, int64_t D, void *stream);

/* Fused integer attention (A1-A3 of MultiHeadAttention_int.qkv_attention,
 * model_int.py:774-1042) for head_dim 64, reading Q/K/V straight from the
 * projection outputs: element (b,t,h,d) of Q is q[b*q_bs + t*ldq + h*64+d]
 * (same for K, V with their strides); y[b*y_bs + t*ldy + h*64 + d].
 * mask_mode 0: none, 1: causal (key j masked when j > Tk-Tq+i, the slice of
 * TextDecoder_int.mask taken at model_int.py:786-799), 2: explicit mask
 * [Tq,Tk]. q, k, v and their row and batch strides must be multiples of
 * 16 bytes (IW_EINVAL otherwise). frac_bits in [1, 30]: calibrated
 * checkpoints carry up to 15, beyond the [1, 14) that the per-op
 * iw_shift_exp admits like the reference's _C.shift_exp. */
int iw_attention(const int8_t *q, int64_t ldq, int64_t q_bs, const int8_t *k, int64_t ldk, int64_t k_bs,
                 const int8_t *v, int64_t ldv, int64_t v_bs, int8_t *y, int64_t ldy, int64_t y_bs, int64_t B,
                 int64_t H, int64_t Tq, int64_t Tk, int mask_mode, const uint8_t *mask, uint8_t qk_multiplier,
                 int8_t qk_shift, int32_t frac_bits, uint8_t av_multiplier, int8_t av_shift, int64_t rsqrt_offset,
                 void *stream);

/* conv1d_{scalar,simd} -- conv1d_scalar.cpp:186-288; pybind.cpp:345-367.
 * x [B,Cin,Tin] int8, weight [Cout,Cin*K] int8, bias [Cout] int32? ->
 * y [B,Cout,Tout] int8, Tout = (Tin + 2*pad - K)/stride + 1. */
int iw_conv1d(const int8_t *x, const int8_t *weight, const int32_t *bias, uint32_t multiplier, int8_t shift,
              int64_t stride, int64_t padding, int8_t *y, int64_t B, int64_t Cin, int64_t Tin, int64_t Cout,
              int64_t K, void *stream);

/* add_requant15_{scalar,simd} -- add_requant15_scalar.cpp:29-80;
 * pybind.cpp:369-384. x [B,T,C] int8, addend [T,C] int8, multiplier
 * uint16 and shift int8 with 1 or C entries -> y [B,T,C] int16. */
int iw_add_requant15(const int8_t *x, const int8_t *addend, const uint16_t *multiplier, const int8_t *shift,
                     int16_t *y, int64_t B, int64_t T, int64_t C, int64_t multiplier_count, int64_t shift_count,
                     void *stream);

/* Token-embedding gather fused with add_requant15: the input row of
 * (b,t) is table[tokens[b*T+t]] and the addend row is pe[offset + t]
 * (TextDecoder_int.forward, model_int.py:1411-1428). */
int iw_embed_add_requant15(const int8_t *table, const int64_t *tokens, const int8_t *pe, int64_t offset,
                           const uint16_t *multiplier, const int8_t *shift, int16_t *y, int64_t B, int64_t T,
                           int64_t C, int64_t multiplier_count, int64_t shift_count, void *stream);

/* classifier_{scalar,simd} -- classifier_scalar.cpp:91-140;
 * pybind.cpp:399-414. x [M,K] int8, weight [N,K] int8 -> y [M,N] int8. */
int iw_classifier(const int8_t *x, const int8_t *weight, uint32_t multiplier, int8_t shift, int8_t *y, int64_t M,
                  int64_t K, int64_t N, void *stream);

/* Row sums of an int8 matrix [M,K] with row stride ldx (the sum(x) of the
 * zero-point term, linear.py:89-91). */
int iw_rowsum_i8(const int8_t *x, int64_t ldx, int64_t M, int64_t K, int32_t *y, void *stream);


/* ------------------------------------------------------------------------
 * Model-level entry points. They expose the fused forms the B200 runner
 * uses for Whisper_int.forward (model_int.py:1064-1484): GEMMs with the
 * requantisation, GeLU, Residual15, positional add and cache layouts in
 * their epilogues, attention over strided projections and head-major
 * caches, and device-side decode state so a decode step can be captured in
 * a CUDA graph and replayed.
 * ---------------------------------------------------------------------- */

/* Epilogue modes of iw_gemm_i8. */
#define IW_GEMM_ACC32 0       /* int32: acc + bias - wz*rowsum                  */
#define IW_GEMM_INT8 1        /* int8: Linear8 / conv / classifier requant      */
#define IW_GEMM_LINEAR32 2    /* int32: Linear32 requant                        */
#define IW_GEMM_LINEAR32_RES 3 /* int16: Linear32 requant + residual15          */

typedef struct iw_gemm_desc {
    const int8_t *x;          /* [M,K], row stride ldx bytes (multiple of 16)  */
    int64_t ldx;
    const int8_t *w;          /* [N,K], row stride ldw bytes (multiple of 16)  */
    int64_t ldw;
    int64_t M, N, K;          /* K multiple of 16 */
    int mode;                 /* IW_GEMM_* */
    void *out;
    int64_t ldo;              /* output row stride in elements */
    const int32_t *bias;      /* [N]? */
    const int8_t *weight_zero;/* [N]? (needs x_rowsum) */
    const int32_t *x_rowsum;  /* [M] sum of each x row */
    const uint32_t *multiplier; /* [N] per channel, or NULL for the scalar pair */
    const int8_t *shift;        /* [N] */
    uint32_t scalar_multiplier;  /* conv1d / classifier requant */
    int32_t scalar_shift;        /* used as max(shift, 0) */
    /* GeLU on the int8 result (gelu_scalar.cpp), lut != NULL enables it */
    const uint8_t *lut;
    const uint8_t *luti_multiplier;
    const int8_t *luti_shift;
    const uint8_t *luto_multiplier;
    const int8_t *luto_shift;
    int luti_per_channel, luto_per_channel;
    /* Residual15 for IW_GEMM_LINEAR32_RES: out = residual15(y, residual, m) */
    const int16_t *residual;
    int64_t ldr;
    uint32_t residual_multiplier;
    /* positional add + requant to INT15 (add_requant15_scalar.cpp) on the
     * int8 result: pos != NULL makes the output int16; row m uses position
     * m % pos_T of pos [pos_T, N]; multiplier/shift per channel or scalar */
    const int8_t *pos;
    int64_t pos_T;
    const uint16_t *pos_multiplier;
    const int8_t *pos_shift;
    int pos_per_channel;
    /* alternative int8 output layouts (0 = row-major [M,N]) */
    int64_t transpose_T;      /* out [B,N,T] with m = b*T + t                  */
    int64_t headmajor_T;      /* out [N/64, B, T, 64] with m = b*T + t          */
    int64_t headmajor_B;
    int32_t *out_rowsum;      /* [M]? accumulate row sums of the int8 output    */
    int tile_n;               /* 0 = automatic, else 64/128/256 */
    /* per-channel GeLU as a lookup table [N][256] (from iw_gelu_table); use
     * instead of the lut and luti/luto parameters on per-channel Linear8
     * outputs */
    const int8_t *gelu_table;
    /* optional V^T output for the tensor-core attention: int8 results of
     * channels n >= vt_col0 go to vt_out[(b*(N-vt_col0) + n-vt_col0)*vt_ld + t]
     * (m = b*vt_T + t) instead of out; vt_col0 a multiple of 64, M a
     * multiple of vt_T, vt_ld >= vt_T and a multiple of 16 */
    int8_t *vt_out;
    int64_t vt_ld;
    int64_t vt_col0;
    int64_t vt_T;
    /* optional self-attention KV-cache output (replaces iw_kv_append after
     * the fused QKV projection): int8 results of channels kv_col0 ..
     * kv_col0 + 2*kv_heads*64 - 1 (keys, then values) go to the head-major
     * caches [B, kv_heads, kv_Tcap, 64] at position p + t for row
     * m = b*kv_T + t, with p = *kv_pos_dev when kv_pos_dev != NULL, else
     * kv_pos; the caller keeps p + kv_T <= kv_Tcap. Those channels are not
     * written to out. kv_col0 + 2*kv_heads*64 == N, kv_col0 % 64 == 0. */
    int8_t *kv_cache_k;
    int8_t *kv_cache_v;
    int64_t kv_col0, kv_heads, kv_T, kv_Tcap, kv_pos;
    const int32_t *kv_pos_dev;
    /* optional: gelu_table rearranged by iw_gelu_table_tiled (16-byte
     * aligned); lets the kernel fetch each 128-channel tile's table with one
     * bulk copy. gelu_table must still be given. */
    const int8_t *gelu_table_tiled;
    /* optional implicit-convolution operand: when x_window_rows > 0, X is
     * M / x_window_rows windows of x_window_rows rows; row r of window w
     * starts at x + w*x_window_stride + r*ldx (bytes; both multiples of 16).
     * ldx may be smaller than K, so K-wide rows overlap: a k-tap, stride-s
     * convolution over a zero-padded channels-last activation [W][rows'][C]
     * is this GEMM with ldx = s*C, K = k*C and weights ordered (tap, channel).
     * Needs the channel-major kernel (IW_EINVAL otherwise). */
    int64_t x_window_rows;
    int64_t x_window_stride;
    /* optional [N] int8, each +1 or -1: the accumulator of channel n is
     * multiplied by weight_sign[n] before the bias is added (NULL = all +1).
     * With weight_zero NULL it lets a caller fold a zero point into the
     * weights exactly: w'[n][k] = s_n * (w[n][k] - wz[n]) gives
     * s_n * acc' = acc - wz[n] * rowsum(x), so no row sums are needed; s_n
     * is chosen per channel so that w' stays in [-128, 127]. Not with
     * weight_zero (IW_EINVAL); needs the channel-major kernel. */
    const int8_t *weight_sign;
} iw_gemm_desc;

/* tcgen05 (sm_100a) int8 GEMM with the epilogue described by *d. */
int iw_gemm_i8(const iw_gemm_desc *d, void *stream);

/* Per-channel GeLU lookup table for iw_gemm_desc.gelu_table:
 * table[n][x+128] = GELU_int of x in [-128,127] with channel n's parameters
 * (gelu_scalar.cpp:10-181; counts 1 or N as in iw_gelu). table is [N,256]. */
int iw_gelu_table(const uint8_t *lut, const uint8_t *luti_multiplier, const int8_t *luti_shift,
                  const uint8_t *luto_multiplier, const int8_t *luto_shift, int64_t luti_count, int64_t luto_count,
                  int64_t N, int8_t *table, void *stream);

/* Rearranges a [N][256] GeLU table into tiled [ceil(N/128)][32768] bytes
 * (16-byte aligned) for iw_gemm_desc.gelu_table_tiled: per 128 channels,
 * byte q*8192 + t*32 + l holds entry t of channel 32q + l (zero past N). */
int iw_gelu_table_tiled(const int8_t *table, int64_t N, int8_t *tiled, void *stream);

typedef struct iw_attn_desc {
    /* element (b,t,h,d) of Q is q[b*q_bs + t*ldq + h*q_hs + d], same for
     * K, V and the output y; head_dim is 64 */
    const int8_t *q; int64_t ldq, q_bs, q_hs;
    const int8_t *k; int64_t ldk, k_bs, k_hs;
    const int8_t *v; int64_t ldv, v_bs, v_hs;
    int8_t *y; int64_t ldy, y_bs, y_hs;
    int64_t B, H, Tq, Tk;
    const int32_t *Tk_dev;    /* optional: key count read on the device       */
    int64_t Tk_cap;           /* upper bound of *Tk_dev                        */
    int mask_mode;            /* 0 none, 1 causal, 2 explicit [Tq,Tk]          */
    const uint8_t *mask;
    uint8_t qk_multiplier; int8_t qk_shift; int32_t frac_bits;
    uint8_t av_multiplier; int8_t av_shift; int32_t rsqrt_offset;
    /* tensor-core path for unmasked self-attention with Tq == Tk and
     * contiguous batches: the shift-exp table of iw_shift_exp_table for this
     * frac_bits, and a V^T buffer [B*H*64, vt_ld] (vt_ld >= Tk, multiple of
     * 16) the call fills. NULL selects the CUDA-core kernel. */
    const uint8_t *exp_table;
    int8_t *vt;
    int64_t vt_ld;
    /* 1: vt already holds V^T (written by the projection GEMM's vt_out), so
     * the call does not transpose V */
    int vt_ready;
    /* optional: the sum of each int8 output row (b, q) is ADDED to
     * row_sum_out[b*Tq + q] (zero it first) -- the zero-point row sums the
     * output projection needs */
    int32_t *row_sum_out;
} iw_attn_desc;

int iw_attention_ex(const iw_attn_desc *d, void *stream);

/* Shift-exp table (attention_scalar.cpp:388-560 as a function of the int16
 * difference to rowmax+1) for the tensor-core attention; table needs 32772
 * bytes (16-byte aligned for the kernel's vector copy into shared memory),
 * frac_bits in [1, 30]. The whole table (at most 32770 entries, frac_bits >=
 * 15) fits the kernel's shared memory. Synchronises `stream`. */
int iw_shift_exp_table(int32_t frac_bits, uint8_t *table, void *stream);

/* LayerNorm32 over rows with strides; optionally writes the row sums of the
 * int8 output (rowsum_out) and zeroes rowsum_zero[rows] for a later
 * accumulating epilogue. */
int iw_layernorm32_ex(const int16_t *x, int64_t ldx, const int8_t *weight, const int32_t *bias,
                      uint8_t ln_multiplier, int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y,
                      int64_t ldy, int64_t rows, int64_t d, int32_t *rowsum_out, int32_t *rowsum_zero, void *stream);

/* iw_layernorm32_ex for LayerNorm64 (no synchronisation: a variance that
 * does not fit INT32 sets bit 1 of the iw_device_status word). */
int iw_layernorm64_ex(const int16_t *x, int64_t ldx, const int8_t *weight, const int32_t *bias,
                      uint8_t ln_multiplier, int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y,
                      int64_t ldy, int64_t rows, int64_t d, int32_t *rowsum_out, int32_t *rowsum_zero, void *stream);

/* Channel-first x [B][C][T] -> channels-last out [B][T+front+back][C] with
 * `front` zero rows before and `back` zero rows after each batch element:
 * the padded input of a convolution run as a windowed GEMM
 * (iw_gemm_desc.x_window_rows). B <= 65535. */
int iw_channels_last_pad(const int8_t *x, int64_t B, int64_t C, int64_t T, int64_t front, int64_t back, int8_t *out,
                         void *stream);
/* Zero `count` rows of `bytes` bytes, `pitch` bytes apart (the padding rows
 * of a windowed GEMM operand). */
int iw_zero_rows(void *p, int64_t count, int64_t bytes, int64_t pitch, void *stream);

/* im2col of the conv stem: row (b,t), column cin*K+k = x[b,cin,t*stride-pad+k]
 * (channels_last: x[b,t',cin]), zero outside; out row stride ldo >= Cin*K. */
int iw_im2col(const int8_t *x, int8_t *out, int64_t B, int64_t Cin, int64_t Tin, int64_t K, int64_t stride,
              int64_t pad, int64_t Tout, int64_t ldo, int channels_last, void *stream);

/* Embedding gather + add_requant15 with the position offset read from the
 * device (*offset_dev) when offset_dev != NULL. */
int iw_embed_add_requant15_dev(const int8_t *table, const int64_t *tokens, const int8_t *pe,
                               const int32_t *offset_dev, int64_t offset, const uint16_t *multiplier,
                               const int8_t *shift, int16_t *y, int64_t B, int64_t T, int64_t C,
                               int64_t multiplier_count, int64_t shift_count, void *stream);

/* Write T positions of K and V (columns k_col.., v_col.. of the rows of
 * src [B*T, lds]) into head-major caches [B,H,Tcap,64] at position
 * *pos_dev (or pos). Replaces the torch.cat KV hooks of
 * Whisper_int.install_kv_cache_hooks (model_int.py:1587-1618). */
int iw_kv_append(const int8_t *src, int64_t lds, int64_t k_col, int64_t v_col, int8_t *k_cache, int8_t *v_cache,
                 int64_t B, int64_t H, int64_t T, int64_t Tcap, int64_t pos, const int32_t *pos_dev, void *stream);

typedef struct iw_greedy_desc {
    const int8_t *logits; int64_t ld; int64_t V;
    float alpha;
    const uint32_t *suppress_bits; const int32_t *blank; int64_t n_blank;
    int64_t eot, timestamp_begin, no_timestamps, max_initial_timestamp_index;
    int32_t *state;           /* [B,4] n_sampled, last, penultimate, last timestamp */
    int64_t *tokens; int64_t ld_tok;
    int32_t *step_dev;        /* column of the next token in tokens */
    int64_t *next;            /* [B] */
} iw_greedy_desc;

/* One greedy decoding step on the device: SuppressBlank, SuppressTokens,
 * ApplyTimestampRules (decoding.py:426-510) and GreedyDecoder.update
 * (decoding.py:280-296). logits rows hold the int8 logits q of V tokens
 * at stride ld >= V; the float logit is q / alpha with alpha > 0
 * (IW_EINVAL otherwise). */
int iw_greedy_step(const iw_greedy_desc *d, int64_t B, void *stream);

/* log_mel_spectrogram (i_whisper/audio.py:216-265) followed by the input
 * quantisation of AudioEncoder_int.forward (model_int.py:1265-1267) for B
 * windows of float32 16 kHz audio [B, n_samples] (row stride lda floats,
 * n_samples > 256): out [B, n_mels, n_samples/160] int8 =
 * clamp(round((max(lg, max_window(lg) - 8)/4 + 1) * input_alpha), +-127)
 * with lg = log10(max(filters @ |STFT|^2, 1e-10)), STFT n_fft 512, hop 160,
 * periodic Hann window, reflect padding, last frame dropped. filters is the
 * [n_mels, 257] float32 mel filterbank on the device (n_mels <= 128). The
 * max is taken per window. Float32 arithmetic: results agree with the
 * reference within one INT8 unit, not bit for bit. */
int iw_log_mel_int8(const float *audio, int64_t B, int64_t n_samples, int64_t lda, const float *filters,
                    int64_t n_mels, float input_alpha, int8_t *out, void *stream);

/* *p += v on the device (advances device-side decode counters). */
int iw_add_i32(int32_t *p, int32_t v, void *stream);

/* ------------------------------------------------------------------------
 * Allocation-free Linear8. This entry point has no counterpart in the
 * reference: it exists for callers that cannot allocate device memory while
 * they run -- work captured into a CUDA graph whose memory pool they do not
 * own, servers that plan all device memory up front and forbid allocator
 * traffic on the request path, or hosts that only hand over raw pointers
 * from another runtime. It computes exactly what iw_linear8 computes, but the
 * row sums of x needed by the weight zero points live in one fixed device
 * array of IW_NOALLOC_MAX_ROWS int32 (256 KiB) that every GPU loading this
 * library keeps until the process exits, instead of a scratch allocation.
 *   - M must not exceed IW_NOALLOC_MAX_ROWS; K must be a multiple of 16 and
 *     x, weight 16-byte aligned (no padding copy is made); otherwise the call
 *     returns IW_EINVAL with a message and launches nothing.
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *   - All calls share the array and it keeps the last call's contents: calls
 *     whose executions overlap on the GPU race, so order them on one stream.
 *   - No cudaMalloc, cudaFree or other allocating routine is called.
 * ---------------------------------------------------------------------- */
#define IW_NOALLOC_MAX_ROWS 65536
int iw_linear8_noalloc(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                       const uint32_t *multiplier, const int8_t *shift, int8_t *y, int64_t M, int64_t K, int64_t N,
                       void *stream);

#ifdef __cplusplus
}
#endif

#endif /* IWHISPER_B200_H */
