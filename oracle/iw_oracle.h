/*
 * iw_oracle.h -- CPU restatement of the I-Whisper integer hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path
 * is compared against; it is never linked into, loaded by, or called from
 * the product library (i_whisper_b200). Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load it.
 *
 * Every function restates the integer semantics of one reference kernel
 * (vcsd-lab/I-Whisper, i_whisper/kernels/csrc/...) in plain C. Citations are
 * given beside each definition in iw_oracle.c. Pointers are host pointers to
 * contiguous row-major arrays. Functions that can fail return 0 on success
 * and a negative code otherwise.
 */
#ifndef IW_ORACLE_H
#define IW_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fixed-point primitives (common/fixedpoint.h) */
int32_t iwo_mulh(int32_t x, uint32_t multiplier);
int32_t iwo_rounding_rshift(int32_t x, uint32_t shift);
int32_t iwo_fisr(int32_t x, uint32_t offset);
void iwo_fisr_vec(const int32_t *x, int32_t *y, int64_t n, uint32_t offset);
void iwo_set_threads(int n);

/* Linear8 / Linear32 (linear8_scalar.cpp, linear32_scalar.cpp) */
void iwo_linear8_accum(const int8_t *x, const int8_t *w, const int32_t *bias,
                       const int8_t *wz, int32_t *y, int64_t M, int64_t K,
                       int64_t N);
void iwo_linear8(const int8_t *x, const int8_t *w, const int32_t *bias,
                 const int8_t *wz, const uint32_t *mult, const int8_t *shift,
                 int8_t *y, int64_t M, int64_t K, int64_t N);
void iwo_linear8_requant(const int32_t *acc, const uint32_t *mult,
                         const int8_t *shift, int32_t *y, int64_t M, int64_t N);
void iwo_linear32(const int8_t *x, const int8_t *w, const int32_t *bias,
                  const int8_t *wz, const uint32_t *mult, const int8_t *shift,
                  int32_t *y, int64_t M, int64_t K, int64_t N);
void iwo_linear32_requant(const int32_t *acc, const uint32_t *mult,
                          const int8_t *shift, int32_t *y, int64_t M, int64_t N);

/* Residual15 (residual15_scalar.cpp) */
void iwo_residual15(const int32_t *branch, const int16_t *residual,
                    uint16_t mult, int16_t *y, int64_t n);

/* LayerNorm32 (layernorm_scalar.cpp) ; returns -1 on unsupported width */
int iwo_layernorm32(const int16_t *x, const int8_t *gamma, const int32_t *beta,
                    uint8_t ln_mult, int8_t ln_shift, uint32_t out_mult,
                    int8_t out_shift, uint32_t rsqrt_offset, int8_t *y,
                    int64_t rows, int64_t d);
int iwo_layernorm32_stats(const int16_t *x, int32_t *mean, int32_t *var,
                          int32_t *renorm_shift, int64_t rows, int64_t d);

/* LayerNorm64 research variant (layernorm_scalar.cpp:230-297, 626-825):
 * returns -1 on an unsupported width, -2 when a row's variance does not fit
 * INT32 (the reference throws std::overflow_error). */
int iwo_layernorm64(const int16_t *x, const int8_t *gamma, const int32_t *beta,
                    uint8_t ln_mult, int8_t ln_shift, uint32_t out_mult,
                    int8_t out_shift, uint32_t rsqrt_offset,
                    int32_t additional_offset, int8_t *y, int64_t rows,
                    int64_t d);
int iwo_layernorm64_stats(const int16_t *x, int32_t *mean, int64_t *var,
                          int64_t rows, int64_t d);

/* GeLU (gelu_scalar.cpp) */
void iwo_gelu(const int8_t *x, const uint8_t *lut, const uint8_t *mi,
              const int8_t *si, const uint8_t *mo, const int8_t *so,
              int8_t *y, int64_t numel, int64_t channels, int64_t n_in,
              int64_t n_out);

/* Attention (attention_scalar.cpp) */
void iwo_qk(const int8_t *q, const int8_t *k, int32_t *y, int64_t B,
            int64_t H, int64_t Tq, int64_t Tk, int64_t D);
void iwo_qk_requant_rowmax(const int8_t *q, const int8_t *k,
                           const uint8_t *mask, int16_t *qk, int16_t *rmax1,
                           int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                           int64_t D, uint8_t mult, int32_t shift);
void iwo_shift_exp(const int16_t *x, const int16_t *rmax1, const uint8_t *mask,
                   uint8_t *p, int32_t *rowsum, int64_t B, int64_t H,
                   int64_t Tq, int64_t Tk, int32_t frac_bits);
void iwo_pv(const uint8_t *p, const int8_t *vt, int32_t *y, int64_t B,
            int64_t H, int64_t Tq, int64_t Tk, int64_t D);
int iwo_pv_norm_requant(const uint8_t *p, const int8_t *vt,
                        const int32_t *rowsum, uint8_t av_mult,
                        int8_t av_shift, uint32_t rsqrt_offset, int8_t *y,
                        int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                        int64_t D);

/* Conv1d (conv1d_scalar.cpp) */
void iwo_conv1d_accum(const int8_t *x, const int8_t *w, const int32_t *bias,
                      int32_t *y, int64_t B, int64_t Cin, int64_t Tin,
                      int64_t Cout, int64_t K, int64_t stride, int64_t pad);
void iwo_conv1d(const int8_t *x, const int8_t *w, const int32_t *bias,
                uint32_t mult, int8_t shift, int8_t *y, int64_t B,
                int64_t Cin, int64_t Tin, int64_t Cout, int64_t K,
                int64_t stride, int64_t pad);

/* Add + requant to INT15 (add_requant15_scalar.cpp) */
void iwo_add_requant15(const int8_t *x, const int8_t *addend,
                       const uint16_t *mult, const int8_t *shift, int16_t *y,
                       int64_t B, int64_t T, int64_t C, int64_t n_mult,
                       int64_t n_shift);

/* Classifier (classifier_scalar.cpp) */
void iwo_classifier_accum(const int8_t *x, const int8_t *w, int32_t *y,
                          int64_t M, int64_t K, int64_t N);
void iwo_classifier(const int8_t *x, const int8_t *w, uint32_t mult,
                    int8_t shift, int8_t *y, int64_t M, int64_t K, int64_t N);

#ifdef __cplusplus
}
#endif

#endif
