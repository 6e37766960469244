// ref_shim.cpp -- C-ABI shim over the reference's own scalar C++ kernels.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile (target `ref`) together
// with the unmodified reference sources
// i_whisper/kernels/csrc/*/*_scalar.cpp of vcsd-lab/I-Whisper, read in
// place from the reference checkout; the result goes to oracle/_ref/ and is
// never committed. It lets the tests check the C restatement
// (iw_oracle.c) against the reference itself, and gives bench.py's
// `--impl reference` arm the reference's own CPU kernels. Each iwr_* symbol
// has the same signature as the iwo_* function of the same name.
#include <cstdint>
#include <stdexcept>

#include "linear8/linear8.h"
#include "linear32/linear32.h"
#include "residual15/residual15.h"
#include "layernorm/layernorm.h"
#include "gelu/gelu.h"
#include "attention/attention.h"
#include "conv1d/conv1d.h"
#include "add_requant15/add_requant15.h"
#include "classifier/classifier.h"

using namespace iwhisper;

extern "C" {

void iwr_linear8_accum(const int8_t *x, const int8_t *w, const int32_t *bias,
                       const int8_t *wz, int32_t *y, int64_t M, int64_t K, int64_t N) {
    linear8_accum_scalar(x, w, bias, wz, y, M, K, N, bias != nullptr, wz != nullptr);
}
void iwr_linear8(const int8_t *x, const int8_t *w, const int32_t *bias, const int8_t *wz,
                 const uint32_t *m, const int8_t *s, int8_t *y, int64_t M, int64_t K, int64_t N) {
    linear8_scalar(x, w, bias, wz, m, s, y, M, K, N, bias != nullptr, wz != nullptr);
}
void iwr_linear32(const int8_t *x, const int8_t *w, const int32_t *bias, const int8_t *wz,
                  const uint32_t *m, const int8_t *s, int32_t *y, int64_t M, int64_t K, int64_t N) {
    linear32_scalar(x, w, bias, wz, m, s, y, M, K, N, bias != nullptr, wz != nullptr);
}
void iwr_residual15(const int32_t *br, const int16_t *r, uint16_t m, int16_t *y, int64_t n) {
    residual15_scalar(br, r, m, y, n);
}
int iwr_layernorm32(const int16_t *x, const int8_t *g, const int32_t *b, uint8_t lm, int8_t ls,
                    uint32_t om, int8_t os, uint32_t off, int8_t *y, int64_t rows, int64_t d) {
    try {
        layernorm32_scalar(x, g, b, lm, ls, om, os, off, y, rows, d, b != nullptr);
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}
int iwr_layernorm32_stats(const int16_t *x, int32_t *mean, int32_t *var, int32_t *rs,
                          int64_t rows, int64_t d) {
    try {
        layernorm32_stats_scalar(x, mean, var, rs, rows, d);
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}
int iwr_layernorm64(const int16_t *x, const int8_t *g, const int32_t *b, uint8_t lm, int8_t ls,
                    uint32_t om, int8_t os, uint32_t off, int32_t add, int8_t *y, int64_t rows, int64_t d) {
    try {
        layernorm64_scalar(x, g, b, lm, ls, om, os, off, add, y, rows, d, b != nullptr);
    } catch (const std::overflow_error &) {
        return -2;
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}
int iwr_layernorm64_stats(const int16_t *x, int32_t *mean, int64_t *var, int64_t rows, int64_t d) {
    try {
        layernorm64_stats_scalar(x, mean, var, rows, d);
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}
void iwr_fisr_vec(const int32_t *x, int32_t *y, int64_t n, uint32_t off) {
    layernorm32_rsqrt_scalar(x, y, n, off);
}
void iwr_gelu(const int8_t *x, const uint8_t *lut, const uint8_t *mi, const int8_t *si,
              const uint8_t *mo, const int8_t *so, int8_t *y, int64_t numel, int64_t ch,
              int64_t ni, int64_t no) {
    gelu_scalar(x, lut, mi, si, mo, so, y, numel, ch, ni, no);
}
void iwr_qk(const int8_t *q, const int8_t *k, int32_t *y, int64_t B, int64_t H, int64_t Tq,
            int64_t Tk, int64_t D) {
    qk_scalar(q, k, y, B, H, Tq, Tk, D);
}
void iwr_qk_requant_rowmax(const int8_t *q, const int8_t *k, const uint8_t *mask, int16_t *qk,
                           int16_t *rmax1, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                           int64_t D, uint8_t m, int32_t s) {
    qk_requant_rowmax_scalar(q, k, reinterpret_cast<const bool *>(mask), qk, rmax1, B, H, Tq,
                             Tk, D, m, s, mask != nullptr);
}
void iwr_shift_exp(const int16_t *x, const int16_t *rmax1, const uint8_t *mask, uint8_t *p,
                   int32_t *rowsum, int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t fb) {
    shift_exp_scalar(x, rmax1, reinterpret_cast<const bool *>(mask), p, rowsum, B, H, Tq, Tk,
                     fb, mask != nullptr);
}
void iwr_pv(const uint8_t *p, const int8_t *vt, int32_t *y, int64_t B, int64_t H, int64_t Tq,
            int64_t Tk, int64_t D) {
    pv_scalar(p, vt, y, B, H, Tq, Tk, D);
}
int iwr_pv_norm_requant(const uint8_t *p, const int8_t *vt, const int32_t *rowsum, uint8_t am,
                        int8_t as, uint32_t off, int8_t *y, int64_t B, int64_t H, int64_t Tq,
                        int64_t Tk, int64_t D) {
    try {
        pv_norm_requant_scalar(p, vt, rowsum, am, as, off, y, B, H, Tq, Tk, D);
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}
void iwr_conv1d_accum(const int8_t *x, const int8_t *w, const int32_t *bias, int32_t *y,
                      int64_t B, int64_t Cin, int64_t Tin, int64_t Cout, int64_t K,
                      int64_t stride, int64_t pad) {
    conv1d_accum_scalar(x, w, bias, y, B, Cin, Tin, Cout, K, stride, pad, bias != nullptr);
}
void iwr_conv1d(const int8_t *x, const int8_t *w, const int32_t *bias, uint32_t m, int8_t s,
                int8_t *y, int64_t B, int64_t Cin, int64_t Tin, int64_t Cout, int64_t K,
                int64_t stride, int64_t pad) {
    conv1d_scalar(x, w, bias, m, s, y, B, Cin, Tin, Cout, K, stride, pad, bias != nullptr);
}
void iwr_add_requant15(const int8_t *x, const int8_t *a, const uint16_t *m, const int8_t *s,
                       int16_t *y, int64_t B, int64_t T, int64_t C, int64_t nm, int64_t ns) {
    add_requant15_scalar(x, a, m, s, y, B, T, C, nm, ns);
}
void iwr_classifier_accum(const int8_t *x, const int8_t *w, int32_t *y, int64_t M, int64_t K,
                          int64_t N) {
    classifier_accum_scalar(x, w, y, M, K, N);
}
void iwr_classifier(const int8_t *x, const int8_t *w, uint32_t m, int8_t s, int8_t *y,
                    int64_t M, int64_t K, int64_t N) {
    classifier_scalar(x, w, m, s, y, M, K, N);
}

}  // extern "C"
