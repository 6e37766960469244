// capi.cu -- extern "C" entry points (include/iwhisper_b200.h).
//
// Argument checking mirrors the TORCH_CHECKs of the reference torch
// wrappers (i_whisper/kernels/csrc/*/*_torch.cpp); every failure returns a
// negative code and records a message for iw_last_error().
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/iwhisper_b200.h"
#include "gemm_i8.cuh"
#include "iw_common.cuh"
#include "kernels.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return IW_OK;
    return fail(IW_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

bool ln_width_ok(int64_t d) { return d == 384 || d == 512 || d == 768 || d == 1024 || d == 1280; }

// Stream-ordered scratch buffer, released on the same stream.
struct Scratch {
    void *p = nullptr;
    cudaStream_t st;
    explicit Scratch(cudaStream_t s) : st(s) {}
    cudaError_t alloc(size_t bytes) { return cudaMallocAsync(&p, bytes ? bytes : 16, st); }
    ~Scratch() {
        if (p) cudaFreeAsync(p, st);
    }
};

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Shared body of Linear8 / Linear32 / accum / fused residual: pads K to a
// multiple of 16 when needed (TMA row-stride rule), computes the row sums
// of x when a zero point is given, then runs the tcgen05 GEMM.
int run_linear(const int8_t *x, const int8_t *w, const int32_t *bias, const int8_t *wz, const uint32_t *mult,
               const int8_t *shift, void *y, int64_t M, int64_t K, int64_t N, iw::EpiMode mode, const int16_t *res,
               uint16_t res_mult, cudaStream_t st, const char *name) {
    if (M < 0 || N <= 0) return fail(IW_EINVAL, "%s: invalid shape M=%lld N=%lld", name, (long long)M, (long long)N);
    if (K <= 0) return fail(IW_EINVAL, "%s: x.size(-1) must be greater than 0", name);
    if (M == 0) return IW_OK;
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(IW_EINVAL, "%s: dimension too large", name);
    Scratch xs(st), ws(st), rs(st);
    const int8_t *xg = x, *wg = w;
    int64_t Kp = K;
    if (K % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) {
        Kp = round_up(K, 16);
        if (int r = cuda_check(xs.alloc((size_t)M * Kp), name)) return r;
        if (int r = cuda_check(ws.alloc((size_t)N * Kp), name)) return r;
        if (int r = cuda_check(iw::pad_rows(x, M, K, (int8_t *)xs.p, Kp, st), name)) return r;
        if (int r = cuda_check(iw::pad_rows(w, N, K, (int8_t *)ws.p, Kp, st), name)) return r;
        xg = (const int8_t *)xs.p;
        wg = (const int8_t *)ws.p;
    }
    iw::EpiParams p;
    p.out = y;
    p.ldo = N;
    p.bias = bias;
    p.wz = wz;
    p.mult = mult;
    p.shift = shift;
    p.per_channel = 1;
    if (wz) {
        if (int r = cuda_check(rs.alloc((size_t)M * 4), name)) return r;
        if (int r = cuda_check(iw::rowsum_i8(xg, Kp, (int)M, (int)Kp, (int32_t *)rs.p, st), name)) return r;
        p.rowsum = (const int32_t *)rs.p;
    }
    if (mode == iw::EPI_L32_RES) {
        p.res = res;
        p.ldr = N;
        p.res_mult = res_mult;
    }
    iw::GemmShape g{xg, Kp, wg, Kp, (int)M, (int)N, (int)Kp};
    return cuda_check(iw::gemm_i8_launch(g, mode, p, st), name);
}

}  // namespace

extern "C" {

const char *iw_last_error(void) { return g_err.c_str(); }

int iw_abi_version(void) { return 1; }

int iw_set_wait_timeout_ns(uint64_t ns) {
    if (ns == 0) return fail(IW_EINVAL, "iw_set_wait_timeout_ns: the bound must be positive");
    const unsigned long long v = ns;
    return cuda_check(cudaMemcpyToSymbol(iw::g_wait_timeout_ns, &v, sizeof(v)), "iw_set_wait_timeout_ns");
}

int iw_selftest_wait_timeout(int32_t *gave_up, void *stream) {
    if (!gave_up) return fail(IW_EINVAL, "iw_selftest_wait_timeout: null result pointer");
    return cuda_check(iw::selftest_wait(gave_up, S(stream)), "iw_selftest_wait_timeout");
}

int iw_device_status(uint32_t *status, int clear) {
    if (int r = cuda_check(cudaDeviceSynchronize(), "iw_device_status")) return r;
    uint32_t v = 0;
    if (int r = cuda_check(cudaMemcpyFromSymbol(&v, iw::g_device_status, sizeof(v)), "iw_device_status")) return r;
    if (status) *status = v;
    if (clear) {
        const uint32_t z = 0;
        if (int r = cuda_check(cudaMemcpyToSymbol(iw::g_device_status, &z, sizeof(z)), "iw_device_status")) return r;
    }
    return IW_OK;
}

int iw_linear8(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
               const uint32_t *multiplier, const int8_t *shift, int8_t *y, int64_t M, int64_t K, int64_t N,
               void *stream) {
    return run_linear(x, weight, bias, weight_zero, multiplier, shift, y, M, K, N, iw::EPI_L8, nullptr, 0, S(stream),
                      "iw_linear8");
}

int iw_linear8_accum(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                     int32_t *y, int64_t M, int64_t K, int64_t N, void *stream) {
    return run_linear(x, weight, bias, weight_zero, nullptr, nullptr, y, M, K, N, iw::EPI_ACC32, nullptr, 0,
                      S(stream), "iw_linear8_accum");
}

int iw_linear8_requant(const int32_t *acc, const uint32_t *multiplier, const int8_t *shift, int32_t *y, int64_t M,
                       int64_t N, void *stream) {
    if (M < 0 || N <= 0) return fail(IW_EINVAL, "iw_linear8_requant: invalid shape M=%lld N=%lld", (long long)M,
                                     (long long)N);
    if (!multiplier || !shift) return fail(IW_EINVAL, "iw_linear8_requant: multiplier and shift are required");
    return cuda_check(iw::requant_rows(acc, multiplier, shift, 0u, y, M * N, N, S(stream)), "iw_linear8_requant");
}

int iw_rounding_rshift(const int32_t *x, uint32_t shift, int32_t *y, int64_t numel, void *stream) {
    if (numel < 0) return fail(IW_EINVAL, "iw_rounding_rshift: invalid numel");
    return cuda_check(iw::requant_rows(x, nullptr, nullptr, shift, y, numel, 1, S(stream)), "iw_rounding_rshift");
}

int iw_linear32(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                const uint32_t *multiplier, const int8_t *shift, int32_t *y, int64_t M, int64_t K, int64_t N,
                void *stream) {
    return run_linear(x, weight, bias, weight_zero, multiplier, shift, y, M, K, N, iw::EPI_L32, nullptr, 0, S(stream),
                      "iw_linear32");
}

int iw_linear32_residual15(const int8_t *x, const int8_t *weight, const int32_t *bias, const int8_t *weight_zero,
                           const uint32_t *multiplier, const int8_t *shift, const int16_t *residual,
                           uint16_t residual_multiplier, int16_t *y, int64_t M, int64_t K, int64_t N, void *stream) {
    if (!residual) return fail(IW_EINVAL, "iw_linear32_residual15: residual is required");
    return run_linear(x, weight, bias, weight_zero, multiplier, shift, y, M, K, N, iw::EPI_L32_RES, residual,
                      residual_multiplier, S(stream), "iw_linear32_residual15");
}

int iw_residual15(const int32_t *branch, const int16_t *residual, uint16_t multiplier, int16_t *y, int64_t numel,
                  void *stream) {
    if (numel < 0) return fail(IW_EINVAL, "iw_residual15: invalid numel");
    return cuda_check(iw::residual15(branch, residual, multiplier, y, numel, S(stream)), "iw_residual15");
}

int iw_layernorm32(const int16_t *x, const int8_t *weight, const int32_t *bias, uint8_t ln_multiplier,
                   int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y, int64_t rows, int64_t d,
                   void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    if (rows < 0 || rows > INT32_MAX) return fail(IW_EINVAL, "iw_layernorm32: invalid row count");
    iw::LnParams p{(int32_t)ln_multiplier, (int32_t)ln_shift, out_multiplier, (uint32_t)(int32_t)out_shift, 13u};
    return cuda_check(iw::layernorm32(x, d, weight, bias, p, y, d, (int)rows, (int)d, nullptr, nullptr, S(stream)),
                      "iw_layernorm32");
}

int iw_layernorm32_stats(const int16_t *x, int32_t *mean, int32_t *variance, int32_t *renorm_shift, int64_t rows,
                         int64_t d, void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    return cuda_check(iw::layernorm32_stats(x, (int)rows, (int)d, mean, variance, renorm_shift, S(stream)),
                      "iw_layernorm32_stats");
}

__global__ void any_negative_kernel(const int32_t *x, int64_t n, int *flag) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        if (x[i] < 0) atomicExch(flag, 1);
}

static int check_nonnegative(const int32_t *x, int64_t n, cudaStream_t st, const char *name, const char *msg,
                             int status = IW_EVALUE) {
    if (n <= 0) return IW_OK;
    Scratch f(st);
    if (int r = cuda_check(f.alloc(sizeof(int)), name)) return r;
    if (int r = cuda_check(cudaMemsetAsync(f.p, 0, sizeof(int), st), name)) return r;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 1024) blocks = 1024;
    any_negative_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, (int *)f.p);
    int h = 0;
    if (int r = cuda_check(cudaMemcpyAsync(&h, f.p, sizeof(int), cudaMemcpyDeviceToHost, st), name)) return r;
    if (int r = cuda_check(cudaStreamSynchronize(st), name)) return r;
    if (h) return fail(status, "%s", msg);
    return IW_OK;
}

int iw_layernorm32_rsqrt(const int32_t *variance, int32_t *invstd, int64_t numel, void *stream) {
    // a TORCH_CHECK in the reference (layernorm_torch.cpp:120-122): RuntimeError, not ValueError
    if (int r = check_nonnegative(variance, numel, S(stream), "iw_layernorm32_rsqrt", "input must be non-negative",
                                  IW_EINVAL))
        return r;
    return cuda_check(iw::fisr_vec(variance, invstd, numel, 13u, S(stream)), "iw_layernorm32_rsqrt");
}

int iw_gelu(const int8_t *x, const uint8_t *lut, const uint8_t *luti_multiplier, const int8_t *luti_shift,
            const uint8_t *luto_multiplier, const int8_t *luto_shift, int8_t *y, int64_t numel, int64_t channels,
            int64_t luti_count, int64_t luto_count, void *stream) {
    if (channels <= 0 && numel > 0) return fail(IW_EINVAL, "iw_gelu: input must have at least one dimension");
    if (!(luti_count == 1 || luti_count == channels))
        return fail(IW_EINVAL, "luti parameters must be scalar or match input.size(-1)");
    if (!(luto_count == 1 || luto_count == channels))
        return fail(IW_EINVAL, "luto parameters must be scalar or match input.size(-1)");
    iw::GeluParams g{lut, luti_multiplier, luti_shift, luto_multiplier, luto_shift, (int)luti_count, (int)luto_count};
    return cuda_check(iw::gelu(x, y, numel, (int)channels, g, S(stream)), "iw_gelu");
}

int iw_qk_requant_rowmax(const int8_t *q, const int8_t *k, const uint8_t *mask, uint8_t multiplier, int8_t shift,
                         int16_t *qk, int16_t *row_max_plus1, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                         int64_t D, void *stream) {
    if (B < 0 || H < 0 || Tq < 0 || Tk < 0 || D < 0) return fail(IW_EINVAL, "iw_qk_requant_rowmax: invalid shape");
    return cuda_check(iw::qk_requant_rowmax(q, k, mask, qk, row_max_plus1, (int)B, (int)H, (int)Tq, (int)Tk, (int)D,
                                            multiplier, (int32_t)shift, S(stream)),
                      "iw_qk_requant_rowmax");
}

int iw_shift_exp(const int16_t *x, const int16_t *row_max_plus1, const uint8_t *mask, int32_t frac_bits, uint8_t *p,
                 int32_t *row_sum, int64_t B, int64_t H, int64_t Tq, int64_t Tk, void *stream) {
    if (!(frac_bits > 0 && frac_bits < 14)) return fail(IW_EINVAL, "frac_bits must be in [1, 14)");
    return cuda_check(iw::shift_exp(x, row_max_plus1, mask, p, row_sum, (int)B, (int)H, (int)Tq, (int)Tk, frac_bits,
                                    S(stream)),
                      "iw_shift_exp");
}

int iw_pv_norm_requant(const uint8_t *p, const int8_t *v, const int32_t *row_sum, uint8_t av_multiplier,
                       int8_t av_shift, int64_t rsqrt_offset, int8_t *y, int64_t B, int64_t H, int64_t Tq,
                       int64_t Tk, int64_t D, void *stream) {
    if (!(rsqrt_offset >= 0 && rsqrt_offset <= 29)) return fail(IW_EINVAL, "rsqrt_offset must be in [0,29]");
    cudaStream_t st = S(stream);
    if (int r = check_nonnegative(row_sum, B * H * Tq, st, "iw_pv_norm_requant", "row_sum must be non-negative"))
        return r;
    Scratch bad(st);
    if (int r = cuda_check(bad.alloc(sizeof(int)), "iw_pv_norm_requant")) return r;
    if (int r = cuda_check(cudaMemsetAsync(bad.p, 0, sizeof(int), st), "iw_pv_norm_requant")) return r;
    return cuda_check(iw::pv_norm_requant(p, v, row_sum, av_multiplier, av_shift, (uint32_t)rsqrt_offset, y, (int)B,
                                          (int)H, (int)Tq, (int)Tk, (int)D, (int *)bad.p, st),
                      "iw_pv_norm_requant");
}

// frac_bits of the fused attention entry points (the model's path). The
// reference's _C.shift_exp wrapper admits [1, 14) (attention_torch.cpp:305;
// iw_shift_exp keeps that check), but its own calibration writes 13-15 into
// checkpoints, which the reference model runs on its torch backend; the
// shift-exp arithmetic (1 << frac_bits in int32, attention_scalar.cpp:388-560)
// is defined up to 30.
static bool fused_frac_bits_ok(int32_t fb) { return fb >= 1 && fb <= 30; }

int iw_attention(const int8_t *q, int64_t ldq, int64_t q_bs, const int8_t *k, int64_t ldk, int64_t k_bs,
                 const int8_t *v, int64_t ldv, int64_t v_bs, int8_t *y, int64_t ldy, int64_t y_bs, int64_t B,
                 int64_t H, int64_t Tq, int64_t Tk, int mask_mode, const uint8_t *mask, uint8_t qk_multiplier,
                 int8_t qk_shift, int32_t frac_bits, uint8_t av_multiplier, int8_t av_shift, int64_t rsqrt_offset,
                 void *stream) {
    if (B < 0 || H < 0 || Tq < 0 || Tk < 0) return fail(IW_EINVAL, "iw_attention: invalid shape");
    if (Tq > Tk && mask_mode == 1) return fail(IW_EINVAL, "iw_attention: causal mask needs Tq <= Tk");
    if (mask_mode == 2 && !mask) return fail(IW_EINVAL, "iw_attention: mask_mode 2 needs a mask");
    if (!fused_frac_bits_ok(frac_bits)) return fail(IW_EINVAL, "frac_bits must be in [1, 30]");
    if (!(rsqrt_offset >= 0 && rsqrt_offset <= 29)) return fail(IW_EINVAL, "rsqrt_offset must be in [0,29]");
    if ((ldq | ldk | ldv | q_bs | k_bs | v_bs) & 15 ||
        (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
        return fail(IW_EINVAL, "iw_attention: Q/K/V rows must be 16-byte aligned");
    iw::AttnArgs a;
    a.q = q; a.ldq = ldq; a.q_bs = q_bs;
    a.k = k; a.ldk = ldk; a.k_bs = k_bs;
    a.v = v; a.ldv = ldv; a.v_bs = v_bs;
    a.out = y; a.ldo = ldy; a.o_bs = y_bs;
    a.Tq = (int)Tq; a.Tk = (int)Tk; a.Tk_dev = nullptr; a.Tk_cap = (int)Tk;
    a.mask_mode = mask_mode; a.mask = mask;
    a.qk_mult = qk_multiplier; a.qk_shift = qk_shift; a.frac_bits = frac_bits;
    a.av_mult = av_multiplier; a.av_shift = av_shift; a.rsqrt_offset = (uint32_t)rsqrt_offset;
    return cuda_check(iw::attention_cc(a, (int)B, (int)H, S(stream)), "iw_attention");
}

int iw_conv1d(const int8_t *x, const int8_t *weight, const int32_t *bias, uint32_t multiplier, int8_t shift,
              int64_t stride, int64_t padding, int8_t *y, int64_t B, int64_t Cin, int64_t Tin, int64_t Cout,
              int64_t K, void *stream) {
    if (stride <= 0) return fail(IW_EINVAL, "stride must be positive");
    if (padding < 0) return fail(IW_EINVAL, "padding must be non-negative");
    if (Cin <= 0) return fail(IW_EINVAL, "input channel count must be positive");
    if (Tin <= 0) return fail(IW_EINVAL, "input length must be positive");
    if (Cout <= 0) return fail(IW_EINVAL, "output channel count must be positive");
    if (K <= 0) return fail(IW_EINVAL, "kernel size must be positive");
    const int64_t num = Tin + 2 * padding - K;
    if (num < 0) return fail(IW_EINVAL, "invalid Conv1d geometry: output length would be non-positive");
    const int64_t Tout = num / stride + 1;
    if (B == 0) return IW_OK;
    cudaStream_t st = S(stream);
    const int64_t Kg = Cin * K, Kp = round_up(Kg, 16);
    const int64_t M = B * Tout;
    Scratch cols(st), ws(st);
    if (int r = cuda_check(cols.alloc((size_t)M * Kp), "iw_conv1d")) return r;
    if (int r = cuda_check(iw::im2col(x, (int8_t *)cols.p, (int)B, (int)Cin, (int)Tin, (int)K, (int)stride,
                                      (int)padding, (int)Tout, Kp, 0, st),
                           "iw_conv1d"))
        return r;
    const int8_t *wg = weight;
    if (Kp != Kg || (reinterpret_cast<uintptr_t>(weight) & 15)) {
        if (int r = cuda_check(ws.alloc((size_t)Cout * Kp), "iw_conv1d")) return r;
        if (int r = cuda_check(iw::pad_rows(weight, Cout, Kg, (int8_t *)ws.p, Kp, st), "iw_conv1d")) return r;
        wg = (const int8_t *)ws.p;
    }
    iw::EpiParams p;
    p.out = y;
    p.ldo = Cout;
    p.bias = bias;
    p.per_channel = 0;
    p.smult = multiplier;
    p.sshift = (uint32_t)(shift > 0 ? shift : 0);
    p.transpose_T = (int)Tout;
    iw::GemmShape g{(const int8_t *)cols.p, Kp, wg, Kp, (int)M, (int)Cout, (int)Kp};
    return cuda_check(iw::gemm_i8_launch(g, iw::EPI_L8, p, st), "iw_conv1d");
}

int iw_add_requant15(const int8_t *x, const int8_t *addend, const uint16_t *multiplier, const int8_t *shift,
                     int16_t *y, int64_t B, int64_t T, int64_t C, int64_t multiplier_count, int64_t shift_count,
                     void *stream) {
    if (!(multiplier_count == 1 || multiplier_count == C)) return fail(IW_EINVAL, "multiplier must contain 1 or C elements");
    if (!(shift_count == 1 || shift_count == C)) return fail(IW_EINVAL, "shift must contain 1 or C elements");
    return cuda_check(iw::add_requant15(x, nullptr, addend, multiplier, shift, y, (int)B, (int)T, (int)C,
                                        (int)multiplier_count, (int)shift_count, 0, nullptr, S(stream)),
                      "iw_add_requant15");
}

int iw_embed_add_requant15(const int8_t *table, const int64_t *tokens, const int8_t *pe, int64_t offset,
                           const uint16_t *multiplier, const int8_t *shift, int16_t *y, int64_t B, int64_t T,
                           int64_t C, int64_t multiplier_count, int64_t shift_count, void *stream) {
    if (!(multiplier_count == 1 || multiplier_count == C)) return fail(IW_EINVAL, "multiplier must contain 1 or C elements");
    if (!(shift_count == 1 || shift_count == C)) return fail(IW_EINVAL, "shift must contain 1 or C elements");
    if (offset < 0) return fail(IW_EINVAL, "iw_embed_add_requant15: negative offset");
    return cuda_check(iw::add_requant15(table, tokens, pe, multiplier, shift, y, (int)B, (int)T, (int)C,
                                        (int)multiplier_count, (int)shift_count, (int)offset, nullptr, S(stream)),
                      "iw_embed_add_requant15");
}

int iw_classifier(const int8_t *x, const int8_t *weight, uint32_t multiplier, int8_t shift, int8_t *y, int64_t M,
                  int64_t K, int64_t N, void *stream) {
    if (K <= 0) return fail(IW_EINVAL, "hidden size must be positive");
    if (N <= 0) return fail(IW_EINVAL, "vocabulary size must be positive");
    if (M == 0) return IW_OK;
    cudaStream_t st = S(stream);
    Scratch xs(st), ws(st);
    const int8_t *xg = x, *wg = weight;
    int64_t Kp = K;
    if (K % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(weight) & 15)) {
        Kp = round_up(K, 16);
        if (int r = cuda_check(xs.alloc((size_t)M * Kp), "iw_classifier")) return r;
        if (int r = cuda_check(ws.alloc((size_t)N * Kp), "iw_classifier")) return r;
        if (int r = cuda_check(iw::pad_rows(x, M, K, (int8_t *)xs.p, Kp, st), "iw_classifier")) return r;
        if (int r = cuda_check(iw::pad_rows(weight, N, K, (int8_t *)ws.p, Kp, st), "iw_classifier")) return r;
        xg = (const int8_t *)xs.p;
        wg = (const int8_t *)ws.p;
    }
    iw::EpiParams p;
    p.out = y;
    p.ldo = N;
    p.per_channel = 0;
    p.smult = multiplier;
    p.sshift = (uint32_t)(shift > 0 ? shift : 0);
    iw::GemmShape g{xg, Kp, wg, Kp, (int)M, (int)N, (int)Kp};
    return cuda_check(iw::gemm_i8_launch(g, iw::EPI_L8, p, st), "iw_classifier");
}

int iw_rowsum_i8(const int8_t *x, int64_t ldx, int64_t M, int64_t K, int32_t *y, void *stream) {
    return cuda_check(iw::rowsum_i8(x, ldx, (int)M, (int)K, y, S(stream)), "iw_rowsum_i8");
}

int iw_gemm_i8(const iw_gemm_desc *d, void *stream) {
    if (!d) return fail(IW_EINVAL, "iw_gemm_i8: null descriptor");
    if (d->M < 0 || d->N <= 0 || d->K <= 0 || d->M > INT32_MAX || d->N > INT32_MAX || d->K > INT32_MAX)
        return fail(IW_EINVAL, "iw_gemm_i8: invalid shape M=%lld N=%lld K=%lld", (long long)d->M, (long long)d->N,
                    (long long)d->K);
    if (d->M == 0) return IW_OK;
    if (d->K % 16 || d->ldx % 16 || d->ldw % 16)
        return fail(IW_EINVAL, "iw_gemm_i8: K and the row strides must be multiples of 16");
    if (d->weight_zero && !d->x_rowsum) return fail(IW_EINVAL, "iw_gemm_i8: weight_zero needs x_rowsum");
    if (d->weight_sign && d->weight_zero)
        return fail(IW_EINVAL, "iw_gemm_i8: weight_sign is for folded zero points (weight_zero must be NULL)");
    if (d->weight_sign && !iw::cm_enabled())
        return fail(IW_EINVAL, "iw_gemm_i8: weight_sign needs the channel-major kernel");
    if (d->mode < 0 || d->mode > 3) return fail(IW_EINVAL, "iw_gemm_i8: bad mode %d", d->mode);
    if ((d->mode == IW_GEMM_LINEAR32 || d->mode == IW_GEMM_LINEAR32_RES) && (!d->multiplier || !d->shift))
        return fail(IW_EINVAL, "iw_gemm_i8: Linear32 needs per-channel multiplier and shift");
    if (d->mode == IW_GEMM_LINEAR32_RES && !d->residual) return fail(IW_EINVAL, "iw_gemm_i8: residual is required");
    if ((d->headmajor_T || d->transpose_T) && d->mode != IW_GEMM_INT8)
        return fail(IW_EINVAL, "iw_gemm_i8: layouts apply to int8 outputs");
    if (d->headmajor_T && (d->N % 64 || d->headmajor_B <= 0 || d->M != d->headmajor_B * d->headmajor_T))
        return fail(IW_EINVAL, "iw_gemm_i8: head-major layout needs N%%64==0 and M == B*T");
    if (d->transpose_T && d->M % d->transpose_T) return fail(IW_EINVAL, "iw_gemm_i8: M must be a multiple of T");
    if (d->vt_out) {
        if (d->mode != IW_GEMM_INT8 || d->headmajor_T || d->transpose_T || d->pos || d->gelu_table)
            return fail(IW_EINVAL, "iw_gemm_i8: vt_out applies to plain int8 row-major outputs");
        if (d->vt_T <= 0 || d->M % d->vt_T || d->vt_col0 < 0 || d->vt_col0 % 64 || d->vt_col0 >= d->N ||
            (d->N - d->vt_col0) % 64 || d->vt_ld < d->vt_T || d->vt_ld % 16 ||
            (reinterpret_cast<uintptr_t>(d->vt_out) & 15))
            return fail(IW_EINVAL, "iw_gemm_i8: invalid vt_out layout");
    }
    iw::EpiParams p;
    p.out = d->out;
    p.ldo = d->ldo;
    p.bias = d->bias;
    p.wz = d->weight_zero;
    p.wsign = d->weight_sign;
    p.rowsum = d->x_rowsum;
    if (d->multiplier) {
        p.per_channel = 1;
        p.mult = d->multiplier;
        p.shift = d->shift;
    } else {
        p.per_channel = 0;
        p.smult = d->scalar_multiplier;
        p.sshift = (uint32_t)(d->scalar_shift > 0 ? d->scalar_shift : 0);
    }
    if (d->lut) {
        p.gelu = 1;
        p.lut = d->lut;
        p.gmi = d->luti_multiplier;
        p.gsi = d->luti_shift;
        p.gmo = d->luto_multiplier;
        p.gso = d->luto_shift;
        p.gelu_in_pc = d->luti_per_channel;
        p.gelu_out_pc = d->luto_per_channel;
    }
    p.res = d->residual;
    p.ldr = d->ldr;
    p.res_mult = d->residual_multiplier;
    if (d->pos) {
        p.posadd = 1;
        p.pe = d->pos;
        p.pe_T = (int)d->pos_T;
        p.pm = d->pos_multiplier;
        p.ps = d->pos_shift;
        p.pos_pc = d->pos_per_channel;
    }
    p.transpose_T = (int)d->transpose_T;
    p.hm_T = (int)d->headmajor_T;
    p.hm_B = (int)d->headmajor_B;
    p.rowsum_out = d->out_rowsum;
    p.gelu_tab = d->gelu_table;
    if (d->gelu_table_tiled) {
        if (!d->gelu_table || (reinterpret_cast<uintptr_t>(d->gelu_table_tiled) & 15))
            return fail(IW_EINVAL, "iw_gemm_i8: gelu_table_tiled needs gelu_table and 16-byte alignment");
        p.gelu_tab_tiled = d->gelu_table_tiled;
    }
    if (d->kv_cache_k) {
        if (!d->kv_cache_v || d->mode != IW_GEMM_INT8 || d->vt_out || d->headmajor_T || d->transpose_T || d->pos ||
            d->kv_heads <= 0 || d->kv_T <= 0 || d->M % d->kv_T || d->kv_col0 < 0 || d->kv_col0 % 64 ||
            d->kv_col0 + 2 * d->kv_heads * 64 != d->N || d->kv_Tcap < d->kv_T ||
            (!d->kv_pos_dev && (d->kv_pos < 0 || d->kv_pos + d->kv_T > d->kv_Tcap)))
            return fail(IW_EINVAL, "iw_gemm_i8: invalid KV-cache output");
        if (!iw::cm_enabled()) {
            // row-major kernel: all channels row-major, then the cache append
            iw::GemmShape g{d->x, d->ldx, d->w, d->ldw, (int)d->M, (int)d->N, (int)d->K};
            if (int r = cuda_check(iw::gemm_i8_launch(g, (iw::EpiMode)d->mode, p, S(stream), d->tile_n), "iw_gemm_i8"))
                return r;
            const int64_t kc = d->kv_col0, vc = d->kv_col0 + d->kv_heads * 64;
            return cuda_check(iw::kv_append(reinterpret_cast<const int8_t *>(d->out), d->ldo, (int)kc, (int)vc,
                                            d->kv_cache_k, d->kv_cache_v, (int)(d->M / d->kv_T), (int)d->kv_heads,
                                            (int)d->kv_T, (int)d->kv_Tcap, (int)d->kv_pos, d->kv_pos_dev, S(stream)),
                              "iw_gemm_i8");
        }
        p.kv_k = d->kv_cache_k;
        p.kv_v = d->kv_cache_v;
        p.kv_c0 = (int)d->kv_col0;
        p.kv_H = (int)d->kv_heads;
        p.kv_T = (int)d->kv_T;
        p.kv_Tcap = (int)d->kv_Tcap;
        p.kv_pos = (int)d->kv_pos;
        p.kv_pos_dev = d->kv_pos_dev;
    }
    if (d->vt_out && !iw::cm_enabled()) {
        // row-major kernel: all channels row-major, then V^T by a transpose
        iw::GemmShape g{d->x, d->ldx, d->w, d->ldw, (int)d->M, (int)d->N, (int)d->K};
        if (int r = cuda_check(iw::gemm_i8_launch(g, (iw::EpiMode)d->mode, p, S(stream), d->tile_n), "iw_gemm_i8"))
            return r;
        const int Tv = (int)d->vt_T, Bv = (int)(d->M / d->vt_T), Hv = (int)((d->N - d->vt_col0) / 64);
        return cuda_check(iw::transpose_v(reinterpret_cast<const int8_t *>(d->out) + d->vt_col0, d->ldo, Bv, Tv, Hv,
                                          d->vt_out, (int)d->vt_ld, S(stream)),
                          "iw_gemm_i8");
    }
    if (d->vt_out) {
        p.tr_out = d->vt_out;
        p.tr_c0 = (int)d->vt_col0;
        p.tr_N = (int)(d->N - d->vt_col0);
        p.tr_T = (int)d->vt_T;
        p.tr_ld = d->vt_ld;
    }
    if (d->gelu_table && (d->lut || d->mode != IW_GEMM_INT8 || !d->multiplier))
        return fail(IW_EINVAL, "iw_gemm_i8: gelu_table needs a per-channel int8 epilogue without lut");
    iw::GemmShape g{d->x, d->ldx, d->w, d->ldw, (int)d->M, (int)d->N, (int)d->K};
    if (d->x_window_rows) {
        if (d->x_window_rows < 0 || d->M % d->x_window_rows || d->x_window_stride < 0 || d->x_window_stride % 16 ||
            d->x_window_rows > INT32_MAX || !iw::cm_enabled() || d->vt_out || d->kv_cache_k || d->headmajor_T ||
            d->transpose_T)
            return fail(IW_EINVAL, "iw_gemm_i8: invalid windowed X (rows dividing M, 16-byte window stride, "
                                   "row-major or positional-add output)");
        g.win_rows = (int)d->x_window_rows;
        g.win_stride = d->x_window_stride;
    }
    return cuda_check(iw::gemm_i8_launch(g, (iw::EpiMode)d->mode, p, S(stream), d->tile_n), "iw_gemm_i8");
}

int iw_gelu_table_tiled(const int8_t *table, int64_t N, int8_t *tiled, void *stream) {
    if (N <= 0 || N > (int64_t)1 << 30) return fail(IW_EINVAL, "iw_gelu_table_tiled: invalid N");
    if (!table || !tiled || (reinterpret_cast<uintptr_t>(tiled) & 15))
        return fail(IW_EINVAL, "iw_gelu_table_tiled: tiled must be 16-byte aligned");
    return cuda_check(iw::gelu_table_tile(table, (int)N, tiled, S(stream)), "iw_gelu_table_tiled");
}

int iw_gelu_table(const uint8_t *lut, const uint8_t *luti_multiplier, const int8_t *luti_shift,
                  const uint8_t *luto_multiplier, const int8_t *luto_shift, int64_t luti_count, int64_t luto_count,
                  int64_t N, int8_t *table, void *stream) {
    if (N <= 0) return fail(IW_EINVAL, "iw_gelu_table: N must be positive");
    if (!(luti_count == 1 || luti_count == N) || !(luto_count == 1 || luto_count == N))
        return fail(IW_EINVAL, "iw_gelu_table: parameter counts must be 1 or N");
    return cuda_check(iw::gelu_table_build(lut, luti_multiplier, luti_shift, luto_multiplier, luto_shift,
                                           (int)luti_count, (int)luto_count, (int)N, table, S(stream)),
                      "iw_gelu_table");
}

int iw_attention_ex(const iw_attn_desc *d, void *stream) {
    if (!d) return fail(IW_EINVAL, "iw_attention_ex: null descriptor");
    if (d->B < 0 || d->H < 0 || d->Tq < 0 || d->Tk < 0) return fail(IW_EINVAL, "iw_attention_ex: invalid shape");
    if (!fused_frac_bits_ok(d->frac_bits)) return fail(IW_EINVAL, "frac_bits must be in [1, 30]");
    if (!(d->rsqrt_offset >= 0 && d->rsqrt_offset <= 29)) return fail(IW_EINVAL, "rsqrt_offset must be in [0,29]");
    if (d->mask_mode == 2 && !d->mask) return fail(IW_EINVAL, "iw_attention_ex: mask_mode 2 needs a mask");
    if (((d->ldq | d->ldk | d->ldv | d->q_bs | d->k_bs | d->v_bs | d->q_hs | d->k_hs | d->v_hs) & 15) ||
        ((reinterpret_cast<uintptr_t>(d->q) | reinterpret_cast<uintptr_t>(d->k) | reinterpret_cast<uintptr_t>(d->v)) &
         15))
        return fail(IW_EINVAL, "iw_attention_ex: Q/K/V rows must be 16-byte aligned");
    iw::AttnArgs a;
    a.q = d->q; a.ldq = d->ldq; a.q_bs = d->q_bs; a.q_hs = d->q_hs;
    a.k = d->k; a.ldk = d->ldk; a.k_bs = d->k_bs; a.k_hs = d->k_hs;
    a.v = d->v; a.ldv = d->ldv; a.v_bs = d->v_bs; a.v_hs = d->v_hs;
    a.out = d->y; a.ldo = d->ldy; a.o_bs = d->y_bs; a.o_hs = d->y_hs;
    a.Tq = (int)d->Tq; a.Tk = (int)d->Tk; a.Tk_dev = d->Tk_dev;
    a.Tk_cap = (int)(d->Tk_cap > 0 ? d->Tk_cap : d->Tk);
    a.mask_mode = d->mask_mode; a.mask = d->mask;
    a.qk_mult = d->qk_multiplier; a.qk_shift = d->qk_shift; a.frac_bits = d->frac_bits;
    a.av_mult = d->av_multiplier; a.av_shift = d->av_shift; a.rsqrt_offset = (uint32_t)d->rsqrt_offset;
    const bool tc = d->exp_table && d->vt && d->mask_mode == 0 && d->Tq == d->Tk && d->Tk > 0 && !d->Tk_dev &&
                    d->q_hs == 64 && d->k_hs == 64 && d->v_hs == 64 && d->y_hs == 64 &&
                    d->q_bs == d->Tq * d->ldq && d->k_bs == d->Tk * d->ldk && d->v_bs == d->Tk * d->ldv &&
                    d->y_bs == d->Tq * d->ldy && (d->ldy % 16) == 0 && (reinterpret_cast<uintptr_t>(d->y) & 15) == 0 &&
                    d->vt_ld >= d->Tk && (d->vt_ld % 16) == 0 && (reinterpret_cast<uintptr_t>(d->vt) & 15) == 0;
    a.rowsum_out = d->row_sum_out;
    if (tc)
        return cuda_check(iw::attention_tc(a, (int)d->B, (int)d->H, d->exp_table, d->vt, (int)d->vt_ld,
                                           d->vt_ready != 0, S(stream)),
                          "iw_attention_ex");
    return cuda_check(iw::attention_cc(a, (int)d->B, (int)d->H, S(stream)), "iw_attention_ex");
}

int iw_shift_exp_table(int32_t frac_bits, uint8_t *table, void *stream) {
    if (!fused_frac_bits_ok(frac_bits)) return fail(IW_EINVAL, "frac_bits must be in [1, 30]");
    cudaStream_t st = S(stream);
    Scratch sc(st);
    if (int r = cuda_check(sc.alloc(2 * sizeof(int)), "iw_shift_exp_table")) return r;
    if (int r = cuda_check(iw::shift_exp_table_build(frac_bits, table, (int *)sc.p, st), "iw_shift_exp_table")) return r;
    int h[2] = {0, 0};
    if (int r = cuda_check(cudaMemcpyAsync(h, sc.p, sizeof(h), cudaMemcpyDeviceToHost, st), "iw_shift_exp_table"))
        return r;
    if (int r = cuda_check(cudaStreamSynchronize(st), "iw_shift_exp_table")) return r;
    if (h[1]) return fail(IW_EVALUE, "shift-exp table for frac_bits %d exceeds the tensor-core kernel", frac_bits);
    return IW_OK;
}

int iw_layernorm32_ex(const int16_t *x, int64_t ldx, const int8_t *weight, const int32_t *bias,
                      uint8_t ln_multiplier, int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y,
                      int64_t ldy, int64_t rows, int64_t d, int32_t *rowsum_out, int32_t *rowsum_zero, void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    iw::LnParams p{(int32_t)ln_multiplier, (int32_t)ln_shift, out_multiplier, (uint32_t)(int32_t)out_shift, 13u};
    return cuda_check(
        iw::layernorm32(x, ldx, weight, bias, p, y, ldy, (int)rows, (int)d, rowsum_out, rowsum_zero, S(stream)),
        "iw_layernorm32_ex");
}

// layernorm_torch.cpp:446-460: LayerNorm64 runs FISR with offset 15 and
// adds 2 to the normalise shift
static iw::LnParams ln64_params(uint8_t ln_multiplier, int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift) {
    iw::LnParams p{(int32_t)ln_multiplier, (int32_t)ln_shift, out_multiplier, (uint32_t)(int32_t)out_shift, 15u};
    p.additional_offset = 2;
    return p;
}

int iw_layernorm64(const int16_t *x, const int8_t *weight, const int32_t *bias, uint8_t ln_multiplier,
                   int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y, int64_t rows, int64_t d,
                   void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    if (rows < 0 || rows > INT32_MAX) return fail(IW_EINVAL, "iw_layernorm64: invalid row count");
    if (rows == 0) return IW_OK;
    cudaStream_t st = S(stream);
    Scratch f(st);
    if (int r = cuda_check(f.alloc(sizeof(int)), "iw_layernorm64")) return r;
    if (int r = cuda_check(cudaMemsetAsync(f.p, 0, sizeof(int), st), "iw_layernorm64")) return r;
    iw::LnParams p = ln64_params(ln_multiplier, ln_shift, out_multiplier, out_shift);
    p.overflow = (int *)f.p;
    if (int r = cuda_check(iw::layernorm32(x, d, weight, bias, p, y, d, (int)rows, (int)d, nullptr, nullptr, st, true),
                           "iw_layernorm64"))
        return r;
    int h = 0;
    if (int r = cuda_check(cudaMemcpyAsync(&h, f.p, sizeof(int), cudaMemcpyDeviceToHost, st), "iw_layernorm64")) return r;
    if (int r = cuda_check(cudaStreamSynchronize(st), "iw_layernorm64")) return r;
    if (h) return fail(IW_EOVERFLOW, "LayerNorm64 variance does not fit INT32");
    return IW_OK;
}

int iw_layernorm64_stats(const int16_t *x, int32_t *mean, int64_t *variance, int64_t rows, int64_t d, void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    if (rows < 0 || rows > INT32_MAX) return fail(IW_EINVAL, "iw_layernorm64_stats: invalid row count");
    return cuda_check(iw::layernorm64_stats(x, (int)rows, (int)d, mean, variance, S(stream)), "iw_layernorm64_stats");
}

int iw_layernorm64_ex(const int16_t *x, int64_t ldx, const int8_t *weight, const int32_t *bias,
                      uint8_t ln_multiplier, int8_t ln_shift, uint32_t out_multiplier, int8_t out_shift, int8_t *y,
                      int64_t ldy, int64_t rows, int64_t d, int32_t *rowsum_out, int32_t *rowsum_zero, void *stream) {
    if (!ln_width_ok(d)) return fail(IW_EINVAL, "unsupported LayerNorm hidden size: %lld", (long long)d);
    const iw::LnParams p = ln64_params(ln_multiplier, ln_shift, out_multiplier, out_shift);
    return cuda_check(
        iw::layernorm32(x, ldx, weight, bias, p, y, ldy, (int)rows, (int)d, rowsum_out, rowsum_zero, S(stream), true),
        "iw_layernorm64_ex");
}

int iw_im2col(const int8_t *x, int8_t *out, int64_t B, int64_t Cin, int64_t Tin, int64_t K, int64_t stride,
              int64_t pad, int64_t Tout, int64_t ldo, int channels_last, void *stream) {
    if (ldo < Cin * K) return fail(IW_EINVAL, "iw_im2col: ldo < Cin*K");
    return cuda_check(iw::im2col(x, out, (int)B, (int)Cin, (int)Tin, (int)K, (int)stride, (int)pad, (int)Tout, ldo,
                                 channels_last, S(stream)),
                      "iw_im2col");
}

int iw_channels_last_pad(const int8_t *x, int64_t B, int64_t C, int64_t T, int64_t front, int64_t back, int8_t *out,
                         void *stream) {
    if (B < 0 || C < 0 || T < 0 || front < 0 || back < 0 || B > 65535 || (T + front + back) > INT32_MAX / 2 ||
        C > INT32_MAX / 2)
        return fail(IW_EINVAL, "iw_channels_last_pad: invalid shape");
    return cuda_check(iw::channels_last_pad(x, (int)B, (int)C, (int)T, (int)front, (int)back, out, S(stream)),
                      "iw_channels_last_pad");
}

int iw_zero_rows(void *p, int64_t count, int64_t bytes, int64_t pitch, void *stream) {
    if (count < 0 || bytes < 0 || pitch < bytes) return fail(IW_EINVAL, "iw_zero_rows: invalid shape");
    if (count == 0 || bytes == 0) return IW_OK;
    return cuda_check(cudaMemset2DAsync(p, (size_t)pitch, 0, (size_t)bytes, (size_t)count, S(stream)), "iw_zero_rows");
}

int iw_embed_add_requant15_dev(const int8_t *table, const int64_t *tokens, const int8_t *pe,
                               const int32_t *offset_dev, int64_t offset, const uint16_t *multiplier,
                               const int8_t *shift, int16_t *y, int64_t B, int64_t T, int64_t C,
                               int64_t multiplier_count, int64_t shift_count, void *stream) {
    if (!(multiplier_count == 1 || multiplier_count == C)) return fail(IW_EINVAL, "multiplier must contain 1 or C elements");
    if (!(shift_count == 1 || shift_count == C)) return fail(IW_EINVAL, "shift must contain 1 or C elements");
    return cuda_check(iw::add_requant15(table, tokens, pe, multiplier, shift, y, (int)B, (int)T, (int)C,
                                        (int)multiplier_count, (int)shift_count, (int)offset, offset_dev, S(stream)),
                      "iw_embed_add_requant15_dev");
}

int iw_kv_append(const int8_t *src, int64_t lds, int64_t k_col, int64_t v_col, int8_t *k_cache, int8_t *v_cache,
                 int64_t B, int64_t H, int64_t T, int64_t Tcap, int64_t pos, const int32_t *pos_dev, void *stream) {
    if ((lds | k_col | v_col) & 3) return fail(IW_EINVAL, "iw_kv_append: columns must be 4-byte aligned");
    return cuda_check(iw::kv_append(src, lds, (int)k_col, (int)v_col, k_cache, v_cache, (int)B, (int)H, (int)T,
                                    (int)Tcap, (int)pos, pos_dev, S(stream)),
                      "iw_kv_append");
}

int iw_greedy_step(const iw_greedy_desc *d, int64_t B, void *stream) {
    if (!d) return fail(IW_EINVAL, "iw_greedy_step: null descriptor");
    if (d->V <= 0 || d->ld < d->V || d->V > INT32_MAX) return fail(IW_EINVAL, "iw_greedy_step: need 0 < V <= ld");
    if (!(d->alpha > 0.f)) return fail(IW_EINVAL, "iw_greedy_step: alpha must be positive");
    iw::GreedyArgs g;
    g.logits = d->logits; g.ld = d->ld; g.V = (int)d->V; g.alpha = d->alpha;
    g.suppress_bits = d->suppress_bits; g.blank = d->blank; g.n_blank = (int)d->n_blank;
    g.eot = (int)d->eot; g.timestamp_begin = (int)d->timestamp_begin; g.no_timestamps = (int)d->no_timestamps;
    g.max_initial_timestamp_index = (int)d->max_initial_timestamp_index;
    g.state = d->state; g.tokens = d->tokens; g.ld_tok = d->ld_tok; g.step_dev = d->step_dev; g.next = d->next;
    return cuda_check(iw::greedy_step(g, (int)B, S(stream)), "iw_greedy_step");
}

int iw_log_mel_int8(const float *audio, int64_t B, int64_t n_samples, int64_t lda, const float *filters,
                    int64_t n_mels, float input_alpha, int8_t *out, void *stream) {
    if (B < 0 || n_samples <= 256 || n_samples > INT32_MAX || lda < n_samples || n_mels <= 0 || n_mels > 128)
        return fail(IW_EINVAL, "iw_log_mel_int8: invalid shape");
    if (B == 0) return IW_OK;
    cudaStream_t st = S(stream);
    const int64_t frames = n_samples / 160;
    Scratch work(st), wmax(st);
    if (int r = cuda_check(work.alloc((size_t)(B * n_mels * frames) * sizeof(float)), "iw_log_mel_int8")) return r;
    if (int r = cuda_check(wmax.alloc((size_t)B * sizeof(int32_t)), "iw_log_mel_int8")) return r;
    return cuda_check(iw::log_mel_int8(audio, (int)B, (int)n_samples, lda, filters, (int)n_mels, input_alpha,
                                       (float *)work.p, (int32_t *)wmax.p, out, st),
                      "iw_log_mel_int8");
}

int iw_add_i32(int32_t *p, int32_t v, void *stream) {
    return cuda_check(iw::add_i32(p, v, S(stream)), "iw_add_i32");
}

}  // extern "C"
