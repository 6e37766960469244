// noalloc.cu -- iw_linear8_noalloc: Linear8 without any device allocation.
//
// iw_linear8 takes a stream-ordered scratch buffer (cudaMallocAsync) for the
// row sums of x that the weight zero-point term needs. Some callers cannot
// allocate device memory at call time: code running inside a captured CUDA
// graph whose memory pool they do not control, inference servers that
// pre-plan every byte of device memory and forbid allocator traffic on the
// request path, or hosts that drive the GPU through another runtime and only
// hand over raw pointers. iw_linear8_noalloc serves them: the row sums live
// in a fixed file-scope device array instead.
//
// The array holds IW_NOALLOC_MAX_ROWS int32 row sums (256 KiB). Every GPU
// that loads this library keeps that much memory reserved until the process
// exits. Every call shares the array, so calls whose executions overlap on
// the GPU (different streams, or different host threads) race on it; order
// such calls on one stream. The row-sum kernel writes all M entries a call
// uses before the GEMM reads them, so nothing has to be cleared between
// calls.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/iwhisper_b200.h"
#include "gemm_i8.cuh"
#include "kernels.cuh"

namespace iw {

static __device__ __align__(256) int32_t g_noalloc_rowsum[IW_NOALLOC_MAX_ROWS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
int32_t *g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_rowsum on the current device, looked up once
// per device (with that device current). In host code the symbol name is a
// host-side stand-in, not a device address, so it must never be passed to a
// kernel directly.
cudaError_t noalloc_scratch(int32_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_rowsum);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = reinterpret_cast<int32_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace iw

extern "C" int iw_linear8_noalloc(const int8_t *x, const int8_t *weight, const int32_t *bias,
                                  const int8_t *weight_zero, const uint32_t *multiplier, const int8_t *shift, int8_t *y,
                                  int64_t M, int64_t K, int64_t N, void *stream) {
    if (M < 0 || N <= 0) return fail(IW_EINVAL, "iw_linear8_noalloc: invalid shape M=%lld N=%lld", (long long)M, (long long)N);
    if (K <= 0) return fail(IW_EINVAL, "iw_linear8_noalloc: x.size(-1) must be greater than 0");
    if (M > IW_NOALLOC_MAX_ROWS)
        return fail(IW_EINVAL, "iw_linear8_noalloc: M=%lld exceeds the %d rows of its fixed scratch array",
                    (long long)M, IW_NOALLOC_MAX_ROWS);
    if (K % 16 != 0)
        return fail(IW_EINVAL, "iw_linear8_noalloc: K=%lld must be a multiple of 16 (no padding buffer is allocated)",
                    (long long)K);
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(weight) & 15))
        return fail(IW_EINVAL, "iw_linear8_noalloc: x and weight must be 16-byte aligned");
    if (N > INT32_MAX || K > INT32_MAX) return fail(IW_EINVAL, "iw_linear8_noalloc: dimension too large");
    if (M == 0) return IW_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    iw::EpiParams p;
    p.out = y;
    p.ldo = N;
    p.bias = bias;
    p.wz = weight_zero;
    p.mult = multiplier;
    p.shift = shift;
    p.per_channel = 1;
    if (weight_zero) {
        int32_t *rs = nullptr;
        if (int r = cuda_check(iw::noalloc_scratch(&rs), "iw_linear8_noalloc")) return r;
        if (int r = cuda_check(iw::rowsum_i8(x, K, (int)M, (int)K, rs, st), "iw_linear8_noalloc")) return r;
        p.rowsum = rs;
    }
    iw::GemmShape g{x, K, weight, K, (int)M, (int)N, (int)K};
    return cuda_check(iw::gemm_i8_launch(g, iw::EPI_L8, p, st), "iw_linear8_noalloc");
}
