// iw_common.cuh -- integer fixed-point arithmetic shared by every kernel.
//
// Device restatements of the reference primitives in
// i_whisper/kernels/csrc/common/fixedpoint.h (vcsd-lab/I-Whisper). All
// wrap-around behaviour is spelled out with uint32 arithmetic.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <utility>
#include <cuda_runtime.h>

#define IW_DEV __device__ __forceinline__

namespace iw {

IW_DEV int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
IW_DEV int32_t wsub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
IW_DEV int32_t wmul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }
__host__ __device__ __forceinline__ int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

// fixedpoint.h:35-44: high word of (int64)x * (uint32)m. Written as the
// unsigned high product corrected for a negative x:
//   (int64)x*m = (uint32)x*m - (x<0 ? m<<32 : 0)
IW_DEV int32_t mulh(int32_t x, uint32_t m) {
    uint32_t hi = __umulhi((uint32_t)x, m);
    return (int32_t)(hi - (x < 0 ? m : 0u));
}

// fixedpoint.h:47-87: shift 0 -> x, shift >= 32 -> 0, else
// (x + 2^(s-1) - signbit) with uint32 wrap, arithmetic shift right.
IW_DEV int32_t rrs(int32_t x, uint32_t s) {
    if (s == 0) return x;
    if (s >= 32) return 0;
    uint32_t v = (uint32_t)x + (1u << (s - 1)) - ((uint32_t)x >> 31);
    return ((int32_t)v) >> s;
}

// Same as rrs for a shift known to lie in [1,31].
IW_DEV int32_t rrs_pos(int32_t x, uint32_t s) {
    uint32_t v = (uint32_t)x + (1u << (s - 1)) - ((uint32_t)x >> 31);
    return ((int32_t)v) >> s;
}

IW_DEV int32_t bit_length_nonneg(int32_t x) { return x == 0 ? 0 : 32 - __clz(x); }

// layernorm_scalar.cpp:309-343 -- int32 -> fp32 bit pattern with the
// mantissa truncated (never rounded).
IW_DEV int32_t int32_to_fp32_bits_trunc(int32_t x) {
    if (x == 0) return 0;
    int32_t e = 31 - __clz(x);
    uint32_t ux = (uint32_t)x;
    uint32_t sig = e <= 23 ? (ux << (23 - e)) : (ux >> (e - 23));
    return (int32_t)(((uint32_t)(e + 127) << 23) | (sig & 0x007FFFFFu));
}

// layernorm_scalar.cpp:345-381 -- fp32 bit pattern -> int32, truncating;
// a left shift of the 24-bit significand keeps only its low 32 bits.
IW_DEV int32_t fp32_bits_to_int32_trunc(int32_t bits) {
    uint32_t raw = (uint32_t)bits;
    int32_t e = (int32_t)((raw >> 23) & 0xFFu) - 127;
    uint64_t sig = (uint64_t)((1u << 23) | (raw & 0x007FFFFFu));
    if (e < 0) return 0;
    uint64_t v;
    if (e >= 23) {
        int32_t sh = e - 23;
        v = sh >= 64 ? 0ull : (sig << sh);
    } else {
        v = sig >> (23 - e);
    }
    return (int32_t)(uint32_t)v;
}

// layernorm_scalar.cpp:383-437 -- integer fast inverse square root in
// Q(off): magic-constant seed computed on the truncated fp32 bit pattern,
// then two Newton steps with wrapping products and rounding shifts.
IW_DEV int32_t fisr(int32_t x, uint32_t off) {
    int32_t i = int32_to_fp32_bits_trunc(x);
    i = (int32_t)0x5f3759dfu - (i >> 1);
    int32_t y = fp32_bits_to_int32_trunc((int32_t)((uint32_t)i + (off << 23)));
    const int32_t three = (int32_t)(3u << off);
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        int32_t xys = rrs(wmul(x, y), off);
        int32_t t = wmul(xys, y);
        y = rrs(wmul(y, wsub(three, t)), off + 1);
    }
    return y;
}

// gelu_scalar.cpp:10-181 -- one element of the LUT GeLU.
IW_DEV int32_t gelu_one(int32_t x, const uint8_t *lut, uint32_t mi, uint32_t si,
                        uint32_t mo, uint32_t so) {
    int32_t idx = rrs(x * (int32_t)mi, si);
    idx = clampi(idx + 8, 0, 15);
    int32_t v = x * (int32_t)lut[idx];
    v = v * (int32_t)mo;
    v = rrs(v, so);
    return clampi(v, -127, 127);
}

// rounding_rshift(x, s) (fixedpoint.h:47-87) with the shift folded into
// constants: s == 0 -> x, s >= 32 -> 0, otherwise
// (int32)((u32)x + 2^(s-1) - (x < 0)) >> s.
struct RrsK {
    int32_t rnd, sgn, sh, z;
};
IW_DEV RrsK rrs_k(uint32_t s) {
    if (s == 0) return {0, 0, 0, -1};
    if (s < 32) return {(int32_t)(1u << (s - 1)), -1, (int32_t)s, -1};
    return {0, 0, 0, 0};
}
IW_DEV int32_t rrs_apply(int32_t x, const RrsK &k) {
    const int32_t t = wadd(wadd(x, k.rnd), (x >> 31) & k.sgn);
    return (t >> k.sh) & k.z;
}

// attention_scalar.cpp:388-560 -- shift-based exp2 of (x - rowmax1) in
// int16 wrapping arithmetic. The caller handles masked lanes.
IW_DEV int32_t shift_exp_one(int32_t x, int32_t xm, int32_t fb) {
    int16_t xs = (int16_t)(x - xm);
    if (xs > 0) return 0;
    int16_t half = (int16_t)(xs >> 1);
    int16_t six = (int16_t)(xs >> 4);
    int16_t fix = (int16_t)((int16_t)(xs + half) - six);
    int16_t xi = (int16_t)(fix >> fb);
    int32_t scale = 1 << fb;
    int16_t ip = (int16_t)((int32_t)xi * scale);
    int16_t fr = (int16_t)(fix - ip);
    int16_t num = (int16_t)(scale + (int32_t)(fr >> 1));
    int16_t e;
    if (xi > 0) {
        e = 0;
    } else {
        int32_t es = -(int32_t)xi;
        e = es >= 16 ? (int16_t)0 : (int16_t)(num >> es);
    }
    if (fb > 7) return (int32_t)(uint8_t)((int32_t)e >> (fb - 7));
    return (int32_t)(uint8_t)e;
}

// Programmatic dependent launch. Kernels launched by launch_pdl may start
// while the previous kernel on the stream is finishing: each kernel does its
// private set-up (shared-memory barriers, TMEM allocation), then pdl_wait()
// blocks until the previous grid has completed and its writes are visible,
// before the kernel touches global memory; pdl_launch() lets the next kernel
// be scheduled. Without the launch attribute both are no-ops.
IW_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
IW_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Device-side status word: set by bounded waits that gave up, read by the
// host after a synchronisation (iw_device_status in the C ABI).
enum : uint32_t {
    IW_DEVERR_NONE = 0,
    IW_DEVERR_WAIT_TIMEOUT = 1u << 0,
    IW_DEVERR_LN64_OVERFLOW = 1u << 1,  // a LayerNorm64 variance did not fit INT32
};

// The library is built as one translation unit (iw_lib.cu), so this single
// definition is shared by every kernel.
__device__ uint32_t g_device_status = 0;

// false when IW_PDL=0 is set in the environment (plain stream-ordered launches)
inline bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("IW_PDL");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// Kernel attributes belong to a device's context: a process that drives
// several GPUs must set them on each. SmemLimit records, per device, the
// dynamic shared-memory limit already set for one kernel; raise_smem_limit
// sets it on the current device the first time a launch there needs more.
// The set-and-record runs under a mutex so that two host threads can never
// leave a smaller limit in place than the one recorded.
constexpr int kMaxDevices = 64;
struct SmemLimit {
    std::atomic<int> bytes[kMaxDevices];  // static storage: zero-initialised
    std::mutex mu;
};

template <typename... KArgs>
inline cudaError_t raise_smem_limit(void (*kernel)(KArgs...), size_t bytes, SmemLimit &lim) {
    if (bytes <= 48 * 1024) return cudaSuccess;  // the default limit
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int want = (int)bytes;
    if (dev < 0 || dev >= kMaxDevices)
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (lim.bytes[dev].load(std::memory_order_acquire) >= want) return cudaSuccess;
    std::lock_guard<std::mutex> g(lim.mu);
    if (lim.bytes[dev].load(std::memory_order_relaxed) >= want) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e == cudaSuccess) lim.bytes[dev].store(want, std::memory_order_release);
    return e;
}

// Streaming multiprocessors of the current device (cached per device).
inline int num_sms() {
    static std::atomic<int> n[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    const int slot = (dev >= 0 && dev < kMaxDevices) ? dev : 0;
    int v = n[slot].load(std::memory_order_relaxed);
    if (v <= 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        n[slot].store(v, std::memory_order_relaxed);
    }
    return v;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace iw
