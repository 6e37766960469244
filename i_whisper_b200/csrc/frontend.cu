// frontend.cu -- the float log-mel frontend of i_whisper/audio.py:216-265 and
// the input quantisation of AudioEncoder_int.forward (model_int.py:1265-1267)
// on the GPU, so raw 16 kHz audio reaches the integer encoder without a
// host round trip.
//
// Per window: reflect-padded frames of 512 samples every 160 (torch.stft
// with center=True), periodic Hann window, a 512-point radix-2 FFT in
// shared memory (float32), power |X|^2 formed as hypot(re, im)^2 like
// torch's abs()**2, the last frame dropped, the mel filterbank applied over
// each filter's non-zero bins, log10 of max(mel, 1e-10). A second kernel
// applies max(lg, window max - 8) / 4 + 1, multiplies by the encoder's
// input_alpha, rounds half to even and clamps to +-127. Float results are
// not bit-identical to torch (summation orders differ); the INT8 output is
// checked against the float64 restatement within one unit.
#include <cuda_runtime.h>

#include <cstdint>

#include "iw_common.cuh"

namespace iw {

constexpr int kFftN = 512;
constexpr int kFftBins = kFftN / 2 + 1;  // 257
constexpr int kHop = 160;
constexpr int kLmThreads = 256;
constexpr int kLmFrames = 24;            // frames per CTA (filters staged once)

// ordered-int image of a float: signed comparison follows the float order
IW_DEV int32_t float_order(float f) {
    const int32_t b = __float_as_int(f);
    return b ^ ((b >> 31) & 0x7FFFFFFF);
}
IW_DEV float float_unorder(int32_t o) { return __int_as_float(o ^ ((o >> 31) & 0x7FFFFFFF)); }

__global__ void __launch_bounds__(kLmThreads) logmel_kernel(const float *__restrict__ audio, int64_t lda,
                                                            int n_samples, int n_frames,
                                                            const float *__restrict__ filters, int n_mels,
                                                            float *__restrict__ logmel, int32_t *__restrict__ wmax) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sm[];
    float *sfilt = sm;                                                  // [n_mels][257]
    float2 *buf = reinterpret_cast<float2 *>(sfilt + n_mels * kFftBins + 1);  // 8-byte aligned below
    buf = reinterpret_cast<float2 *>((reinterpret_cast<uintptr_t>(buf) + 7) & ~uintptr_t(7));
    float *pw = reinterpret_cast<float *>(buf + kFftN);                 // [257]
    __shared__ float2 stw[kFftN / 2];
    __shared__ int32_t sred[kLmThreads / 32];
    const int b = blockIdx.y;
    const int tid = threadIdx.x;
    for (int i = tid; i < n_mels * kFftBins; i += kLmThreads) sfilt[i] = filters[i];
    for (int i = tid; i < kFftN / 2; i += kLmThreads) {
        float s, c;
        sincospif(2.f * (float)i / (float)kFftN, &s, &c);
        stw[i] = make_float2(c, -s);  // e^{-2 pi i j / 512}
    }
    __syncthreads();
    // this thread's mel filter: its first and last non-zero bins
    int lo = 0, hi = -1;
    if (tid < n_mels) {
        for (int k = 0; k < kFftBins; ++k)
            if (sfilt[tid * kFftBins + k] != 0.f) {
                if (hi < 0) lo = k;
                hi = k;
            }
    }
    const float *xa = audio + (int64_t)b * lda;
    int32_t lmax = float_order(-INFINITY);
    const int f0 = blockIdx.x * kLmFrames;
    for (int f = f0; f < min(f0 + kLmFrames, n_frames); ++f) {
        // windowed frame, written at bit-reversed positions
        for (int n = tid; n < kFftN; n += kLmThreads) {
            int i = f * kHop + n - kFftN / 2;
            if (i < 0) i = -i;
            if (i >= n_samples) i = 2 * (n_samples - 1) - i;
            // periodic Hann window (torch.hann_window default)
            const float w = 0.5f - 0.5f * cospif(2.f * (float)n / (float)kFftN);
            buf[__brev((unsigned)n) >> 23] = make_float2(xa[i] * w, 0.f);
        }
        __syncthreads();
        // radix-2 decimation in time, one butterfly per thread per stage
        for (int half = 1; half < kFftN; half <<= 1) {
            const int t = tid;  // 256 butterflies
            const int pos = t & (half - 1);
            const int i0 = ((t - pos) << 1) + pos, i1 = i0 + half;
            const float2 w = stw[pos * (kFftN / 2 / half)];
            const float2 a = buf[i0], c = buf[i1];
            const float2 bb = make_float2(c.x * w.x - c.y * w.y, c.x * w.y + c.y * w.x);
            buf[i0] = make_float2(a.x + bb.x, a.y + bb.y);
            buf[i1] = make_float2(a.x - bb.x, a.y - bb.y);
            __syncthreads();
        }
        for (int k = tid; k < kFftBins; k += kLmThreads) {
            const float m = hypotf(buf[k].x, buf[k].y);
            pw[k] = m * m;
        }
        __syncthreads();
        if (tid < n_mels) {
            float acc = 0.f;
            for (int k = lo; k <= hi; ++k) acc = fmaf(sfilt[tid * kFftBins + k], pw[k], acc);
            const float lg = log10f(fmaxf(acc, 1e-10f));
            logmel[((int64_t)b * n_mels + tid) * n_frames + f] = lg;
            lmax = max(lmax, float_order(lg));
        }
        __syncthreads();  // buf and pw are reused by the next frame
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if ((tid & 31) == 0) sred[tid >> 5] = lmax;
    __syncthreads();
    if (tid == 0) {
        int32_t m = sred[0];
        for (int w = 1; w < kLmThreads / 32; ++w) m = max(m, sred[w]);
        atomicMax(wmax + b, m);
    }
}

__global__ void logmel_quant_kernel(const float *__restrict__ logmel, const int32_t *__restrict__ wmax, int per_window,
                                    int64_t total, float alpha, int8_t *__restrict__ out) {
    pdl_wait();
    pdl_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const float floor_v = float_unorder(wmax[i / per_window]) - 8.0f;
        float v = fmaxf(logmel[i], floor_v);
        v = v / 4.0f + 1.0f;
        v = rintf(v * alpha);
        out[i] = (int8_t)fminf(fmaxf(v, -127.f), 127.f);
    }
}

__global__ void fill_i32_kernel(int32_t *p, int n, int32_t v) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

size_t logmel_smem_bytes(int n_mels) { return (size_t)(n_mels * kFftBins + 1) * 4 + 8 + kFftN * 8 + kFftBins * 4; }

cudaError_t log_mel_int8(const float *audio, int B, int n_samples, int64_t lda, const float *filters, int n_mels,
                         float alpha, float *work, int32_t *wmax, int8_t *out, cudaStream_t st) {
    const int n_frames = n_samples / kHop;  // torch.stft frames minus the dropped last one
    if (B <= 0 || n_frames <= 0) return cudaSuccess;
    fill_i32_kernel<<<(B + 255) / 256, 256, 0, st>>>(wmax, B, INT32_MIN);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = logmel_smem_bytes(n_mels);
    static SmemLimit lim;
    e = raise_smem_limit(logmel_kernel, smem, lim);
    if (e != cudaSuccess) return e;
    dim3 grid((n_frames + kLmFrames - 1) / kLmFrames, B);
    e = launch_pdl(logmel_kernel, grid, kLmThreads, smem, st, audio, lda, n_samples, n_frames, filters, n_mels, work,
                   wmax);
    if (e != cudaSuccess) return e;
    const int64_t total = (int64_t)B * n_mels * n_frames;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    return launch_pdl(logmel_quant_kernel, (unsigned)blocks, 256, 0, st, work, wmax, n_mels * n_frames, total, alpha,
                      out);
}

}  // namespace iw
