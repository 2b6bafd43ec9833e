// Machine-ceiling probes for the B200 roofline: HBM read-stream and copy
// bandwidth, the fp32 FMA rate, and a host triad -- the CUDA counterpart of
// the reference's Metal probe (bench/metal/roofline_probe.mm), read by
// kernelverify_b200.roofline. Measurement infrastructure, not the decode path:
// it is built into its own library, apart from libkvq_b200.
//
// The kernels are plain grid-stride loops over 16-byte vectors sized to the
// whole GPU (a multiple of the SM count); the caller times them with CUDA
// events. Every access stays inside the buffer the caller passes; nothing
// waits on anything.
#include <cuda_runtime.h>

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

constexpr int kThreads = 512;

// Read every 16-byte vector once (streaming loads, no L1 allocation) and fold
// them into one word per block, so the loads cannot be elided.
__global__ void __launch_bounds__(kThreads) read_stream(const uint4* __restrict__ src, size_t n,
                                                        unsigned* __restrict__ sink) {
    uint32_t acc = 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n; i += 4 * stride) {
        const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride);
        const uint4 c = __ldcs(src + i + 2 * stride), d = __ldcs(src + i + 3 * stride);
        acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w;
        acc ^= c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n; i += stride) {
        const uint4 a = __ldcs(src + i);
        acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicXor(sink + blockIdx.x, acc);
}

__global__ void __launch_bounds__(kThreads) copy_stream(const uint4* __restrict__ src,
                                                        uint4* __restrict__ dst, size_t n) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        __stcs(dst + i, __ldcs(src + i));
}

// Eight independent FMA chains per thread; `iters` rounds of all eight.
__global__ void __launch_bounds__(kThreads) fma_chains(float* __restrict__ out, int iters,
                                                       float a, float b) {
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = (float)(threadIdx.x + k) * 1e-3f;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = fmaf(x[k], a, b);
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += x[k];
    if (s == 1234.5f) out[blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the chains live
}

int blocks_for(int per_sm) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * per_sm;
}

}  // namespace

extern "C" {

// Grid sizes the probes launch with (blocks of 512 threads).
int kvq_probe_blocks(int per_sm) { return blocks_for(per_sm > 0 ? per_sm : 4); }

// One read pass over `bytes` (a multiple of 16) of `src`; `sink` holds one
// word per block (kvq_probe_blocks). Returns 0, or -1 for bad arguments, or
// the CUDA error of the launch.
int kvq_probe_read(const void* src, size_t bytes, unsigned* sink, int blocks, void* stream) {
    if (!src || !sink || bytes % 16 || blocks < 1) return -1;
    read_stream<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), bytes / 16, sink);
    return (int)cudaGetLastError();
}

// One copy of `bytes` (a multiple of 16) from src to dst (read + write bytes
// move: 2 x bytes).
int kvq_probe_copy(const void* src, void* dst, size_t bytes, int blocks, void* stream) {
    if (!src || !dst || bytes % 16 || blocks < 1) return -1;
    copy_stream<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), bytes / 16);
    return (int)cudaGetLastError();
}

// blocks x 512 threads x 8 chains x iters FMAs (2 flops each); `out` holds
// blocks x 512 floats and is written only in a case that never happens.
int kvq_probe_fma(float* out, int blocks, int iters, void* stream) {
    if (!out || blocks < 1 || iters < 1) return -1;
    fma_chains<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(out, iters, 0.999f,
                                                                        1e-3f);
    return (int)cudaGetLastError();
}

// Host triad a[i] = b[i] + s * c[i] over three arrays of n doubles on
// `threads` threads, best of `reps`; the GB/s (24 bytes per element) is
// written to *gbs. Returns 0 or -1.
int kvq_probe_host_triad(size_t n, int reps, int threads, double* gbs) {
    if (!gbs || n == 0 || reps < 1 || threads < 1) return -1;
    std::vector<double> a(n, 0.0), b(n, 1.0), c(n, 2.0);
    double best = 0.0;
    for (int r = 0; r < reps; ++r) {
        const auto t0 = std::chrono::steady_clock::now();
        std::vector<std::thread> pool;
        for (int w = 0; w < threads; ++w)
            pool.emplace_back([&, w] {
                const size_t lo = n * w / threads, hi = n * (w + 1) / threads;
                for (size_t i = lo; i < hi; ++i) a[i] = b[i] + 3.0 * c[i];
            });
        for (auto& t : pool) t.join();
        const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (s > 0) {
            const double g = 24.0 * (double)n / s / 1e9;
            if (g > best) best = g;
        }
    }
    *gbs = best;
    return a[n / 2] == 7.0 ? 0 : -1;
}

}  // extern "C"
