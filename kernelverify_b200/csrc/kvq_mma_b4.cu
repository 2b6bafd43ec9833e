// Register-fragment tensor-core partial kernels (fp16 steps, head_dim 128):
// for 4-bit caches the transposed-score kernel (group 64) and the original
// one (groups 32 and 128); for 2-, 3-, 6- and 8-bit caches the byte-code
// kernel (groups 32, 64, 128; at groups 32 and 128 in its 8-column head form).
#include <atomic>

#include "kvq_launch.h"
#include "kvq_mma.cuh"
#include "kvq_mma8.cuh"
#include "kvq_mmat.cuh"

namespace kvq {

constexpr int kMaxDevices = 64;

template <int HT, int GROUP, int PARTS, int BITS>
constexpr auto mma4_kernel() {
    if constexpr (BITS != 4)
        return mma4::partial_kernel_tb<HT, PARTS, BITS, GROUP>;
    else if constexpr (GROUP == 64)
        return mma4::partial_kernel_t<HT, PARTS>;
    else
        return mma4::partial_kernel<HT, GROUP, PARTS>;
}

// The kernel's attributes (dynamic shared memory above 48 KB; a carveout that
// prefers shared memory, so three CTAs fit on an SM), set once per device so
// that later launches, captured ones included, make no attribute calls.
template <int HT, int GROUP, int PARTS, int BITS>
static cudaError_t mma4_prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < kMaxDevices ? 1ull << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    auto kernel = mma4_kernel<HT, GROUP, PARTS, BITS>();
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mma4::smem_bytes<GROUP, BITS>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

template <int HT, int GROUP, int PARTS, int BITS>
static cudaError_t mma4_one(const Problem& P, float* o, float* m, float* l, cudaStream_t stream) {
    cudaError_t e = mma4_prepare<HT, GROUP, PARTS, BITS>();
    if (e != cudaSuccess) return e;
    dim3 grid(P.n_splits, P.n_kv_heads * P.head_tiles, P.b_rows);
    mma4_kernel<HT, GROUP, PARTS, BITS>()<<<grid, mma4::THREADS, mma4::smem_bytes<GROUP, BITS>(),
                                            stream>>>(P, o, m, l);
    return cudaGetLastError();
}

template <int HT, int GROUP, int BITS>
static int mma4_occupancy() {
    constexpr int PARTS = 3;
    static std::atomic<int> cached[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (mma4_prepare<HT, GROUP, PARTS, BITS>() != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, mma4_kernel<HT, GROUP, PARTS, BITS>(),
                                                      mma4::THREADS,
                                                      mma4::smem_bytes<GROUP, BITS>()) != cudaSuccess)
        return 0;
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

template <int BITS>
static int byte_occupancy_w(int ht, int group) {
    if (group == 64) return ht == 4 ? mma4_occupancy<4, 64, BITS>() : mma4_occupancy<8, 64, BITS>();
    return group == 32 ? mma4_occupancy<8, 32, BITS>() : mma4_occupancy<8, 128, BITS>();
}

static int byte_occupancy(int ht, int group, int bits) {
    switch (bits) {
        case 2: return byte_occupancy_w<2>(ht, group);
        case 3: return byte_occupancy_w<3>(ht, group);
        case 6: return byte_occupancy_w<6>(ht, group);
        default: return byte_occupancy_w<8>(ht, group);
    }
}

int mma4_ctas_per_sm(int ht, int group, int bits) {
    int n = 0;
    if (bits != 4) {
        n = byte_occupancy(ht, group, bits);
    } else if (ht == 4)
        n = group == 32 ? mma4_occupancy<4, 32, 4>() : group == 64 ? mma4_occupancy<4, 64, 4>() : mma4_occupancy<4, 128, 4>();
    else
        n = group == 32 ? mma4_occupancy<8, 32, 4>() : group == 64 ? mma4_occupancy<8, 64, 4>() : mma4_occupancy<8, 128, 4>();
    if (n <= 0) {
        cudaGetLastError();  // a failed query leaves no error behind
        n = group == 32 ? 2 : 3;
    }
    return n;
}

int mma4_stage_positions() { return mma4::TP; }

int sm_count() {
    static std::atomic<int> cached[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return 148;
    }
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 148;
    }
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

// The byte-code kernel: at group 64 in its (group, head)-column form for up
// to 4 query heads per cache head; at groups 32 and 128 always in the
// 8-head-column form (a head tile of 4 has the same single tile when at most
// 4 query heads share a cache head, which is when the planner picks 4).
template <int PARTS, int BITS>
static cudaError_t launch_byte(const Problem& P, int ht, int group, float* o, float* m, float* l,
                               cudaStream_t stream) {
    if (group == 64)
        return ht == 4 ? mma4_one<4, 64, PARTS, BITS>(P, o, m, l, stream)
                       : mma4_one<8, 64, PARTS, BITS>(P, o, m, l, stream);
    if (ht == 4 && P.r > 4) return cudaErrorInvalidValue;
    if (group == 32) return mma4_one<8, 32, PARTS, BITS>(P, o, m, l, stream);
    if (group == 128) return mma4_one<8, 128, PARTS, BITS>(P, o, m, l, stream);
    return cudaErrorInvalidValue;
}

template <int PARTS>
static cudaError_t launch_parts(const Problem& P, int ht, int group, int bits, float* o, float* m,
                                float* l, cudaStream_t stream) {
    if (bits != 4) {
        if (ht != 4 && ht != 8) return cudaErrorInvalidValue;
        switch (bits) {
            case 2: return launch_byte<PARTS, 2>(P, ht, group, o, m, l, stream);
            case 3: return launch_byte<PARTS, 3>(P, ht, group, o, m, l, stream);
            case 6: return launch_byte<PARTS, 6>(P, ht, group, o, m, l, stream);
            case 8: return launch_byte<PARTS, 8>(P, ht, group, o, m, l, stream);
        }
        return cudaErrorInvalidValue;
    }
    if (bits != 4) return cudaErrorInvalidValue;
    if (ht == 4) {
        if (group == 32) return mma4_one<4, 32, PARTS, 4>(P, o, m, l, stream);
        if (group == 64) return mma4_one<4, 64, PARTS, 4>(P, o, m, l, stream);
        if (group == 128) return mma4_one<4, 128, PARTS, 4>(P, o, m, l, stream);
    } else if (ht == 8) {
        if (group == 32) return mma4_one<8, 32, PARTS, 4>(P, o, m, l, stream);
        if (group == 64) return mma4_one<8, 64, PARTS, 4>(P, o, m, l, stream);
        if (group == 128) return mma4_one<8, 128, PARTS, 4>(P, o, m, l, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_mma4(const Problem& P, int ht, int group, int bits, int parts, float* o,
                        float* m, float* l, cudaStream_t stream) {
    return parts == 2 ? launch_parts<2>(P, ht, group, bits, o, m, l, stream)
                      : launch_parts<3>(P, ht, group, bits, o, m, l, stream);
}

// ---- the one-kernel sequence split (4-bit, group 64) ----------------------
template <int HT, int PARTS>
static cudaError_t fused_prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < kMaxDevices ? 1ull << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(mma4::partial_kernel_tf<HT, PARTS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mma4::smem_bytes<64, 4>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(mma4::partial_kernel_tf<HT, PARTS>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

template <int HT, int PARTS>
static cudaError_t fused_one(const Problem& P, const fused::Fused& F, cudaStream_t stream) {
    cudaError_t e = fused_prepare<HT, PARTS>();
    if (e != cudaSuccess) return e;
    dim3 grid(P.n_splits, P.n_kv_heads * P.head_tiles, P.b_rows);
    mma4::partial_kernel_tf<HT, PARTS><<<grid, mma4::THREADS, mma4::smem_bytes<64, 4>(), stream>>>(P, F);
    return cudaGetLastError();
}

cudaError_t launch_mma4_fused(const Problem& P, int ht, int parts, const fused::Fused& F,
                              cudaStream_t stream) {
    if (ht == 4) return parts == 2 ? fused_one<4, 2>(P, F, stream) : fused_one<4, 3>(P, F, stream);
    if (ht == 8) return parts == 2 ? fused_one<8, 2>(P, F, stream) : fused_one<8, 3>(P, F, stream);
    return cudaErrorInvalidValue;
}

int mma4_fused_ctas_per_sm(int ht) {
    int n = 0;
    cudaError_t e = ht == 4 ? fused_prepare<4, 3>() : fused_prepare<8, 3>();
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n, ht == 4 ? mma4::partial_kernel_tf<4, 3> : mma4::partial_kernel_tf<8, 3>, mma4::THREADS,
            mma4::smem_bytes<64, 4>());
    if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // namespace kvq
