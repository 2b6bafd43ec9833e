// 5th-generation tensor-core partial kernels (fp16 steps, 4-bit caches,
// head_dim 128, group 64).
#include <atomic>

#include "kvq_launch.h"
#include "kvq_umma.cuh"

namespace kvq {

namespace {
constexpr int kMaxDevices = 64;

// dynamic shared memory above 48 KB and a carveout that keeps two CTAs on an
// SM, set once per device so later (and captured) launches make no attribute call
template <int HT>
cudaError_t umma_prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < kMaxDevices ? 1ull << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    auto kernel = umma::partial_kernel<HT, 64>;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)umma::smem_bytes<HT, 64>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

template <int HT>
cudaError_t umma_one(const Problem& P, float* o, float* m, float* l, cudaStream_t stream) {
    cudaError_t e = umma_prepare<HT>();
    if (e != cudaSuccess) return e;
    dim3 grid(P.n_splits, P.n_kv_heads * P.head_tiles, P.b_rows);
    umma::partial_kernel<HT, 64><<<grid, umma::THREADS, umma::smem_bytes<HT, 64>(), stream>>>(P, o, m, l);
    return cudaGetLastError();
}

template <int HT>
int umma_occupancy() {
    static std::atomic<int> cached[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (umma_prepare<HT>() != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, umma::partial_kernel<HT, 64>, umma::THREADS,
                                                      umma::smem_bytes<HT, 64>()) != cudaSuccess)
        return 0;
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}
}  // namespace

cudaError_t launch_umma4(const Problem& P, int ht, float* o, float* m, float* l, cudaStream_t stream) {
    if (ht == 4) return umma_one<4>(P, o, m, l, stream);
    if (ht == 8) return umma_one<8>(P, o, m, l, stream);
    return cudaErrorInvalidValue;
}

int umma4_ctas_per_sm(int ht) {
    int n = ht == 4 ? umma_occupancy<4>() : umma_occupancy<8>();
    if (n <= 0) {
        cudaGetLastError();
        n = 1;
    }
    return n;
}

}  // namespace kvq
