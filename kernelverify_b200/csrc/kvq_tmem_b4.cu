// The warp-specialised tensor-memory decode kernel (kvq_tmem.cuh): fp16 steps,
// 4-bit caches, head_dim 128, group 64; one persistent CTA per SM.
#include <atomic>

#include "kvq_launch.h"
#include "kvq_tmem.cuh"

namespace kvq {

namespace {
constexpr int kMaxDevices = 64;

// dynamic shared memory above 48 KB, set once per device so later (and
// captured) launches make no attribute call
template <int HT>
cudaError_t tmem_prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < kMaxDevices ? 1ull << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(tmem4::decode_kernel<HT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tmem4::smem_bytes<HT>());
    if (e != cudaSuccess) return e;
    // the warpgroups re-split the registers the CTA launched with: a build
    // whose per-thread count differs would make the softmax warpgroups' request
    // wait forever, so it is never launched
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, tmem4::decode_kernel<HT>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != tmem4::REG_LAUNCH) return cudaErrorInvalidConfiguration;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

template <int HT>
cudaError_t tmem_one(const Problem& P, uint32_t grid, float* o, float* m, float* l, cudaStream_t stream) {
    cudaError_t e = tmem_prepare<HT>();
    if (e != cudaSuccess) return e;
    const uint32_t items = P.b_rows * P.n_kv_heads * P.head_tiles * P.n_splits;
    tmem4::decode_kernel<HT><<<grid, tmem4::THREADS, tmem4::smem_bytes<HT>(), stream>>>(P, items, o, m, l);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_tmem4(const Problem& P, int ht, uint32_t grid, float* o, float* m, float* l,
                         cudaStream_t stream) {
    if (ht == 4) return tmem_one<4>(P, grid, o, m, l, stream);
    if (ht == 8) return tmem_one<8>(P, grid, o, m, l, stream);
    return cudaErrorInvalidValue;
}

int tmem4_tile_positions() { return tmem4::TP; }

}  // namespace kvq
