// Tensor-core partial kernels (fp16 steps, 4-bit caches, head_dim 128).
#include "kvq_launch.h"
#include "kvq_mma.cuh"

namespace kvq {

template <int HT, int GROUP>
static cudaError_t mma4_one(const Problem& P, float* o, float* m, float* l, cudaStream_t stream) {
    constexpr size_t smem = mma4::smem_bytes<GROUP>();
    auto kernel = mma4::partial_kernel<HT, GROUP>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // prefer shared memory over L1 so three CTAs fit on an SM
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    dim3 grid(P.n_splits, P.n_kv_heads * P.head_tiles, P.b_rows);
    kernel<<<grid, mma4::THREADS, smem, stream>>>(P, o, m, l);
    return cudaGetLastError();
}

cudaError_t launch_mma4(const Problem& P, int ht, int group, float* o, float* m, float* l,
                        cudaStream_t stream) {
    if (ht == 4) {
        if (group == 32) return mma4_one<4, 32>(P, o, m, l, stream);
        if (group == 64) return mma4_one<4, 64>(P, o, m, l, stream);
        if (group == 128) return mma4_one<4, 128>(P, o, m, l, stream);
    } else if (ht == 8) {
        if (group == 32) return mma4_one<8, 32>(P, o, m, l, stream);
        if (group == 64) return mma4_one<8, 64>(P, o, m, l, stream);
        if (group == 128) return mma4_one<8, 128>(P, o, m, l, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace kvq
