// Internal launchers, one translation unit per code width (they compile in
// parallel); the C ABI in kvq_abi.cu validates, plans and dispatches to them.
#pragma once

#include <cuda_runtime.h>

#include "kvq_common.cuh"
#include "kvq_fused.cuh"

namespace kvq {

// Heads-per-CTA tiles carried by the library.
constexpr int HEAD_TILES[] = {1, 4, 8};

// Partial kernel over a planned Problem; returns the launch's cudaError_t.
template <int BITS>
cudaError_t launch_partial(const Problem& P, int dtype, int head_dim, int ht, float* part_o,
                           float* part_m, float* part_l, cudaStream_t stream);

template <int BITS>
cudaError_t launch_quantize(const void* w, uint64_t rows, uint32_t head_dim, uint32_t group,
                            int dtype, uint32_t* wq, void* scales, void* biases,
                            const QuantDest& dst, cudaStream_t stream);

template <int BITS>
cudaError_t launch_dequant(const uint32_t* wq, const void* scales, const void* biases,
                           uint64_t rows, uint32_t head_dim, uint32_t group, int dtype,
                           float* out, cudaStream_t stream);

// Register-fragment tensor-core partial kernels: fp16, head_dim 128, ht in
// {4, 8}; 4-bit codes at groups 32/64/128, 8-bit codes at group 64. parts: 3
// (binary32-class combine weights, the default) or 2 (the opt-in fast
// precision)
cudaError_t launch_mma4(const Problem& P, int ht, int group, int bits, int parts, float* part_o,
                        float* part_m, float* part_l, cudaStream_t stream);

// The one-kernel sequence split (kvq_fused.cuh): the 4-bit group-64 split
// stage with the merge, the exchange over the ranks' regions and the final
// merge in its tail; its partials in the region's store, fp16 out through
// F.out. ht in {4, 8}, parts 2 or 3. And its resident CTAs per SM (0 when the
// device cannot be queried).
cudaError_t launch_mma4_fused(const Problem& P, int ht, int parts, const fused::Fused& F,
                              cudaStream_t stream);
int mma4_fused_ctas_per_sm(int ht);

// Merges of n_parts partials; part p's O block starts o_stride floats after
// part p-1's, its m and l ml_stride floats after (stacked partials:
// o_stride = rows * head_dim, ml_stride = rows).
cudaError_t launch_merge(const float* part_o, const float* part_m, const float* part_l,
                         uint32_t n_parts, uint32_t rows, uint32_t head_dim, uint64_t o_stride,
                         uint64_t ml_stride, int out_dtype, void* out, cudaStream_t stream);

cudaError_t launch_merge_partial(const float* part_o, const float* part_m, const float* part_l,
                                 uint32_t n_parts, uint32_t rows, uint32_t head_dim,
                                 float* out_o, float* out_m, float* out_l, cudaStream_t stream);

// 5th-generation tensor-core (tcgen05) partial kernel: fp16, 4-bit, head_dim
// 128, group 64, ht in {4, 8}; and its resident CTAs per SM.
cudaError_t launch_umma4(const Problem& P, int ht, float* part_o, float* part_m, float* part_l,
                         cudaStream_t stream);
int umma4_ctas_per_sm(int ht);

// The warp-specialised tensor-memory kernel (fp16, 4-bit, head_dim 128,
// group 64, ht in {4, 8}): `grid` persistent CTAs, one per SM at most, walk the
// Problem's b_rows x n_kv_heads x head_tiles x n_splits work items.
cudaError_t launch_tmem4(const Problem& P, int ht, uint32_t grid, float* part_o, float* part_m,
                         float* part_l, cudaStream_t stream);
// Positions per tile of that kernel (its split chunks are multiples of it).
int tmem4_tile_positions();

// Resident tensor-core CTAs per SM for (ht, group) on the current device,
// and the device's SM count (both cached per device; fixed fallbacks when the
// device cannot be queried).
int mma4_ctas_per_sm(int ht, int group, int bits);
int sm_count();
// Positions per stage of the register-fragment kernels (split chunks are
// multiples of it).
int mma4_stage_positions();

}  // namespace kvq
