// Device helpers shared by the kvq kernels: element types, the packed-code
// stream, exact integer->float conversion.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "kvq_b200.h"

namespace kvq {

// Compile-time loop: f(std::integral_constant<int, I>) for I in [0, N).
template <int N, int I = 0, typename F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        static_for<N, I + 1>(f);
    }
}

// ---------------------------------------------------------------------------
// element types: q/new_k/new_v/out/scales/biases are all one dtype
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
// round to nearest even, as numpy's astype(float16)
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Exact conversion of a small unsigned integer (< 2^23) to fp32: place it in
// the mantissa of 2^23 and subtract 2^23. Two full-rate instructions, exact.
__device__ __forceinline__ float code_to_f32(uint32_t c) {
    return __fsub_rn(__uint_as_float(0x4B000000u | c), 8388608.0f);
}

// Dequantized value of one code: a rounded multiply then a rounded add,
// never contracted into an FMA, so the value is bit-identical to the
// reference's numpy `scales * q + biases` at fp32 for every scale dtype.
__device__ __forceinline__ float dequant(float s, uint32_t c, float b) {
    return __fadd_rn(__fmul_rn(s, code_to_f32(c)), b);
}

// ---------------------------------------------------------------------------
// The packed code stream: one little-endian bit stream per row, code i at
// stream bit i*BITS. A "chunk" is the smallest run of codes that fills whole
// 32-bit words: 16 codes/1 word at 2 bits, 32/3 at 3, 8/1 at 4, 16/3 at 6,
// 4/1 at 8. Chunks never straddle words, codes inside 3- and 6-bit chunks do.
// ---------------------------------------------------------------------------
template <int BITS> struct Chunk;
template <> struct Chunk<2> { static constexpr int CODES = 16, WORDS = 1; };
template <> struct Chunk<3> { static constexpr int CODES = 32, WORDS = 3; };
template <> struct Chunk<4> { static constexpr int CODES = 8, WORDS = 1; };
template <> struct Chunk<6> { static constexpr int CODES = 16, WORDS = 3; };
template <> struct Chunk<8> { static constexpr int CODES = 4, WORDS = 1; };

// Code j (compile-time) of a chunk held in registers w[0..WORDS).
template <int BITS, int J>
__device__ __forceinline__ uint32_t chunk_code(const uint32_t* w) {
    constexpr int bit = J * BITS;
    constexpr int wi = bit >> 5;
    constexpr int sh = bit & 31;
    constexpr uint32_t mask = (1u << BITS) - 1u;
    if constexpr (sh + BITS <= 32) {
        return (w[wi] >> sh) & mask;
    } else {
        return ((w[wi] >> sh) | (w[wi + 1] << (32 - sh))) & mask;
    }
}

// Code i (run-time) of a row: a two-word window, the straddle rule.
template <int BITS>
__device__ __forceinline__ uint32_t row_code(const uint32_t* row, int i) {
    const int bit = i * BITS;
    const int wi = bit >> 5;
    const int sh = bit & 31;
    uint32_t v = row[wi] >> sh;
    if (sh + BITS > 32) v |= row[wi + 1] << (32 - sh);
    return v & ((1u << BITS) - 1u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Programmatic dependent launch (sm_90 and later). A kernel launched right
// after this one with the programmatic-stream-serialization attribute may
// start once every CTA of this grid has executed launch_dependents or exited
// (the tensor-core split stages do so when their stream ends, so the merge
// that follows is launched while their last CTAs finish; triggering earlier
// put merge CTAs beside still-streaming ones and cost more than it hid); the
// dependent calls pdl_wait() before it reads anything this grid
// wrote -- the wait returns once this grid has completed and its memory is
// visible. Both are no-ops for a kernel launched without that attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch-independent description of one decode problem, built on the host
// from kvq_args (plain values; passed to kernels by value).
struct Problem {
    const void* q;
    const uint32_t* k_wq;
    const void* k_scales;
    const void* k_biases;
    const uint32_t* v_wq;
    const void* v_scales;
    const void* v_biases;
    const void* new_k;
    const void* new_v;
    const int32_t* seq_lens;
    uint32_t b_rows, n_heads, n_kv_heads, t_cached, t_stride;
    uint32_t group_size, has_new_entry;
    uint64_t cache_batch_stride;
    uint32_t t_begin, t_end;
    uint32_t chunk;      // positions per split
    uint32_t n_splits;   // splits per row
    uint32_t r;          // query heads per cache head
    uint32_t head_tiles; // ceil(r / HT)
    float scale;         // 1/sqrt(head_dim)
};

// Where quantized input rows land. The input is [seqs, heads, n_new, DH]
// row-major; input row (b, hk, j) is written to output row
//   b * batch_stride + hk * t_stride + pos_b + j,
// pos_b = positions[b] (device) when positions is set, else `position`.
// Rows whose position reaches t_stride are not written. n_new = 0 is a plain
// quantize: input row r is output row r.
struct QuantDest {
    const int32_t* positions;
    uint32_t position;
    uint32_t heads;
    uint32_t n_new;
    uint32_t t_stride;
    uint64_t batch_stride;
};

}  // namespace kvq
