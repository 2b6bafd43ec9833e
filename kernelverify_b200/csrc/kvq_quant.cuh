// The canonical MLX-affine quantizer + packer, and the fp32 dequantizer, on
// the device. Both are bit-exact restatements of the reference's numpy:
// canonical_quantize (kernelverify/schemas/quant_contract.py:60-104),
// pack_codes (kernelverify/pack/wide_qmv.py:185-201) and dequantize
// (kernelverify/schemas/quant_contract.py:107-113). Bit-exactness needs IEEE
// round-to-nearest division (the default without fast-math) and no FMA
// contraction, so every rounding step is spelled with an _rn intrinsic.
#pragma once

#include "kvq_common.cuh"

namespace kvq {

// sign(x) * floor(|x| + 0.5), the add rounded at fp32
__device__ __forceinline__ float round_half_away(float x) {
    return copysignf(floorf(__fadd_rn(fabsf(x), 0.5f)), x);
}

// One thread per (row, group): the group's step and bias, then its codes,
// packed chunk by chunk (a group is a whole number of chunks: groups are
// multiples of 32 codes and a chunk is at most 32).
template <typename T, int BITS>
__global__ void __launch_bounds__(128)
quantize_kernel(const T* __restrict__ w, uint64_t rows, uint32_t head_dim, uint32_t group,
                uint32_t* __restrict__ wq, T* __restrict__ scales, T* __restrict__ biases,
                QuantDest dst) {
    constexpr int CC = Chunk<BITS>::CODES;
    constexpr int CW = Chunk<BITS>::WORDS;
    const uint32_t groups = head_dim / group;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * groups) return;
    const uint64_t row = idx / groups;
    const uint32_t g = (uint32_t)(idx % groups);
    const T* x = w + row * head_dim + (uint64_t)g * group;
    uint64_t orow = row;
    if (dst.n_new) {
        const uint64_t run = row / dst.n_new;
        const uint32_t j = (uint32_t)(row - run * dst.n_new);
        const uint64_t b = run / dst.heads;
        const uint32_t hk = (uint32_t)(run - b * dst.heads);
        const int32_t pos = dst.positions ? dst.positions[b] : (int32_t)dst.position;
        if (pos < 0) return;
        const uint64_t t = (uint64_t)(uint32_t)pos + j;
        if (t >= dst.t_stride) return;
        orow = b * dst.batch_stride + (uint64_t)hk * dst.t_stride + t;
    }

    float lo = INFINITY, hi = -INFINITY;
    for (uint32_t i = 0; i < group; ++i) {
        const float v = to_f32(x[i]);
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
    }
    hi = fmaxf(hi, 0.0f);
    const float top = (float)((1u << BITS) - 1u);
    float step = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), top), 1e-7f);
    const bool low_side = fabsf(lo) > fabsf(hi);
    step = low_side ? step : -step;
    const float edge = low_side ? lo : hi;
    const float n_edge = round_half_away(__fdiv_rn(edge, step));
    const bool degenerate = n_edge == 0.0f;
    if (!degenerate) step = __fdiv_rn(edge, n_edge);
    const float bias = degenerate ? 0.0f : edge;
    scales[orow * groups + g] = from_f32<T>(step);
    biases[orow * groups + g] = from_f32<T>(bias);

    const uint32_t words_per_row = head_dim * BITS / 32;
    uint32_t* out = wq + orow * words_per_row + (uint64_t)g * group * BITS / 32;
    for (uint32_t c = 0; c < group / CC; ++c) {
        uint32_t acc[CW];
#pragma unroll
        for (int i = 0; i < CW; ++i) acc[i] = 0u;
#pragma unroll
        for (int j = 0; j < CC; ++j) {
            const float v = to_f32(x[c * CC + j]);
            float qv = round_half_away(__fdiv_rn(__fsub_rn(v, bias), step));
            qv = fminf(qv, top);
            const uint32_t code = (uint32_t)(int)qv;
            const int bit = j * BITS, wi = bit >> 5, sh = bit & 31;
            acc[wi] |= code << sh;
            if (sh + BITS > 32) acc[wi + 1] |= code >> (32 - sh);
        }
#pragma unroll
        for (int i = 0; i < CW; ++i) out[c * CW + i] = acc[i];
    }
}

// One thread per (row, chunk): CC fp32 values scale*code + bias.
template <typename T, int BITS>
__global__ void __launch_bounds__(128)
dequant_kernel(const uint32_t* __restrict__ wq, const T* __restrict__ scales,
               const T* __restrict__ biases, uint64_t rows, uint32_t head_dim,
               uint32_t group, float* __restrict__ out) {
    constexpr int CC = Chunk<BITS>::CODES;
    constexpr int CW = Chunk<BITS>::WORDS;
    const uint32_t chunks = head_dim / CC;
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * chunks) return;
    const uint64_t row = idx / chunks;
    const uint32_t c = (uint32_t)(idx % chunks);
    const uint32_t groups = head_dim / group;
    const uint32_t g = c * CC / group;
    const float s = to_f32(scales[row * groups + g]);
    const float b = to_f32(biases[row * groups + g]);
    uint32_t w[CW];
    const uint32_t* src = wq + row * (head_dim * BITS / 32) + (uint64_t)c * CW;
#pragma unroll
    for (int i = 0; i < CW; ++i) w[i] = src[i];
    float* dst = out + row * head_dim + (uint64_t)c * CC;
    static_for<CC>([&](auto J) { dst[J.value] = dequant(s, chunk_code<BITS, J.value>(w), b); });
}

}  // namespace kvq
