// The kv_attention operator with its seven fault seams as one CUDA source --
// TEST INFRASTRUCTURE ONLY (the CUDA mutation battery), never product code.
//
// The reference scores its verifier by mutation: an fp32 port of the
// operator whose keyword seams switch one fault on at a time
// (kernelverify/reference/native_kernels.py:168-221, catalogue entries
// kernelverify/mutation/catalogue.py:153-166), run over the 400-case battery
// (kernelverify/battery/core.py:253-329). This file is that port written for
// the GPU, each fault a compile-time flag of its own kernel instantiation, so
// the battery can ask whether the oracle catches the same faults when they
// happen on the device. The same functions compile for the host as well
// (`kvq_seams_decode` with on_device = 0), which lets a machine without a GPU
// check the source's arithmetic against the reference's recorded verdicts.
//
// Arithmetic follows the numpy port operation by operation: every multiply
// and add is rounded on its own (the device build is compiled without FMA
// contraction, and the device side spells the roundings out), dequantization
// is `scale * code + bias` at fp32, the scores are scaled after the dot
// product, and the softmax divides by the sum of its exponentials. The fp16
// faults round exactly where numpy's float16 arithmetic rounds: a half product
// is the exact product rounded to half, a half sum is the float sum rounded to
// half. Layout: the reference's shared cache (q [B, H, DH]; artefacts
// [HKV, T, ...] as the canonical quantizer packs them; new_k / new_v
// [B, HKV, DH]; out [B, H, DH]).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <vector>

#define HD __host__ __device__

namespace seams {

// The seams (kernelverify/reference/native_kernels.py:168-221).
enum : int {
    SCORES_F16 = 1,           // scores_dtype=float16: scores rounded to half before the softmax
    ACCUM_F16 = 2,            // accum_dtype=float16: the combine accumulated in half
    ACCUM_F16_SEQ = 4,        // accum_dtype=float16-seq: the same as a running sum
    K_SCALES_ROTATED = 8,     // every K group reads its neighbour's scale and bias
    V_BIAS_DROPPED = 16,      // V dequantized without its bias
    NEW_ENTRY_SKIPPED = 32,   // the step's own K/V left out of the softmax and the combine
    DHEAD_SCALE_DROPPED = 64, // scores not multiplied by 1/sqrt(head_dim)
};

constexpr int kMaxT = 8192;   // (T + 1) fp32 scores in a CTA's static shared-memory budget
constexpr int kThreads = 128;

struct Args {
    const void* q;
    const uint32_t* k_wq;
    const void* k_scales;
    const void* k_biases;
    const uint32_t* v_wq;
    const void* v_scales;
    const void* v_biases;
    const void* new_k;
    const void* new_v;
    void* out;
    int b_rows, n_heads, n_kv_heads, t_cached, head_dim, bits, group;
};

HD inline float mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

HD inline float add_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}

HD inline float sub_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}

// a float rounded to the nearest half, read back as a float
HD inline float to_half(float x) { return __half2float(__float2half_rn(x)); }

template <typename T>
HD inline float load(const void* p, size_t i) {
    if constexpr (sizeof(T) == 2)
        return __half2float(reinterpret_cast<const __half*>(p)[i]);
    else
        return reinterpret_cast<const float*>(p)[i];
}

template <typename T>
HD inline void store(void* p, size_t i, float v) {
    if constexpr (sizeof(T) == 2)
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        reinterpret_cast<float*>(p)[i] = v;
}

// Code i of a row: the contiguous little-endian stream, code i at bit i * bits
// (kernelverify/pack/wide_qmv.py:185-201); 3- and 6-bit codes straddle words.
HD inline uint32_t code_at(const uint32_t* row, int i, int bits) {
    const uint32_t bit = (uint32_t)i * (uint32_t)bits, w = bit >> 5, off = bit & 31u;
    uint64_t v = row[w];
    if (off + (uint32_t)bits > 32u) v |= (uint64_t)row[w + 1] << 32;
    return (uint32_t)(v >> off) & ((1u << bits) - 1u);
}

// Element d of artefact row `row` at fp32: scale * code + bias, each rounded
// (kernelverify/schemas/quant_contract.py:107-113). The K-side rotation reads
// group g - 1 (np.roll(scales, 1, axis=1), quant_contract.py:253-256); the
// V-side fault drops the bias (:265-267).
template <typename T, int F, bool IS_K>
HD inline float dequant(const uint32_t* wq, const void* scales, const void* biases, size_t row,
                        int d, const Args& a) {
    const int words = a.head_dim * a.bits / 32, groups = a.head_dim / a.group;
    int g = d / a.group;
    if (IS_K && (F & K_SCALES_ROTATED)) g = (g + groups - 1) % groups;
    const float s = load<T>(scales, row * groups + g);
    const float b = (!IS_K && (F & V_BIAS_DROPPED)) ? 0.0f : load<T>(biases, row * groups + g);
    return add_rn(mul_rn(s, (float)code_at(wq + row * words, d, a.bits)), b);
}

template <int F>
HD inline float finish_score(float dot, int head_dim) {
    const float scale = (F & DHEAD_SCALE_DROPPED) ? 1.0f : 1.0f / sqrtf((float)head_dim);
    const float s = mul_rn(dot, scale);
    return (F & SCORES_F16) ? to_half(s) : s;
}

// Scaled score of cached position t for query row (b, h).
template <typename T, int F>
HD float cached_score(const Args& a, int b, int h, int t) {
    const int hk = h / (a.n_heads / a.n_kv_heads);
    const size_t row = (size_t)hk * a.t_cached + t;
    const size_t qo = ((size_t)b * a.n_heads + h) * a.head_dim;
    float dot = 0.0f;
    for (int d = 0; d < a.head_dim; ++d)
        dot = add_rn(dot, mul_rn(load<T>(a.q, qo + d),
                                 dequant<T, F, true>(a.k_wq, a.k_scales, a.k_biases, row, d, a)));
    return finish_score<F>(dot, a.head_dim);
}

// Scaled score of the step's own key.
template <typename T, int F>
HD float new_score(const Args& a, int b, int h) {
    const int hk = h / (a.n_heads / a.n_kv_heads);
    const size_t qo = ((size_t)b * a.n_heads + h) * a.head_dim;
    const size_t ko = ((size_t)b * a.n_kv_heads + hk) * a.head_dim;
    float dot = 0.0f;
    for (int d = 0; d < a.head_dim; ++d)
        dot = add_rn(dot, mul_rn(load<T>(a.q, qo + d), load<T>(a.new_k, ko + d)));
    return finish_score<F>(dot, a.head_dim);
}

// e^x rounded to fp32 through the double-precision exponential. Each build's
// double exp is within one double ulp of e^x, so both round to the same fp32
// value -- the correctly rounded one -- unless e^x lies within that ulp of an
// fp32 rounding midpoint (a chance near 2^-29 per call): the host and the
// device builds agree bit for bit.
HD inline float exp_rn(float x) { return (float)exp((double)x); }

// exp(s - max) / sum over the n scores, in place.
HD inline void softmax(float* s, int n) {
    float m = s[0];
    for (int i = 1; i < n; ++i) m = fmaxf(m, s[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        s[i] = exp_rn(sub_rn(s[i], m));
        sum = add_rn(sum, s[i]);
    }
    for (int i = 0; i < n; ++i) s[i] = s[i] / sum;
}

// Output element d of row (b, h) from the probabilities p (T cached, then the
// new entry's unless it is skipped). The two half-precision faults compute
// the same running sum: numpy's float16 reduce over the position axis of the
// port's [B, H, T, DH] products accumulates position by position for each
// dim, bit for bit what its float16 accumulate does.
template <typename T, int F>
HD float combine(const Args& a, const float* p, int b, int h, int d) {
    const int hk = h / (a.n_heads / a.n_kv_heads);
    const size_t base = (size_t)hk * a.t_cached;
    float acc = 0.0f;
    for (int t = 0; t < a.t_cached; ++t) {
        const float v = dequant<T, F, false>(a.v_wq, a.v_scales, a.v_biases, base + t, d, a);
        if constexpr ((F & (ACCUM_F16 | ACCUM_F16_SEQ)) != 0)
            acc = to_half(add_rn(acc, to_half(mul_rn(to_half(p[t]), to_half(v)))));
        else
            acc = add_rn(acc, mul_rn(p[t], v));
    }
    if constexpr ((F & NEW_ENTRY_SKIPPED) == 0) {
        const size_t vo = ((size_t)b * a.n_kv_heads + hk) * a.head_dim;
        acc = add_rn(acc, mul_rn(p[a.t_cached], load<T>(a.new_v, vo + d)));
    }
    return acc;
}

template <int F>
HD inline int n_scores(const Args& a) {
    return a.t_cached + ((F & NEW_ENTRY_SKIPPED) ? 0 : 1);
}

// One CTA per query row; the softmax's reductions run on one thread so their
// order is the host build's.
template <typename T, int F>
__global__ void __launch_bounds__(kThreads) seam_kernel(Args a) {
    __shared__ float s[kMaxT + 1];
    const int b = blockIdx.x / a.n_heads, h = blockIdx.x % a.n_heads;
    for (int t = threadIdx.x; t < a.t_cached; t += blockDim.x) s[t] = cached_score<T, F>(a, b, h, t);
    if constexpr ((F & NEW_ENTRY_SKIPPED) == 0)
        if (threadIdx.x == 0) s[a.t_cached] = new_score<T, F>(a, b, h);
    __syncthreads();
    if (threadIdx.x == 0) softmax(s, n_scores<F>(a));
    __syncthreads();
    const size_t o = ((size_t)b * a.n_heads + h) * a.head_dim;
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x)
        store<T>(a.out, o + d, combine<T, F>(a, s, b, h, d));
}

template <typename T, int F>
void seam_host(const Args& a) {
    std::vector<float> s((size_t)a.t_cached + 1);
    for (int b = 0; b < a.b_rows; ++b)
        for (int h = 0; h < a.n_heads; ++h) {
            for (int t = 0; t < a.t_cached; ++t) s[t] = cached_score<T, F>(a, b, h, t);
            if constexpr ((F & NEW_ENTRY_SKIPPED) == 0) s[a.t_cached] = new_score<T, F>(a, b, h);
            softmax(s.data(), n_scores<F>(a));
            const size_t o = ((size_t)b * a.n_heads + h) * a.head_dim;
            for (int d = 0; d < a.head_dim; ++d) store<T>(a.out, o + d, combine<T, F>(a, s.data(), b, h, d));
        }
}

template <typename T, int F>
int run(const Args& a, bool on_device, cudaStream_t stream) {
    if (!on_device) {
        seam_host<T, F>(a);
        return 0;
    }
    seam_kernel<T, F><<<a.b_rows * a.n_heads, kThreads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

template <typename T>
int dispatch(int fault, const Args& a, bool on_device, cudaStream_t stream) {
    switch (fault) {
        case 0: return run<T, 0>(a, on_device, stream);
        case SCORES_F16: return run<T, SCORES_F16>(a, on_device, stream);
        case ACCUM_F16: return run<T, ACCUM_F16>(a, on_device, stream);
        case ACCUM_F16_SEQ: return run<T, ACCUM_F16_SEQ>(a, on_device, stream);
        case K_SCALES_ROTATED: return run<T, K_SCALES_ROTATED>(a, on_device, stream);
        case V_BIAS_DROPPED: return run<T, V_BIAS_DROPPED>(a, on_device, stream);
        case NEW_ENTRY_SKIPPED: return run<T, NEW_ENTRY_SKIPPED>(a, on_device, stream);
        case DHEAD_SCALE_DROPPED: return run<T, DHEAD_SCALE_DROPPED>(a, on_device, stream);
    }
    return -1;
}

}  // namespace seams

// 0 on success, -1 for arguments the seam kernel does not serve, -2 when the
// launch failed. dtype 0: every float input and the output fp16, 1: fp32.
extern "C" int kvq_seams_decode(int on_device, int fault, int dtype, const void* q,
                                const uint32_t* k_wq, const void* k_scales, const void* k_biases,
                                const uint32_t* v_wq, const void* v_scales, const void* v_biases,
                                const void* new_k, const void* new_v, void* out, int b_rows,
                                int n_heads, int n_kv_heads, int t_cached, int head_dim, int bits,
                                int group, void* stream) {
    if (!q || !k_wq || !k_scales || !k_biases || !v_wq || !v_scales || !v_biases || !new_k ||
        !new_v || !out)
        return -1;
    if (b_rows < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads || t_cached < 1 ||
        t_cached > seams::kMaxT || head_dim < 1 || head_dim > 1024 || group < 1 ||
        head_dim % group || (head_dim * bits) % 32 || (dtype != 0 && dtype != 1))
        return -1;
    if (bits != 2 && bits != 3 && bits != 4 && bits != 6 && bits != 8) return -1;
    if ((long long)b_rows * n_heads > 0x7FFFFFFFLL) return -1;
    const seams::Args a{q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, out,
                        b_rows, n_heads, n_kv_heads, t_cached, head_dim, bits, group};
    const auto s = static_cast<cudaStream_t>(stream);
    return dtype == 0 ? seams::dispatch<__half>(fault, a, on_device != 0, s)
                      : seams::dispatch<float>(fault, a, on_device != 0, s);
}
