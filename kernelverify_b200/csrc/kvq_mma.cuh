// Tensor-core partial kernel for fp16 steps over 4-bit caches, head_dim 128.
//
// Data path: one producer warp streams each stage of TP positions -- packed K
// and V codes, K/V scales and biases, six contiguous runs of the cache --
// into a STAGES-deep shared-memory ring with cp.async.bulk (TMA, 1-D) and
// mbarrier transaction counts. Each of the CWARPS consumer warps takes its
// own 16-position block of every stage; each keeps its own online-softmax
// state, and the warps' partials are merged once at the end of the CTA.
//
// Arithmetic (all intermediates fp32 or exact):
//   scores  s[h,t] = scale * sum_g ( k_scale[t,g] * X_g[h,t] + k_bias[t,g] * Qsum_g[h] )
//           X_g[h,t] = sum_{d in g} q[h,d] * code[t,d] on the tensor cores
//           (mma m16n8k16, fp16 operands: q is the fp16 input and codes are
//           small integers, both exact in fp16; products exact, fp32
//           accumulation). The distribution of the per-group dequant over
//           the dot product is a reassociation of the reference's
//           sum_d q_d (s c_d + b) (contract clause C2).
//   combine O[h,d] = sum_t P'[h,t,g] * code[t,d] + sum_t p[h,t] * v_bias[t,g],
//           P' = p * v_scale, carried as three bf16 parts hi + mid + lo that
//           reproduce P' to 2^-23 relative (binary32-class; PARTS = 2 keeps
//           hi + lo, 2^-16, the opt-in fast precision), times the exact bf16
//           codes on the tensor cores (mma m16n8k16 bf16, exact products,
//           fp32 accumulation).
// The MMA shapes are chosen so the score accumulator fragment IS the
// combine's B fragment: S^T = Q * Codes_K^T puts head h = lane/4 and
// positions {2j, 2j+1} (+8) in lane (h, j), which is exactly where
// out^T = Codes_V^T * P' wants P'[pos, h]. No shuffles between the two.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kvq_common.cuh"

namespace kvq {
namespace mma4 {

#ifndef KVQ_MMA_CWARPS
#define KVQ_MMA_CWARPS 4                     // consumer warps
#endif
constexpr int CWARPS = KVQ_MMA_CWARPS;
constexpr int THREADS = 32 * (CWARPS + 1);   // + one producer warp
constexpr int TP = 16 * CWARPS;              // positions per stage: 16 per consumer warp
#ifndef KVQ_MMA_STAGES
#define KVQ_MMA_STAGES 6                     // depth of the shared-memory stage ring
#endif
constexpr int STAGES = KVQ_MMA_STAGES;
constexpr int DH = 128;
constexpr int ROWB = DH / 2;                 // code bytes per row (4-bit)
constexpr uint32_t WAIT_LIMIT = 1u << 22;    // bounded mbarrier waits
#ifndef KVQ_MMA_MINBLOCKS
#define KVQ_MMA_MINBLOCKS 3                  // resident CTAs per SM the register budget targets
#endif

template <int GROUP, int BITS = 4>
struct Layout {
    static constexpr int G = DH / GROUP;
    static constexpr int RB = DH * BITS / 8;              // code bytes per row
    static constexpr int KC = 0;                          // K codes   [TP][RB]
    static constexpr int VC = KC + TP * RB;               // V codes   [TP][RB]
    static constexpr int KS = VC + TP * RB;               // K scales  [TP][G] fp16
    static constexpr int KB = KS + TP * G * 2;
    static constexpr int VS = KB + TP * G * 2;
    static constexpr int VB = VS + TP * G * 2;
    static constexpr int STAGE = VB + TP * G * 2;         // bytes per stage
    static_assert(STAGE % 128 == 0, "stage size");
    // ring depth: 6- and 8-bit stages are 1.5-2x the bytes, so fewer of them
    // keep three CTAs' rings on an SM with about the same bytes in flight (8-bit
    // at group 32, whose scale runs are the longest, one stage fewer again)
    static constexpr int NST = BITS >= 6 ? (STAGES * 2 + 2) / 3 - (BITS == 8 && G == 4 ? 1 : 0)
                                         : STAGES;
    static constexpr int RING = STAGE * NST;
    // per consumer warp: fp32 [16][G] k_scale, k_bias, v_scale, v_bias - 128 v_scale
    // of the warp's 16-position block
    static constexpr int SCR_WARP = 4 * 16 * G * 4;
    static constexpr int SCR = RING;                       // scratch base
    static constexpr int RING_SCR = RING + CWARPS * SCR_WARP;
    // merge area (reuses the ring once it drains): per warp O[8][128], m[8], l[8], bsum[8][G]
    static constexpr int MERGE = CWARPS * (8 * DH + 8 + 8 + 8 * G) * 4 + 8 * 4;
    static constexpr int BYTES = (RING_SCR > MERGE ? RING_SCR : MERGE) + 2 * NST * 8 + 16;
};

template <int GROUP, int BITS = 4>
constexpr size_t smem_bytes() { return Layout<GROUP, BITS>::BYTES; }

// ---- PTX wrappers ------------------------------------------------------------
__device__ __forceinline__ uint32_t s_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(s_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// A wait that gives up after WAIT_LIMIT polls (each poll itself blocks for a
// bounded, hardware-chosen time) and reports it, so no wait here is endless.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(s_addr(dst)),
        "l"(src), "r"(bytes), "r"(s_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- integer helpers with a fixed instruction choice ------------------------
template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "n"(SEL));
    return d;
}
// (x & mask) | magic in one lop3
template <uint32_t MASK, uint32_t MAGIC>
__device__ __forceinline__ uint32_t and_or(uint32_t x) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "n"(MASK), "n"(MAGIC));
    return d;
}
// ---- exact small-integer conversions ----------------------------------------
__device__ __forceinline__ uint32_t h2_sub1024(uint32_t x) {
    __half2 v = __hsub2(*reinterpret_cast<__half2*>(&x), __half2(__half(1024.0f), __half(1024.0f)));
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t h2_hi_nibble(uint32_t x) {  // (1024 + 16n) / 16 - 64 = n
    __half2 v = __hfma2(*reinterpret_cast<__half2*>(&x), __half2(__half(0.0625f), __half(0.0625f)),
                        __half2(__half(-64.0f), __half(-64.0f)));
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t bf2_sub128(uint32_t x) {
    __nv_bfloat162 v = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&x),
                               __nv_bfloat162(__float2bfloat16(128.0f), __float2bfloat16(128.0f)));
    return *reinterpret_cast<uint32_t*>(&v);
}
// word of 8 nibbles n0..n7 -> four half2 registers (n0,n4) (n1,n5) (n2,n6) (n3,n7)
__device__ __forceinline__ void nibbles_f16(uint32_t w, uint32_t (&h)[4]) {
    h[0] = h2_sub1024(and_or<0x000F000Fu, 0x64006400u>(w));
    h[1] = h2_hi_nibble(and_or<0x00F000F0u, 0x64006400u>(w));
    const uint32_t w8 = w >> 8;
    h[2] = h2_sub1024(and_or<0x000F000Fu, 0x64006400u>(w8));
    h[3] = h2_hi_nibble(and_or<0x00F000F0u, 0x64006400u>(w8));
}
// Bytes K and K+1 of words a and b -> four bf16x2 registers of exact code
// values plus 128: (lo(a.K), lo(b.K)), (hi(a.K), hi(b.K)), (lo(a.K+1),
// lo(b.K+1)), (hi(a.K+1), hi(b.K+1)). One byte permute gathers the four
// bytes as [a.K, a.K+1, b.K, b.K+1]; each nibble pair is then one shift and
// one and-or. The combine subtracts 128 * P' through
// the bias term instead of per code:
//   sum_t P'_t (128 + c_t) + sum_t p_t (b_t - 128 s_t) = sum_t p_t (s_t c_t + b_t).
template <int K>
__device__ __forceinline__ void quad_bf16(uint32_t a, uint32_t b, uint32_t& lo0,
                                          uint32_t& hi0, uint32_t& lo1, uint32_t& hi1) {
    constexpr uint32_t sel = K | ((K + 1) << 4) | ((4 + K) << 8) | ((5 + K) << 12);
    const uint32_t u = prmt<sel>(a, b);
    lo0 = and_or<0x000F000Fu, 0x43004300u>(u);
    hi0 = and_or<0x000F000Fu, 0x43004300u>(u >> 4);
    lo1 = and_or<0x000F000Fu, 0x43004300u>(u >> 8);
    hi1 = and_or<0x000F000Fu, 0x43004300u>(u >> 12);
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void bf16x2_to_f32(uint32_t v, float& lo, float& hi) {
    lo = __uint_as_float(v << 16);
    hi = __uint_as_float(v & 0xFFFF0000u);
}
// Split two fp32 values into two packed bf16x2 parts whose sum reproduces
// them to 16+ significant bits: hi is the truncation (the upper half of the
// fp32 word, taken by a byte permute), the residual x - hi is exact in fp32,
// and lo is that residual rounded to nearest bf16. |x - hi - lo| <= 2^-16 |x|.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& p_hi, uint32_t& p_lo) {
    const uint32_t u0 = __float_as_uint(x0), u1 = __float_as_uint(x1);
    p_hi = prmt<0x7632>(u0, u1);
    // hi back as fp32: low half << 16 (an integer multiply), high half masked
    const float2 r = __ffma2_rn(make_float2(__uint_as_float(p_hi * 65536u),
                                            __uint_as_float(p_hi & 0xFFFF0000u)),
                                make_float2(-1.0f, -1.0f), make_float2(x0, x1));
    p_lo = pack_bf16(r.x, r.y);
}

// Three packed bf16x2 parts: hi and mid are truncations (each residual exact
// in fp32), lo is the second residual rounded to nearest bf16, so
// |x - hi - mid - lo| <= 2^-23 |x|: binary32-class, every intermediate of the
// combine at least as precise as fp32 arithmetic (contract clause C1).
__device__ __forceinline__ void split3(float x0, float x1, uint32_t& p_hi, uint32_t& p_mid,
                                       uint32_t& p_lo) {
    const float2 neg1 = make_float2(-1.0f, -1.0f);
    p_hi = prmt<0x7632>(__float_as_uint(x0), __float_as_uint(x1));
    const float2 r = __ffma2_rn(make_float2(__uint_as_float(p_hi * 65536u),
                                            __uint_as_float(p_hi & 0xFFFF0000u)),
                                neg1, make_float2(x0, x1));
    p_mid = prmt<0x7632>(__float_as_uint(r.x), __float_as_uint(r.y));
    const float2 r2 = __ffma2_rn(make_float2(__uint_as_float(p_mid * 65536u),
                                             __uint_as_float(p_mid & 0xFFFF0000u)),
                                 neg1, r);
    p_lo = pack_bf16(r2.x, r2.y);
}

__device__ __forceinline__ float h2f(const __half* p) { return __half2float(*p); }

// 2^x; flushes results below 2^-126 to zero (those weights are negligible
// beside the running maximum's weight of 1)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// G consecutive fp32 values from shared memory (vector loads)
template <int G>
__device__ __forceinline__ void load_f(const float* p, float (&out)[G]) {
    if constexpr (G == 1) {
        out[0] = *p;
    } else if constexpr (G == 2) {
        const float2 f = *reinterpret_cast<const float2*>(p);
        out[0] = f.x; out[1] = f.y;
    } else if constexpr (G == 4) {
        const float4 f = *reinterpret_cast<const float4*>(p);
        out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
    } else {
        const float4 f = *reinterpret_cast<const float4*>(p);
        const float4 h = *reinterpret_cast<const float4*>(p + 4);
        out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
        out[4] = h.x; out[5] = h.y; out[6] = h.z; out[7] = h.w;
    }
}

// G consecutive fp16 values -> fp32
template <int G>
__device__ __forceinline__ void load_g(const __half* p, float (&out)[G]) {
    if constexpr (G == 1) {
        out[0] = __half2float(*p);
    } else if constexpr (G == 2) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
        out[0] = f.x; out[1] = f.y;
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
    }
}

// The producer: one thread streams the split's stages into the ring, each a
// set of six contiguous runs (K codes, V codes, K/V scales and biases) of the
// stage's rows, rounded up to whole 8-row runs; it waits (bounded) for every
// consumer warp to release a slot before refilling it.
template <int GROUP, int BITS = 4>
__device__ __forceinline__ void produce(const Problem& P, unsigned char* smem, uint64_t* full,
                                        uint64_t* empty, int* err_flag, uint32_t lo, uint32_t hi,
                                        int n_stages, uint64_t rowbase) {
    using Lay = Layout<GROUP, BITS>;
    constexpr int G = Lay::G;
    constexpr int RB = Lay::RB;
    constexpr int NST = Lay::NST;
    const uint64_t pol = evict_first_policy();
    const unsigned char* kw = reinterpret_cast<const unsigned char*>(P.k_wq);
    const unsigned char* vw = reinterpret_cast<const unsigned char*>(P.v_wq);
    const unsigned char* ks = static_cast<const unsigned char*>(P.k_scales);
    const unsigned char* kb = static_cast<const unsigned char*>(P.k_biases);
    const unsigned char* vs = static_cast<const unsigned char*>(P.v_scales);
    const unsigned char* vb = static_cast<const unsigned char*>(P.v_biases);
    for (int s = 0; s < n_stages; ++s) {
        const int slot = s % NST, round = s / NST;
        if (s >= NST && !mbar_wait(&empty[slot], (round - 1) & 1)) {
            atomicExch(err_flag, 1);
            break;
        }
        const uint32_t t0 = lo + s * TP;
        const uint32_t n = min((uint32_t)TP, hi - t0);
        const uint32_t nr = (n + 7) & ~7u;
        const uint64_t row = rowbase + t0;
        unsigned char* st = smem + slot * Lay::STAGE;
        mbar_expect_tx(&full[slot], nr * (2 * RB + 4 * G * 2));
        bulk_g2s(st + Lay::KC, kw + row * RB, nr * RB, &full[slot], pol);
        bulk_g2s(st + Lay::VC, vw + row * RB, nr * RB, &full[slot], pol);
        bulk_g2s(st + Lay::KS, ks + row * G * 2, nr * G * 2, &full[slot], pol);
        bulk_g2s(st + Lay::KB, kb + row * G * 2, nr * G * 2, &full[slot], pol);
        bulk_g2s(st + Lay::VS, vs + row * G * 2, nr * G * 2, &full[slot], pol);
        bulk_g2s(st + Lay::VB, vb + row * G * 2, nr * G * 2, &full[slot], pol);
    }
}

// The CTA partial from the consumer warps' partials the caller left in the
// merge area -- mo [CWARPS][8][DH] (O without the bias term), mm / ml
// [CWARPS][8] (reference point in log2 units, l), mb [CWARPS][8][G] (bias
// sums) -- plus the step's own entry when `with_new`; written as (O, m in
// natural-log units, l) rows of split `split`, NaN when `bad`. Every consumer
// thread calls it after the merge area is complete.
// TAGGED: the partial goes out as 8-byte words, the value's bits in the low
// half and `tag` in the high half, row r of split s at
// tagged[(s * rows + r) * (DH + 2)]: O [DH], then m, then l -- each word
// stored whole (a relaxed 64-bit store), so a reader that finds the tag knows
// that word is this step's without any fence (kvq_fused.cuh).
template <int HT, int GROUP, bool TAGGED = false>
__device__ __forceinline__ void finish_partial(const Problem& P, unsigned char* smem, int tid, int warp,
                                               int lane, uint32_t split, uint32_t b, uint32_t hk,
                                               uint32_t h0, int nh, bool with_new, float scale2,
                                               const int* err_flag, float* __restrict__ part_o,
                                               float* __restrict__ part_m, float* __restrict__ part_l,
                                               uint64_t* __restrict__ tagged = nullptr, uint32_t tag = 0) {
    constexpr int G = DH / GROUP;
    constexpr float LN2 = 0.6931471805599453f;
    const uint32_t H = P.n_heads;
    float* mo = reinterpret_cast<float*>(smem);                 // [CWARPS][8][DH]
    float* mm = mo + CWARPS * 8 * DH;                           // [CWARPS][8]
    float* ml = mm + CWARPS * 8;                                // [CWARPS][8]
    float* mb = ml + CWARPS * 8;                                // [CWARPS][8][G]
    float* snew = mb + CWARPS * 8 * G;                          // [8]
    // the step's own entry: s_new[h] = q[h] . new_k / sqrt(DH), at fp32
    if (with_new && warp == 0) {
        const __half* nk = static_cast<const __half*>(P.new_k) + ((size_t)b * P.n_kv_heads + hk) * DH;
        const __half* qb = static_cast<const __half*>(P.q) + ((size_t)b * H + h0) * DH;
        for (int h = 0; h < nh; ++h) {
            float part = 0.0f;
            for (int d = lane; d < DH; d += 32) part = fmaf(__half2float(qb[h * DH + d]), __half2float(nk[d]), part);
            part = warp_sum(part);
            if (lane == 0) snew[h] = part * scale2;
        }
    }
    named_sync(1, CWARPS * 32);
    // ---- merge the warps (and the new entry) into the CTA partial -----------
    const int bad = *(volatile const int*)err_flag;
    const size_t rows = (size_t)P.b_rows * H;
    const __half* nv = static_cast<const __half*>(P.new_v) + ((size_t)b * P.n_kv_heads + hk) * DH;
    for (int idx = tid; idx < nh * DH; idx += CWARPS * 32) {
        const int h = idx / DH, d = idx % DH, g = d / GROUP;
        float M = with_new ? snew[h] : -INFINITY;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) M = fmaxf(M, mm[w * 8 + h]);
        float o = 0.0f, l = 0.0f;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) {
            const float mw = mm[w * 8 + h];
            if (mw == -INFINITY) continue;
            const float e = ex2(mw - M);
            o = fmaf(mo[(w * 8 + h) * DH + d] + mb[(w * 8 + h) * G + g], e, o);
            l = fmaf(ml[w * 8 + h], e, l);
        }
        if (with_new) {
            const float e = ex2(snew[h] - M);
            o = fmaf(__half2float(nv[d]), e, o);
            l += e;
        }
        const size_t row = split * rows + (size_t)b * H + h0 + h;
        if constexpr (TAGGED) {
            uint64_t* w = tagged + row * (DH + 2);
            const uint64_t hi = (uint64_t)tag << 32;
            const auto word = [&](float v) { return hi | __float_as_uint(bad ? __int_as_float(0x7fc00000) : v); };
            // no compiler barrier: nothing else this thread does is ordered
            // against these words (the tags carry their validity)
            asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(w + d), "l"(word(o)));
            if (d == 0) {
                asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(w + DH), "l"(word(M * LN2)),
                             "l"(word(l)));
            }
        } else {
            part_o[row * DH + d] = bad ? __int_as_float(0x7fc00000) : o;
            if (d == 0) {
                part_m[row] = bad ? __int_as_float(0x7fc00000) : M * LN2;  // natural-log units
                part_l[row] = bad ? __int_as_float(0x7fc00000) : l;
            }
        }
    }
}

// -----------------------------------------------------------------------------
template <int HT, int GROUP, int PARTS>
__global__ void __launch_bounds__(THREADS, GROUP == 32 ? 2 : KVQ_MMA_MINBLOCKS)
partial_kernel(Problem P, float* __restrict__ part_o, float* __restrict__ part_m,
               float* __restrict__ part_l) {
    using Lay = Layout<GROUP>;
    constexpr int G = Lay::G;
    constexpr int KSG = GROUP / 16;     // K-side k-steps per group
    constexpr int WPG = GROUP / 32;     // K-side words per lane, row and group
    constexpr int MTG = GROUP / 16;     // V-side M-tiles (16 dims) per group
    constexpr int MT = DH / 16;         // V-side M-tiles
    constexpr int VBYTES = GROUP / 16;  // V-side bytes per lane, row and group
    constexpr float L2E = 1.4426950408889634f;
    const float scale2 = P.scale * L2E;   // scores are kept in log2 units

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (Lay::RING_SCR > Lay::MERGE ? Lay::RING_SCR : Lay::MERGE));
    uint64_t* empty = full + STAGES;
    int* err_flag = reinterpret_cast<int*>(empty + STAGES);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t split = blockIdx.x;
    const uint32_t hk = blockIdx.y / P.head_tiles;
    const uint32_t tile_h = blockIdx.y % P.head_tiles;
    const uint32_t b = blockIdx.z;
    const uint32_t h0 = hk * P.r + tile_h * HT;
    const int nh = min(HT, (int)(P.r - tile_h * HT));
    const uint32_t H = P.n_heads;

    uint32_t len = P.t_cached;
    if (P.seq_lens != nullptr) len = min((uint32_t)max(P.seq_lens[b], 0), P.t_cached);
    const uint32_t end = min(P.t_end, len);
    const uint32_t lo = P.t_begin + split * P.chunk;
    const uint32_t hi = min(end, lo + P.chunk);
    const int n_stages = hi > lo ? (int)((hi - lo + TP - 1) / TP) : 0;
    const bool with_new = P.has_new_entry && split == P.n_splits - 1;
    const uint64_t rowbase = (uint64_t)b * P.cache_batch_stride + (uint64_t)hk * P.t_stride;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);          // the producer's arrive + the stage's bytes
            mbar_init(&empty[s], CWARPS);    // every consumer warp releases every stage
        }
        *err_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == CWARPS) {
        // ---------------- producer: stream stages into the ring ----------------
        if (lane == 0) produce<GROUP>(P, smem, full, empty, err_flag, lo, hi, n_stages, rowbase);
    } else {
        // ---------------- consumers --------------------------------------------
        const int r = lane >> 2, j = lane & 3;
        const int qh = HT == 4 ? (r & 3) : r;          // head of this lane's score row
        const int half = r >> 2;                       // HT = 4: which n-tile the lane keeps
        constexpr int NS = HT == 4 ? 2 : 4;            // scores a lane keeps per block
        const __half* q = static_cast<const __half*>(P.q) + ((size_t)b * H + h0 + qh) * DH;
        const bool qvalid = qh < nh;
        // Q as the K-side A fragment: virtual k (2j,2j+1 | 2j+8,2j+9) of k-step
        // (g, 2wi + half) <-> dims d0 + (0,4 | 1,5) or d0 + (2,6 | 3,7), with
        // d0 = 2 * (g*GROUP/2 + j*GROUP/8 + 4*wi), matching nibbles_f16's pairs.
        uint32_t qa[G][KSG][2];
        float qsum[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float acc = 0.0f;  // this lane's quarter of the group; the other three follow
#pragma unroll
            for (int wi = 0; wi < WPG; ++wi) {
                const int d0 = 2 * (g * (GROUP / 2) + j * (GROUP / 8) + 4 * wi);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int e = d0 + 2 * half;
                    __half2 x0 = qvalid ? __halves2half2(q[e + 0], q[e + 4]) : __half2(0, 0);
                    __half2 x1 = qvalid ? __halves2half2(q[e + 1], q[e + 5]) : __half2(0, 0);
                    acc += __low2float(x0) + __high2float(x0) + __low2float(x1) + __high2float(x1);
                    qa[g][2 * wi + half][0] = *reinterpret_cast<uint32_t*>(&x0);
                    qa[g][2 * wi + half][1] = *reinterpret_cast<uint32_t*>(&x1);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            qsum[g] = acc;
        }

        float m_run = -INFINITY, l_part = 0.0f;
        float bsum[G];
        float oacc[MT][4];
#pragma unroll
        for (int g = 0; g < G; ++g) bsum[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < MT; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;

        // K-side load pattern: lane (nB = r, jB = j) loads row pi(nB) of each
        // 8-position n-tile, pi(n) = (n >> 1) + 4 (n & 1).
        const int krow = (r >> 1) + 4 * (r & 1);

        // Every consumer warp takes every stage: warp w owns the 16-position
        // block w of each 64-position stage. Waiting on every stage in order
        // keeps each warp at most one phase ahead of each barrier, which the
        // parity-based waits require.
        for (int s = 0; s < n_stages; ++s) {
            const int slot = s % STAGES, round = s / STAGES;
            if (!mbar_wait(&full[slot], round & 1)) {
                atomicExch(err_flag, 1);
                break;
            }
            unsigned char* st = smem + slot * Lay::STAGE;
            const uint32_t t0 = lo + s * TP;
            const int blk = warp;
            const int nvalid = (int)min((uint32_t)TP, hi - t0);
            if (nvalid <= blk * 16) {          // no live position in this warp's block
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                continue;
            }

            // fp32 copies of the block's scales and biases, converted once (every
            // score row and P' part reuses them), per position [k_scale (G) |
            // k_bias (G)] with the score scale log2(e)/sqrt(DH) folded in, and
            // [v_scale (G) | v_bias - 128 v_scale (G)]; positions past the
            // logical end get zero V scale and bias so their zero weights meet
            // finite values only.
            float* scr = reinterpret_cast<float*>(smem + Lay::SCR + warp * Lay::SCR_WARP);
            {
                const __half* kss = reinterpret_cast<const __half*>(st + Lay::KS) + blk * 16 * G;
                const __half* kbs = reinterpret_cast<const __half*>(st + Lay::KB) + blk * 16 * G;
                const __half* vss = reinterpret_cast<const __half*>(st + Lay::VS) + blk * 16 * G;
                const __half* vbs = reinterpret_cast<const __half*>(st + Lay::VB) + blk * 16 * G;
                const int nv_blk = nvalid - blk * 16;
                for (int i = lane; i < 16 * G; i += 32) {
                    const int pos = i / G, g = i % G;
                    const bool live = pos < nv_blk;
                    const float vsv = live ? __half2float(vss[i]) : 0.0f;
                    const float vbv = live ? __half2float(vbs[i]) : 0.0f;
                    scr[pos * 2 * G + g] = __half2float(kss[i]) * scale2;
                    scr[pos * 2 * G + G + g] = __half2float(kbs[i]) * scale2;
                    scr[16 * 2 * G + pos * 2 * G + g] = vsv;
                    scr[16 * 2 * G + pos * 2 * G + G + g] = fmaf(vsv, -128.0f, vbv);
                }
                __syncwarp();
            }
            const float* kscr = scr;                 // [16][2G]
            const float* vscr = scr + 16 * 2 * G;    // [16][2G]
            {
                // ---- scores of 16 positions, log2 units. The K-side MMAs give
                // lane (r, j) head qh at positions j, j+4 (n-tile 0) and 8+j,
                // 12+j (n-tile 1). HT = 8: the lane keeps all four. HT = 4: rows
                // r and r+4 carry the same head, so the lane keeps n-tile `half`
                // only and the two halves share the block's scalar work.
                float sc[NS];
                float xs[G][2];
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const unsigned char* rowp = st + Lay::KC + (blk * 16 + nt * 8 + krow) * ROWB;
                    float x[G][4];
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        x[g][0] = x[g][1] = x[g][2] = x[g][3] = 0.0f;
                        uint32_t w[WPG];
                        const uint32_t* src = reinterpret_cast<const uint32_t*>(
                            rowp + g * (GROUP / 2) + j * (GROUP / 8));
#pragma unroll
                        for (int wi = 0; wi < WPG; ++wi) w[wi] = src[wi];
#pragma unroll
                        for (int wi = 0; wi < WPG; ++wi) {
                            uint32_t hcodes[4];
                            nibbles_f16(w[wi], hcodes);
                            mma_f16(x[g], qa[g][2 * wi][0], 0u, qa[g][2 * wi][1], 0u, hcodes[0],
                                    hcodes[1]);
                            mma_f16(x[g], qa[g][2 * wi + 1][0], 0u, qa[g][2 * wi + 1][1], 0u,
                                    hcodes[2], hcodes[3]);
                        }
                    }
                    if constexpr (HT == 4) {
#pragma unroll
                        for (int g = 0; g < G; ++g)
#pragma unroll
                            for (int c = 0; c < 2; ++c)
                                xs[g][c] = (nt == 0 || half) ? x[g][c] : xs[g][c];
                    } else {
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            const int lpos = nt * 8 + j + 4 * c;
                            float kf[2 * G];
                            load_f<2 * G>(kscr + lpos * 2 * G, kf);
                            float acc = 0.0f;
#pragma unroll
                            for (int g = 0; g < G; ++g) acc = fmaf(kf[g], x[g][c], fmaf(kf[G + g], qsum[g], acc));
                            sc[nt * 2 + c] = blk * 16 + lpos < nvalid ? acc : -INFINITY;
                        }
                    }
                }
                if constexpr (HT == 4) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const int lpos = half * 8 + j + 4 * c;
                        float kf[2 * G];
                        load_f<2 * G>(kscr + lpos * 2 * G, kf);
                        float acc = 0.0f;
#pragma unroll
                        for (int g = 0; g < G; ++g) acc = fmaf(kf[g], xs[g][c], fmaf(kf[G + g], qsum[g], acc));
                        sc[c] = blk * 16 + lpos < nvalid ? acc : -INFINITY;
                    }
                }

                // ---- online softmax with lazy rescaling: the reference point
                // m_run moves only when a head's block max exceeds it by more
                // than 2^8, so weights stay <= 256 and O rarely needs rescaling
                float mx = sc[0];
#pragma unroll
                for (int i = 1; i < NS; ++i) mx = fmaxf(mx, sc[i]);
                if (__any_sync(0xffffffffu, mx > m_run + 8.0f)) {
                    // some head's scores outgrew its reference point: take the
                    // head's block max over its lanes and move the point
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                    if constexpr (HT == 4) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const bool grow = mx > m_run + 8.0f;
                    const float m_new = grow ? mx : m_run;
                    const float alpha = ex2(m_run - m_new);   // 0 on the first block, 1 if unchanged
                    m_run = m_new;
                    l_part *= alpha;
#pragma unroll
                    for (int g = 0; g < G; ++g) bsum[g] *= alpha;
                    // O columns belong to heads (2j, 2j+1) (mod 4 when HT = 4): their
                    // alphas live in the lanes whose score row is that head.
                    const int c0h = HT == 4 ? ((2 * j) & 3) : 2 * j;
                    const float2 a01 = make_float2(__shfl_sync(0xffffffffu, alpha, 4 * c0h),
                                                   __shfl_sync(0xffffffffu, alpha, 4 * (c0h + 1)));
#pragma unroll
                    for (int i = 0; i < MT; ++i) {
                        const float2 u = __fmul2_rn(make_float2(oacc[i][0], oacc[i][1]), a01);
                        const float2 v = __fmul2_rn(make_float2(oacc[i][2], oacc[i][3]), a01);
                        oacc[i][0] = u.x; oacc[i][1] = u.y; oacc[i][2] = v.x; oacc[i][3] = v.y;
                    }
                }
                float e[NS];
#pragma unroll
                for (int i = 0; i < NS; ++i) e[i] = ex2(sc[i] - m_run);
                if constexpr (HT == 4) {
                    l_part += e[0] + e[1];
                } else {
                    l_part += (e[0] + e[1]) + (e[2] + e[3]);
                }

                // ---- combine --------------------------------------------------
                // V scale and folded bias of the lane's own positions
                float vsf[NS][G], vbf[NS][G];
#pragma unroll
                for (int i = 0; i < NS; ++i) {
                    const int lpos = HT == 4 ? half * 8 + j + 4 * i : (i >> 1) * 8 + j + 4 * (i & 1);
                    float vf[2 * G];
                    load_f<2 * G>(vscr + lpos * 2 * G, vf);
#pragma unroll
                    for (int g = 0; g < G; ++g) { vsf[i][g] = vf[g]; vbf[i][g] = vf[G + g]; }
                }
                // B fragments (k rows 2j, 2j+1 <-> positions j, j+4; 2j+8, 2j+9
                // <-> 8+j, 12+j; column r): bf0/bf1 for the first MMA of a tile,
                // bs0/bs1 for the second (HT = 8 only).
                uint32_t bf0[G], bf1[G], bs0[G], bs1[G], bt0[G], bt1[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    // bias with the codes' +128 offset folded in: b - 128 s
                    float acc = bsum[g];
#pragma unroll
                    for (int i = 0; i < NS; ++i) acc = fmaf(e[i], vbf[i][g], acc);
                    bsum[g] = acc;
                    if constexpr (HT == 4) {
                        // column r < 4: hi of head r; column r >= 4: lo of head r-4.
                        // The lane has its half's two positions; the other two come
                        // from the partner lane r^4 (lane ^ 16), which holds the
                        // same head: one exchange carries what each side lacks.
                        const float2 v = __fmul2_rn(make_float2(e[0], e[1]), make_float2(vsf[0][g], vsf[1][g]));
                        uint32_t hi, mid, lo;
                        if constexpr (PARTS == 3) {
                            split3(v.x, v.y, hi, mid, lo);
                        } else {
                            split2(v.x, v.y, hi, mid);
                            lo = 0u;
                        }
                        // first MMA: hi (columns 0..3) and mid (or lo at PARTS = 2,
                        // columns 4..7); second MMA (PARTS = 3): lo in columns 0..3
                        const uint32_t recv = __shfl_xor_sync(0xffffffffu, half ? hi : mid, 16);
                        bf0[g] = half ? recv : hi;
                        bf1[g] = half ? mid : recv;
                        if constexpr (PARTS == 3) {
                            const uint32_t recv_lo = __shfl_xor_sync(0xffffffffu, lo, 16);
                            bs0[g] = half ? 0u : lo;
                            bs1[g] = half ? 0u : recv_lo;
                        } else {
                            bs0[g] = bs1[g] = 0u;
                        }
                        bt0[g] = bt1[g] = 0u;
                    } else {
                        const float2 v01 = __fmul2_rn(make_float2(e[0], e[1]), make_float2(vsf[0][g], vsf[1][g]));
                        const float2 v23 = __fmul2_rn(make_float2(e[2], e[3]), make_float2(vsf[2][g], vsf[3][g]));
                        if constexpr (PARTS == 3) {
                            split3(v01.x, v01.y, bf0[g], bs0[g], bt0[g]);
                            split3(v23.x, v23.y, bf1[g], bs1[g], bt1[g]);
                        } else {
                            split2(v01.x, v01.y, bf0[g], bs0[g]);
                            split2(v23.x, v23.y, bf1[g], bs1[g]);
                            bt0[g] = bt1[g] = 0u;
                        }
                    }
                }
                // A fragments: V codes^T, rows = dims, cols = positions
                // (k 2j, 2j+1 <-> pos j, j+4; 2j+8, 2j+9 <-> 8+j, 12+j).
                const int p0 = blk * 16 + j;
                const unsigned char* vrow = st + Lay::VC;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int boff = g * (GROUP / 2) + r * VBYTES;
                    constexpr int NW = (VBYTES + 3) / 4;
                    uint32_t wA[NW], wB[NW], wC[NW], wD[NW];
#pragma unroll
                    for (int k = 0; k < NW; ++k) {
                        if constexpr (VBYTES >= 4) {
                            wA[k] = *reinterpret_cast<const uint32_t*>(vrow + (p0) * ROWB + boff + 4 * k);
                            wB[k] = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 4) * ROWB + boff + 4 * k);
                            wC[k] = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 8) * ROWB + boff + 4 * k);
                            wD[k] = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 12) * ROWB + boff + 4 * k);
                        } else {
                            wA[k] = *reinterpret_cast<const uint16_t*>(vrow + (p0) * ROWB + boff);
                            wB[k] = *reinterpret_cast<const uint16_t*>(vrow + (p0 + 4) * ROWB + boff);
                            wC[k] = *reinterpret_cast<const uint16_t*>(vrow + (p0 + 8) * ROWB + boff);
                            wD[k] = *reinterpret_cast<const uint16_t*>(vrow + (p0 + 12) * ROWB + boff);
                        }
                    }
                    // A fragments of M-tile ii: (a0, a1) from rows (j, j+4) and
                    // (a2, a3) from rows (8+j, 12+j), byte ii of the lane's chunk
                    uint32_t fa[MTG][4];
#pragma unroll
                    for (int ii = 0; ii < MTG; ii += 2) {
                        const int wi = ii >> 2;
                        if constexpr (MTG >= 2) {
                            if ((ii & 3) == 0) {
                                quad_bf16<0>(wA[wi], wB[wi], fa[ii][0], fa[ii][1], fa[ii + 1][0], fa[ii + 1][1]);
                                quad_bf16<0>(wC[wi], wD[wi], fa[ii][2], fa[ii][3], fa[ii + 1][2], fa[ii + 1][3]);
                            } else {
                                quad_bf16<2>(wA[wi], wB[wi], fa[ii][0], fa[ii][1], fa[ii + 1][0], fa[ii + 1][1]);
                                quad_bf16<2>(wC[wi], wD[wi], fa[ii][2], fa[ii][3], fa[ii + 1][2], fa[ii + 1][3]);
                            }
                        }
                    }
#pragma unroll
                    for (int ii = 0; ii < MTG; ++ii) {
                        // a0: (dim row r, pos j, j+4); a1: (row r+8 = high nibble);
                        // a2/a3: the same for positions 8+j, 12+j
                        float (&acc)[4] = oacc[g * MTG + ii];
                        mma_bf16(acc, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bf0[g], bf1[g]);
                        if constexpr (HT == 8 || PARTS == 3)
                            mma_bf16(acc, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bs0[g], bs1[g]);
                        if constexpr (HT == 8 && PARTS == 3)
                            mma_bf16(acc, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bt0[g], bt1[g]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- warp partial: reduce l and bias sums over the 4 lanes of a head --
        l_part += __shfl_xor_sync(0xffffffffu, l_part, 1);
        l_part += __shfl_xor_sync(0xffffffffu, l_part, 2);
        if constexpr (HT == 4) l_part += __shfl_xor_sync(0xffffffffu, l_part, 16);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            bsum[g] += __shfl_xor_sync(0xffffffffu, bsum[g], 1);
            bsum[g] += __shfl_xor_sync(0xffffffffu, bsum[g], 2);
            if constexpr (HT == 4) bsum[g] += __shfl_xor_sync(0xffffffffu, bsum[g], 16);
        }
        if constexpr (HT == 4) {
            // columns 4..7 carry the mid (or lo) parts of heads 0..3: fold them in
#pragma unroll
            for (int i = 0; i < MT; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) oacc[i][c] += __shfl_xor_sync(0xffffffffu, oacc[i][c], 2);
        }
        named_sync(1, CWARPS * 32);  // every consumer is done with the ring
        float* mo = reinterpret_cast<float*>(smem);                 // [CWARPS][8][DH]
        float* mm = mo + CWARPS * 8 * DH;                           // [CWARPS][8]
        float* ml = mm + CWARPS * 8;                                // [CWARPS][8]
        float* mb = ml + CWARPS * 8;                                // [CWARPS][8][G]
        if (j == 0 && r < HT) {
            mm[warp * 8 + r] = m_run;
            ml[warp * 8 + r] = l_part;
#pragma unroll
            for (int g = 0; g < G; ++g) mb[(warp * 8 + r) * G + g] = bsum[g];
        }
        const bool writer = HT == 4 ? (j < 2) : true;
        if (writer) {
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int g = i / MTG, ii = i % MTG;
                const int dlo = 2 * (g * (GROUP / 2) + r * VBYTES + ii);
                const int c0 = 2 * j, c1 = 2 * j + 1;
                mo[(warp * 8 + c0) * DH + dlo] = oacc[i][0];
                mo[(warp * 8 + c1) * DH + dlo] = oacc[i][1];
                mo[(warp * 8 + c0) * DH + dlo + 1] = oacc[i][2];
                mo[(warp * 8 + c1) * DH + dlo + 1] = oacc[i][3];
            }
        }
        // the stream is done: the merge after this grid may launch now (it
        // waits for the grid's completion before it reads a partial)
        pdl_launch_dependents();
        finish_partial<HT, GROUP>(P, smem, tid, warp, lane, split, b, hk, h0, nh, with_new, scale2,
                                  err_flag, part_o, part_m, part_l);
    }
    // a failed wait may leave copies in flight into this CTA's shared memory:
    // let the producer wait for them (bounded) before the CTA retires
    __syncthreads();
    if (tid == CWARPS * 32 && *(volatile int*)err_flag) {
        for (int s = 0; s < STAGES && s < n_stages; ++s) {
            const int last = ((n_stages - 1 - s) / STAGES) * STAGES + s;  // last use of slot s
            (void)mbar_wait(&full[s], (last / STAGES) & 1);
        }
    }
}

}  // namespace mma4
}  // namespace kvq
