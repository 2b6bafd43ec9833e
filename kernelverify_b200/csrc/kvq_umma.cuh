// 5th-generation tensor-core partial kernel (tcgen05 / UMMA, accumulators in
// tensor memory) for fp16 steps over 4-bit caches, head_dim 128.
//
// Work unit: one (batch row, cache head, head tile) x one T split, as the
// other partial kernels. The split is streamed in tiles of TP = 128 positions.
//
// Data path per tile:
//   producer warp  cp.async.bulk the tile's K codes, V codes and the four
//                  fp16 scale/bias arrays into a STAGES-deep ring (mbarrier
//                  transaction counts), exactly as the register-MMA kernel.
//   thread t       (one of 128 consumers) owns position t of the tile: it
//                  unpacks the position's 128 K codes into fp16 (exact small
//                  integers) in a K-major shared-memory operand, and its V
//                  codes into bf16 (128 + code, exact) in an MN-major operand.
//   thread 0       issues the tcgen05.mma's:
//                    S[t, n]   = sum_k Kcodes[t, k] * Qg[k, n]        (TMEM cols 0..15)
//                    O[d, n'] += sum_t Vcodes[t, d] * Pparts[t, n']   (TMEM cols 32..)
//                  Qg holds each head's q restricted to one quantization
//                  group (n = g*8 + h), so S gives the per-group dot
//                  products X_g[t, h] the factored dequant needs:
//                    score[t,h] = sum_g k_scale[t,g] X_g[t,h] + k_bias[t,g] Qsum_g[h].
//                  Pparts holds p * v_scale as two bf16 parts (hi, lo) per
//                  (group, head): n' = (g*2 + part)*HT + h. Rows of O whose
//                  dim is outside group g are computed and ignored.
//   thread t       reads its scores back from TMEM (lane t), applies the lazy
//                  online softmax (the running maximum moves only when a
//                  score exceeds it by 2^8; a CTA-wide vote decides), and
//                  writes its row of Pparts; the V-side bias term
//                  sum_t p_t (b_t - 128 s_t) is summed in registers.
// At the end thread t reads O row t (one dim) from TMEM, the per-thread l and
// bias sums are reduced across the CTA, the step's new entry is merged, and
// the partial (O unnormalised, m, l) is written as the other kernels do.
//
// Precision: K-side products fp16 x fp16 are exact and accumulate in fp32;
// the V-side weights carry 2^-16 relative error (two bf16 parts) against
// exact codes; the kernel serves fp16 outputs only.
#pragma once

#include "kvq_mma.cuh"

namespace kvq {
namespace umma {

using mma4::and_or;
using mma4::bulk_g2s;
using mma4::evict_first_policy;
using mma4::ex2;
using mma4::load_g;
using mma4::mbar_arrive;
using mma4::mbar_expect_tx;
using mma4::mbar_init;
using mma4::mbar_wait;
using mma4::named_sync;
using mma4::nibbles_f16;
using mma4::s_addr;
using mma4::split2;

constexpr int TP = 128;                      // positions per tile = consumer threads
constexpr int CTHREADS = TP;
constexpr int THREADS = CTHREADS + 32;       // + one producer warp
constexpr int DH = 128;
constexpr int ROWB = DH / 2;                 // code bytes per row (4-bit)
constexpr int TMEM_COLS = 64;                // S at column 0, O at column 32
constexpr int S_COL = 0;
constexpr int O_COL = 32;
constexpr int N_S = 16;                      // score columns: group * 8 + head
#ifndef KVQ_UMMA_STAGES
#define KVQ_UMMA_STAGES 2
#endif
constexpr int STAGES = KVQ_UMMA_STAGES;

template <int HT, int GROUP>
struct Layout {
    static constexpr int G = DH / GROUP;
    static constexpr int N_O = 2 * G * HT;                // O columns: (group, part, head)
    // ring stage: K codes [TP][64], V codes [TP][64], then k_scale, k_bias,
    // v_scale, v_bias [TP][G] fp16 each
    static constexpr int KC = 0;
    static constexpr int VC = KC + TP * ROWB;
    static constexpr int KS = VC + TP * ROWB;
    static constexpr int KB = KS + TP * G * 2;
    static constexpr int VS = KB + TP * G * 2;
    static constexpr int VB = VS + TP * G * 2;
    static constexpr int STAGE = VB + TP * G * 2;
    static constexpr int RING = STAGE * STAGES;
    // tensor-core operands (no swizzle, 8 x 16-byte core matrices):
    //   AK  K codes fp16, K-major: (pos t, dim chunk c) at (t%8)*16 + (t/8)*2048 + c*128
    //   AV  V codes bf16, MN-major: (pos t, dim chunk c) at the same offset
    //   BQ  Qg fp16, K-major: (column n, dim chunk c) at (n%8)*16 + (n/8)*2048 + c*128
    //   BP  P parts bf16, MN-major: (pos t, column chunk j) at (t%8)*16 + (t/8)*BP_LBO + j*128
    static constexpr int AK = RING;
    static constexpr int AV = AK + TP * DH * 2;
    static constexpr int BQ = AV + TP * DH * 2;
    static constexpr int BP = BQ + N_S * DH * 2;
    static constexpr int BP_LBO = (N_O / 8) * 128;
    static constexpr int MISC = BP + TP * N_O * 2;
    // misc: barriers, TMEM address, flags, reduction scratch
    static constexpr int BAR = MISC;                       // full[S], empty[S], sdone, vdone
    static constexpr int TMEM_ADDR = BAR + (2 * STAGES + 2) * 8;
    static constexpr int ERR = TMEM_ADDR + 4;
    static constexpr int QSUM = ERR + 12;                  // [G][HT] fp32
    static constexpr int RED = QSUM + G * HT * 4;          // [4 warps][HT] fp32
    static constexpr int BYTES = RED + 4 * HT * 4 + 16;
    static_assert(STAGE % 16 == 0 && AK % 128 == 0 && BQ % 128 == 0 && BP % 128 == 0, "alignment");
};

template <int HT, int GROUP>
constexpr size_t smem_bytes() { return Layout<HT, GROUP>::BYTES; }

// ---- tcgen05 wrappers ---------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(dst)),
                 "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Shared-memory matrix descriptor, no swizzle: start, leading-dimension and
// stride-dimension byte offsets (16-byte units), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: fp32 accumulator, A/B both fp16 or both
// bf16, K- or MN-major operands, N and M.
constexpr uint32_t idesc(bool bf16, bool a_mn, bool b_mn, int n, int m) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate)
        : "memory");
}
// arrive on `bar` once every tcgen05.mma this thread issued has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     s_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// CTA-wide OR over the consumer threads (named barrier 1)
__device__ __forceinline__ bool consumers_any(bool pred) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(pred ? 1u : 0u), "r"(CTHREADS)
        : "memory");
    return out != 0;
}

// word of 8 nibbles n0..n7 -> four bf16x2 registers (128+n0, 128+n4),
// (128+n1, 128+n5), (128+n2, 128+n6), (128+n3, 128+n7): exact
__device__ __forceinline__ void nibbles_bf16(uint32_t w, uint32_t (&h)[4]) {
    h[0] = and_or<0x000F000Fu, 0x43004300u>(w);
    h[1] = and_or<0x000F000Fu, 0x43004300u>(w >> 4);
    h[2] = and_or<0x000F000Fu, 0x43004300u>(w >> 8);
    h[3] = and_or<0x000F000Fu, 0x43004300u>(w >> 12);
}

// Within each 8-dim chunk the operands hold dims in the order nibbles_*
// produce them: element e <-> dim 8c + PERM[e].
__device__ __forceinline__ int chunk_dim(int e) { return (e >> 1) + 4 * (e & 1); }

// -----------------------------------------------------------------------------
template <int HT, int GROUP>
__global__ void __launch_bounds__(THREADS, 2)
partial_kernel(Problem P, float* __restrict__ part_o, float* __restrict__ part_m,
               float* __restrict__ part_l) {
    using Lay = Layout<HT, GROUP>;
    constexpr int G = Lay::G;
    constexpr int N_O = Lay::N_O;
    constexpr float L2E = 1.4426950408889634f;
    constexpr float LN2 = 0.6931471805599453f;
    constexpr uint32_t ID_S = idesc(false, false, false, N_S, 128);
    constexpr uint32_t ID_V = idesc(true, true, true, N_O, 128);
    static_assert(G * 8 <= N_S && HT <= 8, "score columns");
    static_assert(N_O <= 32, "O columns");
    const float scale2 = P.scale * L2E;   // scores in log2 units

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* sdone = empty + STAGES;
    uint64_t* vdone = sdone + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::TMEM_ADDR);
    int* err_flag = reinterpret_cast<int*>(smem + Lay::ERR);
    float* qsum_s = reinterpret_cast<float*>(smem + Lay::QSUM);
    float* red = reinterpret_cast<float*>(smem + Lay::RED);

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
    const int n_tiles = hi > lo ? (int)((hi - lo + TP - 1) / TP) : 0;
    const bool with_new = P.has_new_entry && split == P.n_splits - 1;
    const uint64_t rowbase = (uint64_t)b * P.cache_batch_stride + (uint64_t)hk * P.t_stride;
    const __half* qg = static_cast<const __half*>(P.q) + ((size_t)b * H + h0) * DH;

    // ---- setup: barriers, TMEM, the Qg operand and the per-group q sums ------
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);       // thread 0 releases a stage for all consumers
        }
        mbar_init(sdone, 1);
        mbar_init(vdone, 1);
        *err_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid < CTHREADS) {
        // BQ: 16 columns x 16 dim chunks = 256 chunks of 8 fp16, two per thread
        for (int i = tid; i < N_S * (DH / 8); i += CTHREADS) {
            const int n = i / (DH / 8), c = i % (DH / 8);
            const int g = n / 8, h = n % 8;
            const bool live = h < nh && (c * 8) / GROUP == g;
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const __half x0 = live ? qg[h * DH + c * 8 + chunk_dim(e)] : __half(0.0f);
                const __half x1 = live ? qg[h * DH + c * 8 + chunk_dim(e + 1)] : __half(0.0f);
                __half2 v = __halves2half2(x0, x1);
                w[e / 2] = *reinterpret_cast<uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(smem + Lay::BQ + (n % 8) * 16 + (n / 8) * 2048 + c * 128) =
                make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (tid < G * HT) {
            const int g = tid / HT, h = tid % HT;
            float acc = 0.0f;
            if (h < nh)
                for (int d = 0; d < GROUP; ++d) acc += __half2float(qg[h * DH + g * GROUP + d]);
            qsum_s[g * HT + h] = acc;
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == CTHREADS / 32) {
        // ---------------- producer: stream tiles into the ring -----------------
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            const unsigned char* kw = reinterpret_cast<const unsigned char*>(P.k_wq);
            const unsigned char* vw = reinterpret_cast<const unsigned char*>(P.v_wq);
            const unsigned char* ks = static_cast<const unsigned char*>(P.k_scales);
            const unsigned char* kb = static_cast<const unsigned char*>(P.k_biases);
            const unsigned char* vs = static_cast<const unsigned char*>(P.v_scales);
            const unsigned char* vb = static_cast<const unsigned char*>(P.v_biases);
            for (int s = 0; s < n_tiles; ++s) {
                const int slot = s % STAGES, round = s / STAGES;
                if (s >= STAGES && !mbar_wait(&empty[slot], (round - 1) & 1)) {
                    atomicExch(err_flag, 1);
                    break;
                }
                const uint32_t t0 = lo + s * TP;
                const uint32_t n = min((uint32_t)TP, hi - t0);
                const uint32_t nr = (n + 7) & ~7u;
                const uint64_t row = rowbase + t0;
                unsigned char* st = smem + slot * Lay::STAGE;
                mbar_expect_tx(&full[slot], nr * (2 * ROWB + 4 * G * 2));
                bulk_g2s(st + Lay::KC, kw + row * ROWB, nr * ROWB, &full[slot], pol);
                bulk_g2s(st + Lay::VC, vw + row * ROWB, nr * ROWB, &full[slot], pol);
                bulk_g2s(st + Lay::KS, ks + row * G * 2, nr * G * 2, &full[slot], pol);
                bulk_g2s(st + Lay::KB, kb + row * G * 2, nr * G * 2, &full[slot], pol);
                bulk_g2s(st + Lay::VS, vs + row * G * 2, nr * G * 2, &full[slot], pol);
                bulk_g2s(st + Lay::VB, vb + row * G * 2, nr * G * 2, &full[slot], pol);
            }
        }
    } else {
        // ---------------- consumers: thread t owns position t of each tile -----
        const int t = tid;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const uint32_t s_addr_ak = s_addr(smem + Lay::AK), s_addr_av = s_addr(smem + Lay::AV);
        const uint32_t s_addr_bq = s_addr(smem + Lay::BQ), s_addr_bp = s_addr(smem + Lay::BP);
        const int opoff = (t % 8) * 16 + (t / 8) * 2048;   // AK / AV row offset of position t
        float qsum[G][HT];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int h = 0; h < HT; ++h) qsum[g][h] = qsum_s[g * HT + h];

        float m_run[HT], l_part[HT], bsum[G][HT];
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            m_run[h] = -INFINITY;
            l_part[h] = 0.0f;
#pragma unroll
            for (int g = 0; g < G; ++g) bsum[g][h] = 0.0f;
        }
        bool ok = true;

        for (int s = 0; s < n_tiles; ++s) {
            const int slot = s % STAGES, round = s / STAGES;
            if (!mbar_wait(&full[slot], round & 1)) ok = false;
            // every consumer takes the same branch: a failed wait poisons the
            // output but the tile is still walked so every barrier is matched
            const unsigned char* st = smem + slot * Lay::STAGE;
            const int nvalid = (int)min((uint32_t)TP, hi - (lo + s * TP));
            const bool live = t < nvalid;

            // -- K codes of position t -> AK (fp16, exact) --------------------
            {
                const uint4* src = reinterpret_cast<const uint4*>(st + Lay::KC + t * ROWB);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const uint4 w4 = src[q4];
                    const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint32_t hc[4];
                        nibbles_f16(ws[k], hc);
                        *reinterpret_cast<uint4*>(smem + Lay::AK + opoff + (q4 * 4 + k) * 128) =
                            make_uint4(hc[0], hc[1], hc[2], hc[3]);
                    }
                }
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(1, CTHREADS);
            if (t == 0) {
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < DH / 16; ++k)
                    umma(tmem + S_COL, sdesc(s_addr_ak + k * 256, 128, 2048),
                         sdesc(s_addr_bq + k * 256, 128, 2048), ID_S, k > 0 ? 1u : 0u);
                umma_commit(sdone);
            }

            // -- V codes of position t -> AV (bf16 128+code), once the previous
            //    tile's combine no longer reads AV / BP ------------------------
            if (s > 0 && !mbar_wait(vdone, (s - 1) & 1)) ok = false;
            {
                const uint4* src = reinterpret_cast<const uint4*>(st + Lay::VC + t * ROWB);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const uint4 w4 = src[q4];
                    const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint32_t hc[4];
                        nibbles_bf16(ws[k], hc);
                        *reinterpret_cast<uint4*>(smem + Lay::AV + opoff + (q4 * 4 + k) * 128) =
                            make_uint4(hc[0], hc[1], hc[2], hc[3]);
                    }
                }
            }
            // the position's scales and biases (fp32; score scale folded into K's)
            float ksf[G], kbf[G], vsf[G], vbf[G];
            load_g<G>(reinterpret_cast<const __half*>(st + Lay::KS) + t * G, ksf);
            load_g<G>(reinterpret_cast<const __half*>(st + Lay::KB) + t * G, kbf);
            load_g<G>(reinterpret_cast<const __half*>(st + Lay::VS) + t * G, vsf);
            load_g<G>(reinterpret_cast<const __half*>(st + Lay::VB) + t * G, vbf);

            // -- scores of position t from TMEM lane t -------------------------
            if (!mbar_wait(sdone, s & 1)) ok = false;
            tc_fence_after();
            uint32_t xr[16];
            tmem_ld16(tmem + lane_base + S_COL, xr);
            tmem_wait_ld();
            float sc[HT];
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                float acc = 0.0f;
#pragma unroll
                for (int g = 0; g < G; ++g)
                    acc = fmaf(ksf[g], __uint_as_float(xr[g * 8 + h]), fmaf(kbf[g], qsum[g][h], acc));
                sc[h] = live ? acc * scale2 : -INFINITY;
            }

            // -- lazy online softmax: a CTA-wide vote moves the reference ------
            bool grow = false;
#pragma unroll
            for (int h = 0; h < HT; ++h) grow |= sc[h] > m_run[h] + 8.0f;
            if (consumers_any(grow)) {
                float mx[HT];
#pragma unroll
                for (int h = 0; h < HT; ++h) {
                    float v = sc[h];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
                    mx[h] = v;
                }
                if (lane == 0)
#pragma unroll
                    for (int h = 0; h < HT; ++h) red[warp * HT + h] = mx[h];
                named_sync(1, CTHREADS);
                float alpha[HT];
#pragma unroll
                for (int h = 0; h < HT; ++h) {
                    float v = red[h];
#pragma unroll
                    for (int w = 1; w < CTHREADS / 32; ++w) v = fmaxf(v, red[w * HT + h]);
                    const float m_new = v > m_run[h] + 8.0f ? v : m_run[h];
                    alpha[h] = ex2(m_run[h] - m_new);     // 0 on the first tile
                    m_run[h] = m_new;
                    l_part[h] *= alpha[h];
#pragma unroll
                    for (int g = 0; g < G; ++g) bsum[g][h] *= alpha[h];
                }
                named_sync(1, CTHREADS);   // everyone has read `red`
                if (s > 0) {
                    // O (TMEM lane t, columns (g, part, h)) times its head's alpha
#pragma unroll
                    for (int c0 = 0; c0 < N_O; c0 += 16) {
                        uint32_t ov[16];
                        tmem_ld16(tmem + lane_base + O_COL + c0, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha[(c0 + i) % HT]);
                        tmem_st16(tmem + lane_base + O_COL + c0, ov);
                    }
                    tmem_wait_st();
                }
            }
            float e[HT];
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                e[h] = live ? ex2(sc[h] - m_run[h]) : 0.0f;
                l_part[h] += e[h];
            }

            // -- P' = p * v_scale as two bf16 parts -> BP row t; bias sums -----
            {
                uint32_t pw[N_O / 2];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float vs = live ? vsf[g] : 0.0f;
                    const float vb = live ? fmaf(vsf[g], -128.0f, vbf[g]) : 0.0f;
#pragma unroll
                    for (int h = 0; h < HT; h += 2) {
                        uint32_t phi, plo;
                        split2(e[h] * vs, e[h + 1] * vs, phi, plo);
                        pw[((g * 2 + 0) * HT + h) / 2] = phi;
                        pw[((g * 2 + 1) * HT + h) / 2] = plo;
                        bsum[g][h] = fmaf(e[h], vb, bsum[g][h]);
                        bsum[g][h + 1] = fmaf(e[h + 1], vb, bsum[g][h + 1]);
                    }
                }
#pragma unroll
                for (int j = 0; j < N_O / 8; ++j)
                    *reinterpret_cast<uint4*>(smem + Lay::BP + (t % 8) * 16 + (t / 8) * Lay::BP_LBO + j * 128) =
                        make_uint4(pw[4 * j], pw[4 * j + 1], pw[4 * j + 2], pw[4 * j + 3]);
            }
            fence_async_smem();
            tc_fence_before();
            named_sync(1, CTHREADS);
            if (t == 0) {
                mbar_arrive(&empty[slot]);           // the stage is fully read
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < TP / 16; ++k)
                    umma(tmem + O_COL, sdesc(s_addr_av + k * 2 * 2048, 2048, 128),
                         sdesc(s_addr_bp + k * 2 * Lay::BP_LBO, Lay::BP_LBO, 128), ID_V,
                         (s > 0 || k > 0) ? 1u : 0u);
                umma_commit(vdone);
            }
        }
        if (!ok) atomicExch(err_flag, 1);

        // ---- the CTA partial ----------------------------------------------------
        if (n_tiles > 0 && !mbar_wait(vdone, (n_tiles - 1) & 1)) atomicExch(err_flag, 1);
        tc_fence_after();
        float o[N_O];
        if (n_tiles > 0) {
#pragma unroll
            for (int c0 = 0; c0 < N_O; c0 += 16) {
                uint32_t ov[16];
                tmem_ld16(tmem + lane_base + O_COL + c0, ov);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) o[c0 + i] = __uint_as_float(ov[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < N_O; ++i) o[i] = 0.0f;
        }
        // l and bias sums over all positions: warp sums, then across warps
        float* rl = reinterpret_cast<float*>(smem + Lay::AK);          // [4][HT]
        float* rb = rl + 4 * HT;                                         // [4][G][HT]
        float* snew = rb + 4 * G * HT;                                   // [HT]
        named_sync(1, CTHREADS);   // AK is no longer an MMA operand
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            float v = l_part[h];
#pragma unroll
            for (int x = 16; x > 0; x >>= 1) v += __shfl_xor_sync(0xffffffffu, v, x);
            if (lane == 0) rl[warp * HT + h] = v;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float u = bsum[g][h];
#pragma unroll
                for (int x = 16; x > 0; x >>= 1) u += __shfl_xor_sync(0xffffffffu, u, x);
                if (lane == 0) rb[(warp * G + g) * HT + h] = u;
            }
        }
        if (with_new && warp == 0) {
            const __half* nk = static_cast<const __half*>(P.new_k) + ((size_t)b * P.n_kv_heads + hk) * DH;
            for (int h = 0; h < nh; ++h) {
                float part = 0.0f;
                for (int d = lane; d < DH; d += 32) part = fmaf(__half2float(qg[h * DH + d]), __half2float(nk[d]), part);
                part = warp_sum(part);
                if (lane == 0) snew[h] = part * scale2;
            }
        }
        named_sync(1, CTHREADS);
        // thread t holds dim d of every head: O row t <-> dim 8 (t/8) + chunk_dim(t%8)
        const int d = 8 * (t / 8) + chunk_dim(t % 8);
        const int g = d / GROUP;
        const int bad = *(volatile int*)err_flag;
        const size_t rows = (size_t)P.b_rows * H;
        const __half* nv = static_cast<const __half*>(P.new_v) + ((size_t)b * P.n_kv_heads + hk) * DH;
        const float nvd = with_new ? __half2float(nv[d]) : 0.0f;
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            if (h >= nh) break;
            float l = 0.0f, bs = 0.0f;
#pragma unroll
            for (int w = 0; w < CTHREADS / 32; ++w) {
                l += rl[w * HT + h];
                bs += rb[(w * G + g) * HT + h];
            }
            float ov = 0.0f;
#pragma unroll
            for (int gg = 0; gg < G; ++gg)
                if (gg == g) ov = o[(gg * 2 + 0) * HT + h] + o[(gg * 2 + 1) * HT + h];
            ov += bs;
            float M = m_run[h];
            if (with_new) {
                const float sn = snew[h];
                const float Mx = fmaxf(M, sn);
                const float er = M == -INFINITY ? 0.0f : ex2(M - Mx);
                const float en = ex2(sn - Mx);
                ov = fmaf(nvd, en, ov * er);
                l = fmaf(l, er, en);
                M = Mx;
            }
            const size_t row = split * rows + (size_t)b * H + h0 + h;
            part_o[row * DH + d] = bad ? __int_as_float(0x7fc00000) : ov;
            if (t == 0) {
                part_m[row] = bad ? __int_as_float(0x7fc00000) : M * LN2;   // natural-log units
                part_l[row] = bad ? __int_as_float(0x7fc00000) : l;
            }
        }
        tmem_wait_ld();
        tc_fence_before();
    }
    // a failed wait may leave copies in flight into this CTA's shared memory:
    // the producer waits for them (bounded) before the CTA retires
    __syncthreads();
    if (tid == CTHREADS && *(volatile int*)err_flag) {
        for (int s = 0; s < STAGES && s < n_tiles; ++s) {
            const int last = ((n_tiles - 1 - s) / STAGES) * STAGES + s;
            (void)mbar_wait(&full[s], (last / STAGES) & 1);
        }
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace umma
}  // namespace kvq
