// Split-T partial kernel: one CTA per (T chunk, cache head x head tile, batch
// row). It streams the chunk's packed K and V rows once for all HT query
// heads that read this cache head (the GQA group), and leaves an unnormalised
// partial (O, m, l) per query head for the log-sum-exp merge.
//
// Per tile of TILE positions (one per thread):
//   scores   s[h,t] = (sum_d q[h,d] * (scale_g * code + bias_g)) / sqrt(DH)
//   online softmax: m' = max(m, max_t s), alpha = e^(m - m'),
//                   p = e^(s - m'), l' = alpha l + sum p
//   combine  O[h,:] = alpha O[h,:] + sum_t p[h,t] * dequant(V_t)
// and, in the last split, the step's own new entry (new_k / new_v at full
// precision) as one more position. Every intermediate is fp32; the dequant is
// a rounded multiply then a rounded add per element, the reference kernel's
// arithmetic shape (kernelverify/pack/kv_attention.py:128-157,200-224).
#pragma once

#include "kvq_common.cuh"

namespace kvq {

constexpr int P_THREADS = 256;
constexpr int P_WARPS = P_THREADS / 32;
constexpr int P_TILE = P_THREADS;

template <int HT, int DH>
constexpr size_t partial_smem_bytes() {
    // q[HT][DH] + p[HT][TILE] + red[HT][WARPS] + obuf[WARPS][HT][DH]
    return sizeof(float) * (HT * DH + HT * P_TILE + HT * P_WARPS + P_WARPS * HT * DH);
}

template <typename T, int BITS, int DH, int HT>
__global__ void __launch_bounds__(P_THREADS)
partial_kernel(Problem P, float* __restrict__ part_o, float* __restrict__ part_m,
               float* __restrict__ part_l) {
    constexpr int W = DH * BITS / 32;           // words per row
    constexpr int CC = Chunk<BITS>::CODES;
    constexpr int CW = Chunk<BITS>::WORDS;
    constexpr int L = DH / 32;                  // dims per lane in the combine

    extern __shared__ __align__(16) float smem[];
    float* qs = smem;                                   // [HT][DH]
    float* ps = qs + HT * DH;                           // [HT][TILE]
    float* red = ps + HT * P_TILE;                      // [HT][WARPS]
    float* obuf = red + HT * P_WARPS;                   // [WARPS][HT][DH]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t split = blockIdx.x;
    const uint32_t hk = blockIdx.y / P.head_tiles;
    const uint32_t tile_h = blockIdx.y % P.head_tiles;
    const uint32_t b = blockIdx.z;
    const uint32_t h0 = hk * P.r + tile_h * HT;
    const int nh = min(HT, (int)(P.r - tile_h * HT));
    const uint32_t H = P.n_heads;
    const uint32_t G = DH / P.group_size;

    const T* q = static_cast<const T*>(P.q);
    for (int i = tid; i < HT * DH; i += P_THREADS) {
        const int h = i / DH, d = i % DH;
        qs[i] = h < nh ? to_f32(q[((size_t)b * H + h0 + h) * DH + d]) : 0.0f;
    }

    uint32_t len = P.t_cached;
    if (P.seq_lens != nullptr) len = min((uint32_t)max(P.seq_lens[b], 0), P.t_cached);
    const uint32_t end = min(P.t_end, len);
    const uint32_t lo = P.t_begin + split * P.chunk;
    const uint32_t hi = min(end, lo + P.chunk);
    const bool with_new = P.has_new_entry && split == P.n_splits - 1;

    const uint64_t rowbase = (uint64_t)b * P.cache_batch_stride + (uint64_t)hk * P.t_stride;
    const T* ks = static_cast<const T*>(P.k_scales);
    const T* kb = static_cast<const T*>(P.k_biases);
    const T* vs = static_cast<const T*>(P.v_scales);
    const T* vb = static_cast<const T*>(P.v_biases);

    float m_run[HT], l_run[HT], acc[HT][L];
#pragma unroll
    for (int h = 0; h < HT; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
#pragma unroll
        for (int j = 0; j < L; ++j) acc[h][j] = 0.0f;
    }
    __syncthreads();

    for (uint32_t t0 = lo; t0 < hi; t0 += P_TILE) {
        // ---- scores: one thread per position ---------------------------------
        const uint32_t t = t0 + tid;
        const bool valid = t < hi;
        float s[HT];
#pragma unroll
        for (int h = 0; h < HT; ++h) s[h] = 0.0f;
        if (valid) {
            const uint64_t row = rowbase + t;
            const uint32_t* kw = P.k_wq + row * W;
#pragma unroll 1
            for (int c = 0; c < DH / CC; ++c) {
                uint32_t w[CW];
#pragma unroll
                for (int i = 0; i < CW; ++i) w[i] = __ldg(kw + c * CW + i);
                const int d0 = c * CC;
                const int g = d0 / (int)P.group_size;
                const float sg = to_f32(ks[row * G + g]);
                const float bg = to_f32(kb[row * G + g]);
                float v[CC];
                static_for<CC>([&](auto J) {
                    v[J.value] = dequant(sg, chunk_code<BITS, J.value>(w), bg);
                });
#pragma unroll
                for (int h = 0; h < HT; ++h) {
#pragma unroll
                    for (int j = 0; j < CC; ++j) s[h] = fmaf(qs[h * DH + d0 + j], v[j], s[h]);
                }
            }
#pragma unroll
            for (int h = 0; h < HT; ++h) s[h] = s[h] * P.scale;
        } else {
#pragma unroll
            for (int h = 0; h < HT; ++h) s[h] = -INFINITY;
        }

        // ---- tile max, online rescale ----------------------------------------
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            const float mx = warp_max(s[h]);
            if (lane == 0) red[h * P_WARPS + warp] = mx;
        }
        __syncthreads();
        float m_new[HT], alpha[HT];
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            float mx = red[h * P_WARPS];
#pragma unroll
            for (int i = 1; i < P_WARPS; ++i) mx = fmaxf(mx, red[h * P_WARPS + i]);
            m_new[h] = fmaxf(m_run[h], mx);
            alpha[h] = m_run[h] == -INFINITY ? 0.0f : expf(m_run[h] - m_new[h]);
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            const float p = valid ? expf(s[h] - m_new[h]) : 0.0f;
            ps[h * P_TILE + tid] = p;
            const float sum = warp_sum(p);
            if (lane == 0) red[h * P_WARPS + warp] = sum;
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < P_WARPS; ++i) sum += red[h * P_WARPS + i];
            l_run[h] = l_run[h] * alpha[h] + sum;
            m_run[h] = m_new[h];
#pragma unroll
            for (int j = 0; j < L; ++j) acc[h][j] *= alpha[h];
        }

        // ---- combine: warp w takes positions w, w+WARPS, ...; lane owns L dims
        const int dl = lane * L;
        const int g = dl / (int)P.group_size;
        const int n_here = (int)min((uint32_t)P_TILE, hi - t0);
#pragma unroll 1
        for (int i = warp; i < n_here; i += P_WARPS) {
            const uint64_t row = rowbase + t0 + i;
            const uint32_t* vw = P.v_wq + row * W;
            const float sg = to_f32(vs[row * G + g]);
            const float bg = to_f32(vb[row * G + g]);
            float v[L];
#pragma unroll
            for (int j = 0; j < L; ++j) v[j] = dequant(sg, row_code<BITS>(vw, dl + j), bg);
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                const float p = ps[h * P_TILE + i];
#pragma unroll
                for (int j = 0; j < L; ++j) acc[h][j] = fmaf(p, v[j], acc[h][j]);
            }
        }
        __syncthreads();
    }

    // ---- the step's own entry: new_k / new_v at full precision ---------------
    if (with_new) {
        const T* nk = static_cast<const T*>(P.new_k) + ((size_t)b * P.n_kv_heads + hk) * DH;
        const T* nv = static_cast<const T*>(P.new_v) + ((size_t)b * P.n_kv_heads + hk) * DH;
        const int dl = lane * L;
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < L; ++j) part = fmaf(qs[h * DH + dl + j], to_f32(nk[dl + j]), part);
            const float s_new = warp_sum(part) * P.scale;
            const float m_new = fmaxf(m_run[h], s_new);
            const float alpha = m_run[h] == -INFINITY ? 0.0f : expf(m_run[h] - m_new);
            const float p_new = expf(s_new - m_new);
            l_run[h] = l_run[h] * alpha + p_new;
            m_run[h] = m_new;
#pragma unroll
            for (int j = 0; j < L; ++j) {
                acc[h][j] *= alpha;
                if (warp == 0) acc[h][j] = fmaf(p_new, to_f32(nv[dl + j]), acc[h][j]);
            }
        }
    }

    // ---- cross-warp reduction and the partial's write ------------------------
#pragma unroll
    for (int h = 0; h < HT; ++h) {
#pragma unroll
        for (int j = 0; j < L; ++j) obuf[(warp * HT + h) * DH + lane * L + j] = acc[h][j];
    }
    __syncthreads();
    const size_t rows = (size_t)P.b_rows * H;
    for (int i = tid; i < nh * DH; i += P_THREADS) {
        const int h = i / DH, d = i % DH;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < P_WARPS; ++w) o += obuf[(w * HT + h) * DH + d];
        part_o[((size_t)split * rows + (size_t)b * H + h0 + h) * DH + d] = o;
    }
    if (tid < nh) {
        float mv = 0.0f, lv = 0.0f;
#pragma unroll
        for (int h = 0; h < HT; ++h) {
            if (h == tid) { mv = m_run[h]; lv = l_run[h]; }
        }
        part_m[(size_t)split * rows + (size_t)b * H + h0 + tid] = mv;
        part_l[(size_t)split * rows + (size_t)b * H + h0 + tid] = lv;
    }
}

// Log-sum-exp merge of n_parts partials, one 256-thread block per row.
// Part p's O row starts at part_o + p * o_stride + row * head_dim and its m, l
// at part_m / part_l + p * ml_stride + row, so stacked partials ([P, rows, DH]
// and [P, rows]) and partial records laid end to end are both served.
// The first 32 parts' O rows are loaded up front (warp w: parts w, w+8, w+16,
// w+24; lane owns dims lane, lane+32, ...); meanwhile the parts' m and l are
// staged in shared memory and reduced to the max and to weights e^(m_p - m)
// with l = sum l_p e^(m_p - m); further parts follow four per warp at a time,
// no load waiting on another, and the eight warp sums meet in shared memory. head_dim is a multiple of 32, at most 256; n_parts at
// most MERGE_MAX_PARTS.
// NORMALIZE: out = sum_p O_p e^(m_p - m) / l in TO. Otherwise the merged
// partial (O unnormalised, m, l) in fp32. A part with m = -inf (an empty
// range) adds nothing; a NaN m (a poisoned partial) makes the row NaN.
constexpr int MERGE_THREADS = 256;
constexpr int MERGE_WARPS = MERGE_THREADS / 32;
constexpr int MERGE_MAX_DH = 256;
constexpr int MERGE_MAX_PARTS = 4096;
constexpr int MERGE_UNROLL = 4;

template <typename TO, bool NORMALIZE>
__global__ void __launch_bounds__(MERGE_THREADS)
merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_m,
             const float* __restrict__ part_l, uint32_t n_parts, uint32_t rows,
             uint32_t head_dim, uint64_t o_stride, uint64_t ml_stride, TO* __restrict__ out,
             float* __restrict__ out_m, float* __restrict__ out_l) {
    __shared__ float s_w[MERGE_MAX_PARTS];
    __shared__ float s_l[MERGE_MAX_PARTS];
    __shared__ float s_red[2][MERGE_WARPS];
    __shared__ float s_o[MERGE_WARPS][MERGE_MAX_DH];
    // the partials come from the kernel before this one, which may still be
    // running when this grid starts: wait for it, and read them through L2
    // (the read-only path may keep lines from before the wait)
    pdl_wait();
    const uint32_t row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per_lane = (int)head_dim / 32;
    const float* orow = part_o + (size_t)row * head_dim + lane;

    // the first MERGE_WARPS * MERGE_UNROLL parts' O rows are requested before
    // anything else, so their latency overlaps the m and l phases
    float ov0[MERGE_UNROLL][MERGE_MAX_DH / 32];
#pragma unroll
    for (int u = 0; u < MERGE_UNROLL; ++u) {
        const uint32_t p = warp + u * MERGE_WARPS;
        const float* o = orow + p * o_stride;
#pragma unroll
        for (int k = 0; k < MERGE_MAX_DH / 32; ++k)
            ov0[u][k] = (p < n_parts && k < per_lane) ? __ldcg(o + 32 * k) : 0.0f;
    }
    float m = -INFINITY;
    for (uint32_t p = tid; p < n_parts; p += MERGE_THREADS) {
        const float v = __ldcg(part_m + p * ml_stride + row);
        s_w[p] = v;
        s_l[p] = __ldcg(part_l + p * ml_stride + row);
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    if (lane == 0) s_red[0][warp] = m;
    __syncthreads();
    m = s_red[0][0];
#pragma unroll
    for (int w = 1; w < MERGE_WARPS; ++w) m = fmaxf(m, s_red[0][w]);

    // each thread rewrites only the entries it staged, so no barrier between
    float l = 0.0f;
    for (uint32_t p = tid; p < n_parts; p += MERGE_THREADS) {
        const float v = s_w[p];
        const float w = v == -INFINITY ? 0.0f : expf(v - m);
        s_w[p] = w;
        if (w != 0.0f) l = fmaf(s_l[p], w, l);
    }
    l = warp_sum(l);
    if (lane == 0) s_red[1][warp] = l;
    __syncthreads();
    float lt = 0.0f;
#pragma unroll
    for (int w = 0; w < MERGE_WARPS; ++w) lt += s_red[1][w];

    float acc[MERGE_MAX_DH / 32];
#pragma unroll
    for (int k = 0; k < MERGE_MAX_DH / 32; ++k) acc[k] = 0.0f;
#pragma unroll
    for (int u = 0; u < MERGE_UNROLL; ++u) {
        const uint32_t p = warp + u * MERGE_WARPS;
        const float w = p < n_parts ? s_w[p] : 0.0f;
#pragma unroll
        for (int k = 0; k < MERGE_MAX_DH / 32; ++k)
            if (w != 0.0f) acc[k] = fmaf(ov0[u][k], w, acc[k]);
    }
    for (uint32_t p0 = warp + MERGE_WARPS * MERGE_UNROLL; p0 < n_parts; p0 += MERGE_WARPS * MERGE_UNROLL) {
        float wv[MERGE_UNROLL];
        float ov[MERGE_UNROLL][MERGE_MAX_DH / 32];
#pragma unroll
        for (int j = 0; j < MERGE_UNROLL; ++j) {
            const uint32_t p = p0 + j * MERGE_WARPS;
            wv[j] = p < n_parts ? s_w[p] : 0.0f;
            const float* o = orow + p * o_stride;
#pragma unroll
            for (int k = 0; k < MERGE_MAX_DH / 32; ++k)
                ov[j][k] = (k < per_lane && wv[j] != 0.0f) ? __ldcg(o + 32 * k) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < MERGE_UNROLL; ++j)
#pragma unroll
            for (int k = 0; k < MERGE_MAX_DH / 32; ++k)
                if (wv[j] != 0.0f) acc[k] = fmaf(ov[j][k], wv[j], acc[k]);
    }
#pragma unroll
    for (int k = 0; k < MERGE_MAX_DH / 32; ++k)
        if (k < per_lane) s_o[warp][lane + 32 * k] = acc[k];
    __syncthreads();
    for (uint32_t d = tid; d < head_dim; d += MERGE_THREADS) {
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < MERGE_WARPS; ++w) o += s_o[w][d];
        if constexpr (NORMALIZE) {
            out[(size_t)row * head_dim + d] = from_f32<TO>(o / lt);
        } else {
            out[(size_t)row * head_dim + d] = m == -INFINITY ? 0.0f : o;
        }
    }
    if constexpr (!NORMALIZE) {
        if (tid == 0) {
            out_m[row] = m;
            out_l[row] = lt;
        }
    }
}

// The merge at the split stage's sizes (head_dim 128, at most 64 parts, O
// rows 16-byte aligned): every load of a row -- each warp's parts' O columns
// (a float4 per lane) and their m and l -- is requested at once, one round
// trip, instead of the general kernel's dependent phases. Warp w folds parts
// w, w + 8, ... under its own running maximum; the eight warps then meet in
// shared memory. Same results as merge_kernel up to the order of the fp32
// sums; an empty part (m = -inf) adds nothing, a NaN m poisons the row.
constexpr int MERGE_SMALL_PARTS = 64;

template <typename TO, bool NORMALIZE>
__global__ void __launch_bounds__(MERGE_THREADS)
merge_small_kernel(const float* __restrict__ part_o, const float* __restrict__ part_m,
                   const float* __restrict__ part_l, uint32_t n_parts, uint32_t rows,
                   uint64_t o_stride, uint64_t ml_stride, TO* __restrict__ out,
                   float* __restrict__ out_m, float* __restrict__ out_l) {
    constexpr int DH = 128, PER_WARP = MERGE_SMALL_PARTS / MERGE_WARPS;
    __shared__ float s_m[MERGE_WARPS], s_l[MERGE_WARPS];
    __shared__ float4 s_o[MERGE_WARPS][DH / 4];
    // the partials come from the kernel before this one (see merge_kernel)
    pdl_wait();
    const uint32_t row = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float4 o[PER_WARP];
    float mv[PER_WARP], lv[PER_WARP];
#pragma unroll
    for (int i = 0; i < PER_WARP; ++i) {
        const uint32_t p = warp + i * MERGE_WARPS;
        if (p < n_parts) {
            o[i] = __ldcg(reinterpret_cast<const float4*>(part_o + p * o_stride + (size_t)row * DH) + lane);
            mv[i] = __ldcg(part_m + p * ml_stride + row);
            lv[i] = __ldcg(part_l + p * ml_stride + row);
        } else {
            o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            mv[i] = -INFINITY;
            lv[i] = 0.0f;
        }
    }
    float M = -INFINITY;
    bool poisoned = false;
#pragma unroll
    for (int i = 0; i < PER_WARP; ++i) {
        M = fmaxf(M, mv[i]);
        poisoned |= mv[i] != mv[i];
    }
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < PER_WARP; ++i) {
        const float w = mv[i] == -INFINITY ? 0.0f : expf(mv[i] - M);
        if (w != 0.0f) {
            L = fmaf(lv[i], w, L);
            acc.x = fmaf(o[i].x, w, acc.x);
            acc.y = fmaf(o[i].y, w, acc.y);
            acc.z = fmaf(o[i].z, w, acc.z);
            acc.w = fmaf(o[i].w, w, acc.w);
        }
    }
    if (poisoned) M = L = __int_as_float(0x7fc00000);
    if (lane == 0) {
        s_m[warp] = M;
        s_l[warp] = L;
    }
    s_o[warp][lane] = acc;
    __syncthreads();
    if (warp != 0) return;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < MERGE_WARPS; ++w) m = fmaxf(m, s_m[w]);
    float lt = 0.0f;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < MERGE_WARPS; ++w) {
        if (s_m[w] == -INFINITY) continue;
        const float c = expf(s_m[w] - m);
        const float4 x = s_o[w][lane];
        lt = fmaf(s_l[w], c, lt);
        r.x = fmaf(x.x, c, r.x);
        r.y = fmaf(x.y, c, r.y);
        r.z = fmaf(x.z, c, r.z);
        r.w = fmaf(x.w, c, r.w);
    }
    TO* dst = out + (size_t)row * DH + 4 * lane;
    if constexpr (NORMALIZE) {
        dst[0] = from_f32<TO>(r.x / lt);
        dst[1] = from_f32<TO>(r.y / lt);
        dst[2] = from_f32<TO>(r.z / lt);
        dst[3] = from_f32<TO>(r.w / lt);
    } else {
        // no part at all (m = -inf, l = 0): a zero row; a poisoned one keeps
        // NaN in m as well, so a later merge of this record stays poisoned
        const bool empty = m == -INFINITY && lt == 0.0f;
        if (lt != lt) m = lt;
        dst[0] = empty ? 0.0f : r.x;
        dst[1] = empty ? 0.0f : r.y;
        dst[2] = empty ? 0.0f : r.z;
        dst[3] = empty ? 0.0f : r.w;
        if (lane == 0) {
            out_m[row] = m;
            out_l[row] = lt;
        }
    }
}

}  // namespace kvq
