// Register-fragment tensor-core partial kernel with a transposed score MMA,
// for the group-64 format (fp16 steps, 4-bit caches, head_dim 128).
//
// Same stage ring, producer, scale scratch, combine and CTA merge as
// partial_kernel (kvq_mma.cuh); only the score side differs. Scores are
//   S[pos, n] = sum_k Kcodes[pos, k] * Qn[k, n]
// with the 16 positions of the warp's block as the MMA's M rows and the
// columns n as N: at 4 query heads per cache head n = group * 4 + head, each
// head's q zeroed outside that group, so one MMA chain over all 128 dims gives
// both groups' dot products X_g[pos, h]; at 8 heads n = head and each group
// accumulates in its own chain. That is 8 MMAs of m16n8k16 per block where the
// untransposed form needs 16 with half of every A fragment zero.
//
// The score fragment (positions in rows) is transposed into the combine's B
// fragment (positions along k) with movmatrix: rows are ordered so that
// fragment row r holds position (r >> 1) + 4 (r & 1) and row r + 8 that
// position + 8, which after the transpose puts positions j, j+4 | j+8, j+12 in
// lane (., j) -- the rows the combine's A fragments are built from.
#pragma once

#include "kvq_fused.cuh"
#include "kvq_mma.cuh"

namespace kvq {
namespace mma4 {

// 8x8 b16 transpose across the warp: lane (r, j) gets elements (2j, 2j+1) of
// column r of the matrix whose row r lane (r, j) held at columns 2j, 2j+1
__device__ __forceinline__ uint32_t transpose8x8(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// The split stage's CTA: its split's partial into part_* [n_splits, rows(, DH)],
// or with TAGGED as tagged words into `tagged` (finish_partial).
template <int HT, int PARTS, bool TAGGED = false>
__device__ __forceinline__ void partial_t_body(const Problem& P, float* __restrict__ part_o,
                                               float* __restrict__ part_m, float* __restrict__ part_l,
                                               uint64_t* __restrict__ tagged = nullptr, uint32_t tag = 0) {
    constexpr int GROUP = 64;
    using Lay = Layout<GROUP>;
    constexpr int G = Lay::G;
    constexpr int MTG = GROUP / 16;     // V-side M-tiles per group
    constexpr int MT = DH / 16;         // V-side M-tiles
    constexpr int VBYTES = GROUP / 16;  // V-side bytes per lane, row and group
    constexpr int NACC = HT == 4 ? 1 : G;   // score accumulator chains
    constexpr int NSC = HT == 4 ? 2 : 4;    // scores a lane keeps per block
    constexpr float L2E = 1.4426950408889634f;
    static_assert(HT == 4 || HT == 8, "head tile");
    static_assert(G == 2, "group 64 at head_dim 128");
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
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        *err_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == CWARPS) {
        if (lane == 0) produce<GROUP>(P, smem, full, empty, err_flag, lo, hi, n_stages, rowbase);
    } else {
        const int r = lane >> 2, j = lane & 3;
        // the lane's two score heads 2*hp, 2*hp+1; at HT = 4 the lane keeps
        // fragment row r (half 0) or r + 8 (half 1)
        const int hp = HT == 4 ? (j & 1) : j;
        const int half = HT == 4 ? (j >> 1) : 0;

        // Q as the score MMA's B fragment: column n = r, k-step (c, a) over
        // word wi = 8 (c >> 1) + 2j + (c & 1) of each position row, nibble
        // pairs (0,4 | 1,5) for a = 0 and (2,6 | 3,7) for a = 1.
        uint32_t qb[8][2];
        float qcol[G] = {0.0f, 0.0f};
        {
            const int colh = HT == 4 ? (r & 3) : r;
            const int colg = HT == 4 ? (r >> 2) : -1;
            const bool qvalid = colh < nh;
            const __half* q = static_cast<const __half*>(P.q) + ((size_t)b * H + h0 + colh) * DH;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int g = c >> 1;
                const int wi = 8 * g + 2 * j + (c & 1);
                const bool live = qvalid && (colg < 0 || colg == g);
#pragma unroll
                for (int a = 0; a < 2; ++a) {
                    const int d = 8 * wi + 2 * a;
                    __half2 x0 = live ? __halves2half2(q[d], q[d + 4]) : __half2(0, 0);
                    __half2 x1 = live ? __halves2half2(q[d + 1], q[d + 5]) : __half2(0, 0);
                    qcol[g] += __low2float(x0) + __high2float(x0) + __low2float(x1) + __high2float(x1);
                    qb[2 * c + a][0] = *reinterpret_cast<uint32_t*>(&x0);
                    qb[2 * c + a][1] = *reinterpret_cast<uint32_t*>(&x1);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                qcol[g] += __shfl_xor_sync(0xffffffffu, qcol[g], 1);
                qcol[g] += __shfl_xor_sync(0xffffffffu, qcol[g], 2);
            }
        }
        // per-group q sums of the lane's score heads, from the column lanes
        float qs[G][2];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int col = HT == 4 ? g * 4 + 2 * hp + k : 2 * hp + k;
                qs[g][k] = __shfl_sync(0xffffffffu, qcol[g], 4 * col);
            }

        float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.0f, 0.0f};
        float bsum[G][2];
        float oacc[MT][4];
#pragma unroll
        for (int g = 0; g < G; ++g) bsum[g][0] = bsum[g][1] = 0.0f;
#pragma unroll
        for (int i = 0; i < MT; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;

        const int kr0 = (r >> 1) + 4 * (r & 1);   // position of fragment row r (row r+8: +8)

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
            if (nvalid <= blk * 16) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                continue;
            }
            // fp32 scales and biases of the block (see partial_kernel); at 4
            // heads a lane needs one position's, which it reads from the stage
            // directly (below)
            float* scr = reinterpret_cast<float*>(smem + Lay::SCR + warp * Lay::SCR_WARP);
            if constexpr (HT != 4) {
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
            const float* kscr = scr;
            const float* vscr = scr + 16 * 2 * G;

            // ---- scores: 8 MMAs, fragment rows = positions -----------------
            float acc[NACC][4];
#pragma unroll
            for (int n = 0; n < NACC; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
            {
                const unsigned char* row0 = st + Lay::KC + (blk * 16 + kr0) * ROWB;
                const unsigned char* row1 = row0 + 8 * ROWB;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const uint2 w0 = *reinterpret_cast<const uint2*>(row0 + 4 * (8 * g + 2 * j));
                    const uint2 w1 = *reinterpret_cast<const uint2*>(row1 + 4 * (8 * g + 2 * j));
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int c = 2 * g + cc;
                        uint32_t n0[4], n1[4];
                        nibbles_f16(cc ? w0.y : w0.x, n0);
                        nibbles_f16(cc ? w1.y : w1.x, n1);
                        float (&A)[4] = acc[HT == 4 ? 0 : g];
                        mma_f16(A, n0[0], n1[0], n0[1], n1[1], qb[2 * c][0], qb[2 * c][1]);
                        mma_f16(A, n0[2], n1[2], n0[3], n1[3], qb[2 * c + 1][0], qb[2 * c + 1][1]);
                    }
                }
            }
            // at 4 heads the V code words are read now, so their shared-memory
            // latency hides behind the score epilogue and the softmax
            uint32_t vwq[G][4];
            if constexpr (HT == 4) {
                const int p0h = blk * 16 + j;
                const unsigned char* vrowh = st + Lay::VC;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int boff = g * (GROUP / 2) + r * VBYTES;
                    vwq[g][0] = *reinterpret_cast<const uint32_t*>(vrowh + (p0h) * ROWB + boff);
                    vwq[g][1] = *reinterpret_cast<const uint32_t*>(vrowh + (p0h + 4) * ROWB + boff);
                    vwq[g][2] = *reinterpret_cast<const uint32_t*>(vrowh + (p0h + 8) * ROWB + boff);
                    vwq[g][3] = *reinterpret_cast<const uint32_t*>(vrowh + (p0h + 12) * ROWB + boff);
                }
            }
            // score epilogue: sc[k] (HT = 4) is head 2hp+k at the lane's kept
            // row; sc[2rr + k] (HT = 8) head 2hp+k at row r + 8rr
            float sc[NSC];
            if constexpr (HT == 4) {
                // columns 2j, 2j+1: group 0 (j < 2) or group 1 (j >= 2) of heads
                // 2hp, 2hp+1; the partner lane j^2 holds the other group
                const float s0 = half ? acc[0][0] : acc[0][2];
                const float s1 = half ? acc[0][1] : acc[0][3];
                const float r0 = __shfl_xor_sync(0xffffffffu, s0, 2);
                const float r1 = __shfl_xor_sync(0xffffffffu, s1, 2);
                const float x00 = half ? r0 : acc[0][0], x01 = half ? r1 : acc[0][1];   // group 0
                const float x10 = half ? acc[0][2] : r0, x11 = half ? acc[0][3] : r1;   // group 1
                const int lp = kr0 + 8 * half;
                const bool live = blk * 16 + lp < nvalid;
                // the position's k scales and biases straight from the stage (a
                // dead position's may be any bits: its score is replaced below)
                const int prow = blk * 16 + lp;
                const float2 ks2 = __half22float2(*reinterpret_cast<const __half2*>(st + Lay::KS + prow * 2 * G));
                const float2 kb2 = __half22float2(*reinterpret_cast<const __half2*>(st + Lay::KB + prow * 2 * G));
                const float a0 = scale2 * fmaf(ks2.x, x00, fmaf(ks2.y, x10, fmaf(kb2.x, qs[0][0], kb2.y * qs[1][0])));
                const float a1 = scale2 * fmaf(ks2.x, x01, fmaf(ks2.y, x11, fmaf(kb2.x, qs[0][1], kb2.y * qs[1][1])));
                sc[0] = live ? a0 : -INFINITY;
                sc[1] = live ? a1 : -INFINITY;
            } else {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int lp = kr0 + 8 * rr;
                    float kf[2 * G];
                    load_f<2 * G>(kscr + lp * 2 * G, kf);
                    const bool live = blk * 16 + lp < nvalid;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const float a = fmaf(kf[0], acc[0][2 * rr + k],
                                             fmaf(kf[1], acc[1][2 * rr + k],
                                                  fmaf(kf[2], qs[0][k], kf[3] * qs[1][k])));
                        sc[2 * rr + k] = live ? a : -INFINITY;
                    }
                }
            }

            // ---- online softmax, lazy rescaling (as partial_kernel) ---------
            float mx[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) mx[k] = HT == 4 ? sc[k] : fmaxf(sc[k], sc[2 + k]);
            if (__any_sync(0xffffffffu, mx[0] > m_run[0] + 8.0f || mx[1] > m_run[1] + 8.0f)) {
                float alpha[2];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    float v = mx[k];
                    if constexpr (HT == 4) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
                    const float m_new = v > m_run[k] + 8.0f ? v : m_run[k];
                    alpha[k] = ex2(m_run[k] - m_new);
                    m_run[k] = m_new;
                    l_part[k] *= alpha[k];
#pragma unroll
                    for (int g = 0; g < G; ++g) bsum[g][k] *= alpha[k];
                }
                // O columns 2j, 2j+1 are the lane's own heads
                const float2 a01 = make_float2(alpha[0], alpha[1]);
#pragma unroll
                for (int i = 0; i < MT; ++i) {
                    const float2 u = __fmul2_rn(make_float2(oacc[i][0], oacc[i][1]), a01);
                    const float2 v = __fmul2_rn(make_float2(oacc[i][2], oacc[i][3]), a01);
                    oacc[i][0] = u.x; oacc[i][1] = u.y; oacc[i][2] = v.x; oacc[i][3] = v.y;
                }
            }
            float e[NSC];
#pragma unroll
            for (int i = 0; i < NSC; ++i) e[i] = ex2(sc[i] - m_run[i & 1]);
#pragma unroll
            for (int i = 0; i < NSC; ++i) l_part[i & 1] += e[i];

            // ---- combine: B fragments of P' = p * v_scale by transposition --
            // first MMA (bf), second (bs), third (bt): at HT = 4 the first takes
            // hi (columns 0..3) and mid (columns 4..7; lo at PARTS = 2), the
            // second lo in columns 0..3; at HT = 8 one MMA per part
            uint32_t bf0[G], bf1[G], bs0[G], bs1[G], bt0[G], bt1[G];
            if constexpr (HT == 4) {
                const int lp = kr0 + 8 * half;
                float vf[2 * G];
                {
                    // v scales and biases - 128 v scales from the stage; zero at a
                    // dead position, so its P' and bias term vanish
                    const int prow = blk * 16 + lp;
                    const bool vlive = prow < nvalid;
                    float2 vs2 = __half22float2(*reinterpret_cast<const __half2*>(st + Lay::VS + prow * 2 * G));
                    float2 vb2 = __half22float2(*reinterpret_cast<const __half2*>(st + Lay::VB + prow * 2 * G));
                    vs2.x = vlive ? vs2.x : 0.0f; vs2.y = vlive ? vs2.y : 0.0f;
                    vb2.x = vlive ? vb2.x : 0.0f; vb2.y = vlive ? vb2.y : 0.0f;
                    vf[0] = vs2.x; vf[1] = vs2.y;
                    vf[2] = fmaf(vs2.x, -128.0f, vb2.x); vf[3] = fmaf(vs2.y, -128.0f, vb2.y);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    bsum[g][0] = fmaf(e[0], vf[G + g], bsum[g][0]);
                    bsum[g][1] = fmaf(e[1], vf[G + g], bsum[g][1]);
                    const float2 v = __fmul2_rn(make_float2(e[0], e[1]), make_float2(vf[g], vf[g]));
                    uint32_t phi, pmid, plo;
                    if constexpr (PARTS == 3) {
                        split3(v.x, v.y, phi, pmid, plo);
                    } else {
                        split2(v.x, v.y, phi, pmid);
                        plo = 0u;
                    }
                    // matrix rows r <-> positions kr0 (m0) and kr0 + 8 (m1); the
                    // partner lane j^2 holds the other row's parts of the same heads
                    const uint32_t recv = __shfl_xor_sync(0xffffffffu, half ? phi : pmid, 2);
                    bf0[g] = transpose8x8(half ? recv : phi);
                    bf1[g] = transpose8x8(half ? pmid : recv);
                    if constexpr (PARTS == 3) {
                        const uint32_t recv_lo = __shfl_xor_sync(0xffffffffu, plo, 2);
                        bs0[g] = transpose8x8(half ? 0u : plo);
                        bs1[g] = transpose8x8(half ? 0u : recv_lo);
                    } else {
                        bs0[g] = bs1[g] = 0u;
                    }
                    bt0[g] = bt1[g] = 0u;
                }
            } else {
                float vf[2][2 * G];
                load_f<2 * G>(vscr + kr0 * 2 * G, vf[0]);
                load_f<2 * G>(vscr + (kr0 + 8) * 2 * G, vf[1]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    uint32_t phi[2], pmid[2], plo[2];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        bsum[g][0] = fmaf(e[2 * rr], vf[rr][G + g], bsum[g][0]);
                        bsum[g][1] = fmaf(e[2 * rr + 1], vf[rr][G + g], bsum[g][1]);
                        const float2 v = __fmul2_rn(make_float2(e[2 * rr], e[2 * rr + 1]),
                                                    make_float2(vf[rr][g], vf[rr][g]));
                        if constexpr (PARTS == 3) {
                            split3(v.x, v.y, phi[rr], pmid[rr], plo[rr]);
                        } else {
                            split2(v.x, v.y, phi[rr], pmid[rr]);
                            plo[rr] = 0u;
                        }
                    }
                    bf0[g] = transpose8x8(phi[0]);
                    bf1[g] = transpose8x8(phi[1]);
                    bs0[g] = transpose8x8(pmid[0]);
                    bs1[g] = transpose8x8(pmid[1]);
                    if constexpr (PARTS == 3) {
                        bt0[g] = transpose8x8(plo[0]);
                        bt1[g] = transpose8x8(plo[1]);
                    } else {
                        bt0[g] = bt1[g] = 0u;
                    }
                }
            }
            // A fragments (V codes^T) and the MMAs, as partial_kernel
            const int p0 = blk * 16 + j;
            const unsigned char* vrow = st + Lay::VC;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int boff = g * (GROUP / 2) + r * VBYTES;
                uint32_t wA, wB, wC, wD;
                if constexpr (HT == 4) {
                    wA = vwq[g][0]; wB = vwq[g][1]; wC = vwq[g][2]; wD = vwq[g][3];
                } else {
                    wA = *reinterpret_cast<const uint32_t*>(vrow + (p0) * ROWB + boff);
                    wB = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 4) * ROWB + boff);
                    wC = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 8) * ROWB + boff);
                    wD = *reinterpret_cast<const uint32_t*>(vrow + (p0 + 12) * ROWB + boff);
                }
                uint32_t fa[MTG][4];
                quad_bf16<0>(wA, wB, fa[0][0], fa[0][1], fa[1][0], fa[1][1]);
                quad_bf16<0>(wC, wD, fa[0][2], fa[0][3], fa[1][2], fa[1][3]);
                quad_bf16<2>(wA, wB, fa[2][0], fa[2][1], fa[3][0], fa[3][1]);
                quad_bf16<2>(wC, wD, fa[2][2], fa[2][3], fa[3][2], fa[3][3]);
#pragma unroll
                for (int ii = 0; ii < MTG; ++ii) {
                    float (&o)[4] = oacc[g * MTG + ii];
                    mma_bf16(o, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bf0[g], bf1[g]);
                    if constexpr (HT == 8 || PARTS == 3)
                        mma_bf16(o, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bs0[g], bs1[g]);
                    if constexpr (HT == 8 && PARTS == 3)
                        mma_bf16(o, fa[ii][0], fa[ii][1], fa[ii][2], fa[ii][3], bt0[g], bt1[g]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- warp partial: l and bias sums over the lanes sharing a head --------
#pragma unroll
        for (int k = 0; k < 2; ++k) {
#pragma unroll
            for (int x = 4; x <= 16; x <<= 1) {
                l_part[k] += __shfl_xor_sync(0xffffffffu, l_part[k], x);
#pragma unroll
                for (int g = 0; g < G; ++g) bsum[g][k] += __shfl_xor_sync(0xffffffffu, bsum[g][k], x);
            }
            if constexpr (HT == 4) {
                l_part[k] += __shfl_xor_sync(0xffffffffu, l_part[k], 2);
#pragma unroll
                for (int g = 0; g < G; ++g) bsum[g][k] += __shfl_xor_sync(0xffffffffu, bsum[g][k], 2);
            }
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
        if (r == 0 && (HT == 8 || j < 2)) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int h = 2 * hp + k;
                mm[warp * 8 + h] = m_run[k];
                ml[warp * 8 + h] = l_part[k];
#pragma unroll
                for (int g = 0; g < G; ++g) mb[(warp * 8 + h) * G + g] = bsum[g][k];
            }
        }
        if (HT == 8 || j < 2) {
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
        finish_partial<HT, GROUP, TAGGED>(P, smem, tid, warp, lane, split, b, hk, h0, nh, with_new,
                                          scale2, err_flag, part_o, part_m, part_l, tagged, tag);
    }
    __syncthreads();
    if (tid == CWARPS * 32 && *(volatile int*)err_flag) {
        for (int s = 0; s < STAGES && s < n_stages; ++s) {
            const int last = ((n_stages - 1 - s) / STAGES) * STAGES + s;
            (void)mbar_wait(&full[s], (last / STAGES) & 1);
        }
    }
}

template <int HT, int PARTS>
__global__ void __launch_bounds__(THREADS, KVQ_MMA_MINBLOCKS)
partial_kernel_t(Problem P, float* __restrict__ part_o, float* __restrict__ part_m,
                 float* __restrict__ part_l) {
    partial_t_body<HT, PARTS>(P, part_o, part_m, part_l);
}

// The whole sequence-split step in one launch: the split stage with its
// partial tagged into the region's store, then the merge of the unit's
// splits, the exchange of the ranks' records and the final merge by the
// unit's last CTAs (kvq_fused.cuh).
template <int HT, int PARTS>
__global__ void __launch_bounds__(THREADS, KVQ_MMA_MINBLOCKS)
partial_kernel_tf(Problem P, const __grid_constant__ fused::Fused F) {
    static_assert(THREADS == fused::TAIL_THREADS, "the tail is written for the split stage's CTA size");
    // this step's number: the unit's count in the region + 1 (every CTA of
    // the unit reads it before it writes anything tagged with it)
    const uint32_t unit = blockIdx.z * gridDim.y + blockIdx.y;
    const uint32_t e = fused::ld_relaxed_gpu(fused::epoch_word(F, unit)) + 1u;
    partial_t_body<HT, PARTS, true>(P, nullptr, nullptr, nullptr, fused::partials(F), e);
    extern __shared__ __align__(128) unsigned char smem_tail[];
    fused::tail<HT>(P, F, e, smem_tail);
}

}  // namespace mma4
}  // namespace kvq
