// Register-fragment tensor-core partial kernel over byte codes: fp16 steps,
// head_dim 128, caches of 2-, 3-, 6- or 8-bit codes at groups 32, 64, 128.
//
// The structure is the 4-bit transposed kernel's (kvq_mmat.cuh): the same
// stage ring and producer (rows of DH * BITS / 8 code bytes), score MMAs with
// the 16 positions of a warp's block as M rows, the score fragment transposed
// into the combine's B fragment with movmatrix, the CTA merge. A lane reads
// the packed bits of the codes it needs (an aligned word load and one funnel
// shift bring the first code to bit 0) and spreads them to one code per byte
// in registers; from there every width is the 8-bit arithmetic:
//
// * Scores. Each score k-step covers 16 dims of one group; a lane reads its
//   dims of a row as one run per dim block and turns each code byte into fp16
//   exactly: a byte permute makes 0x64cc = 1024 + c, one subtract leaves c.
//   Q's B fragment follows the same dim order.
// * Combine. A code c = 16 h + l is carried as two bf16 values, both
//   exact: 128 + l (0x4300 | l) and 2048 + 16 h (0x4500 | h), in two MMAs that
//   share the P' fragments, so
//     sum_t P'_t (128 + l_t) + sum_t P'_t (2048 + 16 h_t) = sum_t P'_t c_t + 2176 sum_t P'_t
//   and the 2176 sum_t P'_t = sum_t p_t 2176 s_t is taken out through the bias
//   term (v_bias - 2176 v_scale), as the 4-bit kernel takes out 128. Codes
//   below 16 (2 and 3 bits) have h = 0: the second MMA is left out and the
//   offset is 128. Every M-tile keeps to one group, whose scale P' carries.
#pragma once

#include "kvq_mmat.cuh"

namespace kvq {
namespace mma4 {

// fp16 pairs of the exact code values of a word of four byte codes:
// (c0, c1) and (c2, c3)
__device__ __forceinline__ void bytes_f16(uint32_t w, uint32_t& h01, uint32_t& h23) {
    h01 = h2_sub1024(prmt<0x4140>(w, 0x64646464u));
    h23 = h2_sub1024(prmt<0x4342>(w, 0x64646464u));
}

// Four BITS-bit codes at bits 0 .. 4 BITS - 1 of x -> one code per byte.
template <int BITS>
__device__ __forceinline__ uint32_t spread4(uint32_t x) {
    if constexpr (BITS == 8) {
        return x;
    } else if constexpr (BITS == 2) {
        x &= 0xFFu;
        const uint32_t t = (x | (x << 12)) & 0x000F000Fu;          // (c0 c1 | c2 c3)
        return (t | (t << 6)) & 0x03030303u;
    } else if constexpr (BITS == 3) {
        x &= 0xFFFu;
        const uint32_t t = (x | (x << 10)) & 0x003F003Fu;
        return (t | (t << 5)) & 0x07070707u;
    } else {
        static_assert(BITS == 6, "code width");
        x &= 0xFFFFFFu;
        const uint32_t t = (x & 0xFFFu) | ((x << 4) & 0x0FFF0000u);  // bits 12..15 unused
        return (t & 0x003F003Fu) | ((t << 2) & 0x3F003F00u);
    }
}

// N codes (a multiple of 4) starting at code k0 of a row of packed BITS-bit
// codes -> N / 4 words, one code per byte. Only the 4-byte aligned words that
// hold bits of the run are read, so every read lies in the row (rows are whole
// words).
template <int BITS, int N>
__device__ __forceinline__ void codes_to_bytes(const unsigned char* row, int k0,
                                               uint32_t (&out)[N / 4]) {
    constexpr int NBITS = N * BITS;
    constexpr int NW = (NBITS + 31 + 31) / 32;          // words that can hold the run
    const int bitpos = k0 * BITS;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(row) + (bitpos >> 5);
    const uint32_t sh = (uint32_t)(bitpos & 31);
    uint32_t raw[NW + 1];
#pragma unroll
    for (int i = 0; i < NW; ++i) raw[i] = (32 * i < NBITS + (int)sh) ? w[i] : 0u;
    raw[NW] = 0u;
    uint32_t v[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) v[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
#pragma unroll
    for (int m = 0; m < N / 4; ++m) {
        const int bit = 4 * BITS * m;                   // compile-time after unrolling
        const int wi = bit >> 5, bs = bit & 31;
        const uint32_t x = bs == 0 ? v[wi] : __funnelshift_r(v[wi], wi + 1 < NW ? v[wi + 1] : 0u, bs);
        out[m] = spread4<BITS>(x);
    }
}

// Bytes K, K+1 of words a and b -> the low-nibble (128 + l) and high-nibble
// (2048 + 16 h) bf16 pairs (a.K, b.K) and (a.K+1, b.K+1).
template <int K>
__device__ __forceinline__ void byte_nibbles_bf16(uint32_t a, uint32_t b, uint32_t& lo0,
                                                  uint32_t& hi0, uint32_t& lo1, uint32_t& hi1) {
    constexpr uint32_t sel = K | ((K + 1) << 4) | ((4 + K) << 8) | ((5 + K) << 12);
    const uint32_t u = prmt<sel>(a, b);
    lo0 = and_or<0x000F000Fu, 0x43004300u>(u);
    hi0 = and_or<0x000F000Fu, 0x45004500u>(u >> 4);
    lo1 = and_or<0x000F000Fu, 0x43004300u>(u >> 8);
    hi1 = and_or<0x000F000Fu, 0x45004500u>(u >> 12);
}

// Byte loads of an 8-bit run (16, 8 or 4 codes) with the widest aligned load.
template <int N>
__device__ __forceinline__ void byte_run(const unsigned char* p, uint32_t (&out)[N / 4]) {
    if constexpr (N == 16) {
        const uint4 w = *reinterpret_cast<const uint4*>(p);
        out[0] = w.x; out[1] = w.y; out[2] = w.z; out[3] = w.w;
    } else if constexpr (N == 8) {
        const uint2 w = *reinterpret_cast<const uint2*>(p);
        out[0] = w.x; out[1] = w.y;
    } else {
        out[0] = *reinterpret_cast<const uint32_t*>(p);
    }
}

// N codes of a row starting at code k0, one per byte
template <int BITS, int N>
__device__ __forceinline__ void run_bytes(const unsigned char* row, int k0, uint32_t (&out)[N / 4]) {
    if constexpr (BITS == 8)
        byte_run<N>(row + k0, out);
    else
        codes_to_bytes<BITS, N>(row, k0, out);
}

// Dims are taken in NB blocks of BD: 64-dim blocks up to group 64, one block
// per group at group 32, so every score k-step and every combine M-tile lies
// in one group. Score side: block b holds k-steps b * KPB + i, lane j the
// dims BD b + SRUN j + 4 i + {0, 1 | 2, 3}. Combine side: M-tile b * MTB + mm,
// row r is dim BD b + VRUN r + 2 mm, row r + 8 that dim + 1. At group 64 with
// at most 4 query heads per cache head the score MMA's 8 columns are (group,
// head) pairs (COLS); otherwise columns are heads, with one accumulator chain
// per group.
template <int HT, int PARTS, int BITS, int GROUP>
__global__ void __launch_bounds__(THREADS, KVQ_MMA_MINBLOCKS)
partial_kernel_tb(Problem P, float* __restrict__ part_o, float* __restrict__ part_m,
                  float* __restrict__ part_l) {
    static_assert(BITS == 2 || BITS == 3 || BITS == 6 || BITS == 8, "code width");
    using Lay = Layout<GROUP, BITS>;
    constexpr int G = Lay::G;
    constexpr int RB = Lay::RB;         // code bytes per row
    constexpr int NST = Lay::NST;       // ring depth of this width's layout
    constexpr bool HI = BITS > 4;       // codes of 16 and above: the high-nibble pass
    constexpr int NB = G > 2 ? G : 2;   // dim blocks
    constexpr int BD = DH / NB;         // dims per block (64 or 32)
    constexpr int KPB = BD / 16;        // score k-steps per block
    constexpr int SRUN = BD / 4;        // score-side codes of a lane per (row, block)
    constexpr int VRUN = BD / 8;        // combine-side codes of a lane per (position, block)
    constexpr int MTB = BD / 16;        // M-tiles per block
    constexpr int MT = DH / 16;         // M-tiles
    constexpr bool COLS = HT == 4 && G == 2;
    constexpr int NACC = COLS ? 1 : G;
    constexpr int NSC = COLS ? 2 : 4;
    constexpr float L2E = 1.4426950408889634f;
    constexpr float VOFF = HI ? 2176.0f : 128.0f;   // the code offset the combine carries
    static_assert(HT == 8 || COLS, "head tile 4 only with the (group, head) columns");
    static_assert(NB * KPB == 8 && NB * MTB == MT, "block shape");
    const float scale2 = P.scale * L2E;

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (Lay::RING_SCR > Lay::MERGE ? Lay::RING_SCR : Lay::MERGE));
    uint64_t* empty = full + NST;
    int* err_flag = reinterpret_cast<int*>(empty + NST);

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
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        *err_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == CWARPS) {
        if (lane == 0) produce<GROUP, BITS>(P, smem, full, empty, err_flag, lo, hi, n_stages, rowbase);
    } else {
        const int r = lane >> 2, j = lane & 3;
        const int hp = COLS ? (j & 1) : j;
        const int half = COLS ? (j >> 1) : 0;

        // Q as the score MMA's B fragment: column n = r, k-step c = KPB bb + i
        // over dims BD bb + SRUN j + 4 i + {0, 1} (b0) and {2, 3} (b1)
        uint32_t qb[8][2];
        float qcol[G];
#pragma unroll
        for (int g = 0; g < G; ++g) qcol[g] = 0.0f;
        {
            const int colh = COLS ? (r & 3) : r;
            const int colg = COLS ? (r >> 2) : -1;
            const bool qvalid = colh < nh;
            const __half* q = static_cast<const __half*>(P.q) + ((size_t)b * H + h0 + colh) * DH;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int bb = c / KPB, g = bb * G / NB;
                const int d = BD * bb + SRUN * j + 4 * (c % KPB);
                const bool live = qvalid && (colg < 0 || colg == g);
                __half2 x0 = live ? __halves2half2(q[d], q[d + 1]) : __half2(0, 0);
                __half2 x1 = live ? __halves2half2(q[d + 2], q[d + 3]) : __half2(0, 0);
                qcol[g] += __low2float(x0) + __high2float(x0) + __low2float(x1) + __high2float(x1);
                qb[c][0] = *reinterpret_cast<uint32_t*>(&x0);
                qb[c][1] = *reinterpret_cast<uint32_t*>(&x1);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                qcol[g] += __shfl_xor_sync(0xffffffffu, qcol[g], 1);
                qcol[g] += __shfl_xor_sync(0xffffffffu, qcol[g], 2);
            }
        }
        float qs[G][2];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int col = COLS ? g * 4 + 2 * hp + k : 2 * hp + k;
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
            const int slot = s % NST, round = s / NST;
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
                    scr[16 * 2 * G + pos * 2 * G + G + g] = fmaf(vsv, -VOFF, vbv);
                }
                __syncwarp();
            }
            const float* kscr = scr;
            const float* vscr = scr + 16 * 2 * G;

            // ---- scores: 8 MMAs over the byte codes -----------------------
            float acc[NACC][4];
#pragma unroll
            for (int n = 0; n < NACC; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
            {
                const unsigned char* row0 = st + Lay::KC + (blk * 16 + kr0) * RB;
                const unsigned char* row1 = row0 + 8 * RB;
#pragma unroll
                for (int bb = 0; bb < NB; ++bb) {
                    uint32_t a[SRUN / 4], bw[SRUN / 4];
                    run_bytes<BITS, SRUN>(row0, BD * bb + SRUN * j, a);
                    run_bytes<BITS, SRUN>(row1, BD * bb + SRUN * j, bw);
#pragma unroll
                    for (int i = 0; i < KPB; ++i) {
                        uint32_t a01, a23, b01, b23;
                        bytes_f16(a[i], a01, a23);
                        bytes_f16(bw[i], b01, b23);
                        float (&A)[4] = acc[COLS ? 0 : bb * G / NB];
                        const int c = KPB * bb + i;
                        mma_f16(A, a01, b01, a23, b23, qb[c][0], qb[c][1]);
                    }
                }
            }
            float sc[NSC];
            if constexpr (COLS) {
                const float s0 = half ? acc[0][0] : acc[0][2];
                const float s1 = half ? acc[0][1] : acc[0][3];
                const float r0 = __shfl_xor_sync(0xffffffffu, s0, 2);
                const float r1 = __shfl_xor_sync(0xffffffffu, s1, 2);
                const float x00 = half ? r0 : acc[0][0], x01 = half ? r1 : acc[0][1];   // group 0
                const float x10 = half ? acc[0][2] : r0, x11 = half ? acc[0][3] : r1;   // group 1
                const int lp = kr0 + 8 * half;
                float kf[2 * G];
                load_f<2 * G>(kscr + lp * 2 * G, kf);
                const bool live = blk * 16 + lp < nvalid;
                const float a0 = fmaf(kf[0], x00, fmaf(kf[1], x10, fmaf(kf[2], qs[0][0], kf[3] * qs[1][0])));
                const float a1 = fmaf(kf[0], x01, fmaf(kf[1], x11, fmaf(kf[2], qs[0][1], kf[3] * qs[1][1])));
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
                        float a = 0.0f;
#pragma unroll
                        for (int g = 0; g < G; ++g)
                            a = fmaf(kf[g], acc[g][2 * rr + k], fmaf(kf[G + g], qs[g][k], a));
                        sc[2 * rr + k] = live ? a : -INFINITY;
                    }
                }
            }

            // ---- online softmax, lazy rescaling ----------------------------
            float mx[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) mx[k] = COLS ? sc[k] : fmaxf(sc[k], sc[2 + k]);
            if (__any_sync(0xffffffffu, mx[0] > m_run[0] + 8.0f || mx[1] > m_run[1] + 8.0f)) {
                float alpha[2];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    float v = mx[k];
                    if constexpr (COLS) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
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

            // ---- combine, group by group: B fragments of P' = p * v_scale by
            // transposition, then the group's M-tiles (V codes^T, nibble passes)
            const int p0 = blk * 16 + j;
            const unsigned char* vrow = st + Lay::VC;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                uint32_t bf0, bf1, bs0, bs1, bt0 = 0u, bt1 = 0u;
                if constexpr (COLS) {
                    const int lp = kr0 + 8 * half;
                    const float vs_ = vscr[lp * 2 * G + g], vb_ = vscr[lp * 2 * G + G + g];
                    bsum[g][0] = fmaf(e[0], vb_, bsum[g][0]);
                    bsum[g][1] = fmaf(e[1], vb_, bsum[g][1]);
                    const float2 v = __fmul2_rn(make_float2(e[0], e[1]), make_float2(vs_, vs_));
                    uint32_t phi, pmid, plo;
                    if constexpr (PARTS == 3) {
                        split3(v.x, v.y, phi, pmid, plo);
                    } else {
                        split2(v.x, v.y, phi, pmid);
                        plo = 0u;
                    }
                    const uint32_t recv = __shfl_xor_sync(0xffffffffu, half ? phi : pmid, 2);
                    bf0 = transpose8x8(half ? recv : phi);
                    bf1 = transpose8x8(half ? pmid : recv);
                    if constexpr (PARTS == 3) {
                        const uint32_t recv_lo = __shfl_xor_sync(0xffffffffu, plo, 2);
                        bs0 = transpose8x8(half ? 0u : plo);
                        bs1 = transpose8x8(half ? 0u : recv_lo);
                    } else {
                        bs0 = bs1 = 0u;
                    }
                } else {
                    uint32_t phi[2], pmid[2], plo[2];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const int lp = kr0 + 8 * rr;
                        const float vs_ = vscr[lp * 2 * G + g], vb_ = vscr[lp * 2 * G + G + g];
                        bsum[g][0] = fmaf(e[2 * rr], vb_, bsum[g][0]);
                        bsum[g][1] = fmaf(e[2 * rr + 1], vb_, bsum[g][1]);
                        const float2 v = __fmul2_rn(make_float2(e[2 * rr], e[2 * rr + 1]),
                                                    make_float2(vs_, vs_));
                        if constexpr (PARTS == 3) {
                            split3(v.x, v.y, phi[rr], pmid[rr], plo[rr]);
                        } else {
                            split2(v.x, v.y, phi[rr], pmid[rr]);
                            plo[rr] = 0u;
                        }
                    }
                    bf0 = transpose8x8(phi[0]);
                    bf1 = transpose8x8(phi[1]);
                    bs0 = transpose8x8(pmid[0]);
                    bs1 = transpose8x8(pmid[1]);
                    if constexpr (PARTS == 3) {
                        bt0 = transpose8x8(plo[0]);
                        bt1 = transpose8x8(plo[1]);
                    }
                }
#pragma unroll
                for (int bb = g * NB / G; bb < (g + 1) * NB / G; ++bb) {
                    const int k0 = BD * bb + VRUN * r;
                    uint32_t wA[VRUN / 4], wB[VRUN / 4], wC[VRUN / 4], wD[VRUN / 4];
                    run_bytes<BITS, VRUN>(vrow + (p0) * RB, k0, wA);
                    run_bytes<BITS, VRUN>(vrow + (p0 + 4) * RB, k0, wB);
                    run_bytes<BITS, VRUN>(vrow + (p0 + 8) * RB, k0, wC);
                    run_bytes<BITS, VRUN>(vrow + (p0 + 12) * RB, k0, wD);
#pragma unroll
                    for (int mm = 0; mm < MTB; ++mm) {
                        // M-tile MTB bb + mm: bytes 2mm, 2mm + 1 of the lane's run
                        const uint32_t xa = wA[mm >> 1], xb = wB[mm >> 1];
                        const uint32_t xc = wC[mm >> 1], xd = wD[mm >> 1];
                        uint32_t l0, h0v, l1, h1v, l2, h2v, l3, h3v;
                        if ((mm & 1) == 0) {
                            byte_nibbles_bf16<0>(xa, xb, l0, h0v, l1, h1v);
                            byte_nibbles_bf16<0>(xc, xd, l2, h2v, l3, h3v);
                        } else {
                            byte_nibbles_bf16<2>(xa, xb, l0, h0v, l1, h1v);
                            byte_nibbles_bf16<2>(xc, xd, l2, h2v, l3, h3v);
                        }
                        float (&o)[4] = oacc[bb * MTB + mm];
                        mma_bf16(o, l0, l1, l2, l3, bf0, bf1);
                        if constexpr (HI) mma_bf16(o, h0v, h1v, h2v, h3v, bf0, bf1);
                        if constexpr (HT == 8 || PARTS == 3) {
                            mma_bf16(o, l0, l1, l2, l3, bs0, bs1);
                            if constexpr (HI) mma_bf16(o, h0v, h1v, h2v, h3v, bs0, bs1);
                        }
                        if constexpr (HT == 8 && PARTS == 3) {
                            mma_bf16(o, l0, l1, l2, l3, bt0, bt1);
                            if constexpr (HI) mma_bf16(o, h0v, h1v, h2v, h3v, bt0, bt1);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- warp partial ----------------------------------------------------
#pragma unroll
        for (int k = 0; k < 2; ++k) {
#pragma unroll
            for (int x = 4; x <= 16; x <<= 1) {
                l_part[k] += __shfl_xor_sync(0xffffffffu, l_part[k], x);
#pragma unroll
                for (int g = 0; g < G; ++g) bsum[g][k] += __shfl_xor_sync(0xffffffffu, bsum[g][k], x);
            }
            if constexpr (COLS) {
                l_part[k] += __shfl_xor_sync(0xffffffffu, l_part[k], 2);
#pragma unroll
                for (int g = 0; g < G; ++g) bsum[g][k] += __shfl_xor_sync(0xffffffffu, bsum[g][k], 2);
            }
        }
        if constexpr (COLS) {
#pragma unroll
            for (int i = 0; i < MT; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) oacc[i][c] += __shfl_xor_sync(0xffffffffu, oacc[i][c], 2);
        }
        named_sync(1, CWARPS * 32);  // every consumer is done with the ring
        float* mo = reinterpret_cast<float*>(smem);                 // [CWARPS][8][DH]
        float* mm_ = mo + CWARPS * 8 * DH;                          // [CWARPS][8]
        float* ml = mm_ + CWARPS * 8;                               // [CWARPS][8]
        float* mb = ml + CWARPS * 8;                                // [CWARPS][8][G]
        if (r == 0 && (!COLS || j < 2)) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int h = 2 * hp + k;
                mm_[warp * 8 + h] = m_run[k];
                ml[warp * 8 + h] = l_part[k];
#pragma unroll
                for (int g = 0; g < G; ++g) mb[(warp * 8 + h) * G + g] = bsum[g][k];
            }
        }
        if (!COLS || j < 2) {
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int bb = i / MTB, mm = i % MTB;
                const int d = BD * bb + VRUN * r + 2 * mm;    // row r; row r + 8 is d + 1
                const int c0 = 2 * j, c1 = 2 * j + 1;
                mo[(warp * 8 + c0) * DH + d] = oacc[i][0];
                mo[(warp * 8 + c1) * DH + d] = oacc[i][1];
                mo[(warp * 8 + c0) * DH + d + 1] = oacc[i][2];
                mo[(warp * 8 + c1) * DH + d + 1] = oacc[i][3];
            }
        }
        // the stream is done: the merge after this grid may launch now (it
        // waits for the grid's completion before it reads a partial)
        pdl_launch_dependents();
        finish_partial<HT, GROUP>(P, smem, tid, warp, lane, split, b, hk, h0, nh, with_new, scale2,
                                  err_flag, part_o, part_m, part_l);
    }
    __syncthreads();
    if (tid == CWARPS * 32 && *(volatile int*)err_flag) {
        for (int s = 0; s < NST && s < n_stages; ++s) {
            const int last = ((n_stages - 1 - s) / NST) * NST + s;
            (void)mbar_wait(&full[s], (last / NST) & 1);
        }
    }
}

}  // namespace mma4
}  // namespace kvq
