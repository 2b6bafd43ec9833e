// The one-kernel sequence split: the split stage's CTAs finish the step
// themselves -- the merge of each unit's splits, the exchange of the ranks'
// records over peer memory and the final merge -- in the same launch.
//
// Every word that crosses CTAs or GPUs is a TAGGED word: 8 bytes, the fp32
// value's bits in the low half and the step number e in the high half, stored
// whole by one relaxed 64-bit store and read by relaxed 64-bit loads. A reader
// that finds tag e in a word has that word of this step; nothing else needs
// ordering, so there is no fence and no flag anywhere in the exchange. (A
// gpu-scope release fence at the end of each split CTA -- the classic "fence,
// then take a ticket" merge -- measured 4 us per step on a B200 here: each
// fence stalls the CTAs sharing its SM. Merging CTAs that polled all their
// words with every thread slowed the streaming CTAs as much.)
//
// Per unit (sequence, cache head, head tile) of n splits:
//   1. every CTA writes its split's partial (O unnormalised, m, l per row)
//      into its own region's partial store, tagged e;
//   2. the CTAs of the unit's last k = min(n, 2 HT) split indices merge it,
//      each one slice (64 dims of a head row; slices slot, slot + k, ...):
//      one warp waits (bounded by %globaltimer) until every split's m and l
//      words carry tag e -- a few loads per pause, so a merging CTA that
//      finished early costs the still-streaming CTAs nothing -- then the CTA
//      reads the slice's n partials in one round trip (re-reading any word
//      not yet tagged e), 160 threads as 10 split groups x 16 four-dim
//      columns;
//   3. one rank: the slice, normalised, into `out`. Several ranks: the
//      slice's record words (tagged) are stored into every rank's region at
//      slot [e & 1][this rank], then the CTA reads its own region's slots
//      [e & 1][p] for every rank p until they carry tag e (bounded), and
//      merges the ranks' records by log-sum-exp from local memory.
// The step number lives in the region (one word per unit); every CTA reads
// it at its start, and the unit's slot-0 merging CTA advances it after it has
// seen tag e on all n partials of its slice -- by then every CTA of the unit
// has read it -- so a replayed CUDA graph of the step stays correct and the
// host passes no step number. A rank stores into slot [e & 1][r] of a peer at
// step e + 2 only after its step e + 1 read that peer's step-(e + 1) records,
// which the peer writes in a launch that starts after its step e (and all its
// reads of that slot) finished: the double buffer is never overwritten while
// read. No collective, no multicast: peer stores and local loads only.
//
// Waits: only the k merging CTAs of a unit wait, at most units * k CTAs in
// all (k <= 2 HT), so the unit's other CTAs always find an SM (the host
// checks units * k against the resident capacity). A wait that runs out
// writes the region's status word and NaN rows, and the kernel returns.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "kvq_b200.h"
#include "kvq_common.cuh"

namespace kvq {
namespace fused {

constexpr int MAX_RANKS = KVQ_PEER_MAX_RANKS;
// status word, at the same offset as the two-kernel peer merge's region
constexpr uint64_t STATUS = 8;
constexpr uint32_t STATUS_TIMEOUT = 1;    // a peer's record did not arrive in time
constexpr uint32_t STATUS_SPLITS = 3;     // a unit's partials did not all arrive in time; the
                                          // region's step counts are no longer in step
constexpr uint64_t CTRL = 256;
constexpr uint32_t DH = 128;
constexpr uint32_t WORDS = DH + 2;        // tagged words per row: O [DH], m, l
// partial store capacity in (split, row) pairs: 64 splits of every row, or
// 16384 pairs when that is less (two splits of every row at the least)
constexpr uint64_t MAX_SPLITS = 64;
constexpr uint64_t MIN_PART_ROWS = 16384;

__host__ __device__ constexpr uint64_t align256(uint64_t x) { return (x + 255) / 256 * 256; }

__host__ __device__ constexpr uint64_t part_rows(uint64_t rows) {
    return MAX_SPLITS * rows < MIN_PART_ROWS ? MAX_SPLITS * rows
                                             : (MIN_PART_ROWS > 2 * rows ? MIN_PART_ROWS : 2 * rows);
}

// Byte offsets inside one region (rows = b_rows * n_heads). The per-unit
// arrays are sized by rows (a unit holds at least one row).
struct Layout {
    uint64_t epochs;        // [rows] u32: steps done per unit
    uint64_t partials;      // [part_rows][WORDS] tagged words
    uint64_t part_rows;
    uint64_t records;       // [2][world][rows][WORDS] tagged words
    uint64_t record_bytes;  // one rank's record
    uint64_t total;
};

__host__ __device__ inline Layout region_layout(uint32_t rows, uint32_t world) {
    Layout L{};
    L.epochs = CTRL;
    L.partials = L.epochs + align256(4ull * rows);
    L.part_rows = part_rows(rows);
    L.records = L.partials + align256(8ull * WORDS * L.part_rows);
    L.record_bytes = align256(8ull * WORDS * rows);
    L.total = L.records + 2ull * world * L.record_bytes;
    return L;
}

// Kernel argument: the ranks' regions as mapped here, this rank, the layout.
struct Fused {
    unsigned char* region[MAX_RANKS];
    uint32_t world, rank;
    Layout L;
    uint64_t timeout_ns;
    __half* out;          // [b_rows * n_heads, 128]
};

__device__ __forceinline__ uint32_t* epoch_word(const Fused& F, uint32_t unit) {
    return reinterpret_cast<uint32_t*>(F.region[F.rank] + F.L.epochs) + unit;
}
__device__ __forceinline__ uint64_t* partials(const Fused& F) {
    return reinterpret_cast<uint64_t*>(F.region[F.rank] + F.L.partials);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// two tagged words; SYS: at system scope (words other GPUs store)
template <bool SYS>
__device__ __forceinline__ void ld2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    if constexpr (SYS)
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void st2_sys(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ uint32_t tag_of(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float val_of(uint64_t w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ uint64_t word(float v, uint32_t tag) {
    return ((uint64_t)tag << 32) | __float_as_uint(v);
}

// The six tagged words a thread takes from one row at `w`: O columns c4 ..
// c4 + 3, then the row's m and l.
template <bool SYS>
__device__ __forceinline__ void read6(const uint64_t* w, uint32_t c4, uint64_t (&x)[6]) {
    ld2<SYS>(w + c4, x[0], x[1]);
    ld2<SYS>(w + c4 + 2, x[2], x[3]);
    ld2<SYS>(w + DH, x[4], x[5]);
}
__device__ __forceinline__ bool all_tagged(const uint64_t (&x)[6], uint32_t e) {
    return tag_of(x[0]) == e && tag_of(x[1]) == e && tag_of(x[2]) == e && tag_of(x[3]) == e &&
           tag_of(x[4]) == e && tag_of(x[5]) == e;
}
// Re-read until all six words carry tag e, or the deadline passes (false).
template <bool SYS>
__device__ __forceinline__ bool settle6(const uint64_t* w, uint32_t c4, uint32_t e, uint64_t deadline,
                                        uint64_t (&x)[6]) {
    uint32_t spins = 0;
    while (!all_tagged(x, e)) {
        if ((++spins & 7u) == 0 && globaltimer() > deadline) return false;
        __nanosleep(100);
        read6<SYS>(w, c4, x);
    }
    return true;
}

constexpr int TAIL_THREADS = 160;            // the split stage's CTA size
constexpr int SLICE = 64;                    // dims of a row one merging CTA takes
constexpr int COLS = SLICE / 4;              // 4-dim columns of a slice
constexpr int SGROUPS = TAIL_THREADS / COLS; // split groups summed in parallel
constexpr int BATCH = 6;                     // splits a thread requests at once
static_assert(MAX_RANKS * COLS <= TAIL_THREADS, "one thread per rank and column");

// The tail of one split CTA (all TAIL_THREADS threads, shared memory free):
// this CTA's tagged partial is stored; the CTAs of the unit's last k split
// indices merge and finish the step, each taking slices (half rows) slot,
// slot + k, ....
template <int HT>
__device__ __forceinline__ void tail(const Problem& P, const Fused& F, uint32_t e, unsigned char* smem) {
    __shared__ int s_bad;
    const int tid = threadIdx.x;
    const uint32_t H = P.n_heads;
    const uint32_t rows = P.b_rows * H;
    const uint32_t tile_h = blockIdx.y % P.head_tiles;
    const uint32_t hk = blockIdx.y / P.head_tiles;
    const uint32_t b = blockIdx.z;
    const uint32_t h0 = hk * P.r + tile_h * HT;
    const int nh = min(HT, (int)(P.r - tile_h * HT));
    const int slices = nh * (DH / SLICE);
    const uint32_t unit = b * gridDim.y + blockIdx.y;
    const uint32_t n = P.n_splits;
    constexpr uint32_t KMAX = HT * (DH / SLICE);
    const uint32_t k = n < KMAX ? n : KMAX;
    const uint32_t par = e & 1u;

    // the unit's last k split indices merge; the others are done
    if (blockIdx.x + k < n) return;
    const int slot = (int)(blockIdx.x + k - n);
    unsigned char* self = F.region[F.rank];
    unsigned int* status = reinterpret_cast<unsigned int*>(self + STATUS);
    const uint64_t* part = partials(F);
    const float qnan = __int_as_float(0x7fc00000);
    const uint64_t deadline = globaltimer() + F.timeout_ns;

    // split groups' running max, l and O columns meet in shared memory (the
    // split stage's ring is drained); so do the ranks' records
    float* s_m = reinterpret_cast<float*>(smem);                              // [SGROUPS]
    float* s_l = s_m + SGROUPS;                                               // [SGROUPS]
    float4* s_sum = reinterpret_cast<float4*>(smem + 128);                    // [SGROUPS][COLS]
    float* r_m = reinterpret_cast<float*>(smem + 128 + 16 * SGROUPS * COLS);  // [MAX_RANKS]
    float* r_l = r_m + MAX_RANKS;                                             // [MAX_RANKS]
    float4* r_o = reinterpret_cast<float4*>(r_l + MAX_RANKS);                 // [MAX_RANKS][COLS]
    __syncthreads();                                // the split stage is done with shared memory
    if (tid == 0) s_bad = 0;
    __syncthreads();

    for (int sl = slot; sl < slices; sl += (int)k) {
        const int j = sl / (DH / SLICE);
        const uint32_t row = b * H + h0 + j;
        const int col = tid % COLS, sg = tid / COLS;
        const uint32_t c4 = (uint32_t)(sl % (DH / SLICE)) * SLICE + 4 * col;   // first dim of the column
        // one warp waits until every split's m and l words of the row carry
        // tag e (each lane requests all of its splits at once, then re-reads
        // the missing ones after a pause): a waiting merging CTA costs the
        // streaming CTAs two loads per lane and pause. The O words, stored
        // with them, are then read in one round trip.
        if (tid < 32) {
            constexpr int PER_LANE = (int)(MAX_SPLITS + 31) / 32;
            uint64_t mw[PER_LANE], lw[PER_LANE];
            bool ready = true;
            for (uint32_t s0 = tid; s0 < n && ready; s0 += 32 * PER_LANE) {
#pragma unroll
                for (int u = 0; u < PER_LANE; ++u) {
                    const uint32_t s = s0 + 32 * u;
                    mw[u] = lw[u] = (uint64_t)e << 32;
                    if (s < n) ld2<false>(part + ((size_t)s * rows + row) * WORDS + DH, mw[u], lw[u]);
                }
                uint32_t spins = 0;
                for (;;) {
                    bool all = true;
#pragma unroll
                    for (int u = 0; u < PER_LANE; ++u) all = all && tag_of(mw[u]) == e && tag_of(lw[u]) == e;
                    if (all) break;
                    if ((++spins & 7u) == 0 && globaltimer() > deadline) {
                        ready = false;
                        break;
                    }
                    __nanosleep(200);
#pragma unroll
                    for (int u = 0; u < PER_LANE; ++u) {
                        const uint32_t s = s0 + 32 * u;
                        if (s < n && (tag_of(mw[u]) != e || tag_of(lw[u]) != e))
                            ld2<false>(part + ((size_t)s * rows + row) * WORDS + DH, mw[u], lw[u]);
                    }
                }
            }
            __syncwarp();
        }
        __syncthreads();
        // thread (sg, col) takes splits sg, sg + SGROUPS, ...: BATCH splits'
        // words requested together, then settled (re-read where a tag is not
        // yet e) and folded into a running max (online rescaling; natural-log
        // units, as the partials)
        float M = -INFINITY, lsum = 0.0f;
        bool poisoned = false, ok = true;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t s0 = sg; s0 < n; s0 += SGROUPS * BATCH) {
            uint64_t x[BATCH][6];
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const uint32_t s = s0 + u * SGROUPS;
                if (s < n) read6<false>(part + ((size_t)s * rows + row) * WORDS, c4, x[u]);
            }
            float mv[BATCH];
            float Mb = M;
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const uint32_t s = s0 + u * SGROUPS;
                mv[u] = -INFINITY;
                if (s < n) {
                    if (ok) ok = settle6<false>(part + ((size_t)s * rows + row) * WORDS, c4, e, deadline, x[u]);
                    mv[u] = val_of(x[u][4]);
                }
                Mb = fmaxf(Mb, mv[u]);
                poisoned |= mv[u] != mv[u];
            }
            if (Mb == -INFINITY) continue;           // only empty splits so far
            const float c = M == -INFINITY ? 0.0f : expf(M - Mb);
            acc.x *= c; acc.y *= c; acc.z *= c; acc.w *= c;
            lsum *= c;
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                if (s0 + u * SGROUPS >= n) continue;
                // an empty split (m = -inf) adds nothing; a poisoned one (NaN m)
                // makes the row NaN
                const float w = mv[u] == -INFINITY ? 0.0f : expf(mv[u] - Mb);
                lsum = fmaf(val_of(x[u][5]), w, lsum);
                acc.x = fmaf(val_of(x[u][0]), w, acc.x);
                acc.y = fmaf(val_of(x[u][1]), w, acc.y);
                acc.z = fmaf(val_of(x[u][2]), w, acc.z);
                acc.w = fmaf(val_of(x[u][3]), w, acc.w);
            }
            M = Mb;
        }
        if (!ok) {
            atomicExch(status, STATUS_SPLITS);
            s_bad = 1;
        }
        if (poisoned) M = lsum = qnan;               // a NaN split poisons the row
        if (col == 0) {
            s_m[sg] = M;
            s_l[sg] = lsum;
        }
        s_sum[sg * COLS + col] = acc;
        __syncthreads();
        if (tid < COLS) {
            float m = -INFINITY;
#pragma unroll
            for (int g = 0; g < SGROUPS; ++g) m = fmaxf(m, s_m[g]);
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            float l = 0.0f;
#pragma unroll
            for (int g = 0; g < SGROUPS; ++g) {
                if (s_m[g] == -INFINITY) continue;
                const float w = expf(s_m[g] - m);
                const float4 xs = s_sum[g * COLS + col];
                l = fmaf(s_l[g], w, l);
                o.x = fmaf(xs.x, w, o.x);
                o.y = fmaf(xs.y, w, o.y);
                o.z = fmaf(xs.z, w, o.z);
                o.w = fmaf(xs.w, w, o.w);
            }
            const bool bad = s_bad != 0;
            if (F.world == 1) {
                __half2* dst = reinterpret_cast<__half2*>(F.out + (size_t)row * DH + c4);
                dst[0] = bad ? __floats2half2_rn(qnan, qnan) : __floats2half2_rn(o.x / l, o.y / l);
                dst[1] = bad ? __floats2half2_rn(qnan, qnan) : __floats2half2_rn(o.z / l, o.w / l);
            } else {
                // the slice's record words into every rank's region, slot
                // [par][this rank] (both slices of a row store the same m and
                // l); a NaN m poisons the row on every rank when this one failed
                if (bad) m = qnan;
                for (uint32_t p = 0; p < F.world; ++p) {
                    uint64_t* rec = reinterpret_cast<uint64_t*>(
                                        F.region[p] + F.L.records + (par * F.world + F.rank) * F.L.record_bytes) +
                                    (size_t)row * WORDS;
                    st2_sys(rec + c4, word(o.x, e), word(o.y, e));
                    st2_sys(rec + c4 + 2, word(o.z, e), word(o.w, e));
                    if (col == 0) st2_sys(rec + DH, word(m, e), word(l, e));
                }
            }
        }
        __syncthreads();   // s_m, s_l and s_sum are reused by the next slice
    }
    // every CTA of the unit has read the step number (slot 0 saw all their
    // partials tagged with it): advance it for the next launch
    if (slot == 0 && tid == 0) st_relaxed_gpu(epoch_word(F, unit), e);
    if (F.world == 1) return;

    // every rank's record of this CTA's slices, from the local region: thread
    // (p, col) reads rank p's words of column col, then 16 threads merge the
    // ranks in rank order
    const bool bad_local = s_bad != 0;
    for (int sl = slot; sl < slices; sl += (int)k) {
        const int j = sl / (DH / SLICE);
        const uint32_t row = b * H + h0 + j;
        const int col = tid % COLS, p = tid / COLS;
        const uint32_t c4 = (uint32_t)(sl % (DH / SLICE)) * SLICE + 4 * col;
        bool arrived = true;
        if ((uint32_t)p < F.world) {
            const uint64_t* rec = reinterpret_cast<const uint64_t*>(
                                      self + F.L.records + (par * F.world + p) * F.L.record_bytes) +
                                  (size_t)row * WORDS;
            uint64_t x[6];
            read6<true>(rec, c4, x);
            arrived = settle6<true>(rec, c4, e, deadline, x);
            r_o[p * COLS + col] = make_float4(val_of(x[0]), val_of(x[1]), val_of(x[2]), val_of(x[3]));
            if (col == 0) {
                r_m[p] = val_of(x[4]);
                r_l[p] = val_of(x[5]);
            }
        }
        const bool ok = __syncthreads_and(arrived) != 0;
        if (tid < COLS) {
            float m = -INFINITY;
            for (uint32_t q = 0; q < F.world; ++q) m = fmaxf(m, r_m[q]);
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            float l = 0.0f;
            for (uint32_t q = 0; q < F.world; ++q) {
                const float w = r_m[q] == -INFINITY ? 0.0f : expf(r_m[q] - m);
                if (w != 0.0f) {
                    const float4 xs = r_o[q * COLS + tid];
                    l = fmaf(r_l[q], w, l);
                    o.x = fmaf(xs.x, w, o.x);
                    o.y = fmaf(xs.y, w, o.y);
                    o.z = fmaf(xs.z, w, o.z);
                    o.w = fmaf(xs.w, w, o.w);
                }
            }
            if (!ok && tid == 0) atomicExch(status, STATUS_TIMEOUT);
            const bool bad = bad_local || !ok;
            __half2* dst = reinterpret_cast<__half2*>(F.out + (size_t)row * DH + c4);
            dst[0] = bad ? __floats2half2_rn(qnan, qnan) : __floats2half2_rn(o.x / l, o.y / l);
            dst[1] = bad ? __floats2half2_rn(qnan, qnan) : __floats2half2_rn(o.z / l, o.w / l);
        }
        __syncthreads();   // r_* are reused by the next slice
    }
}

}  // namespace fused
}  // namespace kvq
