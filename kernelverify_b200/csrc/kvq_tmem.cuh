// Warp-specialised, persistent 5th-generation tensor-core decode kernel with
// both MMA A operands in tensor memory, for fp16 steps over 4-bit caches,
// head_dim 128, group 64, up to 8 query heads per cache head.
//
// One CTA per SM walks a list of work items -- (batch row, cache head, head
// tile, T split), consecutive items of a CTA gridDim.x apart -- through one
// continuous pipeline of 128-position tiles. Twenty warps in five
// warpgroups, registers re-split between them with setmaxnreg:
//
//   warpgroup 0 (32 registers): warp 0 producer, cp.async.bulk (1-D TMA) of
//               each tile's K codes, V codes and the four fp16 scale/bias runs
//               into an NST-deep ring (mbarrier transaction bytes); warp 1 the
//               score MMA issuer, S[pos, n] = sum_k Kc[pos, k] Qg[k, n] (A in
//               tensor memory, B = Qg in shared memory); warp 2 the combine
//               MMA issuer, O[d, n'] = sum_pos Vc[d, pos] P'[pos, n'] (A in
//               tensor memory, B = P' in shared memory); one thread each, every
//               MMA a tcgen05.mma kind::f16 with M = 128. Warp 3 idles.
//   warpgroup 1 K unpack: 16-byte reads of the raw K rows (four lanes per
//               row, conflict-free) become exact fp16 1024 + code, stored to
//               tensor memory with 16x256b stores (TMEM lane = position), with
//               each position's scale/bias pairs in four spare columns; per
//               item also the Qg operand (each head's q restricted to one
//               quantisation group, n = group * 8 + head) and its per-group
//               q sums.
//   warpgroup 2 V unpack: ldmatrix.trans reads 8x8 tiles of 16-bit code pairs
//               across positions; each register becomes exact bf16 128 + code
//               of one dim at two positions (TMEM lane = dim).
//   warpgroups 3 and 4 (128 registers) softmax, even and odd tiles: thread =
//               position (TMEM lane). It reads its scores and scales, applies
//                 score[h] = sum_g ks_g (S_gh - 1024 Qsum_gh) + kb_g Qsum_gh,
//               the lazy online softmax (the reference point moves only when a
//               score exceeds it by 2^8, decided by a warpgroup vote), and
//               writes P' = p * v_scale as three bf16 parts (binary32-class,
//               |error| <= 2^-23 |P'|) into the shared-memory B operand; the
//               V-side bias term sum_pos p (b - 128 s) is summed in registers.
//               The same thread owns one dim of O: it reads that row of each
//               of its tiles' O from tensor memory and accumulates it in
//               registers. Each warpgroup keeps its own (O, m, l) over its
//               tiles; the two are merged by log-sum-exp at the item's end.
//
// Every operand hand-off is an mbarrier with bounded waits; tensor memory
// (512 columns) is allocated once per CTA and always freed. Precision: K-side
// products fp16 x fp16 are exact, accumulated in fp32 (with the 1024 offset,
// taken out per group through Qsum); V-side P' parts against exact bf16
// codes; fp16 outputs.
#pragma once

#include "kvq_umma.cuh"

namespace kvq {
namespace tmem4 {

using mma4::and_or;
using mma4::bulk_g2s;
using mma4::evict_first_policy;
using mma4::ex2;
using mma4::mbar_arrive;
using mma4::mbar_expect_tx;
using mma4::mbar_init;
using mma4::mbar_wait;
using mma4::mbar_try_wait;
using mma4::named_sync;
using mma4::s_addr;
using mma4::split3;
using umma::consumers_any;
using umma::fence_async_smem;
using umma::idesc;
using umma::sdesc;
using umma::tc_fence_after;
using umma::tc_fence_before;
using umma::tmem_alloc;
using umma::tmem_dealloc;
using umma::tmem_ld16;
using umma::tmem_relinquish;
using umma::tmem_wait_ld;
using umma::tmem_wait_st;
using umma::umma_commit;

constexpr int TP = 128;                 // positions per tile
constexpr int DH = 128;
constexpr int G = 2;                    // quantisation groups of 64 per row
constexpr int ROWB = DH / 2;            // code bytes per row
#ifndef KVQ_TMEM_STAGES
#define KVQ_TMEM_STAGES 6
#endif
constexpr int NST = KVQ_TMEM_STAGES;    // raw ring depth
constexpr int WARPS = 20;
constexpr int THREADS = 32 * WARPS;
constexpr int W_PROD = 0, W_MMA = 1, W_MMA_C = 2, W_K = 4, W_V = 8, W_S = 12;   // W_S: two warpgroups
// Registers per thread: the launch's (every warp) and, after setmaxnreg, the
// single-thread roles' and the softmax warpgroups'. 4*32*REG_LOW +
// 8*32*REG_LAUNCH + 8*32*REG_SOFTMAX must not exceed THREADS * REG_LAUNCH,
// and the host refuses to launch a build whose register count is not
// REG_LAUNCH (a re-split over budget would wait forever).
constexpr int REG_LAUNCH = 96, REG_LOW = 32, REG_SOFTMAX = 128;
static_assert(4 * 32 * REG_LOW + 8 * 32 * REG_LAUNCH + 8 * 32 * REG_SOFTMAX <= THREADS * REG_LAUNCH,
              "register re-split over the launch budget");
constexpr int XCH_BAR = 3;              // named barrier of both softmax warpgroups (256 threads)
// Buffer depths: K operands (with their scale columns), V operands, score
// accumulators, Qg operands. Score MMAs run up to NAK tiles behind the K unpack
// and NS tiles ahead of the softmax reads, the V unpack NAV tiles ahead of the
// combine MMAs; Qg buffer i is reused NBQ items later.
constexpr int NAK = 2, NAV = 3, NS = 4, NBQ = 3;
constexpr int QRING = 4;                // per-item q-sum slots
constexpr uint32_t TMEM_COLS = 512;

template <int HT>
struct Cfg {
    static_assert(HT == 4 || HT == 8, "head tile");
    // O columns per group, (part, head): HT = 4 pads 12 to 16, HT = 8 uses 24
    static constexpr int GW = HT == 4 ? 16 : 24;
    static constexpr int N_O = G * GW;                 // combine N
    static constexpr int N_S = 16;                     // score N: group * 8 + head
    // tensor memory columns (lane = position for AK and S, lane = dim for AV and O)
    static constexpr uint32_t AK0 = 0;                 // [NAK][64]
    static constexpr uint32_t AV0 = 64 * NAK;          // [NAV][64]
    static constexpr uint32_t S0 = AV0 + 64 * NAV;     // [NS][16]
    static constexpr uint32_t O0 = S0 + 16 * NS;       // [2][N_O]
    // [2][8]: a position's fp16x2 k_scale, k_bias, v_scale, v_bias (columns
    // 0..3), written beside its K operand so the softmax reads them with its scores
    static constexpr uint32_t SC0 = O0 + 2 * N_O;      // [NAK][8]
    static_assert(SC0 + 8 * NAK <= TMEM_COLS, "tensor memory");
    // shared memory
    static constexpr int KC = 0;                       // raw stage: K codes [TP][64]
    static constexpr int VC = KC + TP * ROWB;          //            V codes [TP][64]
    static constexpr int KS = VC + TP * ROWB;          //            fp16 [TP][G] each
    static constexpr int KB = KS + TP * G * 2;
    static constexpr int VS = KB + TP * G * 2;
    static constexpr int VB = VS + TP * G * 2;
    static constexpr int STAGE = VB + TP * G * 2;
    static constexpr int BP = NST * STAGE;             // P' [4]: bf16, MN-major core matrices
    static constexpr int BP_LBO = (N_O / 8) * 128;     // bytes between 8-position row blocks
    static constexpr int BP_BYTES = TP * N_O * 2;
    static constexpr int BQ = BP + 4 * BP_BYTES;       // Qg [NBQ]: fp16, K-major core matrices
    static constexpr int BQ_BYTES = N_S * DH * 2;
    static constexpr int QS = BQ + NBQ * BQ_BYTES;     // fp32 [QRING][G][8] per-group q sums
    static constexpr int XCH = QS + QRING * G * 8 * 4; // fp32 [2][(128 + 2) * HT]: odd -> even warpgroup
    static constexpr int XCH_FLOATS = (128 + 2) * HT;
    static constexpr int BAR = XCH + 2 * XCH_FLOATS * 4;
    // raw_full[NST], raw_empty[NST], ak_full[NAK], s_full[NS], s_empty[NS],
    // av_full[NAV], av_empty[NAV], [2] each of p_full, o_full, o_empty, one
    // drain barrier per issuer, and q_full[QRING]
    static constexpr int NBAR = 2 * NST + NAK + 2 * NS + 2 * NAV + 6 + 2 + QRING;
    static constexpr int MISC = BAR + (NBAR * 8 + 15) / 16 * 16;
    static constexpr int TMEM_SLOT = MISC;             // uint32 TMEM base address
    static constexpr int ERR = MISC + 4;               // int, any role's failed wait
    static constexpr int STALL = MISC + 8;             // int, a stall was reported
    static constexpr int FLAGS = MISC + 16;            // int [2 warpgroups][2][4]: tile votes
    static constexpr int RED = MISC + 80;              // fp32 [2 warpgroups][RED_FLOATS]
    static constexpr int RED_FLOATS = 4 * HT * (1 + G + 1) + HT;
    static constexpr int BYTES = RED + 2 * RED_FLOATS * 4 + 16;
    static_assert(STAGE % 128 == 0 && BP % 1024 == 0 && BQ % 128 == 0 && QS % 16 == 0 &&
                  XCH % 16 == 0 && BAR % 8 == 0 && FLAGS % 16 == 0, "alignment");
};

template <int HT>
constexpr size_t smem_bytes() { return Cfg<HT>::BYTES; }

// ---- PTX wrappers ------------------------------------------------------------
// 16 TMEM lanes x 256 bits, 8 repetitions along the columns: thread t holds,
// per repetition n, lane (t/4) columns 8n + 2(t%4) + {0, 1} in v[4n], v[4n+1]
// and lane (t/4) + 8, the same columns, in v[4n+2], v[4n+3].
__device__ __forceinline__ void tmem_st_16x256b_x8(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_16x256b_x1(uint32_t taddr, uint32_t v0, uint32_t v1, uint32_t v2,
                                                   uint32_t v3) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v0),
                 "r"(v1), "r"(v2), "r"(v3)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Every wait of this kernel gives up after WAIT_NS of device time.
constexpr uint64_t WAIT_NS = 1000000000ull;
// A test that may suspend the thread (up to `hint_ns`) until the phase
// completes, so a waiting warp sleeps instead of re-issuing tests that take
// issue slots from the warps doing work on the same scheduler.
__device__ __forceinline__ bool try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(mma4::s_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Roles with slack (the producer, the K and V unpack run tiles ahead) sleep in
// their waits; the softmax and the MMA issuers, on the critical path, poll.
constexpr uint32_t SLEEP_HINT_NS = 1000000;
template <bool SLEEP = false>
__device__ __forceinline__ bool twait(uint64_t* bar, uint32_t parity) {
    const auto test = [&]() {
        return SLEEP ? try_wait_sleep(bar, parity, SLEEP_HINT_NS) : mma4::mbar_try_wait(bar, parity);
    };
    if (test()) return true;
    const uint64_t t0 = global_ns();
    do {
        if (test()) return true;
    } while (global_ns() - t0 < WAIT_NS);
    return false;
}
// The first wait to give up (over all CTAs of the launches since load)
// records where: {site, tile, CTA, 1}; the kernel's partials are poisoned with
// NaN either way.
__device__ unsigned int g_stall[4];
__device__ __forceinline__ void report_stall(int* first, int site, uint32_t tile) {
    if (atomicCAS(first, 0, 1) == 0 && atomicCAS(&g_stall[3], 0u, 1u) == 0u) {
        g_stall[0] = (unsigned)site;
        g_stall[1] = tile;
        g_stall[2] = blockIdx.x;
    }
}
// Bounded waits on up to three mbarrier phases at once. Every phase is tested
// before any is waited on: a test of a phase that completed long ago still
// takes a shared-memory round trip, and independent tests overlap.
template <bool SLEEP = false>
__device__ __forceinline__ bool wait_all(uint64_t* b0, uint32_t p0, uint64_t* b1 = nullptr,
                                         uint32_t p1 = 0, uint64_t* b2 = nullptr, uint32_t p2 = 0) {
    const bool d0 = mma4::mbar_try_wait(b0, p0);
    const bool d1 = b1 == nullptr || mma4::mbar_try_wait(b1, p1);
    const bool d2 = b2 == nullptr || mma4::mbar_try_wait(b2, p2);
    if (d0 && d1 && d2) return true;
    return (d0 || twait<SLEEP>(b0, p0)) && (d1 || twait<SLEEP>(b1, p1)) && (d2 || twait<SLEEP>(b2, p2));
}
// per-warpgroup register re-split (every thread of the warpgroup executes it)
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
        "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
// D[tmem] (+)= A[tmem] * B[smem descriptor]; kind::f16, one CTA
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t id,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(id), "r"(accumulate)
        : "memory");
}
// four 8x8 b16 tiles, transposed: lanes 8i..8i+7 give tile i's row addresses;
// thread t receives element (row 2(t%4), column t/4) in the low half and
// (row 2(t%4)+1, column t/4) in the high half of x[i]
__device__ __forceinline__ void ldsm_x4_trans(uint32_t saddr, uint32_t (&x)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3])
                 : "r"(saddr));
}
// fp16x2 (1024 + 16c) -> (1024 + c), exact
__device__ __forceinline__ uint32_t h2_hi_to_lo(uint32_t x) {
    __half2 v = __hfma2(*reinterpret_cast<__half2*>(&x), __half2(__half(0.0625f), __half(0.0625f)),
                        __half2(__half(960.0f), __half(960.0f)));
    return *reinterpret_cast<uint32_t*>(&v);
}

// K index k of the score MMA (16 per K-step, 2 per TMEM column) <-> head dim,
// as the K unpack places codes: word i of a lane's 16-byte chunk j holds dims
// 32j + 8i .. +7; its register m (m = 0..3) holds dims (m, m + 4) and goes to
// repetition n = 2i + m/2, column 8n + 2j + m%2.
__device__ __forceinline__ int kdim(int k) {
    const int n = k >> 4, j = (k >> 2) & 3, c = (k >> 1) & 1, hf = k & 1;
    return 32 * j + 8 * (n >> 1) + 2 * (n & 1) + c + 4 * hf;
}
// K index of the combine MMA (positions, 2 per TMEM column) of tile position
// p, as the V unpack places them: repetition n = p/16 holds positions
// 16n + 8c + 2j + {0, 1} in column 8n + 2j + c.
__device__ __forceinline__ int vkpos(int p) {
    const int n = p >> 4, x = p & 15, c = x >> 3, j = (x & 7) >> 1, hf = x & 1;
    return 16 * n + 4 * j + 2 * c + hf;
}
// head dim of combine row (TMEM lane) L: lane 32q + 8s + r holds dim 32q + 4r + s
__device__ __forceinline__ int vdim(int L) { return (L & ~31) + 4 * (L & 7) + ((L & 31) >> 3); }

struct Item {
    uint32_t b, hk, split, lo, hi, h0;
    int nh, n_tiles;
    bool with_new;
    uint64_t rowbase;
};

template <int HT>
__device__ __forceinline__ Item item_of(const Problem& P, uint32_t idx) {
    Item it;
    it.split = idx % P.n_splits;
    uint32_t unit = idx / P.n_splits;
    const uint32_t tile_h = unit % P.head_tiles;
    unit /= P.head_tiles;
    it.hk = unit % P.n_kv_heads;
    it.b = unit / P.n_kv_heads;
    it.h0 = it.hk * P.r + tile_h * HT;
    it.nh = min(HT, (int)(P.r - tile_h * HT));
    uint32_t len = P.t_cached;
    if (P.seq_lens != nullptr) len = min((uint32_t)max(P.seq_lens[it.b], 0), P.t_cached);
    const uint32_t end = min(P.t_end, len);
    it.lo = P.t_begin + it.split * P.chunk;
    it.hi = min(end, it.lo + P.chunk);
    it.n_tiles = it.hi > it.lo ? (int)((it.hi - it.lo + TP - 1) / TP) : 0;
    it.with_new = P.has_new_entry && it.split == P.n_splits - 1;
    it.rowbase = (uint64_t)it.b * P.cache_batch_stride + (uint64_t)it.hk * P.t_stride;
    return it;
}

// -----------------------------------------------------------------------------
template <int HT>
__global__ void __launch_bounds__(THREADS, 1)
decode_kernel(Problem P, uint32_t n_items, float* __restrict__ part_o, float* __restrict__ part_m,
              float* __restrict__ part_l) {
    using C = Cfg<HT>;
    constexpr float L2E = 1.4426950408889634f;
    constexpr float LN2 = 0.6931471805599453f;
    constexpr uint32_t ID_S = idesc(false, false, false, C::N_S, 128);
    constexpr uint32_t ID_V = idesc(true, false, true, C::N_O, 128);
    const float scale2 = P.scale * L2E;   // scores in log2 units

    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::BAR);
    uint64_t* raw_full = bar;
    uint64_t* raw_empty = bar + NST;
    // Tile gt's K operand and scale columns are buffer gt % NAK, its scores
    // gt % NS, its V operand gt % NAV, its P' pair and O buffer gt % 2
    // (softmax warpgroup gt % 2 takes the tile). s_empty (the softmax read a
    // tile's scores and scales, so its scores were computed) frees the tile's
    // K operand and, NBQ - 1 items on, its Qg buffer; av_empty (combine done)
    // frees its V operand, o_full (the same) its P' buffer and O for the
    // softmax warpgroup that owns it.
    uint64_t* ak_full = bar + 2 * NST;    // [NAK]
    uint64_t* s_full = ak_full + NAK;     // [NS]
    uint64_t* s_empty = s_full + NS;      // [NS]
    uint64_t* av_full = s_empty + NS;     // [NAV]
    uint64_t* av_empty = av_full + NAV;   // [NAV]: a tile's combine has read its V operand
    uint64_t* p_full = av_empty + NAV;    // [2]
    uint64_t* o_full = p_full + 2;
    uint64_t* o_empty = p_full + 4;
    uint64_t* drain = p_full + 6;         // [2]: one per MMA issuer
    uint64_t* q_full = p_full + 8;        // [QRING]: an item's q sums are written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::TMEM_SLOT);
    volatile int* err = reinterpret_cast<volatile int*>(smem + C::ERR);
    int* stall = reinterpret_cast<int*>(smem + C::STALL);
    const float* qsums = reinterpret_cast<const float*>(smem + C::QS);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, wg = warp >> 2;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 8);           // every K and V unpack warp
        }
        for (int i = 0; i < NAK; ++i) mbar_init(&ak_full[i], 4);
        for (int i = 0; i < NS; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], 4);
        }
        for (int i = 0; i < NAV; ++i) {
            mbar_init(&av_full[i], 4);
            mbar_init(&av_empty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&p_full[b], 4);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], 4);
            mbar_init(&drain[b], 1);
        }
        for (int s = 0; s < QRING; ++s) mbar_init(&q_full[s], 4);
        *err = 0;
        *stall = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < 16) reinterpret_cast<int*>(smem + C::FLAGS)[tid] = 0;
    if (warp == W_MMA) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    // P' columns past the (group, part, head) ones stay zero for the kernel's life
    for (int i = tid; i < 4 * C::BP_BYTES / 16; i += THREADS)
        reinterpret_cast<uint4*>(smem + C::BP)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (wg == 0) {
        regs_dec<REG_LOW>();
        if (warp == W_PROD && lane == 0) {
            // ------------------------------ producer --------------------------
            const uint64_t pol = evict_first_policy();
            const unsigned char* kw = reinterpret_cast<const unsigned char*>(P.k_wq);
            const unsigned char* vw = reinterpret_cast<const unsigned char*>(P.v_wq);
            const unsigned char* ks = static_cast<const unsigned char*>(P.k_scales);
            const unsigned char* kb = static_cast<const unsigned char*>(P.k_biases);
            const unsigned char* vs = static_cast<const unsigned char*>(P.v_scales);
            const unsigned char* vb = static_cast<const unsigned char*>(P.v_biases);
            uint32_t gt = 0;
            for (uint32_t idx = blockIdx.x; idx < n_items && !*err; idx += gridDim.x) {
                const Item it = item_of<HT>(P, idx);
                for (int i = 0; i < it.n_tiles; ++i, ++gt) {
                    const uint32_t slot = gt % NST, round = gt / NST;
                    if (gt >= NST && !twait<true>(&raw_empty[slot], (round - 1) & 1)) {
                        report_stall(stall, 1, gt);
                        *err = 1;
                        break;
                    }
                    const uint32_t t0 = it.lo + i * TP;
                    const uint32_t n = min((uint32_t)TP, it.hi - t0);
                    const uint32_t nr = (n + 7) & ~7u;
                    const uint64_t row = it.rowbase + t0;
                    unsigned char* st = smem + slot * C::STAGE;
                    mbar_expect_tx(&raw_full[slot], nr * (2 * ROWB + 4 * G * 2));
                    bulk_g2s(st + C::KC, kw + row * ROWB, nr * ROWB, &raw_full[slot], pol);
                    bulk_g2s(st + C::VC, vw + row * ROWB, nr * ROWB, &raw_full[slot], pol);
                    bulk_g2s(st + C::KS, ks + row * G * 2, nr * G * 2, &raw_full[slot], pol);
                    bulk_g2s(st + C::KB, kb + row * G * 2, nr * G * 2, &raw_full[slot], pol);
                    bulk_g2s(st + C::VS, vs + row * G * 2, nr * G * 2, &raw_full[slot], pol);
                    bulk_g2s(st + C::VB, vb + row * G * 2, nr * G * 2, &raw_full[slot], pol);
                }
            }
            // copies still in flight land before the CTA retires: wait (bounded)
            // for every slot's last issued fill
            const uint32_t issued = gt;
            for (uint32_t s = 0; s < NST && s < issued; ++s) {
                const uint32_t last = ((issued - 1 - s) / NST) * NST + s;
                if (!twait(&raw_full[s], (last / NST) & 1)) report_stall(stall, 2, last);
            }
        } else if (warp == W_MMA && lane == 0) {
            // ------------------------- score MMA issuer -----------------------
            const uint32_t bq0 = s_addr(smem + C::BQ);
            uint32_t gt = 0, ni = 0;
            bool ok = true;
            for (uint32_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
                const Item it = item_of<HT>(P, idx);
                if (it.n_tiles == 0) continue;
                // K-step k of the Qg operand starts 256 bytes (16 descriptor units) after k-1's
                const uint64_t qdesc = sdesc(bq0 + (ni % NBQ) * C::BQ_BYTES, 128, 2048);
                for (int i = 0; i < it.n_tiles; ++i, ++gt) {
                    const uint32_t ka = gt % NAK, sb = gt % NS;
                    if (!wait_all(&ak_full[ka], (gt / NAK) & 1, gt >= NS ? &s_empty[sb] : nullptr,
                                  ((gt / NS) & 1) ^ 1)) {
                        report_stall(stall, 3, gt);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + C::S0 + 16 * sb, a = tmem + C::AK0 + 64 * ka;
#pragma unroll
                    for (int k = 0; k < DH / 16; ++k)
                        umma_ts(d, a + 8 * k, qdesc + 16 * k, ID_S, k > 0 ? 1u : 0u);
                    umma_commit(&s_full[sb]);
                }
                ++ni;
            }
            if (!ok) *err = 1;
            // every MMA this thread issued has completed before tensor memory is freed
            umma_commit(&drain[0]);
            if (!twait(&drain[0], 0)) report_stall(stall, 4, gt);
        } else if (warp == W_MMA_C && lane == 0) {
            // ------------------------ combine MMA issuer ----------------------
            const uint32_t bp0 = s_addr(smem + C::BP);
            uint32_t gt = 0;
            bool ok = true;
            for (uint32_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
                const Item it = item_of<HT>(P, idx);
                for (int i = 0; i < it.n_tiles; ++i, ++gt) {
                    const uint32_t b = gt & 1, ph = (gt >> 1) & 1, va = gt % NAV;
                    if (!wait_all(&av_full[va], (gt / NAV) & 1, &p_full[b], ph,
                                  gt >= 2 ? &o_empty[b] : nullptr, ph ^ 1)) {
                        report_stall(stall, 5, gt);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // P' of tile gt: the pair of warpgroup b, alternate tiles of it; K-step
                    // k (16 positions) starts two 8-position row blocks after k-1's
                    const uint32_t pb = 2 * b + ph;
                    const uint64_t pdesc = sdesc(bp0 + pb * C::BP_BYTES, C::BP_LBO, 128);
                    const uint32_t d = tmem + C::O0 + C::N_O * b, a = tmem + C::AV0 + 64 * va;
#pragma unroll
                    for (int k = 0; k < TP / 16; ++k)
                        umma_ts(d, a + 8 * k, pdesc + (uint64_t)((2 * C::BP_LBO) >> 4) * k, ID_V,
                                k > 0 ? 1u : 0u);
                    umma_commit(&o_full[b]);
                    umma_commit(&av_empty[va]);
                }
            }
            if (!ok) *err = 1;
            umma_commit(&drain[1]);
            if (!twait(&drain[1], 0)) report_stall(stall, 6, gt);
        }
    } else if (wg == 1) {
        // ------------------------------ K unpack ------------------------------
        const int q = warp & 3, r = lane >> 2, j = lane & 3;
        const int tq = (warp - W_K) * 32 + lane;               // 0..127
        uint32_t gt = 0, ni = 0;
        bool ok = true;
        for (uint32_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
            const Item it = item_of<HT>(P, idx);
            if (it.n_tiles == 0) continue;
            for (int i = 0; i < it.n_tiles; ++i, ++gt) {
                const uint32_t slot = gt % NST, ka = gt % NAK;
                // s_empty of tile gt - NAK: its scores and scales are read, so its
                // scores were computed: the K operand is free, and the Qg buffer
                // of NBQ items ago (every item has at least one tile)
                const uint32_t old = gt - NAK;
                if (!wait_all<true>(&raw_full[slot], (gt / NST) & 1, gt >= NAK ? &s_empty[old % NS] : nullptr,
                              (old / NS) & 1)) {
                    report_stall(stall, 7, gt);
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (i == 0) {
                    // Qg of this item: column n = g * 8 + h holds q[h] on group
                    // g's dims and zero elsewhere, K-major core matrices
                    const __half* qrow = static_cast<const __half*>(P.q) + ((size_t)it.b * P.n_heads + it.h0) * DH;
                    unsigned char* bq = smem + C::BQ + (ni % NBQ) * C::BQ_BYTES;
#pragma unroll
                    for (int c2 = 0; c2 < 2; ++c2) {
                        const int ci = tq + 128 * c2;                // 256 chunks of 8 fp16
                        const int n = ci >> 4, c = ci & 15;
                        const int g = n >> 3, h = n & 7;
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            const int d0 = kdim(8 * c + e), d1 = kdim(8 * c + e + 1);
                            const __half x0 = (h < it.nh && d0 / 64 == g) ? qrow[h * DH + d0] : __half(0.0f);
                            const __half x1 = (h < it.nh && d1 / 64 == g) ? qrow[h * DH + d1] : __half(0.0f);
                            __half2 v = __halves2half2(x0, x1);
                            w[e / 2] = *reinterpret_cast<uint32_t*>(&v);
                        }
                        *reinterpret_cast<uint4*>(bq + (n % 8) * 16 + (n / 8) * 2048 + c * 128) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    fence_async_smem();
                    // the per-group q sums: lane group of 8 sums 64 dims of (g, h)
                    {
                        const int h = tq >> 4, g = (tq >> 3) & 1, part = tq & 7;
                        float v = 0.0f;
                        if (h < it.nh) {
                            const uint4 u = *reinterpret_cast<const uint4*>(qrow + h * DH + g * 64 + part * 8);
                            const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&uw[k]));
                                v += f.x + f.y;
                            }
                        }
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        v += __shfl_xor_sync(0xffffffffu, v, 4);
                        if (part == 0)
                            reinterpret_cast<float*>(smem + C::QS)[((ni % QRING) * G + g) * 8 + h] = v;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&q_full[ni % QRING]);
                }
                const unsigned char* st = smem + slot * C::STAGE + C::KC;
                const uint32_t col = tmem + C::AK0 + 64 * ka;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t dst[32];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const int p = 32 * q + 16 * half + 8 * rr + r;
                        const uint4 w4 = *reinterpret_cast<const uint4*>(st + p * ROWB + 16 * j);
                        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi) {
                            const uint32_t w = ws[wi];
                            const uint32_t w8 = w >> 8;
                            // register m -> repetition 2wi + m/2, column offset m%2
                            dst[4 * (2 * wi) + 2 * rr + 0] = and_or<0x000F000Fu, 0x64006400u>(w);
                            dst[4 * (2 * wi) + 2 * rr + 1] = h2_hi_to_lo(and_or<0x00F000F0u, 0x64006400u>(w));
                            dst[4 * (2 * wi + 1) + 2 * rr + 0] = and_or<0x000F000Fu, 0x64006400u>(w8);
                            dst[4 * (2 * wi + 1) + 2 * rr + 1] = h2_hi_to_lo(and_or<0x00F000F0u, 0x64006400u>(w8));
                        }
                    }
                    tmem_st_16x256b_x8(col + ((uint32_t)(32 * q + 16 * half) << 16), dst);
                }
                // the rows' scale/bias pairs: lane j = 0 columns 0, 1 (k scale, k
                // bias), j = 1 columns 2, 3 (v scale, v bias), j = 2, 3 unused
                {
                    const unsigned char* sb = smem + slot * C::STAGE + (j == 0 ? C::KS : C::VS);
                    const int d2 = j == 0 ? C::KB - C::KS : C::VB - C::VS;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int p0 = 32 * q + 16 * half + r, p1 = p0 + 8;
                        uint32_t a0 = 0u, a1 = 0u, b0 = 0u, b1 = 0u;
                        if (j < 2) {
                            a0 = *reinterpret_cast<const uint32_t*>(sb + p0 * 4);
                            a1 = *reinterpret_cast<const uint32_t*>(sb + d2 + p0 * 4);
                            b0 = *reinterpret_cast<const uint32_t*>(sb + p1 * 4);
                            b1 = *reinterpret_cast<const uint32_t*>(sb + d2 + p1 * 4);
                        }
                        tmem_st_16x256b_x1(tmem + C::SC0 + 8 * ka + ((uint32_t)(32 * q + 16 * half) << 16),
                                           a0, a1, b0, b1);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&ak_full[ka]);
                    mbar_arrive(&raw_empty[slot]);
                }
            }
            ++ni;
        }
        if (!ok) *err = 1;
    } else if (wg == 2) {
        // ------------------------------ V unpack ------------------------------
        const int q = warp & 3;
        uint32_t gt = 0;
        bool ok = true;
        for (uint32_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
            const Item it = item_of<HT>(P, idx);
            for (int i = 0; i < it.n_tiles; ++i, ++gt) {
                const uint32_t slot = gt % NST, va = gt % NAV;
                // av_empty of tile gt - NAV: its combine has read this V operand
                if (!wait_all<true>(&raw_full[slot], (gt / NST) & 1, gt >= NAV ? &av_empty[va] : nullptr,
                              ((gt / NAV) & 1) ^ 1)) {
                    report_stall(stall, 8, gt);
                    ok = false;
                    break;
                }
                tc_fence_after();
                // lane L gives the row address of tile L/8: repetition pair
                // member L/16, rows 8 (L/8 % 2) .. + 7, this warp's 16 bytes
                const uint32_t vbase = s_addr(smem + slot * C::STAGE + C::VC) + 16 * q;
                uint32_t x[4][4];
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    const int pos = 16 * (2 * pr + (lane >> 4)) + 8 * ((lane >> 3) & 1) + (lane & 7);
                    ldsm_x4_trans(vbase + pos * ROWB, x[pr]);
                }
                const uint32_t col = tmem + C::AV0 + 64 * va;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    // half 0: dims 4u, 4u+1 (lanes r, r+8); half 1: dims 4u+2, 4u+3
                    uint32_t u[32];
#pragma unroll
                    for (int pr = 0; pr < 4; ++pr)
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int n = 2 * pr + (k >> 1), hh = k & 1;
                            const uint32_t xv = half ? x[pr][k] >> 8 : x[pr][k];
                            u[4 * n + hh] = and_or<0x000F000Fu, 0x43004300u>(xv);
                            u[4 * n + 2 + hh] = and_or<0x000F000Fu, 0x43004300u>(xv >> 4);
                        }
                    tmem_st_16x256b_x8(col + ((uint32_t)(32 * q + 16 * half) << 16), u);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&av_full[va]);
                    mbar_arrive(&raw_empty[slot]);
                }
            }
        }
        if (!ok) *err = 1;
    } else {
        // ------------------------------ softmax -------------------------------
        regs_inc<REG_SOFTMAX>();
        const int sp = wg - 3;                   // this warpgroup takes tiles of parity sp
        const int bar_id = 1 + sp;
        const int q = warp & 3;
        const int p = 32 * q + lane;             // tile position = TMEM lane (scores)
        const int d = vdim(32 * q + lane);       // head dim = TMEM lane (O)
        const int gq = q >> 1;                   // group of that dim
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const int kp = vkpos(p);                 // this position's row of P'
        int* flags = reinterpret_cast<int*>(smem + C::FLAGS) + 8 * sp;      // [2][4]
        float* red = reinterpret_cast<float*>(smem + C::RED) + sp * C::RED_FLOATS;
        float* red_l = red;                      // [4][HT]
        float* red_b = red_l + 4 * HT;           // [4][G][HT]
        float* red_m = red_b + 4 * G * HT;       // [4][HT]
        float* snew = red_m + 4 * HT;            // [HT]
        const size_t rows = (size_t)P.b_rows * P.n_heads;
        const uint32_t b = (uint32_t)sp;         // S, P' and O buffer of this warpgroup
        uint32_t gt = 0, ni = 0, xi = 0;
        uint32_t vc = 0;     // votes so far: vote c's words live in flags[c % 2]
        bool bad = false;

        for (uint32_t idx = blockIdx.x; idx < n_items; idx += gridDim.x, ++xi) {
            const Item it = item_of<HT>(P, idx);
            float qs[G][HT];
            bool q_ok = true;        // voted on with this warpgroup's first tile of the item
            if (it.n_tiles > 0) {
                const uint32_t qslot = ni % QRING;
                q_ok = bad || twait(&q_full[qslot], (ni / QRING) & 1);
                if (!q_ok) report_stall(stall, 9, gt);
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int h = 0; h < HT; ++h) qs[g][h] = qsums[(qslot * G + g) * 8 + h];
            }
            float m_run[HT], l_part[HT], bsum[G][HT], o[HT], alpha_p1[HT];
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                m_run[h] = -INFINITY;
                l_part[h] = 0.0f;
                o[h] = 0.0f;
                alpha_p1[h] = 1.0f;
#pragma unroll
                for (int g = 0; g < G; ++g) bsum[g][h] = 0.0f;
            }
            // O of this warpgroup's tile (this thread's dim and group) into the
            // registers: o = o * alpha + O_tile, alpha the reference-point move
            // of that tile
            auto accumulate = [&](const float (&alpha)[HT]) {
                const uint32_t col = tmem + C::O0 + C::N_O * b + C::GW * gq + lane_addr;
                if constexpr (HT == 4) {
                    uint32_t v[16];
                    tmem_ld16(col, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < HT; ++h)
                        o[h] = fmaf(o[h], alpha[h],
                                    __uint_as_float(v[h]) + __uint_as_float(v[HT + h]) +
                                        __uint_as_float(v[2 * HT + h]));
                } else {
                    uint32_t v[24];
                    tmem_ld16(col, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                    tmem_ld8(col + 16, *reinterpret_cast<uint32_t(*)[8]>(&v[16]));
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < HT; ++h)
                        o[h] = fmaf(o[h], alpha[h],
                                    __uint_as_float(v[h]) + __uint_as_float(v[HT + h]) +
                                        __uint_as_float(v[2 * HT + h]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_empty[b]);
            };

            const uint32_t gt0 = gt;
            int last_i = -1;
            bool okw_o = q_ok;       // the previous tile's wait for its O (voted on with this tile)
            for (int i = (int)((sp - gt0) & 1); i < it.n_tiles && !bad; i += 2) {
                const uint32_t g_ = gt0 + i, ph = (g_ >> 1) & 1;
                // the tile's wait first, then one warpgroup vote on the outcome
                // (so every thread takes the same branches). This tile's P'
                // buffer was last read by the combine of tile g_-4, whose O this
                // warpgroup has already taken.
                const uint32_t sb = g_ % NS;
                const bool okw_s = twait(&s_full[sb], (g_ / NS) & 1);
                if (!okw_s) report_stall(stall, 10, g_);
                const bool okw = okw_s && okw_o;
                tc_fence_after();

                // scores of position p, and its scales and biases
                uint32_t xs[16], sv[4];
                tmem_ld16(tmem + C::S0 + 16 * sb + lane_addr, xs);
                tmem_ld4(tmem + C::SC0 + 8 * (g_ % NAK) + lane_addr, sv);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[sb]);
                const int nvalid = (int)min((uint32_t)TP, it.hi - (it.lo + i * TP));
                const bool live = p < nvalid;
                const float2 ks2 = __half22float2(*reinterpret_cast<const __half2*>(&sv[0]));
                const float2 kb2 = __half22float2(*reinterpret_cast<const __half2*>(&sv[1]));
                const float2 vs2 = __half22float2(*reinterpret_cast<const __half2*>(&sv[2]));
                const float2 vb2 = __half22float2(*reinterpret_cast<const __half2*>(&sv[3]));
                const float ksc[G] = {ks2.x * scale2, ks2.y * scale2};
                const float cq[G] = {fmaf(ksc[0], -1024.0f, kb2.x * scale2), fmaf(ksc[1], -1024.0f, kb2.y * scale2)};
                float sc[HT];
                bool grow = false;
#pragma unroll
                for (int h = 0; h < HT; ++h) {
                    float a = 0.0f;
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        a = fmaf(ksc[g], __uint_as_float(xs[8 * g + h]), fmaf(cq[g], qs[g][h], a));
                    sc[h] = live ? a : -INFINITY;
                    grow |= sc[h] > m_run[h] + 8.0f;
                }
                // the warpgroup's vote: per warp (bit 0) some score outgrew its
                // reference point, (bit 1) a wait of the tile failed; every
                // thread reads all four words after the barrier
                {
                    const uint32_t wv = (__any_sync(0xffffffffu, grow) ? 1u : 0u) |
                                        (__any_sync(0xffffffffu, !okw) ? 2u : 0u);
                    if (lane == 0) flags[(vc & 1) * 4 + q] = (int)wv;
                }
                named_sync(bar_id, 128);
                const int4 fl = *reinterpret_cast<const int4*>(flags + (vc & 1) * 4);
                const int fv = fl.x | fl.y | fl.z | fl.w;
                ++vc;
                if (fv & 2) {
                    bad = true;
                    break;
                }
                float alpha[HT];
#pragma unroll
                for (int h = 0; h < HT; ++h) alpha[h] = 1.0f;
                if (fv & 1) {
#pragma unroll
                    for (int h = 0; h < HT; ++h) {
                        float v = sc[h];
#pragma unroll
                        for (int o2 = 16; o2 > 0; o2 >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o2));
                        if (lane == 0) red_m[q * HT + h] = v;
                    }
                    named_sync(bar_id, 128);
#pragma unroll
                    for (int h = 0; h < HT; ++h) {
                        const float v = fmaxf(fmaxf(red_m[h], red_m[HT + h]), fmaxf(red_m[2 * HT + h], red_m[3 * HT + h]));
                        const float m_new = v > m_run[h] + 8.0f ? v : m_run[h];
                        alpha[h] = ex2(m_run[h] - m_new);    // 0 on the warpgroup's first tile
                        m_run[h] = m_new;
                        l_part[h] *= alpha[h];
#pragma unroll
                        for (int g = 0; g < G; ++g) bsum[g][h] *= alpha[h];
                    }
                    named_sync(bar_id, 128);                 // red_m is read by everyone
                }
                float e[HT];
#pragma unroll
                for (int h = 0; h < HT; ++h) {
                    e[h] = live ? ex2(sc[h] - m_run[h]) : 0.0f;
                    l_part[h] += e[h];
                }
                // P' = p * v_scale in three bf16 parts, row kp of this tile's B
                // operand: chunk (g, part) of HT columns; v bias - 128 v_scale
                const float vsf[G] = {live ? vs2.x : 0.0f, live ? vs2.y : 0.0f};
                const float vbf[G] = {live ? fmaf(vs2.x, -128.0f, vb2.x) : 0.0f,
                                      live ? fmaf(vs2.y, -128.0f, vb2.y) : 0.0f};
                unsigned char* prow = smem + C::BP + (2 * b + ph) * C::BP_BYTES + (kp % 8) * 16 + (kp / 8) * C::BP_LBO;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    uint32_t hi[HT / 2], mid[HT / 2], lo[HT / 2];
#pragma unroll
                    for (int h = 0; h < HT; h += 2) {
                        bsum[g][h] = fmaf(e[h], vbf[g], bsum[g][h]);
                        bsum[g][h + 1] = fmaf(e[h + 1], vbf[g], bsum[g][h + 1]);
                        const float2 v = __fmul2_rn(make_float2(e[h], e[h + 1]), make_float2(vsf[g], vsf[g]));
                        split3(v.x, v.y, hi[h / 2], mid[h / 2], lo[h / 2]);
                    }
                    if constexpr (HT == 4) {
                        // columns 16g + (hi 0..3, mid 4..7 | lo 8..11, zero 12..15)
                        *reinterpret_cast<uint4*>(prow + (2 * g) * 128) = make_uint4(hi[0], hi[1], mid[0], mid[1]);
                        *reinterpret_cast<uint4*>(prow + (2 * g + 1) * 128) = make_uint4(lo[0], lo[1], 0u, 0u);
                    } else {
                        // columns 24g + (hi 0..7 | mid 8..15 | lo 16..23)
                        *reinterpret_cast<uint4*>(prow + (3 * g) * 128) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4*>(prow + (3 * g + 1) * 128) = make_uint4(mid[0], mid[1], mid[2], mid[3]);
                        *reinterpret_cast<uint4*>(prow + (3 * g + 2) * 128) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
                fence_async_smem();
                // the O of this warpgroup's previous tile in the item (its combine
                // ran during this tile's work), rescaled by that tile's move. Taken
                // before this tile's P' is published: that combine has then
                // consumed the previous p_full phase, so p_full never runs two
                // phases ahead of the combine issuer's wait (which would alias)
                if (i >= 2) {
                    okw_o = twait(&o_full[b], ph ^ 1);
                    if (!okw_o) report_stall(stall, 11, g_);
                    tc_fence_after();
                    accumulate(alpha_p1);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
#pragma unroll
                for (int h = 0; h < HT; ++h) alpha_p1[h] = alpha[h];
                last_i = i;
            }
            gt = gt0 + (uint32_t)it.n_tiles;
            if (it.n_tiles > 0) ++ni;
            // this warpgroup's last O tile of the item
            if (!bad && last_i >= 0) {
                const uint32_t last = gt0 + (uint32_t)last_i;
                const bool okw_l = twait(&o_full[b], (last >> 1) & 1);
                if (!okw_l) report_stall(stall, 12, last);
                const bool okw = okw_l && okw_o;
                tc_fence_after();
                accumulate(alpha_p1);
                const int wv = __any_sync(0xffffffffu, !okw) ? 2 : 0;
                if (lane == 0) flags[(vc & 1) * 4 + q] = wv;
                named_sync(bar_id, 128);
                const int4 fl = *reinterpret_cast<const int4*>(flags + (vc & 1) * 4);
                ++vc;
                if ((fl.x | fl.y | fl.z | fl.w) & 2) bad = true;
            }

            // ---- the warpgroup's (O, m, l): l and bias sums over its threads --
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                float v = l_part[h];
#pragma unroll
                for (int o2 = 16; o2 > 0; o2 >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
                if (lane == 0) red_l[q * HT + h] = v;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float u = bsum[g][h];
#pragma unroll
                    for (int o2 = 16; o2 > 0; o2 >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o2);
                    if (lane == 0) red_b[(q * G + g) * HT + h] = u;
                }
            }
            const __half* qrow = static_cast<const __half*>(P.q) + ((size_t)it.b * P.n_heads + it.h0) * DH;
            if (sp == 0 && it.with_new && q == 0) {
                const __half* nk = static_cast<const __half*>(P.new_k) + ((size_t)it.b * P.n_kv_heads + it.hk) * DH;
                for (int h = 0; h < it.nh; ++h) {
                    float part = 0.0f;
                    for (int dd = lane; dd < DH; dd += 32)
                        part = fmaf(__half2float(qrow[h * DH + dd]), __half2float(nk[dd]), part);
                    part = warp_sum(part);
                    if (lane == 0) snew[h] = part * scale2;
                }
            }
            named_sync(bar_id, 128);
            float lw[HT], ow[HT];
#pragma unroll
            for (int h = 0; h < HT; ++h) {
                lw[h] = red_l[h] + red_l[HT + h] + red_l[2 * HT + h] + red_l[3 * HT + h];
                ow[h] = o[h] + red_b[(0 * G + gq) * HT + h] + red_b[(1 * G + gq) * HT + h] +
                        red_b[(2 * G + gq) * HT + h] + red_b[(3 * G + gq) * HT + h];
            }
            // ---- the odd tiles' warpgroup hands its (O, m, l) to the even one --
            float* xch = reinterpret_cast<float*>(smem + C::XCH) + (xi & 1) * C::XCH_FLOATS;
            const int tq = 32 * q + lane;
            if (sp == 1) {
#pragma unroll
                for (int h = 0; h < HT; ++h) xch[2 * HT + tq * HT + h] = ow[h];
                if (tq == 0)
#pragma unroll
                    for (int h = 0; h < HT; ++h) {
                        xch[h] = m_run[h];
                        xch[HT + h] = lw[h];
                    }
            }
            if (sp == 1 && bad) *err = 1;
            named_sync(XCH_BAR, 256);
            if (sp == 0) {
                const bool poison = bad || *err != 0;
                const __half* nv = static_cast<const __half*>(P.new_v) + ((size_t)it.b * P.n_kv_heads + it.hk) * DH;
                const float nvd = it.with_new ? __half2float(nv[d]) : 0.0f;
#pragma unroll
                for (int h = 0; h < HT; ++h) {
                    if (h >= it.nh) break;
                    const float m1 = xch[h], l1 = xch[HT + h], o1 = xch[2 * HT + tq * HT + h];
                    float M = fmaxf(m_run[h], m1);
                    const float w0 = m_run[h] == -INFINITY ? 0.0f : ex2(m_run[h] - M);
                    const float w1 = m1 == -INFINITY ? 0.0f : ex2(m1 - M);
                    float ov = fmaf(ow[h], w0, o1 * w1), lv = fmaf(lw[h], w0, l1 * w1);
                    if (it.with_new) {
                        const float sn = snew[h];
                        const float Mx = fmaxf(M, sn);
                        const float er = M == -INFINITY ? 0.0f : ex2(M - Mx);
                        const float en = ex2(sn - Mx);
                        ov = fmaf(nvd, en, ov * er);
                        lv = fmaf(lv, er, en);
                        M = Mx;
                    }
                    const size_t row = it.split * rows + (size_t)it.b * P.n_heads + it.h0 + h;
                    part_o[row * DH + d] = poison ? __int_as_float(0x7fc00000) : ov;
                    if (d == 0) {
                        part_m[row] = poison ? __int_as_float(0x7fc00000) : M * LN2;   // natural-log units
                        part_l[row] = poison ? __int_as_float(0x7fc00000) : lv;
                    }
                }
            }
        }
        if (bad) *err = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace tmem4
}  // namespace kvq
