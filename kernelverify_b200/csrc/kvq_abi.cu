// The C ABI (include/kvq_b200.h): argument validation, the split plan, and
// dispatch to the per-width launchers. Nothing here allocates device memory;
// every failure returns a status and leaves a message for kvq_last_error().
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "kvq_b200.h"
#include "kvq_launch.h"
#include "kvq_partial.cuh"

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(KVQ_ERR_LAUNCH, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// sm_100 check of the current device, cached per device id.
int device_ok() {
    static thread_local int checked[64] = {0};  // 0 unknown, 1 ok, -1 not sm_100
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(KVQ_ERR_UNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64 && checked[dev] != 0)
        return checked[dev] > 0 ? KVQ_OK
                                : fail(KVQ_ERR_UNSUPPORTED, "device %d is not an sm_100 (B200) GPU", dev);
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return fail(KVQ_ERR_UNSUPPORTED, "device query failed: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) checked[dev] = major == 10 ? 1 : -1;
    if (major != 10) return fail(KVQ_ERR_UNSUPPORTED, "device %d is sm_%d0, this library is built for sm_100a", dev, major);
    return KVQ_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool bits_ok(uint32_t b) { return b == 2 || b == 3 || b == 4 || b == 6 || b == 8; }

int check_format(uint32_t head_dim, uint32_t bits, uint32_t group, uint32_t dtype) {
    if (head_dim != 64 && head_dim != 128)
        return fail(KVQ_ERR_INVALID, "head_dim %u is not supported (64 or 128)", head_dim);
    if (!bits_ok(bits)) return fail(KVQ_ERR_INVALID, "bits %u is not supported (2, 3, 4, 6 or 8)", bits);
    if (group != 32 && group != 64 && group != 128)
        return fail(KVQ_ERR_INVALID, "group_size %u is not supported (32, 64 or 128)", group);
    if (head_dim % group)
        return fail(KVQ_ERR_INVALID, "group_size %u does not divide head_dim %u", group, head_dim);
    if (dtype != KVQ_F16 && dtype != KVQ_F32) return fail(KVQ_ERR_INVALID, "dtype %u is not KVQ_F16 or KVQ_F32", dtype);
    return KVQ_OK;
}

constexpr size_t kAlign = 256;
size_t align_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

// The number of resident CTAs the split plan aims to fill: 148 SMs x 4.
constexpr uint64_t kTargetCtas = 148 * 4 * 2;
constexpr uint32_t kMaxSplits = 4096;

enum KernelKind { KERNEL_GENERIC = 0, KERNEL_MMA4 = 1, KERNEL_UMMA4 = 2, KERNEL_TMEM4 = 3 };

// KVQ_KERNEL=generic forces the CUDA-core kernel, KVQ_KERNEL=mma the
// register-fragment tensor-core kernels, KVQ_KERNEL=umma the single-role
// tcgen05 kernel, KVQ_KERNEL=tmem the warp-specialised tensor-memory kernel
// (the last two where they apply: fp16, 4-bit, head_dim 128, group 64).
// Unset, each call takes the fastest eligible kernel (A/B checks of the paths
// use the switch).
int kernel_override() {
    const char* v = getenv("KVQ_KERNEL");
    if (v == nullptr) return -1;
    if (strcmp(v, "generic") == 0) return KERNEL_GENERIC;
    if (strcmp(v, "mma") == 0) return KERNEL_MMA4;
    if (strcmp(v, "umma") == 0) return KERNEL_UMMA4;
    if (strcmp(v, "tmem") == 0) return KERNEL_TMEM4;
    return -1;
}

// KVQ_PRECISION=fast lets the register-fragment tensor-core kernels carry the
// combine's weights p * v_scale as two bf16 parts (2^-16 relative) instead of
// three (2^-23, binary32-class: the contract's working-precision clause C1).
bool fast_precision() {
    const char* v = getenv("KVQ_PRECISION");
    return v != nullptr && strcmp(v, "fast") == 0;
}

// Split plan of the tensor-core kernel. Its CTAs run in waves of the resident
// CTAs (per SM x SMs); a CTA costs its chunk of positions plus a fixed ramp
// (barrier setup, the first copies' latency, the epilogue) worth about two
// 64-position stages. Of the split counts that fill 1..8 whole waves, take the
// one whose waves x (chunk + ramp) is least. Chunks are whole 64-row stages.
constexpr uint64_t kMmaStage = 64;
constexpr uint64_t kMmaRamp = 128;

void mma4_splits(uint64_t span, uint64_t units, int ctas_per_sm, uint32_t* chunk_out,
                 uint32_t* splits_out, uint64_t stage = kMmaStage, uint64_t ramp = kMmaRamp) {
    const uint64_t resident = (uint64_t)ctas_per_sm * kvq::sm_count();
    const auto round_stage = [stage](uint64_t n) {
        n = (n + stage - 1) / stage * stage;
        return n < stage ? stage : n;
    };
    uint64_t best_chunk = round_stage(span), best_splits = 1;
    uint64_t best_cost = ((units + resident - 1) / resident) * (best_chunk + ramp);
    for (uint64_t waves = 1; span && waves <= 8; ++waves) {
        const uint64_t fit = waves * resident / units;
        if (fit <= 1) continue;
        const uint64_t chunk = round_stage((span + fit - 1) / fit);
        const uint64_t splits = (span + chunk - 1) / chunk;
        if (splits > kMaxSplits) break;
        const uint64_t cost = ((units * splits + resident - 1) / resident) * (chunk + ramp);
        if (cost < best_cost) {
            best_cost = cost;
            best_chunk = chunk;
            best_splits = splits;
        }
    }
    const uint64_t kMaxChunk = 0xFFFFFFFFull / stage * stage;
    if (best_chunk > kMaxChunk) {
        best_chunk = kMaxChunk;
        best_splits = (span + best_chunk - 1) / best_chunk;
    }
    *chunk_out = (uint32_t)best_chunk;
    *splits_out = (uint32_t)best_splits;
}

// Split plan of the persistent tensor-memory kernel: one CTA per SM walks
// work items of `chunk` positions (whole 128-position tiles), item i of a CTA
// being its (blockIdx + i * grid)-th. Of the split counts, take the one whose
// busiest CTA streams the fewest tiles (a small per-item cost breaks ties
// toward fewer, longer items, which also keeps the merge short).
void tmem4_splits(uint64_t span, uint64_t units, uint32_t* chunk_out, uint32_t* splits_out,
                  uint32_t* grid_out) {
    const uint64_t tile = (uint64_t)kvq::tmem4_tile_positions();
    const uint64_t sms = (uint64_t)kvq::sm_count();
    const uint64_t tiles = span ? (span + tile - 1) / tile : 1;
    uint64_t best_chunk = tiles, best_splits = 1;
    double best_cost = 1e300;
    for (uint64_t s = 1; s <= tiles && s <= kMaxSplits; ++s) {
        const uint64_t chunk = (tiles + s - 1) / s;
        const uint64_t splits = (tiles + chunk - 1) / chunk;
        if (splits != s) continue;
        const uint64_t items = units * splits;
        const uint64_t per_cta = (items + sms - 1) / sms;
        const double cost = (double)per_cta * ((double)chunk + 0.25);
        if (cost < best_cost) {
            best_cost = cost;
            best_chunk = chunk;
            best_splits = splits;
        }
    }
    const uint64_t items = units * best_splits;
    *chunk_out = (uint32_t)(best_chunk * tile);
    *splits_out = (uint32_t)best_splits;
    *grid_out = (uint32_t)(items < sms ? items : sms);
}

struct Plan {
    kvq::Problem P;
    int kernel;
    int ht;
    uint32_t grid;      // persistent CTAs (tensor-memory kernel)
    uint32_t rows;      // b_rows * n_heads
    size_t part_bytes;  // one fp32 [n_splits, rows, DH] block
    size_t ml_bytes;    // one fp32 [n_splits, rows] block
};

int plan(const kvq_args* a, Plan* pl) {
    if (a == nullptr) return fail(KVQ_ERR_INVALID, "args is NULL");
    int rc = check_format(a->head_dim, a->bits, a->group_size, a->dtype);
    if (rc) return rc;
    if (!a->q || !a->k_wq || !a->k_scales || !a->k_biases || !a->v_wq || !a->v_scales ||
        !a->v_biases || (a->has_new_entry && (!a->new_k || !a->new_v)))
        return fail(KVQ_ERR_INVALID, "a required tensor pointer is NULL");
    if (a->b_rows == 0 || a->n_heads == 0 || a->n_kv_heads == 0)
        return fail(KVQ_ERR_INVALID, "b_rows, n_heads and n_kv_heads must be positive");
    if (a->n_heads % a->n_kv_heads)
        return fail(KVQ_ERR_INVALID, "n_heads %u is not a multiple of n_kv_heads %u", a->n_heads, a->n_kv_heads);
    if (a->b_rows > 65535) return fail(KVQ_ERR_INVALID, "b_rows %u above 65535", a->b_rows);
    if (a->t_cached > a->t_stride)
        return fail(KVQ_ERR_INVALID, "t_cached %u exceeds the physical row stride t_stride %u", a->t_cached, a->t_stride);
    if (a->t_begin > a->t_end) return fail(KVQ_ERR_INVALID, "t_begin %u after t_end %u", a->t_begin, a->t_end);
    const size_t esz = a->dtype == KVQ_F16 ? 2 : 4;
    const void* ptrs[] = {a->q, a->k_scales, a->k_biases, a->v_scales, a->v_biases, a->new_k, a->new_v};
    for (const void* p : ptrs)
        if (p && !aligned(p, esz)) return fail(KVQ_ERR_INVALID, "a tensor pointer is not %zu-byte aligned", esz);
    if (!aligned(a->k_wq, 4) || !aligned(a->v_wq, 4) || (a->seq_lens && !aligned(a->seq_lens, 4)))
        return fail(KVQ_ERR_INVALID, "packed words and seq_lens must be 4-byte aligned");

    kvq::Problem& P = pl->P;
    P.q = a->q; P.k_wq = a->k_wq; P.k_scales = a->k_scales; P.k_biases = a->k_biases;
    P.v_wq = a->v_wq; P.v_scales = a->v_scales; P.v_biases = a->v_biases;
    P.new_k = a->new_k; P.new_v = a->new_v; P.seq_lens = a->seq_lens;
    P.b_rows = a->b_rows; P.n_heads = a->n_heads; P.n_kv_heads = a->n_kv_heads;
    P.t_cached = a->t_cached; P.t_stride = a->t_stride; P.group_size = a->group_size;
    P.has_new_entry = a->has_new_entry ? 1u : 0u;
    P.cache_batch_stride = a->cache_batch_stride;
    P.t_begin = a->t_begin; P.t_end = a->t_end;
    P.r = a->n_heads / a->n_kv_heads;
    // The tensor-core kernels stream 16-byte-aligned runs of 8 rows with TMA:
    // they need fp16 steps, head_dim 128, at most 8 query heads per cache
    // head, and 8-row-aligned geometry (the tcgen05 kernel, when asked for,
    // 4-bit group 64); everything else runs on the CUDA-core kernel.
    const bool tma_ok = aligned(a->k_wq, 16) && aligned(a->v_wq, 16) && aligned(a->k_scales, 16) &&
                        aligned(a->k_biases, 16) && aligned(a->v_scales, 16) &&
                        aligned(a->v_biases, 16) && a->t_stride % 8 == 0 &&
                        a->cache_batch_stride % 8 == 0 && a->t_begin % 8 == 0;
    const bool tc = a->dtype == KVQ_F16 && a->head_dim == 128 && P.r <= 8 && tma_ok;
    const int forced = kernel_override();
    const bool g64b4 = a->group_size == 64 && a->bits == 4;
    if (!tc || forced == KERNEL_GENERIC)
        pl->kernel = KERNEL_GENERIC;
    else if (g64b4 && forced == KERNEL_UMMA4)
        pl->kernel = KERNEL_UMMA4;
    else if (g64b4 && forced == KERNEL_TMEM4)
        pl->kernel = KERNEL_TMEM4;
    else
        pl->kernel = KERNEL_MMA4;
    if (pl->kernel != KERNEL_GENERIC)
        pl->ht = P.r <= 4 ? 4 : 8;
    else
        pl->ht = P.r == 1 ? 1 : (P.r <= 4 ? 4 : 8);
    P.head_tiles = (P.r + pl->ht - 1) / pl->ht;
    P.scale = 1.0f / sqrtf((float)a->head_dim);

    const uint32_t end = a->t_end < a->t_cached ? a->t_end : a->t_cached;
    const uint64_t span = end > a->t_begin ? end - a->t_begin : 0;
    const uint64_t units = (uint64_t)a->b_rows * a->n_kv_heads * P.head_tiles;
    pl->rows = a->b_rows * a->n_heads;
    pl->grid = 0;
    if (pl->kernel == KERNEL_TMEM4) {
        tmem4_splits(span, units, &P.chunk, &P.n_splits, &pl->grid);
        pl->part_bytes = align_up((size_t)P.n_splits * pl->rows * a->head_dim * sizeof(float));
        pl->ml_bytes = align_up((size_t)P.n_splits * pl->rows * sizeof(float));
        return KVQ_OK;
    }
    if (pl->kernel != KERNEL_GENERIC) {
        if (pl->kernel == KERNEL_UMMA4)
            // 128-position tiles; the CTA's fixed work (TMEM, the q operand, the
            // final reduction) is worth about two tiles
            mma4_splits(span, units, kvq::umma4_ctas_per_sm(pl->ht), &P.chunk, &P.n_splits, 128, 256);
        else
            mma4_splits(span, units, kvq::mma4_ctas_per_sm(pl->ht, a->group_size, a->bits), &P.chunk,
                        &P.n_splits, (uint64_t)kvq::mma4_stage_positions(), kMmaRamp);
        pl->part_bytes = align_up((size_t)P.n_splits * pl->rows * a->head_dim * sizeof(float));
        pl->ml_bytes = align_up((size_t)P.n_splits * pl->rows * sizeof(float));
        return KVQ_OK;
    }
    uint64_t chunk = (span * units + kTargetCtas - 1) / kTargetCtas;
    const uint64_t tile = kvq::P_TILE;
    chunk = (chunk + tile - 1) / tile * tile;
    if (chunk < tile) chunk = tile;
    uint64_t splits = span ? (span + chunk - 1) / chunk : 1;
    if (splits > kMaxSplits) {
        chunk = ((span + kMaxSplits - 1) / kMaxSplits + tile - 1) / tile * tile;
        splits = (span + chunk - 1) / chunk;
    }
    P.chunk = (uint32_t)chunk;
    P.n_splits = (uint32_t)splits;
    pl->part_bytes = align_up((size_t)P.n_splits * pl->rows * a->head_dim * sizeof(float));
    pl->ml_bytes = align_up((size_t)P.n_splits * pl->rows * sizeof(float));
    return KVQ_OK;
}

cudaError_t launch_partial_any(const Plan& pl, uint32_t bits, uint32_t dtype, uint32_t dh,
                               float* o, float* m, float* l, cudaStream_t s) {
    if (pl.kernel == KERNEL_TMEM4) return kvq::launch_tmem4(pl.P, pl.ht, pl.grid, o, m, l, s);
    if (pl.kernel == KERNEL_UMMA4) return kvq::launch_umma4(pl.P, pl.ht, o, m, l, s);
    if (pl.kernel == KERNEL_MMA4)
        return kvq::launch_mma4(pl.P, pl.ht, pl.P.group_size, (int)bits, fast_precision() ? 2 : 3,
                                o, m, l, s);
    switch (bits) {
        case 2: return kvq::launch_partial<2>(pl.P, dtype, dh, pl.ht, o, m, l, s);
        case 3: return kvq::launch_partial<3>(pl.P, dtype, dh, pl.ht, o, m, l, s);
        case 4: return kvq::launch_partial<4>(pl.P, dtype, dh, pl.ht, o, m, l, s);
        case 6: return kvq::launch_partial<6>(pl.P, dtype, dh, pl.ht, o, m, l, s);
        case 8: return kvq::launch_partial<8>(pl.P, dtype, dh, pl.ht, o, m, l, s);
    }
    return cudaErrorInvalidValue;
}

int check_workspace(const void* ws, size_t have, size_t need) {
    if (need == 0) return KVQ_OK;
    if (ws == nullptr || have < need)
        return fail(KVQ_ERR_INVALID, "workspace of %zu bytes is smaller than the %zu this call needs", have, need);
    if (!aligned(ws, kAlign)) return fail(KVQ_ERR_INVALID, "workspace is not 256-byte aligned");
    return KVQ_OK;
}

int check_merge(uint32_t n_parts, uint32_t rows, uint32_t head_dim, uint32_t out_dtype) {
    if (n_parts == 0 || rows == 0 || head_dim == 0) return fail(KVQ_ERR_INVALID, "empty merge");
    if (n_parts > (uint32_t)kvq::MERGE_MAX_PARTS)
        return fail(KVQ_ERR_INVALID, "%u parts: at most %d", n_parts, kvq::MERGE_MAX_PARTS);
    if (head_dim > kvq::MERGE_MAX_DH || head_dim % 32)
        return fail(KVQ_ERR_INVALID, "head_dim %u: a multiple of 32 up to %d", head_dim, kvq::MERGE_MAX_DH);
    if (rows > 0x7FFFFFFFu) return fail(KVQ_ERR_INVALID, "too many rows");
    if (out_dtype != KVQ_F16 && out_dtype != KVQ_F32) return fail(KVQ_ERR_INVALID, "bad out_dtype");
    return KVQ_OK;
}

// ---------------------------------------------------------------------------
// Scratch for kvq_decode_noalloc: a file-scope device buffer, present on every
// device that loads this library. Host code may not use its name as a device
// address (on the host it is a stand-in), so the device address is looked up
// with cudaGetSymbolAddress, with the calling device current. It is looked up
// on every call rather than cached: after a device reset the library's device
// code is loaded again and the buffer's address may change, and the lookup of
// an already loaded symbol is a cheap host-side query.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[KVQ_NOALLOC_SCRATCH_BYTES];

int noalloc_scratch(void** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress of the built-in scratch");
    *out = p;
    return KVQ_OK;
}

}  // namespace

namespace kvq {

// The merges are launched as programmatic dependents of the kernel before
// them on the stream (the split stage): their CTAs are launched while it
// streams and wait in pdl_wait() for its completion, which hides the launch
// gap between the two.
template <typename TO, bool NORMALIZE>
static cudaError_t launch_merge_pdl(unsigned blocks, const float* part_o, const float* part_m,
                                   const float* part_l, uint32_t n_parts, uint32_t rows,
                                   uint32_t head_dim, uint64_t o_stride, uint64_t ml_stride, TO* out,
                                   float* out_m, float* out_l, cudaStream_t stream) {
    // the split stage's sizes take the one-round-trip merge
    const bool small = head_dim == 128 && n_parts <= (uint32_t)MERGE_SMALL_PARTS &&
                       aligned(part_o, 16) && o_stride % 4 == 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(MERGE_THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (small)
        return cudaLaunchKernelEx(&cfg, merge_small_kernel<TO, NORMALIZE>, part_o, part_m, part_l,
                                  n_parts, rows, o_stride, ml_stride, out, out_m, out_l);
    return cudaLaunchKernelEx(&cfg, merge_kernel<TO, NORMALIZE>, part_o, part_m, part_l, n_parts,
                              rows, head_dim, o_stride, ml_stride, out, out_m, out_l);
}

cudaError_t launch_merge(const float* part_o, const float* part_m, const float* part_l,
                         uint32_t n_parts, uint32_t rows, uint32_t head_dim, uint64_t o_stride,
                         uint64_t ml_stride, int out_dtype, void* out, cudaStream_t stream) {
    const unsigned blocks = rows;
    cudaError_t e;
    if (out_dtype == KVQ_F16)
        e = launch_merge_pdl<__half, true>(blocks, part_o, part_m, part_l, n_parts, rows, head_dim,
                                           o_stride, ml_stride, static_cast<__half*>(out), nullptr,
                                           nullptr, stream);
    else
        e = launch_merge_pdl<float, true>(blocks, part_o, part_m, part_l, n_parts, rows, head_dim,
                                          o_stride, ml_stride, static_cast<float*>(out), nullptr,
                                          nullptr, stream);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_merge_partial(const float* part_o, const float* part_m, const float* part_l,
                                 uint32_t n_parts, uint32_t rows, uint32_t head_dim,
                                 float* out_o, float* out_m, float* out_l, cudaStream_t stream) {
    const unsigned blocks = rows;
    const cudaError_t e = launch_merge_pdl<float, false>(
        blocks, part_o, part_m, part_l, n_parts, rows, head_dim, (uint64_t)rows * head_dim, rows,
        out_o, out_m, out_l, stream);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace kvq

extern "C" {

int kvq_abi_version(void) { return KVQ_ABI_VERSION; }

const char* kvq_last_error(void) { return g_error.c_str(); }

int kvq_supports(uint32_t head_dim, uint32_t bits, uint32_t group_size, uint32_t dtype) {
    std::string keep = g_error;
    const int ok = check_format(head_dim, bits, group_size, dtype) == KVQ_OK;
    g_error = keep;
    return ok;
}

size_t kvq_workspace_bytes(const kvq_args* a) {
    Plan pl;
    if (plan(a, &pl) != KVQ_OK) return 0;
    return 2 * pl.ml_bytes + pl.part_bytes;
}

int kvq_decode(const kvq_args* a, void* out, void* workspace, size_t workspace_bytes, void* stream) {
    g_error.clear();
    Plan pl;
    int rc = plan(a, &pl);
    if (rc) return rc;
    if (!out) return fail(KVQ_ERR_INVALID, "out is NULL");
    if (!aligned(out, a->dtype == KVQ_F16 ? 2 : 4)) return fail(KVQ_ERR_INVALID, "out is misaligned");
    rc = check_workspace(workspace, workspace_bytes, 2 * pl.ml_bytes + pl.part_bytes);
    if (rc) return rc;
    rc = device_ok();
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    float* po = reinterpret_cast<float*>(ws);
    float* pm = reinterpret_cast<float*>(ws + pl.part_bytes);
    float* pll = reinterpret_cast<float*>(ws + pl.part_bytes + pl.ml_bytes);
    cudaError_t e = launch_partial_any(pl, a->bits, a->dtype, a->head_dim, po, pm, pll, s);
    if (e != cudaSuccess) return cuda_fail(e, "partial kernel launch");
    e = kvq::launch_merge(po, pm, pll, pl.P.n_splits, pl.rows, a->head_dim,
                          (uint64_t)pl.rows * a->head_dim, pl.rows, (int)a->dtype, out, s);
    if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
    return KVQ_OK;
}

int kvq_decode_noalloc(const kvq_args* a, void* out, void* stream) {
    g_error.clear();
    Plan pl;
    int rc = plan(a, &pl);
    if (rc) return rc;
    if (!out) return fail(KVQ_ERR_INVALID, "out is NULL");
    if (!aligned(out, a->dtype == KVQ_F16 ? 2 : 4)) return fail(KVQ_ERR_INVALID, "out is misaligned");
    const size_t need = 2 * pl.ml_bytes + pl.part_bytes;
    if (need > KVQ_NOALLOC_SCRATCH_BYTES)
        return fail(KVQ_ERR_INVALID,
                    "this step needs %zu bytes of scratch for its %u T splits, above the %u "
                    "bytes built into the library; call kvq_decode with a workspace instead",
                    need, pl.P.n_splits, (unsigned)KVQ_NOALLOC_SCRATCH_BYTES);
    rc = device_ok();
    if (rc) return rc;
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(scratch);
    float* po = reinterpret_cast<float*>(ws);
    float* pm = reinterpret_cast<float*>(ws + pl.part_bytes);
    float* pll = reinterpret_cast<float*>(ws + pl.part_bytes + pl.ml_bytes);
    cudaError_t e = launch_partial_any(pl, a->bits, a->dtype, a->head_dim, po, pm, pll, s);
    if (e != cudaSuccess) return cuda_fail(e, "partial kernel launch");
    e = kvq::launch_merge(po, pm, pll, pl.P.n_splits, pl.rows, a->head_dim,
                          (uint64_t)pl.rows * a->head_dim, pl.rows, (int)a->dtype, out, s);
    if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
    return KVQ_OK;
}

int kvq_decode_partial(const kvq_args* a, float* part_o, float* part_m, float* part_l,
                       void* workspace, size_t workspace_bytes, void* stream) {
    g_error.clear();
    Plan pl;
    int rc = plan(a, &pl);
    if (rc) return rc;
    if (!part_o || !part_m || !part_l) return fail(KVQ_ERR_INVALID, "a partial output pointer is NULL");
    if (!aligned(part_o, 4) || !aligned(part_m, 4) || !aligned(part_l, 4))
        return fail(KVQ_ERR_INVALID, "partial outputs must be 4-byte aligned");
    rc = device_ok();
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (pl.P.n_splits == 1) {
        e = launch_partial_any(pl, a->bits, a->dtype, a->head_dim, part_o, part_m, part_l, s);
        if (e != cudaSuccess) return cuda_fail(e, "partial kernel launch");
        return KVQ_OK;
    }
    rc = check_workspace(workspace, workspace_bytes, 2 * pl.ml_bytes + pl.part_bytes);
    if (rc) return rc;
    char* ws = static_cast<char*>(workspace);
    float* po = reinterpret_cast<float*>(ws);
    float* pm = reinterpret_cast<float*>(ws + pl.part_bytes);
    float* pll = reinterpret_cast<float*>(ws + pl.part_bytes + pl.ml_bytes);
    e = launch_partial_any(pl, a->bits, a->dtype, a->head_dim, po, pm, pll, s);
    if (e != cudaSuccess) return cuda_fail(e, "partial kernel launch");
    e = kvq::launch_merge_partial(po, pm, pll, pl.P.n_splits, pl.rows, a->head_dim, part_o, part_m,
                                  part_l, s);
    if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
    return KVQ_OK;
}

uint32_t kvq_split_count(const kvq_args* a) {
    std::string keep = g_error;
    Plan pl;
    const uint32_t n = plan(a, &pl) == KVQ_OK ? pl.P.n_splits : 0;
    g_error = keep;
    return n;
}

int kvq_plan_kernel(const kvq_args* a) {
    g_error.clear();
    Plan pl;
    const int rc = plan(a, &pl);
    if (rc) return rc;
    switch (pl.kernel) {
        case KERNEL_MMA4: return KVQ_KERNEL_TENSOR_CORE;
        case KERNEL_UMMA4:
        case KERNEL_TMEM4: return KVQ_KERNEL_TCGEN05;
        default: return KVQ_KERNEL_CUDA_CORE;
    }
}

int kvq_decode_splits(const kvq_args* a, float* part_o, float* part_m, float* part_l, void* stream) {
    g_error.clear();
    Plan pl;
    int rc = plan(a, &pl);
    if (rc) return rc;
    if (!part_o || !part_m || !part_l) return fail(KVQ_ERR_INVALID, "a partial output pointer is NULL");
    if (!aligned(part_o, 4) || !aligned(part_m, 4) || !aligned(part_l, 4))
        return fail(KVQ_ERR_INVALID, "partial outputs must be 4-byte aligned");
    rc = device_ok();
    if (rc) return rc;
    cudaError_t e = launch_partial_any(pl, a->bits, a->dtype, a->head_dim, part_o, part_m, part_l,
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "partial kernel launch");
    return KVQ_OK;
}

int kvq_lse_merge(const float* part_o, const float* part_m, const float* part_l, uint32_t n_parts,
                  uint32_t rows, uint32_t head_dim, uint32_t out_dtype, void* out, void* stream) {
    g_error.clear();
    if (!part_o || !part_m || !part_l || !out) return fail(KVQ_ERR_INVALID, "a pointer is NULL");
    int rc = check_merge(n_parts, rows, head_dim, out_dtype);
    if (rc) return rc;
    rc = device_ok();
    if (rc) return rc;
    cudaError_t e = kvq::launch_merge(part_o, part_m, part_l, n_parts, rows, head_dim,
                                      (uint64_t)rows * head_dim, rows, (int)out_dtype, out,
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
    return KVQ_OK;
}

int kvq_lse_merge_records(const float* records, uint32_t n_parts, uint32_t rows, uint32_t head_dim,
                          uint32_t out_dtype, void* out, void* stream) {
    g_error.clear();
    if (!records || !out) return fail(KVQ_ERR_INVALID, "a pointer is NULL");
    if (!aligned(records, 4)) return fail(KVQ_ERR_INVALID, "records must be 4-byte aligned");
    int rc = check_merge(n_parts, rows, head_dim, out_dtype);
    if (rc) return rc;
    rc = device_ok();
    if (rc) return rc;
    const uint64_t rec = (uint64_t)rows * (head_dim + 2);
    const float* m = records + (size_t)rows * head_dim;
    cudaError_t e = kvq::launch_merge(records, m, m + rows, n_parts, rows, head_dim, rec, rec,
                                      (int)out_dtype, out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
    return KVQ_OK;
}

int kvq_dequant(const uint32_t* wq, const void* scales, const void* biases, uint64_t rows,
                uint32_t head_dim, uint32_t bits, uint32_t group_size, uint32_t dtype, float* out,
                void* stream) {
    g_error.clear();
    int rc = check_format(head_dim, bits, group_size, dtype);
    if (rc) return rc;
    if (!wq || !scales || !biases || !out) return fail(KVQ_ERR_INVALID, "a pointer is NULL");
    if (rows == 0) return KVQ_OK;
    rc = device_ok();
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaErrorInvalidValue;
    switch (bits) {
        case 2: e = kvq::launch_dequant<2>(wq, scales, biases, rows, head_dim, group_size, dtype, out, s); break;
        case 3: e = kvq::launch_dequant<3>(wq, scales, biases, rows, head_dim, group_size, dtype, out, s); break;
        case 4: e = kvq::launch_dequant<4>(wq, scales, biases, rows, head_dim, group_size, dtype, out, s); break;
        case 6: e = kvq::launch_dequant<6>(wq, scales, biases, rows, head_dim, group_size, dtype, out, s); break;
        case 8: e = kvq::launch_dequant<8>(wq, scales, biases, rows, head_dim, group_size, dtype, out, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "dequant kernel launch");
    return KVQ_OK;
}

static int quantize_rows(const void* w, uint64_t rows, uint32_t head_dim, uint32_t bits,
                         uint32_t group_size, uint32_t dtype, uint32_t* wq, void* scales,
                         void* biases, const kvq::QuantDest& dst, void* stream) {
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaErrorInvalidValue;
    switch (bits) {
        case 2: e = kvq::launch_quantize<2>(w, rows, head_dim, group_size, dtype, wq, scales, biases, dst, s); break;
        case 3: e = kvq::launch_quantize<3>(w, rows, head_dim, group_size, dtype, wq, scales, biases, dst, s); break;
        case 4: e = kvq::launch_quantize<4>(w, rows, head_dim, group_size, dtype, wq, scales, biases, dst, s); break;
        case 6: e = kvq::launch_quantize<6>(w, rows, head_dim, group_size, dtype, wq, scales, biases, dst, s); break;
        case 8: e = kvq::launch_quantize<8>(w, rows, head_dim, group_size, dtype, wq, scales, biases, dst, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "quantize kernel launch");
    return KVQ_OK;
}

int kvq_quantize(const void* w, uint64_t rows, uint32_t head_dim, uint32_t bits, uint32_t group_size,
                 uint32_t dtype, uint32_t* wq, void* scales, void* biases, void* stream) {
    g_error.clear();
    int rc = check_format(head_dim, bits, group_size, dtype);
    if (rc) return rc;
    if (!w || !wq || !scales || !biases) return fail(KVQ_ERR_INVALID, "a pointer is NULL");
    if (rows == 0) return KVQ_OK;
    rc = device_ok();
    if (rc) return rc;
    const kvq::QuantDest dst{nullptr, 0u, 1u, 0u, 0u, 0u};
    return quantize_rows(w, rows, head_dim, bits, group_size, dtype, wq, scales, biases, dst, stream);
}

int kvq_cache_append(const void* w, uint32_t b_rows, uint32_t n_kv_heads, uint32_t n_new,
                     uint32_t head_dim, uint32_t bits, uint32_t group_size, uint32_t dtype,
                     const int32_t* positions, uint32_t position, uint32_t t_stride,
                     uint64_t cache_batch_stride, uint32_t* wq, void* scales, void* biases,
                     void* stream) {
    g_error.clear();
    int rc = check_format(head_dim, bits, group_size, dtype);
    if (rc) return rc;
    if (!w || !wq || !scales || !biases) return fail(KVQ_ERR_INVALID, "a pointer is NULL");
    if (b_rows == 0 || n_kv_heads == 0 || n_new == 0) return KVQ_OK;
    if (t_stride == 0) return fail(KVQ_ERR_INVALID, "t_stride is 0");
    if (!positions && (uint64_t)position + n_new > t_stride)
        return fail(KVQ_ERR_INVALID, "position %u + n_new %u runs past t_stride %u", position,
                    n_new, t_stride);
    if (b_rows > 1 && cache_batch_stride != 0 &&
        cache_batch_stride < (uint64_t)n_kv_heads * t_stride)
        return fail(KVQ_ERR_INVALID, "cache_batch_stride %llu overlaps the %u x %u rows of a "
                    "sequence", (unsigned long long)cache_batch_stride, n_kv_heads, t_stride);
    if (b_rows > 1 && cache_batch_stride == 0)
        return fail(KVQ_ERR_INVALID, "b_rows > 1 needs one cache per sequence "
                    "(cache_batch_stride > 0): appends of a shared cache would collide");
    rc = device_ok();
    if (rc) return rc;
    const uint64_t rows = (uint64_t)b_rows * n_kv_heads * n_new;
    const kvq::QuantDest dst{positions, position, n_kv_heads, n_new, t_stride, cache_batch_stride};
    return quantize_rows(w, rows, head_dim, bits, group_size, dtype, wq, scales, biases, dst, stream);
}

// ---------------------------------------------------------------------------
// The one-kernel sequence split (kvq_fused.cuh)
// ---------------------------------------------------------------------------
static bool tsplit_plan_ok(const kvq_args* a, const Plan& pl) {
    return pl.kernel == KERNEL_MMA4 && a->bits == 4 && a->group_size == 64;
}

// The one-kernel step's split plan: for two CTAs per SM, not the three that
// fit -- with the merge in the same launch, fewer and longer splits measured
// faster at every shard size on a B200 (T = 16384 .. 131072, 8 cache heads:
// fewer partials to merge, fewer streaming CTAs beside each merging one) --
// and within the region's partial store (at most part_rows / rows splits).
static void tsplit_replan(const kvq_args* a, Plan* pl) {
    const uint32_t end = a->t_end < a->t_cached ? a->t_end : a->t_cached;
    const uint64_t span = end > a->t_begin ? end - a->t_begin : 0;
    const uint64_t units = (uint64_t)a->b_rows * a->n_kv_heads * pl->P.head_tiles;
    const uint64_t stage = (uint64_t)kvq::mma4_stage_positions();
    mma4_splits(span, units, 2, &pl->P.chunk, &pl->P.n_splits, stage, kMmaRamp);
    const uint64_t cap = kvq::fused::part_rows(pl->rows) / pl->rows;
    if (pl->P.n_splits > cap) {
        const uint64_t chunk = ((span + cap - 1) / cap + stage - 1) / stage * stage;
        pl->P.chunk = (uint32_t)chunk;
        pl->P.n_splits = (uint32_t)((span + chunk - 1) / chunk);
    }
}

uint32_t kvq_tsplit_split_count(const kvq_args* a) {
    std::string keep = g_error;
    Plan pl;
    uint32_t n = 0;
    if (plan(a, &pl) == KVQ_OK && tsplit_plan_ok(a, pl)) {
        tsplit_replan(a, &pl);
        n = pl.P.n_splits;
    }
    g_error = keep;
    return n;
}

size_t kvq_tsplit_region_bytes(uint32_t rows, uint32_t head_dim, uint32_t world) {
    if (rows == 0 || head_dim != kvq::fused::DH || world == 0 || world > KVQ_PEER_MAX_RANKS) return 0;
    return (size_t)kvq::fused::region_layout(rows, world).total;
}

int kvq_tsplit_supported(const kvq_args* a) {
    std::string keep = g_error;
    Plan pl;
    const int ok = plan(a, &pl) == KVQ_OK && tsplit_plan_ok(a, pl);
    g_error = keep;
    return ok;
}

int kvq_tsplit_decode(const kvq_args* a, void* const* regions, size_t region_bytes, uint32_t world,
                      uint32_t rank, void* out, uint64_t timeout_us, void* stream) {
    g_error.clear();
    Plan pl;
    int rc = plan(a, &pl);
    if (rc) return rc;
    if (!tsplit_plan_ok(a, pl))
        return fail(KVQ_ERR_UNSUPPORTED, "the one-kernel sequence split serves the tensor-core "
                    "kernel's 4-bit group-64 format (fp16, head_dim 128, at most 8 query heads "
                    "per cache head, 8-row-aligned geometry); use kvq_decode_partial and "
                    "kvq_peer_merge");
    if (!regions || !out) return fail(KVQ_ERR_INVALID, "regions or out is NULL");
    if (world == 0 || world > KVQ_PEER_MAX_RANKS || rank >= world)
        return fail(KVQ_ERR_INVALID, "world must be 1..%d and rank < world", KVQ_PEER_MAX_RANKS);
    for (uint32_t p = 0; p < world; ++p)
        if (!regions[p] || !aligned(regions[p], 256))
            return fail(KVQ_ERR_INVALID, "region %u is NULL or not 256-byte aligned", p);
    if (!aligned(out, 8)) return fail(KVQ_ERR_INVALID, "out must be 8-byte aligned");
    const kvq::fused::Layout L = kvq::fused::region_layout(pl.rows, world);
    if (region_bytes < L.total)
        return fail(KVQ_ERR_INVALID, "regions of %zu bytes are smaller than the %llu this step "
                    "needs (kvq_tsplit_region_bytes)", region_bytes, (unsigned long long)L.total);
    tsplit_replan(a, &pl);
    rc = device_ok();
    if (rc) return rc;
    // the merging CTAs wait for the rest of their unit: they must leave room
    // on the device for every other CTA
    const uint64_t units = (uint64_t)a->b_rows * a->n_kv_heads * pl.P.head_tiles;
    const uint64_t kmax = 2ull * (uint32_t)pl.ht;   // merging CTAs per unit: two per head row
    const uint64_t k = pl.P.n_splits < kmax ? pl.P.n_splits : kmax;
    const uint64_t resident = (uint64_t)kvq::mma4_fused_ctas_per_sm(pl.ht) * kvq::sm_count();
    if (units * k >= resident)
        return fail(KVQ_ERR_UNSUPPORTED, "%llu units x %llu merging CTAs would fill the %llu "
                    "resident CTAs; use kvq_decode_partial and kvq_peer_merge",
                    (unsigned long long)units, (unsigned long long)k, (unsigned long long)resident);
    kvq::fused::Fused F{};
    for (uint32_t p = 0; p < world; ++p) F.region[p] = static_cast<unsigned char*>(regions[p]);
    F.world = world;
    F.rank = rank;
    F.L = L;
    F.timeout_ns = (timeout_us ? timeout_us : 2000000ull) * 1000ull;
    F.out = static_cast<__half*>(out);
    cudaError_t e = kvq::launch_mma4_fused(pl.P, pl.ht, fast_precision() ? 2 : 3, F,
                                           static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "one-kernel sequence split launch");
    return KVQ_OK;
}

// ---------------------------------------------------------------------------
// Staging copies for per-token host<->device traffic
// ---------------------------------------------------------------------------
namespace {
// One CTA per 64 KiB, 16 bytes per thread per step: the GPU reads (or
// writes) the host side directly through its mapping, so a copy of a few KB
// costs a kernel launch and one bus round trip rather than a copy engine's
// fixed latency.
__global__ void __launch_bounds__(256) stage_copy_kernel(uint4* __restrict__ dst,
                                                        const uint4* __restrict__ src, size_t n16,
                                                        unsigned char* __restrict__ dst_tail,
                                                        const unsigned char* __restrict__ src_tail,
                                                        uint32_t tail) {
    const size_t per_cta = 4096;   // 16-byte words per CTA
    const size_t lo = (size_t)blockIdx.x * per_cta;
    const size_t hi = lo + per_cta < n16 ? lo + per_cta : n16;
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
    if (blockIdx.x == 0 && threadIdx.x < tail) dst_tail[threadIdx.x] = src_tail[threadIdx.x];
}
}  // namespace

int kvq_stage_copy(void* dst, const void* src, size_t bytes, void* stream) {
    g_error.clear();
    if (bytes == 0) return KVQ_OK;
    if (!dst || !src) return fail(KVQ_ERR_INVALID, "kvq_stage_copy: a pointer is NULL");
    if (!aligned(dst, 16) || !aligned(src, 16))
        return fail(KVQ_ERR_INVALID, "kvq_stage_copy: both pointers must be 16-byte aligned");
    const int rc = device_ok();
    if (rc) return rc;
    // the GPU dereferences both sides: ordinary (pageable) host memory is not
    // mapped into its address space and would fault the device, so it is
    // refused here
    for (const void* p : {static_cast<const void*>(dst), src}) {
        cudaPointerAttributes at{};
        const cudaError_t e = cudaPointerGetAttributes(&at, p);
        if (e != cudaSuccess) return cuda_fail(e, "kvq_stage_copy: pointer query");
        if (at.type == cudaMemoryTypeUnregistered)
            return fail(KVQ_ERR_INVALID, "kvq_stage_copy: %p is pageable host memory; pin it "
                        "(cudaHostAlloc / torch pin_memory) or pass device memory", p);
    }
    const size_t n16 = bytes / 16;
    const uint32_t tail = (uint32_t)(bytes % 16);
    const unsigned blocks = (unsigned)((n16 + 4095) / 4096 > 0 ? (n16 + 4095) / 4096 : 1);
    stage_copy_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint4*>(dst), static_cast<const uint4*>(src), n16,
        static_cast<unsigned char*>(dst) + n16 * 16, static_cast<const unsigned char*>(src) + n16 * 16,
        tail);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KVQ_OK : cuda_fail(e, "staging copy launch");
}

}  // extern "C"
