// Sequence split over peer memory: each rank's partial record lives in an
// exchange region in its own GPU memory, mapped into every peer's address
// space over CUDA IPC (NVLink / NVSwitch); one kernel signals the peers that
// this step's record is ready, waits (bounded) for theirs, and merges all
// ranks' records by log-sum-exp reading them in place with plain loads -- the
// all-gather and the merge in one launch, no NCCL, no multicast.
//
// Region layout (bytes): [0] step counter, [4] blocks done in the current
// merge, [8] status (0 ok, 1 a peer's flag did not arrive in time), [64 + 4p]
// the flag peer p writes (the last step it has published), [256 + parity *
// record] two partial records of rows * (head_dim + 2) floats (O, then m, then
// l), double-buffered by step parity.
//
// Step e (the region's counter + 1) on rank r: the local partial has written
// record e & 1; every block of the merge kernel fences (system scope) and
// stores e into every peer's flag slot r -- the same value from every block,
// so no block's wait depends on another block of this launch being scheduled
// -- then waits until its own flags from every peer are >= e (then reads each
// once with acquire semantics), merges the records of parity e & 1, and the
// last block sets the counter to e. A peer can only overwrite the record of
// parity e & 1 at step e + 2, after its merge of step e + 1 saw this rank's
// flag e + 1, which this rank stores only after its merge of step e has
// finished: the double buffer is never overwritten while read.
//
// The caller names the parity its partial wrote; when that is not e & 1 (the
// caller's step count and the region's disagree) the kernel publishes
// nothing, so no peer merges a record from the wrong slot: the status word
// becomes 2, the rows NaN, and the counter still advances.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>

#include "kvq_b200.h"
#include "kvq_common.cuh"

namespace kvq {
namespace peer {

constexpr int MAX_RANKS = KVQ_PEER_MAX_RANKS;
constexpr uint32_t CTRL_EPOCH = 0, CTRL_DONE = 4, CTRL_STATUS = 8, FLAGS = 64, RECORDS = 256;
constexpr uint32_t STATUS_TIMEOUT = 1, STATUS_PARITY = 2;
constexpr int THREADS = 128;

struct Regions {
    unsigned char* r[MAX_RANKS];
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One block per row; thread d owns dims d, d + THREADS, ...
template <typename TO>
__global__ void __launch_bounds__(THREADS)
peer_merge_kernel(Regions regions, uint32_t world, uint32_t rank, uint32_t parity, uint32_t rows,
                  uint32_t head_dim, uint64_t record_bytes, uint64_t timeout_ns, TO* __restrict__ out) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_bad;
    unsigned char* self = regions.r[rank];
    const uint32_t row = blockIdx.x;
    const int tid = threadIdx.x;

    if (tid == 0) {
        const uint32_t e = *reinterpret_cast<volatile uint32_t*>(self + CTRL_EPOCH) + 1;
        s_epoch = e;
        const bool parity_ok = parity == (e & 1u);
        // this rank's record for step e is complete (the kernels before this
        // one wrote it): every block publishes it to every peer, one
        // system-scope fence ahead of the flag stores
        if (parity_ok) {
            __threadfence_system();
            for (uint32_t p = 0; p < world; ++p)
                st_relaxed_sys(reinterpret_cast<uint32_t*>(regions.r[p] + FLAGS + 4 * rank), e);
        }
        // every peer's record for step e (relaxed polling, then one acquiring
        // read per flag), or give up after timeout_ns
        bool ok = parity_ok;
        const uint64_t t0 = globaltimer();
        for (uint32_t p = 0; p < world && ok; ++p) {
            const uint32_t* flag = reinterpret_cast<const uint32_t*>(self + FLAGS + 4 * p);
            uint32_t spins = 0;
            while (ld_relaxed_sys(flag) < e) {
                if ((++spins & 63u) == 0 && globaltimer() - t0 > timeout_ns) {
                    ok = false;
                    break;
                }
                if (spins > 256) __nanosleep(64);
            }
            if (ok) (void)ld_acquire_sys(flag);
        }
        s_bad = ok ? 0 : 1;
        if (!ok)
            atomicExch(reinterpret_cast<unsigned int*>(self + CTRL_STATUS),
                       parity_ok ? STATUS_TIMEOUT : STATUS_PARITY);
    }
    __syncthreads();

    const uint64_t rec_off = RECORDS + parity * record_bytes;
    const size_t o_floats = (size_t)rows * head_dim;
    float mp[MAX_RANKS], lp[MAX_RANKS];
    float m = -INFINITY;
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
        mp[p] = -INFINITY;
        lp[p] = 0.0f;
        if ((uint32_t)p < world) {
            const float* rec = reinterpret_cast<const float*>(regions.r[p] + rec_off);
            mp[p] = rec[o_floats + row];
            lp[p] = rec[o_floats + rows + row];
            m = fmaxf(m, mp[p]);
        }
    }
    float w[MAX_RANKS];
    float l = 0.0f;
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
        w[p] = ((uint32_t)p < world && mp[p] != -INFINITY) ? expf(mp[p] - m) : 0.0f;
        if (w[p] != 0.0f) l = fmaf(lp[p], w[p], l);
    }
    const bool bad = s_bad != 0;
    for (uint32_t d = tid; d < head_dim; d += THREADS) {
        float ov[MAX_RANKS];
#pragma unroll
        for (int p = 0; p < MAX_RANKS; ++p) {
            const float* rec = reinterpret_cast<const float*>(regions.r[p < (int)world ? p : 0] + rec_off);
            ov[p] = ((uint32_t)p < world && w[p] != 0.0f) ? rec[(size_t)row * head_dim + d] : 0.0f;
        }
        float o = 0.0f;
#pragma unroll
        for (int p = 0; p < MAX_RANKS; ++p)
            if (w[p] != 0.0f) o = fmaf(ov[p], w[p], o);
        out[(size_t)row * head_dim + d] = from_f32<TO>(bad ? __int_as_float(0x7fc00000) : o / l);
    }

    // the last block to finish advances the step counter
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        unsigned int* done = reinterpret_cast<unsigned int*>(self + CTRL_DONE);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile uint32_t*>(self + CTRL_EPOCH) = s_epoch;
            *reinterpret_cast<volatile unsigned int*>(done) = 0u;
            __threadfence();
        }
    }
}

}  // namespace peer
}  // namespace kvq

namespace {
thread_local std::string g_peer_error;

int peer_fail(int code, const char* what, cudaError_t e = cudaSuccess) {
    char buf[256];
    if (e != cudaSuccess)
        snprintf(buf, sizeof buf, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    else
        snprintf(buf, sizeof buf, "%s", what);
    g_peer_error = buf;
    return code;
}

uint64_t record_bytes(uint32_t rows, uint32_t head_dim) {
    const uint64_t b = (uint64_t)rows * (head_dim + 2) * sizeof(float);
    return (b + 255) / 256 * 256;
}
}  // namespace

extern "C" {

size_t kvq_peer_region_bytes(uint32_t rows, uint32_t head_dim) {
    return kvq::peer::RECORDS + 2 * record_bytes(rows, head_dim);
}

size_t kvq_peer_record_offset(uint32_t rows, uint32_t head_dim, uint32_t parity) {
    return kvq::peer::RECORDS + (parity & 1u) * record_bytes(rows, head_dim);
}

const char* kvq_peer_last_error(void) { return g_peer_error.c_str(); }

int kvq_peer_alloc(size_t bytes, void** region, void* ipc_handle) {
    g_peer_error.clear();
    if (!region || !ipc_handle || bytes < kvq::peer::RECORDS)
        return peer_fail(KVQ_ERR_INVALID, "kvq_peer_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return peer_fail(KVQ_ERR_LAUNCH, "cudaMalloc of the exchange region", e);
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, p);
        if (e == cudaSuccess) {
            memcpy(ipc_handle, &h, sizeof h);
            *region = p;
            return KVQ_OK;
        }
    }
    cudaFree(p);
    return peer_fail(KVQ_ERR_LAUNCH, "exchange region setup", e);
}

int kvq_peer_free(void* region) {
    g_peer_error.clear();
    cudaError_t e = cudaFree(region);
    return e == cudaSuccess ? KVQ_OK : peer_fail(KVQ_ERR_LAUNCH, "cudaFree of the exchange region", e);
}

int kvq_peer_open(const void* ipc_handle, void** region) {
    g_peer_error.clear();
    if (!ipc_handle || !region) return peer_fail(KVQ_ERR_INVALID, "kvq_peer_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? KVQ_OK : peer_fail(KVQ_ERR_LAUNCH, "cudaIpcOpenMemHandle", e);
}

int kvq_peer_close(void* region) {
    g_peer_error.clear();
    cudaError_t e = cudaIpcCloseMemHandle(region);
    return e == cudaSuccess ? KVQ_OK : peer_fail(KVQ_ERR_LAUNCH, "cudaIpcCloseMemHandle", e);
}

int kvq_peer_merge(void* const* regions, uint32_t world, uint32_t rank, uint32_t parity, uint32_t rows,
                   uint32_t head_dim, uint32_t out_dtype, void* out, uint64_t timeout_us, void* stream) {
    g_peer_error.clear();
    if (!regions || !out) return peer_fail(KVQ_ERR_INVALID, "kvq_peer_merge: a pointer is NULL");
    if (world == 0 || world > (uint32_t)kvq::peer::MAX_RANKS || rank >= world)
        return peer_fail(KVQ_ERR_INVALID, "kvq_peer_merge: world must be 1..KVQ_PEER_MAX_RANKS and rank < world");
    if (rows == 0 || rows > 0x7FFFFFFFu || head_dim == 0 || head_dim > 1024)
        return peer_fail(KVQ_ERR_INVALID, "kvq_peer_merge: bad rows or head_dim");
    if (out_dtype != KVQ_F16 && out_dtype != KVQ_F32)
        return peer_fail(KVQ_ERR_INVALID, "kvq_peer_merge: bad out_dtype");
    kvq::peer::Regions r;
    for (int p = 0; p < kvq::peer::MAX_RANKS; ++p) r.r[p] = nullptr;
    for (uint32_t p = 0; p < world; ++p) {
        if (!regions[p]) return peer_fail(KVQ_ERR_INVALID, "kvq_peer_merge: a region pointer is NULL");
        r.r[p] = static_cast<unsigned char*>(regions[p]);
    }
    const uint64_t timeout_ns = (timeout_us ? timeout_us : 2000000ull) * 1000ull;
    auto s = static_cast<cudaStream_t>(stream);
    if (out_dtype == KVQ_F16)
        kvq::peer::peer_merge_kernel<__half><<<rows, kvq::peer::THREADS, 0, s>>>(
            r, world, rank, parity & 1u, rows, head_dim, record_bytes(rows, head_dim), timeout_ns,
            static_cast<__half*>(out));
    else
        kvq::peer::peer_merge_kernel<float><<<rows, kvq::peer::THREADS, 0, s>>>(
            r, world, rank, parity & 1u, rows, head_dim, record_bytes(rows, head_dim), timeout_ns,
            static_cast<float*>(out));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KVQ_OK : peer_fail(KVQ_ERR_LAUNCH, "peer merge launch", e);
}

int kvq_peer_status(const void* region, uint32_t* status, void* stream) {
    g_peer_error.clear();
    if (!region || !status) return peer_fail(KVQ_ERR_INVALID, "kvq_peer_status: a pointer is NULL");
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status, static_cast<const unsigned char*>(region) + kvq::peer::CTRL_STATUS,
                                    sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? KVQ_OK : peer_fail(KVQ_ERR_LAUNCH, "reading the exchange status", e);
}

}  // extern "C"
