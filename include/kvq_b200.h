/*
 * kvq_b200.h -- C ABI of the B200 (sm_100a) quantized-KV decode attention.
 *
 * One decode step of attention over an MLX-affine packed K/V cache: per
 * (batch row b, query head h), scores q . dequant(K_t) / sqrt(DH) over the
 * logical cached positions t plus the step's own new entry (new_k at full
 * precision), an fp32 max-shifted softmax over T+1, and the combine
 * sum_t p_t dequant(V_t) + p_new new_v, cast once to the output dtype.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * handle (a cudaStream_t passed as void*; NULL is the legacy default stream).
 * The decode entry points never allocate device memory: scratch space
 * ("workspace") is passed in, sized by kvq_workspace_bytes(). The one
 * allocation the library makes is the sequence-split exchange region of
 * kvq_peer_alloc() (cudaMalloc: it must be IPC-shareable with the peer ranks),
 * made once at setup and released by kvq_peer_free(). Calls are asynchronous on the
 * given stream, reentrant, and return KVQ_OK or a negative status; the
 * message of the calling thread's last failure is kvq_last_error().
 * Nothing here aborts or traps.
 *
 * The packed-cache layout is the reference's (MLX affine):
 *   wq     uint32 [rows, DH*bits/32]  contiguous little-endian code stream per
 *                                     row, code i at bit i*bits (3- and 6-bit
 *                                     codes straddle words)
 *   scales dtype  [rows, DH/group]    per-group scale, stored in the cache's
 *   biases dtype  [rows, DH/group]    dtype (fp16 caches: fp16)
 * A row is one (cache head, position). Row index of (b, kv head hk, t):
 *   b * cache_batch_stride + hk * t_stride + t
 * cache_batch_stride = 0 is the reference's cache shared by every batch row;
 * cache_batch_stride = n_kv_heads * t_stride is one cache per sequence.
 * Query head h reads cache head h / (n_heads / n_kv_heads) (contiguous GQA
 * blocks); new_k/new_v are [b_rows, n_kv_heads, DH].
 */
#ifndef KVQ_B200_H
#define KVQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVQ_ABI_VERSION 1

/* status codes */
#define KVQ_OK 0
#define KVQ_ERR_INVALID (-1)     /* bad shape, bits, group, dtype, alignment or size  */
#define KVQ_ERR_LAUNCH (-2)      /* a CUDA launch or configuration error              */
#define KVQ_ERR_UNSUPPORTED (-3) /* no device, or not an sm_100 device; for
                                    kvq_tsplit_decode also a format it does not serve */

/* element type of q, new_k, new_v, out, scales and biases */
#define KVQ_F16 0
#define KVQ_F32 1

/* "to the end of the sequence" for kvq_args.t_end */
#define KVQ_T_END_ALL 0xFFFFFFFFu

/*
 * One decode step. Replaces the raw-door binding list of kernelverify's
 * kv_attn_decode (kernelverify/pack/kv_attention.py:302-351: q, k_wq,
 * k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, out, n_heads,
 * t_cached, n_kv_heads, t_stride, grid extent b_rows) and extends it with the
 * group size (the reference fixes 64), per-sequence caches, ragged lengths
 * and a T-range shard.
 */
typedef struct kvq_args {
    const void* q;            /* [b_rows, n_heads, head_dim] dtype            */
    const uint32_t* k_wq;     /* packed K codes                                */
    const void* k_scales;     /* K per-group scales, dtype                     */
    const void* k_biases;     /* K per-group biases, dtype                     */
    const uint32_t* v_wq;     /* packed V codes                                */
    const void* v_scales;
    const void* v_biases;
    const void* new_k;        /* [b_rows, n_kv_heads, head_dim] dtype          */
    const void* new_v;
    const int32_t* seq_lens;  /* [b_rows] logical cached lengths, or NULL: every
                                 row has t_cached                              */
    uint32_t b_rows;
    uint32_t n_heads;         /* query heads                                   */
    uint32_t n_kv_heads;      /* cache heads; n_heads % n_kv_heads == 0         */
    uint32_t t_cached;        /* logical cached positions (when seq_lens NULL)  */
    uint32_t t_stride;        /* physical rows per cache head (>= every length);
                                 the tensor-core kernels need it, the batch
                                 stride and t_begin to be multiples of 8 and
                                 every buffer 16-byte aligned, else the
                                 CUDA-core kernel serves the call            */
    uint32_t head_dim;        /* 64 or 128                                     */
    uint32_t bits;            /* 2, 3, 4, 6 or 8                               */
    uint32_t group_size;      /* 32, 64 or 128; divides head_dim               */
    uint32_t dtype;           /* KVQ_F16 or KVQ_F32                            */
    uint32_t has_new_entry;   /* 1: the step's own K/V enter this call          */
    uint64_t cache_batch_stride; /* rows between batch rows' caches; 0 = shared */
    uint32_t t_begin;         /* first position of this call's T range          */
    uint32_t t_end;           /* one past the last (clamped to each length)     */
} kvq_args;

/* Bytes of scratch `kvq_decode` / `kvq_decode_partial` need for these
 * arguments (0 when none); `workspace` must be 256-byte aligned. */
size_t kvq_workspace_bytes(const kvq_args* a);

/*
 * The full step: out [b_rows, n_heads, head_dim] in args->dtype.
 * Long caches are split along T into chunks processed in parallel, each
 * producing an unnormalised partial (O, m, l), merged by a log-sum-exp
 * combine (the reference kernel's T <= 1024 capacity bound does not exist
 * here). Reference: kv_attn_decode, kernelverify/pack/kv_attention.py:85-234.
 */
int kvq_decode(const kvq_args* a, void* out, void* workspace, size_t workspace_bytes,
               void* stream);

/*
 * One T-range shard of the step (positions [t_begin, t_end) of every row,
 * plus the new entry when has_new_entry): the merged partial of that shard,
 *   part_o [b_rows, n_heads, head_dim] fp32, unnormalised, relative to part_m
 *   part_m [b_rows, n_heads]           fp32, max score (-inf: empty shard)
 *   part_l [b_rows, n_heads]           fp32, sum of exp(score - part_m)
 * Sharding a sequence by T range across GPUs and merging the shards with
 * kvq_lse_merge gives the same step as kvq_decode. No reference counterpart
 * (the reference kernel is single-pass, kernelverify/pack/kv_attention.py:53-65).
 */
int kvq_decode_partial(const kvq_args* a, float* part_o, float* part_m, float* part_l,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * Which kernel kvq_decode would run for these arguments (host only, no device
 * work): one of the KVQ_KERNEL_* values, or a negative status when the
 * arguments are invalid. A serving loop checks it once per cache geometry:
 * a call that silently left the tensor-core kernels (an unaligned t_stride,
 * a format they do not carry) still computes the same step, only slower.
 */
#define KVQ_KERNEL_CUDA_CORE 0
#define KVQ_KERNEL_TENSOR_CORE 1   /* register-fragment mma.sync kernels: fp16,
                                      head_dim 128, <= 8 query heads per cache
                                      head, every width and group */
#define KVQ_KERNEL_TCGEN05 2       /* the tcgen05 kernel (KVQ_KERNEL=umma)  */
int kvq_plan_kernel(const kvq_args* a);

/* Number of T splits kvq_decode_splits produces for these arguments (0 when
 * the arguments are invalid). */
uint32_t kvq_split_count(const kvq_args* a);

/*
 * The split stage of kvq_decode on its own: one unnormalised partial per
 * (T split, row), part_o [n_splits, b_rows*n_heads, head_dim] fp32 and
 * part_m/part_l [n_splits, b_rows*n_heads], n_splits = kvq_split_count(a).
 * kvq_lse_merge over them with n_parts = n_splits is kvq_decode's output.
 * Needs no workspace.
 */
int kvq_decode_splits(const kvq_args* a, float* part_o, float* part_m, float* part_l,
                      void* stream);

/*
 * Log-sum-exp merge of n_parts partials of `rows` (= b_rows * n_heads) rows:
 * part_o [n_parts, rows, head_dim], part_m/part_l [n_parts, rows]; part p
 * starts at p * rows rows. m = max_p m_p, l = sum_p l_p e^(m_p - m),
 * out = sum_p O_p e^(m_p - m) / l cast to out_dtype.
 */
int kvq_lse_merge(const float* part_o, const float* part_m, const float* part_l,
                  uint32_t n_parts, uint32_t rows, uint32_t head_dim, uint32_t out_dtype,
                  void* out, void* stream);

/*
 * A partial record: one shard's kvq_decode_partial output in one buffer of
 * KVQ_RECORD_FLOATS(rows, head_dim) floats, O [rows, head_dim] first, then
 * m [rows], then l [rows] (pass part_o = rec, part_m = rec + rows*head_dim,
 * part_l = part_m + rows). An all-gather of every rank's record lays them end
 * to end, and kvq_lse_merge_records merges them there: one collective per
 * step instead of three. No reference counterpart (the reference has no
 * multi-GPU path).
 */
#define KVQ_RECORD_FLOATS(rows, head_dim) ((size_t)(rows) * ((size_t)(head_dim) + 2))
int kvq_lse_merge_records(const float* records, uint32_t n_parts, uint32_t rows,
                          uint32_t head_dim, uint32_t out_dtype, void* out, void* stream);

/*
 * Sequence split over peer memory (no reference counterpart; the reference
 * has no multi-GPU path). Each rank allocates one exchange region in its own
 * GPU memory (kvq_peer_alloc, zeroed, exported as a 64-byte CUDA IPC handle),
 * every rank maps every peer's region (kvq_peer_open, from its own device),
 * and each step:
 *   1. the local partial (kvq_decode_partial) writes this rank's record into
 *      its own region at kvq_peer_record_offset(rows, head_dim, parity) --
 *      O [rows, head_dim], then m [rows], then l [rows], fp32 -- where parity
 *      is (step number + 1) & 1, steps counted from 0 on every rank alike;
 *   2. kvq_peer_merge publishes the record to the peers (a flag store into each
 *      peer's region after a system-scope fence), waits for every peer's flag
 *      of this step in its own region (bounded by timeout_us, 0 = 2 s), and
 *      merges all ranks' records by log-sum-exp reading them over NVLink:
 *      out [rows, head_dim] in out_dtype, identical on every rank.
 * regions[p] is rank p's region as mapped in this process (this rank's own at
 * regions[rank]). A wait that times out sets the region's status word (read
 * it with kvq_peer_status) and writes NaN rows; the kernel always returns.
 * Regions must be freed (kvq_peer_free) only after every peer has closed its
 * mapping (kvq_peer_close).
 */
#define KVQ_PEER_MAX_RANKS 8
#define KVQ_PEER_HANDLE_BYTES 64
size_t kvq_peer_region_bytes(uint32_t rows, uint32_t head_dim);
size_t kvq_peer_record_offset(uint32_t rows, uint32_t head_dim, uint32_t parity);
int kvq_peer_alloc(size_t bytes, void** region, void* ipc_handle);
int kvq_peer_open(const void* ipc_handle, void** region);
int kvq_peer_close(void* region);
int kvq_peer_free(void* region);
int kvq_peer_merge(void* const* regions, uint32_t world, uint32_t rank, uint32_t parity,
                   uint32_t rows, uint32_t head_dim, uint32_t out_dtype, void* out,
                   uint64_t timeout_us, void* stream);
/* status word of a region: 0 ok, 1 a peer's flag did not arrive in time, 2 a
 * merge named a parity other than its step's (nothing was published; the
 * rows are NaN), 3 (kvq_tsplit_decode's regions) a unit's partials did not
 * all arrive in time */
int kvq_peer_status(const void* region, uint32_t* status, void* stream);
/* the calling thread's last error from a kvq_peer_* call ("" when none) */
const char* kvq_peer_last_error(void);

/*
 * The sequence split as ONE kernel per rank per step (no reference
 * counterpart; the reference has no multi-GPU path -- this is its single-GPU
 * door kernelverify/pack/kv_attention.py:369-393 with the cached positions
 * sharded by T range over `world` GPUs). a describes this rank's shard
 * (t_begin 0, t_end = t_cached = the shard's positions; has_new_entry on one
 * rank only). The split stage's CTAs write their partials into this rank's
 * region; the last CTAs of each unit merge them, store each head row's record
 * into every rank's region, read every rank's record of the row from their
 * own region (bounded by timeout_us, 0 = 2 s) and write the merged rows into
 * out [b_rows * n_heads, head_dim] (fp16), identical on every rank. Every
 * exchanged word carries the step number, so no fence or flag is involved.
 * world 1 is the whole sequence on one GPU, a single launch.
 *
 * Regions: one per rank, kvq_tsplit_region_bytes(b_rows * n_heads, head_dim,
 * world) bytes (0 for a head_dim other than 128), allocated zeroed and mapped
 * exactly as for kvq_peer_merge (kvq_peer_alloc / kvq_peer_open /
 * kvq_peer_close / kvq_peer_free); region_bytes is that size. The step count
 * lives in the region, so a CUDA graph of one call replays every later step;
 * every rank must run every step. Status word (kvq_peer_status): 0 ok, 1 a
 * peer's record did not arrive in time (rows NaN), 3 a unit's partials did
 * not all arrive in time (rows NaN; the region's step counts are out of step,
 * so it must be freed and allocated again). No workspace: the partials live in
 * the region (at most 64 splits per row; the split plan is capped to fit).
 * Returns KVQ_ERR_UNSUPPORTED for a format or size this form does not serve
 * (kvq_tsplit_supported says which, without a device): it serves the
 * tensor-core kernel's 4-bit group-64 format, and geometries whose merging
 * CTAs leave room for the rest on the device.
 */
/*
 * Copy `bytes` between device memory and pinned (page-locked, mapped) host
 * memory, either way round, with one small kernel on `stream`: the GPU reads
 * or writes the host side through its mapping. For per-token staging of a
 * decode step's inputs and output, where a copy engine's fixed latency (about
 * 6 us per transfer measured on a B200) is most of the cost. Both pointers
 * 16-byte aligned; host memory must be pinned (cudaHostAlloc / torch
 * pin_memory): pageable host memory is refused with KVQ_ERR_INVALID. No
 * reference counterpart (the reference's unified memory needs
 * no copies).
 */
int kvq_stage_copy(void* dst, const void* src, size_t bytes, void* stream);

size_t kvq_tsplit_region_bytes(uint32_t rows, uint32_t head_dim, uint32_t world);
int kvq_tsplit_supported(const kvq_args* a);
/* splits per unit kvq_tsplit_decode plans for a (0 when it does not serve a) */
uint32_t kvq_tsplit_split_count(const kvq_args* a);
int kvq_tsplit_decode(const kvq_args* a, void* const* regions, size_t region_bytes, uint32_t world,
                      uint32_t rank, void* out, uint64_t timeout_us, void* stream);

/*
 * fp32 dequantized values [rows, head_dim] of a packed artefact: scale * code
 * + bias per group, a rounded multiply then a rounded add -- bit-exact to the
 * reference's _cache_dequant (kernelverify/reference/native_kernels.py:153-165,
 * kernelverify/schemas/quant_contract.py:107-113).
 */
int kvq_dequant(const uint32_t* wq, const void* scales, const void* biases,
                uint64_t rows, uint32_t head_dim, uint32_t bits, uint32_t group_size,
                uint32_t dtype, float* out, void* stream);

/*
 * The canonical MLX-affine quantizer and packer on the device, bit-exact to
 * canonical_quantize + pack_codes
 * (kernelverify/schemas/quant_contract.py:60-104,
 * kernelverify/pack/wide_qmv.py:185-201, as composed by quantize_cache,
 * kernelverify/pack/kv_attention.py:270-283): w [rows, head_dim] dtype in,
 * wq/scales/biases out (scales and biases in dtype).
 */
int kvq_quantize(const void* w, uint64_t rows, uint32_t head_dim, uint32_t bits,
                 uint32_t group_size, uint32_t dtype, uint32_t* wq, void* scales,
                 void* biases, void* stream);

/*
 * Append n_new positions of every (sequence, cache head) to a packed cache
 * with the same quantizer: w [b_rows, n_kv_heads, n_new, head_dim] dtype;
 * row (b, hk, j) is quantized into cache row
 *   b * cache_batch_stride + hk * t_stride + pos_b + j
 * of wq/scales/biases (the cache's base pointers), pos_b = positions[b] read
 * on the device when `positions` is non-NULL (an int32 [b_rows] device
 * array, so a captured decode step appends where the device says), else
 * `position` for every row. Rows at or past t_stride are not written (a
 * device position is not visible to the host check, which covers `position`).
 * b_rows > 1 needs cache_batch_stride >= n_kv_heads * t_stride.
 *
 * The serving cache's update step: the reference's mlx-lm QuantizedKVCache
 * quantizes each step's keys/values into its padded buffers before attention
 * (reached through the runtime patch of bench/spike_mlx_e2e.py:103-123, whose
 * fused arm then reads the padded buffers with the logical length); here the
 * quantizer is the canonical one above, so appended rows are bit-identical to
 * kvq_quantize of the same values.
 */
int kvq_cache_append(const void* w, uint32_t b_rows, uint32_t n_kv_heads, uint32_t n_new,
                     uint32_t head_dim, uint32_t bits, uint32_t group_size, uint32_t dtype,
                     const int32_t* positions, uint32_t position, uint32_t t_stride,
                     uint64_t cache_batch_stride, uint32_t* wq, void* scales, void* biases,
                     void* stream);

/*
 * The full step like kvq_decode, for callers that cannot allocate device
 * memory: a host that binds this library through a plain C FFI and owns no
 * CUDA allocator (a cgo / JNI / ctypes worker), or a serving process that
 * reserves all device memory up front and forbids allocation on its decode
 * path. No counterpart in the reference.
 *
 * Its scratch is a buffer inside the library itself, KVQ_NOALLOC_SCRATCH_BYTES
 * bytes on every GPU that loads the library, held until the process exits.
 * Calls whose split partials need more (kvq_workspace_bytes(a) above the
 * limit) fail with KVQ_ERR_INVALID; use kvq_decode with a workspace instead.
 * Each call looks up the buffer's device address for the current device (so a
 * call after a device reset finds it where the reloaded library put it); the
 * first call on a device also loads the library's device code there, so make
 * that first call before any stream capture. Every call on a
 * device shares the one buffer: calls that overlap on the GPU (two streams,
 * two host threads) race on it and must be serialized by the caller. Nothing
 * in the buffer needs to start at zero: each call writes every partial it
 * reads.
 */
#define KVQ_NOALLOC_SCRATCH_BYTES (16u << 20)
int kvq_decode_noalloc(const kvq_args* a, void* out, void* stream);

/* 1 when this library carries a kernel for the combination, else 0. */
int kvq_supports(uint32_t head_dim, uint32_t bits, uint32_t group_size, uint32_t dtype);

/* The calling thread's last error message ("" when none). */
const char* kvq_last_error(void);

/* KVQ_ABI_VERSION of the loaded library. */
int kvq_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KVQ_B200_H */
