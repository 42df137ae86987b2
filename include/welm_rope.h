/*
 * welm_rope.h — C ABI of the B200 (sm_100a) WeLMv4 in-place partial RoPE.
 *
 * The op rotates the LAST 64 lanes (192..255) of every 256-lane BF16 head of
 * Q [rows, 6, 256] and K [N, 1, 256] in place, with an FP32 cos/sin cache
 * [max_position, 64] (cos in columns 0..31, sin in 32..63) gathered by int64
 * position:
 *     x1 = head[192..223], x2 = head[224..255], c = cache[p, 0..31], s = cache[p, 32..63]
 *     head[192..223] = bf16(x1*c - x2*s)      head[224..255] = bf16(x1*s + x2*c)
 * with each product, the difference and the sum rounded separately in FP32
 * (no fused multiply-add) and one round-to-nearest-even to BF16.  Lanes
 * 0..191 are never written.
 *
 * Each entry point replaces one launch site of the reference benchmark
 * (bench_welmv4_inplace_rope_npu.py); the argument list
 * keeps the reference kernel's runtime arguments in the same order, as plain
 * pointers and 64-bit integers, and adds only `max_position`, an optional
 * device status word and the stream.
 *
 * Conventions for every entry point:
 *   - pointers are device pointers (except the *_host functions and
 *     welm_rope_ordinary_mapped);
 *   - token strides are in ELEMENTS (torch `tensor.stride(0)`); the six Q
 *     heads of a token are contiguous (head stride 256 elements);
 *   - `stream` is a cudaStream_t / CUstream handle (NULL = legacy default
 *     stream) of the current device;
 *   - the call only enqueues work: it never synchronises, never allocates,
 *     never throws and never aborts; it returns a welm_rope_status code;
 *   - `device_status` (may be NULL) is a caller-owned int32 in device memory;
 *     when non-NULL the kernel ORs WELM_ROPE_DEV_* bits into it for tokens or
 *     rows it skipped because an index was out of range.  Out-of-range tokens
 *     are always skipped (left unmodified), never read out of bounds.
 *   - 16-byte aligned bases and token strides that are multiples of 8
 *     elements take the vectorised path; anything else takes a scalar path
 *     with identical results.
 */
#ifndef WELM_ROPE_H_
#define WELM_ROPE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host-side return codes. */
typedef enum welm_rope_status {
  WELM_ROPE_OK = 0,
  WELM_ROPE_ERR_NULL_POINTER = 1, /* a required pointer is NULL                   */
  WELM_ROPE_ERR_BAD_MODE = 2,     /* has_segments not in {0,1}, or mode misuse    */
  WELM_ROPE_ERR_BAD_SIZE = 3,     /* negative or too large N / BS / tiles / P     */
  WELM_ROPE_ERR_BAD_STRIDE = 4,   /* token stride makes rows overlap              */
  WELM_ROPE_ERR_CAPACITY = 5,     /* output buffer too small (tile builder)       */
  WELM_ROPE_ERR_CUDA = 6,         /* the CUDA runtime refused the launch          */
  WELM_ROPE_ERR_TOO_MANY_TOKENS = 7, /* more tokens than the static staging area holds */
  WELM_ROPE_ERR_NOT_MAPPED = 8       /* a host buffer is not page-locked and mapped for the device */
} welm_rope_status;

/* Device-side status bits (ORed into *device_status when it is non-NULL). */
#define WELM_ROPE_DEV_BAD_POSITION 1   /* positions[t] outside [0, max_position)        */
#define WELM_ROPE_DEV_BAD_LAST_INDEX 2 /* last_index[b] outside [0, N)                  */
#define WELM_ROPE_DEV_BAD_TILE 4       /* tile start/end outside [0, N], or > 64 tokens */
#define WELM_ROPE_DEV_BAD_LENGTH 8     /* negative request length (tile builder)        */
#define WELM_ROPE_DEV_BAD_SLOT 16      /* slot_mapping[t] >= num_slots (KV-cache write) */
#define WELM_ROPE_DEV_WAIT_TIMEOUT 32  /* a bounded barrier wait gave up (TMA ceiling)   */

/* Fixed model contract (bench_welmv4_inplace_rope_npu.py:48-58): head_dim 256, rope_dim 64, 6 Q heads,
 * 1 K head, 64-token work tiles. */
#define WELM_ROPE_HEAD_DIM 256
#define WELM_ROPE_ROPE_DIM 64
#define WELM_ROPE_NUM_Q_HEADS 6
#define WELM_ROPE_TILE_TOKENS 64

/*
 * Ordinary prefill / decode: rotate K row t (1 head) and Q row t (6 heads)
 * at positions[t] for every token t covered by the work tiles.
 *
 * Replaces `_candidate_welmv4_inplace_rope_prefill_kernel[(grid,)](q, k,
 * positions, cache, segment_tile_starts_or_placeholder, num_work_tiles, N,
 * q_token_stride, k_token_stride, has_segments)` (bench_welmv4_inplace_rope_npu.py:670-690, bound at
 * bench_welmv4_inplace_rope_npu.py:1267-1322 and 1324-1388) and the per-token decode kernels
 * (bench_welmv4_inplace_rope_npu.py:326-405, 443-526) called with last_index = None.
 *
 *   has_segments == 0: tile i covers tokens [64 i, min(64 i + 64, N)) for
 *       i < num_work_tiles (the reference passes ceil(N/64); with 0 work
 *       tiles nothing is rotated and the call returns WELM_ROPE_OK without
 *       touching any pointer); the segment_tile_starts pointer is not
 *       dereferenced and may be NULL.
 *   has_segments == 1: tile i covers [starts[i], starts[i] + min(64,
 *       starts[i+1] - starts[i])) for i < num_work_tiles; N bounds the tokens.
 * Positions are gathered per token, so no contiguity inside a tile is needed.
 */
int welm_rope_ordinary(void* q, void* k, const int64_t* positions,
                       const float* cos_sin_cache,
                       const int32_t* segment_tile_starts,
                       int64_t num_work_tiles, int64_t n_tokens,
                       int64_t q_token_stride, int64_t k_token_stride,
                       int64_t has_segments, int64_t max_position,
                       int32_t* device_status, void* stream);

/*
 * KV-mirror prefill: Q holds BS rows (one per request); row b is rotated at
 * positions[last_index[b]].  K holds N rows, each rotated at positions[t]
 * for the tokens covered by the work tiles (same tile rules as above).
 *
 * Replaces `_candidate_welmv4_inplace_rope_mirror_prefill_kernel[(grid,)](q,
 * k, positions, cache, last_index, segment_tile_starts_or_placeholder,
 * num_work_tiles, N, BS, q_token_stride, k_token_stride, has_segments)`
 * (bench_welmv4_inplace_rope_npu.py:808-831, bound at bench_welmv4_inplace_rope_npu.py:1176-1205 and 1207-1265) and the
 * frozen per-token kernel called with a last_index tensor (bench_welmv4_inplace_rope_npu.py:371-395).
 */
int welm_rope_mirror(void* q, void* k, const int64_t* positions,
                     const float* cos_sin_cache, const int64_t* last_index,
                     const int32_t* segment_tile_starts, int64_t num_work_tiles,
                     int64_t n_tokens, int64_t batch_size,
                     int64_t q_token_stride, int64_t k_token_stride,
                     int64_t has_segments, int64_t max_position,
                     int32_t* device_status, void* stream);

/*
 * Segmented KV-mirror prefill driven directly by request lengths on the
 * device: no tile table, no last_index tensor and no host round trip between
 * building them and launching.  Request r holds seq_lens[r] consecutive K
 * tokens; K token t < sum(seq_lens) is rotated at positions[t] (the
 * reference's per-request 64-token tiles cover every token of every request);
 * Q row r is rotated at positions[end_r - 1] with end_r = seq_lens[0] + ... +
 * seq_lens[r] (the reference's segmented last_index).  The result equals
 * welm_rope_build_tiles followed by welm_rope_mirror with has_segments = 1.
 * Negative lengths count as 0 and raise WELM_ROPE_DEV_BAD_LENGTH; tokens at or
 * past min(N, sum) are not touched; a Q row whose end_r is 0 or past N raises
 * WELM_ROPE_DEV_BAD_LAST_INDEX and is skipped.  batch_size <=
 * WELM_ROPE_LENS_MAX_BATCH (the lengths are staged in shared memory).
 *
 * On-device tile building fused with the mirror launch; the reference builds
 * tiles on the host (bench_welmv4_inplace_rope_npu.py:1439-1461) before each
 * launch.
 */
#define WELM_ROPE_LENS_MAX_BATCH 2048
int welm_rope_mirror_from_lens(void* q, void* k, const int64_t* positions,
                               const float* cos_sin_cache, const int64_t* seq_lens,
                               int64_t n_tokens, int64_t batch_size,
                               int64_t q_token_stride, int64_t k_token_stride,
                               int64_t max_position, int32_t* device_status,
                               void* stream);

/*
 * KV-mirror prefill fused with the paged KV-cache write and the Q last-row
 * extraction, in one pass:
 *   q_out[b]            = rope(q[last_index[b]]) at positions[last_index[b]]
 *                         (all 6 heads, lanes 0..191 copied, 192..255 rotated)
 *   key_cache[slot[t]]  = rope(k[t]) at positions[t]   (all 256 lanes)
 *   value_cache[slot[t]] = v[t]                        (all 256 lanes)
 * for t < N with slot[t] = slot_mapping[t]; slot < 0 marks a padding token
 * and writes nothing, slot >= num_slots raises WELM_ROPE_DEV_BAD_SLOT and
 * writes nothing; a token whose position is out of range is flagged and not
 * written.  q, k and v are read only (q is the full [N, 6, 256] projection
 * output; q_out holds BS rows); cache rows are `cache_slot_stride` elements
 * apart (256 for [blocks, block_size, 1, 256] and [blocks, 1, block_size, 256]
 * caches with one KV head).  value_cache / v may be NULL to skip the V copy.
 * Every pointer must be 16-byte aligned and every stride a multiple of 8
 * elements.
 *
 * Row 2 of the path's "next" list: the mirror's K output is what gets written
 * to the KV cache (bench_welmv4_inplace_rope_npu.py:17-18 — only the last
 * token per request keeps a Q row); the reference rotates in place and leaves
 * the extraction and the cache write to separate passes.
 */
int welm_rope_mirror_kv_write(const void* q, void* q_out, const void* k, const void* v,
                              const int64_t* positions, const float* cos_sin_cache,
                              const int64_t* last_index, const int64_t* slot_mapping,
                              void* key_cache, void* value_cache, int64_t n_tokens,
                              int64_t batch_size, int64_t q_token_stride,
                              int64_t q_out_token_stride, int64_t k_token_stride,
                              int64_t v_token_stride, int64_t cache_slot_stride,
                              int64_t num_slots, int64_t max_position,
                              int32_t* device_status, void* stream);

/*
 * Segmented 64-token tile-boundary builder on the device.  For request r of
 * length len_r starting at token off_r it emits off_r, off_r+64, ... (< off_r
 * + len_r), then the final total N: int32 starts[T+1], T = sum ceil(len_r/64).
 * Tiles never cross a request boundary.  Optionally also writes
 * last_index[r] = off_r + len_r - 1 (int64).  *num_tiles_out (device int32)
 * receives T; `capacity` is the number of int32 slots in `tile_starts`
 * (T + 1 <= ceil(N/64) + BS + 1 always suffices); entries past capacity are
 * not written and WELM_ROPE_DEV_BAD_TILE is raised.  Negative lengths count
 * as 0 and raise WELM_ROPE_DEV_BAD_LENGTH.
 *
 * Replaces the host loop inside make_inputs (bench_welmv4_inplace_rope_npu.py:1439-1461) and
 * make_last_index (bench_welmv4_inplace_rope_npu.py:1402-1424, segmented branch).
 */
int welm_rope_build_tiles(const int64_t* seq_lens, int64_t batch_size,
                          int32_t* tile_starts, int64_t capacity,
                          int32_t* num_tiles_out, int64_t* last_index_out,
                          int32_t* device_status, void* stream);

/*
 * Host twins of the builder (plain host memory, no CUDA call).  count returns
 * T in *num_tiles_out; build fills starts[0..T] (needs capacity >= T + 1) and,
 * when last_index_out is non-NULL, last_index[0..BS).  Negative lengths are
 * rejected with WELM_ROPE_ERR_BAD_SIZE.  Same reference lines as above.
 */
int welm_rope_count_tiles_host(const int64_t* seq_lens, int64_t batch_size,
                               int64_t* num_tiles_out);
int welm_rope_build_tiles_host(const int64_t* seq_lens, int64_t batch_size,
                               int32_t* tile_starts, int64_t capacity,
                               int64_t* num_tiles_out, int64_t* last_index_out);

/*
 * Copies only the rotated lanes (192..255) of `heads` heads of `rows` rows
 * between host and device memory (direction 0: host -> device, 1: device ->
 * host): the bytes the op reads and writes, a quarter of every head.  Token
 * strides are in elements; heads are 256 lanes apart.  Lanes 0..191 of the
 * destination are not written.  Pinned host memory makes the copy
 * asynchronous on `stream`.  It is a cudaMemcpy2DAsync per call (one when
 * both token strides equal heads * 256, else one per head).
 *
 * No counterpart in the reference (its Q and K always live on the device); it
 * serves callers that keep Q/K in host memory and move them per call.
 */
int welm_rope_copy_rope_lanes(void* dst, const void* src, int64_t rows, int64_t heads,
                              int64_t dst_token_stride, int64_t src_token_stride,
                              int64_t direction, void* stream);

/*
 * Ordinary prefill / decode RoPE on Q/K held in host memory, without any
 * allocation: for callers that cannot allocate device memory — a plugin whose
 * host process owns every byte of device memory through its own allocator, or
 * code on a latency-critical path where cudaMalloc/cudaFree (which may
 * synchronise the device) are not allowed.  The rotated lanes of Q
 * [n_tokens, 6, 256] and K [n_tokens, 1, 256] and the positions are staged
 * through a fixed area inside this library (a static device array of
 * WELM_ROPE_STATIC_MAX_TOKENS tokens, about 1.85 MB, which every GPU that
 * loads the library holds until the process exits), rotated there and copied
 * back, all on `stream`; lanes 0..191 of Q and K are never written.  q, k and
 * positions may be host (pinned for asynchronous copies) or device memory;
 * cos_sin_cache is device memory.  More than WELM_ROPE_STATIC_MAX_TOKENS
 * tokens is rejected with WELM_ROPE_ERR_TOO_MANY_TOKENS (split larger batches
 * into several calls).
 *
 * The first call on each device looks up the staging area's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  The address is kept for the life of the
 * process, so do not use this entry after a cudaDeviceReset of that device
 * (the reset unloads the library's device code and the kept address may no
 * longer be mapped).  Every call shares the one staging area: calls
 * whose work overlaps on the GPU (different streams, or different host
 * threads without ordering) race on it and must be serialised by the caller.
 * The area is fully rewritten by each call before it is read, so the previous
 * call's leftovers never reach a result.
 *
 * No counterpart in the reference: it keeps Q and K on the device and
 * allocates freely.
 */
#define WELM_ROPE_STATIC_MAX_TOKENS 2048
int welm_rope_ordinary_host_static(void* q, void* k, const int64_t* positions,
                                   const float* cos_sin_cache, int64_t n_tokens,
                                   int64_t q_token_stride, int64_t k_token_stride,
                                   int64_t max_position, int32_t* device_status,
                                   void* stream);

/*
 * Ordinary prefill / decode RoPE on Q [n_tokens, 6, 256] and K [n_tokens, 1,
 * 256] that stay in page-locked host memory, without staging: one kernel reads
 * each 128-byte rope slice (lanes 192..255 of a head) straight from host
 * memory over PCIe, rotates it and writes it back, so the two bus directions
 * overlap and lanes 0..191 never cross the bus.  q and k must be page-locked
 * AND mapped into the device's address space (cudaHostAlloc / cudaMallocHost,
 * torch's pin_memory(), or cudaHostRegister with cudaHostRegisterMapped), each
 * within one allocation; positions may be such host memory or device memory
 * of the current device; cos_sin_cache is device memory.  Other memory is
 * rejected with WELM_ROPE_ERR_NOT_MAPPED before anything is launched.  Bases
 * must be 16-byte aligned and token strides multiples of 8 elements
 * (WELM_ROPE_ERR_BAD_STRIDE otherwise).
 *
 * Stream-ordered like the device entries: the host buffers hold the result
 * once `stream` has been synchronised, and the host must not touch them in
 * between.  Allocates nothing; out-of-range positions leave their token
 * unchanged and raise WELM_ROPE_DEV_BAD_POSITION.
 *
 * No counterpart in the reference (its Q and K always live on the device); it
 * serves callers that keep Q/K in host memory.
 */
int welm_rope_ordinary_mapped(void* q, void* k, const int64_t* positions,
                              const float* cos_sin_cache, int64_t n_tokens,
                              int64_t q_token_stride, int64_t k_token_stride,
                              int64_t max_position, int32_t* device_status,
                              void* stream);

/*
 * Measurement kernels: the practical ceilings the RoPE kernels are timed
 * against on the same bytes.  They rotate nothing and have no counterpart in
 * the reference, whose benchmark compares against the NPU's nominal peak only.
 *
 * welm_rope_ceiling_copy copies `bytes` (a multiple of 16; both pointers
 * 16-byte aligned, device memory) from src to dst in 16-byte vectors (one per
 * thread up to a full-occupancy wave, four per thread above), launched like
 * the op.  welm_rope_ceiling_slices reads the rope
 * slices (lanes 192..255) of K row t (1 head) and Q row t (6 heads) for
 * t < n_tokens and writes them back unchanged: the ordinary kernel's accesses
 * without positions, cos/sin and arithmetic (16-byte aligned bases, strides a
 * multiple of 8 elements, else WELM_ROPE_ERR_BAD_STRIDE).
 * welm_rope_ceiling_gather performs only the ordinary kernel's position and
 * cos/sin gather for tokens t < n_tokens (the same items, launch shape and
 * pre-wait hints and prefetches; 16-byte aligned cache, else
 * WELM_ROPE_ERR_BAD_STRIDE) and writes nothing but, when the values it read
 * fold to a fixed magic word (they do not for any real cache), one int32 to
 * `sink`: its L2 and DRAM counters are those of the gather alone.
 *
 * welm_rope_ceiling_tma_slices moves the same slices as
 * welm_rope_ceiling_slices through shared memory with the Tensor Memory
 * Accelerator: `ctas` persistent CTAs (0: two per SM), each with a ring of
 * `stages` (2, 4 or 6; else WELM_ROPE_ERR_BAD_MODE) 16-token tiles loaded by
 * tiled cp.async.bulk.tensor and stored back unchanged by bulk-tensor stores,
 * the first tiles prefetched into L2 before the dependency wait.  Strides of
 * at least one row (1536 and 256 elements) and multiples of 8 elements,
 * 16-byte aligned bases (else WELM_ROPE_ERR_BAD_STRIDE); n_tokens at most
 * 2^31 - 17 (else WELM_ROPE_ERR_BAD_SIZE); WELM_ROPE_ERR_CUDA when the driver
 * cannot encode the tensor maps.  A barrier wait that gives up ORs
 * WELM_ROPE_DEV_WAIT_TIMEOUT into device_status (when non-NULL) and ends
 * that CTA's work.
 */
int welm_rope_ceiling_copy(void* dst, const void* src, int64_t bytes, void* stream);
int welm_rope_ceiling_slices(void* q, void* k, int64_t n_tokens, int64_t q_token_stride,
                             int64_t k_token_stride, void* stream);
int welm_rope_ceiling_gather(const int64_t* positions, const float* cos_sin_cache, int64_t n_tokens,
                             int64_t max_position, int32_t* sink, void* stream);
int welm_rope_ceiling_tma_slices(void* q, void* k, int64_t n_tokens, int64_t q_token_stride,
                                 int64_t k_token_stride, int32_t ctas, int32_t stages, int32_t* device_status,
                                 void* stream);

/* Human-readable name of a welm_rope_status code (static storage). */
const char* welm_rope_status_string(int status);

/* ABI version of this header: (major << 16) | minor.  A minor bump only adds
 * entry points or status codes; a major bump changes an existing signature.
 * 1.1 added welm_rope_ordinary_mapped and WELM_ROPE_ERR_NOT_MAPPED; 1.2 the
 * two measurement kernels welm_rope_ceiling_copy and welm_rope_ceiling_slices;
 * 1.3 the measurement kernel welm_rope_ceiling_gather; 1.4 the measurement
 * kernel welm_rope_ceiling_tma_slices and WELM_ROPE_DEV_WAIT_TIMEOUT. */
#define WELM_ROPE_ABI_VERSION ((1 << 16) | 4)
int welm_rope_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* WELM_ROPE_H_ */
