// rope_ceiling.cu — measurement kernels: the practical ceilings the RoPE
// kernels are timed against on the same bytes.  They rotate nothing, read no
// positions and no cos/sin cache, and are not part of the op.
//
// * welm_rope_ceiling_copy: a streaming device copy launched like the op (PDL
//   attribute, pdl_enter before the first access, and the source lines of
//   each thread's first round prefetched into L2 before the wait, as the op
//   does): one 16-byte vector per thread up to one full-occupancy wave of
//   threads, four per thread (all loaded before any is stored) in one wave
//   above that.  With one vector per thread at every size, 33.7 MB took
//   8.9 us against 6.7-7.1 us for the runtime's device-to-device copy; at
//   8.7 MB it took 2.80 against 3.26.
// * welm_rope_ceiling_slices: the ordinary dense kernels' own access pattern —
//   the same item mapping (seven heads per thread, or one head per thread for
//   launches of at most 3328 tokens), launch shape, pre-wait prefetch of the
//   slice lines, and 16-byte loads and stores of the rope slices of K and the
//   six Q heads, in place — without the position and cos/sin gather and
//   without the arithmetic.  Its time is the floor of that access pattern:
//   what the op would take if the rotation were free.
// * welm_rope_ceiling_tma_slices: the same slices moved through shared memory
//   by the Tensor Memory Accelerator instead of the threads' own loads and
//   stores — persistent CTAs, each with a ring of 16-token tiles loaded by
//   tiled cp.async.bulk.tensor and stored back unchanged by bulk-tensor
//   stores — so the register path can be compared with TMA staging on the
//   op's own buffers.

#include <cudaTypedefs.h>

#include "rope_host.cuh"

namespace {

// kPer vectors per thread per round, all loaded before any is stored; vector
// j of a round sits `threads` apart, so every load and store is coalesced.
template <int kPer>
__global__ void __launch_bounds__(kBlock) ceiling_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                              int64_t vectors) {
  const int64_t threads = int64_t(gridDim.x) * blockDim.x;
  {  // before the wait: one prefetch per 128-byte source line of the first round
    const int64_t base = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int64_t v = base + j * threads;
      if (v < vectors && (v & 7) == 0) prefetch_line(src + v);
    }
  }
  pdl_enter();
  for (int64_t base = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; base < vectors; base += threads * kPer) {
    uint4 v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (base + j * threads < vectors) v[j] = __ldg(src + base + j * threads);
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (base + j * threads < vectors) dst[base + j * threads] = v[j];
  }
}

// Writes the loaded slices back XORed with `salt`.  The caller passes 0, so
// the data is unchanged; the compiler cannot know that, so it keeps every
// store, which it could drop for a plain store of a just-loaded value.
template <int NH>
__device__ __forceinline__ void store_back(Slices<true, NH>& x, uint32_t salt) {
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    x.x1[h].x ^= salt;
    x.x2[h].x ^= salt;
    Io<true>::store8(x.base + h * kHeadDim, x.x1[h]);
    Io<true>::store8(x.base + h * kHeadDim + kHalf, x.x2[h]);
  }
}

__global__ void __launch_bounds__(kBlock, 5) ceiling_slices_kernel(uint16_t* q, uint16_t* k, int64_t q_stride,
                                                                   int64_t k_stride, int32_t items, uint32_t salt) {
  const int stride = gridDim.x * blockDim.x;
  const int first = blockIdx.x * blockDim.x + threadIdx.x;
  if (first < items) prefetch_token<true>(q, k, q_stride, k_stride, first >> kPartShift, first & (kParts - 1));
  pdl_enter();
  for (int item = first; item < items; item += stride) {
    const int part = item & (kParts - 1);
    const int64_t tok = item >> kPartShift;
    const int next = item + stride;
    if (next < items) prefetch_token<true>(q, k, q_stride, k_stride, next >> kPartShift, next & (kParts - 1));
    Slices<true, 1> kx;
    Slices<true, kQHeads> qx;
    kx.load(k + tok * k_stride, part);
    qx.load(q + tok * q_stride, part);
    store_back(kx, salt);
    store_back(qx, salt);
  }
}

// The same for launches that the ordinary path runs one head per thread
// (item = ((token * 7 + head) * 4 + part), head 0 the K head).
__global__ void __launch_bounds__(kBlock) ceiling_slices_head_kernel(uint16_t* q, uint16_t* k, int64_t q_stride,
                                                                     int64_t k_stride, int32_t items,
                                                                     uint32_t salt) {
  const int item = blockIdx.x * blockDim.x + threadIdx.x;  // the grid covers every item once
  const int part = item & (kParts - 1);
  const int slice = item >> kPartShift;
  const int64_t tok = slice / kHeadsPerToken;
  const int head = slice - int(tok) * kHeadsPerToken;
  uint16_t* row = head == 0 ? k + tok * k_stride : q + tok * q_stride + (head - 1) * kHeadDim;
  if (item < items && part == 0 && items >= kHeadPrefetchMinItems) prefetch_row_slices<1>(row, 0);
  pdl_enter();
  if (item >= items) return;
  Slices<true, 1> x;
  x.load(row, part);
  store_back(x, salt);
}

// The ordinary kernels' gather alone: item (token, part) reads the token's
// position (a hint before the wait, prefetching the cos/sin lines it names,
// then the real value) and its part of the cos/sin row, and folds the values
// it read into one word.
__global__ void __launch_bounds__(kBlock) ceiling_gather_kernel(const int64_t* positions, const float* cache,
                                                                int32_t items, int64_t max_position,
                                                                int32_t* sink) {
  const int stride = gridDim.x * blockDim.x;
  const int first = blockIdx.x * blockDim.x + threadIdx.x;
  if (first < items)
    prefetch_cos_sin_row(cache, max_position, hint_load(positions + (first >> kPartShift)), first & (kParts - 1));
  pdl_enter();
  uint32_t fold = 0;
  for (int item = first; item < items; item += stride) {
    const int part = item & (kParts - 1);
    const int64_t pos = __ldg(positions + (item >> kPartShift));
    if (pos < 0 || pos >= max_position) continue;
    CosSin cs;
    Io<true>::load_cos_sin(cache + pos * kRopeDim, part, cs);
#pragma unroll
    for (int i = 0; i < kLanes; ++i) fold ^= __float_as_uint(cs.c[i]) ^ (__float_as_uint(cs.s[i]) << 1);
  }
  if (fold == 0x9e3779b9u && sink != nullptr) *sink = int32_t(fold);
}

// ---------------------------------------------------------------------------
// TMA-staged slice mover.  Tile i holds tokens [16 i, 16 i + 16): the rope
// lanes (x = 192..255) of Q's six heads as one 3-D box {64 lanes, 6 heads, 16
// tokens} (12 KB) and of K as one 2-D box {64 lanes, 16 tokens} (2 KB).  CTA
// b takes tiles b, b + G, b + 2G, ... through a ring of S stages: one elected
// thread arms the stage's mbarrier with the 14 KB it expects, issues both
// loads, waits for them, issues both stores from the same shared memory and,
// once the stores have read it, refills the stage with the tile S steps
// ahead.  Loads past the last token fill zeros and stores past it are
// clipped, so ragged N needs no special case.  Before the dependency wait the
// CTA's first S tiles are prefetched into L2 (a prefetch returns no data, so
// it cannot see stale values).  Every barrier wait gives up after a bounded
// number of polls, raises WELM_ROPE_DEV_WAIT_TIMEOUT and ends the CTA's work.
// ---------------------------------------------------------------------------
constexpr int kTmaTileTokens = 16;
constexpr int kTmaQBytes = kRopeDim * 2 * kQHeads * kTmaTileTokens;
constexpr int kTmaKBytes = kRopeDim * 2 * kTmaTileTokens;
constexpr int kTmaStageBytes = kTmaQBytes + kTmaKBytes;
constexpr int kTmaWaitPolls = 1 << 22;

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arm(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void tma_tile_load(uint8_t* stage, const CUtensorMap* qmap, const CUtensorMap* kmap,
                                              int tile, uint64_t* bar) {
  const int z = tile * kTmaTileTokens;
  mbar_arm(bar, kTmaStageBytes);
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(stage)), "l"(qmap), "r"(kRopeLane0), "r"(0), "r"(z), "r"(smem_u32(bar))
      : "memory");
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(stage + kTmaQBytes)), "l"(kmap), "r"(kRopeLane0), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_tile_store(const uint8_t* stage, const CUtensorMap* qmap,
                                               const CUtensorMap* kmap, int tile) {
  const int z = tile * kTmaTileTokens;
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];"
               ::"l"(qmap), "r"(kRopeLane0), "r"(0), "r"(z), "r"(smem_u32(stage))
               : "memory");
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(kmap), "r"(kRopeLane0), "r"(z), "r"(smem_u32(stage + kTmaQBytes))
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int S>
__global__ void __launch_bounds__(kBlock) ceiling_tma_slices_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                    const __grid_constant__ CUtensorMap kmap,
                                                                    int tiles, int32_t* status) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[S];
  const bool leader = threadIdx.x == 0;
  if (leader) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < S; ++i) {  // before the wait: L2 prefetch of the first tiles
      const int t = blockIdx.x + i * gridDim.x;
      if (t >= tiles) break;
      asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];"
                   ::"l"(&qmap), "r"(kRopeLane0), "r"(0), "r"(t * kTmaTileTokens) : "memory");
      asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
                   ::"l"(&kmap), "r"(kRopeLane0), "r"(t * kTmaTileTokens) : "memory");
    }
  }
  __syncthreads();
  pdl_enter();
  if (!leader) return;
  for (int i = 0; i < S; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= tiles) break;
    tma_tile_load(ring + i * kTmaStageBytes, &qmap, &kmap, t, &full[i]);
  }
  for (int i = 0;; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= tiles) break;
    const int s = i % S;
    uint8_t* stage = ring + s * kTmaStageBytes;
    bool landed = false;
    for (int poll = 0; poll < kTmaWaitPolls && !landed; ++poll) landed = mbar_poll(&full[s], (i / S) & 1);
    if (!landed) {
      raise_status(status, WELM_ROPE_DEV_WAIT_TIMEOUT);
      break;
    }
    tma_tile_store(stage, &qmap, &kmap, t);
    const int next = t + S * gridDim.x;
    if (next < tiles) {
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the stores have read the stage
      tma_tile_load(stage, &qmap, &kmap, next, &full[s]);
    }
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The driver's tensor-map encoder, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult found;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor maps of Q ({256 lanes, 6 heads, N tokens}) and K ({256 lanes, N
// tokens}) with the tile boxes above; false when the driver refuses them.
bool encode_slice_maps(void* q, void* k, int64_t n_tokens, int64_t q_stride, int64_t k_stride, CUtensorMap& qmap,
                       CUtensorMap& kmap) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint32_t unit[3] = {1, 1, 1};
  const cuuint64_t qdim[3] = {cuuint64_t(kHeadDim), cuuint64_t(kQHeads), cuuint64_t(n_tokens)};
  const cuuint64_t qstride[2] = {cuuint64_t(kHeadDim) * 2, cuuint64_t(q_stride) * 2};
  const cuuint32_t qbox[3] = {cuuint32_t(kRopeDim), cuuint32_t(kQHeads), cuuint32_t(kTmaTileTokens)};
  const cuuint64_t kdim[2] = {cuuint64_t(kHeadDim), cuuint64_t(n_tokens)};
  const cuuint64_t kstride[1] = {cuuint64_t(k_stride) * 2};
  const cuuint32_t kbox[2] = {cuuint32_t(kRopeDim), cuuint32_t(kTmaTileTokens)};
  return encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, qdim, qstride, qbox, unit,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
         encode(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, kdim, kstride, kbox, unit,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int S>
int launch_tma_slices(const CUtensorMap& qmap, const CUtensorMap& kmap, int tiles, int ctas, int32_t* status,
                      cudaStream_t stream) {
  const size_t smem = size_t(S) * kTmaStageBytes;
  if (cudaFuncSetAttribute(ceiling_tma_slices_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess) {
    cudaGetLastError();
    return WELM_ROPE_ERR_CUDA;
  }
  return launch(ceiling_tma_slices_kernel<S>, unsigned(ctas), kBlock, smem, stream, qmap, kmap, tiles, status);
}

}  // namespace

extern "C" {

int welm_rope_ceiling_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || bytes % 16 != 0) return WELM_ROPE_ERR_BAD_SIZE;
  const int64_t vectors = bytes / 16;
  if (vectors > kMaxItems) return WELM_ROPE_ERR_BAD_SIZE;
  if (vectors == 0) return WELM_ROPE_OK;
  if (!dst || !src) return WELM_ROPE_ERR_NULL_POINTER;
  if (!aligned16(dst) || !aligned16(src)) return WELM_ROPE_ERR_BAD_STRIDE;
  // Up to one full-occupancy wave of threads (16 CTAs of 128 per SM): one
  // vector per thread.  Above that, four per thread in at most one wave.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = current_sm_count();
  const int64_t wave = int64_t(sms > 0 ? sms : 1) * 16 * kBlock;
  const auto* s4 = static_cast<const uint4*>(src);
  auto* d4 = static_cast<uint4*>(dst);
  if (vectors <= wave)
    return launch(ceiling_copy_kernel<1>, unsigned((vectors + kBlock - 1) / kBlock), kBlock, 0, st, s4, d4, vectors);
  const int64_t need = (vectors + 4 * kBlock - 1) / (4 * kBlock);
  const int64_t grid = need < wave / kBlock ? need : wave / kBlock;
  return launch(ceiling_copy_kernel<4>, unsigned(grid), kBlock, 0, st, s4, d4, vectors);
}

int welm_rope_ceiling_slices(void* q, void* k, int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                             void* stream) {
  if (n_tokens < 0 || n_tokens > kMaxItems / kParts) return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!q || !k) return WELM_ROPE_ERR_NULL_POINTER;
  if (n_tokens > 1 && (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  if (!aligned16(q) || !aligned16(k) || q_token_stride % 8 != 0 || k_token_stride % 8 != 0)
    return WELM_ROPE_ERR_BAD_STRIDE;  // the 16-byte vector path only
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LaunchShape shape;
  if (head_split_shape(n_tokens, shape))
    return launch(ceiling_slices_head_kernel, shape.grid, shape.block, 0, st, static_cast<uint16_t*>(q),
                  static_cast<uint16_t*>(k), q_token_stride, k_token_stride,
                  int32_t(n_tokens * kHeadsPerToken * kParts), uint32_t(0));
  const int64_t items = n_tokens * kParts;
  shape = stream_shape(items);
  return launch(ceiling_slices_kernel, shape.grid, shape.block, 0, st,
                static_cast<uint16_t*>(q), static_cast<uint16_t*>(k), q_token_stride, k_token_stride,
                int32_t(items), uint32_t(0));
}

int welm_rope_ceiling_gather(const int64_t* positions, const float* cos_sin_cache, int64_t n_tokens,
                             int64_t max_position, int32_t* sink, void* stream) {
  if (n_tokens < 0 || max_position < 0 || n_tokens > kMaxItems / kParts) return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!positions || !cos_sin_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (!aligned16(cos_sin_cache)) return WELM_ROPE_ERR_BAD_STRIDE;
  const int64_t items = n_tokens * kParts;
  const LaunchShape shape = stream_shape(items);
  return launch(ceiling_gather_kernel, shape.grid, shape.block, 0, static_cast<cudaStream_t>(stream), positions,
                cos_sin_cache, int32_t(items), max_position, sink);
}

int welm_rope_ceiling_tma_slices(void* q, void* k, int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                                 int32_t ctas, int32_t stages, int32_t* device_status, void* stream) {
  if (n_tokens < 0 || n_tokens > int64_t(INT32_MAX) - kTmaTileTokens || ctas < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (stages != 2 && stages != 4 && stages != 6) return WELM_ROPE_ERR_BAD_MODE;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!q || !k) return WELM_ROPE_ERR_NULL_POINTER;
  if (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim || !aligned16(q) || !aligned16(k) ||
      q_token_stride % 8 != 0 || k_token_stride % 8 != 0)
    return WELM_ROPE_ERR_BAD_STRIDE;  // tensor maps need 16-byte bases and strides
  CUtensorMap qmap, kmap;
  if (!encode_slice_maps(q, k, n_tokens, q_token_stride, k_token_stride, qmap, kmap)) return WELM_ROPE_ERR_CUDA;
  const int tiles = int((n_tokens + kTmaTileTokens - 1) / kTmaTileTokens);
  const int sms = current_sm_count();
  int grid = ctas > 0 ? ctas : 2 * (sms > 0 ? sms : 1);
  if (grid > tiles) grid = tiles;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (stages) {
    case 2: return launch_tma_slices<2>(qmap, kmap, tiles, grid, device_status, st);
    case 4: return launch_tma_slices<4>(qmap, kmap, tiles, grid, device_status, st);
    default: return launch_tma_slices<6>(qmap, kmap, tiles, grid, device_status, st);
  }
}

}  // extern "C"
