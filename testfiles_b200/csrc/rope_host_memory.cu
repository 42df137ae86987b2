// rope_host_memory.cu — Q/K held in host memory: the rope-lane copy helper,
// the allocation-free staged entry and the mapped (zero-staging) entry.

#include "rope_host.cuh"

namespace {

// ---------------------------------------------------------------------------
// Allocation-free host entry (welm_rope_ordinary_host_static): a static staging
// area in device memory holds the rope lanes of up to kStaticTokens tokens in
// a compact layout — Q [tokens][6][64], K [tokens][64] (bf16) — plus their
// positions.  Host code must not use the array's name as an address (it is a
// host-side stand-in); it looks the device address up once per device.
// ---------------------------------------------------------------------------
constexpr int kStaticTokens = WELM_ROPE_STATIC_MAX_TOKENS;
constexpr size_t kStageQBytes = size_t(kStaticTokens) * kQHeads * kRopeDim * sizeof(uint16_t);
constexpr size_t kStageKBytes = size_t(kStaticTokens) * kRopeDim * sizeof(uint16_t);
constexpr size_t kStagePosBytes = size_t(kStaticTokens) * sizeof(int64_t);
constexpr size_t kStageBytes = kStageQBytes + kStageKBytes + kStagePosBytes;

static __device__ __align__(256) unsigned char g_static_stage[kStageBytes];

// Rotates staged rows: one item = (token, part) as in the other kernels, over
// the compact staging layout (head stride 64, rope lanes from 0).
__global__ void __launch_bounds__(kBlock)
rope_staged_kernel(uint16_t* q, uint16_t* k, const int64_t* positions, const float* cache,
                   int32_t items, int64_t max_position, int32_t* status) {
  pdl_enter();
  const int stride = gridDim.x * blockDim.x;
  for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < items; item += stride) {
    const int part = item & (kParts - 1);
    const int tok = item >> kPartShift;
    const int64_t pos = __ldg(positions + tok);
    uint16_t* kb = k + size_t(tok) * kRopeDim + part * kLanes;
    uint16_t* qb = q + size_t(tok) * kQHeads * kRopeDim + part * kLanes;
    uint4 kx1 = Io<true>::load8(kb), kx2 = Io<true>::load8(kb + kHalf);
    uint4 qx1[kQHeads], qx2[kQHeads];
#pragma unroll
    for (int h = 0; h < kQHeads; ++h) {
      qx1[h] = Io<true>::load8(qb + h * kRopeDim);
      qx2[h] = Io<true>::load8(qb + h * kRopeDim + kHalf);
    }
    if (pos < 0 || pos >= max_position) {
      if (part == 0) raise_status(status, WELM_ROPE_DEV_BAD_POSITION);
      continue;  // the staged lanes go back unchanged
    }
    CosSin cs;
    Io<true>::load_cos_sin(cache + pos * kRopeDim, part, cs);
    rotate8(kx1, kx2, cs);
    Io<true>::store8(kb, kx1);
    Io<true>::store8(kb + kHalf, kx2);
#pragma unroll
    for (int h = 0; h < kQHeads; ++h) {
      rotate8(qx1[h], qx2[h], cs);
      Io<true>::store8(qb + h * kRopeDim, qx1[h]);
      Io<true>::store8(qb + h * kRopeDim + kHalf, qx2[h]);
    }
  }
}

// ---------------------------------------------------------------------------
// Mapped-host entry (welm_rope_ordinary_mapped): Q and K stay in page-locked
// host memory mapped into the device's address space, and the kernel moves
// only the rope slices over PCIe, reading and writing in the same pass so the
// two bus directions overlap.  One piece = the 128-byte rope slice (64 lanes)
// of one head of one token; pieces are numbered token-major (6 Q heads, then
// K).  Eight consecutive threads own a piece, 16 bytes each, so every warp
// request covers whole 128-byte slices — the request size at which the
// bus's reads and writes run near their bulk-copy rate.  Thread sub =
// lane & 7 holds x1 lanes 8*sub.. (sub < 4) or the matching x2 lanes
// (sub >= 4); the other half of its pair arrives by shuffle, both threads
// rotate the pair with the same rotate8 and each stores its own half.
// ---------------------------------------------------------------------------
constexpr int kMappedBlock = 256;
constexpr int kMappedPieces = kQHeads + 1;  // pieces per token
constexpr int kPieceThreads = 8;            // 16-byte vectors per piece

struct MappedArgs {
  uint16_t* q;
  uint16_t* k;
  const int64_t* positions;
  const float* cache;
  int64_t q_stride;
  int64_t k_stride;
  int64_t max_position;
  int64_t pieces;   // n_tokens * kMappedPieces
  int64_t threads;  // pieces * kPieceThreads rounded up to whole warps
  int32_t* status;
};

__global__ void __launch_bounds__(kMappedBlock) rope_mapped_kernel(const MappedArgs a) {
  pdl_enter();
  const int sub = threadIdx.x & (kPieceThreads - 1);
  const int part = sub & (kParts - 1);
  const bool upper = sub >= kParts;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  // a.threads is a multiple of 32 and so is the stride: every lane of a warp
  // runs the same iterations, which the shuffles below need.
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < a.threads; t += stride) {
    const int64_t piece = t / kPieceThreads;
    const bool valid = piece < a.pieces;
    int64_t tok = 0, pos = 0;
    int j = 0;
    uint16_t* addr = nullptr;
    uint4 mine = make_uint4(0u, 0u, 0u, 0u);
    if (valid) {
      tok = piece / kMappedPieces;
      j = int(piece - tok * kMappedPieces);
      uint16_t* row = j < kQHeads ? a.q + tok * a.q_stride + j * kHeadDim : a.k + tok * a.k_stride;
      addr = row + kRopeLane0 + (upper ? kHalf : 0) + part * kLanes;
      mine = *reinterpret_cast<const uint4*>(addr);
      pos = a.positions[tok];
    }
    uint4 other;
    other.x = __shfl_xor_sync(0xffffffffu, mine.x, kParts);
    other.y = __shfl_xor_sync(0xffffffffu, mine.y, kParts);
    other.z = __shfl_xor_sync(0xffffffffu, mine.z, kParts);
    other.w = __shfl_xor_sync(0xffffffffu, mine.w, kParts);
    if (!valid) continue;
    if (pos < 0 || pos >= a.max_position) {
      if (sub == 0 && j == kQHeads) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
      continue;  // the token stays as it was
    }
    CosSin cs;
    Io<true>::load_cos_sin(a.cache + pos * kRopeDim, part, cs);
    uint4 x1 = upper ? other : mine;
    uint4 x2 = upper ? mine : other;
    rotate8(x1, x2, cs);
    *reinterpret_cast<uint4*>(addr) = upper ? x2 : x1;
  }
}

// Device address of g_static_stage on the current device, looked up once per
// device (with that device current) and cached; nullptr if the lookup fails.
unsigned char* static_stage_for_current_device() {
  static std::atomic<unsigned char*> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  unsigned char* p = cache[dev].load(std::memory_order_acquire);
  if (p != nullptr) return p;
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_static_stage) != cudaSuccess || addr == nullptr) {
    cudaGetLastError();
    return nullptr;
  }
  p = static_cast<unsigned char*>(addr);
  cache[dev].store(p, std::memory_order_release);
  return p;
}

// Copies the rope lanes of `heads` heads of `rows` rows between a full-layout
// tensor (token stride `full_stride` elements, heads 256 apart) and the
// compact staging layout (rows of heads x 64 lanes).
cudaError_t copy_compact(void* compact, void* full, int64_t rows, int heads, int64_t full_stride,
                         bool to_stage, cudaStream_t s) {
  constexpr size_t kElem = sizeof(uint16_t);
  constexpr size_t kWidth = size_t(kRopeDim) * kElem;  // 128 bytes
  char* c = static_cast<char*>(compact);
  char* f = static_cast<char*>(full) + size_t(kRopeLane0) * kElem;
  if (rows == 1 || full_stride == int64_t(heads) * kHeadDim) {  // one 2D copy over rows * heads
    const size_t fp = size_t(kHeadDim) * kElem;
    return to_stage ? cudaMemcpy2DAsync(c, kWidth, f, fp, kWidth, size_t(rows * heads), cudaMemcpyDefault, s)
                    : cudaMemcpy2DAsync(f, fp, c, kWidth, kWidth, size_t(rows * heads), cudaMemcpyDefault, s);
  }
  const size_t cp = kWidth * size_t(heads), fp = size_t(full_stride) * kElem;
  for (int h = 0; h < heads; ++h) {
    char* ch = c + size_t(h) * kWidth;
    char* fh = f + size_t(h) * kHeadDim * kElem;
    const cudaError_t e = to_stage ? cudaMemcpy2DAsync(ch, cp, fh, fp, kWidth, size_t(rows), cudaMemcpyDefault, s)
                                   : cudaMemcpy2DAsync(fh, fp, ch, cp, kWidth, size_t(rows), cudaMemcpyDefault, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// The device address of [p, p + bytes) for a kernel on the current device:
// page-locked host memory mapped into the device's address space (both ends
// mapped, at device addresses `bytes - 1` apart), or — when `allow_device` —
// device memory of the current device.  nullptr for anything else (pageable
// host memory, another device's memory, an unknown pointer).
void* mapped_range(const void* p, size_t bytes, bool allow_device) {
  if (p == nullptr || bytes == 0) return nullptr;
  int dev = 0;
  cudaPointerAttributes first{}, last{};
  const char* end = static_cast<const char*>(p) + (bytes - 1);
  if (cudaGetDevice(&dev) != cudaSuccess || cudaPointerGetAttributes(&first, p) != cudaSuccess ||
      cudaPointerGetAttributes(&last, end) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (first.type == cudaMemoryTypeHost && last.type == cudaMemoryTypeHost) {
    if (first.devicePointer == nullptr || last.devicePointer == nullptr) return nullptr;
    const char* d0 = static_cast<const char*>(first.devicePointer);
    const char* d1 = static_cast<const char*>(last.devicePointer);
    if (size_t(d1 - d0) != bytes - 1) return nullptr;
    return first.devicePointer;
  }
  if (allow_device && first.type == cudaMemoryTypeDevice && last.type == cudaMemoryTypeDevice &&
      first.device == dev && last.device == dev)
    return const_cast<void*>(p);
  return nullptr;
}

}  // namespace

extern "C" {

int welm_rope_copy_rope_lanes(void* dst, const void* src, int64_t rows, int64_t heads,
                              int64_t dst_token_stride, int64_t src_token_stride, int64_t direction,
                              void* stream) {
  if (rows < 0 || heads < 0 || heads > 64) return WELM_ROPE_ERR_BAD_SIZE;
  if (direction != 0 && direction != 1) return WELM_ROPE_ERR_BAD_MODE;
  if (rows == 0 || heads == 0) return WELM_ROPE_OK;
  if (!dst || !src) return WELM_ROPE_ERR_NULL_POINTER;
  if (rows > 1 && (dst_token_stride < heads * kHeadDim || src_token_stride < heads * kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  const cudaMemcpyKind kind = direction == 0 ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr size_t kElem = sizeof(uint16_t);
  constexpr size_t kWidth = size_t(kRopeDim) * kElem;                // 128 bytes per head
  constexpr size_t kHeadPitch = size_t(kHeadDim) * kElem;            // 512 bytes
  const size_t lane0 = size_t(kRopeLane0) * kElem;                   // 384 bytes
  char* d = static_cast<char*>(dst);
  const char* p = static_cast<const char*>(src);
  cudaError_t err = cudaSuccess;
  if ((rows == 1 || (dst_token_stride == heads * kHeadDim && src_token_stride == heads * kHeadDim))) {
    err = cudaMemcpy2DAsync(d + lane0, kHeadPitch, p + lane0, kHeadPitch, kWidth, size_t(rows * heads), kind, s);
  } else {
    for (int64_t h = 0; h < heads && err == cudaSuccess; ++h) {
      const size_t off = lane0 + size_t(h) * kHeadPitch;
      err = cudaMemcpy2DAsync(d + off, size_t(dst_token_stride) * kElem, p + off,
                              size_t(src_token_stride) * kElem, kWidth, size_t(rows), kind, s);
    }
  }
  if (err != cudaSuccess) {
    cudaGetLastError();
    return WELM_ROPE_ERR_CUDA;
  }
  return WELM_ROPE_OK;
}

int welm_rope_ordinary_host_static(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                                   int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                                   int64_t max_position, int32_t* device_status, void* stream) {
  if (n_tokens < 0 || max_position < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens > kStaticTokens) return WELM_ROPE_ERR_TOO_MANY_TOKENS;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!q || !k || !positions || !cos_sin_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (n_tokens > 1 && (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  if (!aligned16(cos_sin_cache)) return WELM_ROPE_ERR_BAD_STRIDE;  // the staged kernel reads 16-byte vectors
  unsigned char* stage = static_stage_for_current_device();
  if (stage == nullptr) return WELM_ROPE_ERR_CUDA;
  uint16_t* sq = reinterpret_cast<uint16_t*>(stage);
  uint16_t* sk = reinterpret_cast<uint16_t*>(stage + kStageQBytes);
  int64_t* sp = reinterpret_cast<int64_t*>(stage + kStageQBytes + kStageKBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = copy_compact(sq, q, n_tokens, kQHeads, q_token_stride, true, s);
  if (e == cudaSuccess) e = copy_compact(sk, k, n_tokens, 1, k_token_stride, true, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(sp, positions, size_t(n_tokens) * sizeof(int64_t), cudaMemcpyDefault, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return WELM_ROPE_ERR_CUDA;
  }
  const int32_t items = int32_t(n_tokens * kParts);
  const int rc = launch(rope_staged_kernel, unsigned((items + kBlock - 1) / kBlock), kBlock, 0, s, sq, sk,
                        static_cast<const int64_t*>(sp), cos_sin_cache, items, max_position, device_status);
  if (rc != WELM_ROPE_OK) return rc;
  e = copy_compact(sq, q, n_tokens, kQHeads, q_token_stride, false, s);
  if (e == cudaSuccess) e = copy_compact(sk, k, n_tokens, 1, k_token_stride, false, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return WELM_ROPE_ERR_CUDA;
  }
  return WELM_ROPE_OK;
}

int welm_rope_ordinary_mapped(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                              int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                              int64_t max_position, int32_t* device_status, void* stream) {
  if (n_tokens < 0 || max_position < 0 || n_tokens > kMaxItems / (kMappedPieces * kPieceThreads))
    return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!q || !k || !positions || !cos_sin_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (n_tokens > 1 && (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  // 16-byte vectors everywhere: aligned bases and token strides of 8 elements
  if (!aligned16(q) || !aligned16(k) || !aligned16(cos_sin_cache) ||
      (n_tokens > 1 && (q_token_stride % 8 != 0 || k_token_stride % 8 != 0)))
    return WELM_ROPE_ERR_BAD_STRIDE;
  constexpr size_t kElem = sizeof(uint16_t);
  const size_t q_bytes = (size_t(n_tokens - 1) * size_t(q_token_stride) + kQHeads * kHeadDim) * kElem;
  const size_t k_bytes = (size_t(n_tokens - 1) * size_t(k_token_stride) + kHeadDim) * kElem;
  void* dq = mapped_range(q, q_bytes, false);
  void* dk = mapped_range(k, k_bytes, false);
  void* dp = mapped_range(positions, size_t(n_tokens) * sizeof(int64_t), true);
  if (dq == nullptr || dk == nullptr || dp == nullptr) return WELM_ROPE_ERR_NOT_MAPPED;

  MappedArgs a{};
  a.q = static_cast<uint16_t*>(dq);
  a.k = static_cast<uint16_t*>(dk);
  a.positions = static_cast<const int64_t*>(dp);
  a.cache = cos_sin_cache;
  a.q_stride = q_token_stride;
  a.k_stride = k_token_stride;
  a.max_position = max_position;
  a.pieces = n_tokens * kMappedPieces;
  a.threads = (a.pieces * kPieceThreads + 31) / 32 * 32;
  a.status = device_status;
  const int sms = current_sm_count();
  const int64_t need = (a.threads + kMappedBlock - 1) / kMappedBlock;
  const int64_t cap = sms > 0 ? int64_t(sms) * 32 : need;
  return launch(rope_mapped_kernel, unsigned(need < cap ? need : cap), kMappedBlock, 0,
                static_cast<cudaStream_t>(stream), a);
}

}  // extern "C"
