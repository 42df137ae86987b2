// rope_tiles.cu — the segmented 64-token tile-boundary builder: device
// kernel and host twins.

#include "rope_host.cuh"

namespace {

// ---------------------------------------------------------------------------
// Segmented tile-boundary builder: one CTA, requests processed in chunks of
// kBuildThreads with a running carry (tokens, tiles).  Within a chunk the
// per-request tile counts and lengths are scanned with warp shuffles, then the
// chunk's tile starts are written cooperatively (each thread finds the
// request of its tile by binary search over the chunk's inclusive scan).
// ---------------------------------------------------------------------------
constexpr int kBuildThreads = 1024;
constexpr int kBuildWarps = kBuildThreads / 32;

__device__ __forceinline__ void block_inclusive_scan2(int64_t& x, int64_t& y, int64_t* wx, int64_t* wy) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t tx = __shfl_up_sync(0xffffffffu, x, d);
    const int64_t ty = __shfl_up_sync(0xffffffffu, y, d);
    if (lane >= d) { x += tx; y += ty; }
  }
  if (lane == 31) { wx[warp] = x; wy[warp] = y; }
  __syncthreads();
  if (warp == 0) {
    int64_t vx = lane < kBuildWarps ? wx[lane] : 0;
    int64_t vy = lane < kBuildWarps ? wy[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int64_t tx = __shfl_up_sync(0xffffffffu, vx, d);
      const int64_t ty = __shfl_up_sync(0xffffffffu, vy, d);
      if (lane >= d) { vx += tx; vy += ty; }
    }
    if (lane < kBuildWarps) { wx[lane] = vx; wy[lane] = vy; }
  }
  __syncthreads();
  if (warp > 0) { x += wx[warp - 1]; y += wy[warp - 1]; }
}

__global__ void __launch_bounds__(kBuildThreads)
build_tiles_kernel(const int64_t* __restrict__ lens, int32_t bs, int32_t* __restrict__ starts,
                   int64_t capacity, int32_t* __restrict__ num_tiles_out,
                   int64_t* __restrict__ last_index_out, int32_t* status) {
  __shared__ int64_t s_tok[kBuildThreads];   // inclusive token scan of the chunk
  __shared__ int64_t s_tile[kBuildThreads];  // inclusive tile scan of the chunk
  __shared__ int64_t wx[kBuildWarps], wy[kBuildWarps];
  pdl_enter();
  int64_t carry_tok = 0, carry_tile = 0;     // identical in every thread
  for (int base = 0; base < bs; base += kBuildThreads) {
    const int r = base + threadIdx.x;
    int64_t len = 0;
    if (r < bs) {
      len = lens[r];
      if (len < 0) {
        raise_status(status, WELM_ROPE_DEV_BAD_LENGTH);
        len = 0;
      }
    }
    int64_t tok = len, tiles = (len + kTile - 1) / kTile;
    block_inclusive_scan2(tok, tiles, wx, wy);
    s_tok[threadIdx.x] = tok;
    s_tile[threadIdx.x] = tiles;
    if (r < bs && last_index_out != nullptr) last_index_out[r] = carry_tok + tok - 1;
    __syncthreads();
    const int chunk = min(kBuildThreads, bs - base);
    const int64_t chunk_tiles = s_tile[chunk - 1];
    for (int64_t t = threadIdx.x; t < chunk_tiles; t += kBuildThreads) {
      int lo = 0, hi = chunk - 1;
      while (lo < hi) {  // first request whose inclusive tile count exceeds t
        const int mid = (lo + hi) >> 1;
        if (s_tile[mid] > t) hi = mid; else lo = mid + 1;
      }
      const int64_t first_tile = lo > 0 ? s_tile[lo - 1] : 0;
      const int64_t first_tok = lo > 0 ? s_tok[lo - 1] : 0;
      const int64_t out = carry_tile + t;
      const int64_t value = carry_tok + first_tok + (t - first_tile) * kTile;
      if (out < capacity && value <= INT32_MAX) {
        starts[out] = int32_t(value);
      } else {
        raise_status(status, WELM_ROPE_DEV_BAD_TILE);
      }
    }
    carry_tok += s_tok[chunk - 1];
    carry_tile += chunk_tiles;
    __syncthreads();  // the next chunk overwrites s_tok / s_tile
  }
  if (threadIdx.x == 0) {
    if (carry_tile < capacity && carry_tok <= INT32_MAX) {
      starts[carry_tile] = int32_t(carry_tok);
    } else {
      raise_status(status, WELM_ROPE_DEV_BAD_TILE);
    }
    *num_tiles_out = carry_tile <= INT32_MAX ? int32_t(carry_tile) : -1;
  }
}

}  // namespace

extern "C" {

int welm_rope_build_tiles(const int64_t* seq_lens, int64_t batch_size, int32_t* tile_starts,
                          int64_t capacity, int32_t* num_tiles_out, int64_t* last_index_out,
                          int32_t* device_status, void* stream) {
  if (batch_size < 0 || batch_size > INT32_MAX || capacity < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (capacity < 1) return WELM_ROPE_ERR_CAPACITY;  // starts[T] always needs a slot
  if (!tile_starts || !num_tiles_out || (batch_size > 0 && !seq_lens))
    return WELM_ROPE_ERR_NULL_POINTER;
  return launch(build_tiles_kernel, 1, kBuildThreads, 0, static_cast<cudaStream_t>(stream), seq_lens,
                int32_t(batch_size), tile_starts, capacity, num_tiles_out, last_index_out,
                device_status);
}

int welm_rope_count_tiles_host(const int64_t* seq_lens, int64_t batch_size,
                               int64_t* num_tiles_out) {
  if (batch_size < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (!num_tiles_out || (batch_size > 0 && !seq_lens)) return WELM_ROPE_ERR_NULL_POINTER;
  int64_t tiles = 0;
  for (int64_t r = 0; r < batch_size; ++r) {
    if (seq_lens[r] < 0) return WELM_ROPE_ERR_BAD_SIZE;
    tiles += (seq_lens[r] + kTile - 1) / kTile;
  }
  *num_tiles_out = tiles;
  return WELM_ROPE_OK;
}

int welm_rope_build_tiles_host(const int64_t* seq_lens, int64_t batch_size, int32_t* tile_starts,
                               int64_t capacity, int64_t* num_tiles_out,
                               int64_t* last_index_out) {
  int64_t tiles = 0;
  const int rc = welm_rope_count_tiles_host(seq_lens, batch_size, &tiles);
  if (rc != WELM_ROPE_OK) return rc;
  if (!tile_starts) return WELM_ROPE_ERR_NULL_POINTER;
  if (capacity < tiles + 1) return WELM_ROPE_ERR_CAPACITY;
  int64_t token = 0, t = 0;
  for (int64_t r = 0; r < batch_size; ++r) {
    for (int64_t off = 0; off < seq_lens[r]; off += kTile) {
      if (token + off > INT32_MAX) return WELM_ROPE_ERR_BAD_SIZE;
      tile_starts[t++] = int32_t(token + off);
    }
    token += seq_lens[r];
    if (last_index_out) last_index_out[r] = token - 1;
  }
  if (token > INT32_MAX) return WELM_ROPE_ERR_BAD_SIZE;
  tile_starts[t] = int32_t(token);
  if (num_tiles_out) *num_tiles_out = tiles;
  return WELM_ROPE_OK;
}

}  // extern "C"
