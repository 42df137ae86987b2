// rope_mirror.cu — KV-mirror kernels (one head per item over dense tokens or
// tile slots, and the variant driven by request lengths) and their C entries.

#include "rope_host.cuh"

namespace {

// KV-mirror semantics: the BS Q rows are rotated at positions[last_index[b]]
// (bench_welmv4_inplace_rope_npu.py:839-854), K token t at positions[t]
// (bench_welmv4_inplace_rope_npu.py:856-919).  Q rows and K rows are disjoint
// tensors, so the two phases need no ordering.
//
// ---------------------------------------------------------------------------
// KV-mirror prefill, one head per item.  Items [0, q_items) are Q heads, item
// = (row * 6 + head) * 4 + part.  The K items follow: with has_segments = 0
// one per (token, part); with a tile table one per (tile, slot, part), 64
// slots per tile, slot j of tile i holding token starts[i] + j when j <
// min(64, starts[i+1] - starts[i]) (bench_welmv4_inplace_rope_npu.py:856-867),
// so no token-to-tile search is needed.  Every thread holds one head's two
// 16-byte vectors and its cos/sin (at most 64 registers), so under
// programmatic dependent launch most or all of the next launch's CTAs are
// resident while this one runs, and before their dependency wait each item
// does what needs none of the previous launch's results:
//   * reads as hints its token's position (Q heads: last_index, then the
//     position it names; slots: starts[i], then the position of the token it
//     gives), prefetching the slice line and the cos/sin lines they name.
// After the wait one round of loads finishes an item in the common case: the
// data and position at the hinted token next to the real table entries (or
// last_index), and cos/sin at the hinted position (RowGather).  An item keeps
// what it loaded on hints only when the real chain names the same token and
// position; otherwise it reloads, so results equal the plain dependent
// chain's for every input.
// ---------------------------------------------------------------------------
template <bool kVec, Source kSrc>
__global__ void __launch_bounds__(kBlock, 8) rope_mirror_head_kernel(const RopeArgs a) {
  static_assert(kSrc == Source::kDense || kSrc == Source::kTileSlots, "dense or slot items");
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  const int part = item & (kParts - 1);
  const bool is_q = item < a.q_items;
  const int k_item = item - a.q_items;
  const bool is_k = !is_q && k_item < a.k_items;
  const int q_slice = is_q ? (item >> kPartShift) : 0;
  const int row = q_slice / kQHeads;
  const int head = q_slice - row * kQHeads;
  const int slot = k_item >> kPartShift;

  // Before the wait: hints and prefetches only.
  int64_t src_hint = -1, pos_hint = -1, tok_hint = -1;
  uint16_t* q_row = a.q + int64_t(row) * a.q_stride + head * kHeadDim;
  if (is_q) {
    if (kVec && part == 0) prefetch_row_slices<1>(q_row, 0);
    src_hint = hint_load(a.last_index + row);
    if (src_hint >= 0 && src_hint < a.n_tokens) pos_hint = hint_load(a.positions + src_hint);
  } else if (is_k) {
    if (kSrc == Source::kDense) {
      tok_hint = slot;
    } else {
      const int tile = slot / kTile, j = slot - tile * kTile;
      const int64_t b = hint_load_s32(a.tile_starts + tile), e = hint_load_s32(a.tile_starts + tile + 1);
      if (j < e - b && j < kTile && b + j >= 0 && b + j < a.n_tokens) tok_hint = b + j;
    }
    if (tok_hint >= 0) {
      if (kVec && part == 0) prefetch_row_slices<1>(a.k + tok_hint * a.k_stride, 0);
      pos_hint = hint_load(a.positions + tok_hint);
    }
  }
  // Unlike the ordinary streaming kernel, the mirror keeps its cos/sin
  // prefetch before the wait even though it waits on the hint: every CTA of
  // the next launch is resident about 1.5 us early, and without it the
  // contiguous mirror (16384 distinct rows from DRAM) slowed from 2.26 to
  // 2.75 us.
  prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, part);
  pdl_enter();

  Slices<kVec, 1> x;
  RowGather<kVec> g;
  if (is_q) {
    x.load(q_row, part);
    const int64_t src = __ldg(a.last_index + row);
    g.issue(a, src_hint, pos_hint, part);
    const bool flag = part == 0 && head == 0;  // one report per row
    if (src < 0 || src >= a.n_tokens) {
      if (flag) raise_status(a.status, WELM_ROPE_DEV_BAD_LAST_INDEX);
    } else if (!g.finish(a, g.position(a, src), part)) {
      if (flag) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    } else {
      x.rotate_store(g.cs);
    }
  } else if (is_k) {
    int64_t pos = 0;
    if (tok_hint >= 0) {  // loads on the hinted token (after the wait: current data)
      x.load(a.k + tok_hint * a.k_stride, part);
      pos = __ldg(a.positions + tok_hint);
    }
    g.issue(a, -1, pos_hint, part);
    int64_t tok;
    if (slot_token<kSrc>(a, slot, part, tok)) {  // the real token (slots: the real table entries)
      if (tok != tok_hint) {
        x.load(a.k + tok * a.k_stride, part);
        pos = __ldg(a.positions + tok);
      }
      if (g.finish(a, pos, part)) {
        x.rotate_store(g.cs);
      } else if (part == 0) {
        raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// KV mirror from request lengths.  Every CTA stages the BS lengths into shared
// memory (cp.async) while its K-token loads and cache gathers fly; after the
// one barrier each warp derives what it needs with shuffles, without further
// CTA-wide synchronisation: K token t is rotated iff t < sum(lengths), Q row
// r uses src = end_r - 1 with end_r = lengths[0] + ... + lengths[r].  Before
// the dependency wait, warps holding Q rows run the same scan over hint
// copies of the lengths so each row's source position and cos/sin row can be
// loaded speculatively; the real scan keeps them only if the hints held.  One
// item per thread, one head per item: Q heads, then K tokens.  Measured on one
// B200 (graph replay, L2-cold sets, us per launch) against the previous
// six-head-row kernel without data prefetch: N=16384 BS=128 uneven 3.71 ->
// 3.34, N=16384 BS=32 3.21 -> 2.70, N=9616 BS=8 2.83 -> 2.36, N=8192 BS=2
// 2.68 -> 2.27.  A preferred shared-memory carveout of 50 % was slower.
// ---------------------------------------------------------------------------
constexpr int kLensCap = WELM_ROPE_LENS_MAX_BATCH;

// Warp-cooperative prefix over the staged lengths (negative entries count as
// 0): returns the total and, for `row` in [0, n), end_row = s[0] + ... +
// s[row].  Every lane of the warp must call it (it shuffles).
template <typename Load>
__device__ __forceinline__ int64_t warp_request_ends(Load load, int n, int row, int64_t& end_row, bool& negative) {
  const int lane = threadIdx.x & 31;
  const int chunk = (n + 31) >> 5;
  const int lo = min(n, lane * chunk), hi = min(n, lo + chunk);
  int64_t part_sum = 0;
  for (int i = lo; i < hi; ++i) {
    const int64_t v = load(i);
    negative |= v < 0;
    part_sum += v > 0 ? v : 0;
  }
  negative = __any_sync(0xffffffffu, negative);
  int64_t incl = part_sum;  // inclusive scan of the lanes' chunk sums
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += t;
  }
  const int64_t total = __shfl_sync(0xffffffffu, incl, 31);
  const int c = row >= 0 && row < n ? row / chunk : 0;  // the chunk holding `row`
  const int64_t before = __shfl_sync(0xffffffffu, incl - part_sum, c);
  end_row = before;
  if (row >= 0 && row < n) {
    for (int i = c * chunk; i <= row; ++i) {
      const int64_t v = load(i);
      end_row += v > 0 ? v : 0;
    }
  }
  return total;
}

// The same from request lengths, one head per item: items [0, q_items) are
// Q heads (row * 6 + head) * 4 + part, then K tokens token * 4 + part.  Before
// the wait, warps holding Q items run the length scan on hint copies of the
// lengths to find each row's source token and warm its position and cos/sin
// lines; every item prefetches its slice line.  After the wait the lengths
// are staged in shared memory (cp.async) while the data loads fly, and after
// the one barrier each warp derives the total and its rows' ends with
// shuffles; the Q heads keep their speculative loads only if the hints held.
template <bool kVec>
__global__ void __launch_bounds__(kBlock, 8) rope_mirror_lens_head_kernel(const RopeArgs a, const int64_t* lens,
                                                                          int batch) {
  extern __shared__ int64_t s_len[];
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  const int part = item & (kParts - 1);
  const bool is_q = item < a.q_items;
  const int k_item = item - a.q_items;
  const bool is_k = !is_q && k_item < a.k_items;
  const int64_t tok = is_k ? (k_item >> kPartShift) : 0;
  const int q_slice = is_q ? (item >> kPartShift) : 0;
  const int row = q_slice / kQHeads;
  const int head = q_slice - row * kQHeads;
  uint16_t* slice_row = is_q ? a.q + int64_t(row) * a.q_stride + head * kHeadDim : a.k + tok * a.k_stride;

  // Before the wait: hints and prefetches only.
  prefetch_lines(lens, int64_t(batch) * sizeof(int64_t));
  int64_t src_hint = -1, pos_hint = -1;
  if ((item & ~31) < a.q_items) {  // warp-uniform: the scan shuffles
    int64_t end_hint = 0;
    bool neg_hint = false;
    warp_request_ends([&](int i) { return hint_load(lens + i); }, batch, is_q ? row : -1, end_hint, neg_hint);
    if (is_q) {
      src_hint = end_hint - 1;
      if (src_hint >= 0 && src_hint < a.n_tokens) pos_hint = hint_load(a.positions + src_hint);
    }
  }
  if (is_q || is_k) {
    if (kVec && part == 0) prefetch_row_slices<1>(slice_row, 0);
    if (is_k) pos_hint = hint_load(a.positions + tok);
  }
  prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, part);
  pdl_enter();

  for (int j = threadIdx.x; j < batch; j += blockDim.x)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(s_len + j)), "l"(lens + j) : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
  Slices<kVec, 1> x;
  RowGather<kVec> g;
  bool pos_ok = false;
  if (is_q) {
    x.load(slice_row, part);
    g.issue(a, src_hint, pos_hint, part);
  } else if (is_k) {
    const int64_t pos = __ldg(a.positions + tok);
    x.load(slice_row, part);
    g.issue(a, -1, pos_hint, part);
    pos_ok = g.finish(a, pos, part);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  int64_t end_row = 0;
  bool negative = false;
  const int64_t total = warp_request_ends([&](int i) { return s_len[i]; }, batch, is_q ? row : -1, end_row, negative);
  if (is_q) {
    const bool flag = part == 0 && head == 0;  // one report per row
    const int64_t src = end_row - 1;
    if (src < 0 || src >= a.n_tokens) {
      if (flag) raise_status(a.status, WELM_ROPE_DEV_BAD_LAST_INDEX);
    } else if (!g.finish(a, g.position(a, src), part)) {
      if (flag) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    } else {
      x.rotate_store(g.cs);
    }
  } else if (is_k && tok < total) {
    if (pos_ok) {
      x.rotate_store(g.cs);
    } else if (part == 0) {
      raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    }
  }
  if (negative && blockIdx.x == 0 && threadIdx.x == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_LENGTH);
}

template <typename Kernel>
int launch_heads(Kernel kernel, int64_t total, const RopeArgs& a, cudaStream_t s) {
  const int sms = current_sm_count();
  if (sms > 0 && total <= int64_t(sms) * kBlock) return launch(kernel, unsigned((total + 31) / 32), 32u, 0, s, a);
  return launch(kernel, unsigned((total + kBlock - 1) / kBlock), kBlock, 0, s, a);
}

template <bool kVec>
int launch_mirror(const Plan& plan, const RopeArgs& a, int64_t rows, cudaStream_t s) {
  RopeArgs h = a;
  h.q_items = int32_t(rows * kQHeads * kParts);
  if (plan.src == Source::kDense)
    return launch_heads(rope_mirror_head_kernel<kVec, Source::kDense>, int64_t(h.q_items) + plan.token_items, h, s);
  // tile slots for every table size: 64 slots per tile
  h.k_items = int32_t(int64_t(a.num_tiles) * kTile * kParts);
  return launch_heads(rope_mirror_head_kernel<kVec, Source::kTileSlots>, int64_t(h.q_items) + h.k_items, h, s);
}

}  // namespace

extern "C" {

int welm_rope_mirror(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                     const int64_t* last_index, const int32_t* segment_tile_starts,
                     int64_t num_work_tiles, int64_t n_tokens, int64_t batch_size,
                     int64_t q_token_stride, int64_t k_token_stride, int64_t has_segments,
                     int64_t max_position, int32_t* device_status, void* stream) {
  if (has_segments != 0 && has_segments != 1) return WELM_ROPE_ERR_BAD_MODE;
  if (num_work_tiles < 0 || n_tokens < 0 || batch_size < 0 || max_position < 0)
    return WELM_ROPE_ERR_BAD_SIZE;
  if (num_work_tiles > kMaxItems / (kTile * kParts) || n_tokens > kMaxItems / kParts ||
      batch_size > kMaxItems / kParts)
    return WELM_ROPE_ERR_BAD_SIZE;
  const Plan plan = n_tokens > 0 ? plan_tokens(has_segments, num_work_tiles, n_tokens) : Plan{Source::kDense, 0, 0};
  const int64_t rows = n_tokens > 0 ? batch_size : 0;  // Q rows need a valid last_index target
  const int64_t k_items = has_segments ? num_work_tiles * kTile * kParts : plan.token_items;
  if (rows * kQHeads * kParts + k_items > kMaxItems) return WELM_ROPE_ERR_BAD_SIZE;
  if (plan.token_items == 0 && rows == 0) return WELM_ROPE_OK;
  if (!positions || !cos_sin_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (rows > 0 && (!q || !last_index)) return WELM_ROPE_ERR_NULL_POINTER;
  if (plan.token_items > 0 && !k) return WELM_ROPE_ERR_NULL_POINTER;
  if (has_segments && plan.token_items > 0 && !segment_tile_starts) return WELM_ROPE_ERR_NULL_POINTER;
  if ((rows > 1 && q_token_stride < kQHeads * kHeadDim) || (n_tokens > 1 && k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;

  RopeArgs a{};
  a.q = static_cast<uint16_t*>(q);
  a.k = static_cast<uint16_t*>(k);
  a.positions = positions;
  a.cache = cos_sin_cache;
  a.last_index = last_index;
  a.tile_starts = segment_tile_starts;
  a.q_stride = q_token_stride;
  a.k_stride = k_token_stride;
  a.n_tokens = n_tokens;
  a.max_position = max_position;
  a.status = device_status;
  a.q_items = int32_t(rows * kParts);
  a.k_items = int32_t(plan.token_items);
  a.num_tiles = int32_t(num_work_tiles);
  const bool vec = aligned16(q) && aligned16(k) && aligned16(cos_sin_cache) &&
                   (rows <= 1 || q_token_stride % 8 == 0) &&
                   (n_tokens <= 1 || k_token_stride % 8 == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return vec ? launch_mirror<true>(plan, a, rows, s) : launch_mirror<false>(plan, a, rows, s);
}

int welm_rope_mirror_from_lens(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                               const int64_t* seq_lens, int64_t n_tokens, int64_t batch_size,
                               int64_t q_token_stride, int64_t k_token_stride, int64_t max_position,
                               int32_t* device_status, void* stream) {
  if (n_tokens < 0 || batch_size < 0 || max_position < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (batch_size > kLensCap || n_tokens > (kMaxItems - int64_t(kLensCap) * kQHeads * kParts) / kParts)
    return WELM_ROPE_ERR_BAD_SIZE;
  if (batch_size == 0 || n_tokens == 0) return WELM_ROPE_OK;  // no request, or no token to rotate
  if (!q || !k || !positions || !cos_sin_cache || !seq_lens) return WELM_ROPE_ERR_NULL_POINTER;
  if ((batch_size > 1 && q_token_stride < kQHeads * kHeadDim) || (n_tokens > 1 && k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  if ((reinterpret_cast<uintptr_t>(seq_lens) & 7u) != 0) return WELM_ROPE_ERR_BAD_STRIDE;  // 8-byte cp.async
  RopeArgs a{};
  a.q = static_cast<uint16_t*>(q);
  a.k = static_cast<uint16_t*>(k);
  a.positions = positions;
  a.cache = cos_sin_cache;
  a.q_stride = q_token_stride;
  a.k_stride = k_token_stride;
  a.n_tokens = n_tokens;
  a.max_position = max_position;
  a.status = device_status;
  a.q_items = int32_t(batch_size * kQHeads * kParts);
  a.k_items = int32_t(n_tokens * kParts);
  const bool vec = aligned16(q) && aligned16(k) && aligned16(cos_sin_cache) &&
                   (batch_size <= 1 || q_token_stride % 8 == 0) && (n_tokens <= 1 || k_token_stride % 8 == 0);
  const int64_t total = int64_t(a.q_items) + a.k_items;
  const size_t smem = size_t(batch_size) * sizeof(int64_t);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int b = int(batch_size);
  const int sms = current_sm_count();
  const unsigned block = sms > 0 && total <= int64_t(sms) * kBlock ? 32u : unsigned(kBlock);
  const unsigned grid = unsigned((total + block - 1) / block);
  return vec ? launch(rope_mirror_lens_head_kernel<true>, grid, block, smem, s, a, seq_lens, b)
             : launch(rope_mirror_lens_head_kernel<false>, grid, block, smem, s, a, seq_lens, b);
}

}  // extern "C"
