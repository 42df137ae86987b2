// rope_ordinary.cu — ordinary prefill / decode kernels (one head per thread
// for small dense launches, the streaming dense kernel above that, and the
// segmented kernel over a staged tile table or tile slots) and the C entry
// welm_rope_ordinary.

#include "rope_host.cuh"

namespace {

// ---------------------------------------------------------------------------
// Ordinary prefill / decode: K head + 6 Q heads of token t at positions[t];
// the cache row is gathered once for all seven heads.
// ---------------------------------------------------------------------------
template <bool kVec>
__device__ __forceinline__ void ordinary_token(const RopeArgs& a, int64_t tok, int part, int64_t pos_hint) {
  const int64_t pos = __ldg(a.positions + tok);
  Slices<kVec, 1> kx;
  Slices<kVec, kQHeads> qx;
  kx.load(a.k + tok * a.k_stride, part);
  qx.load(a.q + tok * a.q_stride, part);
  RowGather<kVec> g;
  g.issue(a, -1, pos_hint, part);
  if (!g.finish(a, pos, part)) {
    if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    return;
  }
  kx.rotate_store(g.cs);
  qx.rotate_store(g.cs);
}

template <bool kVec, Source kSrc>
__global__ void __launch_bounds__(kBlock) rope_ordinary_kernel(const RopeArgs a) {
  extern __shared__ int32_t s_tab[];
  const int item0 = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t pos_hint = -1;
  if (kSrc == Source::kTileTable) prefetch_lines(a.tile_starts, int64_t(a.num_tiles + 1) * sizeof(int32_t));
  if (kSrc != Source::kTileSlots && item0 < a.k_items) {  // tokens are items: warm the first item's row
    prefetch_token<kVec>(a.q, a.k, a.q_stride, a.k_stride, item0 >> kPartShift, item0 & (kParts - 1));
    pos_hint = hint_load(a.positions + (item0 >> kPartShift));
    prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, item0 & (kParts - 1));
  }
  pdl_enter();
  if constexpr (kSrc == Source::kTileTable) {
    // One item per thread: tokens [0, k_items / 4), then one check per tile.
    stage_table_async(s_tab, a.tile_starts, a.num_tiles + 1);
    const int item = blockIdx.x * blockDim.x + threadIdx.x;
    const int part = item & (kParts - 1);
    const bool is_token = item < a.k_items;
    const int64_t tok = is_token ? (item >> kPartShift) : 0;
    Slices<kVec, 1> kx;
    Slices<kVec, kQHeads> qx;
    RowGather<kVec> g;
    bool pos_ok = false;
    if (is_token) {
      const int64_t pos = __ldg(a.positions + tok);
      kx.load(a.k + tok * a.k_stride, part);
      qx.load(a.q + tok * a.q_stride, part);
      g.issue(a, -1, pos_hint, part);
      pos_ok = g.finish(a, pos, part);
    } else if (item - a.k_items < a.num_tiles) {
      check_tile(a, item - a.k_items);
    }
    stage_table_wait();  // every thread of the CTA reaches this once
    if (is_token && table_covers(s_tab, a.num_tiles, tok)) {
      if (pos_ok) {
        kx.rotate_store(g.cs);
        qx.rotate_store(g.cs);
      } else if (part == 0) {
        raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
      }
    }
  } else {
    const int stride = gridDim.x * blockDim.x;
    for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < a.k_items; item += stride) {
      const int part = item & (kParts - 1);
      int64_t tok;
      if (slot_token<kSrc>(a, item >> kPartShift, part, tok))
        ordinary_token<kVec>(a, tok, part, item == item0 ? pos_hint : -1);
    }
  }
}

// ---------------------------------------------------------------------------
// Dense prefill above the one-head range (the bench workload, M = 16384).
// One item (token, part) per thread, in CTAs small enough in registers (at
// most 102, five CTAs per SM) that while one launch runs, a large part of the
// next launch in the stream is already resident beside it: under programmatic
// dependent launch the next launch's CTAs start as soon as every CTA of this
// one has passed its dependency wait, and they use the time before their own
// wait to ask L2 for every line their item will read — the token's rope-slice
// lines (prefetch.global.L2), its position line (the hint load) and its
// cos/sin lines at the hinted position.  A prefetch into L2 cannot return
// stale data (L2 is where the previous grid's writes land), so results are
// unchanged, but DRAM keeps streaming the next launch's reads while this one
// drains, and after the wait its loads hit L2.  Measured on one B200 at
// M = 16384 (graph replay, L2-cold rotating buffers, us per launch): the
// one-wave kernel without the data prefetch 6.99; with it 6.07.  What did not
// help: a grid of two CTAs per SM looping over items (7.6: each thread's items
// then pay their latency chains one after another), splitting a token's seven
// heads into two rounds to fit two whole launches per SM (7.5), 16-byte
// cp.async reads into a shared-memory scratch slot instead of the prefetch
// (6.6: the real reads delay the completing launch, and the static shared
// array shrinks L1), and 4 or 6 CTAs per SM (6.4 and 8.5).
// Launches above one item per thread (more than 4 CTAs per SM) loop, each
// thread prefetching its next item's lines before it works on the current.
// ---------------------------------------------------------------------------
// Token of a streaming item before the wait, from hint copies of the tile
// table (slots) or the item itself (dense); -1 when the slot looks empty.
template <Source kSrc>
__device__ __forceinline__ int64_t stream_token_hint(const RopeArgs& a, int item) {
  const int slot = item >> kPartShift;
  if (kSrc == Source::kDense) return slot;
  const int tile = slot / kTile, j = slot - tile * kTile;
  const int64_t b = hint_load_s32(a.tile_starts + tile), e = hint_load_s32(a.tile_starts + tile + 1);
  return j < e - b && j < kTile && b + j >= 0 && b + j < a.n_tokens ? b + j : -1;
}

// kDense: item = token * 4 + part.  kTileSlots (segmented tables whose tiles
// are mostly full): item = slot * 4 + part, 64 slots per tile, slot j of tile
// i holding token starts[i] + j (slot_token); before the wait the table
// entries are read as hints to find the token whose lines to prefetch.
template <bool kVec, Source kSrc>
__global__ void __launch_bounds__(kBlock, 5) rope_ordinary_stream_kernel(const RopeArgs a) {
  static_assert(kSrc == Source::kDense || kSrc == Source::kTileSlots, "dense or slot items");
  const int stride = gridDim.x * blockDim.x;
  const int first = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t hint = -1, tok_hint = -1;
  if (first < a.k_items) {  // before the wait: the first item's lines
    tok_hint = stream_token_hint<kSrc>(a, first);
    if (tok_hint >= 0) {
      // The position is read as a hint but not waited for: the cos/sin loads
      // at the hinted position start right after the wait (ordinary_token's
      // RowGather).  Prefetching the cos/sin lines here would stall the
      // thread on the hint before it reaches the wait; CTAs that start late
      // then release late (M=16384: 5.80 us without that prefetch, 6.15 with).
      prefetch_token<kVec>(a.q, a.k, a.q_stride, a.k_stride, tok_hint, first & (kParts - 1));
      hint = hint_load(a.positions + tok_hint);
    }
  }
  pdl_enter();
  for (int item = first; item < a.k_items; item += stride) {
    const int part = item & (kParts - 1);
    if (kSrc == Source::kDense) {
      const int next = item + stride;
      if (next < a.k_items) prefetch_token<kVec>(a.q, a.k, a.q_stride, a.k_stride, next >> kPartShift, next & (kParts - 1));
    }
    int64_t tok;
    if (slot_token<kSrc>(a, item >> kPartShift, part, tok))
      ordinary_token<kVec>(a, tok, part, tok == tok_hint ? hint : -1);
    hint = tok_hint = -1;
  }
}

// Small dense launches: one head per thread instead of seven.  Item =
// ((token * 7 + head) * 4 + part), head 0 the K head and 1..6 the Q heads, so
// four consecutive lanes cover one head's rope slice and a warp covers eight
// heads.  A decode-sized launch then spreads its loads and stores over seven
// times as many threads and SMs; every thread gathers its part of the cos/sin
// row itself (L1/L2 hits after the first).  Same arithmetic, same results.
template <bool kVec, bool kPrefetch>
__global__ void __launch_bounds__(kBlock) rope_ordinary_head_kernel(const RopeArgs a) {
  const int item = blockIdx.x * blockDim.x + threadIdx.x;  // the grid covers every item once
  const int part = item & (kParts - 1);
  const int slice = item >> kPartShift;
  const int64_t tok = slice / kHeadsPerToken;
  const int head = slice - int(tok) * kHeadsPerToken;
  const bool live = item < a.k_items;
  int64_t pos_hint = -1;
  if (live) {  // before the wait: the position and the cos/sin lines (and, with kPrefetch, the slice line)
    if (kPrefetch && kVec && part == 0)
      prefetch_row_slices<1>(head == 0 ? a.k + tok * a.k_stride : a.q + tok * a.q_stride + (head - 1) * kHeadDim, 0);
    pos_hint = hint_load(a.positions + tok);
    if (head == 0) prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, part);
  }
  pdl_enter();
  if (!live) return;
  const int64_t pos = __ldg(a.positions + tok);
  Slices<kVec, 1> x;
  x.load(head == 0 ? a.k + tok * a.k_stride : a.q + tok * a.q_stride + (head - 1) * kHeadDim, part);
  RowGather<kVec> g;
  g.issue(a, -1, pos_hint, part);
  if (!g.finish(a, pos, part)) {
    if (part == 0 && head == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    return;
  }
  x.rotate_store(g.cs);
}

// Segmented launches run the streaming kernel over tile slots when at least
// half of the slots can hold a token (2 N >= 64 T), else the token-mapped
// kernel over the staged table (or its slot source for tables too large to
// stage), which never launches a thread for an empty slot.  Measured on one
// B200 (graph replay, L2-cold sets, us per launch, staged table -> slots): the
// reference's segmented cases M=4096/8 requests 2.87 -> 2.76, M=8192/32 4.18 ->
// 4.05, M=9616/8 uneven 4.90 -> 4.55, M=16384/8 uneven 6.43 -> 6.15,
// M=16384/64 6.53 -> 6.29, M=16384/128 uneven (80 % of slots live) 6.68 ->
// 6.44.
bool stream_slots(int64_t num_tiles, int64_t n_tokens) { return num_tiles > 0 && 2 * n_tokens >= num_tiles * kTile; }

template <bool kVec>
int launch_ordinary(const Plan& plan, const RopeArgs& a, cudaStream_t s) {
  if (plan.src == Source::kDense) {
    const int64_t items = plan.token_items * kHeadsPerToken;
    LaunchShape shape;
    if (head_split_shape(plan.token_items / kParts, shape)) {
      RopeArgs h = a;
      h.k_items = int32_t(items);
      return items >= kHeadPrefetchMinItems ? launch(rope_ordinary_head_kernel<kVec, true>, shape.grid, shape.block, 0, s, h)
                                            : launch(rope_ordinary_head_kernel<kVec, false>, shape.grid, shape.block, 0, s, h);
    }
    shape = stream_shape(plan.token_items);
    return launch(rope_ordinary_stream_kernel<kVec, Source::kDense>, shape.grid, shape.block, 0, s, a);
  }
  if (stream_slots(a.num_tiles, a.n_tokens)) {
    RopeArgs h = a;
    h.k_items = int32_t(int64_t(a.num_tiles) * kTile * kParts);
    // one item per thread at every size: a slot's token comes from the table,
    // so a thread looping over slots could not prefetch its next one
    LaunchShape shape = stream_shape(h.k_items);
    if (shape.block == unsigned(kBlock)) shape.grid = unsigned((int64_t(h.k_items) + kBlock - 1) / kBlock);
    return launch(rope_ordinary_stream_kernel<kVec, Source::kTileSlots>, shape.grid, shape.block, 0, s, h);
  }
  switch (plan.src) {
    case Source::kTileTable: return launch_plan(rope_ordinary_kernel<kVec, Source::kTileTable>, plan, a, s);
    default: return launch_plan(rope_ordinary_kernel<kVec, Source::kTileSlots>, plan, a, s);
  }
}

}  // namespace

extern "C" {

int welm_rope_ordinary(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                       const int32_t* segment_tile_starts, int64_t num_work_tiles,
                       int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                       int64_t has_segments, int64_t max_position, int32_t* device_status,
                       void* stream) {
  if (has_segments != 0 && has_segments != 1) return WELM_ROPE_ERR_BAD_MODE;
  if (num_work_tiles < 0 || n_tokens < 0 || max_position < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (num_work_tiles > kMaxItems / (kTile * kParts) || n_tokens > kMaxItems / kParts)
    return WELM_ROPE_ERR_BAD_SIZE;
  const Plan plan = plan_tokens(has_segments, num_work_tiles, n_tokens);
  if (plan.token_items == 0) return WELM_ROPE_OK;  // nothing to rotate
  if (!q || !k || !positions || !cos_sin_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (has_segments && !segment_tile_starts) return WELM_ROPE_ERR_NULL_POINTER;
  if (n_tokens > 1 && (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;

  RopeArgs a{};
  a.q = static_cast<uint16_t*>(q);
  a.k = static_cast<uint16_t*>(k);
  a.positions = positions;
  a.cache = cos_sin_cache;
  a.tile_starts = segment_tile_starts;
  a.q_stride = q_token_stride;
  a.k_stride = k_token_stride;
  a.n_tokens = n_tokens;
  a.max_position = max_position;
  a.status = device_status;
  a.k_items = int32_t(plan.token_items);
  a.num_tiles = int32_t(num_work_tiles);
  const bool vec = aligned16(q) && aligned16(k) && aligned16(cos_sin_cache) &&
                   (n_tokens <= 1 || (q_token_stride % 8 == 0 && k_token_stride % 8 == 0));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return vec ? launch_ordinary<true>(plan, a, s) : launch_ordinary<false>(plan, a, s);
}

}  // extern "C"
