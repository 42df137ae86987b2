// welm_rope.cu — sm_100a kernels and C ABI for WeLMv4's in-place partial RoPE.
//
// Semantics follow the reference's oracle `apply_reference` /
// `reference_outputs` (bench_welmv4_inplace_rope_npu.py:1489-1521): for every
// rotated row, lanes 192..223 (x1) and 224..255 (x2) of each 256-lane head
// become bf16(x1*c - x2*s) and bf16(x1*s + x2*c), where c and s are the cos and
// sin halves of the FP32 cache row at the row's position.  Products, the
// difference and the sum are each rounded in FP32 (__fmul_rn/__fsub_rn/
// __fadd_rn: no FMA contraction), then one round-to-nearest-even to BF16,
// exactly as the reference's separate torch elementwise ops round.
//
// Work decomposition (B200-first, not the reference's 56-program tile loop):
//   * one work item = (row, part): a thread owns 8 lanes of x1 and the
//     matching 8 lanes of x2 of every head of that row, i.e. two 16-byte
//     vectors per head; 4 threads cover a row's 128-byte rope slice per head;
//   * the thread loads its 8 cos + 8 sin values once (four 16-byte loads) and
//     reuses them from registers for all heads of the row (7 for the ordinary
//     op: 1 K + 6 Q), so each cache row crosses HBM once per token;
//   * every data load of the row is issued before the position-dependent
//     cache load, so the position -> cache dependency overlaps the data
//     stream; the grid is sized so a whole prefill is resident in one wave.
//   * 64-token work tiles are kept only as the segment / masking unit of the
//     reference's contract; positions are gathered per token, so no
//     contiguity inside a tile is assumed (bench_welmv4_inplace_rope_npu.py:714-715
//     assumes it, the oracle does not).

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <utility>

#include "welm_rope.h"

namespace {

constexpr int kHeadDim = WELM_ROPE_HEAD_DIM;        // 256 lanes per head
constexpr int kRopeDim = WELM_ROPE_ROPE_DIM;        // 64 rotated lanes
constexpr int kHalf = kRopeDim / 2;                 // 32: x1 / x2 width
constexpr int kRopeLane0 = kHeadDim - kRopeDim;     // 192: first rotated lane
constexpr int kQHeads = WELM_ROPE_NUM_Q_HEADS;      // 6
constexpr int kTile = WELM_ROPE_TILE_TOKENS;        // 64
constexpr int kLanes = 8;                           // x1 lanes owned by one thread
constexpr int kParts = kHalf / kLanes;              // 4 threads per row slice
constexpr int kPartShift = 2;                       // log2(kParts)
constexpr int kBlock = 128;                         // threads per CTA
constexpr int kMaxDevices = 64;

static_assert(kParts == (1 << kPartShift), "part count must be a power of two");

struct RopeArgs {
  uint16_t* q;                 // BF16 bits
  uint16_t* k;                 // BF16 bits
  const int64_t* positions;    // [N]
  const float* cache;          // [max_position, 64]
  const int64_t* last_index;   // [BS] (mirror only)
  const int32_t* tile_starts;  // [num_tiles + 1] (segmented only)
  int64_t q_stride;            // elements between Q rows
  int64_t k_stride;            // elements between K rows
  int64_t n_tokens;            // K rows / positions length
  int64_t max_position;        // cache rows
  int32_t* status;             // optional device status word
  int32_t q_items;             // Q-row items (mirror): BS * kParts
  int32_t k_items;             // token items: tokens (or tile slots) * kParts
  int32_t num_tiles;           // work tiles (segmented)
};

struct CosSin {
  float c[kLanes];
  float s[kLanes];
};

// Cold path, kept out of line so the hot loop's register allocation and load
// scheduling do not depend on it.
__device__ __noinline__ void raise_status(int32_t* status, int bit) {
  if (status != nullptr) atomicOr(status, bit);
}

// Programmatic dependent launch: wait until every grid this launch depends on
// has completed and its memory is visible (a no-op when the launch carries no
// programmatic dependency), then let the next grid in the stream begin its own
// launch while this one runs.  Every kernel calls this before its first global
// memory access, so ordering with any producer is preserved.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Work done BEFORE pdl_enter(), while the previous grid may still run: a
// thread reads its position as a hint only (ld.global.cg: served from L2,
// never allocated in L1, so no stale L1 line can answer the real loads made
// after the wait) and prefetches that cos/sin row into L2.  A prefetch cannot
// change a result — L2 is where writes of the previous grid land — and a
// stale or garbage hint only fetches a useless line; hints outside the cache
// are ignored.  The results use the positions read after the wait.
__device__ __forceinline__ int64_t hint_load(const int64_t* p) {
  int64_t v;
  asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

// Prefetches the 128-byte lines of [p, p + bytes) into L2 (one line per thread
// of the CTA; every CTA stages the whole table, so every CTA asks for it).
__device__ __forceinline__ void prefetch_lines(const void* p, int64_t bytes) {
  const char* base = static_cast<const char*>(p);
  for (int64_t off = int64_t(threadIdx.x) * 128; off < bytes; off += int64_t(blockDim.x) * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
}

__device__ __forceinline__ void prefetch_cos_sin_row(const float* cache, int64_t max_position, int64_t pos_hint,
                                                     int part) {
  if (part < 2 && pos_hint >= 0 && pos_hint < max_position)  // part 0: cos line, part 1: sin line
    asm volatile("prefetch.global.L2 [%0];" ::"l"(cache + pos_hint * kRopeDim + part * kHalf));
}

// ---------------------------------------------------------------------------
// Loads / stores.  kVec: 16-byte vectors (bases 16-byte aligned, strides a
// multiple of 8 elements); otherwise 2-byte scalars with the same results.
// ---------------------------------------------------------------------------
template <bool kVec>
struct Io;

template <>
struct Io<true> {
  static __device__ __forceinline__ uint4 load8(const uint16_t* p) {
    return *reinterpret_cast<const uint4*>(p);
  }
  static __device__ __forceinline__ void store8(uint16_t* p, const uint4& v) {
    *reinterpret_cast<uint4*>(p) = v;
  }
  static __device__ __forceinline__ void load_cos_sin(const float* row, int part, CosSin& cs) {
    const float4* c = reinterpret_cast<const float4*>(row + part * kLanes);
    const float4* s = reinterpret_cast<const float4*>(row + kHalf + part * kLanes);
    const float4 c0 = __ldg(c), c1 = __ldg(c + 1), s0 = __ldg(s), s1 = __ldg(s + 1);
    cs.c[0] = c0.x; cs.c[1] = c0.y; cs.c[2] = c0.z; cs.c[3] = c0.w;
    cs.c[4] = c1.x; cs.c[5] = c1.y; cs.c[6] = c1.z; cs.c[7] = c1.w;
    cs.s[0] = s0.x; cs.s[1] = s0.y; cs.s[2] = s0.z; cs.s[3] = s0.w;
    cs.s[4] = s1.x; cs.s[5] = s1.y; cs.s[6] = s1.z; cs.s[7] = s1.w;
  }
};

template <>
struct Io<false> {
  static __device__ __forceinline__ uint4 load8(const uint16_t* p) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = uint32_t(p[2 * i]) | (uint32_t(p[2 * i + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  static __device__ __forceinline__ void store8(uint16_t* p, const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[2 * i] = uint16_t(w[i] & 0xffffu);
      p[2 * i + 1] = uint16_t(w[i] >> 16);
    }
  }
  static __device__ __forceinline__ void load_cos_sin(const float* row, int part, CosSin& cs) {
#pragma unroll
    for (int i = 0; i < kLanes; ++i) {
      cs.c[i] = __ldg(row + part * kLanes + i);
      cs.s[i] = __ldg(row + kHalf + part * kLanes + i);
    }
  }
};

// ---------------------------------------------------------------------------
// Arithmetic: one rotated pair per lane, FP32 with separate roundings.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // RNE, lo in the low half
  return *reinterpret_cast<const uint32_t*>(&v);
}

// x1 (8 lanes) and x2 (the matching 8 lanes) are rotated in place.
__device__ __forceinline__ void rotate8(uint4& x1, uint4& x2, const CosSin& cs) {
  uint32_t a[4] = {x1.x, x1.y, x1.z, x1.w};
  uint32_t b[4] = {x2.x, x2.y, x2.z, x2.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a0 = bf16_lo(a[i]), a1 = bf16_hi(a[i]);
    const float b0 = bf16_lo(b[i]), b1 = bf16_hi(b[i]);
    const float c0 = cs.c[2 * i], c1 = cs.c[2 * i + 1];
    const float s0 = cs.s[2 * i], s1 = cs.s[2 * i + 1];
    const float o0 = __fsub_rn(__fmul_rn(a0, c0), __fmul_rn(b0, s0));
    const float o1 = __fsub_rn(__fmul_rn(a1, c1), __fmul_rn(b1, s1));
    const float p0 = __fadd_rn(__fmul_rn(a0, s0), __fmul_rn(b0, c0));
    const float p1 = __fadd_rn(__fmul_rn(a1, s1), __fmul_rn(b1, c1));
    a[i] = pack_bf16x2(o0, o1);
    b[i] = pack_bf16x2(p0, p1);
  }
  x1 = make_uint4(a[0], a[1], a[2], a[3]);
  x2 = make_uint4(b[0], b[1], b[2], b[3]);
}

// ---------------------------------------------------------------------------
// Row pieces.  Slices<NH> holds NH heads (head stride 256 lanes) of one row for
// one part; its loads are issued by load() and consumed by rotate_store(), so
// callers can put the position / cache gather and the tile check in between.
// ---------------------------------------------------------------------------
template <bool kVec, int NH>
struct Slices {
  uint16_t* base;
  uint4 x1[NH], x2[NH];
  __device__ __forceinline__ void load(uint16_t* row, int part) {
    base = row + kRopeLane0 + part * kLanes;
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      x1[h] = Io<kVec>::load8(base + h * kHeadDim);
      x2[h] = Io<kVec>::load8(base + h * kHeadDim + kHalf);
    }
  }
  __device__ __forceinline__ void rotate_store(const CosSin& cs) {
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      rotate8(x1[h], x2[h], cs);
      Io<kVec>::store8(base + h * kHeadDim, x1[h]);
      Io<kVec>::store8(base + h * kHeadDim + kHalf, x2[h]);
    }
  }
};

// Gathers this part's cos/sin at `pos`; false when pos is outside the cache
// (nothing is read then).
template <bool kVec>
__device__ __forceinline__ bool gather_cos_sin(const RopeArgs& a, int64_t pos, int part, CosSin& cs) {
  if (pos < 0 || pos >= a.max_position) return false;
  Io<kVec>::load_cos_sin(a.cache + pos * kRopeDim, part, cs);
  return true;
}

// Loads whose place in the instruction stream is pinned (volatile asm), so
// they are issued where written — before the checks that decide whether
// their values are used.
__device__ __forceinline__ int64_t pinned_load_s64(const int64_t* p) {
  int64_t v;
  asm volatile("ld.global.nc.s64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 pinned_load_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Cos/sin gather for a row whose position is known only at the end of a
// dependent chain (position, or last_index -> position).  issue() starts, AFTER
// the dependency wait, the loads that the chain would make if its values
// equalled the hints read before the wait: positions[src_hint] and the cos/sin
// row at pos_hint.  position() / finish() keep those values when the real src
// and position equal the hints — the loads then read exactly the data the
// chain would have read — and fall back to the real chain otherwise.  So the
// common case costs one round trip instead of two or three, and every result
// is the one the plain chain gives.  Hints < 0 disable the speculation.
template <bool kVec>
struct RowGather {
  CosSin cs;
  int64_t src_hint = -1, pos_hint = -1, pos_spec = 0;
  bool src_spec = false, row_spec = false;
  __device__ __forceinline__ void issue(const RopeArgs& a, int64_t sh, int64_t ph, int part) {
    src_hint = sh;
    pos_hint = ph;
    src_spec = sh >= 0 && sh < a.n_tokens;
    if (src_spec) pos_spec = pinned_load_s64(a.positions + sh);
    row_spec = kVec && ph >= 0 && ph < a.max_position;
    if (row_spec) {
      const float* row = a.cache + ph * kRopeDim;
      const float4 c0 = pinned_load_f4(row + part * kLanes), c1 = pinned_load_f4(row + part * kLanes + 4);
      const float4 s0 = pinned_load_f4(row + kHalf + part * kLanes), s1 = pinned_load_f4(row + kHalf + part * kLanes + 4);
      cs.c[0] = c0.x; cs.c[1] = c0.y; cs.c[2] = c0.z; cs.c[3] = c0.w;
      cs.c[4] = c1.x; cs.c[5] = c1.y; cs.c[6] = c1.z; cs.c[7] = c1.w;
      cs.s[0] = s0.x; cs.s[1] = s0.y; cs.s[2] = s0.z; cs.s[3] = s0.w;
      cs.s[4] = s1.x; cs.s[5] = s1.y; cs.s[6] = s1.z; cs.s[7] = s1.w;
    }
  }
  // Position of the row for the real src (already checked to be in [0, N)).
  __device__ __forceinline__ int64_t position(const RopeArgs& a, int64_t src) const {
    return src_spec && src == src_hint ? pos_spec : __ldg(a.positions + src);
  }
  // Cos/sin for the real position; false when it is outside the cache.
  __device__ __forceinline__ bool finish(const RopeArgs& a, int64_t pos, int part) {
    if (row_spec && pos == pos_hint) return true;
    return gather_cos_sin<kVec>(a, pos, part, cs);
  }
};

// ---------------------------------------------------------------------------
// Token sources.  Tile semantics are the reference kernels'
// (bench_welmv4_inplace_rope_npu.py:700-718, 856-867): tile i covers
// [starts[i], starts[i] + min(64, starts[i+1] - starts[i])).
//   kDense:     has_segments = 0; token = slot, slots = min(N, 64 * tiles).
//   kTileTable: has_segments = 1 with at most kTableCap table entries;
//               items are tokens 0..N-1 in order, so every load is issued at
//               once, and a token is rotated iff a tile covers it (ordinary:
//               binary search of the table staged in shared memory; mirror:
//               a warp-cooperative search of the global table while the
//               loads fly).  Exact for any non-decreasing table; other tables
//               are flagged.
//   kTileSlots: has_segments = 1 with a large table; 64 slots per tile,
//               token = starts[tile] + slot (one extra dependent load).
// ---------------------------------------------------------------------------
enum class Source { kDense, kTileTable, kTileSlots };

constexpr int kTableCap = 2048;  // staged table entries (8 KB of shared memory)
// warp_table_covers searches two levels of at most 32 x 64 entries
static_assert(kTableCap <= 32 * 64, "the warp search covers at most 2048 table entries");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Starts copying tile_starts[0..n) into shared memory (4-byte cp.async; the
// table is only 4-byte aligned).
__device__ __forceinline__ void stage_table_async(int32_t* s_tab, const int32_t* g_tab, int n) {
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(s_tab + j)), "l"(g_tab + j)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void stage_table_wait() {
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
}

// Whether a non-decreasing tile table rotates token t: the last tile starting
// at or before t must hold t within its first 64 tokens.
__device__ __forceinline__ bool table_covers(const int32_t* s_tab, int num_tiles, int64_t t) {
  int lo = 0, hi = num_tiles + 1;  // first entry greater than t
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (s_tab[mid] <= t) lo = mid + 1; else hi = mid;
  }
  const int i = lo - 1;
  return i >= 0 && i < num_tiles && t - s_tab[i] < kTile;
}

// Warp-cooperative coverage test on the global tile table (read-only path;
// its lines were prefetched into L2 in the PDL window and are read only after
// the wait): a 32-way ballot search finds the last entry at or before the
// warp's first token t_ref in two rounds of parallel loads (instead of
// log2(T) dependent ones), then each lane steps forward to its own token
// t >= t_ref.  Same answer as table_covers for every non-decreasing table;
// for other tables (flagged by the check items) the answer is arbitrary, but
// every index read stays in [0, num_tiles].  All 32 lanes must call it.
__device__ __forceinline__ bool warp_table_covers(const int32_t* g_tab, int num_tiles, int64_t t_ref, int64_t t) {
  constexpr unsigned kAll = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int entries = num_tiles + 1;
  const int stride = (entries + 31) >> 5;
  const int e0 = lane * stride;
  const int blocks = __popc(__ballot_sync(kAll, e0 < entries && __ldg(g_tab + e0) <= t_ref));
  int i = -1;
  if (blocks > 0) {  // warp-uniform
    const int base = (blocks - 1) * stride;
    const int e1 = base + lane, e2 = base + 32 + lane;
    const bool le1 = lane < stride && e1 < entries && __ldg(g_tab + e1) <= t_ref;
    const bool le2 = 32 + lane < stride && e2 < entries && __ldg(g_tab + e2) <= t_ref;
    i = base + __popc(__ballot_sync(kAll, le1)) + __popc(__ballot_sync(kAll, le2)) - 1;
  }
  while (i < num_tiles && __ldg(g_tab + i + 1) <= t) ++i;
  return i >= 0 && i < num_tiles && t - __ldg(g_tab + i) < kTile;
}

// Tile validation item: flags a tile that starts below 0, ends past N, runs
// backwards or holds more than 64 tokens.
__device__ __forceinline__ void check_tile(const RopeArgs& a, int tile) {
  const int64_t begin = __ldg(a.tile_starts + tile);
  const int64_t end = __ldg(a.tile_starts + tile + 1);
  if (begin < 0 || end < begin || end - begin > kTile || end > a.n_tokens)
    raise_status(a.status, WELM_ROPE_DEV_BAD_TILE);
}

// Slot -> token for kDense and kTileSlots.  False when the slot is empty (a
// short tile's tail) or its token is outside [0, N) (never touched).
template <Source kSrc>
__device__ __forceinline__ bool slot_token(const RopeArgs& a, int slot, int part, int64_t& tok) {
  if (kSrc == Source::kDense) {
    tok = slot;
    return true;
  }
  const int tile = slot / kTile;
  const int j = slot - tile * kTile;
  const int64_t begin = __ldg(a.tile_starts + tile);
  const int64_t end = __ldg(a.tile_starts + tile + 1);
  if (j == 0 && part == 0 && (begin < 0 || end < begin || end - begin > kTile || end > a.n_tokens))
    raise_status(a.status, WELM_ROPE_DEV_BAD_TILE);
  const int64_t count = end - begin < kTile ? end - begin : kTile;
  if (j >= count) return false;
  tok = begin + j;
  return tok >= 0 && tok < a.n_tokens;
}

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
// KV-mirror prefill.  Items [0, q_items) are the BS Q rows (6 heads at
// positions[last_index[b]], bench_welmv4_inplace_rope_npu.py:839-854); the
// next k_items are K tokens (1 head at positions[t],
// bench_welmv4_inplace_rope_npu.py:856-919).  Q rows and K rows are disjoint
// tensors, so the two phases need no ordering.  A Q row's data loads are
// issued before its last_index -> position -> cache chain.
// ---------------------------------------------------------------------------
// g has been issued (with or without hints) before src is known.
template <bool kVec>
__device__ __forceinline__ void finish_q_row(const RopeArgs& a, Slices<kVec, kQHeads>& qx, int64_t src,
                                             RowGather<kVec>& g, int part) {
  if (src < 0 || src >= a.n_tokens) {
    if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_LAST_INDEX);
    return;
  }
  if (!g.finish(a, g.position(a, src), part)) {
    if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    return;
  }
  qx.rotate_store(g.cs);
}

template <bool kVec>
__device__ __forceinline__ void mirror_q_row(const RopeArgs& a, int b, int part, int64_t src_hint,
                                             int64_t pos_hint) {
  Slices<kVec, kQHeads> qx;
  qx.load(a.q + int64_t(b) * a.q_stride, part);
  const int64_t src = __ldg(a.last_index + b);
  RowGather<kVec> g;
  g.issue(a, src_hint, pos_hint, part);
  finish_q_row<kVec>(a, qx, src, g, part);
}

template <bool kVec>
__device__ __forceinline__ void mirror_k_token(const RopeArgs& a, int64_t tok, int part, int64_t pos_hint) {
  const int64_t pos = __ldg(a.positions + tok);
  Slices<kVec, 1> kx;
  kx.load(a.k + tok * a.k_stride, part);
  RowGather<kVec> g;
  g.issue(a, -1, pos_hint, part);
  if (!g.finish(a, pos, part)) {
    if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    return;
  }
  kx.rotate_store(g.cs);
}

// At most 128 registers: 4 CTAs per SM keep a 16384-token launch in one wave.
template <bool kVec, Source kSrc>
__global__ void __launch_bounds__(kBlock, 4) rope_mirror_kernel(const RopeArgs a) {
  // warm the first item's cos/sin row (Q rows: through a last_index hint)
  const int item0 = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t src_hint = -1, pos_hint = -1;
  if (kSrc == Source::kTileTable) prefetch_lines(a.tile_starts, int64_t(a.num_tiles + 1) * sizeof(int32_t));
  if (item0 < a.q_items) {
    src_hint = hint_load(a.last_index + (item0 >> kPartShift));
    if (src_hint >= 0 && src_hint < a.n_tokens) pos_hint = hint_load(a.positions + src_hint);
  } else if (kSrc != Source::kTileSlots && item0 - a.q_items < a.k_items) {
    pos_hint = hint_load(a.positions + ((item0 - a.q_items) >> kPartShift));
  }
  prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, item0 & (kParts - 1));
  pdl_enter();
  if constexpr (kSrc == Source::kTileTable) {
    // One item per thread: Q rows, then tokens [0, k_items / 4), then one
    // check per tile.  Phase 1 issues the loads of whatever item the thread
    // owns; the coverage search (warp-uniform, no barrier) runs while they
    // fly; phase 2 finishes the item.
    const int item = blockIdx.x * blockDim.x + threadIdx.x;
    const int part = item & (kParts - 1);
    const bool is_q = item < a.q_items;
    const int k_item = item - a.q_items;
    const bool is_token = !is_q && k_item < a.k_items;
    const int64_t tok = is_token ? (k_item >> kPartShift) : 0;
    Slices<kVec, kQHeads> qx;
    Slices<kVec, 1> kx;
    RowGather<kVec> g;
    int64_t src = 0, pos = 0;
    if (is_q) {
      qx.load(a.q + int64_t(item >> kPartShift) * a.q_stride, part);
      src = __ldg(a.last_index + (item >> kPartShift));
      g.issue(a, src_hint, pos_hint, part);
    } else if (is_token) {
      pos = __ldg(a.positions + tok);
      kx.load(a.k + tok * a.k_stride, part);
      g.issue(a, -1, pos_hint, part);
    } else if (k_item - a.k_items < a.num_tiles) {
      check_tile(a, k_item - a.k_items);
    }
    // the coverage search runs while the loads above are in flight
    const int first_k = max(item & ~31, a.q_items) - a.q_items;  // the warp's first K item
    const int64_t t_ref = first_k < a.k_items ? int64_t(first_k >> kPartShift) : 0;
    const bool covered = warp_table_covers(a.tile_starts, a.num_tiles, t_ref, is_token ? tok : t_ref);
    if (is_q) {
      finish_q_row<kVec>(a, qx, src, g, part);
    } else if (is_token && covered) {
      if (g.finish(a, pos, part)) {
        kx.rotate_store(g.cs);
      } else if (part == 0) {
        raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
      }
    }
  } else {
    const int stride = gridDim.x * blockDim.x;
    const int total = a.q_items + a.k_items;
    for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < total; item += stride) {
      const int part = item & (kParts - 1);
      const bool first = item == item0;
      if (item < a.q_items) {
        mirror_q_row<kVec>(a, item >> kPartShift, part, first ? src_hint : -1, first ? pos_hint : -1);
      } else {
        int64_t tok;
        if (slot_token<kSrc>(a, (item - a.q_items) >> kPartShift, part, tok))
          mirror_k_token<kVec>(a, tok, part, first ? pos_hint : -1);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// KV mirror from request lengths.  Every CTA stages the BS lengths into shared
// memory (cp.async) while its K-token loads and cache gathers fly; after the
// one barrier each warp derives what it needs with shuffles, without further
// CTA-wide synchronisation: K token t is rotated iff t < sum(lengths), Q row
// r uses src = end_r - 1 with end_r = lengths[0] + ... + lengths[r].  One
// item per thread: Q rows, then K tokens.
// ---------------------------------------------------------------------------
constexpr int kLensCap = WELM_ROPE_LENS_MAX_BATCH;

// Warp-cooperative prefix over the staged lengths (negative entries count as
// 0): returns the total and, for `row` in [0, n), end_row = s[0] + ... +
// s[row].  Every lane of the warp must call it (it shuffles).
__device__ __forceinline__ int64_t warp_request_ends(const int64_t* s, int n, int row, int64_t& end_row,
                                                     bool& negative) {
  const int lane = threadIdx.x & 31;
  const int chunk = (n + 31) >> 5;
  const int lo = min(n, lane * chunk), hi = min(n, lo + chunk);
  int64_t part_sum = 0;
  for (int i = lo; i < hi; ++i) {
    const int64_t v = s[i];
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
      const int64_t v = s[i];
      end_row += v > 0 ? v : 0;
    }
  }
  return total;
}

// At most 128 registers, so 4 CTAs fit per SM and a 16384-token launch
// (516 CTAs) stays resident in one wave on 148 SMs.
template <bool kVec>
__global__ void __launch_bounds__(kBlock, 4) rope_mirror_lens_kernel(const RopeArgs a, const int64_t* lens, int batch) {
  extern __shared__ int64_t s_len[];
  // K tokens: warm the first item's cos/sin row; the lengths every CTA stages
  int64_t pos_hint = -1;
  prefetch_lines(lens, int64_t(batch) * sizeof(int64_t));
  {
    const int item0 = blockIdx.x * blockDim.x + threadIdx.x;
    if (item0 >= a.q_items && item0 - a.q_items < a.k_items) {
      pos_hint = hint_load(a.positions + ((item0 - a.q_items) >> kPartShift));
      prefetch_cos_sin_row(a.cache, a.max_position, pos_hint, item0 & (kParts - 1));
    }
  }
  pdl_enter();
  for (int j = threadIdx.x; j < batch; j += blockDim.x) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(s_len + j)), "l"(lens + j) : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  const int part = item & (kParts - 1);
  const bool is_q = item < a.q_items;
  const int k_item = item - a.q_items;
  const bool is_token = !is_q && k_item < a.k_items;
  const int64_t tok = is_token ? (k_item >> kPartShift) : 0;
  Slices<kVec, kQHeads> qx;
  Slices<kVec, 1> kx;
  RowGather<kVec> g;
  bool pos_ok = false;
  if (is_q) {
    qx.load(a.q + int64_t(item >> kPartShift) * a.q_stride, part);
  } else if (is_token) {
    const int64_t pos = __ldg(a.positions + tok);
    kx.load(a.k + tok * a.k_stride, part);
    g.issue(a, -1, pos_hint, part);
    pos_ok = g.finish(a, pos, part);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  int64_t end_row = 0;
  bool negative = false;
  const int64_t total = warp_request_ends(s_len, batch, is_q ? (item >> kPartShift) : -1, end_row, negative);
  if (is_q) {
    finish_q_row<kVec>(a, qx, end_row - 1, g, part);  // g was not issued: plain chain
  } else if (is_token && tok < total) {
    if (pos_ok) {
      kx.rotate_store(g.cs);
    } else if (part == 0) {
      raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
    }
  }
  if (negative && blockIdx.x == 0 && threadIdx.x == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_LENGTH);
}

// ---------------------------------------------------------------------------
// KV mirror fused with the paged KV-cache write and the Q last-row extraction.
// Items: Q rows first — one per (request, head, part), 24 per row — then K
// tokens, one per (token, part).  A thread owns 48 lanes of the 192 copied
// lanes (six 16-byte chunks) plus its 8 x1 / 8 x2 rotated lanes of a head; a
// K thread also copies 64 lanes of V (eight 16-byte chunks).
// ---------------------------------------------------------------------------
struct KvArgs {
  const uint16_t* q;
  uint16_t* q_out;
  const uint16_t* k;
  const uint16_t* v;
  const int64_t* positions;
  const float* cache;
  const int64_t* last_index;
  const int64_t* slots;
  uint16_t* key_cache;
  uint16_t* value_cache;
  int64_t q_stride, q_out_stride, k_stride, v_stride, slot_stride;
  int64_t num_slots, n_tokens, max_position;
  int32_t* status;
  int32_t q_items, k_items;
};

constexpr int kNope = kRopeLane0;          // 192 copied lanes per head
constexpr int kNopeChunks = kNope / kParts / 8;  // 6 chunks of 8 lanes per thread
constexpr int kVChunks = kHeadDim / kParts / 8;  // 8 chunks of 8 lanes per thread

// One head of one row: this part's copied lanes and rotated lanes.
struct HeadPiece {
  uint4 nope[kNopeChunks];
  uint4 x1, x2;
  __device__ __forceinline__ void load(const uint16_t* head, int part) {
    const uint16_t* n = head + part * (kNope / kParts);
#pragma unroll
    for (int c = 0; c < kNopeChunks; ++c) nope[c] = *reinterpret_cast<const uint4*>(n + 8 * c);
    x1 = *reinterpret_cast<const uint4*>(head + kRopeLane0 + part * kLanes);
    x2 = *reinterpret_cast<const uint4*>(head + kRopeLane0 + kHalf + part * kLanes);
  }
  __device__ __forceinline__ void store(uint16_t* head, int part) const {
    uint16_t* n = head + part * (kNope / kParts);
#pragma unroll
    for (int c = 0; c < kNopeChunks; ++c) *reinterpret_cast<uint4*>(n + 8 * c) = nope[c];
    *reinterpret_cast<uint4*>(head + kRopeLane0 + part * kLanes) = x1;
    *reinterpret_cast<uint4*>(head + kRopeLane0 + kHalf + part * kLanes) = x2;
  }
};

__global__ void __launch_bounds__(kBlock) rope_mirror_kv_write_kernel(const KvArgs a) {
  {  // warm the first item's cos/sin row (Q rows: through a last_index hint)
    const int item0 = blockIdx.x * blockDim.x + threadIdx.x;
    const int part0 = item0 & (kParts - 1);
    if (item0 < a.q_items) {
      const int64_t src = hint_load(a.last_index + item0 / (kQHeads * kParts));
      if (src >= 0 && src < a.n_tokens)
        prefetch_cos_sin_row(a.cache, a.max_position, hint_load(a.positions + src), part0);
    } else if (item0 - a.q_items < a.k_items) {
      prefetch_cos_sin_row(a.cache, a.max_position, hint_load(a.positions + ((item0 - a.q_items) >> kPartShift)),
                           part0);
    }
  }
  pdl_enter();
  const int stride = gridDim.x * blockDim.x;
  const int total = a.q_items + a.k_items;
  for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < total; item += stride) {
    const int part = item & (kParts - 1);
    if (item < a.q_items) {
      const int b = item / (kQHeads * kParts);
      const int h = (item >> kPartShift) % kQHeads;
      const int64_t src = __ldg(a.last_index + b);
      if (src < 0 || src >= a.n_tokens) {
        if (part == 0 && h == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_LAST_INDEX);
        continue;
      }
      const int64_t pos = __ldg(a.positions + src);
      HeadPiece piece;
      piece.load(a.q + src * a.q_stride + h * kHeadDim, part);
      CosSin cs;
      if (pos < 0 || pos >= a.max_position) {
        if (part == 0 && h == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
        continue;
      }
      Io<true>::load_cos_sin(a.cache + pos * kRopeDim, part, cs);
      rotate8(piece.x1, piece.x2, cs);
      piece.store(a.q_out + int64_t(b) * a.q_out_stride + h * kHeadDim, part);
    } else {
      const int64_t tok = (item - a.q_items) >> kPartShift;
      const int64_t slot = __ldg(a.slots + tok);
      const int64_t pos = __ldg(a.positions + tok);
      HeadPiece kp;
      kp.load(a.k + tok * a.k_stride, part);
      uint4 vv[kVChunks];
      const bool with_v = a.v != nullptr && a.value_cache != nullptr;
      if (with_v) {
        const uint16_t* vsrc = a.v + tok * a.v_stride + part * (kHeadDim / kParts);
#pragma unroll
        for (int c = 0; c < kVChunks; ++c) vv[c] = *reinterpret_cast<const uint4*>(vsrc + 8 * c);
      }
      if (pos < 0 || pos >= a.max_position) {
        if (part == 0 && slot >= 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
        continue;
      }
      CosSin cs;
      Io<true>::load_cos_sin(a.cache + pos * kRopeDim, part, cs);
      if (slot < 0) continue;  // padding token
      if (slot >= a.num_slots) {
        if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_SLOT);
        continue;
      }
      rotate8(kp.x1, kp.x2, cs);
      kp.store(a.key_cache + slot * a.slot_stride, part);
      if (with_v) {
        uint16_t* vdst = a.value_cache + slot * a.slot_stride + part * (kHeadDim / kParts);
#pragma unroll
        for (int c = 0; c < kVChunks; ++c) *reinterpret_cast<uint4*>(vdst + 8 * c) = vv[c];
      }
    }
  }
}

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

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
constexpr int64_t kMaxItems = int64_t(1) << 30;  // item indices stay in int32

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_sm_count() {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  if (dev < kMaxDevices) {
    const int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < kMaxDevices) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

// Grid for `items` work items of a grid-stride kernel: enough CTAs for one
// item per thread, capped at 16 CTAs of 128 threads per SM (more than these
// kernels keep resident) so larger inputs loop.
unsigned grid_for(int64_t items) {
  const int sms = current_sm_count();
  const int64_t need = (items + kBlock - 1) / kBlock;
  const int64_t cap = sms > 0 ? int64_t(sms) * 16 : need;
  return unsigned(need < cap ? need : cap);
}

// Launches carry the programmatic-stream-serialization attribute (PDL) unless
// the environment sets WELM_ROPE_PDL=0: the grid may be scheduled while the
// previous kernel in the stream drains, and waits in pdl_enter() before it
// touches memory.
bool pdl_enabled() {
  static const bool enabled = [] {
    const char* v = std::getenv("WELM_ROPE_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return enabled;
}

template <typename... Params, typename... Args>
int launch(void (*kernel)(Params...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    cudaGetLastError();  // clear the launch error so later calls start clean
    return WELM_ROPE_ERR_CUDA;
  }
  return WELM_ROPE_OK;
}

// How the token phase is laid out for one call (see Source).
struct Plan {
  Source src;
  int64_t token_items;  // items of the token phase
  int64_t check_items;  // tile validation items (kTileTable only)
};

Plan plan_tokens(int64_t has_segments, int64_t num_work_tiles, int64_t n_tokens) {
  if (!has_segments) {
    const int64_t covered = num_work_tiles * kTile;
    return {Source::kDense, (covered < n_tokens ? covered : n_tokens) * kParts, 0};
  }
  if (num_work_tiles == 0 || n_tokens == 0) return {Source::kTileSlots, 0, 0};
  if (num_work_tiles + 1 <= kTableCap) return {Source::kTileTable, n_tokens * kParts, num_work_tiles};
  return {Source::kTileSlots, num_work_tiles * kTile * kParts, 0};
}

template <typename Kernel>
int launch_plan(Kernel kernel, const Plan& plan, const RopeArgs& a, cudaStream_t stream, bool staged_table = true) {
  const int64_t total = int64_t(a.q_items) + plan.token_items + plan.check_items;
  if (plan.src == Source::kTileTable) {
    const size_t smem = staged_table ? (size_t(a.num_tiles + 1) * sizeof(int32_t) + 15) & ~size_t(15) : 0;
    return launch(kernel, unsigned((total + kBlock - 1) / kBlock), kBlock, smem, stream, a);
  }
  return launch(kernel, grid_for(total), kBlock, 0, stream, a);
}

template <bool kVec>
int launch_ordinary(const Plan& plan, const RopeArgs& a, cudaStream_t s) {
  switch (plan.src) {
    case Source::kDense: return launch_plan(rope_ordinary_kernel<kVec, Source::kDense>, plan, a, s);
    case Source::kTileTable: return launch_plan(rope_ordinary_kernel<kVec, Source::kTileTable>, plan, a, s);
    default: return launch_plan(rope_ordinary_kernel<kVec, Source::kTileSlots>, plan, a, s);
  }
}

template <bool kVec>
int launch_mirror(const Plan& plan, const RopeArgs& a, cudaStream_t s) {
  switch (plan.src) {
    case Source::kDense: return launch_plan(rope_mirror_kernel<kVec, Source::kDense>, plan, a, s);
    case Source::kTileTable: return launch_plan(rope_mirror_kernel<kVec, Source::kTileTable>, plan, a, s, false);
    default: return launch_plan(rope_mirror_kernel<kVec, Source::kTileSlots>, plan, a, s);
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

int welm_rope_abi_version(void) { return WELM_ROPE_ABI_VERSION; }

const char* welm_rope_status_string(int status) {
  switch (status) {
    case WELM_ROPE_OK: return "ok";
    case WELM_ROPE_ERR_NULL_POINTER: return "a required pointer is NULL";
    case WELM_ROPE_ERR_BAD_MODE: return "has_segments must be 0 or 1 (segmented mode needs segment_tile_starts)";
    case WELM_ROPE_ERR_BAD_SIZE: return "negative or too large size argument";
    case WELM_ROPE_ERR_BAD_STRIDE: return "token stride makes rows overlap";
    case WELM_ROPE_ERR_CAPACITY: return "output buffer too small";
    case WELM_ROPE_ERR_CUDA: return "CUDA launch failed";
    case WELM_ROPE_ERR_TOO_MANY_TOKENS:
      return "n_tokens exceeds WELM_ROPE_STATIC_MAX_TOKENS (2048) of the static staging area; split the batch";
    case WELM_ROPE_ERR_NOT_MAPPED:
      return "a host buffer is not page-locked and mapped for the device (pin it, e.g. cudaHostAlloc or pin_memory)";
    default: return "unknown welm_rope status";
  }
}

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
  if (rows * kParts + plan.token_items + plan.check_items > kMaxItems) return WELM_ROPE_ERR_BAD_SIZE;
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
  return vec ? launch_mirror<true>(plan, a, s) : launch_mirror<false>(plan, a, s);
}

int welm_rope_mirror_from_lens(void* q, void* k, const int64_t* positions, const float* cos_sin_cache,
                               const int64_t* seq_lens, int64_t n_tokens, int64_t batch_size,
                               int64_t q_token_stride, int64_t k_token_stride, int64_t max_position,
                               int32_t* device_status, void* stream) {
  if (n_tokens < 0 || batch_size < 0 || max_position < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (batch_size > kLensCap || n_tokens > kMaxItems / kParts - kLensCap) return WELM_ROPE_ERR_BAD_SIZE;
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
  a.q_items = int32_t(batch_size * kParts);
  a.k_items = int32_t(n_tokens * kParts);
  const bool vec = aligned16(q) && aligned16(k) && aligned16(cos_sin_cache) &&
                   (batch_size <= 1 || q_token_stride % 8 == 0) && (n_tokens <= 1 || k_token_stride % 8 == 0);
  const int64_t total = int64_t(a.q_items) + a.k_items;
  const unsigned grid = unsigned((total + kBlock - 1) / kBlock);
  const size_t smem = size_t(batch_size) * sizeof(int64_t);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int b = int(batch_size);
  return vec ? launch(rope_mirror_lens_kernel<true>, grid, kBlock, smem, s, a, seq_lens, b)
             : launch(rope_mirror_lens_kernel<false>, grid, kBlock, smem, s, a, seq_lens, b);
}

int welm_rope_mirror_kv_write(const void* q, void* q_out, const void* k, const void* v,
                              const int64_t* positions, const float* cos_sin_cache, const int64_t* last_index,
                              const int64_t* slot_mapping, void* key_cache, void* value_cache, int64_t n_tokens,
                              int64_t batch_size, int64_t q_token_stride, int64_t q_out_token_stride,
                              int64_t k_token_stride, int64_t v_token_stride, int64_t cache_slot_stride,
                              int64_t num_slots, int64_t max_position, int32_t* device_status, void* stream) {
  if (n_tokens < 0 || batch_size < 0 || num_slots < 0 || max_position < 0) return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens > kMaxItems / kParts || batch_size > kMaxItems / (kParts * kQHeads) ||
      n_tokens * kParts + batch_size * kParts * kQHeads > kMaxItems)
    return WELM_ROPE_ERR_BAD_SIZE;
  const int64_t rows = n_tokens > 0 ? batch_size : 0;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!k || !positions || !cos_sin_cache || !slot_mapping || !key_cache) return WELM_ROPE_ERR_NULL_POINTER;
  if (rows > 0 && (!q || !q_out || !last_index)) return WELM_ROPE_ERR_NULL_POINTER;
  if ((v == nullptr) != (value_cache == nullptr)) return WELM_ROPE_ERR_NULL_POINTER;
  const int64_t row = kQHeads * kHeadDim;
  if ((rows > 0 && (q_token_stride < row || q_out_token_stride < row)) || (n_tokens > 1 && k_token_stride < kHeadDim) ||
      (v && n_tokens > 1 && v_token_stride < kHeadDim) || (num_slots > 1 && cache_slot_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  const bool aligned = aligned16(k) && aligned16(cos_sin_cache) && aligned16(key_cache) &&
                       (!v || (aligned16(v) && aligned16(value_cache) && v_token_stride % 8 == 0)) &&
                       (rows == 0 || (aligned16(q) && aligned16(q_out) && q_token_stride % 8 == 0 &&
                                      q_out_token_stride % 8 == 0)) &&
                       k_token_stride % 8 == 0 && cache_slot_stride % 8 == 0;
  if (!aligned) return WELM_ROPE_ERR_BAD_STRIDE;
  KvArgs a{};
  a.q = static_cast<const uint16_t*>(q);
  a.q_out = static_cast<uint16_t*>(q_out);
  a.k = static_cast<const uint16_t*>(k);
  a.v = static_cast<const uint16_t*>(v);
  a.positions = positions;
  a.cache = cos_sin_cache;
  a.last_index = last_index;
  a.slots = slot_mapping;
  a.key_cache = static_cast<uint16_t*>(key_cache);
  a.value_cache = static_cast<uint16_t*>(value_cache);
  a.q_stride = q_token_stride;
  a.q_out_stride = q_out_token_stride;
  a.k_stride = k_token_stride;
  a.v_stride = v_token_stride;
  a.slot_stride = cache_slot_stride;
  a.num_slots = num_slots;
  a.n_tokens = n_tokens;
  a.max_position = max_position;
  a.status = device_status;
  a.q_items = int32_t(rows * kQHeads * kParts);
  a.k_items = int32_t(n_tokens * kParts);
  const int64_t total = int64_t(a.q_items) + a.k_items;
  return launch(rope_mirror_kv_write_kernel, grid_for(total), kBlock, 0, static_cast<cudaStream_t>(stream), a);
}

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
