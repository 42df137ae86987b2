// rope_device.cuh — device building blocks shared by every kernel family of
// the sm_100a in-place partial RoPE (constants, argument block, loads and
// stores, the rotation, row gathers, token sources and tile-table helpers).
// Everything lives in an anonymous namespace: each translation unit that
// includes this header gets its own copy of the inline helpers.
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
//   * a thread owns 8 lanes of x1 and the matching 8 lanes of x2 of a head,
//     i.e. two 16-byte vectors; 4 threads ("parts") cover a head's 128-byte
//     rope slice.  A work item is (row, part) with seven heads (the ordinary
//     streaming and segmented kernels: each cos/sin row then crosses HBM once
//     per token and is reused from registers for 1 K + 6 Q heads), or
//     (row, head, part) with one head (small ordinary launches and the KV
//     mirror, so more threads share a launch and fewer registers are held);
//   * the thread loads its 8 cos + 8 sin values once (four 16-byte loads);
//   * launches use programmatic dependent launch: before the dependency wait
//     a thread only reads hints and prefetches lines into L2, which cannot
//     change a result, and after it every data load of the item is issued
//     before the position-dependent cache load (or next to a speculative one
//     at the hinted position), so the position -> cache dependency overlaps
//     the data stream;
//   * 64-token work tiles are kept only as the segment / masking unit of the
//     reference's contract; positions are gathered per token, so no
//     contiguity inside a tile is assumed (bench_welmv4_inplace_rope_npu.py:714-715
//     assumes it, the oracle does not).

#ifndef WELM_ROPE_DEVICE_CUH_
#define WELM_ROPE_DEVICE_CUH_

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

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
constexpr int kHeadsPerToken = 1 + kQHeads;         // K head + 6 Q heads
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
  int32_t q_items;             // Q items (mirror): BS * kParts, or BS * 6 * kParts one head per item
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
// thread reads its position (and table entries or last_index) as hints only
// (ld.global.cg: served from L2, never allocated in L1, so no stale L1 line
// can answer the real loads made after the wait), and prefetches into L2 the
// lines its item will read: its rope slices and, in some kernels, the cos/sin
// row at the hinted position.  A prefetch cannot change a result — L2 is where
// writes of the previous grid land — and a stale or garbage hint only fetches
// a useless line; hints outside the cache are ignored.  The results use the
// values read after the wait.
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

__device__ __forceinline__ void prefetch_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Prefetches the rope-slice lines of one row of NH heads (head stride 256
// lanes) into L2, the row's four parts sharing the work: part p takes heads
// p, p + 4, ...  A head's 64 rope lanes are 128 bytes at byte offset 384 of
// the head: one 128-byte line when the row is 128-byte aligned (packed and
// fused-QKV layouts from an aligned base), else two, and then both are asked
// for.  Every address lies inside the row's rope slices.
template <int NH>
__device__ __forceinline__ void prefetch_row_slices(const uint16_t* row, int part) {
  const uint16_t* slice = row + kRopeLane0;
  const bool straddles = (reinterpret_cast<uintptr_t>(slice) & 127u) != 0;
#pragma unroll
  for (int h = part; h < NH; h += kParts) {
    prefetch_line(slice + h * kHeadDim);
    if (straddles) prefetch_line(slice + h * kHeadDim + kRopeDim - 1);
  }
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

// The rope-slice lines of token `tok` that part `part` prefetches: the
// token's seven slices (K, then Q heads 0..5) are shared out so that part p
// takes slices p and p + 4.  The scalar path's rows need not be 16-byte
// aligned, so it prefetches nothing.
template <bool kVec>
__device__ __forceinline__ void prefetch_token(const uint16_t* q, const uint16_t* k, int64_t q_stride,
                                               int64_t k_stride, int64_t tok, int part) {
  if (!kVec) return;
  const uint16_t* qrow = q + tok * q_stride;
  if (part == 0) {
    prefetch_row_slices<1>(k + tok * k_stride, 0);
    prefetch_row_slices<1>(qrow + 3 * kHeadDim, 0);
  } else {
    prefetch_row_slices<1>(qrow + (part - 1) * kHeadDim, 0);
    if (part < 3) prefetch_row_slices<1>(qrow + (part + 3) * kHeadDim, 0);
  }
}

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
//   kTileTable: (ordinary) has_segments = 1 with at most kTableCap table
//               entries; items are tokens 0..N-1 in order, so every load is
//               issued at once, and a token is rotated iff a tile covers it
//               (binary search of the table staged in shared memory).  Exact
//               for any non-decreasing table; other tables are flagged.
//   kTileSlots: has_segments = 1; 64 slots per tile, token = starts[tile] +
//               slot (one extra dependent load).  The ordinary kernel uses it
//               for large tables, the mirror for every table.  A table whose
//               tiles overlap (not non-decreasing, flagged) may reach a token
//               from two slots.
// ---------------------------------------------------------------------------
enum class Source { kDense, kTileTable, kTileSlots };

constexpr int kTableCap = 2048;  // table entries of the kTileTable source (8 KB when staged in shared memory)

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

// Reads a 32-bit value as a hint before the dependency wait (see hint_load).
__device__ __forceinline__ int32_t hint_load_s32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
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

}  // namespace

#endif  // WELM_ROPE_DEVICE_CUH_
