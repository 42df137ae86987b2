// rope_kv_write.cu — KV mirror fused with the Q last-row gather and the
// paged KV-cache store, and its C entry welm_rope_mirror_kv_write.

#include "rope_host.cuh"

namespace {

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
    const uint16_t* n = head + part * 8;
#pragma unroll
    for (int c = 0; c < kNopeChunks; ++c) nope[c] = *reinterpret_cast<const uint4*>(n + 8 * kParts * c);
    x1 = *reinterpret_cast<const uint4*>(head + kRopeLane0 + part * kLanes);
    x2 = *reinterpret_cast<const uint4*>(head + kRopeLane0 + kHalf + part * kLanes);
  }
  __device__ __forceinline__ void store(uint16_t* head, int part) const {
    uint16_t* n = head + part * 8;
#pragma unroll
    for (int c = 0; c < kNopeChunks; ++c) *reinterpret_cast<uint4*>(n + 8 * kParts * c) = nope[c];
    *reinterpret_cast<uint4*>(head + kRopeLane0 + part * kLanes) = x1;
    *reinterpret_cast<uint4*>(head + kRopeLane0 + kHalf + part * kLanes) = x2;
  }
};

__global__ void __launch_bounds__(kBlock) rope_mirror_kv_write_kernel(const KvArgs a) {
  // warm the first item's cos/sin row (Q rows: through a last_index hint);
  // a K token also keeps its position hint for the speculative gather below
  const int item0 = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t pos_hint = -1;
  // Before the wait the item's head rows are prefetched too, each part taking
  // one 128-byte line of every 512-byte head row it reads (Q: the source
  // row's head through the last_index hint; K: the K and V rows, and the
  // slot-mapping line).  Like every pre-wait access these only warm L2.
  // Measured on one B200 (graph replay, L2-cold sets, us per launch):
  // N=16384 BS=128 7.34 -> 6.38, N=8192 BS=8 4.56 -> 3.94, N=BS=128 unchanged.
  {
    const int part0 = item0 & (kParts - 1);
    if (item0 < a.q_items) {
      const int64_t src = hint_load(a.last_index + item0 / (kQHeads * kParts));
      if (src >= 0 && src < a.n_tokens) {
        prefetch_line(a.q + src * a.q_stride + ((item0 >> kPartShift) % kQHeads) * kHeadDim + part0 * 64);
        prefetch_cos_sin_row(a.cache, a.max_position, hint_load(a.positions + src), part0);
      }
    } else if (item0 - a.q_items < a.k_items) {
      const int64_t tok = (item0 - a.q_items) >> kPartShift;
      prefetch_line(a.k + tok * a.k_stride + part0 * 64);
      if (a.v != nullptr) prefetch_line(a.v + tok * a.v_stride + part0 * 64);
      if (part0 == 1 && (reinterpret_cast<uintptr_t>(a.slots + tok) & 127u) < sizeof(int64_t))
        prefetch_line(a.slots + tok);
      // the position hint feeds the speculative cos/sin loads after the wait;
      // it is not waited for here (prefetching its cos/sin lines before the
      // wait stalled late CTAs: N=8192 BS=8 4.18 us with it, 3.94 without)
      pos_hint = hint_load(a.positions + tok);
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
      // speculative cos/sin at the position hint, issued with the real loads
      CosSin cs;
      const bool spec = item == item0 && pos_hint >= 0 && pos_hint < a.max_position;
      if (spec) {
        const float* row = a.cache + pos_hint * kRopeDim;
        const float4 c0 = pinned_load_f4(row + part * kLanes), c1 = pinned_load_f4(row + part * kLanes + 4);
        const float4 s0 = pinned_load_f4(row + kHalf + part * kLanes);
        const float4 s1 = pinned_load_f4(row + kHalf + part * kLanes + 4);
        cs.c[0] = c0.x; cs.c[1] = c0.y; cs.c[2] = c0.z; cs.c[3] = c0.w;
        cs.c[4] = c1.x; cs.c[5] = c1.y; cs.c[6] = c1.z; cs.c[7] = c1.w;
        cs.s[0] = s0.x; cs.s[1] = s0.y; cs.s[2] = s0.z; cs.s[3] = s0.w;
        cs.s[4] = s1.x; cs.s[5] = s1.y; cs.s[6] = s1.z; cs.s[7] = s1.w;
      }
      const int64_t slot = __ldg(a.slots + tok);
      const int64_t pos = __ldg(a.positions + tok);
      HeadPiece kp;
      kp.load(a.k + tok * a.k_stride, part);
      uint4 vv[kVChunks];
      const bool with_v = a.v != nullptr && a.value_cache != nullptr;
      if (with_v) {
        const uint16_t* vsrc = a.v + tok * a.v_stride + part * 8;
#pragma unroll
        for (int c = 0; c < kVChunks; ++c) vv[c] = *reinterpret_cast<const uint4*>(vsrc + 8 * kParts * c);
      }
      if (pos < 0 || pos >= a.max_position) {
        if (part == 0 && slot >= 0) raise_status(a.status, WELM_ROPE_DEV_BAD_POSITION);
        continue;
      }
      if (!(spec && pos == pos_hint)) Io<true>::load_cos_sin(a.cache + pos * kRopeDim, part, cs);
      if (slot < 0) continue;  // padding token
      if (slot >= a.num_slots) {
        if (part == 0) raise_status(a.status, WELM_ROPE_DEV_BAD_SLOT);
        continue;
      }
      rotate8(kp.x1, kp.x2, cs);
      kp.store(a.key_cache + slot * a.slot_stride, part);
      if (with_v) {
        uint16_t* vdst = a.value_cache + slot * a.slot_stride + part * 8;
#pragma unroll
        for (int c = 0; c < kVChunks; ++c) *reinterpret_cast<uint4*>(vdst + 8 * kParts * c) = vv[c];
      }
    }
  }
}

}  // namespace

extern "C" {

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
  const LaunchShape shape = shape_for(total);
  return launch(rope_mirror_kv_write_kernel, shape.grid, shape.block, 0, static_cast<cudaStream_t>(stream), a);
}

}  // extern "C"
