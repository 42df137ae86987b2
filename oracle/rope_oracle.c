/*
 * rope_oracle.c — plain-C restatement of the reference's CPU algorithm for the
 * in-place partial RoPE.  TEST INFRASTRUCTURE ONLY: it checks the product
 * and is never part of it; tests/ and the C-ABI smoke program link it,
 * nothing else does.
 *
 * welm_oracle_apply restates apply_reference (bench_welmv4_inplace_rope_npu.py:
 * 1489-1505): every head of every row is copied, then lanes 192..223 (x1) and
 * 224..255 (x2) become bf16(x1*c - x2*s) and bf16(x1*s + x2*c) with c, s the
 * cos / sin halves of cache[pos].  Each product, the difference and the sum are
 * separate IEEE float operations (build with -ffp-contract=off so no FMA is
 * formed) and the BF16 conversion is round-to-nearest-even on the bit pattern,
 * as torch rounds float to bfloat16.  A NaN becomes a quiet NaN; its payload is
 * not pinned (torch's own CPU conversions differ: 0xFFFF on the vectorised
 * path, 0x7FC0 on the scalar one), so tests compare NaN lanes as NaN.
 *
 * welm_oracle_build_tiles restates the segmented tile builder inside
 * make_inputs (bench_welmv4_inplace_rope_npu.py:1439-1461).
 */
#include <stdint.h>
#include <string.h>

#define HEAD_DIM 256
#define ROPE_DIM 64
#define HALF_ROPE 32
#define ROPE_LANE0 (HEAD_DIM - ROPE_DIM)
#define TILE_TOKENS 64

static float bf16_to_float(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static uint16_t float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);  /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* out[r] = rope(data[r]) at rope_positions[r] for r < rows; rows are
 * `token_stride` elements apart in both buffers, `heads` heads of 256 lanes
 * each.  Returns the number of rows whose position was outside
 * [0, max_position) (those rows are copied unrotated). */
int64_t welm_oracle_apply(const uint16_t* data, uint16_t* out, int64_t rows, int64_t heads,
                          int64_t token_stride, const int64_t* rope_positions, const float* cache,
                          int64_t max_position) {
  int64_t bad = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* src = data + r * token_stride;
    uint16_t* dst = out + r * token_stride;
    memmove(dst, src, (size_t)(heads * HEAD_DIM) * sizeof(uint16_t));
    const int64_t pos = rope_positions[r];
    if (pos < 0 || pos >= max_position) {
      ++bad;
      continue;
    }
    const float* cs = cache + pos * ROPE_DIM;
    for (int64_t h = 0; h < heads; ++h) {
      const uint16_t* x = src + h * HEAD_DIM + ROPE_LANE0;
      uint16_t* y = dst + h * HEAD_DIM + ROPE_LANE0;
      for (int i = 0; i < HALF_ROPE; ++i) {
        const float x1 = bf16_to_float(x[i]);
        const float x2 = bf16_to_float(x[HALF_ROPE + i]);
        const float c = cs[i], s = cs[HALF_ROPE + i];
        const float x1c = x1 * c, x2s = x2 * s, x1s = x1 * s, x2c = x2 * c;
        y[i] = float_to_bf16(x1c - x2s);
        y[HALF_ROPE + i] = float_to_bf16(x1s + x2c);
      }
    }
  }
  return bad;
}

/* Tile starts of requests with lengths lens[0..bs): for each request its
 * 64-token tile starts, then the total.  Writes T + 1 entries (the caller
 * sizes `starts` with welm_oracle_count_tiles + 1) and returns T. */
int64_t welm_oracle_count_tiles(const int64_t* lens, int64_t bs) {
  int64_t tiles = 0;
  for (int64_t r = 0; r < bs; ++r) tiles += lens[r] > 0 ? (lens[r] + TILE_TOKENS - 1) / TILE_TOKENS : 0;
  return tiles;
}

int64_t welm_oracle_build_tiles(const int64_t* lens, int64_t bs, int32_t* starts) {
  int64_t token = 0, t = 0;
  for (int64_t r = 0; r < bs; ++r) {
    for (int64_t off = 0; off < lens[r]; off += TILE_TOKENS) starts[t++] = (int32_t)(token + off);
    if (lens[r] > 0) token += lens[r];
  }
  starts[t] = (int32_t)token;
  return t;
}
