/*
 * c_abi_smoke.c — a plain C99 caller of the library's C ABI (include/welm_rope.h),
 * the way a non-Python host binds it: no torch, only the CUDA runtime for
 * device memory.  Each entry's result is checked bit for bit against the C
 * oracle (oracle/rope_oracle.c).
 *
 * Covers: welm_rope_ordinary (dense and segmented), welm_rope_mirror
 * (segmented), welm_rope_build_tiles (device) against welm_rope_build_tiles_host
 * and the oracle builder, welm_rope_ordinary_mapped on page-locked host
 * buffers (and its refusal of pageable ones), host-side validation (a NULL
 * pointer is refused with its status string) and the device status word
 * staying zero.
 *
 * Exit status 0 = every check passed.  Built and run by tests/test_c_abi.py.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "welm_rope.h"

int64_t welm_oracle_apply(const uint16_t* data, uint16_t* out, int64_t rows, int64_t heads,
                          int64_t token_stride, const int64_t* rope_positions, const float* cache,
                          int64_t max_position);
int64_t welm_oracle_count_tiles(const int64_t* lens, int64_t bs);
int64_t welm_oracle_build_tiles(const int64_t* lens, int64_t bs, int32_t* starts);

#define HD WELM_ROPE_HEAD_DIM
#define NQ WELM_ROPE_NUM_Q_HEADS
#define MAX_POS 8192

static int failures = 0;

#define CHECK_CUDA(x)                                                              \
  do {                                                                             \
    cudaError_t e_ = (x);                                                          \
    if (e_ != cudaSuccess) {                                                       \
      fprintf(stderr, "%s:%d CUDA %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
      exit(2);                                                                     \
    }                                                                              \
  } while (0)

#define EXPECT(cond, what)                                  \
  do {                                                      \
    if (!(cond)) {                                          \
      fprintf(stderr, "FAILED: %s (line %d)\n", what, __LINE__); \
      ++failures;                                           \
    }                                                       \
  } while (0)

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static uint32_t next_u32(void) {
  rng_state = rng_state * 6364136223846793005ull + 1442695040888963407ull;
  return (uint32_t)(rng_state >> 32);
}
/* A finite BF16 value in about [-4, 4). */
static uint16_t random_bf16(void) {
  const float f = ((float)(next_u32() >> 8) / 16777216.0f - 0.5f) * 8.0f;
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return (uint16_t)(u >> 16);
}

static void* device_copy(const void* host, size_t bytes) {
  void* d = NULL;
  CHECK_CUDA(cudaMalloc(&d, bytes ? bytes : 16));
  if (bytes) CHECK_CUDA(cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice));
  return d;
}

static int same_bits(const uint16_t* a, const uint16_t* b, size_t n, const char* what) {
  for (size_t i = 0; i < n; ++i)
    if (a[i] != b[i]) {
      fprintf(stderr, "%s: first difference at element %zu (%#x vs %#x)\n", what, i, a[i], b[i]);
      return 0;
    }
  return 1;
}

static void check_ordinary(const float* cache, const float* d_cache, int64_t n, int segmented) {
  const size_t qn = (size_t)n * NQ * HD, kn = (size_t)n * HD;
  uint16_t* q = malloc(qn * 2);
  uint16_t* k = malloc(kn * 2);
  uint16_t* q_want = malloc(qn * 2);
  uint16_t* k_want = malloc(kn * 2);
  int64_t* pos = malloc((size_t)n * 8);
  for (size_t i = 0; i < qn; ++i) q[i] = random_bf16();
  for (size_t i = 0; i < kn; ++i) k[i] = random_bf16();
  for (int64_t i = 0; i < n; ++i) pos[i] = (int64_t)(next_u32() % MAX_POS);

  /* two requests (n/3 and the rest) as a 64-token tile table */
  int64_t lens[2] = {n / 3, n - n / 3};
  const int64_t tiles = welm_oracle_count_tiles(lens, 2);
  int32_t* starts = malloc((size_t)(tiles + 1) * 4);
  welm_oracle_build_tiles(lens, 2, starts);

  void* dq = device_copy(q, qn * 2);
  void* dk = device_copy(k, kn * 2);
  int64_t* dpos = device_copy(pos, (size_t)n * 8);
  int32_t* dstarts = device_copy(starts, (size_t)(tiles + 1) * 4);
  int32_t zero = 0, status = -1;
  int32_t* dstatus = device_copy(&zero, 4);

  /* without a table the reference's contract is num_work_tiles = ceil(N / 64) */
  const int64_t work_tiles = segmented ? tiles : (n + WELM_ROPE_TILE_TOKENS - 1) / WELM_ROPE_TILE_TOKENS;
  const int rc = welm_rope_ordinary(dq, dk, dpos, d_cache, segmented ? dstarts : NULL, work_tiles, n, NQ * HD, HD,
                                    segmented, MAX_POS, dstatus, NULL);
  EXPECT(rc == WELM_ROPE_OK, welm_rope_status_string(rc));
  CHECK_CUDA(cudaDeviceSynchronize());
  uint16_t* q_got = malloc(qn * 2);
  uint16_t* k_got = malloc(kn * 2);
  CHECK_CUDA(cudaMemcpy(q_got, dq, qn * 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(k_got, dk, kn * 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(&status, dstatus, 4, cudaMemcpyDeviceToHost));

  /* every tile here is full or the request's tail, so every token rotates */
  EXPECT(welm_oracle_apply(q, q_want, n, NQ, NQ * HD, pos, cache, MAX_POS) == 0, "oracle positions in range");
  EXPECT(welm_oracle_apply(k, k_want, n, 1, HD, pos, cache, MAX_POS) == 0, "oracle positions in range");
  EXPECT(same_bits(q_got, q_want, qn, segmented ? "ordinary segmented Q" : "ordinary dense Q"), "ordinary Q");
  EXPECT(same_bits(k_got, k_want, kn, segmented ? "ordinary segmented K" : "ordinary dense K"), "ordinary K");
  EXPECT(status == 0, "device status stays zero");

  CHECK_CUDA(cudaFree(dq));
  CHECK_CUDA(cudaFree(dk));
  CHECK_CUDA(cudaFree(dpos));
  CHECK_CUDA(cudaFree(dstarts));
  CHECK_CUDA(cudaFree(dstatus));
  free(q); free(k); free(q_want); free(k_want); free(q_got); free(k_got); free(pos); free(starts);
}

static void check_mirror(const float* cache, const float* d_cache) {
  int64_t lens[5] = {100, 1, 64, 300, 35};
  const int64_t bs = 5;
  int64_t n = 0;
  for (int r = 0; r < bs; ++r) n += lens[r];

  /* the host builder, the device builder and the oracle builder agree */
  int64_t tiles = -1;
  EXPECT(welm_rope_count_tiles_host(lens, bs, &tiles) == WELM_ROPE_OK, "count tiles");
  EXPECT(tiles == welm_oracle_count_tiles(lens, bs), "tile count");
  int32_t* starts = malloc((size_t)(tiles + 1) * 4);
  int32_t* want_starts = malloc((size_t)(tiles + 1) * 4);
  int64_t last_index[5], built = -1;
  EXPECT(welm_rope_build_tiles_host(lens, bs, starts, tiles + 1, &built, last_index) == WELM_ROPE_OK, "host builder");
  welm_oracle_build_tiles(lens, bs, want_starts);
  EXPECT(built == tiles && memcmp(starts, want_starts, (size_t)(tiles + 1) * 4) == 0, "host builder table");
  int64_t end = 0;
  for (int r = 0; r < bs; ++r) {
    end += lens[r];
    EXPECT(last_index[r] == end - 1, "last index");
  }

  int64_t* dlens = device_copy(lens, sizeof lens);
  int32_t* dstarts = NULL;
  int32_t* dcount = NULL;
  int64_t* dlast = NULL;
  CHECK_CUDA(cudaMalloc((void**)&dstarts, (size_t)(tiles + 1) * 4));
  CHECK_CUDA(cudaMalloc((void**)&dcount, 4));
  CHECK_CUDA(cudaMalloc((void**)&dlast, sizeof last_index));
  int32_t zero = 0, status = -1, dev_tiles = -1;
  int32_t* dstatus = device_copy(&zero, 4);
  int rc = welm_rope_build_tiles(dlens, bs, dstarts, tiles + 1, dcount, dlast, dstatus, NULL);
  EXPECT(rc == WELM_ROPE_OK, welm_rope_status_string(rc));
  CHECK_CUDA(cudaDeviceSynchronize());
  int32_t* dev_starts = malloc((size_t)(tiles + 1) * 4);
  int64_t dev_last[5];
  CHECK_CUDA(cudaMemcpy(dev_starts, dstarts, (size_t)(tiles + 1) * 4, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(&dev_tiles, dcount, 4, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(dev_last, dlast, sizeof dev_last, cudaMemcpyDeviceToHost));
  EXPECT(dev_tiles == tiles, "device tile count");
  EXPECT(memcmp(dev_starts, want_starts, (size_t)(tiles + 1) * 4) == 0, "device builder table");
  EXPECT(memcmp(dev_last, last_index, sizeof dev_last) == 0, "device last index");

  /* segmented KV-mirror prefill: Q holds one row per request, K every token */
  const size_t qn = (size_t)bs * NQ * HD, kn = (size_t)n * HD;
  uint16_t* q = malloc(qn * 2);
  uint16_t* k = malloc(kn * 2);
  uint16_t* q_want = malloc(qn * 2);
  uint16_t* k_want = malloc(kn * 2);
  int64_t* pos = malloc((size_t)n * 8);
  int64_t q_pos[5];
  for (size_t i = 0; i < qn; ++i) q[i] = random_bf16();
  for (size_t i = 0; i < kn; ++i) k[i] = random_bf16();
  for (int64_t i = 0; i < n; ++i) pos[i] = (int64_t)(next_u32() % MAX_POS);
  for (int r = 0; r < bs; ++r) q_pos[r] = pos[last_index[r]];

  void* dq = device_copy(q, qn * 2);
  void* dk = device_copy(k, kn * 2);
  int64_t* dpos = device_copy(pos, (size_t)n * 8);
  rc = welm_rope_mirror(dq, dk, dpos, d_cache, dlast, dstarts, tiles, n, bs, NQ * HD, HD, 1, MAX_POS, dstatus,
                        NULL);
  EXPECT(rc == WELM_ROPE_OK, welm_rope_status_string(rc));
  CHECK_CUDA(cudaDeviceSynchronize());
  uint16_t* q_got = malloc(qn * 2);
  uint16_t* k_got = malloc(kn * 2);
  CHECK_CUDA(cudaMemcpy(q_got, dq, qn * 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(k_got, dk, kn * 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(&status, dstatus, 4, cudaMemcpyDeviceToHost));
  welm_oracle_apply(q, q_want, bs, NQ, NQ * HD, q_pos, cache, MAX_POS);
  welm_oracle_apply(k, k_want, n, 1, HD, pos, cache, MAX_POS);
  EXPECT(same_bits(q_got, q_want, qn, "mirror Q rows"), "mirror Q");
  EXPECT(same_bits(k_got, k_want, kn, "mirror K"), "mirror K");
  EXPECT(status == 0, "device status stays zero");

  CHECK_CUDA(cudaFree(dlens));
  CHECK_CUDA(cudaFree(dstarts));
  CHECK_CUDA(cudaFree(dcount));
  CHECK_CUDA(cudaFree(dlast));
  CHECK_CUDA(cudaFree(dstatus));
  CHECK_CUDA(cudaFree(dq));
  CHECK_CUDA(cudaFree(dk));
  CHECK_CUDA(cudaFree(dpos));
  free(starts); free(want_starts); free(dev_starts);
  free(q); free(k); free(q_want); free(k_want); free(q_got); free(k_got); free(pos);
}

/* Q/K stay in page-locked host memory; the kernel reads and writes them over
 * the bus.  Positions are host memory too. */
static void check_mapped(const float* cache, const float* d_cache, int64_t n) {
  const size_t qn = (size_t)n * NQ * HD, kn = (size_t)n * HD;
  uint16_t *q = NULL, *k = NULL;
  int64_t* pos = NULL;
  CHECK_CUDA(cudaMallocHost((void**)&q, qn * 2));
  CHECK_CUDA(cudaMallocHost((void**)&k, kn * 2));
  CHECK_CUDA(cudaMallocHost((void**)&pos, (size_t)n * 8));
  uint16_t* q_want = malloc(qn * 2);
  uint16_t* k_want = malloc(kn * 2);
  for (size_t i = 0; i < qn; ++i) q[i] = random_bf16();
  for (size_t i = 0; i < kn; ++i) k[i] = random_bf16();
  for (int64_t i = 0; i < n; ++i) pos[i] = (int64_t)(next_u32() % MAX_POS);
  EXPECT(welm_oracle_apply(q, q_want, n, NQ, NQ * HD, pos, cache, MAX_POS) == 0, "oracle positions in range");
  EXPECT(welm_oracle_apply(k, k_want, n, 1, HD, pos, cache, MAX_POS) == 0, "oracle positions in range");

  /* pageable memory is refused before anything is launched */
  uint16_t* pageable = malloc(qn * 2);
  memcpy(pageable, q, qn * 2);
  int rc = welm_rope_ordinary_mapped(pageable, k, pos, d_cache, n, NQ * HD, HD, MAX_POS, NULL, NULL);
  EXPECT(rc == WELM_ROPE_ERR_NOT_MAPPED, "pageable Q is refused");
  EXPECT(memcmp(pageable, q, qn * 2) == 0, "refused call wrote nothing");

  int32_t zero = 0, status = -1;
  int32_t* dstatus = device_copy(&zero, 4);
  rc = welm_rope_ordinary_mapped(q, k, pos, d_cache, n, NQ * HD, HD, MAX_POS, dstatus, NULL);
  EXPECT(rc == WELM_ROPE_OK, welm_rope_status_string(rc));
  CHECK_CUDA(cudaDeviceSynchronize());
  CHECK_CUDA(cudaMemcpy(&status, dstatus, 4, cudaMemcpyDeviceToHost));
  EXPECT(same_bits(q, q_want, qn, "mapped Q"), "mapped Q");
  EXPECT(same_bits(k, k_want, kn, "mapped K"), "mapped K");
  EXPECT(status == 0, "device status stays zero");

  CHECK_CUDA(cudaFree(dstatus));
  CHECK_CUDA(cudaFreeHost(q));
  CHECK_CUDA(cudaFreeHost(k));
  CHECK_CUDA(cudaFreeHost(pos));
  free(pageable); free(q_want); free(k_want);
}

int main(void) {
  EXPECT(welm_rope_abi_version() == WELM_ROPE_ABI_VERSION, "library and header ABI versions agree");
  /* host validation happens before any CUDA call and names the problem */
  const int bad = welm_rope_ordinary(NULL, NULL, NULL, NULL, NULL, 1, 4, NQ * HD, HD, 0, MAX_POS, NULL, NULL);
  EXPECT(bad == WELM_ROPE_ERR_NULL_POINTER, "NULL q is refused");
  EXPECT(strlen(welm_rope_status_string(bad)) > 0, "status string");
  /* zero work tiles: nothing to rotate, so nothing is dereferenced */
  EXPECT(welm_rope_ordinary(NULL, NULL, NULL, NULL, NULL, 0, 4, NQ * HD, HD, 0, MAX_POS, NULL, NULL) == WELM_ROPE_OK,
         "zero work tiles is a no-op");

  float* cache = malloc((size_t)MAX_POS * WELM_ROPE_ROPE_DIM * sizeof(float));
  for (size_t i = 0; i < (size_t)MAX_POS * WELM_ROPE_ROPE_DIM; ++i)
    cache[i] = (float)(next_u32() >> 8) / 8388608.0f - 1.0f;
  float* d_cache = device_copy(cache, (size_t)MAX_POS * WELM_ROPE_ROPE_DIM * sizeof(float));

  check_ordinary(cache, d_cache, 1000, 0);
  check_ordinary(cache, d_cache, 777, 1);
  check_mirror(cache, d_cache);
  check_mapped(cache, d_cache, 1234);

  CHECK_CUDA(cudaFree(d_cache));
  free(cache);
  if (failures) {
    fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  printf("c-abi ok\n");
  return 0;
}
