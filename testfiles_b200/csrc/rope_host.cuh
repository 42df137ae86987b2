// rope_host.cuh — host-side launch plumbing shared by the C entry points:
// SM count, grid sizing, the PDL launch wrapper and the token-source plan.

#ifndef WELM_ROPE_HOST_CUH_
#define WELM_ROPE_HOST_CUH_

#include <atomic>
#include <cstdlib>
#include <utility>

#include "rope_device.cuh"

namespace {
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

// Grid and block for `total` work items of a grid-stride kernel.  A launch
// with more than two warps of items but fewer than two full 128-thread CTAs
// per SM runs in warp-sized CTAs instead.  Its tokens then spread evenly over
// the SMs rather than queueing on a few SMs' bandwidth (one 128-thread CTA
// holds 32 tokens).  Measured on one B200 (graph replay, us): decode M=32
// 1.73 -> 1.44 and M=128 1.70 -> 1.47, prefill M=1024 2.23 -> 1.96 and
// M=6145 3.62 -> 3.47, fused KV write N=BS=128 1.86 -> 1.51.  At 16 tokens or
// fewer one CTA is as fast or faster, and from M=16384 the 128-thread grid is.
struct LaunchShape {
  unsigned grid;
  unsigned block;
};

LaunchShape shape_for(int64_t total) {
  constexpr int kSmallBlock = 32;
  const int sms = current_sm_count();
  if (sms > 0 && total > 2 * kSmallBlock && total <= 2 * int64_t(sms) * kBlock)
    return {unsigned((total + kSmallBlock - 1) / kSmallBlock), unsigned(kSmallBlock)};
  return {grid_for(total), unsigned(kBlock)};
}

// Dense launches of at most this many tokens run one head per thread (the
// ordinary one-head kernel, and the slice ceiling that mirrors it); larger
// ones run the streaming kernel.  Measured on one B200 (graph replay, L2-cold
// sets, us per launch): against a seven-heads-per-thread launch without
// prefetch, M=1 1.12 -> 0.86, M=128 1.47 -> 1.15, M=1024 1.96 -> 1.70; one
// head per thread against the streaming kernel, M=2048 1.91 vs 2.23, M=2561
// 2.08 vs 2.23, M=3072 2.29 vs 2.36, M=3585 2.54 vs 2.50, M=4096 2.70 vs 2.59.
constexpr int64_t kHeadSplitMaxTokens = 3328;

// One-head launches prefetch their slice lines before the wait from this many
// items (1536 tokens) up.  Measured on one B200 (graph replay, L2-cold sets,
// us per launch, without -> with the prefetch): M=1536 1.89 -> 1.77, M=2048
// 2.07 -> 1.91, M=4096 2.85 -> 2.56; below that it only adds latency: M=1
// 0.83 -> 0.90, M=8 0.93 -> 0.99, M=1281 1.89 -> 1.94.
constexpr int64_t kHeadPrefetchMinItems = int64_t(1536) * kHeadsPerToken * kParts;

// One-head launches of at most this many 128-thread CTAs' worth of items
// (decode batches up to 22 tokens) run in 128-thread CTAs rather than the
// warp-sized CTAs of shape_for.  Measured on four B200 boxes (graph replay,
// us per launch, warp-sized -> 128-thread CTAs): M=8 0.93 -> 0.90 and 1.00
// -> 0.99, M=12 1.05 -> 0.99, M=16 1.08 -> 0.90 / 0.92 / 0.99, M=20 1.07 ->
// 1.02.  From seven CTAs up it depends on the box: M=32 1.09 -> 0.93 on two
// boxes but 1.09 -> 1.18 on the other two, so larger batches keep the warp-
// sized CTAs.  256-thread CTAs were slower still (M=40 1.18, M=128 1.47).
constexpr int64_t kHeadFewCtas = 5;

// Launch shape of a one-head launch over `tokens` tokens: true when it
// applies, that is at most kHeadSplitMaxTokens tokens and a grid that gives
// every (token, head, part) item its own thread.
bool head_split_shape(int64_t tokens, LaunchShape& shape) {
  if (tokens > kHeadSplitMaxTokens) return false;
  const int64_t items = tokens * kHeadsPerToken * kParts;
  shape = items <= kHeadFewCtas * kBlock ? LaunchShape{unsigned((items + kBlock - 1) / kBlock), unsigned(kBlock)}
                                         : shape_for(items);
  return int64_t(shape.grid) * shape.block >= items;
}

// CTAs per SM of one streaming launch (rope_ordinary_stream_kernel): below the
// five its registers allow, so part of the next launch fits beside it.
constexpr int kStreamCtasPerSm = 4;

// CTAs of a streaming launch over `items` items: warp-sized CTAs, one item
// per thread, while the launch is at most three 128-thread CTAs per SM (so its
// tokens spread over every SM; M=9616 as 301 CTAs of 128 threads left three
// SMs a third CTA: 4.35 us, against 3.90 in warp-sized CTAs), else one item
// per thread up to kStreamCtasPerSm CTAs per SM, looping above that.
LaunchShape stream_shape(int64_t items) {
  const int sms = current_sm_count();
  if (sms > 0 && items > 64 && items <= 3 * int64_t(sms) * kBlock) return {unsigned((items + 31) / 32), 32u};
  const int64_t need = (items + kBlock - 1) / kBlock;
  const int64_t cap = sms > 0 ? int64_t(sms) * kStreamCtasPerSm : need;
  return {unsigned(need < cap ? need : cap), unsigned(kBlock)};
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
int launch_plan(Kernel kernel, const Plan& plan, const RopeArgs& a, cudaStream_t stream) {
  const int64_t total = int64_t(a.q_items) + plan.token_items + plan.check_items;
  if (plan.src == Source::kTileTable) {
    // One item per thread.  Up to one 128-thread CTA's worth of items per SM
    // the launch runs in warp-sized CTAs, so it spreads over all SMs instead
    // of leaving most with one CTA.  Measured on one B200 (graph replay, us):
    // segmented prefill M=4096 (8 requests) 3.55 -> 3.23; at M=8192 (32
    // requests, above this limit) warp-sized CTAs were slower, 4.43 -> 4.66.
    const size_t smem = (size_t(a.num_tiles + 1) * sizeof(int32_t) + 15) & ~size_t(15);
    const int sms = current_sm_count();
    if (sms > 0 && total <= int64_t(sms) * kBlock)
      return launch(kernel, unsigned((total + 31) / 32), 32u, smem, stream, a);
    return launch(kernel, unsigned((total + kBlock - 1) / kBlock), kBlock, smem, stream, a);
  }
  const LaunchShape shape = shape_for(total);
  return launch(kernel, shape.grid, shape.block, 0, stream, a);
}

}  // namespace

#endif  // WELM_ROPE_HOST_CUH_
