// rope_ceiling.cu — measurement kernels: the practical ceilings the RoPE
// kernels are timed against on the same bytes.  They rotate nothing, read no
// positions and no cos/sin cache, and are not part of the op.
//
// * welm_rope_ceiling_copy: a streaming device copy, one 16-byte vector per
//   thread, launched like the op (PDL attribute, pdl_enter before the first
//   access).  It is the best copy found for the op's byte counts, faster at
//   these sizes than the runtime's device-to-device copy.
// * welm_rope_ceiling_slices: the ordinary kernel's own access pattern — the
//   same item mapping, launch shape and 16-byte loads and stores of the rope
//   slices of K and the six Q heads, in place — without the position and
//   cos/sin gather and without the arithmetic.  Its time is the floor of that
//   access pattern: what the op would take if the rotation were free.

#include "rope_host.cuh"

namespace {

__global__ void __launch_bounds__(kBlock) ceiling_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                              int64_t vectors) {
  pdl_enter();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < vectors) dst[i] = __ldg(src + i);
}

// Writes the loaded slices back XORed with `salt`.  The caller passes 0, so
// the data is unchanged; the compiler cannot know that, so it keeps every
// store, which it could drop for a plain store of a just-loaded value.
template <int NH>
__device__ __forceinline__ void store_back(Slices<true, NH>& x, uint32_t salt) {
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    x.x1[h].x ^= salt;
    x.x2[h].x ^= salt;
    Io<true>::store8(x.base + h * kHeadDim, x.x1[h]);
    Io<true>::store8(x.base + h * kHeadDim + kHalf, x.x2[h]);
  }
}

__global__ void __launch_bounds__(kBlock) ceiling_slices_kernel(uint16_t* q, uint16_t* k, int64_t q_stride,
                                                                int64_t k_stride, int32_t items, uint32_t salt) {
  pdl_enter();
  const int stride = gridDim.x * blockDim.x;
  for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < items; item += stride) {
    const int part = item & (kParts - 1);
    const int64_t tok = item >> kPartShift;
    Slices<true, 1> kx;
    Slices<true, kQHeads> qx;
    kx.load(k + tok * k_stride, part);
    qx.load(q + tok * q_stride, part);
    store_back(kx, salt);
    store_back(qx, salt);
  }
}

}  // namespace

extern "C" {

int welm_rope_ceiling_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || bytes % 16 != 0) return WELM_ROPE_ERR_BAD_SIZE;
  const int64_t vectors = bytes / 16;
  if (vectors > kMaxItems) return WELM_ROPE_ERR_BAD_SIZE;
  if (vectors == 0) return WELM_ROPE_OK;
  if (!dst || !src) return WELM_ROPE_ERR_NULL_POINTER;
  if (!aligned16(dst) || !aligned16(src)) return WELM_ROPE_ERR_BAD_STRIDE;
  const unsigned grid = unsigned((vectors + kBlock - 1) / kBlock);
  return launch(ceiling_copy_kernel, grid, kBlock, 0, static_cast<cudaStream_t>(stream),
                static_cast<const uint4*>(src), static_cast<uint4*>(dst), vectors);
}

int welm_rope_ceiling_slices(void* q, void* k, int64_t n_tokens, int64_t q_token_stride, int64_t k_token_stride,
                             void* stream) {
  if (n_tokens < 0 || n_tokens > kMaxItems / kParts) return WELM_ROPE_ERR_BAD_SIZE;
  if (n_tokens == 0) return WELM_ROPE_OK;
  if (!q || !k) return WELM_ROPE_ERR_NULL_POINTER;
  if (n_tokens > 1 && (q_token_stride < kQHeads * kHeadDim || k_token_stride < kHeadDim))
    return WELM_ROPE_ERR_BAD_STRIDE;
  if (!aligned16(q) || !aligned16(k) || q_token_stride % 8 != 0 || k_token_stride % 8 != 0)
    return WELM_ROPE_ERR_BAD_STRIDE;  // the 16-byte vector path only
  const int64_t items = n_tokens * kParts;
  const LaunchShape shape = shape_for(items);
  return launch(ceiling_slices_kernel, shape.grid, shape.block, 0, static_cast<cudaStream_t>(stream),
                static_cast<uint16_t*>(q), static_cast<uint16_t*>(k), q_token_stride, k_token_stride,
                int32_t(items), uint32_t(0));
}

}  // extern "C"
