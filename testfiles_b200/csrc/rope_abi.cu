// rope_abi.cu — ABI version and status strings of the C interface.

#include "welm_rope.h"

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

}  // extern "C"
