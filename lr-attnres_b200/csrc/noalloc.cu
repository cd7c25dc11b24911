// attnres_lrid_backward_noalloc: the LRID read backward for callers that may
// not allocate device memory, with its scratch in a fixed static device array.
//
// The backward needs scratch for its per-CTA partial sums of the parameter
// gradients (static query, gate, logit bias); attnres_lrid_backward takes that
// scratch from the caller. Some callers cannot provide it: code that runs
// where cudaMalloc is forbidden or unavailable (inside a custom allocator's
// own callbacks, a host-side plugin given only fixed buffers, or a runtime
// that reserved all device memory up front). This entry point uses
// g_noalloc_scratch instead, a static array that each GPU loading the library
// keeps until the process exits.
#include <stdio.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "plan.h"

namespace {

constexpr size_t kNoallocScratchBytes = 4u << 20;  // 4 MiB per device

// Per-device scratch for the partial sums. Its name in host code is only a
// host-side handle: the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_mu;
// device ordinal -> device address of the scratch. The cache assumes the
// device's primary context lives as long as the process: after a
// cudaDeviceReset the module is loaded again and the cached address is stale.
std::unordered_map<int, void*> g_addr;

// Looks up the scratch's device address once per device (that device current).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return attnres::record_error(ATTNRES_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_addr.find(dev);
  if (it != g_addr.end()) {
    *out = it->second;
    return ATTNRES_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return attnres::record_error(ATTNRES_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch failed");
  g_addr[dev] = p;
  *out = p;
  return ATTNRES_OK;
}

}  // namespace

extern "C" {

size_t attnres_noalloc_scratch_bytes(void) { return kNoallocScratchBytes; }

int attnres_lrid_backward_noalloc(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                  int num_heads, int dtype, const void* const* values,
                                  const int64_t* value_row_strides, const void* const* keys,
                                  const int64_t* key_row_strides, int query_mode, const void* query,
                                  const void* query_gate, const void* query_dynamic, float logit_scale,
                                  int key_norm, float key_eps, const float* logit_bias, int output_norm,
                                  float output_eps, const void* grad_output, const void* normed_output,
                                  const float* output_inv_rms, void* const* grad_values,
                                  void* const* grad_keys, void* grad_query, float* grad_query_gate,
                                  void* grad_query_dynamic, float* grad_logit_bias, void* stream) {
  // A per-token query with no logit-bias gradient has no parameter gradient
  // to sum: that call uses no scratch, whatever its size.
  const bool uses_scratch = query_mode != ATTNRES_QUERY_DYNAMIC || grad_logit_bias != nullptr;
  const size_t need = attnres_lrid_backward_workspace_bytes(num_sources, num_tokens, value_dim, key_dim,
                                                            num_heads, dtype);
  if (need == 0 && uses_scratch)
    return attnres::record_error(ATTNRES_ERR_INVALID_ARGUMENT,
                                 "attnres_lrid_backward_noalloc: invalid geometry or no CUDA device");
  if (uses_scratch && need > kNoallocScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "attnres_lrid_backward_noalloc: this geometry needs %zu bytes of scratch, more than the "
             "%zu-byte static scratch; use attnres_lrid_backward with a caller workspace",
             need, kNoallocScratchBytes);
    return attnres::record_error(ATTNRES_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  // Every partial row the kernels read is written by the same call first, so
  // nothing in the scratch has to start at zero.
  return attnres_lrid_backward(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                               value_row_strides, keys, key_row_strides, query_mode, query, query_gate,
                               query_dynamic, logit_scale, key_norm, key_eps, logit_bias, output_norm,
                               output_eps, grad_output, normed_output, output_inv_rms, grad_values,
                               grad_keys, grad_query, grad_query_gate, grad_query_dynamic,
                               grad_logit_bias, scratch, kNoallocScratchBytes, stream);
}

}  // extern "C"
