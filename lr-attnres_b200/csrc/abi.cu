// extern "C" entry points of libattnres_b200.so: argument validation, launch
// planning, and error reporting. Declared in include/attnres_b200.h.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>

#include "common.cuh"
#include "plan.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(ATTNRES_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

int elem_size(int dtype) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return 4;
    case ATTNRES_DTYPE_F16:
    case ATTNRES_DTYPE_BF16: return 2;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Common checks of the source tables. `need_keys` is false for the base read.
int check_sources(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                  const int64_t* vstr, const void* const* keys, const int64_t* kstr,
                  bool need_keys) {
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (S < 1 || S > ATTNRES_MAX_SOURCES)
    return fail(ATTNRES_ERR_UNSUPPORTED, "num_sources=%d outside [1, %d]", S, ATTNRES_MAX_SOURCES);
  if (N < 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "num_tokens=%lld is negative", N);
  if (d < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "value_dim=%d must be positive", d);
  if (!values || !vstr) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "values/value_row_strides is NULL");
  if (need_keys) {
    if (H < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "num_heads=%d must be positive", H);
    if (R < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key_dim=%d must be positive", R);
    if (d % H || R % H)
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "value_dim=%d and key_dim=%d must divide by num_heads=%d",
                  d, R, H);
    if (!keys || !kstr) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "keys/key_row_strides is NULL");
  }
  for (int s = 0; s < S; ++s) {
    if (N > 0 && !values[s]) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "values[%d] is NULL", s);
    if (vstr[s] < d) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "value_row_strides[%d]=%lld < value_dim",
                                 s, (long long)vstr[s]);
    if (need_keys) {
      if (N > 0 && !keys[s]) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "keys[%d] is NULL", s);
      if (kstr[s] < R) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key_row_strides[%d]=%lld < key_dim",
                                   s, (long long)kstr[s]);
    }
  }
  return ATTNRES_OK;
}

// True when every value row (and the extra dense buffers) admits 16-byte packs.
bool values_vectorizable(int S, int esz, const void* const* values, const int64_t* vstr,
                         const void* const* extra, int n_extra) {
  for (int s = 0; s < S; ++s)
    if (!aligned16(values[s]) || (vstr[s] * esz) % 16) return false;
  for (int i = 0; i < n_extra; ++i)
    if (extra[i] && !aligned16(extra[i])) return false;
  return true;
}

// Which LRID kernel to use. The streaming warp pipeline (bulk copies into
// per-warp rings) serves every layout whose rows are 16-byte aligned and split
// into 512-byte chunks per head; the register-streaming kernel serves every
// other layout (unaligned or odd-width rows, odd head counts). Tests set
// ATTNRES_B200_PATH=simt to run the register-streaming kernel on layouts the
// streaming pipeline would take.
enum PathChoice { PATH_AUTO, PATH_SIMT };

PathChoice path_choice() {
  const char* v = getenv("ATTNRES_B200_PATH");
  return (v && !strcmp(v, "simt")) ? PATH_SIMT : PATH_AUTO;
}

// Key rows (and per-token queries) admit 16-byte bulk copies.
bool keys_bulk_copyable(int S, int R, int esz, const void* const* keys, const int64_t* kstr,
                        const void* qdyn) {
  if ((static_cast<long long>(R) * esz) % 16) return false;
  for (int s = 0; s < S; ++s)
    if (!aligned16(keys[s]) || (kstr[s] * esz) % 16) return false;
  return qdyn == nullptr || aligned16(qdyn);
}

int check_query(int qmode, const void* q, const void* gate, const void* qdyn) {
  switch (qmode) {
    case ATTNRES_QUERY_STATIC:
      if (!q) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "static query is NULL");
      return ATTNRES_OK;
    case ATTNRES_QUERY_DYNAMIC:
      if (!qdyn) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "query_dynamic is NULL");
      return ATTNRES_OK;
    case ATTNRES_QUERY_GATED:
      if (!q || !gate || !qdyn)
        return fail(ATTNRES_ERR_INVALID_ARGUMENT, "gated query needs query, query_gate and query_dynamic");
      return ATTNRES_OK;
    default:
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown query_mode %d", qmode);
  }
}

int check_norm(int mode, bool allow_per_head) {
  if (mode == ATTNRES_NORM_NONE || mode == ATTNRES_NORM_ROW) return ATTNRES_OK;
  if (mode == ATTNRES_NORM_PER_HEAD && allow_per_head) return ATTNRES_OK;
  return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unsupported output_norm mode %d", mode);
}

}  // namespace

int attnres::record_error(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" {

int attnres_abi_version(void) { return ATTNRES_ABI_VERSION; }

const char* attnres_last_error(void) { return g_last_error.c_str(); }

int attnres_device_status(unsigned* status, int reset) {
  if (!status) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "status is NULL");
  unsigned s1 = 0, s2 = 0;
  cudaError_t e = attnres::read_warp_status(&s2, reset != 0);
  unsigned s3 = 0;
  if (e == cudaSuccess) e = attnres::read_keyproj_status(&s3, reset != 0);
  unsigned s4 = 0;
  if (e == cudaSuccess) e = attnres::read_keyproj_bwd_status(&s4, reset != 0);
  s3 |= s4;
  if (e == cudaSuccess) e = attnres::read_kvfused_status(&s4, reset != 0);
  s3 |= s4;
  if (e == cudaSuccess) e = attnres::read_kvbwd_status(&s4, reset != 0);
  s3 |= s4;
  if (e != cudaSuccess) return cuda_fail(e, "attnres_device_status");
  *status = s1 | s2 | s3;
  return ATTNRES_OK;
}

int attnres_lrid_forward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                         int num_heads, int dtype, const void* const* values,
                         const int64_t* value_row_strides, const void* const* keys,
                         const int64_t* key_row_strides, int query_mode, const void* query,
                         const void* query_gate, const void* query_dynamic, float logit_scale,
                         int key_norm, float key_eps, const float* logit_bias, int output_norm,
                         float output_eps, void* output, float* output_inv_rms, float* alpha_out,
                         float* key_inv_rms_out, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                         value_row_strides, keys, key_row_strides, true);
  if (rc) return rc;
  if ((rc = check_query(query_mode, query, query_gate, query_dynamic))) return rc;
  if ((rc = check_norm(output_norm, true))) return rc;
  if (num_tokens > 0 && !output) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "output is NULL");
  const int esz = elem_size(dtype);
  const void* extra[1] = {output};
  const bool vec = values_vectorizable(num_sources, esz, values, value_row_strides, extra, 1);
  attnres::LridPlan plan;
  const char* why = "";
  rc = attnres::make_lrid_plan(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, vec,
                               output_norm, &plan, &why);
  if (rc) return fail(rc, "%s", why);
  if (num_tokens == 0) return ATTNRES_OK;
  attnres::LridIO io{values, value_row_strides, keys, key_row_strides, query_mode, query,
                     query_gate, query_dynamic, logit_scale, key_norm, key_eps, logit_bias,
                     output_norm, output_eps, output, output_inv_rms, alpha_out, key_inv_rms_out};
  const PathChoice pc = path_choice();
  const bool has_qd = query_mode != ATTNRES_QUERY_STATIC;
  const bool bulk = pc != PATH_SIMT && vec && plan.vec == 16 / esz &&
                    keys_bulk_copyable(num_sources, key_dim, esz, keys, key_row_strides,
                                       has_qd ? query_dynamic : nullptr);
  attnres::TmaLayout wl{};
  int nw = 0;
  const bool warp = bulk && attnres::lrid_warp_plan(plan, esz, false, false, has_qd, output_norm, &wl, &nw);
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaError_t e = warp ? attnres::lrid_warp_forward_launch(dtype, plan, wl, nw, io, cs)
                       : attnres::lrid_forward_launch(dtype, plan, io, cs);
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_forward launch");
  return ATTNRES_OK;
}

size_t attnres_lrid_backward_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                             int key_dim, int num_heads, int dtype) {
  if (elem_size(dtype) == 0 || num_sources < 1 || num_sources > ATTNRES_MAX_SOURCES ||
      num_tokens < 0 || num_heads < 1 || value_dim < 1 || key_dim < 1 ||
      value_dim % num_heads || key_dim % num_heads)
    return 0;
  attnres::LridPlan plan;
  const char* why = "";
  // The pack width (and with it the grid) depends on pointer alignment, which
  // is unknown here: size for the larger of the two launch shapes.
  size_t best = 0;
  for (int v = 0; v < 2; ++v) {
    if (attnres::make_lrid_plan(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype,
                                v == 1, ATTNRES_NORM_NONE, &plan, &why))
      continue;
    size_t b = 0;
    if (attnres::lrid_workspace(dtype, plan, &b) != cudaSuccess) return 0;
    if (b > best) best = b;
    for (int variant = 0; variant < 4 && v == 1; ++variant) {
      attnres::TmaLayout tl{};
      const bool y = variant & 1, qd = variant & 2;
      int nw = 0;
      if (!attnres::lrid_warp_plan(plan, elem_size(dtype), true, y, qd, y ? ATTNRES_NORM_ROW : ATTNRES_NORM_NONE,
                                   &tl, &nw))
        continue;
      if (attnres::lrid_warp_workspace(dtype, plan, tl, nw, &b) != cudaSuccess) return 0;
      if (b > best) best = b;
    }
  }
  return best;
}

int attnres_lrid_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                          int num_heads, int dtype, const void* const* values,
                          const int64_t* value_row_strides, const void* const* keys,
                          const int64_t* key_row_strides, int query_mode, const void* query,
                          const void* query_gate, const void* query_dynamic, float logit_scale,
                          int key_norm, float key_eps, const float* logit_bias, int output_norm,
                          float output_eps, const void* grad_output, const void* normed_output,
                          const float* output_inv_rms, void* const* grad_values,
                          void* const* grad_keys, void* grad_query, float* grad_query_gate,
                          void* grad_query_dynamic, float* grad_logit_bias, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                         value_row_strides, keys, key_row_strides, true);
  if (rc) return rc;
  if ((rc = check_query(query_mode, query, query_gate, query_dynamic))) return rc;
  if ((rc = check_norm(output_norm, true))) return rc;
  if (!grad_keys) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_keys is NULL");
  if (num_tokens > 0) {
    if (!grad_output) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_output is NULL");
    if (output_norm != ATTNRES_NORM_NONE && (!normed_output || !output_inv_rms))
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "output norm backward needs normed_output and output_inv_rms");
    for (int s = 0; s < num_sources; ++s)
      if ((grad_values && !grad_values[s]) || !grad_keys[s])
        return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_values[%d]/grad_keys[%d] is NULL", s, s);
  }
  if (!grad_query) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_query is NULL");
  if (query_mode == ATTNRES_QUERY_GATED && (!grad_query_gate || (num_tokens > 0 && !grad_query_dynamic)))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "gated query needs grad_query_gate and grad_query_dynamic");
  const int esz = elem_size(dtype);
  const void* extra[2 + ATTNRES_MAX_SOURCES];
  int n_extra = 0;
  extra[n_extra++] = grad_output;
  extra[n_extra++] = output_norm != ATTNRES_NORM_NONE ? normed_output : nullptr;
  for (int s = 0; s < num_sources && grad_values; ++s) extra[n_extra++] = grad_values[s];
  const bool vec = values_vectorizable(num_sources, esz, values, value_row_strides, extra, n_extra);
  attnres::LridPlan plan;
  const char* why = "";
  rc = attnres::make_lrid_plan(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, vec,
                               output_norm, &plan, &why);
  if (rc) return fail(rc, "%s", why);
  const PathChoice pc = path_choice();
  const bool has_qd = query_mode != ATTNRES_QUERY_STATIC;
  const bool has_y = output_norm != ATTNRES_NORM_NONE;
  const bool bulk = pc != PATH_SIMT && vec && plan.vec == 16 / esz &&
                    keys_bulk_copyable(num_sources, key_dim, esz, keys, key_row_strides,
                                       has_qd ? query_dynamic : nullptr);
  attnres::TmaLayout wl{};
  int nw = 0;
  const bool warp = bulk && attnres::lrid_warp_plan(plan, esz, true, has_y, has_qd, output_norm, &wl, &nw);
  const bool need_ws = query_mode != ATTNRES_QUERY_DYNAMIC || grad_logit_bias != nullptr;
  if (need_ws) {
    size_t need = 0;
    cudaError_t e = warp ? attnres::lrid_warp_workspace(dtype, plan, wl, nw, &need)
                         : attnres::lrid_workspace(dtype, plan, &need);
    if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_backward workspace query");
    if (!workspace || workspace_bytes < need)
      return fail(ATTNRES_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
    if (!aligned16(workspace)) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  }
  attnres::LridIO io{values, value_row_strides, keys, key_row_strides, query_mode, query,
                     query_gate, query_dynamic, logit_scale, key_norm, key_eps, logit_bias,
                     output_norm, output_eps, nullptr, nullptr, nullptr, nullptr};
  attnres::LridGradIO gio{grad_output, normed_output, output_inv_rms, grad_values, grad_keys,
                          grad_query, grad_query_gate, grad_query_dynamic, grad_logit_bias, workspace};
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaError_t e = warp ? attnres::lrid_warp_backward_launch(dtype, plan, wl, nw, io, gio, cs)
                       : attnres::lrid_backward_launch(dtype, plan, io, gio, cs);
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_backward launch");
  return ATTNRES_OK;
}

int attnres_base_forward(int num_sources, int64_t num_tokens, int value_dim, int dtype,
                         const void* const* values, const int64_t* value_row_strides,
                         const void* query, int key_norm, float key_eps, const float* logit_bias,
                         int output_norm, float output_eps, void* output, float* output_inv_rms,
                         void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, 0, 1, dtype, values,
                         value_row_strides, nullptr, nullptr, false);
  if (rc) return rc;
  if ((rc = check_norm(output_norm, false))) return rc;
  if (!query) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "query is NULL");
  if (num_tokens > 0 && !output) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "output is NULL");
  const void* extra[2] = {output, query};
  const bool vec = values_vectorizable(num_sources, elem_size(dtype), values, value_row_strides, extra, 2);
  attnres::BasePlan plan;
  const char* why = "";
  rc = attnres::make_base_plan(num_sources, num_tokens, value_dim, dtype, vec, &plan, &why);
  if (rc) return fail(rc, "%s", why);
  if (num_tokens == 0) return ATTNRES_OK;
  attnres::BaseIO io{};
  io.values = values;
  io.vstr = value_row_strides;
  io.q = query;
  io.key_norm = key_norm;
  io.key_eps = key_eps;
  io.bias = logit_bias;
  io.out_norm = output_norm;
  io.out_eps = output_eps;
  io.out = output;
  io.out_inv = output_inv_rms;
  cudaError_t e = attnres::base_forward_launch(dtype, plan, io, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_base_forward launch");
  return ATTNRES_OK;
}

size_t attnres_base_backward_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                             int dtype) {
  if (elem_size(dtype) == 0 || num_sources < 1 || num_sources > ATTNRES_MAX_SOURCES ||
      num_tokens < 0 || value_dim < 1)
    return 0;
  size_t best = 0;
  for (int v = 0; v < 2; ++v) {
    attnres::BasePlan plan;
    const char* why = "";
    if (attnres::make_base_plan(num_sources, num_tokens, value_dim, dtype, v == 1, &plan, &why))
      continue;
    size_t b = 0;
    if (attnres::base_workspace(dtype, plan, &b) != cudaSuccess) return 0;
    if (b > best) best = b;
  }
  return best;
}

int attnres_base_backward(int num_sources, int64_t num_tokens, int value_dim, int dtype,
                          const void* const* values, const int64_t* value_row_strides,
                          const void* query, int key_norm, float key_eps, const float* logit_bias,
                          int output_norm, float output_eps, const void* grad_output,
                          const void* normed_output, const float* output_inv_rms,
                          void* const* grad_values, float* grad_query, float* grad_logit_bias,
                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, 0, 1, dtype, values,
                         value_row_strides, nullptr, nullptr, false);
  if (rc) return rc;
  if ((rc = check_norm(output_norm, false))) return rc;
  if (!query || !grad_query) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "query/grad_query is NULL");
  if (!grad_values) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_values is NULL");
  if (num_tokens > 0) {
    if (!grad_output) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_output is NULL");
    if (output_norm != ATTNRES_NORM_NONE && (!normed_output || !output_inv_rms))
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "output norm backward needs normed_output and output_inv_rms");
    for (int s = 0; s < num_sources; ++s)
      if (!grad_values[s]) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_values[%d] is NULL", s);
  }
  const void* extra[3 + ATTNRES_MAX_SOURCES];
  int n_extra = 0;
  extra[n_extra++] = grad_output;
  extra[n_extra++] = query;
  extra[n_extra++] = output_norm != ATTNRES_NORM_NONE ? normed_output : nullptr;
  for (int s = 0; s < num_sources; ++s) extra[n_extra++] = grad_values[s];
  const bool vec = values_vectorizable(num_sources, elem_size(dtype), values, value_row_strides, extra, n_extra);
  attnres::BasePlan plan;
  const char* why = "";
  rc = attnres::make_base_plan(num_sources, num_tokens, value_dim, dtype, vec, &plan, &why);
  if (rc) return fail(rc, "%s", why);
  size_t need = 0;
  cudaError_t e = attnres::base_workspace(dtype, plan, &need);
  if (e != cudaSuccess) return cuda_fail(e, "attnres_base_backward workspace query");
  if (!workspace || workspace_bytes < need)
    return fail(ATTNRES_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
  if (!aligned16(workspace)) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  attnres::BaseIO io{};
  io.values = values;
  io.vstr = value_row_strides;
  io.q = query;
  io.key_norm = key_norm;
  io.key_eps = key_eps;
  io.bias = logit_bias;
  io.out_norm = output_norm;
  io.out_eps = output_eps;
  io.grad_output = grad_output;
  io.normed_output = normed_output;
  io.output_inv_rms = output_inv_rms;
  io.grad_values = grad_values;
  io.grad_query = grad_query;
  io.grad_bias = grad_logit_bias;
  io.workspace = workspace;
  e = attnres::base_backward_launch(dtype, plan, io, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_base_backward launch");
  return ATTNRES_OK;
}

int attnres_lrid_key_projection(int num_sources, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                                const void* const* values, const int64_t* value_row_strides,
                                const void* weight, int64_t weight_row_stride, int value_norm,
                                float value_eps, void* keys, float* inv_rms, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, 1, dtype, values, value_row_strides,
                         nullptr, nullptr, false);
  if (rc) return rc;
  if (key_dim < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key_dim=%d must be positive", key_dim);
  if (!weight || weight_row_stride < value_dim)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "weight is NULL or its row stride is below value_dim");
  if (num_tokens > 0 && !keys) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "keys is NULL");
  if (value_norm && num_tokens > 0 && !inv_rms)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "value_norm needs an inv_rms output");
  bool used_tc = false;
  cudaError_t e = attnres::keyproj_launch(num_sources, num_tokens, value_dim, key_dim, dtype, values,
                                          value_row_strides, weight, weight_row_stride, value_norm, value_eps,
                                          keys, inv_rms, path_choice() != PATH_SIMT,
                                          static_cast<cudaStream_t>(stream), &used_tc);
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_key_projection launch");
  return ATTNRES_OK;
}

int attnres_lrid_fused_key_projection(int64_t num_tokens, int in_dim, int rank, int query_rank, int num_heads,
                                      int dtype, const void* x, int64_t x_row_stride, const void* weight,
                                      int64_t weight_row_stride, int key_norm, float eps, void* key_query,
                                      void* key, float* key_inv_rms, void* stream) {
  if (num_tokens < 0 || in_dim < 1 || rank < 1 || query_rank < 0 || num_heads < 1 || rank % num_heads)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT,
                "attnres_lrid_fused_key_projection: bad geometry (tokens %lld, in_dim %d, rank %d, query_rank %d, "
                "heads %d)", static_cast<long long>(num_tokens), in_dim, rank, query_rank, num_heads);
  if (dtype != ATTNRES_DTYPE_F32 && dtype != ATTNRES_DTYPE_F16 && dtype != ATTNRES_DTYPE_BF16)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "attnres_lrid_fused_key_projection: unknown dtype %d", dtype);
  if (num_tokens == 0) return ATTNRES_OK;
  if (!x || !weight || !key_query || x_row_stride < in_dim || weight_row_stride < in_dim)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT,
                "attnres_lrid_fused_key_projection: NULL pointer or a row stride below in_dim");
  if (key_norm && (!key || !key_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "attnres_lrid_fused_key_projection: key_norm needs key and key_inv_rms");
  bool eligible = false;
  cudaError_t e = attnres::fused_key_projection_launch(num_tokens, in_dim, rank, query_rank, num_heads, dtype, x,
                                                       x_row_stride, weight, weight_row_stride, key_norm, eps,
                                                       key_query, key, key_inv_rms,
                                                       static_cast<cudaStream_t>(stream), &eligible);
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_fused_key_projection launch");
  if (!eligible)
    return fail(ATTNRES_ERR_UNSUPPORTED,
                "attnres_lrid_fused_key_projection: needs 16-bit data, in_dim %% 64 == 0, rank + query_rank a "
                "multiple of 16 in [16, 256], a head width that is a multiple of 16 with key_norm, and 16-byte "
                "aligned rows");
  return ATTNRES_OK;
}

int attnres_lrid_key_projection_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                         int num_heads, int dtype, const void* const* values,
                                         const int64_t* value_row_strides, void* const* grad_values,
                                         const void* grad_normed, const void* grad_keys, const void* keys,
                                         const float* inv_rms, const void* grad_output, const float* alpha,
                                         int value_norm, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                         value_row_strides, nullptr, nullptr, false);
  if (rc) return rc;
  if (num_heads < 1 || value_dim % num_heads)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "value_dim must divide by num_heads");
  if (num_tokens > 0 && (!grad_values || !grad_normed || !grad_keys || !keys || (value_norm && !inv_rms)))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key projection backward: NULL buffer");
  if ((grad_output == nullptr) != (alpha == nullptr))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_output and alpha go together");
  cudaError_t e = attnres::keyproj_bwd_combine_launch(num_sources, num_tokens, value_dim, key_dim, num_heads,
                                                      dtype, values, value_row_strides, grad_values,
                                                      grad_normed, grad_keys, keys, inv_rms, grad_output,
                                                      alpha, value_norm, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_key_projection_backward launch");
  return ATTNRES_OK;
}

int attnres_lrid_key_from_value_forward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                        int num_heads, int dtype, const void* const* values,
                                        const int64_t* value_row_strides, const void* weight,
                                        int64_t weight_row_stride, int value_norm, float value_eps,
                                        const void* query, float logit_scale, int key_norm, float key_eps,
                                        const float* logit_bias, void* output, void* keys, float* value_inv_rms,
                                        float* alpha_out, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values, value_row_strides,
                         nullptr, nullptr, false);
  if (rc) return rc;
  if (num_tokens == 0) return ATTNRES_OK;
  if (!weight || !query || !output || !keys || (value_norm && !value_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key-from-value forward: NULL weight/query/output/keys/inv_rms");
  const char* why = "";
  if (!attnres::kvfused_eligible(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                                 value_row_strides, weight, weight_row_stride, &why))
    return fail(ATTNRES_ERR_UNSUPPORTED, "key-from-value forward: %s", why);
  if (!aligned16(output) || !aligned16(keys))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "key-from-value forward: output and keys must be 16-byte aligned");
  cudaError_t e = attnres::kvfused_forward_launch(
      num_sources, num_tokens, value_dim, num_heads, dtype, values, value_row_strides, weight, weight_row_stride,
      value_norm, value_eps, query, logit_scale, key_norm, key_eps, logit_bias, output, keys, value_inv_rms,
      alpha_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_key_from_value_forward launch");
  return ATTNRES_OK;
}

size_t attnres_lrid_key_projection_backward_tc_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                                               int key_dim, int num_heads, int dtype) {
  return attnres::keyproj_bwd_tc_workspace(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype);
}

int attnres_lrid_key_projection_backward_tc(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                            int num_heads, int dtype, const void* const* values,
                                            const int64_t* value_row_strides, const void* weight,
                                            int64_t weight_row_stride, const void* const* grad_keys,
                                            const void* keys, const float* inv_rms, const void* grad_output,
                                            const float* alpha, int value_norm, void* const* grad_values,
                                            float* grad_weight, void* workspace, size_t workspace_bytes,
                                            void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                         value_row_strides, nullptr, nullptr, false);
  if (rc) return rc;
  if (num_tokens == 0) return ATTNRES_OK;
  const size_t need = attnres::keyproj_bwd_tc_workspace(num_sources, num_tokens, value_dim, key_dim, num_heads,
                                                         dtype);
  if (need == 0)
    return fail(ATTNRES_ERR_UNSUPPORTED,
                "fused projection backward needs f16/bf16, key_dim 64, value_dim/num_heads a multiple of 128, "
                "at most 24 sources");
  if (!weight || !grad_keys || !keys || !grad_output || !alpha || !grad_values || !grad_weight || !workspace ||
      (value_norm && !inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "fused projection backward: NULL buffer");
  if (workspace_bytes < need)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (weight_row_stride < value_dim) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "weight_row_stride < value_dim");
  if (!aligned16(grad_output) || !aligned16(keys) || !aligned16(workspace))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_output, keys and workspace must be 16-byte aligned");
  for (int s = 0; s < num_sources; ++s) {
    if (!grad_keys[s] || !grad_values[s] || !aligned16(grad_keys[s]) || !aligned16(grad_values[s]))
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_keys[%d] / grad_values[%d] NULL or not 16-byte aligned", s,
                  s);
    if (!aligned16(values[s]) || (value_row_strides[s] * 2) % 16)
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "values[%d] must be 16-byte aligned with 16-byte row strides", s);
  }
  cudaError_t e = attnres::keyproj_bwd_tc_launch(
      num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values, value_row_strides, weight,
      weight_row_stride, grad_keys, keys, inv_rms, grad_output, alpha, value_norm, grad_values, grad_weight,
      workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_key_projection_backward_tc launch");
  return ATTNRES_OK;
}

size_t attnres_lrid_key_from_value_backward_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                                             int key_dim, int num_heads, int dtype) {
  return attnres::kvbwd_fused_workspace(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype);
}

int attnres_lrid_key_from_value_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                         int num_heads, int dtype, const void* const* values,
                                         const int64_t* value_row_strides, const void* weight,
                                         int64_t weight_row_stride, const void* keys, int value_norm,
                                         const float* value_inv_rms, const float* alpha, const void* query,
                                         float logit_scale, int key_norm, float key_eps, const void* grad_output,
                                         const void* output, void* const* grad_values, float* grad_weight,
                                         float* grad_query, float* grad_logit_bias, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values,
                         value_row_strides, nullptr, nullptr, false);
  if (rc) return rc;
  if (num_tokens == 0) return ATTNRES_OK;
  const size_t need = attnres::kvbwd_fused_workspace(num_sources, num_tokens, value_dim, key_dim, num_heads, dtype);
  if (need == 0)
    return fail(ATTNRES_ERR_UNSUPPORTED,
                "one-pass key-from-value backward needs f16/bf16, key_dim 64, 2..24 sources, num_heads 1/2/4/8, "
                "value_dim/num_heads a multiple of 256, value_dim <= 4096");
  if (!weight || !keys || !alpha || !query || !grad_output || !output || !grad_values || !grad_weight ||
      !grad_query || !workspace || (value_norm && !value_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "one-pass key-from-value backward: NULL buffer");
  if (workspace_bytes < need)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (weight_row_stride < value_dim) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "weight_row_stride < value_dim");
  if (!aligned16(grad_output) || !aligned16(output) || !aligned16(keys) || !aligned16(workspace) ||
      !aligned16(weight) || (weight_row_stride * 2) % 16)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT,
                "grad_output, output, keys, weight rows and workspace must be 16-byte aligned");
  for (int s = 0; s < num_sources; ++s) {
    if (!grad_values[s] || !aligned16(grad_values[s]))
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "grad_values[%d] NULL or not 16-byte aligned", s);
    if (!aligned16(values[s]) || (value_row_strides[s] * 2) % 16)
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "values[%d] must be 16-byte aligned with 16-byte row strides", s);
  }
  cudaError_t e = attnres::kvbwd_fused_launch(
      num_sources, num_tokens, value_dim, key_dim, num_heads, dtype, values, value_row_strides, weight,
      weight_row_stride, keys, value_norm ? value_inv_rms : nullptr, alpha, query, logit_scale, key_norm, key_eps,
      grad_output, output, grad_values, grad_weight, grad_query, grad_logit_bias, workspace, workspace_bytes,
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_lrid_key_from_value_backward launch");
  return ATTNRES_OK;
}

int attnres_block_summary_forward(int64_t num_elements, int dtype, const void* partial, const void* x,
                                  const float* scale_device, float scale, void* sum, void* source,
                                  void* stream) {
  if (num_elements < 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "num_elements < 0");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_elements > 0 && (!x || !source)) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary: NULL x/source");
  cudaError_t e = attnres::summary_forward_launch(num_elements, dtype, partial, x, scale_device, scale, sum, source,
                                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_block_summary_forward launch");
  return ATTNRES_OK;
}

size_t attnres_block_summary_backward_workspace_bytes(int64_t num_elements) {
  if (num_elements <= 0) return 0;
  return sizeof(float) * static_cast<size_t>(attnres::summary_bwd_grid(num_elements));
}

int attnres_block_summary_backward(int64_t num_elements, int dtype, const void* grad_source, const void* grad_sum,
                                   const void* sum, const float* scale_device, float scale, void* grad_partial,
                                   float* grad_scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (num_elements < 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "num_elements < 0");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_elements > 0 && !grad_partial) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary: NULL grad_partial");
  const bool want_dc = grad_scale && grad_source && num_elements > 0;
  if (want_dc) {
    if (!sum) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary: the scale gradient needs the saved sum");
    if (!workspace || workspace_bytes < attnres_block_summary_backward_workspace_bytes(num_elements))
      return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary: workspace too small");
  }
  cudaError_t e = attnres::summary_backward_launch(num_elements, dtype, grad_source, grad_sum, sum, scale_device,
                                                   scale, grad_partial, grad_scale, static_cast<float*>(workspace),
                                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_block_summary_backward launch");
  return ATTNRES_OK;
}

int attnres_block_summary_norm_forward(int64_t num_rows, int row_width, int dtype, const void* partial,
                                       const void* x, float eps, void* sum, void* source, float* inv_rms,
                                       void* stream) {
  if (num_rows < 0 || row_width < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary norm: bad shape");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_rows > 0 && (!x || !source || !inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary norm: NULL x/source/inv_rms");
  cudaError_t e = attnres::summary_norm_launch(false, num_rows, row_width, dtype, partial, x, eps, sum, source,
                                               inv_rms, nullptr, nullptr, nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_block_summary_norm_forward launch");
  return ATTNRES_OK;
}

int attnres_block_summary_norm_backward(int64_t num_rows, int row_width, int dtype, const void* grad_source,
                                        const void* grad_sum, const void* sum, const float* inv_rms,
                                        void* grad_total, void* stream) {
  if (num_rows < 0 || row_width < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary norm: bad shape");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_rows > 0 && (!grad_source || !sum || !inv_rms || !grad_total))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "block summary norm backward: NULL buffer");
  cudaError_t e = attnres::summary_norm_launch(true, num_rows, row_width, dtype, nullptr, nullptr, 0.f,
                                               const_cast<void*>(sum), nullptr, const_cast<float*>(inv_rms),
                                               grad_source, grad_sum, grad_total, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_block_summary_norm_backward launch");
  return ATTNRES_OK;
}

static int check_phase2(int mode, int64_t N, int d, int R, int dtype, const void* v, const void* key,
                        const float* logit, const void* q, const void* prev, const float* lse) {
  if (mode < ATTNRES_PHASE2_LRID || mode > ATTNRES_PHASE2_LOGIT)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown phase-2 mode %d", mode);
  if (N < 0 || d < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: num_tokens < 0 or value_dim < 1");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (mode == ATTNRES_PHASE2_LRID && R < 1) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: key_dim < 1");
  if (N == 0) return ATTNRES_OK;
  if (!v || !prev || !lse) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: NULL partial value / interblock");
  if (mode == ATTNRES_PHASE2_LRID && (!key || !q)) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: NULL key/query");
  if (mode == ATTNRES_PHASE2_BASE && !q) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: NULL query");
  if (mode == ATTNRES_PHASE2_LOGIT && !logit) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: NULL partial logit");
  return ATTNRES_OK;
}

int attnres_phase2_forward(int mode, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                           const void* partial_value, const void* partial_key, const float* partial_logit,
                           const void* query, float logit_scale, int key_norm, float key_eps, float logit_bias,
                           const float* logit_bias_device, const void* interblock_output,
                           const float* interblock_lse, int normalize_output, float output_eps, void* output,
                           float* output_inv_rms, void* stream) {
  int rc = check_phase2(mode, num_tokens, value_dim, key_dim, dtype, partial_value, partial_key, partial_logit, query,
                        interblock_output, interblock_lse);
  if (rc) return rc;
  if (num_tokens == 0) return ATTNRES_OK;
  if (!output || (normalize_output && !output_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2: NULL output / output_inv_rms");
  cudaError_t e = attnres::phase2_run(false, mode, num_tokens, value_dim, key_dim, dtype, partial_value, partial_key,
                                      partial_logit, query, logit_scale, key_norm, key_eps, logit_bias,
                                      logit_bias_device, interblock_output, interblock_lse, normalize_output,
                                      output_eps, output, output_inv_rms, nullptr, nullptr, nullptr, nullptr, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_phase2_forward launch");
  return ATTNRES_OK;
}

size_t attnres_phase2_backward_workspace_bytes(int mode, int64_t num_tokens, int value_dim, int key_dim) {
  return attnres::phase2_workspace(mode, num_tokens, value_dim, key_dim);
}

int attnres_phase2_backward(int mode, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                            const void* partial_value, const void* partial_key, const float* partial_logit,
                            const void* query, float logit_scale, int key_norm, float key_eps, float logit_bias,
                            const float* logit_bias_device, const void* interblock_output,
                            const float* interblock_lse, int normalize_output, const void* output,
                            const float* output_inv_rms, const void* grad_output, void* grad_partial_value,
                            void* grad_partial_key, float* grad_partial_logit, void* grad_interblock_output,
                            float* grad_interblock_lse, float* grad_query, float* grad_bias, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int rc = check_phase2(mode, num_tokens, value_dim, key_dim, dtype, partial_value, partial_key, partial_logit, query,
                        interblock_output, interblock_lse);
  if (rc) return rc;
  if (num_tokens == 0) {
    if (grad_query) cudaMemsetAsync(grad_query, 0, sizeof(float) * (mode == ATTNRES_PHASE2_LRID ? key_dim : value_dim),
                                    static_cast<cudaStream_t>(stream));
    if (grad_bias) cudaMemsetAsync(grad_bias, 0, sizeof(float), static_cast<cudaStream_t>(stream));
    return ATTNRES_OK;
  }
  if (!grad_output || !grad_partial_value || !grad_interblock_output || !grad_interblock_lse)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2 backward: NULL gradient buffer");
  if (mode == ATTNRES_PHASE2_LRID && !grad_partial_key)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2 backward: NULL grad_partial_key");
  if (mode == ATTNRES_PHASE2_LOGIT && !grad_partial_logit)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2 backward: NULL grad_partial_logit");
  if (normalize_output && (!output || !output_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2 backward: the normalised output and its inverse rms are needed");
  const bool need_ws = (grad_query && mode != ATTNRES_PHASE2_LOGIT) || grad_bias;
  if (need_ws && (!workspace || workspace_bytes < attnres::phase2_workspace(mode, num_tokens, value_dim, key_dim)))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase 2 backward: workspace too small");
  cudaError_t e = attnres::phase2_run(true, mode, num_tokens, value_dim, key_dim, dtype, partial_value, partial_key,
                                      partial_logit, query, logit_scale, key_norm, key_eps, logit_bias,
                                      logit_bias_device, interblock_output, interblock_lse, normalize_output, 0.f,
                                      nullptr, nullptr, grad_output, output, output_inv_rms, grad_partial_value,
                                      grad_partial_key, grad_partial_logit, grad_interblock_output,
                                      grad_interblock_lse, grad_query, grad_bias, workspace,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_phase2_backward launch");
  return ATTNRES_OK;
}

int attnres_head_rms_norm_forward(int64_t rows, int width, int num_heads, int dtype, const void* x,
                                  int64_t x_row_stride, float eps, void* y, float* inv_rms, void* stream) {
  if (rows < 0 || width < 1 || num_heads < 1 || width % num_heads)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm: width must divide by num_heads");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (x_row_stride < width) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm: x_row_stride < width");
  if (rows > 0 && (!x || !y)) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm: NULL x/y");
  cudaError_t e = attnres::headnorm_launch(false, dtype, rows, width, num_heads, x, x_row_stride, eps, nullptr,
                                           nullptr, y, inv_rms, width, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_head_rms_norm_forward launch");
  return ATTNRES_OK;
}

int attnres_head_rms_norm_backward(int64_t rows, int width, int num_heads, int dtype, const void* grad_y,
                                   const void* x, int64_t x_row_stride, const float* inv_rms, void* grad_x,
                                   int64_t grad_x_row_stride, void* stream) {
  if (rows < 0 || width < 1 || num_heads < 1 || width % num_heads)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm: width must divide by num_heads");
  if (elem_size(dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (grad_x_row_stride < width || x_row_stride < width)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm: a row stride < width");
  if (rows > 0 && (!grad_y || !x || !inv_rms || !grad_x))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "head rms norm backward: NULL buffer");
  cudaError_t e = attnres::headnorm_launch(true, dtype, rows, width, num_heads, grad_y, x_row_stride, 0.f, x,
                                           inv_rms, grad_x, nullptr, grad_x_row_stride,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_head_rms_norm_backward launch");
  return ATTNRES_OK;
}

int attnres_phase1_forward(int num_sources, int num_queries, int64_t num_tokens, int value_dim, int dtype,
                           const void* const* values, const int64_t* value_row_strides, const void* logits,
                           int logit_dtype, int output_norm, float output_eps, void* output, float* lse,
                           float* output_inv_rms, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, 0, 1, dtype, values, value_row_strides, nullptr,
                         nullptr, false);
  if (rc) return rc;
  if (num_queries < 1 || num_queries > 16)
    return fail(ATTNRES_ERR_UNSUPPORTED, "num_queries=%d outside [1, 16]", num_queries);
  if (elem_size(logit_dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown logit dtype %d", logit_dtype);
  if ((rc = check_norm(output_norm, false))) return rc;
  if (num_tokens > 0 && (!logits || !output || !lse))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase1 forward: NULL logits/output/lse");
  if (num_tokens == 0) return ATTNRES_OK;
  const void* extra[1] = {output};
  const bool vec = values_vectorizable(num_sources, elem_size(dtype), values, value_row_strides, extra, 1);
  cudaError_t e = attnres::phase1_launch(dtype, logit_dtype, num_sources, num_queries, num_tokens, value_dim, vec,
                                         values, value_row_strides, logits, output_norm != ATTNRES_NORM_NONE,
                                         output_eps, output, lse, output_inv_rms, nullptr, nullptr, nullptr,
                                         nullptr, nullptr, nullptr, false, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_phase1_forward launch");
  return ATTNRES_OK;
}

int attnres_phase1_backward(int num_sources, int num_queries, int64_t num_tokens, int value_dim, int dtype,
                            const void* const* values, const int64_t* value_row_strides, const void* logits,
                            int logit_dtype, int output_norm, float output_eps, const void* grad_output,
                            const float* grad_lse, const void* normed_output, const float* output_inv_rms,
                            void* const* grad_values, void* grad_logits, void* stream) {
  int rc = check_sources(num_sources, num_tokens, value_dim, 0, 1, dtype, values, value_row_strides, nullptr,
                         nullptr, false);
  if (rc) return rc;
  if (num_queries < 1 || num_queries > 16)
    return fail(ATTNRES_ERR_UNSUPPORTED, "num_queries=%d outside [1, 16]", num_queries);
  if (elem_size(logit_dtype) == 0) return fail(ATTNRES_ERR_INVALID_ARGUMENT, "unknown logit dtype %d", logit_dtype);
  if ((rc = check_norm(output_norm, false))) return rc;
  if (num_tokens == 0) return ATTNRES_OK;
  if (!logits || !grad_output || !grad_values || !grad_logits)
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase1 backward: NULL buffer");
  if (output_norm != ATTNRES_NORM_NONE && (!normed_output || !output_inv_rms))
    return fail(ATTNRES_ERR_INVALID_ARGUMENT, "phase1 backward with output norm needs normed_output/output_inv_rms");
  const void* extra[2 + ATTNRES_MAX_SOURCES];
  int n_extra = 0;
  extra[n_extra++] = grad_output;
  extra[n_extra++] = output_norm != ATTNRES_NORM_NONE ? normed_output : nullptr;
  for (int s = 0; s < num_sources; ++s) extra[n_extra++] = grad_values[s];
  const bool vec = values_vectorizable(num_sources, elem_size(dtype), values, value_row_strides, extra, n_extra);
  cudaError_t e = attnres::phase1_launch(dtype, logit_dtype, num_sources, num_queries, num_tokens, value_dim, vec,
                                         values, value_row_strides, logits, output_norm != ATTNRES_NORM_NONE,
                                         output_eps, nullptr, nullptr, nullptr, grad_output, normed_output,
                                         output_inv_rms, grad_lse, grad_values, grad_logits, true,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attnres_phase1_backward launch");
  return ATTNRES_OK;
}

}  // extern "C"
