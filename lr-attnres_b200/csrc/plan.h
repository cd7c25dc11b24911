// Host/device launch plans and argument bundles of the AttnRes read kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace attnres {

// Thread layout of one LRID launch (computed on the host by make_lrid_plan).
struct LridPlan {
  int S, d, R, H, dv, dk;
  long long N;
  int vec;    // elements per value pack (16 bytes worth, or 1 for unaligned rows)
  int nvh;    // packs per head row = dv / vec
  int tph;    // value threads per head (power of two)
  int cph;    // packs per value thread = ceil(nvh / tph)
  int lph;    // key lanes per head (power of two <= 32)
  int kpl;    // key elements per lane = ceil(dk / lph)
  int tpt;    // threads per token row (power of two, >= 32)
  int tpc;    // token rows per CTA
  int wph;    // warps per head = max(1, tph / 32)
  int out_norm_group;  // threads in one output-norm reduction group
  long long ntiles;
};

struct LridIO {
  const void* const* values;
  const int64_t* vstr;
  const void* const* keys;
  const int64_t* kstr;
  int qmode;
  const void* q;
  const void* gate;
  const void* qdyn;
  float scale;
  int key_norm;
  float key_eps;
  const float* bias;
  int out_norm;
  float out_eps;
  void* out;
  float* out_inv;
  float* alpha_out;
  float* kinv_out;
};

struct LridGradIO {
  const void* grad_output;
  const void* normed_output;
  const float* output_inv_rms;
  void* const* grad_values;
  void* const* grad_keys;
  void* grad_query;
  float* grad_gate;
  void* grad_query_dynamic;
  float* grad_bias;
  void* workspace;
};

// Shared-memory layout of the streaming (bulk-copy) kernels.
struct TmaLayout {
  int stages;       // ring depth
  int stage_bytes;  // bytes per stage: keys [S][tpc][R], values [S][tpc][d], g, y, query
  int off_v, off_g, off_y, off_qd;  // region offsets inside a stage
  int stage_off;    // offset of stage 0 from the start of dynamic shared memory
  int smem_bytes;   // total dynamic shared memory
  int key_lanes;    // lanes per key segment (power of two <= 32)
  int key_packs;    // 16-byte packs per key lane (1 or 4)
};

// Returns 0 and fills *p, or an attnres_status with a message in *why.
int make_lrid_plan(int S, long long N, int d, int R, int H, int dtype, bool full_vec, int out_norm,
                   LridPlan* p, const char** why);
cudaError_t lrid_workspace(int dtype, const LridPlan& p, size_t* bytes);
cudaError_t lrid_forward_launch(int dtype, const LridPlan& p, const LridIO& io, cudaStream_t st);
cudaError_t lrid_backward_launch(int dtype, const LridPlan& p, const LridIO& io,
                                 const LridGradIO& gio, cudaStream_t st);


// Warp-per-token bulk-copy variant (row widths that split into 32-lane chunks per head).
bool lrid_warp_plan(const LridPlan& base, int esz, bool bwd, bool has_y, bool has_qd, int out_norm,
                    TmaLayout* L, int* consumer_warps);
cudaError_t lrid_warp_workspace(int dtype, const LridPlan& p, const TmaLayout& L, int nw, size_t* bytes);
cudaError_t lrid_warp_forward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                     const LridIO& io, cudaStream_t st);
cudaError_t lrid_warp_backward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                      const LridIO& io, const LridGradIO& gio, cudaStream_t st);
cudaError_t read_warp_status(unsigned* status, bool reset);

// Base AttnRes read (keys are the rms-normed values): one value row of d
// columns per token, `tpt` threads per token, `cpt` packs per thread.
struct BasePlan {
  int S, d;
  long long N;
  int vec, nv, tpt, cpt, tpc, wpt;
  long long ntiles;
};

struct BaseIO {
  const void* const* values;
  const int64_t* vstr;
  const void* q;
  int key_norm;
  float key_eps;
  const float* bias;
  int out_norm;
  float out_eps;
  void* out;
  float* out_inv;
  // backward
  const void* grad_output;
  const void* normed_output;
  const float* output_inv_rms;
  void* const* grad_values;
  float* grad_query;
  float* grad_bias;
  void* workspace;
};

int make_base_plan(int S, long long N, int d, int dtype, bool full_vec, BasePlan* p,
                   const char** why);
cudaError_t base_workspace(int dtype, const BasePlan& p, size_t* bytes);
cudaError_t base_forward_launch(int dtype, const BasePlan& p, const BaseIO& io, cudaStream_t st);
cudaError_t base_backward_launch(int dtype, const BasePlan& p, const BaseIO& io, cudaStream_t st);

}  // namespace attnres

namespace attnres {
// out[c] = sum over rows r of partials[r*stride + c0 + c], in a fixed order.
void launch_reduce_partials(const float* partials, int nrows, int stride, int c0, int ncols,
                            float* out, cudaStream_t st);
}  // namespace attnres

namespace attnres {
// Records `msg` as attnres_last_error() for the calling host thread; returns code.
int record_error(int code, const char* msg);
}  // namespace attnres

namespace attnres {
// Key-from-value projection (keyproj.cu).
cudaError_t keyproj_launch(int S, long long N, int d, int R, int dtype, const void* const* values,
                           const int64_t* vstr, const void* w, long long w_stride, int value_norm, float eps,
                           void* keys, float* inv_rms, bool allow_tc, cudaStream_t st, bool* used_tc);
cudaError_t keyproj_bwd_combine_launch(int S, long long N, int d, int R, int H, int dtype,
                                       const void* const* values, const int64_t* vstr,
                                       void* const* grad_values, const void* dn, const void* dk,
                                       const void* keys, const float* inv_rms, const void* g,
                                       const float* alpha, int value_norm, cudaStream_t st);
// Key/query columns of the fused output projection with the per-head key norm
// in the tensor-core kernel's epilogue (keyproj.cu); *eligible = false (nothing
// launched) when the shapes or alignments are outside that kernel.
cudaError_t fused_key_projection_launch(long long N, int din, int rank, int query_rank, int H, int dtype,
                                        const void* x, long long x_stride, const void* w, long long w_stride,
                                        int key_norm, float eps, void* kq, void* key, float* key_inv,
                                        cudaStream_t st, bool* eligible);
cudaError_t read_keyproj_status(unsigned* status, bool reset);

// Fused tcgen05 backward of the key projection (keyproj_bwd.cu). Workspace 0
// means the shapes do not fit the kernel.
size_t keyproj_bwd_tc_workspace(int S, long long N, int d, int R, int H, int dtype);
cudaError_t keyproj_bwd_tc_launch(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                                  const int64_t* vstr, const void* w, long long w_stride,
                                  const void* const* grad_keys, const void* keys, const float* inv_rms,
                                  const void* g, const float* alpha, int value_norm, void* const* grad_values,
                                  float* grad_weight, void* workspace, size_t workspace_bytes, cudaStream_t st);
cudaError_t read_keyproj_bwd_status(unsigned* status, bool reset);

// Key-from-value read backward in one pass over the values (kvbwd.cu): read
// backward, key-norm backward and key-projection backward fused, static query.
// Workspace 0 means the shapes do not fit the kernel.
size_t kvbwd_fused_workspace(int S, long long N, int d, int R, int H, int dtype);
cudaError_t kvbwd_fused_launch(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                               const int64_t* vstr, const void* w, long long w_stride, const void* keys,
                               const float* inv_rms, const float* alpha, const void* query, float scale,
                               int key_norm, float key_eps, const void* g, const void* out,
                               void* const* grad_values, float* grad_weight, float* grad_query,
                               float* grad_bias, void* workspace, size_t workspace_bytes, cudaStream_t st);
cudaError_t read_kvbwd_status(unsigned* status, bool reset);

// Key-from-value read forward in one kernel (kvfused.cu): projection, key
// norm, softmax and weighted sum; saves keys [S][N][64], value inverse rms
// [S][N] and alpha [N][H][S] for the backward.
bool kvfused_eligible(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                      const int64_t* vstr, const void* w, long long w_stride, const char** why);
cudaError_t kvfused_forward_launch(int S, long long N, int d, int H, int dtype, const void* const* values,
                                   const int64_t* vstr, const void* w, long long w_stride, int value_norm,
                                   float value_eps, const void* q, float scale, int key_norm, float key_eps,
                                   const float* bias, void* out, void* keys, float* vinv, float* alpha,
                                   cudaStream_t st);
cudaError_t read_kvfused_status(unsigned* status, bool reset);

// Cached-logit phase 2 (phase2.cu).
size_t phase2_workspace(int mode, long long N, int d, int R);
cudaError_t phase2_run(bool bwd, int mode, long long N, int d, int R, int dtype, const void* v, const void* key,
                       const float* logit, const void* q, float scale, int key_norm, float key_eps, float bias,
                       const float* bias_dev, const void* prev, const float* lse, int onorm, float out_eps,
                       void* out, float* out_inv, const void* g, const void* y, const float* y_inv, void* dv,
                       void* dkey, float* dlogit, void* dprev, float* dlse, float* grad_query, float* grad_bias,
                       void* workspace, cudaStream_t st);

// Per-head key RMS norm (headnorm.cu).
cudaError_t headnorm_launch(bool bwd, int dtype, long long rows, int width, int heads, const void* a, long long as,
                            float eps, const void* b, const float* inv_in, void* out, float* inv_out, long long os,
                            cudaStream_t st);

// Block summary (summary.cu).
int summary_bwd_grid(long long n);
// Block summary with the value norm: forward (bwd false) sum / source / inv,
// backward (bwd true) g_total from g_source, g_sum and the saved sum and inv.
cudaError_t summary_norm_launch(bool bwd, long long rows, int d, int dtype, const void* partial, const void* x,
                                float eps, void* sum, void* source, float* inv, const void* g_source,
                                const void* g_sum, void* g_total, cudaStream_t st);
cudaError_t summary_forward_launch(long long n, int dtype, const void* partial, const void* x,
                                   const float* scale_dev, float scale, void* sum, void* source,
                                   cudaStream_t st);
cudaError_t summary_backward_launch(long long n, int dtype, const void* g_source, const void* g_sum,
                                    const void* sum, const float* scale_dev, float scale, void* g_total,
                                    float* grad_scale, float* partials, cudaStream_t st);
}  // namespace attnres

namespace attnres {
// Cached-logit multi-query read (phase1.cu).
cudaError_t phase1_launch(int dtype, int logit_dtype, int S, int Q, long long N, int d, bool full_vec,
                          const void* const* values, const int64_t* vstr, const void* logits, int out_norm,
                          float out_eps, void* out, float* lse, float* out_inv, const void* g, const void* y,
                          const float* y_inv, const float* glse, void* const* grad_values, void* dlogits,
                          bool bwd, cudaStream_t st);
}  // namespace attnres
