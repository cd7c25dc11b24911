/*
 * attnres_b200.h — C ABI of the B200 (sm_100a) block Attention-Residual
 * depth-routing read ("AttnRes" / low-rank "LRID" read), forward and backward.
 *
 * The ABI takes plain device pointers, element strides and sizes; it never
 * allocates device memory and never synchronises the host. Every call enqueues
 * its kernels on the caller's CUDA stream (`stream` is a cudaStream_t; NULL is
 * the legacy default stream).
 *
 * Geometry used throughout:
 *   S  = num_sources   depth sources read by one residual site (1..ATTNRES_MAX_SOURCES)
 *   N  = num_tokens    token rows (B*T); row n of source s starts at base_s + n*row_stride_s
 *   d  = value_dim     value width, split into H heads of dv = d/H columns
 *   R  = key_dim       low-rank key width, split into H heads of dk = R/H columns
 *   H  = num_heads     depth heads
 *
 * All value/key/query/output tensors of one call share one element type
 * (`dtype`, an attnres_dtype). The last dimension of every source is dense
 * (element stride 1); rows may be strided (e.g. keys that are a column slice of
 * a wider projection). Outputs are dense row-major.
 *
 * Status codes: 0 on success, otherwise an attnres_status; a message for the
 * last failure on the calling host thread is returned by attnres_last_error().
 *
 * Reference interfaces replaced (paths inside jon123boss/LR-AttnRes):
 *   attnres_lrid_forward   <- torch.library op attnres::lrid_read_list
 *                             (attnres_ops.py:4636-4722) and the Triton kernel
 *                             _lrid_attnres_list_read_kernel (attnres_ops.py:331-445),
 *                             plus _lrid_read_list_triton (attnres_ops.py:4533-4629)
 *   attnres_lrid_backward  <- attnres::lrid_read_list_backward (attnres_ops.py:4725-4802),
 *                             _lrid_attnres_list_backward_kernel (attnres_ops.py:602-746)
 *                             and _lrid_read_list_backward_triton (attnres_ops.py:4373-4456)
 *   attnres_base_forward   <- _attnres_read_list_triton / _attnres_list_read_kernel
 *                             (attnres_ops.py:2301-2342, :267-328)
 *   attnres_base_backward  <- _attnres_read_list_backward_triton /
 *                             _attnres_list_backward_kernel (attnres_ops.py:2378-2421, :448-535)
 */
#ifndef ATTNRES_B200_H
#define ATTNRES_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATTNRES_ABI_VERSION 1
#define ATTNRES_MAX_SOURCES 64

typedef enum attnres_dtype {
  ATTNRES_DTYPE_F32 = 0,
  ATTNRES_DTYPE_F16 = 1,
  ATTNRES_DTYPE_BF16 = 2
} attnres_dtype;

typedef enum attnres_status {
  ATTNRES_OK = 0,
  ATTNRES_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad enum */
  ATTNRES_ERR_UNSUPPORTED = 2,      /* shape/alignment outside what the kernels handle */
  ATTNRES_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
  ATTNRES_ERR_WORKSPACE = 4         /* workspace missing or smaller than required */
} attnres_status;

/* How the depth query is formed (model.py:2102-2115 of the reference). */
typedef enum attnres_query_mode {
  ATTNRES_QUERY_STATIC = 0,  /* query [H, dk], shared by all tokens                     */
  ATTNRES_QUERY_DYNAMIC = 1, /* query_dynamic [N, H, dk], one query per token           */
  ATTNRES_QUERY_GATED = 2    /* q_t = query[H,dk] + gate[H] * query_dynamic[N,H,dk]      */
} attnres_query_mode;

/* RMS normalisation of the read output. */
typedef enum attnres_norm_mode {
  ATTNRES_NORM_NONE = 0,
  ATTNRES_NORM_PER_HEAD = 1, /* rms over each head's dv columns; inv-rms saved as [N, H] */
  ATTNRES_NORM_ROW = 2       /* rms over all d columns;          inv-rms saved as [N]    */
} attnres_norm_mode;

int attnres_abi_version(void);
const char* attnres_last_error(void);

/*
 * Health word of the bulk-copy kernels on the current device. A kernel that
 * waits on a shared-memory pipeline barrier gives up after ~2 s instead of
 * hanging, sets a bit here and returns (its outputs are then invalid):
 *   1 = consumers timed out waiting for a stage, 2 = producer timed out
 *   waiting for a stage to drain, 4 = producer timed out draining its copies.
 * Synchronous (reads device memory). reset != 0 clears the word afterwards.
 * No reference counterpart (the reference's Triton kernels have no waits).
 */
int attnres_device_status(unsigned* status, int reset);

/*
 * LRID read, forward. Replaces attnres::lrid_read_list (attnres_ops.py:4636).
 *   logit[n,h,s] = logit_scale * <khat[s,n,h,:], q[n,h,:]> + logit_bias[s]
 *   khat         = key_norm ? k * rsqrt(mean(k^2) + key_eps) : k     (per head of dk)
 *   alpha        = softmax over s (fp32)
 *   out[n,h,:]   = sum_s alpha[n,h,s] * V[s,n,h,:]   (fp32 accumulate, rounded to dtype)
 * query / query_gate / query_dynamic are dtype; unused ones may be NULL.
 * logit_bias: float[S] or NULL. output_inv_rms: float[N,H] (PER_HEAD) or float[N]
 * (ROW) or NULL. alpha_out / key_inv_rms_out: float[N,H,S] or NULL.
 */
int attnres_lrid_forward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                         int num_heads, int dtype,
                         const void* const* values, const int64_t* value_row_strides,
                         const void* const* keys, const int64_t* key_row_strides,
                         int query_mode, const void* query, const void* query_gate,
                         const void* query_dynamic, float logit_scale, int key_norm,
                         float key_eps, const float* logit_bias, int output_norm,
                         float output_eps, void* output, float* output_inv_rms,
                         float* alpha_out, float* key_inv_rms_out, void* stream);

/*
 * Bytes of device workspace attnres_lrid_backward needs for this geometry on
 * the current device (deterministic per-CTA partial sums of the parameter
 * gradients). Returns 0 when the geometry is invalid.
 */
size_t attnres_lrid_backward_workspace_bytes(int num_sources, int64_t num_tokens,
                                             int value_dim, int key_dim, int num_heads,
                                             int dtype);

/*
 * LRID read, backward. Replaces attnres::lrid_read_list_backward (attnres_ops.py:4725).
 * Softmax weights are recomputed from the keys (same arithmetic as the forward).
 *   grad_values[s] : dtype [N, d] dense  = alpha * g'            (g' = output-norm backward of g);
 *                    grad_values == NULL skips these writes (callers that form dV themselves)
 *   grad_keys[s]   : dtype [N, R] dense  = key-norm backward of dlogit*scale*q
 *   grad_query     : STATIC/GATED: float [H, dk] summed over tokens (deterministic order)
 *                    DYNAMIC     : dtype [N, H, dk] per token
 *   grad_query_gate    : GATED only, float [H]
 *   grad_query_dynamic : GATED only, dtype [N, H, dk] (= gate * per-token dq)
 *   grad_logit_bias    : float [S] or NULL
 * normed_output / output_inv_rms: the forward's normalised output and inv-rms,
 * required when output_norm != NONE.
 * The per-token gradients are written once; the summed ones are reduced in a
 * fixed order, so repeated calls are bitwise identical.
 */
int attnres_lrid_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                          int num_heads, int dtype,
                          const void* const* values, const int64_t* value_row_strides,
                          const void* const* keys, const int64_t* key_row_strides,
                          int query_mode, const void* query, const void* query_gate,
                          const void* query_dynamic, float logit_scale, int key_norm,
                          float key_eps, const float* logit_bias, int output_norm,
                          float output_eps, const void* grad_output, const void* normed_output,
                          const float* output_inv_rms, void* const* grad_values,
                          void* const* grad_keys, void* grad_query, float* grad_query_gate,
                          void* grad_query_dynamic, float* grad_logit_bias, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * LRID read backward that allocates nothing: for callers that cannot call
 * cudaMalloc or hand over a device workspace (a custom allocator's own
 * callbacks, plugins that receive only fixed buffers, runtimes that reserve
 * all device memory up front). Same arguments and results as
 * attnres_lrid_backward minus the workspace: the scratch for the parameter
 * gradients' partial sums is a static device array of
 * attnres_noalloc_scratch_bytes() bytes (4 MiB) that every GPU loading the
 * library holds until the process exits. Geometries needing more scratch are
 * rejected with ATTNRES_ERR_UNSUPPORTED. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture. All calls share the one array: calls that
 * overlap on the GPU (other streams, other threads) race on it.
 * No counterpart in the reference.
 */
int attnres_lrid_backward_noalloc(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                  int num_heads, int dtype,
                                  const void* const* values, const int64_t* value_row_strides,
                                  const void* const* keys, const int64_t* key_row_strides,
                                  int query_mode, const void* query, const void* query_gate,
                                  const void* query_dynamic, float logit_scale, int key_norm,
                                  float key_eps, const float* logit_bias, int output_norm,
                                  float output_eps, const void* grad_output,
                                  const void* normed_output, const float* output_inv_rms,
                                  void* const* grad_values, void* const* grad_keys,
                                  void* grad_query, float* grad_query_gate,
                                  void* grad_query_dynamic, float* grad_logit_bias, void* stream);

/* Size in bytes of the static scratch used by attnres_lrid_backward_noalloc. */
size_t attnres_noalloc_scratch_bytes(void);

/*
 * Key-from-value projection of the LRID read (lrid_key_from_value, unshared):
 *   keys[s][n][:] = inv_rms[s][n] * (V_s[n] @ W^T),
 *   inv_rms = value_norm ? rsqrt(mean(V_s[n]^2) + value_eps) : 1
 * i.e. rms_norm(V_s) @ value_key_proj.weight^T. Replaces
 * LRIDFusedProjection.project_key_from_value (model.py:348-356) and the value
 * norm of model.py:344-346. weight: dtype [R, d] (row stride weight_row_stride).
 * keys: dtype [S][N][R] dense; inv_rms: float [S][N] (needed by the backward).
 * bf16/fp16 with d % 64 == 0, R % 16 == 0 (16..256) and 16-byte aligned rows
 * run on tcgen05 tensor cores (TMA-fed, accumulators in TMEM); any other
 * layout on CUDA cores.
 */
int attnres_lrid_key_projection(int num_sources, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                                const void* const* values, const int64_t* value_row_strides,
                                const void* weight, int64_t weight_row_stride, int value_norm,
                                float value_eps, void* keys, float* inv_rms, void* stream);

/*
 * Backward of the value rms-norm in the key projection, combined into
 * grad_values (dense [N, d] each):
 *   grad_values[s][n] = base + inv * (dn - (V*inv) * <dK, key> / d)
 * grad_normed = dn = dK @ W: dtype [S][N][d]; grad_keys = dK: dtype [S][N][R];
 * keys / inv_rms: the forward's outputs. base = alpha[n,h,s] * grad_output[n]
 * when grad_output (dtype [N, d]) and alpha (float [N, H, S], the forward's
 * softmax weights) are given -- the read backward then runs with
 * grad_values == NULL -- otherwise the current grad_values (read-modify-write).
 * The weight gradient sum_s (inv_s * dK_s)^T @ V_s is a plain GEMM left to
 * the caller. Replaces the autograd backward of model.py:344-356.
 */
int attnres_lrid_key_projection_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                         int num_heads, int dtype, const void* const* values,
                                         const int64_t* value_row_strides, void* const* grad_values,
                                         const void* grad_normed, const void* grad_keys, const void* keys,
                                         const float* inv_rms, const void* grad_output, const float* alpha,
                                         int value_norm, void* stream);

/*
 * Key-from-value LRID read, forward, in one kernel (replaces the reference's
 * LRIDFusedProjection.project_key_from_value, model.py:344-356, followed by
 * lrid_attention_residual_read, attnres_ops.py:4852): per source
 *   keys_s = rms_norm(V_s) @ weight^T  (value_norm; eps = value_eps)
 * rounded to the value dtype, then the LRID read with per-head key norm,
 * static query [num_heads, key_dim / num_heads], logit_scale, optional
 * logit_bias [S] and no output norm. Writes output [N, value_dim], keys
 * [S][N][key_dim] (dtype), value_inv_rms [S][N] (may be NULL without
 * value_norm) and alpha_out [N][num_heads][S] (float, may be NULL) -- what
 * attnres_lrid_backward (grad_values = NULL) and
 * attnres_lrid_key_projection_backward_tc need. f16/bf16, key_dim 64, 2..32
 * sources, value_dim and value_dim / num_heads multiples of 64, num_heads a
 * power of two <= 8, 16-byte aligned rows; other shapes return
 * ATTNRES_ERR_UNSUPPORTED (use attnres_lrid_key_projection +
 * attnres_lrid_forward).
 */
int attnres_lrid_key_from_value_forward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                        int num_heads, int dtype, const void* const* values,
                                        const int64_t* value_row_strides, const void* weight,
                                        int64_t weight_row_stride, int value_norm, float value_eps,
                                        const void* query, float logit_scale, int key_norm, float key_eps,
                                        const float* logit_bias, void* output, void* keys, float* value_inv_rms,
                                        float* alpha_out, void* stream);

/*
 * Fused backward of the key projection on the tensor cores, for the one-pass
 * key-from-value read backward (the read ran with grad_values == NULL):
 *   dKs = inv * dK,  coef = inv * <dKs, key> / d
 *   grad_values[s][n] = alpha[n,h,s] * grad_output[n] + (dKs_s @ W)[n] - V_s[n] * coef[s][n]
 *   grad_weight (float [R][d], overwritten) = sum_s dKs_s^T @ V_s
 * grad_keys: one dtype [N, R] dense array per source; keys dtype [S][N][R];
 * weight: dtype [R, d] with row stride weight_row_stride. f16/bf16, R == 64,
 * (value_dim / num_heads) % 128 == 0, num_sources <= 24. The workspace query
 * returns 0 when the shapes do not fit (use attnres_lrid_key_projection_backward
 * with a separate dn = dK @ W then). Deterministic. Replaces the autograd
 * backward of model.py:344-356 (rms_norm + value_key_proj), weight gradient
 * included.
 */
size_t attnres_lrid_key_projection_backward_tc_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                                               int key_dim, int num_heads, int dtype);
int attnres_lrid_key_projection_backward_tc(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                            int num_heads, int dtype, const void* const* values,
                                            const int64_t* value_row_strides, const void* weight,
                                            int64_t weight_row_stride, const void* const* grad_keys,
                                            const void* keys, const float* inv_rms, const void* grad_output,
                                            const float* alpha, int value_norm, void* const* grad_values,
                                            float* grad_weight, void* workspace, size_t workspace_bytes,
                                            void* stream);

/*
 * Key-from-value LRID read backward in one pass over the values (static query,
 * no output norm): the read backward, the key RMS-norm backward and the key
 * projection backward fused, so each value row is read once and each value
 * gradient row written once. keys dtype [S][N][R] and alpha float [N][H][S]
 * as saved by the forward (attnres_lrid_key_projection + attnres_lrid_forward,
 * or attnres_lrid_key_from_value_forward); output dtype [N][value_dim] is the
 * forward's output; query dtype [num_heads * key_dim / num_heads].
 *   grad_values[s][n]     = alpha g + dKs_s @ W - V_s coef  (dtype, written)
 *   grad_weight [R][d]    = sum_s dKs_s^T @ V_s            (float, overwritten)
 *   grad_query [R]        = summed query gradient           (float, overwritten)
 *   grad_logit_bias [S]   = summed bias gradient, or NULL   (float, overwritten)
 * The softmax backward uses sum_j alpha_j <g, V_j> = <g, output>, so the
 * 16-bit output's rounding enters the logit gradient (well inside the 16-bit
 * tolerance). f16/bf16, key_dim 64, 2..24 sources, num_heads 1/2/4/8,
 * value_dim / num_heads a multiple of 256, value_dim <= 4096; the workspace
 * query returns 0 otherwise (use the read backward followed by
 * attnres_lrid_key_projection_backward_tc). Deterministic. Launched as
 * thread-block clusters of value_dim / 128 CTAs (16, a non-portable cluster
 * size, for value_dim 2048) that exchange partial dots through distributed
 * shared memory; a wait that runs out (~2 s) sets a bit in
 * attnres_device_status(). Measured slower than the two-kernel path at config
 * 4 (12-16 ms against 5.4 ms): the exchange round trip keeps each ring stage
 * resident too long. Replaces the autograd backward of the read
 * (attnres_ops.py:4725, lrid_read_list_backward) together with that of
 * model.py:344-356 (rms_norm + value_key_proj).
 */
size_t attnres_lrid_key_from_value_backward_workspace_bytes(int num_sources, int64_t num_tokens, int value_dim,
                                                             int key_dim, int num_heads, int dtype);
int attnres_lrid_key_from_value_backward(int num_sources, int64_t num_tokens, int value_dim, int key_dim,
                                         int num_heads, int dtype, const void* const* values,
                                         const int64_t* value_row_strides, const void* weight,
                                         int64_t weight_row_stride, const void* keys, int value_norm,
                                         const float* value_inv_rms, const float* alpha, const void* query,
                                         float logit_scale, int key_norm, float key_eps, const void* grad_output,
                                         const void* output, void* const* grad_values, float* grad_weight,
                                         float* grad_query, float* grad_logit_bias, void* workspace,
                                         size_t workspace_bytes, void* stream);

/*
 * Block summary of block Attention Residuals, one pass over the rows:
 *   sum = partial + x (partial may be NULL),  source = sum * c
 * with c = *scale_device when scale_device is not NULL (a learned scale,
 * already in the value dtype's precision), else `scale` (count^-alpha).
 * sum may be NULL when only the source is wanted. dtype arrays of
 * num_elements elements. Replaces the running sum and the
 * _attnres_block_summary / _lrid_block_source value scaling of
 * model.py:990-1028 (call sites model.py:2377-2389, :2451-2463).
 */
int attnres_block_summary_forward(int64_t num_elements, int dtype, const void* partial, const void* x,
                                  const float* scale_device, float scale, void* sum, void* source,
                                  void* stream);
/*
 * Backward: grad_partial (the gradient of both partial and x) =
 * round(round(grad_source * c) + grad_sum); either input may be NULL. With
 * grad_scale (float, one element) the scale gradient sum(grad_source * sum)
 * is reduced deterministically using a workspace of
 * attnres_block_summary_backward_workspace_bytes(num_elements) bytes.
 */
size_t attnres_block_summary_backward_workspace_bytes(int64_t num_elements);
int attnres_block_summary_backward(int64_t num_elements, int dtype, const void* grad_source, const void* grad_sum,
                                   const void* sum, const float* scale_device, float scale, void* grad_partial,
                                   float* grad_scale, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Block summary with the value norm (attnres_block_value_norm): the block
 * source is the RMS-normed running sum instead of the scaled one
 * (model.py:991-992, :1004-1005; replaces F.rms_norm(partial + x)):
 *   sum = partial + x (partial may be NULL),  source = rms_norm(sum)
 * over rows of row_width elements, eps = `eps` (F.rms_norm's default is the
 * fp32 eps for fp32, fp16 and bf16 rows). inv_rms (float, num_rows) receives
 * each row's inverse rms for the backward; sum may be NULL.
 */
int attnres_block_summary_norm_forward(int64_t num_rows, int row_width, int dtype, const void* partial,
                                       const void* x, float eps, void* sum, void* source, float* inv_rms,
                                       void* stream);
/*
 * Backward of the above: grad_total (the gradient of both partial and x) =
 * round(round(rms_norm_backward(grad_source)) + grad_sum), from the saved sum
 * and inv_rms; grad_sum may be NULL.
 */
int attnres_block_summary_norm_backward(int64_t num_rows, int row_width, int dtype, const void* grad_source,
                                        const void* grad_sum, const void* sum, const float* inv_rms,
                                        void* grad_total, void* stream);

/*
 * Key/query columns of the fused output projection with the key norm in the
 * GEMM's epilogue: key_query[n, :] = round(x[n, :] @ weight^T) for the
 * rank + query_rank rows of weight (the projection weight's rows after the
 * output columns); with key_norm, key[n, h*dk + j] = round(kq[n, h*dk + j] *
 * inv[n, h]), inv = rsqrt(mean_j kq[n, h*dk + j]^2 + eps) over the rounded
 * values, dk = rank / num_heads, and key_inv_rms float [N, num_heads].
 * key_query dtype [N, rank + query_rank] dense, key dtype [N, rank] dense.
 * Replaces, for the key and query columns, the F.linear of
 * LRIDFusedProjection.forward (model.py:363-374) and _norm_lrid_key
 * (model.py:33-36) as applied at model.py:375-379; the output columns stay a
 * plain GEMM. tcgen05 tensor cores (TMA-fed, accumulators in TMEM, the norm
 * from TMEM in the epilogue); returns ATTNRES_ERR_UNSUPPORTED, launching
 * nothing, unless: bf16/fp16, in_dim % 64 == 0, rank + query_rank a multiple
 * of 16 in [16, 256], dk % 16 == 0 with key_norm, 16-byte aligned rows.
 */
int attnres_lrid_fused_key_projection(int64_t num_tokens, int in_dim, int rank, int query_rank, int num_heads,
                                      int dtype, const void* x, int64_t x_row_stride, const void* weight,
                                      int64_t weight_row_stride, int key_norm, float eps, void* key_query,
                                      void* key, float* key_inv_rms, void* stream);

/*
 * Per-head RMS norm of key rows: y[r, h*dk + j] = x[r, h*dk + j] * inv_rms[r, h],
 * inv_rms = rsqrt(mean_j x^2 + eps), dk = width / num_heads, fp32 math, y and
 * grad dense [rows, width]; x may be a strided slice (x_row_stride elements),
 * e.g. the key columns of a projection output. inv_rms float [rows, num_heads]
 * (may be NULL in the forward). Backward: grad_x = inv * (grad_y - y <grad_y, y> / dk)
 * with y = x * inv recomputed in fp32 from the pre-norm rows x (row stride
 * x_row_stride), written with row stride grad_x_row_stride. Replaces _norm_lrid_key
 * (model.py:33-36) as LRIDFusedProjection.forward applies it (model.py:375-379).
 */
int attnres_head_rms_norm_forward(int64_t rows, int width, int num_heads, int dtype, const void* x,
                                  int64_t x_row_stride, float eps, void* y, float* inv_rms, void* stream);
int attnres_head_rms_norm_backward(int64_t rows, int width, int num_heads, int dtype, const void* grad_y,
                                   const void* x, int64_t x_row_stride, const float* inv_rms, void* grad_x,
                                   int64_t grad_x_row_stride, void* stream);

/* Phase-2 key modes: the partial block's logit from an LRID key, from the base
 * key rms_norm(partial_value), or given. */
enum { ATTNRES_PHASE2_LRID = 0, ATTNRES_PHASE2_BASE = 1, ATTNRES_PHASE2_LOGIT = 2 };

/*
 * Cached-logit phase 2: merge the live partial block into the phase-1 result.
 *   logit = scale * <k_hat, query> + bias   (LRID: k = partial_key [N, key_dim],
 *           scale = logit_scale; BASE: k = partial_value, scale 1; LOGIT: given
 *           float partial_logit [N]); k_hat = rms-normalised k when key_norm
 *   p = sigmoid(logit - interblock_lse[n]),  out = prev + p * (partial - prev)
 * optionally rms-normalised per row (output_inv_rms float [N] then written).
 * partial_value, interblock_output, output: dtype [N, value_dim] dense;
 * query: dtype [key_dim] (LRID) or [value_dim] (BASE); bias = *logit_bias_device
 * when not NULL, else logit_bias. Replaces lrid_attention_residual_phase2
 * (attnres_ops.py:4075-4139), attention_residual_phase2 (:3964-4019) and
 * attention_residual_phase2_from_logit (:4043-4072).
 */
int attnres_phase2_forward(int mode, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                           const void* partial_value, const void* partial_key, const float* partial_logit,
                           const void* query, float logit_scale, int key_norm, float key_eps, float logit_bias,
                           const float* logit_bias_device, const void* interblock_output,
                           const float* interblock_lse, int normalize_output, float output_eps, void* output,
                           float* output_inv_rms, void* stream);
/*
 * Phase-2 backward. grad_partial_value / grad_interblock_output: dtype [N, value_dim];
 * grad_interblock_lse: float [N]; grad_partial_key (LRID): dtype [N, key_dim];
 * grad_partial_logit (LOGIT): float [N]; grad_query (float [key_dim] or
 * [value_dim]) and grad_bias (float, one element) may be NULL and are summed
 * over tokens in a fixed order (deterministic) with a workspace of
 * attnres_phase2_backward_workspace_bytes(...) bytes. With normalize_output the
 * forward's output and output_inv_rms are passed back. Replaces the autograd
 * backward of the same functions (Triton kernel attnres_ops.py:2058-2121).
 */
size_t attnres_phase2_backward_workspace_bytes(int mode, int64_t num_tokens, int value_dim, int key_dim);
int attnres_phase2_backward(int mode, int64_t num_tokens, int value_dim, int key_dim, int dtype,
                            const void* partial_value, const void* partial_key, const float* partial_logit,
                            const void* query, float logit_scale, int key_norm, float key_eps, float logit_bias,
                            const float* logit_bias_device, const void* interblock_output,
                            const float* interblock_lse, int normalize_output, const void* output,
                            const float* output_inv_rms, const void* grad_output, void* grad_partial_value,
                            void* grad_partial_key, float* grad_partial_logit, void* grad_interblock_output,
                            float* grad_interblock_lse, float* grad_query, float* grad_bias, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Cached-logit block read ("phase 1"): Q reads of the same S sources whose
 * logits were computed once. Replaces attention_residual_phase1_from_logits
 * (attnres_ops.py:3910-3961) and its Triton kernels (:933-989, :1069-1140).
 *   alpha = softmax over s of logits[q][:][n]; output[q][n] = sum_s alpha V_s[n]
 *   lse[q][n] = logsumexp over s;  optional rms norm of each output row (ROW)
 * logits: logit_dtype [Q][S][N] dense; output: dtype [Q][N][d] dense;
 * lse, output_inv_rms: float [Q][N]. Q <= 16.
 */
int attnres_phase1_forward(int num_sources, int num_queries, int64_t num_tokens, int value_dim, int dtype,
                           const void* const* values, const int64_t* value_row_strides, const void* logits,
                           int logit_dtype, int output_norm, float output_eps, void* output, float* lse,
                           float* output_inv_rms, void* stream);

/*
 * Phase-1 backward: grad_values[s] (dtype [N, d] dense) = sum_q alpha g'_q;
 * grad_logits (logit_dtype [Q][S][N]) = alpha * (<g'_q, V_s> - sum_r alpha <g'_q, V_r>)
 *                                       + grad_lse[q][n] * alpha   (grad_lse may be NULL).
 */
int attnres_phase1_backward(int num_sources, int num_queries, int64_t num_tokens, int value_dim, int dtype,
                            const void* const* values, const int64_t* value_row_strides, const void* logits,
                            int logit_dtype, int output_norm, float output_eps, const void* grad_output,
                            const float* grad_lse, const void* normed_output, const float* output_inv_rms,
                            void* const* grad_values, void* grad_logits, void* stream);

/*
 * Base AttnRes read, forward (keys are the values themselves).
 * Replaces _attnres_read_list_triton (attnres_ops.py:2301) /
 * _attnres_list_read_kernel (attnres_ops.py:267).
 *   khat = key_norm ? v * rsqrt(mean(v^2) + key_eps) : v ;  logit = <khat, query> + bias
 * query: dtype [d]. output_norm: NONE or ROW; output_inv_rms float[N] or NULL.
 */
int attnres_base_forward(int num_sources, int64_t num_tokens, int value_dim, int dtype,
                         const void* const* values, const int64_t* value_row_strides,
                         const void* query, int key_norm, float key_eps,
                         const float* logit_bias, int output_norm, float output_eps,
                         void* output, float* output_inv_rms, void* stream);

size_t attnres_base_backward_workspace_bytes(int num_sources, int64_t num_tokens,
                                             int value_dim, int dtype);

/*
 * Base AttnRes read, backward. Replaces _attnres_read_list_backward_triton
 * (attnres_ops.py:2378) / _attnres_list_backward_kernel (attnres_ops.py:448).
 *   grad_values[s] : dtype [N, d] dense = alpha*g' + key-norm backward of dlogit*q
 *   grad_query     : float [d] summed over tokens in a fixed order
 */
int attnres_base_backward(int num_sources, int64_t num_tokens, int value_dim, int dtype,
                          const void* const* values, const int64_t* value_row_strides,
                          const void* query, int key_norm, float key_eps,
                          const float* logit_bias, int output_norm, float output_eps,
                          const void* grad_output, const void* normed_output,
                          const float* output_inv_rms, void* const* grad_values,
                          float* grad_query, float* grad_logit_bias, void* workspace,
                          size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTNRES_B200_H */
