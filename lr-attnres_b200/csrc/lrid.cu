// LRID (low-rank key) block Attention-Residual read: forward and backward.
//
// Semantics follow the reference's unfused PyTorch path
// (_lrid_read_torch_list, attnres_ops.py:4195-4232) and its Triton kernels
// (_lrid_attnres_list_read_kernel attnres_ops.py:331-445,
//  _lrid_attnres_list_backward_kernel attnres_ops.py:602-746), with all
// arithmetic in fp32.
//
// Work decomposition (one CTA = `tpc` token rows, persistent grid):
//   * value threads: each token row gets `tpt` threads; head h owns `tph`
//     consecutive threads, each streaming VEC-wide packs of the head's dv
//     columns (cph packs per thread) from every source row.
//   * key threads: the same threads re-mapped as `lph` lanes per head; lane l
//     owns key elements l, l+lph, ... of the head's dk columns, so a head's
//     sum-of-squares and query dot are `lph`-lane butterfly sums.
//   * per (token, head): softmax over the S sources by one warp, lane = source.
// The backward writes per-CTA partial sums of the parameter gradients (static
// query, gate, logit bias) into a workspace; attnres_reduce_partials() sums
// them in a fixed order, so the result is bitwise reproducible.
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "plan.h"
#include "lrid_args.cuh"
#include "launch_cache.h"

namespace attnres {


// Sum over the `gsz` consecutive threads of an aligned group (gsz a power of
// two). Groups wider than a warp combine per-warp sums through `red` in warp
// order. Every thread of the CTA must call with the same gsz.
__device__ __forceinline__ float block_group_sum(float v, int gsz, float* red) {
  if (gsz <= 32) return group_sum(v, gsz);
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int nw = gsz >> 5;
  const int w0 = (threadIdx.x / gsz) * nw;
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w0 + w];
  __syncthreads();
  return tot;
}

constexpr int kSrcBatch = 8;  // source rows loaded back-to-back per thread

// Packed (VEC > 1) variants run at most 256 threads per CTA, which leaves the
// register file to the unrolled source batches; the element-wise fallback for
// unaligned rows may need up to 1024.
template <typename T, int VEC, int MAXC, int KPLMAX, bool BWD>
__global__ void __launch_bounds__(VEC > 1 ? 256 : 1024) lrid_kernel(const __grid_constant__ LridArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const LridPlan& P = a.p;
  const int S = P.S, H = P.H, dk = P.dk, dv = P.dv, d = P.d, R = P.R;
  const int tpt = P.tpt, tpc = P.tpc, tph = P.tph, lph = P.lph, kpl = P.kpl, cph = P.cph;
  const int nvh = P.nvh, wph = P.wph;

  // source table copied to shared memory (uniform, broadcast reads)
  const T** sv = reinterpret_cast<const T**>(smem_raw);
  const T** sk = sv + S;
  long long* svs = reinterpret_cast<long long*>(sk + S);
  long long* sks = svs + S;
  T** sgv = reinterpret_cast<T**>(sks + S);
  T** sgk = sgv + S;
  float* fs = reinterpret_cast<float*>(sgk + S);
  const int A = tpc * H * S;
  float* sm_logit = fs;         // logits, then dlogits (backward)
  float* sm_alpha = fs + A;
  float* sm_kinv = fs + 2 * A;
  float* sm_qk = fs + 3 * A;    // <q, khat> per (token, head, source)
  float* sm_dwp = fs + 4 * A;   // backward: per-warp partial <g', v_s>
  float* sm_red = sm_dwp + (BWD ? A * wph : 0);
  float* sm_dqe = sm_red + (blockDim.x >> 5);
  float* sm_gate = sm_dqe + tpc * R;

  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    sv[i] = static_cast<const T*>(a.v[i]);
    sk[i] = static_cast<const T*>(a.k[i]);
    svs[i] = a.vs[i];
    sks[i] = a.ks[i];
    if (BWD) {
      sgv[i] = static_cast<T*>(a.gv[i]);
      sgk[i] = static_cast<T*>(a.gk[i]);
    }
  }
  __syncthreads();

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int slot = tid / tpt, it = tid % tpt;
  const int kh = it / lph, kl = it % lph;
  const bool kvalid = kh < H;
  const bool kwarp = ((it & ~31) / lph) < H;
  const int vh = it / tph, vj = it % tph;
  const bool vvalid = vh < H;
  const int hgrp = P.out_norm_group;  // threads per output-norm group
  const int width = (a.out_norm == ATTNRES_NORM_ROW) ? d : dv;

  const T* qp = static_cast<const T*>(a.q);
  const T* qdp = static_cast<const T*>(a.qdyn);
  float qs[KPLMAX];
#pragma unroll
  for (int i = 0; i < KPLMAX; ++i) {
    const int e = kl + i * lph;
    qs[i] = (a.qmode != ATTNRES_QUERY_DYNAMIC && kvalid && i < kpl && e < dk)
                ? load_f(qp + kh * dk + e)
                : 0.f;
  }
  const float gate_h =
      (a.qmode == ATTNRES_QUERY_GATED && kvalid) ? load_f(static_cast<const T*>(a.gate) + kh) : 0.f;

  float dq_acc[KPLMAX];
#pragma unroll
  for (int i = 0; i < KPLMAX; ++i) dq_acc[i] = 0.f;
  float dgate_acc = 0.f, dbias_acc = 0.f;

  for (long long tile = blockIdx.x; tile < P.ntiles; tile += gridDim.x) {
    const long long t = tile * tpc + slot;
    const bool tv = t < P.N;

    // ---- per-token query (dynamic / gated) -------------------------------
    float q[KPLMAX], qd[KPLMAX];
#pragma unroll
    for (int i = 0; i < KPLMAX; ++i) {
      const int e = kl + i * lph;
      qd[i] = 0.f;
      if (a.qmode != ATTNRES_QUERY_STATIC && kvalid && tv && i < kpl && e < dk)
        qd[i] = load_f(qdp + t * R + kh * dk + e);
      q[i] = (a.qmode == ATTNRES_QUERY_STATIC) ? qs[i]
             : (a.qmode == ATTNRES_QUERY_DYNAMIC) ? qd[i]
                                                  : qs[i] + gate_h * qd[i];
    }

    // ---- key phase: key rms-norm, logits ----------------------------------
    if (kwarp) {
      for (int s = 0; s < S; ++s) {
        const T* kp = sk[s] + t * sks[s] + kh * dk;
        float ss = 0.f, dot = 0.f;
#pragma unroll
        for (int i = 0; i < KPLMAX; ++i) {
          const int e = kl + i * lph;
          if (i < kpl && kvalid && tv && e < dk) {
            const float x = load_f(kp + e);
            ss = fmaf(x, x, ss);
            dot = fmaf(x, q[i], dot);
          }
        }
        ss = group_sum(ss, lph);
        dot = group_sum(dot, lph);
        if (kvalid && kl == 0) {
          const float kinv = a.key_norm ? rsqrtf(ss / dk + a.key_eps) : 1.f;
          const float qk = dot * kinv;
          const int idx = (slot * H + kh) * S + s;
          sm_logit[idx] = qk * a.scale + (a.bias ? a.bias[s] : 0.f);
          sm_kinv[idx] = kinv;
          sm_qk[idx] = qk;
        }
      }
    }
    __syncthreads();

    // ---- softmax over sources: one warp per (token, head) ------------------
    for (int pair = warp; pair < tpc * H; pair += nwarps) {
      const int base = pair * S;
      const long long tp = tile * tpc + pair / H;
      const int h = pair % H;
      float m = -INFINITY;
      for (int s = lane; s < S; s += 32) m = fmaxf(m, sm_logit[base + s]);
      m = warp_max(m);
      float sum = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float e = expf(sm_logit[base + s] - m);
        sm_alpha[base + s] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      for (int s = lane; s < S; s += 32) {
        const float al = sm_alpha[base + s] / sum;
        sm_alpha[base + s] = al;
        if (!BWD && tp < P.N) {
          if (a.alpha_out) a.alpha_out[(tp * H + h) * S + s] = al;
          if (a.kinv_out) a.kinv_out[(tp * H + h) * S + s] = sm_kinv[base + s];
        }
      }
    }
    __syncthreads();

    const float* al = sm_alpha + (slot * H + (vvalid ? vh : 0)) * S;

    if constexpr (!BWD) {
      // ---- forward value phase: out = sum_s alpha_s * V_s ------------------
      T* outp = static_cast<T*>(a.out);
      float acc[MAXC][VEC];
      float ssq = 0.f;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[c][e] = 0.f;
        const int vidx = vj + c * tph;
        if (c < cph && vvalid && tv && vidx < nvh) {
          const int col = vh * dv + vidx * VEC;
          for (int s0 = 0; s0 < S; s0 += kSrcBatch) {
            Pack<T, VEC> r[kSrcBatch];
#pragma unroll
            for (int j = 0; j < kSrcBatch; ++j)
              if (s0 + j < S) r[j] = load_stream<T, VEC>(sv[s0 + j] + t * svs[s0 + j] + col);
#pragma unroll
            for (int j = 0; j < kSrcBatch; ++j) {
              if (s0 + j < S) {
                const float w = al[s0 + j];
#pragma unroll
                for (int e = 0; e < VEC; ++e) acc[c][e] = fmaf(w, Elem<T>::to_f(r[j].e[e]), acc[c][e]);
              }
            }
          }
          if (a.out_norm == ATTNRES_NORM_NONE) {
            store_pack<T, VEC>(outp + t * d + col, acc[c]);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) ssq = fmaf(acc[c][e], acc[c][e], ssq);
          }
        }
      }
      if (a.out_norm != ATTNRES_NORM_NONE) {
        const float tot = block_group_sum(ssq, hgrp, sm_red);
        const float inv = rsqrtf(tot / width + a.out_eps);
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int vidx = vj + c * tph;
          if (c < cph && vvalid && tv && vidx < nvh) {
            const int col = vh * dv + vidx * VEC;
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[c][e] *= inv;
            store_pack<T, VEC>(outp + t * d + col, acc[c]);
          }
        }
        if (a.out_inv && tv && vvalid && vj == 0) {
          if (a.out_norm == ATTNRES_NORM_PER_HEAD) a.out_inv[t * H + vh] = inv;
          else if (vh == 0) a.out_inv[t] = inv;
        }
      }
    } else {
      // ---- backward value phase -------------------------------------------
      const T* gp_ = static_cast<const T*>(a.g);
      const T* yp_ = static_cast<const T*>(a.y);
      float gp[MAXC][VEC], yv[MAXC][VEC];
      float gy = 0.f;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int vidx = vj + c * tph;
#pragma unroll
        for (int e = 0; e < VEC; ++e) gp[c][e] = yv[c][e] = 0.f;
        if (c < cph && vvalid && tv && vidx < nvh) {
          const int col = vh * dv + vidx * VEC;
          const Pack<T, VEC> gr = load_pack<T, VEC>(gp_ + t * d + col);
#pragma unroll
          for (int e = 0; e < VEC; ++e) gp[c][e] = Elem<T>::to_f(gr.e[e]);
          if (a.out_norm != ATTNRES_NORM_NONE) {
            const Pack<T, VEC> yr = load_pack<T, VEC>(yp_ + t * d + col);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              yv[c][e] = Elem<T>::to_f(yr.e[e]);
              gy = fmaf(gp[c][e], yv[c][e], gy);
            }
          }
        }
      }
      if (a.out_norm != ATTNRES_NORM_NONE) {
        const float tot = block_group_sum(gy, hgrp, sm_red);
        float inv = 0.f;
        if (tv && vvalid)
          inv = (a.out_norm == ATTNRES_NORM_PER_HEAD) ? a.y_inv[t * H + vh] : a.y_inv[t];
        const float mdot = tot / width;
#pragma unroll
        for (int c = 0; c < MAXC; ++c)
#pragma unroll
          for (int e = 0; e < VEC; ++e) gp[c][e] = inv * (gp[c][e] - yv[c][e] * mdot);
      }

      const int rg = tph < 32 ? tph : 32;
      for (int s0 = 0; s0 < S; s0 += kSrcBatch) {
        Pack<T, VEC> r[kSrcBatch][MAXC];
#pragma unroll
        for (int j = 0; j < kSrcBatch; ++j)
#pragma unroll
          for (int c = 0; c < MAXC; ++c) {
            const int vidx = vj + c * tph;
            if (s0 + j < S && c < cph && vvalid && tv && vidx < nvh)
              r[j][c] = load_stream<T, VEC>(sv[s0 + j] + t * svs[s0 + j] + vh * dv + vidx * VEC);
          }
#pragma unroll
        for (int j = 0; j < kSrcBatch; ++j) {
          if (s0 + j < S) {
            const int s = s0 + j;
            const float w = vvalid ? al[s] : 0.f;
            float dwp = 0.f;
#pragma unroll
            for (int c = 0; c < MAXC; ++c) {
              const int vidx = vj + c * tph;
              if (c < cph && vvalid && tv && vidx < nvh) {
                float gvv[VEC];
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  dwp = fmaf(gp[c][e], Elem<T>::to_f(r[j][c].e[e]), dwp);
                  gvv[e] = w * gp[c][e];
                }
                if (sgv[s]) store_pack<T, VEC>(sgv[s] + t * d + vh * dv + vidx * VEC, gvv);
              }
            }
            dwp = group_sum(dwp, rg);
            if ((vj & 31) == 0 && vvalid) sm_dwp[((slot * H + vh) * S + s) * wph + (vj >> 5)] = dwp;
          }
        }
      }
      __syncthreads();

      // ---- dlogit_s = alpha_s (dw_s - sum_r alpha_r dw_r) -------------------
      for (int pair = warp; pair < tpc * H; pair += nwarps) {
        const int base = pair * S;
        const long long tp = tile * tpc + pair / H;
        float part = 0.f;
        for (int s = lane; s < S; s += 32) {
          float dw = 0.f;
          for (int w = 0; w < wph; ++w) dw += sm_dwp[(base + s) * wph + w];
          sm_dwp[(base + s) * wph] = dw;
          part = fmaf(sm_alpha[base + s], dw, part);
        }
        const float wd = warp_sum(part);
        for (int s = lane; s < S; s += 32) {
          const float alp = sm_alpha[base + s];
          sm_logit[base + s] = (tp < P.N) ? alp * (sm_dwp[(base + s) * wph] - wd) : 0.f;
        }
      }
      __syncthreads();

      if (a.want_bias_grad && tid < S)
        for (int pair = 0; pair < tpc * H; ++pair) dbias_acc += sm_logit[pair * S + tid];

      // ---- key phase 2: dK, dq --------------------------------------------
      if (kwarp) {
        float dqt[KPLMAX];
#pragma unroll
        for (int i = 0; i < KPLMAX; ++i) dqt[i] = 0.f;
        for (int s = 0; s < S; ++s) {
          const int idx = (slot * H + (kvalid ? kh : 0)) * S + s;
          const float c1 = sm_logit[idx] * a.scale;
          const float kinv = sm_kinv[idx];
          const float c2 = a.key_norm ? c1 * sm_qk[idx] / dk : 0.f;
          const T* kp = sk[s] + t * sks[s] + kh * dk;
          T* gkp = sgk[s] + t * R + kh * dk;
#pragma unroll
          for (int i = 0; i < KPLMAX; ++i) {
            const int e = kl + i * lph;
            if (i < kpl && kvalid && tv && e < dk) {
              const float khat = load_f(kp + e) * kinv;
              const float gk = c1 * q[i];
              const float dkv = a.key_norm ? kinv * (gk - khat * c2) : gk;
              gkp[e] = Elem<T>::from_f(dkv);
              dqt[i] = fmaf(c1, khat, dqt[i]);
            }
          }
        }
        T* dqp = static_cast<T*>(a.dq_tok);
#pragma unroll
        for (int i = 0; i < KPLMAX; ++i) {
          const int e = kl + i * lph;
          if (i < kpl && kvalid && tv && e < dk) {
            if (a.qmode == ATTNRES_QUERY_STATIC) {
              dq_acc[i] += dqt[i];
            } else if (a.qmode == ATTNRES_QUERY_DYNAMIC) {
              dqp[t * R + kh * dk + e] = Elem<T>::from_f(dqt[i]);
            } else {
              dqp[t * R + kh * dk + e] = Elem<T>::from_f(gate_h * dqt[i]);
              dq_acc[i] += dqt[i];
              dgate_acc = fmaf(dqt[i], qd[i], dgate_acc);
            }
          }
        }
      }
    }
    __syncthreads();
  }

  if constexpr (BWD) {
    // ---- per-CTA partial sums of the parameter gradients, fixed order -------
    if (a.partials == nullptr) return;
    for (int i = tid; i < tpc * R; i += blockDim.x) sm_dqe[i] = 0.f;
    __syncthreads();
    if (kvalid) {
#pragma unroll
      for (int i = 0; i < KPLMAX; ++i) {
        const int e = kl + i * lph;
        if (i < kpl && e < dk) sm_dqe[slot * R + kh * dk + e] = dq_acc[i];
      }
    }
    const float gsum = group_sum(dgate_acc, lph);
    if (kvalid && kl == 0) sm_gate[slot * H + kh] = gsum;
    __syncthreads();
    float* row = a.partials + static_cast<long long>(blockIdx.x) * a.part_stride;
    for (int e = tid; e < R; e += blockDim.x) {
      float s = 0.f;
      for (int sl = 0; sl < tpc; ++sl) s += sm_dqe[sl * R + e];
      row[e] = s;
    }
    for (int h = tid; h < H; h += blockDim.x) {
      float s = 0.f;
      for (int sl = 0; sl < tpc; ++sl) s += sm_gate[sl * H + h];
      row[R + h] = s;
    }
    if (tid < S) row[R + H + tid] = dbias_acc;
  }
}

// Fixed-order sum of per-CTA partial rows: out[c] = sum_r partials[r][c].
// One CTA per column; thread i takes rows i, i+256, ...; then a fixed tree.
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partials,
                                                              int nrows, int stride, int c0,
                                                              int ncols, float* __restrict__ out) {
  __shared__ float red[256];
  const int c = blockIdx.x;
  if (c >= ncols) return;
  float s = 0.f;
  for (int r = threadIdx.x; r < nrows; r += blockDim.x)
    s += partials[static_cast<long long>(r) * stride + c0 + c];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[c] = red[0];
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
void launch_reduce_partials(const float* partials, int nrows, int stride, int c0, int ncols,
                            float* out, cudaStream_t st) {
  if (ncols <= 0 || out == nullptr) return;
  reduce_partials_kernel<<<ncols, 256, 0, st>>>(partials, nrows, stride, c0, ncols, out);
}

int make_lrid_plan(int S, long long N, int d, int R, int H, int dtype, bool full_vec, int out_norm,
                   LridPlan* p, const char** why) {
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  LridPlan q{};
  q.S = S; q.N = N; q.d = d; q.R = R; q.H = H;
  q.dv = d / H; q.dk = R / H;
  if (q.dk > 512) { *why = "key head width R/H must be <= 512"; return ATTNRES_ERR_UNSUPPORTED; }
  const int full = 16 / esz;
  q.lph = next_pow2(q.dk) < 32 ? next_pow2(q.dk) : 32;
  q.kpl = ceil_div_i(q.dk, q.lph);
  // Packed layout when rows are 16-byte aligned and a CTA of <= 256 threads
  // covers a token row; otherwise the element-wise layout (<= 1024 threads).
  for (int attempt = 0; attempt < 2; ++attempt) {
    q.vec = (attempt == 0 && full_vec && q.dv % full == 0) ? full : 1;
    const int maxc = q.vec == full ? 1 : 4;
    q.nvh = q.dv / q.vec;
    q.tph = next_pow2(ceil_div_i(q.nvh, maxc));
    q.cph = ceil_div_i(q.nvh, q.tph);
    int need = 32;
    if (H * q.tph > need) need = H * q.tph;
    if (H * q.lph > need) need = H * q.lph;
    q.tpt = next_pow2(need);
    if (q.vec == 1 || q.tpt <= 256) break;
  }
  if (q.tpt > 1024) {
    *why = "value/key head layout needs more than 1024 threads per token row";
    return ATTNRES_ERR_UNSUPPORTED;
  }
  q.tpc = q.tpt >= 256 ? 1 : 256 / q.tpt;
  q.wph = q.tph >= 32 ? q.tph / 32 : 1;
  q.out_norm_group = out_norm == ATTNRES_NORM_ROW ? q.tpt : q.tph;
  q.ntiles = (N + q.tpc - 1) / q.tpc;
  *p = q;
  return ATTNRES_OK;
}

using KernelFn = void (*)(LridArgs);

template <typename T, int VEC, int MAXC, int KPLMAX>
KernelFn pick_dir(bool bwd) {
  return bwd ? lrid_kernel<T, VEC, MAXC, KPLMAX, true> : lrid_kernel<T, VEC, MAXC, KPLMAX, false>;
}

template <typename T, int VEC, int MAXC>
KernelFn pick_kpl(const LridPlan& p, bool bwd) {
  return p.kpl <= 2 ? pick_dir<T, VEC, MAXC, 2>(bwd) : pick_dir<T, VEC, MAXC, 16>(bwd);
}

template <typename T>
KernelFn pick_vec(const LridPlan& p, bool bwd) {
  constexpr int FULL = 16 / sizeof(T);
  return p.vec == FULL ? pick_kpl<T, FULL, 1>(p, bwd) : pick_kpl<T, 1, 4>(p, bwd);
}

static KernelFn pick_kernel(int dtype, const LridPlan& p, bool bwd) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return pick_vec<float>(p, bwd);
    case ATTNRES_DTYPE_F16: return pick_vec<__half>(p, bwd);
    default: return pick_vec<__nv_bfloat16>(p, bwd);
  }
}

static size_t lrid_smem_bytes(const LridPlan& p, int block, bool bwd) {
  const size_t A = static_cast<size_t>(p.tpc) * p.H * p.S;
  size_t bytes = 6 * sizeof(void*) * p.S;
  bytes += sizeof(float) * (4 * A + (bwd ? A * p.wph : 0) + block / 32 +
                            static_cast<size_t>(p.tpc) * p.R + static_cast<size_t>(p.tpc) * p.H);
  return bytes;
}

struct LaunchShape {
  KernelFn fn;
  int block;
  size_t smem;
  int grid;
};

static int device_sm_count() {
  int n = 0;
  return cached_sm_count(&n) == cudaSuccess ? n : 0;
}

// Launch geometry for one plan; deterministic for a given device and plan, so
// the workspace query and the backward launch agree on the grid.
static cudaError_t lrid_launch_shape(int dtype, const LridPlan& p, bool bwd, LaunchShape* ls) {
  ls->fn = pick_kernel(dtype, p, bwd);
  ls->block = p.tpc * p.tpt;
  ls->smem = lrid_smem_bytes(p, ls->block, bwd);
  cudaError_t e = cudaSuccess;
  if (ls->smem > 48 * 1024) {
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(ls->fn), static_cast<int>(ls->smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 0;
  e = cached_occupancy(&per_sm, reinterpret_cast<const void*>(ls->fn), ls->block, ls->smem);
  if (e != cudaSuccess) return e;
  const int nsm = device_sm_count();
  if (nsm <= 0 || per_sm <= 0) return cudaErrorInvalidConfiguration;
  const long long cap = static_cast<long long>(nsm) * per_sm;
  ls->grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.ntiles, cap)));
  return cudaSuccess;
}

int lrid_partial_stride(const LridPlan& p) { return p.R + p.H + p.S; }

cudaError_t lrid_workspace(int dtype, const LridPlan& p, size_t* bytes) {
  LaunchShape ls;
  cudaError_t e = lrid_launch_shape(dtype, p, true, &ls);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(float) * static_cast<size_t>(ls.grid) * lrid_partial_stride(p);
  return cudaSuccess;
}

static void fill_tables(LridArgs& a, const LridPlan& p, const void* const* values,
                        const int64_t* vstr, const void* const* keys, const int64_t* kstr) {
  for (int s = 0; s < p.S; ++s) {
    a.v[s] = values[s];
    a.k[s] = keys[s];
    a.vs[s] = vstr[s];
    a.ks[s] = kstr[s];
  }
}

cudaError_t lrid_forward_launch(int dtype, const LridPlan& p, const LridIO& io, cudaStream_t st) {
  LridArgs a{};
  a.p = p;
  fill_tables(a, p, io.values, io.vstr, io.keys, io.kstr);
  a.qmode = io.qmode;
  a.q = io.q;
  a.gate = io.gate;
  a.qdyn = io.qdyn;
  a.scale = io.scale;
  a.key_norm = io.key_norm;
  a.key_eps = io.key_eps;
  a.bias = io.bias;
  a.out_norm = io.out_norm;
  a.out_eps = io.out_eps;
  a.out = io.out;
  a.out_inv = io.out_inv;
  a.alpha_out = io.alpha_out;
  a.kinv_out = io.kinv_out;
  LaunchShape ls;
  cudaError_t e = lrid_launch_shape(dtype, p, false, &ls);
  if (e != cudaSuccess) return e;
  ls.fn<<<ls.grid, ls.block, ls.smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t lrid_backward_launch(int dtype, const LridPlan& p, const LridIO& io,
                                 const LridGradIO& gio, cudaStream_t st) {
  LridArgs a{};
  a.p = p;
  fill_tables(a, p, io.values, io.vstr, io.keys, io.kstr);
  for (int s = 0; s < p.S; ++s) {
    a.gv[s] = gio.grad_values ? gio.grad_values[s] : nullptr;
    a.gk[s] = gio.grad_keys[s];
  }
  a.qmode = io.qmode;
  a.q = io.q;
  a.gate = io.gate;
  a.qdyn = io.qdyn;
  a.scale = io.scale;
  a.key_norm = io.key_norm;
  a.key_eps = io.key_eps;
  a.bias = io.bias;
  a.out_norm = io.out_norm;
  a.out_eps = io.out_eps;
  a.g = gio.grad_output;
  a.y = gio.normed_output;
  a.y_inv = gio.output_inv_rms;
  a.dq_tok = (io.qmode == ATTNRES_QUERY_DYNAMIC) ? gio.grad_query : gio.grad_query_dynamic;
  a.want_bias_grad = gio.grad_bias != nullptr;
  LaunchShape ls;
  cudaError_t e = lrid_launch_shape(dtype, p, true, &ls);
  if (e != cudaSuccess) return e;
  const int stride = lrid_partial_stride(p);
  const bool need_partials = io.qmode != ATTNRES_QUERY_DYNAMIC || gio.grad_bias != nullptr;
  a.partials = need_partials ? static_cast<float*>(gio.workspace) : nullptr;
  a.part_stride = stride;
  ls.fn<<<ls.grid, ls.block, ls.smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || !need_partials) return e;
  if (io.qmode != ATTNRES_QUERY_DYNAMIC) {
    launch_reduce_partials(a.partials, ls.grid, stride, 0, p.R,
                           static_cast<float*>(gio.grad_query), st);
    if (io.qmode == ATTNRES_QUERY_GATED)
      launch_reduce_partials(a.partials, ls.grid, stride, p.R, p.H, gio.grad_gate, st);
  }
  launch_reduce_partials(a.partials, ls.grid, stride, p.R + p.H, p.S, gio.grad_bias, st);
  return cudaGetLastError();
}

}  // namespace attnres
