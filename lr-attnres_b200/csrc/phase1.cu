// Cached-logit block read ("phase 1"): Q reads of the same S sources with
// precomputed logits, forward and backward.
//
// Semantics of attention_residual_phase1_from_logits (attnres_ops.py:3910-3961,
// PyTorch path :3955-3961; Triton kernels _attnres_phase1_logits_forward_kernel
// :933-989 and _attnres_phase1_logits_backward_weights_kernel :1069-1140):
//   alpha[q,n,:] = softmax_s(logits[q,:,n])           (fp32)
//   out[q,n,:]   = sum_s alpha[q,n,s] * V_s[n,:]       (opt. rms norm of each output row)
//   lse[q,n]     = logsumexp_s(logits[q,:,n])
// Backward (g' = output-norm backward of grad_out[q,n]):
//   dV_s[n]        = sum_q alpha[q,n,s] * g'_q
//   dlogits[q,s,n] = alpha[q,n,s] * (<g'_q, V_s> - sum_r alpha[q,n,r] <g'_q, V_r>) + dlse[q,n] * alpha[q,n,s]
// Layout: sources are row-strided [N, d]; logits / dlogits dense [Q][S][N];
// out dense [Q][N][d]; lse / inv-rms [Q][N].
// Work split: `tpt` threads per token row (cpt packs each), `tpc` rows per
// CTA; logits are loaded token-fastest (coalesced); a warp computes each
// (token, query) softmax; values are re-read per query from L1.
#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "launch_cache.h"

namespace attnres {

constexpr int kP1MaxQ = 16;

struct Phase1Args {
  const void* v[kMaxSources];
  long long vs[kMaxSources];
  void* gv[kMaxSources];
  const void* logits;  // [Q][S][N], logit dtype
  int logit_dtype;
  void* out;           // [Q][N][d]
  float* lse;          // [Q][N]
  float* out_inv;      // [Q][N] or null
  const void* g;       // [Q][N][d]
  const void* y;       // saved normalised output [Q][N][d]
  const float* y_inv;  // [Q][N]
  const float* glse;   // [Q][N] or null
  void* dlogits;       // [Q][S][N], logit dtype
  long long N;
  long long ntiles;
  int S, Q, d, tpt, tpc, cpt, nv, wpt, out_norm;
  float out_eps;
};

__device__ __forceinline__ float load_any(const void* p, int dtype, long long i) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return static_cast<const float*>(p)[i];
    case ATTNRES_DTYPE_F16: return __half2float(static_cast<const __half*>(p)[i]);
    default: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
}

__device__ __forceinline__ void store_any(void* p, int dtype, long long i, float x) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: static_cast<float*>(p)[i] = x; break;
    case ATTNRES_DTYPE_F16: static_cast<__half*>(p)[i] = __float2half_rn(x); break;
    default: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  }
}

// Sum over the tpt threads of a token row (power of two >= 32) via per-warp
// partials in `red` (fixed order). Every thread of the CTA must call.
__device__ __forceinline__ float row_sum(float v, int tpt, float* red) {
  v = warp_sum(v);
  if (tpt == 32) return v;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int nw = tpt >> 5, w0 = (threadIdx.x / tpt) * nw;
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w0 + w];
  __syncthreads();
  return tot;
}

template <typename T, int VEC, int MAXC, bool BWD>
__global__ void __launch_bounds__(1024) phase1_kernel(const __grid_constant__ Phase1Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int S = a.S, Q = a.Q, d = a.d, tpt = a.tpt, tpc = a.tpc, cpt = a.cpt, nv = a.nv, wpt = a.wpt;
  const T** sv = reinterpret_cast<const T**>(smem_raw);
  long long* svs = reinterpret_cast<long long*>(sv + S);
  T** sgv = reinterpret_cast<T**>(svs + S);
  float* fs = reinterpret_cast<float*>(sgv + S);
  const int A = tpc * Q * S;
  float* sm_alpha = fs;                 // [tpc][Q][S]
  float* sm_dw = fs + A;                // [tpc][Q][S][wpt] (backward)
  float* sm_red = sm_dw + (BWD ? A * wpt : 0);
  float* sm_mdot = sm_red + (blockDim.x >> 5);  // [tpc][Q] (backward, output norm)
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    sv[i] = static_cast<const T*>(a.v[i]);
    svs[i] = a.vs[i];
    if (BWD) sgv[i] = static_cast<T*>(a.gv[i]);
  }
  __syncthreads();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int slot = tid / tpt, it = tid % tpt, wi = it >> 5;

  for (long long tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
    const long long t0 = tile * tpc;
    const long long t = t0 + slot;
    const bool tv = t < a.N;
    // ---- logits (token-fastest, coalesced) -> softmax per (token, query) ----
    for (int i = tid; i < A; i += blockDim.x) {
      const int sl = i % tpc, qs = i / tpc;  // qs = q * S + s
      const long long tt = t0 + sl;
      sm_alpha[(sl * Q + qs / S) * S + qs % S] =
          tt < a.N ? load_any(a.logits, a.logit_dtype, static_cast<long long>(qs) * a.N + tt) : 0.f;
    }
    __syncthreads();
    for (int pair = warp; pair < tpc * Q; pair += nwarps) {
      float* al = sm_alpha + pair * S;
      const long long tp = t0 + pair / Q;
      const int q = pair % Q;
      float m = -INFINITY;
      for (int s = lane; s < S; s += 32) m = fmaxf(m, al[s]);
      m = warp_max(m);
      float sum = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float e = expf(al[s] - m);
        al[s] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      for (int s = lane; s < S; s += 32) al[s] = al[s] / sum;
      if (!BWD && lane == 0 && tp < a.N) a.lse[q * a.N + tp] = m + logf(sum);
    }
    __syncthreads();
    const float* al = sm_alpha + slot * Q * S;

    if constexpr (!BWD) {
      T* outp = static_cast<T*>(a.out);
      for (int q = 0; q < Q; ++q) {
        float acc[MAXC][VEC];
        float ssq = 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int vi = it + c * tpt;
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[c][e] = 0.f;
          if (c < cpt && vi < nv && tv) {
            for (int s = 0; s < S; ++s) {
              const float w = al[q * S + s];
              const Pack<T, VEC> r = load_pack<T, VEC>(sv[s] + t * svs[s] + vi * VEC);
#pragma unroll
              for (int e = 0; e < VEC; ++e) acc[c][e] = fmaf(w, Elem<T>::to_f(r.e[e]), acc[c][e]);
            }
#pragma unroll
            for (int e = 0; e < VEC; ++e) ssq = fmaf(acc[c][e], acc[c][e], ssq);
          }
        }
        float inv = 1.f;
        if (a.out_norm) {
          inv = rsqrtf(row_sum(ssq, tpt, sm_red) / d + a.out_eps);
          if (a.out_inv && tv && it == 0) a.out_inv[q * a.N + t] = inv;
        }
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int vi = it + c * tpt;
          if (c < cpt && vi < nv && tv) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[c][e] *= inv;
            store_pack<T, VEC>(outp + (static_cast<long long>(q) * a.N + t) * d + vi * VEC, acc[c]);
          }
        }
      }
    } else {
      const T* gp = static_cast<const T*>(a.g);
      const T* yp = static_cast<const T*>(a.y);
      // output-norm backward needs <g_q, y_q> per query first
      if (a.out_norm) {
        for (int q = 0; q < Q; ++q) {
          float gy = 0.f;
#pragma unroll
          for (int c = 0; c < MAXC; ++c) {
            const int vi = it + c * tpt;
            if (c < cpt && vi < nv && tv) {
              const long long off = (static_cast<long long>(q) * a.N + t) * d + vi * VEC;
              const Pack<T, VEC> gr = load_pack<T, VEC>(gp + off), yr = load_pack<T, VEC>(yp + off);
#pragma unroll
              for (int e = 0; e < VEC; ++e) gy = fmaf(Elem<T>::to_f(gr.e[e]), Elem<T>::to_f(yr.e[e]), gy);
            }
          }
          const float tot = row_sum(gy, tpt, sm_red);
          if (it == 0) sm_mdot[slot * Q + q] = tot / d;
        }
        __syncthreads();
      }
      for (int s = 0; s < S; ++s) {
        float dwp[kP1MaxQ];
#pragma unroll
        for (int q = 0; q < kP1MaxQ; ++q) dwp[q] = 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int vi = it + c * tpt;
          if (c < cpt && vi < nv && tv) {
            const Pack<T, VEC> vr = load_pack<T, VEC>(sv[s] + t * svs[s] + vi * VEC);
            float dv[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) dv[e] = 0.f;
#pragma unroll
            for (int q = 0; q < kP1MaxQ; ++q) {
              if (q < Q) {
                const long long off = (static_cast<long long>(q) * a.N + t) * d + vi * VEC;
                const Pack<T, VEC> gr = load_pack<T, VEC>(gp + off);
                float yinv = 0.f, mdot = 0.f;
                Pack<T, VEC> yr;
                if (a.out_norm) {
                  yr = load_pack<T, VEC>(yp + off);
                  yinv = a.y_inv[q * a.N + t];
                  mdot = sm_mdot[slot * Q + q];
                }
                const float w = al[q * S + s];
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  float g = Elem<T>::to_f(gr.e[e]);
                  if (a.out_norm) g = yinv * (g - Elem<T>::to_f(yr.e[e]) * mdot);
                  dv[e] = fmaf(w, g, dv[e]);
                  dwp[q] = fmaf(g, Elem<T>::to_f(vr.e[e]), dwp[q]);
                }
              }
            }
            store_pack<T, VEC>(sgv[s] + t * d + vi * VEC, dv);
          }
        }
#pragma unroll
        for (int q = 0; q < kP1MaxQ; ++q) {
          if (q < Q) {
            const float r = warp_sum(dwp[q]);
            if (lane == 0) sm_dw[((slot * Q + q) * S + s) * wpt + wi] = r;
          }
        }
      }
      __syncthreads();
      // dlogits: combine the per-warp partial dots, then write token-fastest
      for (int pair = warp; pair < tpc * Q; pair += nwarps) {
        const int sl = pair / Q, q = pair % Q;
        const long long tp = t0 + sl;
        float part = 0.f;
        for (int s = lane; s < S; s += 32) {
          float dw = 0.f;
          for (int w = 0; w < wpt; ++w) dw += sm_dw[((sl * Q + q) * S + s) * wpt + w];
          sm_dw[((sl * Q + q) * S + s) * wpt] = dw;
          part = fmaf(sm_alpha[pair * S + s], dw, part);
        }
        const float wd = warp_sum(part);
        const float gl = (a.glse && tp < a.N) ? a.glse[q * a.N + tp] : 0.f;
        for (int s = lane; s < S; s += 32) {
          const float alp = sm_alpha[pair * S + s];
          sm_dw[((sl * Q + q) * S + s) * wpt] = alp * (sm_dw[((sl * Q + q) * S + s) * wpt] - wd) + gl * alp;
        }
      }
      __syncthreads();
      for (int i = tid; i < A; i += blockDim.x) {
        const int sl = i % tpc, qs = i / tpc;
        const long long tt = t0 + sl;
        if (tt < a.N)
          store_any(a.dlogits, a.logit_dtype, static_cast<long long>(qs) * a.N + tt,
                    sm_dw[((sl * Q + qs / S) * S + qs % S) * wpt]);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using P1Fn = void (*)(Phase1Args);

template <typename T>
static P1Fn pick_p1_t(int vec, bool bwd) {
  constexpr int FULL = 16 / sizeof(T);
  if (vec == FULL) return bwd ? phase1_kernel<T, FULL, 1, true> : phase1_kernel<T, FULL, 1, false>;
  return bwd ? phase1_kernel<T, 1, 4, true> : phase1_kernel<T, 1, 4, false>;
}

cudaError_t phase1_launch(int dtype, int logit_dtype, int S, int Q, long long N, int d, bool full_vec,
                          const void* const* values, const int64_t* vstr, const void* logits, int out_norm,
                          float out_eps, void* out, float* lse, float* out_inv, const void* g, const void* y,
                          const float* y_inv, const float* glse, void* const* grad_values, void* dlogits,
                          bool bwd, cudaStream_t st) {
  if (Q < 1 || Q > kP1MaxQ) return cudaErrorInvalidValue;
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const int full = 16 / esz;
  Phase1Args a{};
  const int vec = (full_vec && d % full == 0) ? full : 1;
  const int maxc = vec == full ? 1 : 4;
  a.nv = d / vec;
  int tpt = next_pow2(ceil_div_i(a.nv, maxc));
  if (tpt < 32) tpt = 32;
  if (tpt > 1024) return cudaErrorInvalidValue;
  a.tpt = tpt;
  a.cpt = ceil_div_i(a.nv, tpt);
  a.tpc = tpt >= 256 ? 1 : 256 / tpt;
  a.wpt = tpt / 32;
  a.S = S;
  a.Q = Q;
  a.d = d;
  a.N = N;
  a.ntiles = (N + a.tpc - 1) / a.tpc;
  for (int s = 0; s < S; ++s) {
    a.v[s] = values[s];
    a.vs[s] = vstr[s];
    a.gv[s] = grad_values ? grad_values[s] : nullptr;
  }
  a.logits = logits;
  a.logit_dtype = logit_dtype;
  a.out = out;
  a.lse = lse;
  a.out_inv = out_inv;
  a.g = g;
  a.y = y;
  a.y_inv = y_inv;
  a.glse = glse;
  a.dlogits = dlogits;
  a.out_norm = out_norm;
  a.out_eps = out_eps;
  P1Fn fn;
  switch (dtype) {
    case ATTNRES_DTYPE_F32: fn = pick_p1_t<float>(vec, bwd); break;
    case ATTNRES_DTYPE_F16: fn = pick_p1_t<__half>(vec, bwd); break;
    default: fn = pick_p1_t<__nv_bfloat16>(vec, bwd);
  }
  const int block = a.tpc * tpt;
  const size_t A = static_cast<size_t>(a.tpc) * Q * S;
  const size_t smem = 3 * sizeof(void*) * S +
                      sizeof(float) * (A + (bwd ? A * a.wpt : 0) + block / 32 + static_cast<size_t>(a.tpc) * Q);
  cudaError_t e;
  if (smem > 48 * 1024) {
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 0, nsm = 0;
  e = cached_occupancy(&per_sm, reinterpret_cast<const void*>(fn), block, smem);
  if (e != cudaSuccess) return e;
  e = cached_sm_count(&nsm);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const long long grid = std::max<long long>(1, std::min<long long>(a.ntiles, static_cast<long long>(nsm) * per_sm));
  fn<<<static_cast<int>(grid), block, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace attnres
