// Base block Attention-Residual read (keys = rms-normed values): forward and
// backward.
//
// Semantics follow the reference's PyTorch path _attnres_read_torch_list
// (attnres_ops.py:2193-2214) and the Triton kernels _attnres_list_read_kernel
// (attnres_ops.py:267-328) / _attnres_list_backward_kernel
// (attnres_ops.py:448-535), computed in fp32:
//   khat_s = key_norm ? v_s * rsqrt(mean(v_s^2) + eps) : v_s
//   logit_s = <khat_s, q> + bias_s ; alpha = softmax_s ; out = sum_s alpha_s v_s
// Backward (g' = output-norm backward of g, qk_s = <khat_s, q>):
//   dlogit_s = alpha_s (<g', v_s> - sum_r alpha_r <g', v_r>)
//   dV_s = alpha_s g' + key_norm ? kinv_s dlogit_s (q - khat_s qk_s / d) : dlogit_s q
//   dq = sum_tokens sum_s dlogit_s khat_s   (per-CTA partials, fixed-order reduce)
#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "launch_cache.h"

namespace attnres {

struct BaseArgs {
  BasePlan p;
  const void* v[kMaxSources];
  long long vs[kMaxSources];
  void* gv[kMaxSources];
  const void* q;
  int key_norm;
  float key_eps;
  const float* bias;
  int out_norm;
  float out_eps;
  void* out;
  float* out_inv;
  const void* g;
  const void* y;
  const float* y_inv;
  float* partials;
  int part_stride;
  int want_bias_grad;
};

template <typename T, int VEC, int MAXC, bool BWD>
__global__ void __launch_bounds__(1024) base_kernel(const __grid_constant__ BaseArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const BasePlan& P = a.p;
  const int S = P.S, d = P.d, tpt = P.tpt, tpc = P.tpc, cpt = P.cpt, nv = P.nv, wpt = P.wpt;
  const T** sv = reinterpret_cast<const T**>(smem_raw);
  long long* svs = reinterpret_cast<long long*>(sv + S);
  T** sgv = reinterpret_cast<T**>(svs + S);
  float* fs = reinterpret_cast<float*>(sgv + S);
  const int A = tpc * S;
  float* sm_part = fs;                 // [tpc][S][wpt][3] per-warp partial sums
  float* sm_alpha = sm_part + A * wpt * 3;
  float* sm_kinv = sm_alpha + A;
  float* sm_qk = sm_kinv + A;
  float* sm_dl = sm_qk + A;
  float* sm_red = sm_dl + A;           // [blockDim/32]
  float* sm_dqe = sm_red + (blockDim.x >> 5);  // [tpc][d]

  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    sv[i] = static_cast<const T*>(a.v[i]);
    svs[i] = a.vs[i];
    if (BWD) sgv[i] = static_cast<T*>(a.gv[i]);
  }
  __syncthreads();

  const int tid = threadIdx.x, lane = tid & 31;
  const int slot = tid / tpt, it = tid % tpt;
  const int wi = it >> 5;  // warp index within the token row
  const int rg = tpt < 32 ? tpt : 32;
  const T* qp = static_cast<const T*>(a.q);

  float qv[MAXC][VEC], dq_acc[MAXC][VEC];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int vi = it + c * tpt;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      dq_acc[c][e] = 0.f;
      qv[c][e] = (c < cpt && vi < nv) ? load_f(qp + vi * VEC + e) : 0.f;
    }
  }
  float dbias_acc = 0.f;

  for (long long tile = blockIdx.x; tile < P.ntiles; tile += gridDim.x) {
    const long long t = tile * tpc + slot;
    const bool tv = t < P.N;

    float gp[MAXC][VEC], yv[MAXC][VEC];
    if constexpr (BWD) {
      const T* gptr = static_cast<const T*>(a.g);
      const T* yptr = static_cast<const T*>(a.y);
      float gy = 0.f;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int vi = it + c * tpt;
#pragma unroll
        for (int e = 0; e < VEC; ++e) gp[c][e] = yv[c][e] = 0.f;
        if (c < cpt && vi < nv && tv) {
          const Pack<T, VEC> gr = load_pack<T, VEC>(gptr + t * d + vi * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) gp[c][e] = Elem<T>::to_f(gr.e[e]);
          if (a.out_norm != ATTNRES_NORM_NONE) {
            const Pack<T, VEC> yr = load_pack<T, VEC>(yptr + t * d + vi * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              yv[c][e] = Elem<T>::to_f(yr.e[e]);
              gy = fmaf(gp[c][e], yv[c][e], gy);
            }
          }
        }
      }
      if (a.out_norm != ATTNRES_NORM_NONE) {
        // row reduction over tpt threads
        float tot = group_sum(gy, rg);
        if (tpt > 32) {
          if (lane == 0) sm_red[tid >> 5] = tot;
          __syncthreads();
          tot = 0.f;
          for (int w = 0; w < wpt; ++w) tot += sm_red[slot * wpt + w];
          __syncthreads();
        }
        const float inv = tv ? a.y_inv[t] : 0.f;
        const float mdot = tot / d;
#pragma unroll
        for (int c = 0; c < MAXC; ++c)
#pragma unroll
          for (int e = 0; e < VEC; ++e) gp[c][e] = inv * (gp[c][e] - yv[c][e] * mdot);
      }
    }

    // ---- pass 1: per source sum-of-squares, <v,q>, and (backward) <g',v> ----
    for (int s = 0; s < S; ++s) {
      float p0 = 0.f, p1 = 0.f, p2 = 0.f;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int vi = it + c * tpt;
        if (c < cpt && vi < nv && tv) {
          const Pack<T, VEC> r = load_pack<T, VEC>(sv[s] + t * svs[s] + vi * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float x = Elem<T>::to_f(r.e[e]);
            p0 = fmaf(x, x, p0);
            p1 = fmaf(x, qv[c][e], p1);
            if (BWD) p2 = fmaf(x, gp[c][e], p2);
          }
        }
      }
      p0 = group_sum(p0, rg);
      p1 = group_sum(p1, rg);
      if (BWD) p2 = group_sum(p2, rg);
      if ((it & 31) == 0) {
        float* dst = sm_part + ((slot * S + s) * wpt + wi) * 3;
        dst[0] = p0;
        dst[1] = p1;
        dst[2] = p2;
      }
    }
    __syncthreads();

    // ---- softmax (and dlogit) over sources: one warp per token row ----------
    for (int sl = tid >> 5; sl < tpc; sl += blockDim.x >> 5) {
      const long long tp = tile * tpc + sl;
      float m = -INFINITY;
      for (int s = lane; s < S; s += 32) {
        float ss = 0.f, dot = 0.f, dw = 0.f;
        for (int w = 0; w < wpt; ++w) {
          const float* src = sm_part + ((sl * S + s) * wpt + w) * 3;
          ss += src[0];
          dot += src[1];
          dw += src[2];
        }
        const float kinv = a.key_norm ? rsqrtf(ss / d + a.key_eps) : 1.f;
        const float qk = dot * kinv;
        const float logit = qk + (a.bias ? a.bias[s] : 0.f);
        sm_kinv[sl * S + s] = kinv;
        sm_qk[sl * S + s] = qk;
        sm_alpha[sl * S + s] = logit;
        sm_dl[sl * S + s] = dw;
        m = fmaxf(m, logit);
      }
      m = warp_max(m);
      float sum = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float e = expf(sm_alpha[sl * S + s] - m);
        sm_alpha[sl * S + s] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      float wd = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float al = sm_alpha[sl * S + s] / sum;
        sm_alpha[sl * S + s] = al;
        wd = fmaf(al, sm_dl[sl * S + s], wd);
      }
      if (BWD) {
        wd = warp_sum(wd);
        for (int s = lane; s < S; s += 32) {
          const float al = sm_alpha[sl * S + s];
          sm_dl[sl * S + s] = (tp < P.N) ? al * (sm_dl[sl * S + s] - wd) : 0.f;
        }
      }
    }
    __syncthreads();

    if constexpr (!BWD) {
      // ---- pass 2: out = sum_s alpha_s v_s ---------------------------------
      T* outp = static_cast<T*>(a.out);
      float acc[MAXC][VEC];
      float ssq = 0.f;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int vi = it + c * tpt;
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[c][e] = 0.f;
        if (c < cpt && vi < nv && tv) {
          for (int s = 0; s < S; ++s) {
            const float w = sm_alpha[slot * S + s];
            const Pack<T, VEC> r = load_pack<T, VEC>(sv[s] + t * svs[s] + vi * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[c][e] = fmaf(w, Elem<T>::to_f(r.e[e]), acc[c][e]);
          }
#pragma unroll
          for (int e = 0; e < VEC; ++e) ssq = fmaf(acc[c][e], acc[c][e], ssq);
        }
      }
      float inv = 1.f;
      if (a.out_norm != ATTNRES_NORM_NONE) {
        float tot = group_sum(ssq, rg);
        if (tpt > 32) {
          if (lane == 0) sm_red[tid >> 5] = tot;
          __syncthreads();
          tot = 0.f;
          for (int w = 0; w < wpt; ++w) tot += sm_red[slot * wpt + w];
        }
        inv = rsqrtf(tot / d + a.out_eps);
        if (a.out_inv && tv && it == 0) a.out_inv[t] = inv;
      }
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int vi = it + c * tpt;
        if (c < cpt && vi < nv && tv) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[c][e] *= inv;
          store_pack<T, VEC>(outp + t * d + vi * VEC, acc[c]);
        }
      }
    } else {
      // ---- pass 2: dV_s and dq ---------------------------------------------
      if (a.want_bias_grad && tid < S)
        for (int sl = 0; sl < tpc; ++sl) dbias_acc += sm_dl[sl * S + tid];
      for (int s = 0; s < S; ++s) {
        const float al = sm_alpha[slot * S + s];
        const float dl = sm_dl[slot * S + s];
        const float kinv = sm_kinv[slot * S + s];
        const float c2 = a.key_norm ? dl * sm_qk[slot * S + s] / d : 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          const int vi = it + c * tpt;
          if (c < cpt && vi < nv && tv) {
            const Pack<T, VEC> r = load_pack<T, VEC>(sv[s] + t * svs[s] + vi * VEC);
            float o[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              const float khat = Elem<T>::to_f(r.e[e]) * kinv;
              const float gk = a.key_norm ? kinv * (dl * qv[c][e] - khat * c2) : dl * qv[c][e];
              o[e] = fmaf(al, gp[c][e], gk);
              dq_acc[c][e] = fmaf(dl, khat, dq_acc[c][e]);
            }
            store_pack<T, VEC>(sgv[s] + t * d + vi * VEC, o);
          }
        }
      }
    }
    __syncthreads();
  }

  if constexpr (BWD) {
    if (a.partials == nullptr) return;
    for (int i = tid; i < tpc * d; i += blockDim.x) sm_dqe[i] = 0.f;
    __syncthreads();
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int vi = it + c * tpt;
      if (c < cpt && vi < nv)
#pragma unroll
        for (int e = 0; e < VEC; ++e) sm_dqe[slot * d + vi * VEC + e] = dq_acc[c][e];
    }
    __syncthreads();
    float* row = a.partials + static_cast<long long>(blockIdx.x) * a.part_stride;
    for (int e = tid; e < d; e += blockDim.x) {
      float s = 0.f;
      for (int sl = 0; sl < tpc; ++sl) s += sm_dqe[sl * d + e];
      row[e] = s;
    }
    if (tid < S) row[d + tid] = dbias_acc;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using BaseFn = void (*)(BaseArgs);

template <typename T>
static BaseFn pick_base_t(const BasePlan& p, bool bwd) {
  constexpr int FULL = 16 / sizeof(T);
  if (p.vec == FULL) return bwd ? base_kernel<T, FULL, 1, true> : base_kernel<T, FULL, 1, false>;
  return bwd ? base_kernel<T, 1, 4, true> : base_kernel<T, 1, 4, false>;
}

static BaseFn pick_base(int dtype, const BasePlan& p, bool bwd) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return pick_base_t<float>(p, bwd);
    case ATTNRES_DTYPE_F16: return pick_base_t<__half>(p, bwd);
    default: return pick_base_t<__nv_bfloat16>(p, bwd);
  }
}

int make_base_plan(int S, long long N, int d, int dtype, bool full_vec, BasePlan* p,
                   const char** why) {
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const int full = 16 / esz;
  BasePlan q{};
  q.S = S; q.N = N; q.d = d;
  q.vec = (full_vec && d % full == 0) ? full : 1;
  const int maxc = q.vec == full ? 1 : 4;
  q.nv = d / q.vec;
  int tpt = next_pow2(ceil_div_i(q.nv, maxc));
  if (tpt < 32) tpt = 32;
  if (tpt > 1024) {
    *why = "value width too large for the base AttnRes read (needs > 1024 threads per row)";
    return ATTNRES_ERR_UNSUPPORTED;
  }
  q.tpt = tpt;
  q.cpt = ceil_div_i(q.nv, tpt);
  q.tpc = tpt >= 256 ? 1 : 256 / tpt;
  q.wpt = tpt / 32;
  q.ntiles = (N + q.tpc - 1) / q.tpc;
  *p = q;
  return ATTNRES_OK;
}

static size_t base_smem(const BasePlan& p, int block) {
  const size_t A = static_cast<size_t>(p.tpc) * p.S;
  return 3 * sizeof(void*) * p.S +
         sizeof(float) * (A * p.wpt * 3 + 4 * A + block / 32 + static_cast<size_t>(p.tpc) * p.d);
}

struct BaseShape {
  BaseFn fn;
  int block, grid;
  size_t smem;
};

static cudaError_t base_shape(int dtype, const BasePlan& p, bool bwd, BaseShape* bs) {
  bs->fn = pick_base(dtype, p, bwd);
  bs->block = p.tpc * p.tpt;
  bs->smem = base_smem(p, bs->block);
  cudaError_t e;
  if (bs->smem > 48 * 1024) {
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(bs->fn), static_cast<int>(bs->smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 0, nsm = 0;
  e = cached_occupancy(&per_sm, reinterpret_cast<const void*>(bs->fn), bs->block, bs->smem);
  if (e != cudaSuccess) return e;
  e = cached_sm_count(&nsm);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  const long long cap = static_cast<long long>(nsm) * per_sm;
  bs->grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.ntiles, cap)));
  return cudaSuccess;
}

cudaError_t base_workspace(int dtype, const BasePlan& p, size_t* bytes) {
  BaseShape bs;
  cudaError_t e = base_shape(dtype, p, true, &bs);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(float) * static_cast<size_t>(bs.grid) * (p.d + p.S);
  return cudaSuccess;
}

static void fill_base(BaseArgs& a, const BasePlan& p, const BaseIO& io) {
  a.p = p;
  for (int s = 0; s < p.S; ++s) {
    a.v[s] = io.values[s];
    a.vs[s] = io.vstr[s];
    a.gv[s] = io.grad_values ? io.grad_values[s] : nullptr;
  }
  a.q = io.q;
  a.key_norm = io.key_norm;
  a.key_eps = io.key_eps;
  a.bias = io.bias;
  a.out_norm = io.out_norm;
  a.out_eps = io.out_eps;
  a.out = io.out;
  a.out_inv = io.out_inv;
  a.g = io.grad_output;
  a.y = io.normed_output;
  a.y_inv = io.output_inv_rms;
  a.want_bias_grad = io.grad_bias != nullptr;
}

cudaError_t base_forward_launch(int dtype, const BasePlan& p, const BaseIO& io, cudaStream_t st) {
  BaseArgs a{};
  fill_base(a, p, io);
  BaseShape bs;
  cudaError_t e = base_shape(dtype, p, false, &bs);
  if (e != cudaSuccess) return e;
  bs.fn<<<bs.grid, bs.block, bs.smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t base_backward_launch(int dtype, const BasePlan& p, const BaseIO& io, cudaStream_t st) {
  BaseArgs a{};
  fill_base(a, p, io);
  BaseShape bs;
  cudaError_t e = base_shape(dtype, p, true, &bs);
  if (e != cudaSuccess) return e;
  a.partials = static_cast<float*>(io.workspace);
  a.part_stride = p.d + p.S;
  bs.fn<<<bs.grid, bs.block, bs.smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  launch_reduce_partials(a.partials, bs.grid, a.part_stride, 0, p.d, io.grad_query, st);
  launch_reduce_partials(a.partials, bs.grid, a.part_stride, p.d, p.S, io.grad_bias, st);
  return cudaGetLastError();
}

}  // namespace attnres
