// Cached-logit phase 2 of block Attention Residuals: the live partial block is
// merged into the phase-1 result (attnres_ops.py:4075-4160 with LRID keys,
// :3964-4040 / :2630-2642 with the base key rms_norm(partial_value),
// :4043-4072 given the partial logit; Triton kernels :2013-2121):
//   logit = scale <k_hat, q> + bias        (k_hat = key * kinv when key_norm)
//   p     = sigmoid(logit - lse_prev)
//   out   = prev + p (v - prev)            (optionally rms-normalised per row)
// Backward (g' = the output-norm backward of g when normalised):
//   dv = p g' (+ the base key's norm backward), dprev = (1 - p) g',
//   dlogit = p (1 - p) <g', v - prev>, dlse = -dlogit, dkey = norm backward of
//   dlogit scale q, dq = sum_t dlogit scale k_hat, dbias = sum_t dlogit.
// One warp per token row, 16-byte packs; fp32 math. dq is reduced without
// atomics: the per-token weight dlogit * scale * kinv goes to a workspace,
// then a weighted column sum over fixed token ranges and a fixed-order
// combine (deterministic; the reference uses atomic adds).
#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "launch_cache.h"

namespace attnres {

struct Phase2Args {
  int mode;  // ATTNRES_PHASE2_*
  long long N;
  int d, R;
  const void* v;     // partial value [N, d]
  const void* prev;  // interblock output [N, d]
  const float* lse;  // interblock lse [N]
  const void* key;   // LRID partial key [N, R]
  const float* logit;  // given partial logit [N] (LOGIT mode)
  const void* q;     // [R] (LRID) or [d] (BASE), value dtype
  float scale;
  int key_norm;
  float key_eps;
  float bias;
  const float* bias_dev;
  int onorm;
  float out_eps;
  void* out;
  float* out_inv;
  // backward
  const void* g;
  const void* y;       // saved (normalised) output, with onorm
  const float* y_inv;  // saved output inverse rms, with onorm
  void* dv;
  void* dprev;
  float* dlse;
  void* dkey;
  float* dlogit;
  float* wq;  // per-token dq weight dlogit * scale * kinv, or null
};

template <typename T>
__device__ __forceinline__ float ldf(const void* p, long long i) {
  return Elem<T>::to_f(static_cast<const T*>(p)[i]);
}

// Key statistics of token t: raw <k, q> and the key's inverse rms (1 without
// key norm). The key is the partial key row (LRID) or the value row (BASE).
template <typename T, int VEC>
__device__ __forceinline__ void phase2_key(const Phase2Args& a, long long t, int lane, float& dot, float& kinv) {
  float ss = 0.f, dt = 0.f;
  if (a.mode == ATTNRES_PHASE2_LRID) {
    for (int r = lane; r < a.R; r += 32) {
      const float k = ldf<T>(a.key, t * a.R + r);
      ss = fmaf(k, k, ss);
      dt = fmaf(k, ldf<T>(a.q, r), dt);
    }
  } else {
    const T* vr = static_cast<const T*>(a.v) + t * a.d;
    const T* qr = static_cast<const T*>(a.q);
    for (int c = lane * VEC; c < a.d; c += 32 * VEC) {
      const Pack<T, VEC> vp = load_pack<T, VEC>(vr + c);
      const Pack<T, VEC> qp = load_pack<T, VEC>(qr + c);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float k = Elem<T>::to_f(vp.e[e]);
        ss = fmaf(k, k, ss);
        dt = fmaf(k, Elem<T>::to_f(qp.e[e]), dt);
      }
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dt);
  const int kd = a.mode == ATTNRES_PHASE2_LRID ? a.R : a.d;
  kinv = a.key_norm ? rsqrtf(ss / kd + a.key_eps) : 1.f;
}

template <typename T, int VEC>
__device__ __forceinline__ float phase2_logit(const Phase2Args& a, long long t, int lane, float& dot, float& kinv) {
  float lg;
  dot = 0.f;
  kinv = 1.f;
  if (a.mode == ATTNRES_PHASE2_LOGIT) {
    lg = a.logit[t];
  } else {
    phase2_key<T, VEC>(a, t, lane, dot, kinv);
    lg = dot * kinv * (a.mode == ATTNRES_PHASE2_LRID ? a.scale : 1.f);
  }
  return lg + (a.bias_dev ? *a.bias_dev : a.bias);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

template <typename T, int VEC>
__global__ void __launch_bounds__(256) phase2_fwd_kernel(const __grid_constant__ Phase2Args a) {
  const int lane = threadIdx.x & 31;
  const long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= a.N) return;
  float dot, kinv;
  const float p = sigmoidf_(phase2_logit<T, VEC>(a, t, lane, dot, kinv) - a.lse[t]);
  const T* vr = static_cast<const T*>(a.v) + t * a.d;
  const T* pr = static_cast<const T*>(a.prev) + t * a.d;
  T* orow = static_cast<T*>(a.out) + t * a.d;
  float inv = 1.f;
  if (a.onorm) {
    float ss = 0.f;
    for (int c = lane * VEC; c < a.d; c += 32 * VEC) {
      const Pack<T, VEC> vp = load_pack<T, VEC>(vr + c), pp = load_pack<T, VEC>(pr + c);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float pv = Elem<T>::to_f(pp.e[e]);
        const float m = fmaf(p, Elem<T>::to_f(vp.e[e]) - pv, pv);
        ss = fmaf(m, m, ss);
      }
    }
    inv = rsqrtf(warp_sum(ss) / a.d + a.out_eps);
    if (lane == 0) a.out_inv[t] = inv;
  }
  for (int c = lane * VEC; c < a.d; c += 32 * VEC) {
    const Pack<T, VEC> vp = load_pack<T, VEC>(vr + c), pp = load_pack<T, VEC>(pr + c);
    float o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float pv = Elem<T>::to_f(pp.e[e]);
      o[e] = fmaf(p, Elem<T>::to_f(vp.e[e]) - pv, pv) * inv;
    }
    store_pack<T, VEC>(orow + c, o);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) phase2_bwd_kernel(const __grid_constant__ Phase2Args a) {
  const int lane = threadIdx.x & 31;
  const long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= a.N) return;
  const int d = a.d;
  const T* vr = static_cast<const T*>(a.v) + t * d;
  const T* pr = static_cast<const T*>(a.prev) + t * d;
  const T* gr = static_cast<const T*>(a.g) + t * d;
  const T* yr = a.onorm ? static_cast<const T*>(a.y) + t * d : nullptr;
  const float yinv = a.onorm ? a.y_inv[t] : 1.f;
  // output-norm backward needs <g, y> / d
  float gyd = 0.f;
  if (a.onorm) {
    float s = 0.f;
    for (int c = lane * VEC; c < d; c += 32 * VEC) {
      const Pack<T, VEC> gp = load_pack<T, VEC>(gr + c), yp = load_pack<T, VEC>(yr + c);
#pragma unroll
      for (int e = 0; e < VEC; ++e) s = fmaf(Elem<T>::to_f(gp.e[e]), Elem<T>::to_f(yp.e[e]), s);
    }
    gyd = warp_sum(s) / d;
  }
  float dot, kinv;
  const float p = sigmoidf_(phase2_logit<T, VEC>(a, t, lane, dot, kinv) - a.lse[t]);
  // <g', v - prev>
  float mg = 0.f;
  for (int c = lane * VEC; c < d; c += 32 * VEC) {
    const Pack<T, VEC> vp = load_pack<T, VEC>(vr + c), pp = load_pack<T, VEC>(pr + c),
                       gp = load_pack<T, VEC>(gr + c);
    Pack<T, VEC> yp;
    if (a.onorm) yp = load_pack<T, VEC>(yr + c);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float gg = Elem<T>::to_f(gp.e[e]);
      if (a.onorm) gg = yinv * (gg - Elem<T>::to_f(yp.e[e]) * gyd);
      mg = fmaf(gg, Elem<T>::to_f(vp.e[e]) - Elem<T>::to_f(pp.e[e]), mg);
    }
  }
  const float dl = p * (1.f - p) * warp_sum(mg);
  const float sc = a.mode == ATTNRES_PHASE2_LRID ? a.scale : 1.f;
  const float c1 = dl * sc;  // d logit / d <k_hat, q> * ... : dk_hat = c1 q
  // <dk_hat, k_hat> / dim = c1 <q, k_hat> / dim = c1 dot kinv / dim
  const int kd = a.mode == ATTNRES_PHASE2_LRID ? a.R : d;
  const float cross = a.key_norm ? c1 * dot * kinv / kd : 0.f;
  // dv, dprev (+ the base key's norm backward)
  const bool base = a.mode == ATTNRES_PHASE2_BASE;
  const T* qr = static_cast<const T*>(a.q);
  T* dvr = static_cast<T*>(a.dv) + t * d;
  T* dpr = static_cast<T*>(a.dprev) + t * d;
  for (int c = lane * VEC; c < d; c += 32 * VEC) {
    const Pack<T, VEC> gp = load_pack<T, VEC>(gr + c);
    Pack<T, VEC> yp, vp, qp;
    if (a.onorm) yp = load_pack<T, VEC>(yr + c);
    if (base) {
      vp = load_pack<T, VEC>(vr + c);
      qp = load_pack<T, VEC>(qr + c);
    }
    float ov[VEC], op[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float gg = Elem<T>::to_f(gp.e[e]);
      if (a.onorm) gg = yinv * (gg - Elem<T>::to_f(yp.e[e]) * gyd);
      ov[e] = p * gg;
      op[e] = (1.f - p) * gg;
      if (base) {
        const float qv = Elem<T>::to_f(qp.e[e]);
        ov[e] += a.key_norm ? kinv * (c1 * qv - Elem<T>::to_f(vp.e[e]) * kinv * cross) : c1 * qv;
      }
    }
    store_pack<T, VEC>(dvr + c, ov);
    store_pack<T, VEC>(dpr + c, op);
  }
  if (a.mode == ATTNRES_PHASE2_LRID) {
    T* dk = static_cast<T*>(a.dkey) + t * a.R;
    for (int r = lane; r < a.R; r += 32) {
      const float qv = ldf<T>(a.q, r);
      const float k = ldf<T>(a.key, t * a.R + r);
      const float g = a.key_norm ? kinv * (c1 * qv - k * kinv * cross) : c1 * qv;
      dk[r] = Elem<T>::from_f(g);
    }
  }
  if (lane == 0) {
    a.dlse[t] = -dl;
    if (a.dlogit) a.dlogit[t] = dl;
    if (a.wq) a.wq[t] = c1 * kinv;
  }
}

// partials[b][c] = sum over the token range of block b, in token order, of
// w[t] * K[t][c] (K = partial key [N, C] or partial value [N, C]).
template <typename T>
__global__ void __launch_bounds__(256) phase2_wsum_kernel(const float* __restrict__ w, const void* keys, long long N,
                                                          int C, long long rows_per_block, float* partials) {
  const long long t0 = static_cast<long long>(blockIdx.x) * rows_per_block;
  const long long t1 = t0 + rows_per_block < N ? t0 + rows_per_block : N;
  const T* K = static_cast<const T*>(keys);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float s = 0.f;
    for (long long t = t0; t < t1; ++t) s = fmaf(w[t], Elem<T>::to_f(K[t * C + c]), s);
    partials[static_cast<long long>(blockIdx.x) * C + c] = s;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool p2_al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
static cudaError_t phase2_launch_t(const Phase2Args& a, bool bwd, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const unsigned grid = static_cast<unsigned>((a.N + 7) / 8);
  if (bwd) {
    if (vec) phase2_bwd_kernel<T, V><<<grid, 256, 0, st>>>(a);
    else phase2_bwd_kernel<T, 1><<<grid, 256, 0, st>>>(a);
  } else {
    if (vec) phase2_fwd_kernel<T, V><<<grid, 256, 0, st>>>(a);
    else phase2_fwd_kernel<T, 1><<<grid, 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

static cudaError_t phase2_dispatch(int dtype, const Phase2Args& a, bool bwd, bool vec, cudaStream_t st) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return phase2_launch_t<float>(a, bwd, vec, st);
    case ATTNRES_DTYPE_F16: return phase2_launch_t<__half>(a, bwd, vec, st);
    default: return phase2_launch_t<__nv_bfloat16>(a, bwd, vec, st);
  }
}

static bool phase2_vec(const Phase2Args& a, int esz, bool bwd) {
  const int V = 16 / esz;
  if (a.d % V) return false;
  const void* rows[] = {a.v, a.prev, a.out, a.g, a.y, a.dv, a.dprev,
                        a.mode == ATTNRES_PHASE2_BASE ? a.q : nullptr};
  for (const void* p : rows)
    if (p && !p2_al16(p)) return false;
  (void)bwd;
  return true;
}

// dq blocks: token ranges over about 4 CTAs per SM
static int phase2_wsum_blocks(long long N) {
  int nsm = 148;
  if (cached_sm_count(&nsm) != cudaSuccess) nsm = 148;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(N, 4LL * nsm)));
}

// Workspace: [dq weight per token | dlogit per token | dq partial rows].
static size_t p2_vec_bytes(long long N) { return (static_cast<size_t>(N) * 4 + 255) & ~size_t(255); }

size_t phase2_workspace(int mode, long long N, int d, int R) {
  if (N <= 0) return 0;
  const int C = mode == ATTNRES_PHASE2_LRID ? R : (mode == ATTNRES_PHASE2_BASE ? d : 0);
  return 2 * p2_vec_bytes(N) + sizeof(float) * static_cast<size_t>(phase2_wsum_blocks(N)) * C;
}

cudaError_t phase2_forward_launch(int dtype, const Phase2Args& a, cudaStream_t st) {
  if (a.N == 0) return cudaSuccess;
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  return phase2_dispatch(dtype, a, false, phase2_vec(a, esz, false), st);
}

cudaError_t phase2_backward_launch(int dtype, Phase2Args a, float* grad_query, float* grad_bias, void* workspace,
                                   cudaStream_t st) {
  if (a.N == 0) return cudaSuccess;
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const bool keyed = a.mode != ATTNRES_PHASE2_LOGIT;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  float* w = (keyed && grad_query) ? reinterpret_cast<float*>(ws) : nullptr;
  float* partials = reinterpret_cast<float*>(ws + 2 * p2_vec_bytes(a.N));
  a.wq = w;
  if (grad_bias && a.dlogit == nullptr) a.dlogit = reinterpret_cast<float*>(ws + p2_vec_bytes(a.N));
  cudaError_t e = phase2_dispatch(dtype, a, true, phase2_vec(a, esz, true), st);
  if (e != cudaSuccess) return e;
  if (w) {
    const int C = a.mode == ATTNRES_PHASE2_LRID ? a.R : a.d;
    const int nb = phase2_wsum_blocks(a.N);
    const long long rows = (a.N + nb - 1) / nb;
    const void* K = a.mode == ATTNRES_PHASE2_LRID ? a.key : a.v;
    switch (dtype) {
      case ATTNRES_DTYPE_F32: phase2_wsum_kernel<float><<<nb, 256, 0, st>>>(w, K, a.N, C, rows, partials); break;
      case ATTNRES_DTYPE_F16: phase2_wsum_kernel<__half><<<nb, 256, 0, st>>>(w, K, a.N, C, rows, partials); break;
      default: phase2_wsum_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(w, K, a.N, C, rows, partials);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    launch_reduce_partials(partials, nb, C, 0, C, grad_query, st);
  }
  if (grad_bias) launch_reduce_partials(a.dlogit, static_cast<int>(a.N), 1, 0, 1, grad_bias, st);  // sum_t dlogit
  return cudaGetLastError();
}

cudaError_t phase2_run(bool bwd, int mode, long long N, int d, int R, int dtype, const void* v, const void* key,
                       const float* logit, const void* q, float scale, int key_norm, float key_eps, float bias,
                       const float* bias_dev, const void* prev, const float* lse, int onorm, float out_eps,
                       void* out, float* out_inv, const void* g, const void* y, const float* y_inv, void* dv,
                       void* dkey, float* dlogit, void* dprev, float* dlse, float* grad_query, float* grad_bias,
                       void* workspace, cudaStream_t st) {
  Phase2Args a{};
  a.mode = mode;
  a.N = N;
  a.d = d;
  a.R = R;
  a.v = v;
  a.prev = prev;
  a.lse = lse;
  a.key = key;
  a.logit = logit;
  a.q = q;
  a.scale = scale;
  a.key_norm = key_norm;
  a.key_eps = key_eps;
  a.bias = bias;
  a.bias_dev = bias_dev;
  a.onorm = onorm;
  a.out_eps = out_eps;
  a.out = out;
  a.out_inv = out_inv;
  if (!bwd) return phase2_forward_launch(dtype, a, st);
  a.g = g;
  a.y = y;
  a.y_inv = y_inv;
  a.dv = dv;
  a.dprev = dprev;
  a.dlse = dlse;
  a.dkey = dkey;
  a.dlogit = dlogit;
  return phase2_backward_launch(dtype, a, grad_query, grad_bias, workspace, st);
}

}  // namespace attnres
