// Block summary of block Attention Residuals (the reference model's
// _attnres_block_summary / _lrid_block_source, model.py:990-1028, with the
// running sums of model.py:2377-2389 and :2451-2463):
//   sum    = partial + x                (the running block sum; partial may be absent)
//   source = sum * c                    (c = count^-alpha, or a learned scale)
// computed in one pass (the reference runs an add and a multiply, five passes
// over the rows; this is four), rounded like the reference's dtype ops:
// sum = round(partial + x), source = round(float(sum) * c).
// Backward, one pass: d_sum_total = round(round(g_source * c) + g_sum), which
// is the gradient of both partial and x, and d c = sum over elements of
// g_source * sum, reduced per CTA and then in a fixed order (deterministic).
// HBM-bound elementwise work: 16-byte packs, grid-stride over up to 16 CTAs per SM.
#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "launch_cache.h"

namespace attnres {

// One 16-byte pack per thread per pass and up to 16 CTAs of 256 threads per
// SM (8 resident): measured 93 % of the copy bandwidth on B200, against 68 %
// for four packs per thread on fewer CTAs.
constexpr int kSummaryUnroll = 1;
constexpr int kSummaryCtasPerSm = 16;

struct SummaryArgs {
  const void* partial;  // nullable (first sublayer of a block)
  const void* x;
  const float* scale_dev;  // nullable: use `scale`
  float scale;
  void* sum;     // nullable: only the scaled source is wanted
  void* source;
  long long n;
};

struct SummaryBwdArgs {
  const void* g_source;  // nullable
  const void* g_sum;     // nullable
  const void* sum;       // saved forward sum; needed for the scale gradient
  const float* scale_dev;
  float scale;
  void* g_total;    // gradient of partial and of x
  float* partials;  // per-CTA partial sums of g_source * sum, or null
  long long n;
};

template <typename T, int VEC>
__global__ void __launch_bounds__(256) summary_fwd_kernel(const __grid_constant__ SummaryArgs a) {
  const float c = a.scale_dev ? *a.scale_dev : a.scale;
  const T* x = static_cast<const T*>(a.x);
  const T* p = static_cast<const T*>(a.partial);
  T* sm = static_cast<T*>(a.sum);
  T* src = static_cast<T*>(a.source);
  const long long nv = a.n / VEC;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  // kSummaryUnroll packs per thread per pass, all loads issued before any use
  constexpr int U = kSummaryUnroll;
  for (long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < nv; i0 += U * step) {
    Pack<T, VEC> xv[U], pv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * step;
      if (i < nv) {
        xv[u] = load_stream<T, VEC>(x + i * VEC);
        if (p) pv[u] = load_stream<T, VEC>(p + i * VEC);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * step;
      if (i >= nv) break;
      Pack<T, VEC> yv, sv;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float y = Elem<T>::to_f(xv[u].e[e]) + (p ? Elem<T>::to_f(pv[u].e[e]) : 0.f);
        yv.e[e] = Elem<T>::from_f(y);
        sv.e[e] = Elem<T>::from_f(Elem<T>::to_f(yv.e[e]) * c);
      }
      if (sm) *reinterpret_cast<Pack<T, VEC>*>(sm + i * VEC) = yv;
      *reinterpret_cast<Pack<T, VEC>*>(src + i * VEC) = sv;
    }
  }
  // ragged tail (n % VEC elements)
  const long long t0 = nv * VEC;
  const long long ti = t0 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (ti < a.n) {
    const float y = Elem<T>::to_f(x[ti]) + (p ? Elem<T>::to_f(p[ti]) : 0.f);
    const T yt = Elem<T>::from_f(y);
    if (sm) sm[ti] = yt;
    src[ti] = Elem<T>::from_f(Elem<T>::to_f(yt) * c);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) summary_bwd_kernel(const __grid_constant__ SummaryBwdArgs a) {
  __shared__ float red[8];
  const float c = a.scale_dev ? *a.scale_dev : a.scale;
  const T* gs = static_cast<const T*>(a.g_source);
  const T* gm = static_cast<const T*>(a.g_sum);
  const T* y = static_cast<const T*>(a.sum);
  T* gt = static_cast<T*>(a.g_total);
  const bool want_dc = a.partials != nullptr && gs != nullptr;
  float dc = 0.f;
  const long long nv = a.n / VEC;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  constexpr int U = kSummaryUnroll;
  for (long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < nv; i0 += U * step) {
    Pack<T, VEC> sv[U], mv[U], yv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * step;
      if (i < nv) {
        if (gs) sv[u] = load_stream<T, VEC>(gs + i * VEC);
        if (gm) mv[u] = load_stream<T, VEC>(gm + i * VEC);
        if (want_dc) yv[u] = load_stream<T, VEC>(y + i * VEC);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * step;
      if (i >= nv) break;
      Pack<T, VEC> ov;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float g = 0.f;
        if (gs) {
          const float gsf = Elem<T>::to_f(sv[u].e[e]);
          g = Elem<T>::to_f(Elem<T>::from_f(gsf * c));
          if (want_dc) dc = fmaf(gsf, Elem<T>::to_f(yv[u].e[e]), dc);
        }
        if (gm) g += Elem<T>::to_f(mv[u].e[e]);
        ov.e[e] = Elem<T>::from_f(g);
      }
      *reinterpret_cast<Pack<T, VEC>*>(gt + i * VEC) = ov;
    }
  }
  const long long t0 = nv * VEC;
  const long long ti = t0 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (ti < a.n) {
    float g = 0.f;
    if (gs) {
      const float gsf = Elem<T>::to_f(gs[ti]);
      g = Elem<T>::to_f(Elem<T>::from_f(gsf * c));
      if (want_dc) dc = fmaf(gsf, Elem<T>::to_f(y[ti]), dc);
    }
    if (gm) g += Elem<T>::to_f(gm[ti]);
    gt[ti] = Elem<T>::from_f(g);
  }
  if (!want_dc) return;
  // fixed-order CTA reduction: warp shuffles, then the 8 warp sums in order
  dc = warp_sum(dc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w];
    a.partials[blockIdx.x] = s;
  }
}

// ---------------------------------------------------------------------------
// Block summary with the value norm (attnres_block_value_norm,
// model.py:991-992 and :1004-1005): sum = round(partial + x), source =
// round(rms_norm(sum)) over each row of `d` elements (fp32 eps, as
// F.rms_norm takes for 16-bit inputs). One warp per row; the inverse rms is
// saved for the backward.
// Backward: d_sum_total = round(round(inv * (g - s_hat * mean(g . s_hat))) + g_sum)
// with s_hat = sum * inv -- the gradient of partial and of x.
// ---------------------------------------------------------------------------
struct SummaryNormArgs {
  const void* partial;  // nullable
  const void* x;
  void* sum;  // nullable
  void* source;
  float* inv;  // [rows]
  const void* g_source;
  const void* g_sum;  // nullable
  void* g_total;
  long long rows;
  int d;
  float eps;
};

template <typename T, int VEC>
__global__ void __launch_bounds__(256) summary_norm_fwd_kernel(const __grid_constant__ SummaryNormArgs a) {
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= a.rows) return;
  const int np = a.d / VEC;
  const T* x = static_cast<const T*>(a.x) + row * a.d;
  const T* p = a.partial ? static_cast<const T*>(a.partial) + row * a.d : nullptr;
  T* sm = a.sum ? static_cast<T*>(a.sum) + row * a.d : nullptr;
  T* src = static_cast<T*>(a.source) + row * a.d;
  float ss = 0.f;
  for (int i = lane; i < np; i += 32) {
    const Pack<T, VEC> xv = load_pack<T, VEC>(x + i * VEC);
    Pack<T, VEC> pv;
    if (p) pv = load_pack<T, VEC>(p + i * VEC);
    Pack<T, VEC> yv;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      yv.e[e] = Elem<T>::from_f(Elem<T>::to_f(xv.e[e]) + (p ? Elem<T>::to_f(pv.e[e]) : 0.f));
      const float y = Elem<T>::to_f(yv.e[e]);
      ss = fmaf(y, y, ss);
    }
    if (sm) *reinterpret_cast<Pack<T, VEC>*>(sm + i * VEC) = yv;
  }
  const float inv = rsqrtf(warp_sum(ss) / a.d + a.eps);
  if (lane == 0) a.inv[row] = inv;
  // second pass over the row (L1 / L2 resident) for the normalised source
  for (int i = lane; i < np; i += 32) {
    const Pack<T, VEC> xv = load_pack<T, VEC>(x + i * VEC);
    Pack<T, VEC> pv;
    if (p) pv = load_pack<T, VEC>(p + i * VEC);
    float o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float y = Elem<T>::to_f(Elem<T>::from_f(Elem<T>::to_f(xv.e[e]) + (p ? Elem<T>::to_f(pv.e[e]) : 0.f)));
      o[e] = y * inv;
    }
    store_pack<T, VEC>(src + i * VEC, o);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) summary_norm_bwd_kernel(const __grid_constant__ SummaryNormArgs a) {
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= a.rows) return;
  const int np = a.d / VEC;
  const T* g = static_cast<const T*>(a.g_source) + row * a.d;
  const T* gm = a.g_sum ? static_cast<const T*>(a.g_sum) + row * a.d : nullptr;
  const T* y = static_cast<const T*>(a.sum) + row * a.d;
  T* gt = static_cast<T*>(a.g_total) + row * a.d;
  const float inv = a.inv[row];
  float gy = 0.f;
  for (int i = lane; i < np; i += 32) {
    const Pack<T, VEC> gv = load_pack<T, VEC>(g + i * VEC);
    const Pack<T, VEC> yv = load_pack<T, VEC>(y + i * VEC);
#pragma unroll
    for (int e = 0; e < VEC; ++e) gy = fmaf(Elem<T>::to_f(gv.e[e]), Elem<T>::to_f(yv.e[e]) * inv, gy);
  }
  const float m = warp_sum(gy) / a.d;
  for (int i = lane; i < np; i += 32) {
    const Pack<T, VEC> gv = load_pack<T, VEC>(g + i * VEC);
    const Pack<T, VEC> yv = load_pack<T, VEC>(y + i * VEC);
    Pack<T, VEC> mv;
    if (gm) mv = load_pack<T, VEC>(gm + i * VEC);
    float o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float sh = Elem<T>::to_f(yv.e[e]) * inv;
      float dx = Elem<T>::to_f(Elem<T>::from_f(inv * (Elem<T>::to_f(gv.e[e]) - sh * m)));
      if (gm) dx += Elem<T>::to_f(mv.e[e]);
      o[e] = dx;
    }
    store_pack<T, VEC>(gt + i * VEC, o);
  }
}

template <typename T>
static cudaError_t summary_norm_t(bool bwd, const SummaryNormArgs& a, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const unsigned grid = static_cast<unsigned>((a.rows * 32 + 255) / 256);
  if (vec) {
    if (bwd) summary_norm_bwd_kernel<T, V><<<grid, 256, 0, st>>>(a);
    else summary_norm_fwd_kernel<T, V><<<grid, 256, 0, st>>>(a);
  } else {
    if (bwd) summary_norm_bwd_kernel<T, 1><<<grid, 256, 0, st>>>(a);
    else summary_norm_fwd_kernel<T, 1><<<grid, 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

static bool al16n(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t summary_norm_launch(bool bwd, long long rows, int d, int dtype, const void* partial, const void* x,
                                float eps, void* sum, void* source, float* inv, const void* g_source,
                                const void* g_sum, void* g_total, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  SummaryNormArgs a{partial, x, sum, source, inv, g_source, g_sum, g_total, rows, d, eps};
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const void* ptrs[] = {partial, x, sum, source, g_source, g_sum, g_total};
  bool vec = (static_cast<long long>(d) * esz) % 16 == 0;
  for (const void* q : ptrs) vec = vec && (q == nullptr || al16n(q));
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return summary_norm_t<float>(bwd, a, vec, st);
    case ATTNRES_DTYPE_F16: return summary_norm_t<__half>(bwd, a, vec, st);
    default: return summary_norm_t<__nv_bfloat16>(bwd, a, vec, st);
  }
}

static int summary_grid(long long n, int vec) {
  int nsm = 148;
  if (cached_sm_count(&nsm) != cudaSuccess) nsm = 148;
  const long long need = (n / vec + 256 * kSummaryUnroll - 1) / (256 * kSummaryUnroll) + 1;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(need, static_cast<long long>(kSummaryCtasPerSm) * nsm)));
}

int summary_bwd_grid(long long n) { return summary_grid(n, 1); }

template <typename T>
static cudaError_t summary_fwd_t(const SummaryArgs& a, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (vec) {
    summary_fwd_kernel<T, V><<<summary_grid(a.n, V), 256, 0, st>>>(a);
  } else {
    summary_fwd_kernel<T, 1><<<summary_grid(a.n, 1), 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t summary_bwd_t(const SummaryBwdArgs& a, bool vec, int grid, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (vec) summary_bwd_kernel<T, V><<<grid, 256, 0, st>>>(a);
  else summary_bwd_kernel<T, 1><<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t summary_forward_launch(long long n, int dtype, const void* partial, const void* x,
                                   const float* scale_dev, float scale, void* sum, void* source,
                                   cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  SummaryArgs a{partial, x, scale_dev, scale, sum, source, n};
  const bool vec = al16(x) && al16(source) && (!partial || al16(partial)) && (!sum || al16(sum));
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return summary_fwd_t<float>(a, vec, st);
    case ATTNRES_DTYPE_F16: return summary_fwd_t<__half>(a, vec, st);
    default: return summary_fwd_t<__nv_bfloat16>(a, vec, st);
  }
}

cudaError_t summary_backward_launch(long long n, int dtype, const void* g_source, const void* g_sum,
                                    const void* sum, const float* scale_dev, float scale, void* g_total,
                                    float* grad_scale, float* partials, cudaStream_t st) {
  if (n == 0) {
    if (grad_scale) return cudaMemsetAsync(grad_scale, 0, sizeof(float), st);
    return cudaSuccess;
  }
  const int grid = summary_bwd_grid(n);
  const bool want_dc = grad_scale != nullptr && g_source != nullptr;
  SummaryBwdArgs a{g_source, g_sum, sum, scale_dev, scale, g_total, want_dc ? partials : nullptr, n};
  const bool vec = al16(g_total) && (!g_source || al16(g_source)) && (!g_sum || al16(g_sum)) &&
                   (!want_dc || al16(sum));
  cudaError_t e;
  switch (dtype) {
    case ATTNRES_DTYPE_F32: e = summary_bwd_t<float>(a, vec, grid, st); break;
    case ATTNRES_DTYPE_F16: e = summary_bwd_t<__half>(a, vec, grid, st); break;
    default: e = summary_bwd_t<__nv_bfloat16>(a, vec, grid, st);
  }
  if (e != cudaSuccess) return e;
  if (grad_scale) {
    if (want_dc) launch_reduce_partials(partials, grid, 1, 0, 1, grad_scale, st);
    else e = cudaMemsetAsync(grad_scale, 0, sizeof(float), st);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace attnres
