// Per-head RMS norm of LRID key rows (the reference model's _norm_lrid_key,
// model.py:33-36, applied by LRIDFusedProjection.forward, model.py:363-388):
//   y[r, h*dk + j] = x[r, h*dk + j] * inv[r, h],  inv = rsqrt(mean_j x^2 + eps)
// computed in fp32 and rounded to the key dtype, reading the key slice in
// place from the projection output through a row stride (no split copy).
// Backward: gx = inv * (gy - y * <gy, y> / dk), y = x * inv recomputed in
// fp32 from the (strided) pre-norm rows.
// One thread per (row, head); rows are short (dk <= 256).
#include "common.cuh"
#include "plan.h"

namespace attnres {

template <typename T>
__global__ void __launch_bounds__(256) headnorm_fwd_kernel(long long rows, int width, int heads,
                                                           const T* __restrict__ x, long long xs, float eps,
                                                           T* __restrict__ y, float* __restrict__ inv) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * heads) return;
  const long long r = i / heads;
  const int h = static_cast<int>(i - r * heads);
  const int dk = width / heads;
  const T* xr = x + r * xs + h * dk;
  float ss = 0.f;
  for (int j = 0; j < dk; ++j) {
    const float v = Elem<T>::to_f(xr[j]);
    ss = fmaf(v, v, ss);
  }
  const float iv = rsqrtf(ss / dk + eps);
  T* yr = y + r * width + h * dk;
  for (int j = 0; j < dk; ++j) yr[j] = Elem<T>::from_f(Elem<T>::to_f(xr[j]) * iv);
  if (inv) inv[i] = iv;
}

template <typename T>
__global__ void __launch_bounds__(256) headnorm_bwd_kernel(long long rows, int width, int heads,
                                                           const T* __restrict__ gy, const T* __restrict__ x,
                                                           long long xs, const float* __restrict__ inv,
                                                           T* __restrict__ gx, long long gxs) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * heads) return;
  const long long r = i / heads;
  const int h = static_cast<int>(i - r * heads);
  const int dk = width / heads;
  const T* gr = gy + r * width + h * dk;
  const T* xr = x + r * xs + h * dk;
  const float iv = inv[i];
  // y = x * inv recomputed in fp32 from the pre-norm key
  float s = 0.f;
  for (int j = 0; j < dk; ++j) s = fmaf(Elem<T>::to_f(gr[j]), Elem<T>::to_f(xr[j]) * iv, s);
  const float c = s / dk;
  T* o = gx + r * gxs + h * dk;
  for (int j = 0; j < dk; ++j) o[j] = Elem<T>::from_f(iv * (Elem<T>::to_f(gr[j]) - Elem<T>::to_f(xr[j]) * iv * c));
}

template <typename T>
static cudaError_t headnorm_t(bool bwd, long long rows, int width, int heads, const void* a, long long as,
                              float eps, const void* b, const float* inv_in, void* out, float* inv_out, long long os,
                              cudaStream_t st) {
  const long long n = rows * heads;
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  if (bwd)
    headnorm_bwd_kernel<T><<<grid, 256, 0, st>>>(rows, width, heads, static_cast<const T*>(a),
                                                 static_cast<const T*>(b), as, inv_in, static_cast<T*>(out), os);
  else
    headnorm_fwd_kernel<T><<<grid, 256, 0, st>>>(rows, width, heads, static_cast<const T*>(a), as, eps,
                                                 static_cast<T*>(out), inv_out);
  return cudaGetLastError();
}

cudaError_t headnorm_launch(bool bwd, int dtype, long long rows, int width, int heads, const void* a, long long as,
                            float eps, const void* b, const float* inv_in, void* out, float* inv_out, long long os,
                            cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return headnorm_t<float>(bwd, rows, width, heads, a, as, eps, b, inv_in, out, inv_out, os, st);
    case ATTNRES_DTYPE_F16: return headnorm_t<__half>(bwd, rows, width, heads, a, as, eps, b, inv_in, out, inv_out, os, st);
    default: return headnorm_t<__nv_bfloat16>(bwd, rows, width, heads, a, as, eps, b, inv_in, out, inv_out, os, st);
  }
}

}  // namespace attnres
