// Device helpers shared by the AttnRes read kernels: element types, 16/8/4-byte
// streaming vector loads, and deterministic lane-group reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/attnres_b200.h"

namespace attnres {

constexpr int kMaxSources = ATTNRES_MAX_SOURCES;

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T> struct Elem;

template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// A VEC-element slice of one row, moved as one aligned memory transaction.
template <typename T, int VEC> struct alignas(sizeof(T) * VEC) Pack {
  T e[VEC];
};

// Read-only streaming load of one pack. Values are read exactly once per
// kernel, so the 16/8/4-byte forms skip L1 allocation.
template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> load_stream(const T* p) {
  Pack<T, VEC> r;
  constexpr int B = sizeof(T) * VEC;
  if constexpr (B == 16) {
    uint4 u;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "l"(p));
    *reinterpret_cast<uint4*>(&r) = u;
  } else if constexpr (B == 8) {
    uint2 u;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(u.x), "=r"(u.y)
                 : "l"(p));
    *reinterpret_cast<uint2*>(&r) = u;
  } else if constexpr (B == 4) {
    uint32_t u;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(u) : "l"(p));
    *reinterpret_cast<uint32_t*>(&r) = u;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.e[i] = __ldg(p + i);
  }
  return r;
}

// Plain (L1-cached) load of one pack; used for data that is read again
// shortly (the upstream gradient, the saved output).
template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> load_pack(const T* p) {
  return *reinterpret_cast<const Pack<T, VEC>*>(p);
}

template <typename T, int VEC>
__device__ __forceinline__ void store_pack(T* p, const float (&x)[VEC]) {
  Pack<T, VEC> r;
#pragma unroll
  for (int i = 0; i < VEC; ++i) r.e[i] = Elem<T>::from_f(x[i]);
  *reinterpret_cast<Pack<T, VEC>*>(p) = r;
}

// acc[e] = fma(w, x[e], acc[e]) over one pack, two lanes per instruction with
// sm_100's packed fp32 FMA (each lane rounds exactly like fmaf). bf16 halves
// widen to fp32 by a shift / mask of their 32-bit word.
__device__ __forceinline__ void fma2(float& a0, float& a1, float w, float x0, float x1) {
  asm("{\n\t.reg .b64 xa, wa, aa;\n\t"
      "mov.b64 xa, {%2, %3};\n\tmov.b64 wa, {%4, %4};\n\tmov.b64 aa, {%0, %1};\n\t"
      "fma.rn.f32x2 aa, wa, xa, aa;\n\tmov.b64 {%0, %1}, aa;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(w));
}

template <typename T, int VEC> __device__ __forceinline__ void unpack2(const Pack<T, VEC>&, int, float&, float&);

template <typename T, int VEC>
__device__ __forceinline__ void axpy_pack(float (&acc)[VEC], float w, const Pack<T, VEC>& x) {
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) {
    float x0, x1;
    unpack2<T, VEC>(x, i, x0, x1);
    fma2(acc[2 * i], acc[2 * i + 1], w, x0, x1);
  }
}

__device__ __forceinline__ void mul2(float& y0, float& y1, float w, float x0, float x1) {
  asm("{\n\t.reg .b64 xa, wa, ya;\n\t"
      "mov.b64 xa, {%2, %3};\n\tmov.b64 wa, {%4, %4};\n\t"
      "mul.rn.f32x2 ya, wa, xa;\n\tmov.b64 {%0, %1}, ya;\n\t}"
      : "=f"(y0), "=f"(y1)
      : "f"(x0), "f"(x1), "f"(w));
}

__device__ __forceinline__ void fma2v(float& a0, float& a1, float g0, float g1, float x0, float x1) {
  asm("{\n\t.reg .b64 xa, ga, aa;\n\t"
      "mov.b64 xa, {%2, %3};\n\tmov.b64 ga, {%4, %5};\n\tmov.b64 aa, {%0, %1};\n\t"
      "fma.rn.f32x2 aa, ga, xa, aa;\n\tmov.b64 {%0, %1}, aa;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(g0), "f"(g1));
}

// Widen element pair i of a pack to fp32.
template <typename T, int VEC>
__device__ __forceinline__ void unpack2(const Pack<T, VEC>& x, int i, float& x0, float& x1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t u = reinterpret_cast<const uint32_t*>(x.e)[i];
    x0 = __uint_as_float(u << 16);
    x1 = __uint_as_float(u & 0xffff0000u);
  } else {
    x0 = Elem<T>::to_f(x.e[2 * i]);
    x1 = Elem<T>::to_f(x.e[2 * i + 1]);
  }
}

// acc + sum_e g[e] * x[e], even and odd elements in two packed chains.
template <typename T, int VEC>
__device__ __forceinline__ float dot_pack(float acc, const float (&g)[VEC], const Pack<T, VEC>& x) {
  float a0 = acc, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) {
    float x0, x1;
    unpack2<T, VEC>(x, i, x0, x1);
    fma2v(a0, a1, g[2 * i], g[2 * i + 1], x0, x1);
  }
  return a0 + a1;
}

// ---------------------------------------------------------------------------
// sm_100 mixed-precision FMA: fp32 accumulator += 16-bit a * 16-bit b, the
// operands widened inside the FMA (no separate conversion instructions). The
// 16-bit halves of a 32-bit word are taken as register halves.
// ---------------------------------------------------------------------------
template <typename T> struct Mixed16;
template <> struct Mixed16<__nv_bfloat16> {
  // a0 += lo(x) * w, a1 += hi(x) * w
  static __device__ __forceinline__ void fma_w(float& a0, float& a1, uint32_t x, uint16_t w) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "fma.rn.f32.bf16 %0, l, %3, %0;\n\tfma.rn.f32.bf16 %1, h, %3, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(x), "h"(w));
  }
  // a0 += lo(x) * lo(y), a1 += hi(x) * hi(y)
  static __device__ __forceinline__ void fma_pp(float& a0, float& a1, uint32_t x, uint32_t y) {
    asm("{\n\t.reg .b16 xl, xh, yl, yh;\n\tmov.b32 {xl, xh}, %2;\n\tmov.b32 {yl, yh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, xl, yl, %0;\n\tfma.rn.f32.bf16 %1, xh, yh, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(x), "r"(y));
  }
  // one chain each, element order lo then hi: ss += k*k, dot += k*q
  static __device__ __forceinline__ void key_step(float& ss, float& dot, uint32_t k, uint32_t q) {
    asm("{\n\t.reg .b16 kl, kh, ql, qh;\n\tmov.b32 {kl, kh}, %2;\n\tmov.b32 {ql, qh}, %3;\n\t"
        "fma.rn.f32.bf16 %0, kl, kl, %0;\n\tfma.rn.f32.bf16 %1, kl, ql, %1;\n\t"
        "fma.rn.f32.bf16 %0, kh, kh, %0;\n\tfma.rn.f32.bf16 %1, kh, qh, %1;\n\t}"
        : "+f"(ss), "+f"(dot)
        : "r"(k), "r"(q));
  }
  // one chain, element order lo then hi: ss += k*k
  static __device__ __forceinline__ void sq_step(float& ss, uint32_t k) {
    asm("{\n\t.reg .b16 kl, kh;\n\tmov.b32 {kl, kh}, %1;\n\t"
        "fma.rn.f32.bf16 %0, kl, kl, %0;\n\tfma.rn.f32.bf16 %0, kh, kh, %0;\n\t}"
        : "+f"(ss)
        : "r"(k));
  }
  static __device__ __forceinline__ uint16_t bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
};
template <> struct Mixed16<__half> {
  static __device__ __forceinline__ void fma_w(float& a0, float& a1, uint32_t x, uint16_t w) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "fma.rn.f32.f16 %0, l, %3, %0;\n\tfma.rn.f32.f16 %1, h, %3, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(x), "h"(w));
  }
  static __device__ __forceinline__ void fma_pp(float& a0, float& a1, uint32_t x, uint32_t y) {
    asm("{\n\t.reg .b16 xl, xh, yl, yh;\n\tmov.b32 {xl, xh}, %2;\n\tmov.b32 {yl, yh}, %3;\n\t"
        "fma.rn.f32.f16 %0, xl, yl, %0;\n\tfma.rn.f32.f16 %1, xh, yh, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(x), "r"(y));
  }
  // one chain each, element order lo then hi: ss += k*k, dot += k*q
  static __device__ __forceinline__ void key_step(float& ss, float& dot, uint32_t k, uint32_t q) {
    asm("{\n\t.reg .b16 kl, kh, ql, qh;\n\tmov.b32 {kl, kh}, %2;\n\tmov.b32 {ql, qh}, %3;\n\t"
        "fma.rn.f32.f16 %0, kl, kl, %0;\n\tfma.rn.f32.f16 %1, kl, ql, %1;\n\t"
        "fma.rn.f32.f16 %0, kh, kh, %0;\n\tfma.rn.f32.f16 %1, kh, qh, %1;\n\t}"
        : "+f"(ss), "+f"(dot)
        : "r"(k), "r"(q));
  }
  // one chain, element order lo then hi: ss += k*k
  static __device__ __forceinline__ void sq_step(float& ss, uint32_t k) {
    asm("{\n\t.reg .b16 kl, kh;\n\tmov.b32 {kl, kh}, %1;\n\t"
        "fma.rn.f32.f16 %0, kl, kl, %0;\n\tfma.rn.f32.f16 %0, kh, kh, %0;\n\t}"
        : "+f"(ss)
        : "r"(k));
  }
  static __device__ __forceinline__ uint16_t bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
};

template <typename T> constexpr bool kIs16 = std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value;

// acc[e] += w16 * x[e] over one pack (16-bit T; w16 = the weight in T's bits)
template <typename T, int VEC>
__device__ __forceinline__ void axpy_pack16(float (&acc)[VEC], uint16_t w16, const Pack<T, VEC>& x) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(x.e);
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) Mixed16<T>::fma_w(acc[2 * i], acc[2 * i + 1], u[i], w16);
}

// acc + sum_e x[e] * y[e] over two packs (16-bit T), even and odd elements in
// two chains like dot_pack (identical rounding: the widening is exact)
template <typename T, int VEC>
__device__ __forceinline__ float dot_pack16(float acc, const Pack<T, VEC>& x, const Pack<T, VEC>& y) {
  const uint32_t* ux = reinterpret_cast<const uint32_t*>(x.e);
  const uint32_t* uy = reinterpret_cast<const uint32_t*>(y.e);
  float a0 = acc, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) Mixed16<T>::fma_pp(a0, a1, uy[i], ux[i]);
  return a0 + a1;
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p) {
  return Elem<T>::to_f(__ldg(p));
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
// Sum over aligned groups of `g` lanes (g a power of two <= 32). Every lane of
// the warp must execute the call. The butterfly order is fixed, so the result
// is deterministic and identical on every lane of the group.
__device__ __forceinline__ float group_sum(float v, int g) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < g) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__host__ __device__ constexpr int ceil_div_i(int a, int b) { return (a + b - 1) / b; }

inline int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace attnres
