// Key-from-value LRID read, forward, in one persistent kernel: the key
// projection keys_s = rms_norm(V_s) @ W^T (model.py:344-356) fused with the
// depth softmax and the weighted sum (the read of attnres_ops.py:4195-4232).
//
// A CTA takes token tiles of 8 tokens x all S sources. Each tile streams its
// value rows through shared memory twice, in 64-column chunks (one 128-byte
// swizzle span of 16-bit elements):
//   phase A: TMA loads the chunk of every source (one 8-row box per source,
//     rows (s mod 16) * 8 + t of a 128-row UMMA tile per group of 16 sources)
//     plus the chunk of W; one thread issues tcgen05.mma M=128 N=64 K=16 per
//     group into a TMEM accumulator (V_rows @ W^T); the 4 epilogue warps sum
//     the squares of their row from the same staged tile. After the last
//     chunk the epilogue scales by the inverse rms, rounds the keys to the
//     value dtype (saved for the backward), applies the per-head key norm,
//     forms the logits and the softmax over sources (saved: alpha);
//   phase B: the same chunks again -- now L2 hits: phase A loads them with an
//     evict-last policy, phase B with evict-first, and one tile of all CTAs
//     is ~80 MB -- and the epilogue warps form out = sum_s alpha_s V_s.
// So V crosses HBM once per step instead of twice (a projection kernel, then
// a read kernel). Warp 0 issues the TMA loads, warp 1 the MMAs, warps 2-5
// consume. The ring of stages is used strictly in order by every role; every
// mbarrier wait is bounded and reports through a status word; TMEM is freed.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "tma.cuh"
#include "umma.cuh"

namespace attnres {

constexpr int kKvfMaxSources = 32;   // two 16-source UMMA groups
constexpr int kKvfTokens = 8;        // tokens per tile (one 8-row box per source)
constexpr int kKvfMaxStages = 8;
constexpr int kKvfR = 64;            // key rank
constexpr int kKvfK = 64;            // columns per chunk
constexpr int kKvfMaxHeads = 8;
constexpr int kKvfThreads = 6 * 32;  // TMA, MMA, 4 epilogue warps

static __device__ unsigned int g_kvf_status = 0;

struct KvfArgs {
  CUtensorMap vmap[kKvfMaxSources];  // V_s as [N rows, d cols], box 64 x 8
  CUtensorMap wmap;                  // W as [R rows, d cols], box 64 x 64
  const void* q;                     // static query [H, dk] (value dtype)
  const float* bias;                 // [S] or null
  void* out;                         // [N, d]
  void* keys;                        // [S][N][R]
  float* vinv;                       // [S][N]
  float* alpha;                      // [N][H][S]
  long long N, ntiles;
  int S, d, H, G, stages, value_norm, key_norm;
  float value_eps, key_eps, scale;
  uint32_t idesc;
};

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tiled 2-D TMA load with an L2 cache policy
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

template <typename T, int H>
__global__ void __launch_bounds__(kKvfThreads, 1) kvfused_fwd_kernel(const __grid_constant__ KvfArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.S, d = a.d, G = a.G, NST = a.stages;
  constexpr uint32_t kRowBytes = kKvfK * sizeof(T);              // 128
  constexpr uint32_t kGroupBytes = 128 * kRowBytes;              // one 128-row UMMA tile
  constexpr uint32_t kBoxBytes = kKvfTokens * kRowBytes;         // one source's 8 rows
  constexpr uint32_t kWBytes = kKvfR * kRowBytes;
  const uint32_t stage_bytes = G * kGroupBytes + kWBytes;
  unsigned char* stages = base;
  float* lg = reinterpret_cast<float*>(stages + NST * stage_bytes);  // [8][H][32] logits
  float* al = lg + kKvfTokens * H * 32;                                // [8][H][32] weights
  float* qs = al + kKvfTokens * H * 32;                                // [64] query
  uint64_t* full = reinterpret_cast<uint64_t*>(qs + kKvfR);
  uint64_t* empty = full + kKvfMaxStages;
  uint64_t* acc_full = empty + kKvfMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = d / kKvfK;
  constexpr uint32_t kTmemCols = 256;  // 2 accumulators x 2 groups x 64 columns

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 4);  // the MMA thread + the 4 epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // wait for the previous launch before taking TMEM, so no CTA holds tensor
  // memory while it waits
  pdl_wait_then_release();
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: phase A then phase B chunks of every tile --
    // lane 0 waits for the stage and posts the byte count; lane s issues the
    // box of source s (the issue of 17+ small boxes spread over the warp)
    const uint64_t keep = l2_policy_evict_last(), drop = l2_policy_evict_first();
    long long it = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
      const int t0 = static_cast<int>(tile * kKvfTokens);
      for (int ph = 0; ph < 2 && ok; ++ph) {
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = static_cast<int>(it % NST);
          const uint32_t par = static_cast<uint32_t>((it / NST) & 1);
          int good = 1;
          if (lane == 0) {
            if (*abort_flag || !mbar_wait_bounded(&empty[st], par ^ 1u)) {
              atomicOr(&g_kvf_status, kStatusEmptyWaitTimeout);
              *abort_flag = 1;
              good = 0;
            } else {
              mbar_arrive_expect_tx(&full[st], S * kBoxBytes + (ph == 0 ? kWBytes : 0));
            }
          }
          if (!__shfl_sync(0xffffffffu, good, 0)) {
            ok = false;
            break;
          }
          unsigned char* sa = stages + st * stage_bytes;
          if (lane < S)
            tma_load_2d_hint(sa + (lane >> 4) * kGroupBytes + (lane & 15) * kBoxBytes, &a.vmap[lane], kc * kKvfK,
                             t0, &full[st], ph == 0 ? keep : drop);
          if (ph == 0 && lane == 31) tma_load_2d(sa + G * kGroupBytes, &a.wmap, kc * kKvfK, 0, &full[st]);
          __syncwarp();
        }
      }
    }
    if (!ok && lane == 0) {
      // let the copies already issued land before the CTA can exit
      for (long long j = (it > NST ? it - NST : 0); j < it; ++j)
        if (!mbar_wait_bounded(&full[j % NST], static_cast<uint32_t>((j / NST) & 1)))
          atomicOr(&g_kvf_status, kStatusDrainTimeout);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ---------------------------------------------
    if (lane == 0) {
      long long it = 0, tcount = 0;
      bool issued_any = false, ok = true;
      for (long long tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x, ++tcount) {
        const int ab = static_cast<int>(tcount & 1);
        if (*abort_flag || !mbar_wait_bounded(&acc_empty[ab], static_cast<uint32_t>(((tcount >> 1) & 1) ^ 1))) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dbase = tmem_base + ab * 128;
        for (int ph = 0; ph < 2 && ok; ++ph) {
          for (int kc = 0; kc < nk; ++kc, ++it) {
            const int st = static_cast<int>(it % NST);
            if (*abort_flag || !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / NST) & 1))) {
              atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
              *abort_flag = 1;
              ok = false;
              break;
            }
            if (ph == 1) {
              mbar_arrive(&empty[st]);  // phase B needs no MMA: keep the stage count
              continue;
            }
            tc_fence_after();
            const unsigned char* sa = stages + st * stage_bytes;
            const uint64_t db = umma_desc_sw128(sa + G * kGroupBytes);
            for (int g = 0; g < G; ++g) {
              const uint64_t da = umma_desc_sw128(sa + g * kGroupBytes);
#pragma unroll
              for (int k = 0; k < kKvfK / 16; ++k)  // K = 16 per instruction: +32 bytes in the swizzle atom
                umma_f16(dbase + g * kKvfR, da + 2 * k, db + 2 * k, a.idesc, (kc > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&empty[st]);
            issued_any = true;
            if (kc == nk - 1) umma_commit(&acc_full[ab]);
          }
        }
      }
      umma_commit(done);
      if (issued_any && !mbar_wait_bounded(done, 0)) atomicOr(&g_kvf_status, kStatusDrainTimeout);
    }
  } else {
    // ---------------- epilogue: 4 warps ----------------------------------------
    const int e = threadIdx.x - 64;        // 0..127
    const int q = warp & 3;                // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;           // row of each group's 128-row tile
    const int rt = r & 7, rs = r >> 3;     // its token and source within the group
    const int ew = e >> 5;                 // epilogue warp 0..3
    constexpr int DK = kKvfR / H;
    const int dvh = d / H;
    // the static query, rounded to T as the reference casts it, in shared memory
    if (e < kKvfR) qs[e] = Elem<T>::to_f(static_cast<const T*>(a.q)[e]);
    consumer_sync(128);
    T* keys = static_cast<T*>(a.keys);
    T* out = static_cast<T*>(a.out);
    long long it = 0, tcount = 0;
    for (long long tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++tcount) {
      const long long t0 = tile * kKvfTokens;
      bool ok = true;
      // ---- phase A: sums of squares of this thread's rows ----------------
      float ss[2] = {0.f, 0.f};
      for (int kc = 0; kc < nk; ++kc, ++it) {
        const int st = static_cast<int>(it % NST);
        if (*abort_flag || !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / NST) & 1))) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (a.value_norm) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            if (g >= G || g * 16 + rs >= S) continue;
            const unsigned char* rowp = stages + st * stage_bytes + g * kGroupBytes + r * kRowBytes;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const Pack<T, 8> p = *reinterpret_cast<const Pack<T, 8>*>(rowp + ((c ^ rt) * 16));
              const uint32_t* pw = reinterpret_cast<const uint32_t*>(p.e);
#pragma unroll
              for (int i = 0; i < 4; ++i) Mixed16<T>::sq_step(ss[g], pw[i]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      const int ab = static_cast<int>(tcount & 1);
      if (ok && (*abort_flag || !mbar_wait_bounded(&acc_full[ab], static_cast<uint32_t>((tcount >> 1) & 1)))) {
        atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
        *abort_flag = 1;
        ok = false;
      }
      if (consumer_sync_or(128, !ok)) break;
      tc_fence_after();
      // ---- keys (saved in T), per-head key norm and logits -----------------
      const long long tok = t0 + rt;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        if (g >= G) break;
        const int s = g * 16 + rs;
        const bool valid = s < S && tok < a.N;
        const float inv = a.value_norm ? rsqrtf(ss[g] / d + a.value_eps) : 1.f;
        float kss[H], dot[H];
#pragma unroll
        for (int h = 0; h < H; ++h) kss[h] = dot[h] = 0.f;
        T* kp = keys + (static_cast<long long>(s) * a.N + tok) * kKvfR;
#pragma unroll
        for (int c0 = 0; c0 < kKvfR; c0 += 16) {
          float v[16];
          tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ab * 128 + g * kKvfR + c0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            v[i] = Elem<T>::to_f(Elem<T>::from_f(v[i] * inv));  // the key, rounded to T
            kss[(c0 + i) / DK] = fmaf(v[i], v[i], kss[(c0 + i) / DK]);
            dot[(c0 + i) / DK] = fmaf(v[i], qs[c0 + i], dot[(c0 + i) / DK]);
          }
          if (valid) {
            float o0[8], o1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              o0[i] = v[i];
              o1[i] = v[8 + i];
            }
            store_pack<T, 8>(kp + c0, o0);
            store_pack<T, 8>(kp + c0 + 8, o1);
          }
        }
        if (s < S) {
          if (valid && a.vinv) a.vinv[static_cast<long long>(s) * a.N + tok] = inv;
          const float b = a.bias ? a.bias[s] : 0.f;
#pragma unroll
          for (int h = 0; h < H; ++h) {
            const float kinv = a.key_norm ? rsqrtf(kss[h] / DK + a.key_eps) : 1.f;
            lg[(rt * H + h) * 32 + s] = dot[h] * kinv * a.scale + b;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      consumer_sync(128);
      // ---- softmax over sources per (token, head) --------------------------
      for (int p = ew; p < kKvfTokens * H; p += 4) {
        const float l = lane < S ? lg[p * 32 + lane] : -INFINITY;
        const float m = warp_max(l);
        const float ex = lane < S ? expf(l - m) : 0.f;
        const float w = ex / warp_sum(ex);
        // weights rounded to T, as the reference casts them (attnres_ops.py:4229)
        al[p * 32 + lane] = Elem<T>::to_f(Elem<T>::from_f(w));
        const long long tk = t0 + p / H;
        if (lane < S && tk < a.N && a.alpha) a.alpha[(tk * H + p % H) * S + lane] = w;
      }
      consumer_sync(128);
      // ---- phase B: out = sum_s alpha_s V_s, 4 columns of one token per thread
      const int tt = e >> 4, piece = e & 15, u = piece >> 1, half = piece & 1;
      const long long otok = t0 + tt;
      const unsigned col = ((u ^ tt) * 16) + half * 8;
      for (int kc = 0; kc < nk; ++kc, ++it) {
        const int st = static_cast<int>(it % NST);
        if (ok && (*abort_flag || !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / NST) & 1)))) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
          ok = false;
        }
        if (ok) {
          const int h = (kc * kKvfK) / dvh;
          const float* w = al + (tt * H + h) * 32;
          const unsigned char* rowt = stages + st * stage_bytes + tt * kRowBytes + col;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int s = 0; s < S; ++s) {
            const Pack<T, 4> v =
                *reinterpret_cast<const Pack<T, 4>*>(rowt + (s >> 4) * kGroupBytes + (s & 15) * kBoxBytes);
            const float ws = w[s];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(ws, Elem<T>::to_f(v.e[i]), acc[i]);
          }
          if (otok < a.N) store_pack<T, 4>(out + otok * d + kc * kKvfK + piece * 4, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      if (consumer_sync_or(128, !ok)) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool kvfused_eligible(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                      const int64_t* vstr, const void* w, long long w_stride, const char** why) {
  *why = "";
  if (dtype != ATTNRES_DTYPE_BF16 && dtype != ATTNRES_DTYPE_F16) return *why = "needs f16/bf16 rows", false;
  if (R != kKvfR) return *why = "needs key_dim 64", false;
  if (S < 2 || S > kKvfMaxSources) return *why = "needs 2..32 sources", false;
  if (N < 1 || d % kKvfK) return *why = "needs value_dim a multiple of 64", false;
  if (H < 1 || H > kKvfMaxHeads || (H & (H - 1)) || (d / H) % kKvfK) return *why = "needs a power-of-two head count with (value_dim / heads) % 64 == 0", false;
  if (N > 0x7fffffffLL) return *why = "too many tokens for 32-bit TMA coordinates", false;
  if (!aligned16p(w) || (w_stride * 2) % 16) return *why = "weight rows must be 16-byte aligned", false;
  for (int s = 0; s < S; ++s)
    if (!aligned16p(values[s]) || (vstr[s] * 2) % 16) return *why = "value rows must be 16-byte aligned", false;
  return encode_fn() != nullptr || (*why = "no cuTensorMapEncodeTiled", false);
}

cudaError_t kvfused_forward_launch(int S, long long N, int d, int H, int dtype, const void* const* values,
                                   const int64_t* vstr, const void* w, long long w_stride, int value_norm,
                                   float value_eps, const void* q, float scale, int key_norm, float key_eps,
                                   const float* bias, void* out, void* keys, float* vinv, float* alpha,
                                   cudaStream_t st) {
  KvfArgs a{};
  for (int s = 0; s < S; ++s)
    if (!encode_2d(&a.vmap[s], dtype, values[s], N, d, vstr[s], kKvfTokens)) return cudaErrorInvalidValue;
  if (!encode_2d(&a.wmap, dtype, w, kKvfR, d, w_stride, kKvfR)) return cudaErrorInvalidValue;
  a.q = q;
  a.bias = bias;
  a.out = out;
  a.keys = keys;
  a.vinv = vinv;
  a.alpha = alpha;
  a.N = N;
  a.ntiles = (N + kKvfTokens - 1) / kKvfTokens;
  a.S = S;
  a.d = d;
  a.H = H;
  a.G = (S + 15) / 16;
  a.value_norm = value_norm;
  a.key_norm = key_norm;
  a.value_eps = value_eps;
  a.key_eps = key_eps;
  a.scale = scale;
  a.idesc = umma_idesc_f16(dtype == ATTNRES_DTYPE_BF16 ? 1u : 0u, 0u, 0u, 128, kKvfR);
  const size_t stage_bytes = static_cast<size_t>(a.G) * 128 * kKvfK * 2 + kKvfR * kKvfK * 2;
  const size_t fixed = 1024 + 2 * sizeof(float) * kKvfTokens * H * 32 + sizeof(float) * kKvfR + 256;
  int dev = 0, cap = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
  a.stages = static_cast<int>(std::min<size_t>(kKvfMaxStages, (static_cast<size_t>(cap) - fixed) / stage_bytes));
  if (a.stages < 2) return cudaErrorInvalidConfiguration;
  const size_t smem = fixed + static_cast<size_t>(a.stages) * stage_bytes;
  const bool bf = dtype == ATTNRES_DTYPE_BF16;
  void (*fn)(KvfArgs) = nullptr;
  switch (H) {
    case 1: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 1> : kvfused_fwd_kernel<__half, 1>; break;
    case 2: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 2> : kvfused_fwd_kernel<__half, 2>; break;
    case 4: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 4> : kvfused_fwd_kernel<__half, 4>; break;
    default: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 8> : kvfused_fwd_kernel<__half, 8>; break;
  }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int nsm = 0;
  if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(std::max<long long>(1, std::min<long long>(a.ntiles, nsm))));
  cfg.blockDim = dim3(kKvfThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t read_kvfused_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_kvf_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_kvf_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
