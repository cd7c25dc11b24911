// Key-from-value projection of the LRID read (lrid_key_from_value):
//   keys[s][t][:] = inv_rms(V_s[t]) * (V_s[t] @ W^T),  inv_rms = rsqrt(mean(V_s[t]^2) + eps)
// i.e. rms_norm(V_s) @ W^T of the reference's LRIDFusedProjection.project_key_from_value
// (model.py:348-356, value norm model.py:344-346, W = value_key_proj.weight [R, d]).
//
// sm_100a kernel: the dense contraction runs on the 5th-generation tensor cores.
//   * warp 0 (one thread): TMA tiled loads (cp.async.bulk.tensor.2d, 128-byte
//     swizzle, no multicast) of a 128-row x 64-column tile of V_s and the
//     matching 64-column slice of W into a ring of shared-memory stages;
//   * warp 1 (one thread): tcgen05.mma.cta_group::1.kind::f16, M=128, N=R,
//     K=16, accumulating a 128 x R fp32 tile in tensor memory (two
//     accumulator buffers, so the next tile's MMAs overlap this tile's
//     epilogue); tcgen05.commit releases stages and publishes accumulators;
//   * warps 2-5 (one V row per thread): sum of squares of the row from the
//     same shared-memory tiles (so the rms scale costs no extra pass over V),
//     then tcgen05.ld of the accumulator row, scale, round, store.
// Every mbarrier wait is bounded (~2 s); TMEM is always released.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "plan.h"
#include "tma.cuh"
#include "umma.cuh"
#include "launch_cache.h"

namespace attnres {

constexpr int kKpMaxSources = 24;
constexpr int kKpStages = 4;
constexpr int kKpRows = 128;  // UMMA M
constexpr int kKpK = 64;      // columns per stage (one 128-byte swizzle span of bf16)

static __device__ unsigned int g_kp_status = 0;

struct KeyProjArgs {
  CUtensorMap vmap[kKpMaxSources];  // V_s as [N rows, d cols]
  CUtensorMap wmap;                 // W as [R rows, d cols]
  void* keys;                       // [S][N][R] dtype
  float* inv_rms;                   // [S][N], or with keys_normed [N][H]; or null
  // Per-head key norm of the fused output projection (S == 1, no value norm):
  // the first nrm_cols columns of each row, in H heads, rms-normalised from
  // their dtype-rounded values into keys_normed [N][nrm_cols]; null = off.
  void* keys_normed;
  long long N;
  long long ntiles;
  int S, R, d, tiles_per_src, value_norm, H, nrm_cols;
  float eps;
  uint32_t idesc;
};

template <typename T>
__global__ void __launch_bounds__(192, 1) keyproj_tc_kernel(const __grid_constant__ KeyProjArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stage tiles must start on 1024-byte boundaries (128-byte swizzle atoms)
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int R = a.R, d = a.d;
  const uint32_t a_bytes = kKpRows * kKpK * sizeof(T);
  const uint32_t b_bytes = R * kKpK * sizeof(T);
  const uint32_t stage_bytes = a_bytes + b_bytes;
  unsigned char* stages = base;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kKpStages * stage_bytes);
  uint64_t* empty = full + kKpStages;
  uint64_t* acc_full = empty + kKpStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = d / kKpK;
  const uint32_t tmem_cols = (2 * R <= 32) ? 32 : (2 * R <= 64 ? 64 : (2 * R <= 128 ? 128 : (2 * R <= 256 ? 256 : 512)));

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKpStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 4);  // MMA commit + 4 epilogue warps (sum of squares)
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer -------------------------------------------
    if (lane == 0) {
      long long it = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
        const int s = static_cast<int>(tile / a.tiles_per_src);
        const int t0 = static_cast<int>((tile % a.tiles_per_src) * kKpRows);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = static_cast<int>(it % kKpStages);
          const uint32_t par = static_cast<uint32_t>((it / kKpStages) & 1);
          if (*abort_flag || !mbar_wait_bounded(&empty[st], par ^ 1u)) {
            atomicOr(&g_kp_status, kStatusEmptyWaitTimeout);
            *abort_flag = 1;
            ok = false;
            break;
          }
          unsigned char* sa = stages + st * stage_bytes;
          mbar_arrive_expect_tx(&full[st], stage_bytes);
          tma_load_2d(sa, &a.vmap[s], kc * kKpK, t0, &full[st]);
          tma_load_2d(sa + a_bytes, &a.wmap, kc * kKpK, 0, &full[st]);
        }
      }
      if (!ok) {
        for (long long j = (it > kKpStages ? it - kKpStages : 0); j < it; ++j)
          if (!mbar_wait_bounded(&full[j % kKpStages], static_cast<uint32_t>((j / kKpStages) & 1)))
            atomicOr(&g_kp_status, kStatusDrainTimeout);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer -----------------------------------------------
    if (lane == 0) {
      long long it = 0, tcount = 0;
      bool issued_any = false;
      for (long long tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++tcount) {
        const int ab = static_cast<int>(tcount & 1);
        if (*abort_flag || !mbar_wait_bounded(&acc_empty[ab], static_cast<uint32_t>(((tcount >> 1) & 1) ^ 1))) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + ab * R;
        bool ok = true;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = static_cast<int>(it % kKpStages);
          if (*abort_flag || !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / kKpStages) & 1))) {
            atomicOr(&g_kp_status, kStatusFullWaitTimeout);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const unsigned char* sa = stages + st * stage_bytes;
          const uint64_t da = umma_desc_sw128(sa), db = umma_desc_sw128(sa + a_bytes);
#pragma unroll
          for (int k = 0; k < kKpK / 16; ++k)  // K = 16 per instruction: +32 bytes in the swizzle atom
            umma_f16(dcol, da + 2 * k, db + 2 * k, a.idesc, (kc > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
          issued_any = true;
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
      }
      // all MMAs of this CTA retired before the accumulators are freed
      umma_commit(done);
      if (issued_any && !mbar_wait_bounded(done, 0)) atomicOr(&g_kp_status, kStatusDrainTimeout);
    }
  } else {
    // ---------------- epilogue: 4 warps, one accumulator row per thread --------
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;   // row of the 128-row tile
    long long it = 0, tcount = 0;
    T* keys = static_cast<T*>(a.keys);
    for (long long tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++tcount) {
      const int s = static_cast<int>(tile / a.tiles_per_src);
      const long long t = (tile % a.tiles_per_src) * kKpRows + row;
      float ss = 0.f;
      bool ok = true;
      for (int kc = 0; kc < nk; ++kc, ++it) {
        const int st = static_cast<int>(it % kKpStages);
        if (*abort_flag || !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / kKpStages) & 1))) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (a.value_norm) {
          const unsigned char* rowp = stages + st * stage_bytes + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const Pack<T, 8> p = *reinterpret_cast<const Pack<T, 8>*>(rowp + ((c ^ (row & 7)) * 16));
            const uint32_t* pw = reinterpret_cast<const uint32_t*>(p.e);
#pragma unroll
            for (int e = 0; e < 4; ++e) Mixed16<T>::sq_step(ss, pw[e]);  // widened inside the FMA
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      if (!ok) break;
      const int ab = static_cast<int>(tcount & 1);
      if (*abort_flag || !mbar_wait_bounded(&acc_full[ab], static_cast<uint32_t>((tcount >> 1) & 1))) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const float inv = a.value_norm ? rsqrtf(ss / d + a.eps) : 1.f;
      T* kp = keys + (static_cast<long long>(s) * a.N + t) * R;
      for (int c0 = 0; c0 < R; c0 += 16) {
        float v[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ab * R + c0, v);
        if (t < a.N) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = v[h * 8 + e] * inv;
            store_pack<T, 8>(kp + c0 + h * 8, o);
          }
        }
      }
      if (a.keys_normed != nullptr) {
        // F.rms_norm per head of the rounded projection (model.py:33-36): the
        // sum of squares of the head's dtype-rounded values, then each rounded
        // value times the inverse rms, rounded once more
        const int dk = a.nrm_cols / a.H;
        T* np = static_cast<T*>(a.keys_normed) + t * a.nrm_cols;
        for (int h = 0; h < a.H; ++h) {
          float hs = 0.f;
          for (int c0 = h * dk; c0 < (h + 1) * dk; c0 += 16) {
            float v[16];
            tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ab * R + c0, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float r = Elem<T>::to_f(Elem<T>::from_f(v[e]));
              hs = fmaf(r, r, hs);
            }
          }
          const float hinv = rsqrtf(hs / dk + a.eps);
          for (int c0 = h * dk; c0 < (h + 1) * dk; c0 += 16) {
            float v[16];
            tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ab * R + c0, v);
            if (t < a.N) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                float o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = Elem<T>::to_f(Elem<T>::from_f(v[hh * 8 + e])) * hinv;
                store_pack<T, 8>(np + c0 + hh * 8, o);
              }
            }
          }
          if (a.inv_rms && t < a.N) a.inv_rms[t * a.H + h] = hinv;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if (a.inv_rms && a.keys_normed == nullptr && t < a.N) a.inv_rms[static_cast<long long>(s) * a.N + t] = inv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// Generic (any dtype / width) projection on CUDA cores: one warp per row.
struct KeyProjSimtArgs {
  const void* v[ATTNRES_MAX_SOURCES];
  long long vs[ATTNRES_MAX_SOURCES];
  const void* w;
  long long w_stride;
  void* keys;
  float* inv_rms;
  long long N;
  int S, d, R, value_norm;
  float eps;
};

template <typename T>
__global__ void __launch_bounds__(256) keyproj_simt_kernel(const __grid_constant__ KeyProjSimtArgs a) {
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(a.S) * a.N) return;
  const int s = static_cast<int>(row / a.N);
  const long long t = row % a.N;
  const T* v = static_cast<const T*>(a.v[s]) + t * a.vs[s];
  const T* w = static_cast<const T*>(a.w);
  float ss = 0.f;
  for (int j = lane; j < a.d; j += 32) {
    const float x = Elem<T>::to_f(v[j]);
    ss = fmaf(x, x, ss);
  }
  ss = warp_sum(ss);
  const float inv = a.value_norm ? rsqrtf(ss / a.d + a.eps) : 1.f;
  T* out = static_cast<T*>(a.keys) + row * a.R;
  for (int r = 0; r < a.R; ++r) {
    float acc = 0.f;
    for (int j = lane; j < a.d; j += 32) acc = fmaf(Elem<T>::to_f(v[j]), Elem<T>::to_f(w[r * a.w_stride + j]), acc);
    acc = warp_sum(acc);
    if (lane == 0) out[r] = Elem<T>::from_f(acc * inv);
  }
  if (lane == 0 && a.inv_rms) a.inv_rms[row] = inv;
}

// Backward of the value rms-norm of the projection, combined into grad_values:
//   dV[s][t] = base + inv * (dn - (V * inv) * <dK, key> / d),   dn = dK @ W (given)
// (<dn, V*inv> = <dK, key> because key = (V*inv) @ W^T). base is either the
// read backward's alpha * g (alpha [N,H,S] saved by the forward, g the upstream
// gradient: the read then skips its own dV writes) or the current grad_values
// (read-modify-write). One warp per (source, token) row, VEC-wide packs.
struct KeyProjBwdArgs {
  const void* v[ATTNRES_MAX_SOURCES];
  long long vs[ATTNRES_MAX_SOURCES];
  void* gv[ATTNRES_MAX_SOURCES];  // [N, d] dense
  const void* dn;                 // [S][N][d] dense
  const void* dk;                 // [S][N][R]
  const void* keys;               // [S][N][R]
  const float* inv_rms;           // [S][N]
  const void* g;                  // [N, d] upstream gradient, or null (read-modify-write)
  const float* alpha;             // [N, H, S] softmax weights, with g
  long long N;
  int S, d, R, H, value_norm;
};

template <typename T, int VEC>
__global__ void __launch_bounds__(256) keyproj_bwd_combine_kernel(const __grid_constant__ KeyProjBwdArgs a) {
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(a.S) * a.N) return;
  const int s = static_cast<int>(row / a.N);
  const long long t = row % a.N;
  const T* dk = static_cast<const T*>(a.dk) + row * a.R;
  const T* kk = static_cast<const T*>(a.keys) + row * a.R;
  float c = 0.f;
  for (int r = lane; r < a.R; r += 32) c = fmaf(Elem<T>::to_f(dk[r]), Elem<T>::to_f(kk[r]), c);
  c = a.value_norm ? warp_sum(c) / a.d : 0.f;
  const float inv = a.value_norm ? a.inv_rms[row] : 1.f;
  const T* v = static_cast<const T*>(a.v[s]) + t * a.vs[s];
  const T* dn = static_cast<const T*>(a.dn) + row * a.d;
  const T* g = a.g ? static_cast<const T*>(a.g) + t * a.d : nullptr;
  T* gv = static_cast<T*>(a.gv[s]) + t * a.d;
  const int dv = a.d / a.H;
  for (int j = lane * VEC; j < a.d; j += 32 * VEC) {
    const Pack<T, VEC> vp = load_stream<T, VEC>(v + j);
    const Pack<T, VEC> np = load_stream<T, VEC>(dn + j);
    Pack<T, VEC> bp;
    float al = 0.f;
    if (g) {
      bp = load_pack<T, VEC>(g + j);
      al = a.alpha[(t * a.H + j / dv) * a.S + s];
    } else {
      bp = load_pack<T, VEC>(gv + j);
    }
    float o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float base = g ? al * Elem<T>::to_f(bp.e[e]) : Elem<T>::to_f(bp.e[e]);
      const float y = Elem<T>::to_f(vp.e[e]) * inv;
      o[e] = base + inv * (Elem<T>::to_f(np.e[e]) - y * c);
    }
    store_pack<T, VEC>(gv + j, o);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool tc_eligible(int S, long long N, int d, int R, int dtype, const void* const* values, const int64_t* vstr,
                        const void* w, long long w_stride) {
  if (dtype == ATTNRES_DTYPE_F32 || S > kKpMaxSources || N < 1) return false;
  if (d % kKpK || R % 16 || R < 16 || R > 256) return false;
  if (N > 0x7fffffffLL) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  for (int s = 0; s < S; ++s)
    if (!al16(values[s]) || (vstr[s] * 2) % 16) return false;
  return al16(w) && (w_stride * 2) % 16 == 0 && encode_fn() != nullptr;
}

// Fills the shape fields and the instruction descriptor of `a` (sources,
// tensor maps, outputs and norm fields set by the caller) and launches the
// tensor-core kernel: one CTA per 128-row tile, up to two CTAs per SM.
static cudaError_t launch_tc(KeyProjArgs& a, long long N, int d, int R, int dtype, int nsm, cudaStream_t st) {
  a.N = N;
  a.R = R;
  a.d = d;
  a.tiles_per_src = static_cast<int>((N + kKpRows - 1) / kKpRows);
  a.ntiles = static_cast<long long>(a.tiles_per_src) * a.S;
  // kind::f16 instruction descriptor: D f32, A/B bf16 (1) or f16 (0), both K-major, N>>3, M>>4
  const uint32_t ab = dtype == ATTNRES_DTYPE_BF16 ? 1u : 0u;
  a.idesc = (1u << 4) | (ab << 7) | (ab << 10) | (static_cast<uint32_t>(R >> 3) << 17) |
            (static_cast<uint32_t>(kKpRows >> 4) << 24);
  const size_t smem = 1024 + kKpStages * (kKpRows + R) * kKpK * 2 + 256;
  auto fn = dtype == ATTNRES_DTYPE_BF16 ? keyproj_tc_kernel<__nv_bfloat16> : keyproj_tc_kernel<__half>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cached_occupancy(&per_sm, reinterpret_cast<const void*>(fn), 192, smem);
  if (e != cudaSuccess) return e;
  per_sm = std::max(1, std::min(per_sm, 2));
  const long long grid = std::min<long long>(a.ntiles, static_cast<long long>(nsm) * per_sm);
  fn<<<static_cast<int>(grid), 192, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t fused_key_projection_launch(long long N, int din, int rank, int query_rank, int H, int dtype,
                                        const void* x, long long x_stride, const void* w, long long w_stride,
                                        int key_norm, float eps, void* kq, void* key, float* key_inv,
                                        cudaStream_t st, bool* eligible) {
  // x [N, din] (row stride x_stride), w the key/query rows [rank + query_rank, din];
  // kq [N][rank + query_rank] (pre-norm, dtype-rounded), key [N][rank], key_inv [N][H]
  const int R = rank + query_rank;
  *eligible = false;
  if (H < 1 || rank % H) return cudaSuccess;
  if (key_norm && ((rank / H) % 16 || key == nullptr || key_inv == nullptr)) return cudaSuccess;
  const int64_t xs = x_stride;
  if (N < 1 || !tc_eligible(1, N, din, R, dtype, &x, &xs, w, w_stride)) return cudaSuccess;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(kq) || (key_norm && !al16(key))) return cudaSuccess;
  KeyProjArgs a{};
  if (!encode_2d(&a.vmap[0], dtype, x, N, din, x_stride, kKpRows) || !encode_2d(&a.wmap, dtype, w, R, din, w_stride, R))
    return cudaSuccess;
  int nsm = 0;
  cudaError_t e = cached_sm_count(&nsm);
  if (e != cudaSuccess) return e;
  a.keys = kq;
  a.S = 1;
  a.value_norm = 0;
  a.eps = eps;
  a.H = H;
  a.nrm_cols = rank;
  a.keys_normed = key_norm ? key : nullptr;
  a.inv_rms = key_norm ? key_inv : nullptr;
  *eligible = true;
  return launch_tc(a, N, din, R, dtype, nsm, st);
}

cudaError_t keyproj_launch(int S, long long N, int d, int R, int dtype, const void* const* values,
                           const int64_t* vstr, const void* w, long long w_stride, int value_norm, float eps,
                           void* keys, float* inv_rms, bool allow_tc, cudaStream_t st, bool* used_tc) {
  // keys / inv_rms are dense [S][N][R] / [S][N]
  *used_tc = false;
  if (N == 0) return cudaSuccess;
  int nsm = 0;
  cudaError_t e = cached_sm_count(&nsm);
  if (e != cudaSuccess) return e;
  if (allow_tc && tc_eligible(S, N, d, R, dtype, values, vstr, w, w_stride)) {
    KeyProjArgs a{};
    bool ok = true;
    for (int s = 0; s < S && ok; ++s) ok = encode_2d(&a.vmap[s], dtype, values[s], N, d, vstr[s], kKpRows);
    ok = ok && encode_2d(&a.wmap, dtype, w, R, d, w_stride, R);
    if (ok) {
      a.keys = keys;
      a.inv_rms = inv_rms;
      a.S = S;
      a.value_norm = value_norm;
      a.eps = eps;
      *used_tc = true;
      return launch_tc(a, N, d, R, dtype, nsm, st);
    }
  }
  KeyProjSimtArgs g{};
  for (int s = 0; s < S; ++s) {
    g.v[s] = values[s];
    g.vs[s] = vstr[s];
  }
  g.w = w;
  g.w_stride = w_stride;
  g.keys = keys;
  g.inv_rms = inv_rms;
  g.N = N;
  g.S = S;
  g.d = d;
  g.R = R;
  g.value_norm = value_norm;
  g.eps = eps;
  const long long rows = static_cast<long long>(S) * N;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  switch (dtype) {
    case ATTNRES_DTYPE_F32: keyproj_simt_kernel<float><<<grid, 256, 0, st>>>(g); break;
    case ATTNRES_DTYPE_F16: keyproj_simt_kernel<__half><<<grid, 256, 0, st>>>(g); break;
    default: keyproj_simt_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(g);
  }
  return cudaGetLastError();
}

cudaError_t keyproj_bwd_combine_launch(int S, long long N, int d, int R, int H, int dtype,
                                       const void* const* values, const int64_t* vstr,
                                       void* const* grad_values, const void* dn, const void* dk,
                                       const void* keys, const float* inv_rms, const void* g,
                                       const float* alpha, int value_norm, cudaStream_t st) {
  const long long rows = static_cast<long long>(S) * N;
  if (rows == 0) return cudaSuccess;
  KeyProjBwdArgs a{};
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const int full = 16 / esz;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  bool vec = (d % full) == 0 && (d / H) % full == 0 && al16(dn) && (!g || al16(g));
  for (int s = 0; s < S; ++s) {
    a.v[s] = values[s];
    a.vs[s] = vstr[s];
    a.gv[s] = grad_values[s];
    vec = vec && al16(values[s]) && (vstr[s] * esz) % 16 == 0 && al16(grad_values[s]);
  }
  a.dn = dn;
  a.dk = dk;
  a.keys = keys;
  a.inv_rms = inv_rms;
  a.g = g;
  a.alpha = alpha;
  a.N = N;
  a.S = S;
  a.d = d;
  a.R = R;
  a.H = H;
  a.value_norm = value_norm;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  switch (dtype) {
    case ATTNRES_DTYPE_F32:
      if (vec) keyproj_bwd_combine_kernel<float, 4><<<grid, 256, 0, st>>>(a);
      else keyproj_bwd_combine_kernel<float, 1><<<grid, 256, 0, st>>>(a);
      break;
    case ATTNRES_DTYPE_F16:
      if (vec) keyproj_bwd_combine_kernel<__half, 8><<<grid, 256, 0, st>>>(a);
      else keyproj_bwd_combine_kernel<__half, 1><<<grid, 256, 0, st>>>(a);
      break;
    default:
      if (vec) keyproj_bwd_combine_kernel<__nv_bfloat16, 8><<<grid, 256, 0, st>>>(a);
      else keyproj_bwd_combine_kernel<__nv_bfloat16, 1><<<grid, 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t read_keyproj_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_kp_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_kp_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
