// Fused backward of the key-from-value projection (lrid_key_from_value) on the
// 5th-generation tensor cores. With keys k_s = inv_s * (V_s @ W^T) (the
// reference's LRIDFusedProjection.project_key_from_value, model.py:344-356)
// and dK_s the read backward's key gradient, write dKs = inv * dK. Then
//   dV_s = alpha_s * g + dKs_s @ W - V_s * coef_s,   coef = inv * <dKs, k> / d
//   dW   = sum_s dKs_s^T @ V_s
// (<dn, V*inv> = <dK, k> because k = (V*inv) @ W^T; without the value norm
// inv = 1 and coef = 0). alpha * g is the read's own value gradient, so the
// read backward runs without writing dV and each dV row is written once.
//
// Kernels:
//   * kpb_prepass_kernel: dKs (dtype [S][N][64]) and {alpha, coef} (f32 pairs
//     [S][H][N]);
//   * kpb_transpose_w_kernel: Wt = W^T (dtype [d][64]);
//   * keyproj_bwd_tc_kernel, persistent, one 128-column slice of d per CTA.
//     The CTA walks its token tiles (128 tokens) and, inside each, the S
//     sources; the slice of g is loaded once per token tile and the slice of W
//     (Wt, 16 KB) once per CTA:
//       - warp 0 (one thread): TMA loads (128-byte swizzle, no multicast) of
//         the dKs tile [128 x 64] and the V_s slice [128 x 128] into a
//         three-stage ring, and of the g slice into a double buffer;
//       - warp 1 (one thread): tcgen05.mma kind::f16 M=128:
//           dn[128 tok x 128 col]  = dKs (K-major) x Wt (K-major), N=128, into
//             one of two TMEM accumulators;
//           dWt[128 col x 64]     += V^T (MN-major) x dKs (MN-major), N=64, a
//             TMEM accumulator that lives across all of the CTA's tiles;
//       - warps 3-10 (one token row x 64 columns per thread, two warps per
//         TMEM lane quarter): dV = alpha g + dn - V coef from TMEM and the
//         staged tiles, written over the V tile once the dWt MMA has read it;
//       - warp 2: TMA store of each finished dV tile, one tile behind the
//         epilogue, then frees the stage.
//     At the end each CTA writes its dWt slice to a partial buffer;
//   * kpb_reduce_dw_kernel sums the partials of each slice in a fixed order
//     (deterministic) into dW (f32 [64][d]).
// Every mbarrier wait is bounded (~2 s, a status bit on timeout); TMEM is
// always released.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "tma.cuh"
#include "umma.cuh"
#include "launch_cache.h"

namespace attnres {

constexpr int kKpbMaxSources = 24;
constexpr int kKpbRows = 128;   // tokens per tile (UMMA M of dn)
constexpr int kKpbCols = 128;   // columns of d per CTA slice (UMMA N of dn, M of dWt)
constexpr int kKpbR = 64;       // key rank
constexpr int kKpbStages = 3;
constexpr uint32_t kKpbKBytes = kKpbRows * kKpbR * 2;          // dKs tile, 16 KB
constexpr uint32_t kKpbAtom = kKpbRows * kTmaBoxCols * 2;       // one 64-column box, 16 KB
constexpr uint32_t kKpbStageBytes = kKpbKBytes + 2 * kKpbAtom;  // dKs | V (2 boxes; dV after the epilogue)
constexpr uint32_t kKpbGBytes = 2 * kKpbAtom;                   // g slice of a token tile
constexpr uint32_t kKpbTmemCols = 512;                          // dn x2 (256) + dWt (64), power of two
constexpr int kKpbEpiWarps = 8;                                // two per TMEM lane quarter
constexpr int kKpbThreads = (3 + kKpbEpiWarps) * 32;            // producer, MMA, store, epilogue
constexpr size_t kKpbSmem = 1024 + kKpbKBytes + 2 * kKpbGBytes + kKpbStages * kKpbStageBytes + 256;

static __device__ unsigned int g_kpb_status = 0;

struct KpbArgs {
  CUtensorMap vmap[kKpbMaxSources];   // V_s as [N rows, d cols]
  CUtensorMap gvmap[kKpbMaxSources];  // dV_s as [N, d] (TMA stores)
  CUtensorMap gmap;                   // g as [N, d]
  CUtensorMap kmap;                   // dKs as [S][N][64]
  CUtensorMap wtmap;                  // Wt as [d, 64]
  const float2* ac;                   // [S][H][N]: {alpha, coef}
  float* partials;                    // [grid][128][64]
  long long N;
  int S, d, H, nch, ntt;
  uint32_t idesc_dn, idesc_dw;
};

template <typename T>
__global__ void __launch_bounds__(kKpbThreads, 1) keyproj_bwd_tc_kernel(const __grid_constant__ KpbArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* wt_tile = base;                  // [128 cols][64] K-major, 16 KB
  unsigned char* gbuf = base + kKpbKBytes;        // 2 x g slice
  unsigned char* stages = gbuf + 2 * kKpbGBytes;  // kKpbStages x (dKs | V)
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kKpbStages * kKpbStageBytes);
  uint64_t* empty = full + kKpbStages;   // stage free: its dV tile has been read by the store
  uint64_t* vfree = empty + kKpbStages;  // the dWt MMA has finished reading the stage's V
  uint64_t* acc_full = vfree + kKpbStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* gfull = acc_empty + 2;
  uint64_t* gempty = gfull + 2;
  uint64_t* wt_full = gempty + 2;
  uint64_t* done = wt_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ch = blockIdx.x % a.nch;   // column slice of this CTA
  const int grp = blockIdx.x / a.nch;  // token tiles grp, grp + G, ...
  const int G = gridDim.x / a.nch;
  const int S = a.S;
  const int c_base = ch * kKpbCols;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKpbStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&vfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kKpbEpiWarps);
      mbar_init(&gfull[i], 1);
      mbar_init(&gempty[i], kKpbEpiWarps);
    }
    mbar_init(wt_full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kKpbTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool has_tiles = grp < a.ntt;

  if (warp == 0) {
    // ---------------- TMA producer -------------------------------------------
    if (lane == 0 && has_tiles) {
      mbar_arrive_expect_tx(wt_full, kKpbKBytes);
      tma_load_2d(wt_tile, &a.wtmap, 0, c_base, wt_full);
      long long it = 0;
      int k = 0;  // token tiles of this CTA so far
      bool ok = true;
      for (int tt = grp; tt < a.ntt && ok; tt += G, ++k) {
        const int t0 = tt * kKpbRows;
        const int gb = k & 1;
        if (*abort_flag || !mbar_wait_bounded(&gempty[gb], static_cast<uint32_t>(((k >> 1) & 1) ^ 1))) {
          atomicOr(&g_kpb_status, kStatusEmptyWaitTimeout);
          *abort_flag = 1;
          break;
        }
        unsigned char* gp = gbuf + gb * kKpbGBytes;
        mbar_arrive_expect_tx(&gfull[gb], kKpbGBytes);
        tma_load_2d(gp, &a.gmap, c_base, t0, &gfull[gb]);
        tma_load_2d(gp + kKpbAtom, &a.gmap, c_base + kTmaBoxCols, t0, &gfull[gb]);
        for (int s = 0; s < S; ++s, ++it) {
          const int st = static_cast<int>(it % kKpbStages);
          const uint32_t par = static_cast<uint32_t>((it / kKpbStages) & 1);
          if (*abort_flag || !mbar_wait_bounded(&empty[st], par ^ 1u)) {
            atomicOr(&g_kpb_status, kStatusEmptyWaitTimeout);
            *abort_flag = 1;
            ok = false;
            break;
          }
          unsigned char* sp = stages + st * kKpbStageBytes;
          mbar_arrive_expect_tx(&full[st], kKpbStageBytes);
          tma_load_3d(sp, &a.kmap, 0, t0, s, &full[st]);
          tma_load_2d(sp + kKpbKBytes, &a.vmap[s], c_base, t0, &full[st]);
          tma_load_2d(sp + kKpbKBytes + kKpbAtom, &a.vmap[s], c_base + kTmaBoxCols, t0, &full[st]);
        }
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA can exit
        for (long long j = (it > kKpbStages ? it - kKpbStages : 0); j < it; ++j)
          if (!mbar_wait_bounded(&full[j % kKpbStages], static_cast<uint32_t>((j / kKpbStages) & 1)))
            atomicOr(&g_kpb_status, kStatusDrainTimeout);
        for (int j = (k > 2 ? k - 2 : 0); j < k; ++j)
          if (!mbar_wait_bounded(&gfull[j & 1], static_cast<uint32_t>((j >> 1) & 1)))
            atomicOr(&g_kpb_status, kStatusDrainTimeout);
      }
      if (!mbar_wait_bounded(wt_full, 0)) atomicOr(&g_kpb_status, kStatusDrainTimeout);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer -----------------------------------------------
    if (lane == 0 && has_tiles) {
      bool issued_any = false;
      if (!mbar_wait_bounded(wt_full, 0)) {
        atomicOr(&g_kpb_status, kStatusFullWaitTimeout);
        *abort_flag = 1;
      } else {
        tc_fence_after();
        const uint64_t dwt = umma_desc_sw128(wt_tile);
        const uint32_t d_dw = tmem_base + 2 * kKpbCols;
        long long it = 0;
        for (int tt = grp; tt < a.ntt && !*abort_flag; tt += G) {
          for (int s = 0; s < S; ++s, ++it) {
            const int st = static_cast<int>(it % kKpbStages);
            const int ab = static_cast<int>(it & 1);
            if (*abort_flag ||
                !mbar_wait_bounded(&acc_empty[ab], static_cast<uint32_t>(((it >> 1) & 1) ^ 1)) ||
                !mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / kKpbStages) & 1))) {
              atomicOr(&g_kpb_status, kStatusFullWaitTimeout);
              *abort_flag = 1;
              break;
            }
            tc_fence_after();
            const unsigned char* sp = stages + st * kKpbStageBytes;
            // dn = dKs x Wt^T: K = 64 in four K=16 steps (+32 bytes inside the swizzle atom)
            const uint64_t dk = umma_desc_sw128(sp);
#pragma unroll
            for (int k = 0; k < kKpbR / 16; ++k)
              umma_f16(tmem_base + ab * kKpbCols, dk + 2 * k, dwt + 2 * k, a.idesc_dn, k > 0 ? 1u : 0u);
            umma_commit(&acc_full[ab]);
            // dWt += V^T x dKs over the tile's 128 tokens: K = 16 tokens per step,
            // two 1024-byte row groups (+2048 bytes) per step
            const uint64_t dv = umma_desc_sw128_mn(sp + kKpbKBytes, kKpbAtom);
            const uint64_t dkm = umma_desc_sw128_mn(sp, kKpbAtom);
#pragma unroll
            for (int k = 0; k < kKpbRows / 16; ++k)
              umma_f16(d_dw, dv + 128 * k, dkm + 128 * k, a.idesc_dw, (it > 0 || k > 0) ? 1u : 0u);
            umma_commit(&vfree[st]);
            issued_any = true;
          }
        }
      }
      umma_commit(done);
      if (issued_any && !mbar_wait_bounded(done, 0)) atomicOr(&g_kpb_status, kStatusDrainTimeout);
    }
  } else if (warp == 2) {
    // ---------------- dV tile stores (one tile behind the epilogue) -------------
    // Meets the epilogue warps at named barrier 2 once per tile (the OR of
    // their stop predicates makes every participant leave on the same tile),
    // then stores the tile, waits until the TMA has read it and frees the stage.
    long long it = 0;
    bool stopped = !has_tiles;
    for (int tt = grp; tt < a.ntt && !stopped; tt += G) {
      const int t0 = tt * kKpbRows;
      for (int s = 0; s < S; ++s, ++it) {
        stopped = consumer_sync_or(kKpbEpiWarps * 32 + 32, *abort_flag != 0);
        if (stopped) break;
        if (lane == 0) {
          const int st = static_cast<int>(it % kKpbStages);
          const unsigned char* tile = stages + st * kKpbStageBytes + kKpbKBytes;
          tma_store_2d(&a.gvmap[s], c_base, t0, tile);
          tma_store_2d(&a.gvmap[s], c_base + kTmaBoxCols, t0, tile + kKpbAtom);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(&empty[st]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) bulk_wait_group0();
  } else {
    // ---------------- epilogue: 8 warps, one token row x 64 columns per thread ---
    // dV overwrites the V half-row it was computed from (the dWt MMA has read it
    // by then: vfree), so the stage's V boxes become the dV tile of the store.
    // A failed (timed-out) wait never skips named barrier 2: every epilogue warp
    // reaches it each tile.
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int half = (warp - 3) >> 2;     // 64-column half (= V box) of the slice
    const int row = q * 32 + lane;        // token row of the tile / column row of dWt
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int dvh = a.d / a.H;
    const int h = c_base / dvh;
    long long it = 0;
    int k = 0;
    bool stopped = !has_tiles;
    for (int tt = grp; tt < a.ntt && !stopped; tt += G, ++k) {
      const int t0 = tt * kKpbRows;
      const long long t = static_cast<long long>(t0) + row;
      const bool live = t < a.N;
      const int gb = k & 1;
      bool good = !*abort_flag && mbar_wait_bounded(&gfull[gb], static_cast<uint32_t>((k >> 1) & 1));
      if (!good) *abort_flag = 1;
      const unsigned char* grow = gbuf + gb * kKpbGBytes + half * kKpbAtom + row * 128;
      const float2* acp = a.ac + static_cast<long long>(h) * a.N + (live ? t : 0);
      const long long acs = static_cast<long long>(a.H) * a.N;  // next source
      float2 acn = *acp;                                          // {alpha, coef} of source 0
      for (int s = 0; s < S; ++s, ++it) {
        const int st = static_cast<int>(it % kKpbStages);
        const int ab = static_cast<int>(it & 1);
        const float al = live ? acn.x : 0.f;
        const float cf = live ? acn.y : 0.f;
        if (s + 1 < S) acn = acp[(s + 1) * acs];  // one tile ahead
        const uint32_t sph = static_cast<uint32_t>((it / kKpbStages) & 1);
        good = good && !*abort_flag && mbar_wait_bounded(&full[st], sph) &&
               mbar_wait_bounded(&acc_full[ab], static_cast<uint32_t>((it >> 1) & 1)) &&
               mbar_wait_bounded(&vfree[st], sph);
        if (!good) *abort_flag = 1;
        if (good) {
          tc_fence_after();
          unsigned char* vrow = stages + st * kKpbStageBytes + kKpbKBytes + half * kKpbAtom + row * 128;
          const uint32_t tcol = tmem_base + lane_off + ab * kKpbCols + half * kTmaBoxCols;
          // the thread's 64 dn columns: four TMEM loads, one wait
          uint32_t dr[4][16];
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_ld16_nowait(tcol + 16 * j, dr[j]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_regs_ready(dr[j]);
#pragma unroll
          for (int hh = 0; hh < 8; ++hh) {
            const int off = (hh ^ (row & 7)) << 4;
            const Pack<T, 8> vp = *reinterpret_cast<const Pack<T, 8>*>(vrow + off);
            const Pack<T, 8> gp = *reinterpret_cast<const Pack<T, 8>*>(grow + off);
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              o[e] = fmaf(al, Elem<T>::to_f(gp.e[e]),
                          __uint_as_float(dr[hh >> 1][(hh & 1) * 8 + e]) - Elem<T>::to_f(vp.e[e]) * cf);
            store_pack<T, 8>(reinterpret_cast<T*>(vrow + off), o);
          }
          tc_fence_before();
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&acc_empty[ab]);
            if (s == S - 1) mbar_arrive(&gempty[gb]);
          }
        }
        // the whole dV tile is in shared memory: hand it to the store warp
        stopped = consumer_sync_or(kKpbEpiWarps * 32 + 32, !good || *abort_flag != 0);
        if (stopped) break;
      }
    }
    const bool ok = has_tiles && !stopped;
    // this CTA's slice of dWt: lane = column of the slice, this warp's 32 of
    // the 64 fp32 columns (= r)
    float* part = a.partials + (static_cast<long long>(blockIdx.x) * kKpbCols + row) * kKpbR + half * 32;
    if (ok && mbar_wait_bounded(done, 0)) {
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < 32; c0 += 16) {
        float v[16];
        tmem_ld16(tmem_base + lane_off + 2 * kKpbCols + half * 32 + c0, v);
#pragma unroll
        for (int e = 0; e < 16; e += 4)
          *reinterpret_cast<float4*>(part + c0 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      }
    } else {
      if (has_tiles) atomicOr(&g_kpb_status, kStatusFullWaitTimeout);
      for (int c0 = 0; c0 < 32; c0 += 4) *reinterpret_cast<float4*>(part + c0) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kKpbTmemCols);
  }
}

// dKs = inv * dK (rounded to T) and coef = inv * <inv * dK, k> / d, with
// eight lanes per (source, token) row of 64 (one 16-byte pack each); the
// softmax weight is copied next to coef in source-major order, so the fused
// kernel's epilogue reads one coalesced {alpha, coef} pair per row and tile.
struct KpbPrepArgs {
  const void* dk[kKpbMaxSources];  // [N, 64] dense per source
  const void* keys;                // [S][N][64]
  const float* inv_rms;            // [S][N], or null without the value norm
  const float* alpha;              // [N][H][S] softmax weights of the forward
  void* dks;                       // [S][N][64]
  float2* ac;                      // [S][H][N]: {alpha, coef}
  long long N;
  int S, d, H;
};

template <typename T>
__global__ void __launch_bounds__(256) kpb_prepass_kernel(const __grid_constant__ KpbPrepArgs a) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int sub = threadIdx.x & 7;
  const long long rows = static_cast<long long>(a.S) * a.N;
  const bool live = row < rows;
  const long long r = live ? row : 0;
  const int s = static_cast<int>(r / a.N);
  const long long t = r - static_cast<long long>(s) * a.N;
  const float inv = a.inv_rms ? a.inv_rms[r] : 1.f;
  const Pack<T, 8> gp = *reinterpret_cast<const Pack<T, 8>*>(static_cast<const T*>(a.dk[s]) + t * kKpbR + sub * 8);
  const Pack<T, 8> kp = *reinterpret_cast<const Pack<T, 8>*>(static_cast<const T*>(a.keys) + r * kKpbR + sub * 8);
  float o[8], c = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o[e] = inv * Elem<T>::to_f(gp.e[e]);
    c = fmaf(o[e], Elem<T>::to_f(kp.e[e]), c);
  }
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  if (!live) return;
  store_pack<T, 8>(static_cast<T*>(a.dks) + r * kKpbR + sub * 8, o);
  const float cf = a.inv_rms ? inv * c / a.d : 0.f;
  for (int h = sub; h < a.H; h += 8)
    a.ac[(static_cast<long long>(s) * a.H + h) * a.N + t] = make_float2(a.alpha[(t * a.H + h) * a.S + s], cf);
}

// Wt[c][r] = W[r][c]; W is [64, d] with a row stride.
template <typename T>
__global__ void __launch_bounds__(256) kpb_transpose_w_kernel(const T* __restrict__ w, long long wstride, int d,
                                                              T* __restrict__ wt) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(d) * kKpbR) return;
  const int c = static_cast<int>(i / kKpbR), r = static_cast<int>(i % kKpbR);
  wt[i] = w[r * wstride + c];
}

// dW[r][slice * 128 + c] = sum over the slice's CTAs, in CTA order, of
// partials[cta][c][r].
__global__ void __launch_bounds__(256) kpb_reduce_dw_kernel(const float* __restrict__ partials, int nch, int G,
                                                            int d, float* __restrict__ dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over [64][d]
  if (i >= kKpbR * d) return;
  const int r = i / d, col = i % d;
  const int ch = col / kKpbCols, c = col % kKpbCols;
  float acc = 0.f;
  for (int g = 0; g < G; ++g) acc += partials[(static_cast<long long>(g * nch + ch) * kKpbCols + c) * kKpbR + r];
  dw[i] = acc;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static bool kpb_shape(int S, long long N, int d, int R, int H, int dtype, int* nch, int* G, int* ntt) {
  if (dtype == ATTNRES_DTYPE_F32 || R != kKpbR || S < 1 || S > kKpbMaxSources || N < 1) return false;
  if (H < 1 || d % kKpbCols || d % H || (d / H) % kKpbCols || N > 0x7fffffffLL) return false;
  if (encode_fn() == nullptr) return false;
  int nsm = 0;
  if (cached_sm_count(&nsm) != cudaSuccess) return false;
  *nch = d / kKpbCols;
  *ntt = static_cast<int>((N + kKpbRows - 1) / kKpbRows);
  *G = std::max(1, std::min(nsm / *nch, *ntt));
  return true;
}

size_t keyproj_bwd_tc_workspace(int S, long long N, int d, int R, int H, int dtype) {
  int nch, G, ntt;
  if (!kpb_shape(S, N, d, R, H, dtype, &nch, &G, &ntt)) return 0;
  return align256(static_cast<size_t>(d) * kKpbR * 2) + align256(static_cast<size_t>(S) * N * kKpbR * 2) +
         align256(static_cast<size_t>(S) * H * N * 8) + align256(static_cast<size_t>(nch) * G * kKpbCols * kKpbR * 4);
}

cudaError_t keyproj_bwd_tc_launch(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                                  const int64_t* vstr, const void* w, long long w_stride,
                                  const void* const* grad_keys, const void* keys, const float* inv_rms,
                                  const void* g, const float* alpha, int value_norm, void* const* grad_values,
                                  float* grad_weight, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  int nch, G, ntt;
  if (!kpb_shape(S, N, d, R, H, dtype, &nch, &G, &ntt)) return cudaErrorNotSupported;
  if (workspace_bytes < keyproj_bwd_tc_workspace(S, N, d, R, H, dtype)) return cudaErrorInvalidValue;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  void* wt = ws;
  ws += align256(static_cast<size_t>(d) * kKpbR * 2);
  void* dks = ws;
  ws += align256(static_cast<size_t>(S) * N * kKpbR * 2);
  float2* ac = reinterpret_cast<float2*>(ws);
  ws += align256(static_cast<size_t>(S) * H * N * 8);
  float* partials = reinterpret_cast<float*>(ws);
  const bool bf = dtype == ATTNRES_DTYPE_BF16;

  // W^T and the scaled key gradient
  {
    const long long n = static_cast<long long>(d) * kKpbR;
    const unsigned grid = static_cast<unsigned>((n + 255) / 256);
    if (bf)
      kpb_transpose_w_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), w_stride,
                                                                    d, static_cast<__nv_bfloat16*>(wt));
    else
      kpb_transpose_w_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w), w_stride, d,
                                                             static_cast<__half*>(wt));
    KpbPrepArgs p{};
    for (int s = 0; s < S; ++s) p.dk[s] = grad_keys[s];
    p.keys = keys;
    p.inv_rms = value_norm ? inv_rms : nullptr;
    p.alpha = alpha;
    p.dks = dks;
    p.ac = ac;
    p.N = N;
    p.S = S;
    p.d = d;
    p.H = H;
    const long long threads = static_cast<long long>(S) * N * 8;
    const unsigned pg = static_cast<unsigned>((threads + 255) / 256);
    if (bf) kpb_prepass_kernel<__nv_bfloat16><<<pg, 256, 0, st>>>(p);
    else kpb_prepass_kernel<__half><<<pg, 256, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }

  KpbArgs a{};
  bool ok = true;
  for (int s = 0; s < S && ok; ++s) {
    ok = encode_2d(&a.vmap[s], dtype, values[s], N, d, vstr[s], kKpbRows);
    ok = ok && encode_2d(&a.gvmap[s], dtype, grad_values[s], N, d, d, kKpbRows);
  }
  ok = ok && encode_2d(&a.gmap, dtype, g, N, d, d, kKpbRows);
  ok = ok && encode_3d(&a.kmap, dtype, dks, S, N, kKpbR, kKpbRows);
  ok = ok && encode_2d(&a.wtmap, dtype, wt, d, kKpbR, kKpbR, kKpbCols);
  if (!ok) return cudaErrorInvalidValue;
  a.ac = ac;
  a.partials = partials;
  a.N = N;
  a.S = S;
  a.d = d;
  a.H = H;
  a.nch = nch;
  a.ntt = ntt;
  const uint32_t ab = bf ? 1u : 0u;
  a.idesc_dn = umma_idesc_f16(ab, 0, 0, kKpbRows, kKpbCols);
  a.idesc_dw = umma_idesc_f16(ab, 1, 1, kKpbCols, kKpbR);
  const size_t smem = kKpbSmem;
  auto fn = bf ? keyproj_bwd_tc_kernel<__nv_bfloat16> : keyproj_bwd_tc_kernel<__half>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  fn<<<nch * G, kKpbThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int n = kKpbR * d;
  kpb_reduce_dw_kernel<<<(n + 255) / 256, 256, 0, st>>>(partials, nch, G, d, grad_weight);
  return cudaGetLastError();
}

cudaError_t read_keyproj_bwd_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_kpb_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_kpb_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
