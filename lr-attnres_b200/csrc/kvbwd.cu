// Key-from-value LRID read backward in one pass over the values: the read
// backward (attnres_ops.py:4195-4232 differentiated, with a static query) and
// the backward of the key projection keys_s = inv_s * (V_s @ W^T)
// (LRIDFusedProjection.project_key_from_value, model.py:344-356) fused, so
// that every value row crosses HBM once and every dV row is written once.
//
// Per (token t, source s, head h), with alpha the forward's softmax weights
// and out the forward's output:
//   dw_s   = <g_h, V_s,h>                      (a dot over the head's columns)
//   dl_s   = alpha_s (dw_s - <g_h, out_h>)     (softmax backward: sum_j alpha_j
//                                               dw_j = <g, sum_j alpha_j V_j>)
//   dK_s   = kinv (c1 q - khat c2),  c1 = dl scale, c2 = c1 <khat, q> / dk
//            (key RMS norm backward; dK_s = c1 q without the key norm)
//   dKs_s  = inv_s dK_s,  coef_s = inv_s <dKs_s, k_s> / d
//   dV_s   = alpha_s g + dKs_s @ W - V_s coef_s
//   dW    += dKs_s^T @ V_s,   dq += c1 khat,   dbias_s += dl_s
//
// The weight W (R = 64 rows) is too large to sit next to a whole value row in
// one SM, so each CTA owns one 128-column slice of d and the d / 128 slices
// of a token tile form one thread-block cluster (16 CTAs for d = 2048). Per
// stage every CTA forms the partial dots <g, V> of its slice for the tile's
// 128 rows and bulk-copies the 512 bytes into every other CTA's exchange slot
// (cp.async.bulk shared::cta -> shared::cluster, completing on that CTA's
// exchange mbarrier, no multicast); each CTA then sums the slices' partials
// in rank order, so all of them form identical dKs rows. Before its sources a
// token tile streams one pseudo-stage, the slice of the forward output, whose
// exchanged dots give <g, out> per head.
//
// CTA roles (20 warps; the control warpgroup hands registers to the others):
//   warp 0: TMA loads (128-byte swizzle, no multicast) of W^T's slice once and,
//     per stage, the V_s (or output) slice [128 tokens x 128 columns] into a
//     four-stage ring;
//   warp 1: per source stage, tcgen05.mma kind::f16 M=128:
//       dn[128 tok x 128 col] = dKs (K-major) x Wt (K-major), N=128, into one
//         of two TMEM accumulators;
//       dWt[128 col x 64]    += V^T (MN-major) x dKs (MN-major), N=64, a TMEM
//         accumulator that lives across the CTA's tiles;
//   warps 2-3: idle (the control warpgroup hands its registers to the rows);
//   warps 4-11 (one token row x 64 columns per thread): at step i the exchange
//     of stage i-1 and its dKs row half (written into a swizzled tile, the
//     MMA operand) and {alpha, coef}, then the partial dots of stage i (published to the
//     cluster); dKs_j = inv dl (u0 q_j - u1 k_j) and
//     coef = sum_h dl_h w_h with {u0, u1, w} per (source, token, head) from a
//     prepass over the keys, so nothing after the exchange reduces over j;
//   warps 12-19 (one token row x 64 columns per thread, TMEM lane quarter =
//     warp % 4): dV = alpha g + dn - V coef from TMEM and the staged V,
//     stored straight to global memory; a ring stage is free once these warps
//     and the MMAs have read it.
// The slice-0 CTA of each tile writes dl; a follow-up kernel sums dq and dbias
// from dl and the keys, another sums the dW partials, both in a fixed order.
// Every wait is bounded (~2 s) and reports through a status bit; TMEM is
// always released; no CTA leaves before its cluster (the exchange writes into
// the partners' shared memory).
//
// Measured at config 4 (S=17, 131 072 tokens, d=2048, bf16) on a B200: 12-16 ms
// against 5.4 ms for the read backward followed by the projection backward,
// although V crosses HBM once here. Per-role %globaltimer stamps show every
// stage held in the ring for ~15 us (load, dots, the exchange round trip of
// ~2.5 us through the cluster, dKs, MMAs, dV), so four 32 KB stages turn over
// every ~4-5 us where the CTA's share of HBM needs ~1.6 us; more stages or
// exchange slots do not fit beside them in shared memory. The path is selected
// with ATTNRES_KV_BWD=one and parity-tested; the two-kernel path is the default.
#include <cuda.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "plan.h"
#include "tma.cuh"
#include "umma.cuh"
#include "cluster.cuh"
#include "launch_cache.h"

namespace attnres {

constexpr int kKvbMaxSources = 24;
constexpr int kKvbRows = 128;     // tokens per tile
constexpr int kKvbCols = 128;     // columns of d per CTA slice
constexpr int kKvbR = 64;         // key rank
constexpr int kKvbStages = 4;     // value ring
constexpr int kKvbSlots = 4;      // exchange ring (see the slot-reuse note in the dot warps)
constexpr int kKvbMaxCluster = 16;
constexpr uint32_t kKvbAtom = kKvbRows * kTmaBoxCols * 2;  // one 64-column box, 16 KB
constexpr uint32_t kKvbStageBytes = 2 * kKvbAtom;          // V slice (dV after the epilogue)
constexpr uint32_t kKvbKBytes = kKvbRows * kKvbR * 2;      // dKs tile / Wt slice, 16 KB
constexpr uint32_t kKvbXBytes = kKvbRows * 4;              // one slice's partial dots of a stage
constexpr uint32_t kKvbTmemCols = 512;                     // dn x2 (256) + dWt (64)
constexpr int kKvbThreads = 20 * 32;
// Register split (setmaxnreg): the kernel launches with 96 registers per
// thread (640 x 96 = 61 440); the control warpgroup gives back down to 40 and
// the four row warpgroups take 104: 128 x 40 + 512 x 104 = 58 368.
constexpr int kKvbLaunchRegs = 96;
constexpr int kKvbCtlRegs = 40;
constexpr int kKvbEpiRegs = 104;
static_assert(128 * kKvbCtlRegs + 512 * kKvbEpiRegs <= kKvbThreads * kKvbLaunchRegs, "register split exceeds the launch");
constexpr size_t kKvbSmem = 1024 + 3 * kKvbKBytes + kKvbStages * kKvbStageBytes +
                            kKvbSlots * kKvbMaxCluster * kKvbXBytes + 4 * kKvbRows * 8 + 256 + 512 + 512;

static __device__ unsigned int g_kvb_status = 0;

struct KvbArgs {
  CUtensorMap vmap[kKvbMaxSources];   // V_s as [N rows, d cols]
  CUtensorMap omap;                   // forward output as [N, d]
  CUtensorMap wtmap;                  // Wt as [d, 64]
  void* dv[kKvbMaxSources];           // dV_s, [N, d] dense
  const void* g;                      // [N, d] dense
  const void* keys;                   // [S][N][64]
  const float* vinv;                  // [S][N], or null without the value norm
  const float* alpha;                 // [N][H][S]
  const float4* prep;                 // [S][N][H]: {u0, u1, w, 0} (kvb_prep_kernel)
  const void* q;                      // static query, 64 values
  float* dl;                          // [S][N][H]
  float* partials;                    // [grid][128][64] dWt
  long long N;
  int S, d, nch, ntt, key_norm;
  float scale, key_eps;
  uint32_t idesc_dn, idesc_dw;
};

// Named barrier `id` over `n` threads, OR-reducing a predicate.
__device__ __forceinline__ bool kvb_sync_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

template <typename T>
__device__ __forceinline__ void kvb_zero(Pack<T, 8>& p) {
#pragma unroll
  for (int e = 0; e < 8; ++e) p.e[e] = Elem<T>::from_f(0.f);
}

template <typename T, int H>
__global__ void __launch_bounds__(kKvbThreads, 1) kvb_fused_kernel(const __grid_constant__ KvbArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* wt_tile = base;                    // [128 cols][64] K-major
  unsigned char* dks_tiles = base + kKvbKBytes;     // 2 x [128 tok][64] K-major
  unsigned char* stages = dks_tiles + 2 * kKvbKBytes;
  float* xbuf = reinterpret_cast<float*>(stages + kKvbStages * kKvbStageBytes);  // [slot][rank][128]
  float2* acs = reinterpret_cast<float2*>(xbuf + kKvbSlots * kKvbMaxCluster * kKvbRows);  // [4][128]
  float* q_s = reinterpret_cast<float*>(acs + 4 * kKvbRows);  // 64 fp32, then 128 fp32 half-row partials
  uint64_t* full = reinterpret_cast<uint64_t*>(q_s + kKvbR + kKvbRows);
  uint64_t* empty = full + kKvbStages;
  uint64_t* acc_full = empty + kKvbStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* dks_full = acc_empty + 2;
  uint64_t* dks_free = dks_full + 2;
  uint64_t* ac_full = dks_free + 2;     // 4: {alpha, coef} of a source stage ready
  uint64_t* xbar = ac_full + 4;         // kKvbSlots: a stage's partials from every slice landed
  uint64_t* pfree = xbar + kKvbSlots;   // the dot warps are done with a tile's output pseudo-stage
  uint64_t* wt_full = pfree + 1;
  uint64_t* done = wt_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = a.nch;                                   // cluster size = column slices
  const int ch = static_cast<int>(cluster_rank());       // column slice of this CTA
  const long long grp = cluster_id_x();                  // token tiles grp, grp + G, ...
  const long long G = cluster_count_x();
  const int S = a.S, S1 = a.S + 1;  // stages per tile: the output pseudo-stage, then the sources
  const int c_base = ch * kKvbCols;
  const long long ntiles = grp < a.ntt ? (a.ntt - grp + G - 1) / G : 0;
  const long long I = ntiles * S1;  // stages of this CTA (the same for every CTA of the cluster)
  const uint32_t xtx = static_cast<uint32_t>(C - 1) * kKvbXBytes;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKvbStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 9);  // the dV warps have read V and the MMAs have finished with it
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
      mbar_init(&dks_full[i], 8);
      mbar_init(&dks_free[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&ac_full[i], 8);
    for (int i = 0; i < kKvbSlots; ++i) mbar_init(&xbar[i], 1);
    mbar_init(pfree, 8);
    mbar_init(wt_full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    // arm the first generation of every exchange slot before any partner can send
    for (int i = 0; i < kKvbSlots; ++i) mbar_arrive_expect_tx(&xbar[i], xtx);
  }
  if (threadIdx.x < kKvbR) q_s[threadIdx.x] = Elem<T>::to_f(static_cast<const T*>(a.q)[threadIdx.x]);
  if (warp == 1) tmem_alloc(tmem_slot, kKvbTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers are initialised before any exchange copy
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool row_ok = true;  // row warps: no wait has failed

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kKvbCtlRegs));
    if (warp == 0) {
      // ---------------- TMA producer -----------------------------------------
      if (lane == 0 && I > 0) {
        mbar_arrive_expect_tx(wt_full, kKvbKBytes);
        tma_load_2d(wt_tile, &a.wtmap, 0, c_base, wt_full);
        long long i = 0;
        for (; i < I; ++i) {
          const int st = static_cast<int>(i % kKvbStages);
          if (*abort_flag || !mbar_wait_bounded(&empty[st], static_cast<uint32_t>(((i / kKvbStages) & 1) ^ 1))) {
            atomicOr(&g_kvb_status, kStatusEmptyWaitTimeout);
            *abort_flag = 1;
            break;
          }
          const int pos = static_cast<int>(i % S1);
          const int t0 = static_cast<int>((grp + (i / S1) * G) * kKvbRows);
          const CUtensorMap* map = pos == 0 ? &a.omap : &a.vmap[pos - 1];
          unsigned char* sp = stages + st * kKvbStageBytes;
          mbar_arrive_expect_tx(&full[st], kKvbStageBytes);
          tma_load_2d(sp, map, c_base, t0, &full[st]);
          tma_load_2d(sp + kKvbAtom, map, c_base + kTmaBoxCols, t0, &full[st]);
        }
        if (*abort_flag) {
          // let the copies already issued land before the CTA can exit
          for (long long j = (i > kKvbStages ? i - kKvbStages : 0); j < i; ++j)
            if (!mbar_wait_bounded(&full[j % kKvbStages], static_cast<uint32_t>((j / kKvbStages) & 1)))
              atomicOr(&g_kvb_status, kStatusDrainTimeout);
        }
        if (!mbar_wait_bounded(wt_full, 0)) atomicOr(&g_kvb_status, kStatusDrainTimeout);
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ---------------------------------------------
      if (lane == 0 && I > 0) {
        bool issued_any = false;
        if (!mbar_wait_bounded(wt_full, 0)) {
          atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
        } else {
          tc_fence_after();
          const uint64_t dwt = umma_desc_sw128(wt_tile);
          const uint32_t d_dw = tmem_base + 2 * kKvbCols;
          long long m = 0;  // source stages so far
          for (long long i = 0; i < I && !*abort_flag; ++i) {
            const int st = static_cast<int>(i % kKvbStages);
            if (i % S1 == 0) {
              // output pseudo-stage: dots only (the commit is the MMA side's
              // share of freeing the stage)
              umma_commit(&empty[st]);
              continue;
            }
            const int ab = static_cast<int>(m & 1);
            const uint32_t mph = static_cast<uint32_t>((m >> 1) & 1);
            if (!mbar_wait_bounded(&acc_empty[ab], mph ^ 1u) || !mbar_wait_bounded(&dks_full[ab], mph) ||
                !mbar_wait_bounded(&full[st], static_cast<uint32_t>((i / kKvbStages) & 1))) {
              atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
              *abort_flag = 1;
              break;
            }
            tc_fence_after();
            const unsigned char* sp = stages + st * kKvbStageBytes;
            const unsigned char* kp = dks_tiles + ab * kKvbKBytes;
            const uint64_t dk = umma_desc_sw128(kp);
#pragma unroll
            for (int k = 0; k < kKvbR / 16; ++k)
              umma_f16(tmem_base + ab * kKvbCols, dk + 2 * k, dwt + 2 * k, a.idesc_dn, k > 0 ? 1u : 0u);
            umma_commit(&acc_full[ab]);
            const uint64_t dv = umma_desc_sw128_mn(sp, kKvbAtom);
            const uint64_t dkm = umma_desc_sw128_mn(kp, kKvbAtom);
#pragma unroll
            for (int k = 0; k < kKvbRows / 16; ++k)
              umma_f16(d_dw, dv + 128 * k, dkm + 128 * k, a.idesc_dw, (m > 0 || k > 0) ? 1u : 0u);
            umma_commit(&empty[st]);
            umma_commit(&dks_free[ab]);
            issued_any = true;
            ++m;
          }
        }
        umma_commit(done);
        if (issued_any && !mbar_wait_bounded(done, 0)) atomicOr(&g_kvb_status, kStatusDrainTimeout);
      }
    }
  } else if (warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kKvbEpiRegs));
    // ---------------- dot / exchange / dKs warps: a token row x 64 columns ----
    // Slot reuse: this CTA copies stage i into the partners' slot (i mod 4)
    // only after its own B(i-1), which needed every partner's stage i-1; a
    // partner that sent stage i-1 had finished its B(i-2) and re-armed that
    // slot's earlier generations, so generation i-4 has been read everywhere.
    constexpr int DK = kKvbR / H;
    const int row = ((warp - 4) & 3) * 32 + lane;
    const int half = (warp - 4) >> 2;  // 64-column half (= V box) and 32 key dims
    const int hown = c_base / (a.d / H);  // head of this CTA's columns
    const int cph = C / H;                // slices per head
    const T* gsrc = static_cast<const T*>(a.g);
    const T* ksrc = static_cast<const T*>(a.keys);
    float* xhalf = reinterpret_cast<float*>(acs + 4 * kKvbRows) + kKvbR;  // [128] half-1 partials
    Pack<T, 8> gA[8];  // g of the thread's 64 columns for the current tile
#pragma unroll
    for (int c = 0; c < 8; ++c) kvb_zero<T>(gA[c]);
    float gout[H];
#pragma unroll
    for (int h = 0; h < H; ++h) gout[h] = 0.f;
    bool good = I > 0;
    // A warp that fails a wait only clears `good`: the next stage's barrier
    // (bar 3, OR of the failures) takes all eight warps out of the loop
    // together, so none is left waiting there.
    for (long long it = 0; it < I + 1; ++it) {
      // ---- B(it-1): the slices' partials, dl, dKs half row, {alpha, coef} -----
      const long long jb = it - 1;
      if (jb >= 0 && good) do {  // a failed wait leaves through `break` to this stage's barrier
        const int pos = static_cast<int>(jb % S1);
        const int slot = static_cast<int>(jb % kKvbSlots);
        const long long t = (grp + (jb / S1) * G) * kKvbRows + row;
        const bool live = t < a.N;
        const int s = pos > 0 ? pos - 1 : 0;
        const long long tr = live ? t : 0;
        const long long m = (jb / S1) * S + pos - 1;
        Pack<T, 8> kr[4];
        float al[H];
        float4 pr[H];
        float inv = 1.f;
        if (pos > 0) {  // loads first: their latency overlaps the exchange wait
          const long long r = static_cast<long long>(s) * a.N + tr;
          const T* kp = ksrc + r * kKvbR + half * 32;
#pragma unroll
          for (int c = 0; c < 4; ++c) kr[c] = load_pack<T, 8>(kp + 8 * c);
#pragma unroll
          for (int h = 0; h < H; ++h) {
            al[h] = a.alpha[(tr * H + h) * S + s];
            pr[h] = a.prep[r * H + h];
          }
          if (a.vinv) inv = a.vinv[r];
        }
        good = !*abort_flag && mbar_wait_bounded(&xbar[slot], static_cast<uint32_t>((jb / kKvbSlots) & 1));
        if (good && row == 0 && half == 0) mbar_arrive_expect_tx(&xbar[slot], xtx);  // arm the next generation
        if (good && pos > 0)
          good = mbar_wait_bounded(&dks_free[m & 1], static_cast<uint32_t>(((m >> 1) & 1) ^ 1));
        if (!good) {
          *abort_flag = 1;
          atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
          break;
        }
        const float* xs = xbuf + slot * kKvbMaxCluster * kKvbRows + row;
        float dw[H];
#pragma unroll
        for (int h = 0; h < H; ++h) {
          float acc = 0.f;
          for (int e = h * cph; e < (h + 1) * cph; ++e) acc += xs[e * kKvbRows];
          dw[h] = acc;
        }
        if (pos == 0) {
#pragma unroll
          for (int h = 0; h < H; ++h) gout[h] = dw[h];
        } else {
          float dl[H], coef = 0.f, alo = 0.f;
#pragma unroll
          for (int h = 0; h < H; ++h) {
            dl[h] = live ? al[h] * (dw[h] - gout[h]) : 0.f;
            coef = fmaf(dl[h], pr[h].z, coef);
            alo = h == hown ? al[h] : alo;
            if (ch == 0 && half == 0 && live) a.dl[(static_cast<long long>(s) * a.N + t) * H + h] = dl[h];
          }
          unsigned char* krow = dks_tiles + static_cast<int>(m & 1) * kKvbKBytes + row * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int j = half * 32 + c * 8 + e;
              const int h = j / DK;
              const float u = fmaf(-pr[h].y, Elem<T>::to_f(kr[c].e[e]), pr[h].x * q_s[j]);
              // dK is rounded to T, as the read backward writes it
              o[e] = inv * Elem<T>::to_f(Elem<T>::from_f(dl[h] * u));
            }
            store_pack<T, 8>(reinterpret_cast<T*>(krow + (((half * 4 + c) ^ (row & 7)) << 4)), o);
          }
          if (half == 0) acs[(m & 3) * kKvbRows + row] = make_float2(live ? alo : 0.f, live ? coef : 0.f);
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&dks_full[m & 1]);
            mbar_arrive(&ac_full[m & 3]);
          }
        }
      } while (0);
      // ---- A(it): partial dot of the row over this slice, sent to the cluster
      if (it < I) {
        const int pos = static_cast<int>(it % S1);
        const long long t = (grp + (it / S1) * G) * kKvbRows + row;
        const bool live = t < a.N;
        const int slot = static_cast<int>(it % kKvbSlots);
        if (pos == 0) {
          const T* gp = gsrc + (live ? t : 0) * a.d + c_base + half * kTmaBoxCols;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            gA[c] = load_pack<T, 8>(gp + 8 * c);
            if (!live) kvb_zero<T>(gA[c]);
          }
        }
        const int st = static_cast<int>(it % kKvbStages);
        good = good && !*abort_flag && mbar_wait_bounded(&full[st], static_cast<uint32_t>((it / kKvbStages) & 1));
        float* xrow = xbuf + (slot * kKvbMaxCluster + ch) * kKvbRows;
        float p = 0.f;
        if (good) {
          const unsigned char* vrow = stages + st * kKvbStageBytes + half * kKvbAtom + row * 128;
          float p2 = 0.f;
#pragma unroll
          for (int c = 0; c < 8; c += 2) {
            const Pack<T, 8> v0 = *reinterpret_cast<const Pack<T, 8>*>(vrow + ((c ^ (row & 7)) << 4));
            const Pack<T, 8> v1 = *reinterpret_cast<const Pack<T, 8>*>(vrow + (((c + 1) ^ (row & 7)) << 4));
            p = dot_pack16<T, 8>(p, v0, gA[c]);
            p2 = dot_pack16<T, 8>(p2, v1, gA[c + 1]);
          }
          p += p2;
          if (half == 1) xhalf[row] = p;
        }
        // the eight warps meet twice (a failed one too, so nobody is left
        // waiting): the half-1 partials, then the row sums; then lanes 1..C-1
        // of the first warp each copy the slice's 128 sums into one partner
        if (kvb_sync_or(3, 256, !good)) {
          good = false;
        } else {
          if (half == 0) xrow[row] = p + xhalf[row];
          if (kvb_sync_or(3, 256, false)) good = false;
          if (good && warp == 4 && lane > 0 && lane < C) {
            fence_async_shared();
            const uint32_t dst = static_cast<uint32_t>((ch + lane) % C);
            bulk_s2cluster(map_to_rank(smem_u32(xrow), dst), xrow, kKvbXBytes,
                           map_to_rank(smem_u32(&xbar[slot]), dst));
          }
        }
        if (!good) {
          *abort_flag = 1;
          atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
          break;
        }
        // the output slice of a pseudo-stage is no longer read: the dV warps
        // may let the store warp free its ring stage
        if (pos == 0 && lane == 0) mbar_arrive(pfree);
      }
    }
    row_ok = good;
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kKvbEpiRegs));
    // ---------------- dV warps: one token row x 64 columns per thread ---------
    // dV goes straight from registers to global memory (each thread writes 128
    // contiguous bytes of its row), so a ring stage is free as soon as these
    // warps have read its V and the MMAs have finished with it.
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 12) >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const T* gsrc = static_cast<const T*>(a.g);
    Pack<T, 8> gC[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) kvb_zero<T>(gC[c]);
    bool good = I > 0;
    for (long long jc = 0; jc < I && good; ++jc) {
      const int pos = static_cast<int>(jc % S1);
      const int st = static_cast<int>(jc % kKvbStages);
      const long long t = (grp + (jc / S1) * G) * kKvbRows + row;
      const bool live = t < a.N;
      if (pos == 0) {
        const T* gp = gsrc + (live ? t : 0) * a.d + c_base + half * kTmaBoxCols;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          gC[c] = load_pack<T, 8>(gp + 8 * c);
          if (!live) kvb_zero<T>(gC[c]);
        }
        // the stage is freed after this step: wait until the dot warps have
        // read the tile's output slice
        good = !*abort_flag && mbar_wait_bounded(pfree, static_cast<uint32_t>((jc / S1) & 1));
      } else {
        const long long m = (jc / S1) * S + pos - 1;
        const int ab = static_cast<int>(m & 1);
        good = !*abort_flag && mbar_wait_bounded(&ac_full[m & 3], static_cast<uint32_t>((m >> 2) & 1)) &&
               mbar_wait_bounded(&full[st], static_cast<uint32_t>((jc / kKvbStages) & 1)) &&
               mbar_wait_bounded(&acc_full[ab], static_cast<uint32_t>((m >> 1) & 1));
        if (good) {
          tc_fence_after();
          const float2 ac = acs[(m & 3) * kKvbRows + row];
          const unsigned char* vrow = stages + st * kKvbStageBytes + half * kKvbAtom + row * 128;
          const uint32_t tcol = tmem_base + lane_off + ab * kKvbCols + half * kTmaBoxCols;
          T* drow = static_cast<T*>(a.dv[pos - 1]) + (live ? t : 0) * a.d + c_base + half * kTmaBoxCols;
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {  // 32 dn columns per TMEM wait
            uint32_t dr[2][16];
            tmem_ld16_nowait(tcol + 32 * hb, dr[0]);
            tmem_ld16_nowait(tcol + 32 * hb + 16, dr[1]);
            tmem_ld_wait();
            tmem_regs_ready(dr[0]);
            tmem_regs_ready(dr[1]);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const int c = hb * 4 + cc;
              const Pack<T, 8> vp = *reinterpret_cast<const Pack<T, 8>*>(vrow + ((c ^ (row & 7)) << 4));
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                o[e] = fmaf(ac.x, Elem<T>::to_f(gC[c].e[e]),
                            __uint_as_float(dr[cc >> 1][(cc & 1) * 8 + e]) - Elem<T>::to_f(vp.e[e]) * ac.y);
              if (live) store_pack<T, 8>(drow + 8 * c, o);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[ab]);
        }
      }
      if (!good) {
        *abort_flag = 1;
        atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // this CTA's slice of dWt: lane = column of the slice, this warp's 32 of
    // the 64 fp32 columns (= r)
    float* part = a.partials + (static_cast<long long>(blockIdx.x) * kKvbCols + row) * kKvbR + half * 32;
    if (I > 0 && good && mbar_wait_bounded(done, 0)) {
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < 32; c0 += 16) {
        float v[16];
        tmem_ld16(tmem_base + lane_off + 2 * kKvbCols + half * 32 + c0, v);
#pragma unroll
        for (int e = 0; e < 16; e += 4)
          *reinterpret_cast<float4*>(part + c0 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      }
    } else {
      if (I > 0) atomicOr(&g_kvb_status, kStatusFullWaitTimeout);
      for (int c0 = 0; c0 < 32; c0 += 4) *reinterpret_cast<float4*>(part + c0) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    row_ok = good;
  }
  if (!row_ok && threadIdx.x == 128) {
    // after a failed wait, give exchange copies still in flight (ours into the
    // partners, theirs into this CTA) time to land before the cluster can exit
    const unsigned long long t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 100000ull) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kKvbTmemCols);
  }
}

// Per (source s, token t, head h), from the key row k (dk = 64 / H dims of
// the head) with kinv = rsqrt(<k, k> / dk + eps) (1 without the key norm) and
// kq = <k, q>:  u0 = scale kinv,  u1 = u0 kinv^2 kq / dk (0 without the key
// norm),  w = inv^2 (u0 kq - u1 <k, k>) / d (0 without the value norm), so that
// dK_j = dl (u0 q_j - u1 k_j) and coef = sum_h dl_h w_h. Eight lanes per row.
template <typename T, int H>
__global__ void __launch_bounds__(256) kvb_prep_kernel(const T* __restrict__ keys, const float* __restrict__ vinv,
                                                       const T* __restrict__ q, long long rows, int d, float scale,
                                                       int key_norm, float key_eps, float4* __restrict__ prep) {
  constexpr int DK = kKvbR / H;
  constexpr int LPH = DK / 8;  // lanes per head
  const long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int sub = threadIdx.x & 7;
  const bool live = r < rows;
  const long long rr = live ? r : 0;
  const Pack<T, 8> kp = load_pack<T, 8>(keys + rr * kKvbR + sub * 8);
  const Pack<T, 8> qp = load_pack<T, 8>(q + sub * 8);
  float ss = 0.f, kq = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x = Elem<T>::to_f(kp.e[e]);
    ss = fmaf(x, x, ss);
    kq = fmaf(x, Elem<T>::to_f(qp.e[e]), kq);
  }
#pragma unroll
  for (int o = 1; o < LPH; o <<= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    kq += __shfl_xor_sync(0xffffffffu, kq, o);
  }
  if (!live || sub % LPH) return;
  const float kinv = key_norm ? rsqrtf(ss / DK + key_eps) : 1.f;
  const float u0 = scale * kinv;
  const float u1 = key_norm ? u0 * kinv * kinv * kq / DK : 0.f;
  const float inv = vinv ? vinv[rr] : 0.f;
  const float w = inv * inv * (u0 * kq - u1 * ss) / d;
  prep[rr * H + sub / LPH] = make_float4(u0, u1, w, 0.f);
}

// Wt[c][r] = W[r][c]; W is [64, d] with a row stride.
template <typename T>
__global__ void __launch_bounds__(256) kvb_transpose_w_kernel(const T* __restrict__ w, long long wstride, int d,
                                                              T* __restrict__ wt) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(d) * kKvbR) return;
  const int c = static_cast<int>(i / kKvbR), r = static_cast<int>(i % kKvbR);
  wt[i] = w[r * wstride + c];
}

// dq partials: block b sums scale * dl * khat over rows [b * rows_per, ...)
// of the flattened [S][N] rows, eight lanes per row (one 8-dim pack each),
// then over its warps in order; writes dqp[b][64].
constexpr int kKvbParamBlocks = 296;

template <typename T, int H>
__global__ void __launch_bounds__(256) kvb_dq_kernel(const T* __restrict__ keys, const float* __restrict__ dl,
                                                     long long rows, long long rows_per, float scale, int key_norm,
                                                     float key_eps, float* __restrict__ dqp) {
  constexpr int DK = kKvbR / H;
  constexpr int LPH = DK / 8;  // lanes per head
  __shared__ float red[8][kKvbR];
  const int sub = threadIdx.x & 7;
  const int h = (sub * 8) / DK;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const long long r0 = static_cast<long long>(blockIdx.x) * rows_per;
  const long long r1 = min(rows, r0 + rows_per);
  for (long long base = r0; base < r1; base += 32) {
    // every lane takes part in the shuffles; rows past r1 add 0
    const long long r = base + (threadIdx.x >> 3);
    const bool live = r < r1;
    const long long rr = live ? r : r0;
    const Pack<T, 8> kp = load_pack<T, 8>(keys + rr * kKvbR + sub * 8);
    float x[8], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x[e] = Elem<T>::to_f(kp.e[e]);
      ss = fmaf(x[e], x[e], ss);
    }
#pragma unroll
    for (int o = 1; o < LPH; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float kinv = key_norm ? rsqrtf(ss / DK + key_eps) : 1.f;
    const float c1 = live ? dl[rr * H + h] * scale : 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(c1, x[e] * kinv, acc[e]);
  }
  // lanes with the same sub: xor 8, 16 inside the warp, then warps in order
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 8);
    acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 16);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) < 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) red[w][sub * 8 + e] = acc[e];
  }
  __syncthreads();
  if (threadIdx.x < kKvbR) {
    float v = 0.f;
    for (int i = 0; i < 8; ++i) v += red[i][threadIdx.x];
    dqp[static_cast<long long>(blockIdx.x) * kKvbR + threadIdx.x] = v;
  }
}

// dq[j] = sum over blocks, in order, of dqp[b][j]; dbias[s] = sum over t and h
// of dl[s][t][h] (one CTA per source, fixed-order tree).
__global__ void __launch_bounds__(256) kvb_param_sum_kernel(const float* __restrict__ dqp, int nblk,
                                                            const float* __restrict__ dl, long long per_source,
                                                            float* __restrict__ dq, float* __restrict__ dbias) {
  __shared__ float red[256];
  if (blockIdx.x == 0) {
    if (threadIdx.x < kKvbR) {
      float v = 0.f;
      for (int b = 0; b < nblk; ++b) v += dqp[static_cast<long long>(b) * kKvbR + threadIdx.x];
      dq[threadIdx.x] = v;
    }
    return;
  }
  const int s = blockIdx.x - 1;
  const float* p = dl + static_cast<long long>(s) * per_source;
  float v = 0.f;
  for (long long i = threadIdx.x; i < per_source; i += 256) v += p[i];
  red[threadIdx.x] = v;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) dbias[s] = red[0];
}

// dW[r][slice * 128 + c] = sum over the slice's CTAs, in CTA order, of
// partials[cta][c][r].
__global__ void __launch_bounds__(256) kvb_reduce_dw_kernel(const float* __restrict__ partials, int nch, int G,
                                                            int d, float* __restrict__ dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over [64][d]
  if (i >= kKvbR * d) return;
  const int r = i / d, col = i % d;
  const int ch = col / kKvbCols, c = col % kKvbCols;
  float acc = 0.f;
  for (int g = 0; g < G; ++g) acc += partials[(static_cast<long long>(g * nch + ch) * kKvbCols + c) * kKvbR + r];
  dw[i] = acc;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static size_t kvb_align(size_t x) { return (x + 255) & ~size_t(255); }

using KvbFn = void (*)(KvbArgs);

static KvbFn kvb_fn(int H, bool bf) {
  switch (H) {
    case 1: return bf ? kvb_fused_kernel<__nv_bfloat16, 1> : kvb_fused_kernel<__half, 1>;
    case 2: return bf ? kvb_fused_kernel<__nv_bfloat16, 2> : kvb_fused_kernel<__half, 2>;
    case 4: return bf ? kvb_fused_kernel<__nv_bfloat16, 4> : kvb_fused_kernel<__half, 4>;
    default: return bf ? kvb_fused_kernel<__nv_bfloat16, 8> : kvb_fused_kernel<__half, 8>;
  }
}

static void kvb_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* at, int C, unsigned clusters, cudaStream_t st) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3(static_cast<unsigned>(C) * clusters);
  cfg->blockDim = dim3(kKvbThreads);
  cfg->dynamicSmemBytes = kKvbSmem;
  cfg->stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(C);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg->attrs = at;
  cfg->numAttrs = 1;
}

// Clusters of C CTAs (one per SM) resident at once, per device and kernel
// variant; 0 when the cluster shape cannot launch.
static int kvb_max_clusters(int C, int H, bool bf) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, C, H, bf ? 1 : 0);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  KvbFn fn = kvb_fn(H, bf);
  int n = 0;
  if (ensure_dynamic_smem(reinterpret_cast<const void*>(fn), static_cast<int>(kKvbSmem)) == cudaSuccess &&
      (C <= 8 || cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    int nsm = 0;
    if (cached_sm_count(&nsm) == cudaSuccess) {
      kvb_config(&cfg, at, C, static_cast<unsigned>(std::max(1, nsm / C)), nullptr);
      if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
    }
  }
  cudaGetLastError();  // a refused cluster shape is an answer, not an error
  cache[key] = n;
  return n;
}

static bool kvb_shape(int S, long long N, int d, int R, int H, int dtype, int* nch, int* G, int* ntt) {
  if (dtype == ATTNRES_DTYPE_F32 || R != kKvbR || S < 2 || S > kKvbMaxSources || N < 1) return false;
  if (!(H == 1 || H == 2 || H == 4 || H == 8)) return false;
  // (d / H) % 256: each head owns an even number of slices
  if (d % H || (d / H) % (2 * kKvbCols) || N > 0x7fffffffLL) return false;
  *nch = d / kKvbCols;
  if (*nch > kKvbMaxCluster) return false;
  if (encode_fn() == nullptr) return false;
  const int mc = kvb_max_clusters(*nch, H, dtype == ATTNRES_DTYPE_BF16);
  if (mc < 1) return false;
  *ntt = static_cast<int>((N + kKvbRows - 1) / kKvbRows);
  *G = std::max(1, std::min(mc, *ntt));
  return true;
}

size_t kvbwd_fused_workspace(int S, long long N, int d, int R, int H, int dtype) {
  int nch, G, ntt;
  if (!kvb_shape(S, N, d, R, H, dtype, &nch, &G, &ntt)) return 0;
  return kvb_align(static_cast<size_t>(d) * kKvbR * 2) +                    // Wt
         kvb_align(static_cast<size_t>(nch) * G * kKvbCols * kKvbR * 4) +   // dWt partials
         kvb_align(static_cast<size_t>(S) * N * H * 4) +                    // dl
         kvb_align(static_cast<size_t>(S) * N * H * 16) +                   // {u0, u1, w}
         kvb_align(static_cast<size_t>(kKvbParamBlocks) * kKvbR * 4);       // dq partials
}

cudaError_t kvbwd_fused_launch(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                               const int64_t* vstr, const void* w, long long w_stride, const void* keys,
                               const float* inv_rms, const float* alpha, const void* query, float scale,
                               int key_norm, float key_eps, const void* g, const void* out,
                               void* const* grad_values, float* grad_weight, float* grad_query,
                               float* grad_bias, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  int nch, G, ntt;
  if (!kvb_shape(S, N, d, R, H, dtype, &nch, &G, &ntt)) return cudaErrorNotSupported;
  if (workspace_bytes < kvbwd_fused_workspace(S, N, d, R, H, dtype)) return cudaErrorInvalidValue;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  void* wt = ws;
  ws += kvb_align(static_cast<size_t>(d) * kKvbR * 2);
  float* partials = reinterpret_cast<float*>(ws);
  ws += kvb_align(static_cast<size_t>(nch) * G * kKvbCols * kKvbR * 4);
  float* dl = reinterpret_cast<float*>(ws);
  ws += kvb_align(static_cast<size_t>(S) * N * H * 4);
  float4* prep = reinterpret_cast<float4*>(ws);
  ws += kvb_align(static_cast<size_t>(S) * N * H * 16);
  float* dqp = reinterpret_cast<float*>(ws);
  const bool bf = dtype == ATTNRES_DTYPE_BF16;
  cudaError_t e;
  {
    const long long n = static_cast<long long>(d) * kKvbR;
    const unsigned grid = static_cast<unsigned>((n + 255) / 256);
    if (bf)
      kvb_transpose_w_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), w_stride,
                                                                    d, static_cast<__nv_bfloat16*>(wt));
    else
      kvb_transpose_w_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w), w_stride, d,
                                                             static_cast<__half*>(wt));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  {
    const long long rows = static_cast<long long>(S) * N;
    const unsigned pg = static_cast<unsigned>((rows * 8 + 255) / 256);
#define KVB_PREP(TT, HH)                                                                                          \
  kvb_prep_kernel<TT, HH><<<pg, 256, 0, st>>>(static_cast<const TT*>(keys), inv_rms, static_cast<const TT*>(query), \
                                              rows, d, scale, key_norm, key_eps, prep)
    switch (H) {
      case 1: if (bf) KVB_PREP(__nv_bfloat16, 1); else KVB_PREP(__half, 1); break;
      case 2: if (bf) KVB_PREP(__nv_bfloat16, 2); else KVB_PREP(__half, 2); break;
      case 4: if (bf) KVB_PREP(__nv_bfloat16, 4); else KVB_PREP(__half, 4); break;
      default: if (bf) KVB_PREP(__nv_bfloat16, 8); else KVB_PREP(__half, 8); break;
    }
#undef KVB_PREP
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  KvbArgs a{};
  bool ok = true;
  for (int s = 0; s < S && ok; ++s) {
    ok = encode_2d(&a.vmap[s], dtype, values[s], N, d, vstr[s], kKvbRows);
  }
  ok = ok && encode_2d(&a.omap, dtype, out, N, d, d, kKvbRows);
  ok = ok && encode_2d(&a.wtmap, dtype, wt, d, kKvbR, kKvbR, kKvbCols);
  if (!ok) return cudaErrorInvalidValue;
  for (int s2 = 0; s2 < S; ++s2) a.dv[s2] = grad_values[s2];
  a.g = g;
  a.keys = keys;
  a.vinv = inv_rms;
  a.alpha = alpha;
  a.prep = prep;
  a.q = query;
  a.dl = dl;
  a.partials = partials;
  a.N = N;
  a.S = S;
  a.d = d;
  a.nch = nch;
  a.ntt = ntt;
  a.key_norm = key_norm;
  a.scale = scale;
  a.key_eps = key_eps;
  const uint32_t ab = bf ? 1u : 0u;
  a.idesc_dn = umma_idesc_f16(ab, 0, 0, kKvbRows, kKvbCols);
  a.idesc_dw = umma_idesc_f16(ab, 1, 1, kKvbCols, kKvbR);
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute at[1];
  kvb_config(&cfg, at, nch, static_cast<unsigned>(G), st);
  if ((e = cudaLaunchKernelEx(&cfg, kvb_fn(H, bf), a)) != cudaSuccess) return e;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const long long rows = static_cast<long long>(S) * N;
  const long long per = (rows + kKvbParamBlocks - 1) / kKvbParamBlocks;
  switch (H) {
    case 1: bf ? kvb_dq_kernel<__nv_bfloat16, 1><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp)
               : kvb_dq_kernel<__half, 1><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __half*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp); break;
    case 2: bf ? kvb_dq_kernel<__nv_bfloat16, 2><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp)
               : kvb_dq_kernel<__half, 2><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __half*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp); break;
    case 4: bf ? kvb_dq_kernel<__nv_bfloat16, 4><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp)
               : kvb_dq_kernel<__half, 4><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __half*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp); break;
    default: bf ? kvb_dq_kernel<__nv_bfloat16, 8><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp)
                : kvb_dq_kernel<__half, 8><<<kKvbParamBlocks, 256, 0, st>>>(static_cast<const __half*>(keys), dl, rows, per, scale, key_norm, key_eps, dqp); break;
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  kvb_param_sum_kernel<<<1 + (grad_bias ? S : 0), 256, 0, st>>>(dqp, kKvbParamBlocks, dl, N * H, grad_query,
                                                                 grad_bias);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int n = kKvbR * d;
  kvb_reduce_dw_kernel<<<(n + 255) / 256, 256, 0, st>>>(partials, nch, G, d, grad_weight);
  return cudaGetLastError();
}

cudaError_t read_kvbwd_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_kvb_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_kvb_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
