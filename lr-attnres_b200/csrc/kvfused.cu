// Key-from-value LRID read, forward, in one kernel: the key projection
// keys_s = rms_norm(V_s) @ W^T (model.py:344-356) fused with the depth softmax
// and the weighted sum (the read of attnres_ops.py:4195-4232), so V crosses
// HBM once.
//
// A cluster of C = d / 512 CTAs (C in {2, 4, 8}) splits the value columns: CTA
// `rank` owns columns [512 rank, 512 rank + 512) and, for the key step, tokens
// [rank * 32 / C, (rank + 1) * 32 / C) of every 32-token tile. It keeps its
// slice of W (64 x 512) in tensor memory for the whole launch as the A operand
// of tcgen05.mma (A from TMEM, M = 64 key dims), so the projection reads only
// the value tile from shared memory. Tiles are walked source by source; per
// (tile, source):
//   warp 0   TMA-loads the source's 32 x 512 value tile (one 3-D box, 128-byte
//            swizzle, chunk-major) into a ring stage;
//   warp 1   issues 32 MMAs (N = 32 tokens, K = 16) -> partial keys^T [64 x 32]
//            over this CTA's columns, in a double-buffered TMEM accumulator;
//   WG-A     (4 warps) sums the squares of each token's 512 columns, reads the
//            partial keys from TMEM into an outbox [32 tokens][64 keys | ss]
//            and bulk-copies each owner's token rows into the owner's receive
//            slot (cp.async.bulk shared::cta -> shared::cluster, completing on
//            the owner's mbarrier): a reduce-scatter;
//   WG-K     (2 warps) adds the C partials of its owned tokens in rank order,
//            forms the keys (rounded to the value type, saved for the
//            backward), the per-head key norm and the logits, and stores the
//            logits into every CTA of the cluster (st.async, completing on the
//            receiver's mbarrier);
//   WG-B     (8 warps) folds the source into an online softmax over this CTA's
//            columns, in registers: acc = acc * exp(m - m') + exp(l - m') V_s.
// After the last source the CTA writes its columns of out = acc / Z and the
// owned tokens' exact softmax weights (saved for the backward). A receive slot
// is reused only after every reader returned a credit (a 16-byte st.async that
// completes on the writer's credit barrier). Every wait is bounded and reports
// through a status word; TMEM is freed; no TMA multicast.
//
// Measured limiter (config 4, B200): a ring stage is released only when the
// logits of its source have come back through the cluster, ~10 us after its
// load is issued, and five 32 KB stages fit in shared memory, so a stage turns
// over every ~2.2 us instead of the 0.74 us one SM's share of HBM allows.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "plan.h"
#include "tma.cuh"
#include "umma.cuh"
#include "cluster.cuh"
#include "launch_cache.h"

namespace attnres {

constexpr int kKvT = 32;                 // tokens per tile (MMA N)
constexpr int kKvSlice = 512;            // value columns per CTA
constexpr int kKvR = 64;                 // key rank (MMA M)
constexpr int kKvBoxes = kKvSlice / 64;  // 64-column boxes per stage
constexpr uint32_t kKvStageBytes = kKvT * kKvSlice * 2;
constexpr uint32_t kKvBoxBytes = kKvStageBytes / kKvBoxes;
constexpr int kKvRow = kKvR + 4;         // floats per token row of a partial: 64 keys, ss, pad
constexpr uint32_t kKvTileBytes = kKvT * kKvRow * 4;  // one CTA's partials of a tile
constexpr int kKvMaxS = 32;
constexpr int kKvMaxH = 4;
constexpr int kKvKSlots = 2;             // partial-key receive slots (and outboxes)
constexpr int kKvLSlots = 4;             // logit receive slots (and outboxes)
constexpr int kKvMaxStages = 8;
constexpr int kKvThreads = 16 * 32;      // TMA, MMA, 4 WG-A, 2 WG-K, 8 WG-B warps
constexpr int kKvWgK = 192, kKvWgB = 256;  // first thread of WG-K, WG-B
constexpr uint32_t kKvTmemCols = 512;    // A: 256 columns, D: 2 x 32
constexpr uint32_t kKvDCol = 256;

static __device__ unsigned int g_kvf_status = 0;

struct KvfArgs {
  CUtensorMap vmap[kKvMaxS];  // V_s as {64 columns, N rows, d / 64 chunks}, box {64, 32, 8}
  const void* w;              // W [R, d] (value dtype), row stride wstride
  long long wstride;
  const void* q;              // static query [H, dk] (value dtype)
  const float* bias;          // [S] or null
  void* out;                  // [N, d]
  void* keys;                 // [S][N][R]
  float* vinv;                // [S][N]
  float* alpha;               // [N][H][S]
  long long N, ntiles;
  int S, d, stages, value_norm, key_norm;
  float value_eps, key_eps, scale;
  uint32_t idesc;
};

// Waits of this kernel: try_wait without a suspend-time hint (the hardware's
// own short wait), so a waiting thread sees the phase flip promptly; bounded
// like mbar_wait_bounded.
__device__ __forceinline__ bool kv_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool kv_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns = kWaitLimitNs) {
  if (kv_try(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (kv_try(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ bool named_sync_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---- tensor-memory helpers --------------------------------------------------
// D (+)= A(TMEM) * B(shared), kind::f16, A K-major in tensor memory
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :
      : "r"(tmem_d), "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
// 32 consecutive 32-bit columns of this thread's lane
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <typename T, int H>
__global__ void __launch_bounds__(kKvThreads, 1) kvfused_fwd_kernel(const __grid_constant__ KvfArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.S, d = a.d, NST = a.stages;
  const int C = d / kKvSlice;
  const int TPC = kKvT / C;                       // tokens owned per CTA in the key step
  const uint32_t kmsg = TPC * kKvRow * 4;         // one sender's partials for one owner
  const uint32_t lmsg = TPC * H * 4;              // one owner's logits
  const uint32_t rank = cluster_rank();
  unsigned char* stages = base;
  float* slotk = reinterpret_cast<float*>(stages + NST * kKvStageBytes);  // [KS][C senders][TPC][68]
  float* outk = slotk + kKvKSlots * (kKvTileBytes / 4);                     // [KS][32][68]
  float* slotl = outk + kKvKSlots * (kKvTileBytes / 4);                     // [LS][32][H]
  float* lg = slotl + kKvLSlots * kKvT * kKvMaxH;                           // [32][H][32] logits
  float* qs = lg + kKvT * kKvMaxH * 32;                                     // [64] query
  float* bs = qs + kKvR;                                                    // [32] logit bias
  float* pad = bs + kKvMaxS;  // [2][8][4]: landing pads of the credit signals, then a 16-byte source
  uint64_t* full = reinterpret_cast<uint64_t*>(pad + 2 * 8 * 4 + 4);
  uint64_t* empty = full + kKvMaxStages;
  uint64_t* accf = empty + kKvMaxStages;
  uint64_t* acce = accf + 2;
  uint64_t* recvk = acce + 2;
  uint64_t* credk = recvk + kKvKSlots;
  uint64_t* recvl = credk + kKvKSlots;
  uint64_t* credl = recvl + kKvLSlots;
  uint64_t* done = credl + kKvLSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nclusters = cluster_count_x();
  const long long cid = cluster_id_x();

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 4 + 8);  // MMA commit + WG-A warps + WG-B warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);
    }
    for (int p = 0; p < kKvKSlots; ++p) {
      mbar_init(&recvk[p], 1);
      mbar_init(&credk[p], 1);
    }
    for (int p = 0; p < kKvLSlots; ++p) {
      mbar_init(&recvl[p], 1);
      mbar_init(&credl[p], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int p = 0; p < kKvKSlots; ++p) mbar_arrive_expect_tx(&recvk[p], C * kmsg);
    for (int p = 0; p < kKvLSlots; ++p) mbar_arrive_expect_tx(&recvl[p], C * lmsg);
    // a credit is a 16-byte signal copy from each reader of the slot
    for (int p = 0; p < kKvKSlots; ++p) mbar_arrive_expect_tx(&credk[p], C * 16);
    for (int p = 0; p < kKvLSlots; ++p) mbar_arrive_expect_tx(&credl[p], C * 16);
  }
  // the previous launch's writes (and its tensor memory) are released first
  pdl_wait_then_release();
  if (warp == 1) tmem_alloc(tmem_slot, kKvTmemCols);
  if (threadIdx.x >= kKvWgB) {
    const int f = threadIdx.x - kKvWgB;
    if (f < kKvR) qs[f] = Elem<T>::to_f(static_cast<const T*>(a.q)[f]);
    if (f < S) bs[f] = a.bias ? a.bias[f] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp >= 2 && warp < 6) {
    // W's slice into tensor memory: key dim m = 16 * quadrant + lane (lanes
    // 16-31 of each quadrant are unused by the M = 64 layout; they get zeros),
    // element k of the slice in column k / 2 (two 16-bit elements per column)
    const int qd = warp & 3;
    const int m = qd * 16 + lane;
    const T* wrow = static_cast<const T*>(a.w) + static_cast<long long>(m) * a.wstride + rank * kKvSlice;
#pragma unroll 1
    for (int piece = 0; piece < kKvSlice / 64; ++piece) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (lane < 16) v = *reinterpret_cast<const uint4*>(wrow + piece * 64 + i * 8);
        r[4 * i] = v.x;
        r[4 * i + 1] = v.y;
        r[4 * i + 2] = v.z;
        r[4 * i + 3] = v.w;
      }
      tmem_st32(tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + piece * 32, r);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // every CTA's barriers are initialised before any cross-CTA traffic
  cluster_sync_all();

  const long long per_tile = S;
  const long long ntile_mine = cid < a.ntiles ? (a.ntiles - 1 - cid) / nclusters + 1 : 0;
  const long long total = ntile_mine * per_tile;

  if (warp == 0) {
    // ---------------- TMA producer --------------------------------------------
    long long j = 0;
    bool ok = true;
    for (; j < total && ok; ++j) {
      const long long tile = cid + (j / per_tile) * nclusters;
      const int s = static_cast<int>(j % per_tile);
      const int st = static_cast<int>(j % NST);
      int good = 1;
      if (lane == 0) {
        if (*abort_flag || !kv_wait(&empty[st], static_cast<uint32_t>(((j / NST) & 1) ^ 1))) {
          atomicOr(&g_kvf_status, kStatusEmptyWaitTimeout);
          *abort_flag = 1;
          good = 0;
        } else {
          mbar_arrive_expect_tx(&full[st], kKvStageBytes);
        }
      }
      if (!__shfl_sync(0xffffffffu, good, 0)) {
        ok = false;
        break;
      }
      if (lane == 0)
        tma_load_3d(stages + st * kKvStageBytes, &a.vmap[s], 0, static_cast<int>(tile * kKvT),
                    static_cast<int>(rank) * kKvBoxes, &full[st]);
      __syncwarp();
    }
    if (!ok && lane == 0) {
      // let the copies already issued land before the CTA can exit
      for (long long i = (j > NST ? j - NST : 0); i < j; ++i)
        if (!kv_wait(&full[i % NST], static_cast<uint32_t>((i / NST) & 1), 20000000ull))
          atomicOr(&g_kvf_status, kStatusDrainTimeout);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------------------------------------
    if (lane == 0) {
      bool issued = false;
      for (long long j = 0; j < total; ++j) {
        const int st = static_cast<int>(j % NST);
        const int b = static_cast<int>(j & 1);
        if (*abort_flag || !kv_wait(&full[st], static_cast<uint32_t>((j / NST) & 1)) ||
            !kv_wait(&acce[b], static_cast<uint32_t>(((j >> 1) & 1) ^ 1))) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const unsigned char* sa = stages + st * kKvStageBytes;
        const uint32_t dcol = tmem_base + kKvDCol + b * kKvT;
#pragma unroll 1
        for (int c = 0; c < kKvBoxes; ++c) {
          const uint64_t bd = umma_desc_sw128(sa + c * kKvBoxBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K = 16 per MMA: 8 TMEM columns of A, 32 bytes of B
            umma_f16_ts(dcol, tmem_base + c * 32 + k * 8, bd + 2 * k, a.idesc, (c | k) ? 1u : 0u);
        }
        umma_commit(&empty[st]);
        umma_commit(&accf[b]);
        issued = true;
      }
      umma_commit(done);
      if (issued && !kv_wait(done, 0)) atomicOr(&g_kvf_status, kStatusDrainTimeout);
    }
  } else if (warp < 6) {
    // ---------------- WG-A: sums of squares, partial keys, reduce-scatter -----
    const int e = threadIdx.x - 64;
    const int qd = warp & 3;
    const int tk = e >> 2, qq = e & 3;
    for (long long j = 0; j < total; ++j) {
      const int st = static_cast<int>(j % NST);
      const int b = static_cast<int>(j & 1);
      const int p = static_cast<int>(j % kKvKSlots);
      bool ok = !*abort_flag && kv_wait(&full[st], static_cast<uint32_t>((j / NST) & 1));
      float ss = 0.f;
      if (ok && a.value_norm) {
        float s4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const unsigned char* rowp = stages + st * kKvStageBytes + (2 * qq + cc) * kKvBoxBytes + tk * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((u ^ (tk & 7)) * 16));
            Mixed16<T>::sq_step(s4[0], v.x);
            Mixed16<T>::sq_step(s4[1], v.y);
            Mixed16<T>::sq_step(s4[2], v.z);
            Mixed16<T>::sq_step(s4[3], v.w);
          }
        }
        ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      ok = ok && kv_wait(&accf[b], static_cast<uint32_t>((j >> 1) & 1));
      ok = __all_sync(0xffffffffu, ok);
      uint32_t r0[16], r1[16];
      if (ok) {
        tc_fence_after();
        const uint32_t ta = tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + kKvDCol + b * kKvT;
        tmem_ld16_nowait(ta, r0);
        tmem_ld16_nowait(ta + 16, r1);
        tmem_ld_wait();
        tmem_regs_ready(r0);
        tmem_regs_ready(r1);
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
      // outbox p and every owner's slot p are free once each owner returned its
      // credit for the previous partials through slot p (then the credit
      // barrier expects the next round)
      if (j >= kKvKSlots) {
        ok = ok && mbar_wait_cluster(&credk[p], static_cast<uint32_t>((j / kKvKSlots - 1) & 1));
        if (ok && e == 0) mbar_arrive_expect_tx(&credk[p], C * 16);
      }
      float* ob = outk + p * (kKvTileBytes / 4);
      if (ok) {
        if (lane < 16) {
          const int m = qd * 16 + lane;
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            ob[t * kKvRow + m] = __uint_as_float(r0[t]);
            ob[(t + 16) * kKvRow + m] = __uint_as_float(r1[t]);
          }
        }
        if (qq == 0) ob[tk * kKvRow + kKvR] = ss;
        fence_async_shared();
      }
      if (named_sync_or(3, 128, !ok)) {
        if (e == 0) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      if (e < C) {
        // owner e's token rows -> owner e's slot p, at this sender's place
        const uint32_t dst = map_to_rank(smem_u32(slotk + (p * C + rank) * (kmsg / 4)), e);
        bulk_s2cluster(dst, ob + e * TPC * kKvRow, kmsg, map_to_rank(smem_u32(&recvk[p]), e));
      }
    }
  } else if (warp < 8) {
    // ---------------- WG-K: keys and logits of the owned tokens ---------------
    const int g = threadIdx.x - kKvWgK;
    constexpr int DK = kKvR / H;
    T* keys = static_cast<T*>(a.keys);
    for (long long j = 0; j < total; ++j) {
      const long long tile = cid + (j / per_tile) * nclusters;
      const int s = static_cast<int>(j % per_tile);
      const int pk = static_cast<int>(j % kKvKSlots);
      const int pl = static_cast<int>(j % kKvLSlots);
      bool ok = !*abort_flag && mbar_wait_cluster(&recvk[pk], static_cast<uint32_t>((j / kKvKSlots) & 1));
      // the logit outbox and every CTA's logit slot pl are free again
      if (j >= kKvLSlots) {
        ok = ok && mbar_wait_cluster(&credl[pl], static_cast<uint32_t>((j / kKvLSlots - 1) & 1));
        if (ok && g == 0) mbar_arrive_expect_tx(&credl[pl], C * 16);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        for (int item = g; item < TPC * 8; item += 64) {
          const int lt = item >> 3, pp = item & 7;  // owned token, key dims 4pp.., 32+4pp..
          float kv[8], sst = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) kv[i] = 0.f;
          for (int r = 0; r < C; ++r) {
            const float* row = slotk + (pk * C + r) * (kmsg / 4) + lt * kKvRow;
            const float4 x0 = *reinterpret_cast<const float4*>(row + 4 * pp);
            const float4 x1 = *reinterpret_cast<const float4*>(row + 32 + 4 * pp);
            kv[0] += x0.x;
            kv[1] += x0.y;
            kv[2] += x0.z;
            kv[3] += x0.w;
            kv[4] += x1.x;
            kv[5] += x1.y;
            kv[6] += x1.z;
            kv[7] += x1.w;
            sst += row[kKvR];
          }
          const float inv = a.value_norm ? rsqrtf(sst / d + a.value_eps) : 1.f;
          float kss[H], dot[H];
#pragma unroll
          for (int h = 0; h < H; ++h) kss[h] = dot[h] = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int dim = i < 4 ? 4 * pp + i : 32 + 4 * pp + i - 4;
            kv[i] = Elem<T>::to_f(Elem<T>::from_f(kv[i] * inv));  // the key, rounded to T
#pragma unroll
            for (int hh = 0; hh < H; ++hh)
              if (hh == dim / DK) {
                kss[hh] = fmaf(kv[i], kv[i], kss[hh]);
                dot[hh] = fmaf(kv[i], qs[dim], dot[hh]);
              }
          }
#pragma unroll
          for (int h = 0; h < H; ++h) {
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
              kss[h] += __shfl_xor_sync(0xffffffffu, kss[h], o);
              dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], o);
            }
          }
          const long long tok = tile * kKvT + rank * TPC + lt;
          if (tok < a.N) {
            T* kp = keys + (static_cast<long long>(s) * a.N + tok) * kKvR;
            const float k0[4] = {kv[0], kv[1], kv[2], kv[3]}, k1[4] = {kv[4], kv[5], kv[6], kv[7]};
            store_pack<T, 4>(kp + 4 * pp, k0);
            store_pack<T, 4>(kp + 32 + 4 * pp, k1);
            if (pp == 0 && a.vinv) a.vinv[static_cast<long long>(s) * a.N + tok] = inv;
          }
          if (pp < C) {
            // this token's logits into cluster CTA pp's slot pl
            const uint32_t dst = map_to_rank(smem_u32(slotl + (pl * kKvT + rank * TPC + lt) * H), pp);
            const uint32_t bar = map_to_rank(smem_u32(&recvl[pl]), pp);
#pragma unroll
            for (int h = 0; h < H; ++h) {
              const float kinv = a.key_norm ? rsqrtf(kss[h] / DK + a.key_eps) : 1.f;
              st_async_f32(dst + 4 * h, dot[h] * kinv * a.scale + bs[s], bar);
            }
          }
        }
      }
      if (named_sync_or(5, 64, !ok)) {
        if (g == 0) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      // slot pk is read: open its next phase, then signal each sender
      if (g == 0) mbar_arrive_expect_tx(&recvk[pk], C * kmsg);
      if (g >= 32 && g < 32 + C)
        st_async_signal(map_to_rank(smem_u32(pad + (0 * 8 + rank) * 4), g - 32),
                        map_to_rank(smem_u32(&credk[pk]), g - 32));
    }
  } else {
    // ---------------- WG-B: online softmax and output ------------------------
    const int f = threadIdx.x - kKvWgB;
    const int tk = f >> 3, pp = f & 7;  // token, and 16-byte piece pp of each 64-column box
    const int dvh = d / H;
    T* out = static_cast<T*>(a.out);
    float acc[kKvBoxes][8];
    float mrun[H], zrun[H];
#pragma unroll
    for (int h = 0; h < H; ++h) {
      mrun[h] = -INFINITY;
      zrun[h] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < kKvBoxes; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
    // the head of each of this thread's boxes
    int hbox[kKvBoxes];
#pragma unroll
    for (int c = 0; c < kKvBoxes; ++c) hbox[c] = H > 1 ? (static_cast<int>(rank) * kKvSlice + c * 64) / dvh : 0;
    for (long long j = 0; j < total; ++j) {
      const long long tile = cid + (j / per_tile) * nclusters;
      const int s = static_cast<int>(j % per_tile);
      const int st = static_cast<int>(j % NST);
      const int pl = static_cast<int>(j % kKvLSlots);
      const long long tok = tile * kKvT + tk;
      bool ok = !*abort_flag && mbar_wait_cluster(&recvl[pl], static_cast<uint32_t>((j / kKvLSlots) & 1));
      float l[H];
#pragma unroll
      for (int h = 0; h < H; ++h) l[h] = ok ? slotl[(pl * kKvT + tk) * H + h] : 0.f;
      if (named_sync_or(4, 256, !ok)) {
        if (f == 0) {
          atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      // logit slot pl is read: open its next phase, then signal each owner
      if (f == 0) mbar_arrive_expect_tx(&recvl[pl], C * lmsg);
      if (f >= 32 && f < 32 + C)
        st_async_signal(map_to_rank(smem_u32(pad + (1 * 8 + rank) * 4), f - 32),
                        map_to_rank(smem_u32(&credl[pl]), f - 32));
      float corr[H], pw[H];
#pragma unroll
      for (int h = 0; h < H; ++h) {
        if (pp == 0) lg[(tk * H + h) * 32 + s] = l[h];
        const float mn = fmaxf(mrun[h], l[h]);
        corr[h] = mrun[h] == -INFINITY ? 0.f : expf(mrun[h] - mn);
        pw[h] = expf(l[h] - mn);
        zrun[h] = fmaf(zrun[h], corr[h], pw[h]);
        mrun[h] = mn;
      }
      // fold this source's columns (still in the ring stage) into the sums
      ok = !*abort_flag && kv_wait(&full[st], static_cast<uint32_t>((j / NST) & 1));
      if (ok) {
        const unsigned char* rowp = stages + st * kKvStageBytes + tk * 128 + ((pp ^ (tk & 7)) * 16);
#pragma unroll
        for (int c = 0; c < kKvBoxes; ++c) {
          const Pack<T, 8> v = *reinterpret_cast<const Pack<T, 8>*>(rowp + c * kKvBoxBytes);
          float cr = corr[0], w = pw[0];
#pragma unroll
          for (int hh = 1; hh < H; ++hh)
            if (hh == hbox[c]) {
              cr = corr[hh];
              w = pw[hh];
            }
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[c][i] = fmaf(acc[c][i], cr, w * Elem<T>::to_f(v.e[i]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (!ok) {
        atomicOr(&g_kvf_status, kStatusFullWaitTimeout);
        *abort_flag = 1;
      }
      if (s == S - 1) {
        // ---- the tile's output columns and the owned tokens' weights --------
        if (tok < a.N) {
#pragma unroll
          for (int c = 0; c < kKvBoxes; ++c) {
            float z = zrun[0];
#pragma unroll
            for (int hh = 1; hh < H; ++hh)
              if (hh == hbox[c]) z = zrun[hh];
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = acc[c][i] / z;
            store_pack<T, 8>(out + tok * d + static_cast<long long>(rank) * kKvSlice + c * 64 + pp * 8, o);
          }
        }
        __syncwarp();
        if (tok < a.N && tk / TPC == static_cast<int>(rank) && a.alpha) {
#pragma unroll
          for (int h = 0; h < H; ++h)
            for (int s2 = pp; s2 < S; s2 += 8)
              a.alpha[(tok * H + h) * S + s2] = expf(lg[(tk * H + h) * 32 + s2] - mrun[h]) / zrun[h];
        }
        __syncwarp();
#pragma unroll
        for (int h = 0; h < H; ++h) {
          mrun[h] = -INFINITY;
          zrun[h] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < kKvBoxes; ++c)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // no cluster CTA still sends into this CTA's shared memory
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kKvTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// V [N rows, d cols] (row stride in elements) as a 3-D map {64 columns, rows,
// d / 64 column chunks}: one box {64, 32, 8} is a CTA's 32 x 512 tile, landing
// chunk-major ([8][32 rows][128 bytes], 128-byte swizzle) in one copy.
static bool encode_row_chunks(CUtensorMap* map, int dtype, const void* ptr, long long rows, int cols,
                              long long row_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols / 64)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * 2, 128};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kKvT), static_cast<cuuint32_t>(kKvBoxes)};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == ATTNRES_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static size_t kvf_fixed_bytes() {
  return 1024 + 2 * static_cast<size_t>(kKvKSlots) * kKvTileBytes + sizeof(float) * kKvLSlots * kKvT * kKvMaxH +
         sizeof(float) * (kKvT * kKvMaxH * 32 + kKvR + kKvMaxS + 2 * 8 * 4 + 4) +
         8 * (2 * kKvMaxStages + 4 + 2 * kKvKSlots + 2 * kKvLSlots + 1) + 16;
}

bool kvfused_eligible(int S, long long N, int d, int R, int H, int dtype, const void* const* values,
                      const int64_t* vstr, const void* w, long long w_stride, const char** why) {
  *why = "";
  if (dtype != ATTNRES_DTYPE_BF16 && dtype != ATTNRES_DTYPE_F16) return *why = "needs f16/bf16 rows", false;
  if (R != kKvR) return *why = "needs key_dim 64", false;
  if (S < 2 || S > kKvMaxS) return *why = "needs 2..32 sources", false;
  if (N < 1 || (d != 2 * kKvSlice && d != 4 * kKvSlice && d != 8 * kKvSlice))
    return *why = "needs value_dim 1024, 2048 or 4096", false;
  if (H != 1 && H != 2 && H != 4) return *why = "needs 1, 2 or 4 heads", false;
  if ((d / H) % 64) return *why = "needs (value_dim / heads) % 64 == 0", false;
  if (N > 0x7fffffffLL) return *why = "too many tokens for 32-bit TMA coordinates", false;
  if (!aligned16p(w) || (w_stride * 2) % 16) return *why = "weight rows must be 16-byte aligned", false;
  for (int s = 0; s < S; ++s)
    if (!aligned16p(values[s]) || (vstr[s] * 2) % 16) return *why = "value rows must be 16-byte aligned", false;
  int cap = 0;
  if (cached_smem_optin(&cap) != cudaSuccess) return *why = "no device", false;
  if (static_cast<size_t>(cap) < kvf_fixed_bytes() + 2 * kKvStageBytes) return *why = "not enough shared memory", false;
  return encode_fn() != nullptr || (*why = "no cuTensorMapEncodeTiled", false);
}

cudaError_t kvfused_forward_launch(int S, long long N, int d, int H, int dtype, const void* const* values,
                                   const int64_t* vstr, const void* w, long long w_stride, int value_norm,
                                   float value_eps, const void* q, float scale, int key_norm, float key_eps,
                                   const float* bias, void* out, void* keys, float* vinv, float* alpha,
                                   cudaStream_t st) {
  KvfArgs a{};
  for (int s = 0; s < S; ++s) {
    if (!encode_row_chunks(&a.vmap[s], dtype, values[s], N, d, vstr[s])) return cudaErrorInvalidValue;
  }
  const int C = d / kKvSlice;
  a.w = w;
  a.wstride = w_stride;
  a.q = q;
  a.bias = bias;
  a.out = out;
  a.keys = keys;
  a.vinv = vinv;
  a.alpha = alpha;
  a.N = N;
  a.ntiles = (N + kKvT - 1) / kKvT;
  a.S = S;
  a.d = d;
  a.value_norm = value_norm;
  a.key_norm = key_norm;
  a.value_eps = value_eps;
  a.key_eps = key_eps;
  a.scale = scale;
  a.idesc = umma_idesc_f16(dtype == ATTNRES_DTYPE_BF16 ? 1u : 0u, 0u, 0u, kKvR, kKvT);
  int cap = 0, nsm = 0;
  cudaError_t e = cached_smem_optin(&cap);
  if (e != cudaSuccess) return e;
  if ((e = cached_sm_count(&nsm)) != cudaSuccess) return e;
  const size_t fixed = kvf_fixed_bytes();
  a.stages = static_cast<int>(std::min<size_t>(kKvMaxStages, (static_cast<size_t>(cap) - fixed) / kKvStageBytes));
  if (a.stages < 2) return cudaErrorInvalidConfiguration;
  const size_t smem = fixed + static_cast<size_t>(a.stages) * kKvStageBytes;
  const bool bf = dtype == ATTNRES_DTYPE_BF16;
  void (*fn)(KvfArgs) = nullptr;
  switch (H) {
    case 1: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 1> : kvfused_fwd_kernel<__half, 1>; break;
    case 2: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 2> : kvfused_fwd_kernel<__half, 2>; break;
    default: fn = bf ? kvfused_fwd_kernel<__nv_bfloat16, 4> : kvfused_fwd_kernel<__half, 4>; break;
  }
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kKvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(C);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // as many clusters as are resident at once (one CTA per SM), each walking
  // its tiles
  cfg.gridDim = dim3(static_cast<unsigned>(C * std::max(1, nsm / C)));
  int max_clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&max_clusters, fn, &cfg);
  if (e != cudaSuccess) return e;
  if (max_clusters < 1) return cudaErrorInvalidConfiguration;
  const long long nclusters = std::max<long long>(1, std::min<long long>(a.ntiles, max_clusters));
  cfg.gridDim = dim3(static_cast<unsigned>(C * nclusters));
  cfg.numAttrs = 2;
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
