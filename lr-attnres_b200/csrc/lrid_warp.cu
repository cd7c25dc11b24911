// LRID block Attention-Residual read, forward and backward: self-fed warps
// streaming one token row at a time through a private bulk-copy ring.
//
// Arithmetic and semantics are those of lrid.cu / lrid_tma.cu (fp32, the
// reference's _lrid_read_torch_list attnres_ops.py:4195-4232 and the backward
// of _lrid_attnres_list_backward_kernel attnres_ops.py:602-746). Layout:
//   * every warp of a persistent CTA owns whole token rows (t = blockIdx.x +
//     (warp + k * warps) * gridDim.x) and a private ring of NSW stages;
//   * a token is a sequence of units: unit 0 = the S key rows (+ the token's
//     query), units 1..C = one 512-byte column chunk of all S value rows (+ the
//     upstream-gradient chunk in the backward);
//   * lane 0 issues the cp.async.bulk copies of unit j + NSW - 1 right after
//     the warp has finished unit j - 1 in that stage, so NSW - 1 units of every
//     warp are always in flight while the warp computes the current one;
//   * all reductions are warp shuffles; nothing waits on another warp until
//     the final fixed-order sum of the parameter gradients.
// A warp holds only one small unit while it computes, so most of the shared
// memory is in flight: that is what keeps HBM busy (a single-token-stage
// design held most of its ring in compute). The ring of each warp is used
// strictly in order, so one mbarrier per stage (parity = use count & 1) is
// unambiguous. Waits are bounded (~2 s) and report through a status word.
// Row widths must split into 512-byte chunks per head: (d/H) % (32*VEC) == 0.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "lrid_args.cuh"
#include "tma.cuh"

namespace attnres {

static __device__ unsigned int g_warp_status = 0;

constexpr int kStreamMaxWarps = 20;
constexpr int kStreamMaxStages = 4;

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Backward warps per CTA: up to 16, or 12 above 16 sources, where the larger
// per-source register arrays need more registers per thread (and shared memory
// holds no more warps' rings anyway).
constexpr int kStreamBwdWarps = 16;
constexpr int kStreamBwdWarpsManySources = 12;

template <typename T, int KP, int SMAX, bool BWD>
__global__ void __launch_bounds__(BWD ? (SMAX > 16 ? kStreamBwdWarpsManySources : kStreamBwdWarps) * 32 : 640, 1) lrid_stream_kernel(const __grid_constant__ LridArgs a) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int KE = KP * VEC;
  constexpr int CW = 32 * VEC;  // columns per chunk unit (512 bytes per row)
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const LridPlan& P = a.p;
  const TmaLayout& L = a.tma;
  const int S = P.S, H = P.H, dk = P.dk, dv = P.dv, d = P.d, R = P.R;
  const int NSW = L.stages;
  const int NW = blockDim.x >> 5;
  const int KL = L.key_lanes;
  const bool has_qd = a.qmode != ATTNRES_QUERY_STATIC;
  const int SH = S * H;
  const int SP = (S + 3) & ~3;  // per-head row stride of the scratch arrays (16-byte rows)
  const int HSP = H * SP;
  const int C = d / CW, cph = dv / CW, U1 = C + 1;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);  // [NW][NSW]
  long long* tokq_all = reinterpret_cast<long long*>(bars + kStreamMaxWarps * kStreamMaxStages);  // [NW][NSW]
  const T** sv = reinterpret_cast<const T**>(tokq_all + kStreamMaxWarps * kStreamMaxStages);
  const T** sk = sv + S;
  long long* svs = reinterpret_cast<long long*>(sk + S);
  long long* sks = svs + S;
  T** sgv = reinterpret_cast<T**>(sks + S);
  T** sgk = sgv + S;
  float* ep = reinterpret_cast<float*>(sgk + S);  // epilogue [NW][R + H + S]
  unsigned char* wscr0 = smem_raw + L.off_y;      // per-warp scratch, L.off_qd bytes each
  unsigned char* stage0 = smem_raw + L.stage_off;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (lane == 0) {
    for (int i = 0; i < NSW; ++i) mbar_init(&bars[w * NSW + i], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < S; i += blockDim.x) {
    sv[i] = static_cast<const T*>(a.v[i]);
    sk[i] = static_cast<const T*>(a.k[i]);
    svs[i] = a.vs[i];
    sks[i] = a.ks[i];
    sgv[i] = static_cast<T*>(a.gv[i]);
    sgk[i] = static_cast<T*>(a.gk[i]);
  }
  __syncthreads();

  // per-warp scratch: logit | alpha | kinv | qk | dw (each [H][S] fp32), then
  // (backward) a copy of the token's key rows [S][R] and query [R]
  float* sm_logit = reinterpret_cast<float*>(wscr0 + static_cast<size_t>(w) * L.off_qd);
  float* sm_alpha = sm_logit + HSP;
  float* sm_kinv = sm_alpha + HSP;
  float* sm_qk = sm_kinv + HSP;
  float* sm_dw = sm_qk + HSP;
  T* kcopy = reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(sm_logit) + L.off_v);
  T* qcopy = kcopy + S * R;
  unsigned char* ring = stage0 + static_cast<size_t>(w) * NSW * L.stage_bytes;
  uint64_t* wbars = bars + w * NSW;

  // Token schedule. Static: this warp takes tokens first, first + step, ...
  // Dynamic (a.claim set): the warp takes the next unclaimed token from a
  // global counter each time its copy issue reaches a new token, so warps on
  // faster SMs take more tokens and all warps finish within about one token.
  const long long N = P.N;
  const long long step = static_cast<long long>(NW) * gridDim.x;
  long long stat_next = blockIdx.x + static_cast<long long>(w) * gridDim.x;
  // Lane 0 keeps one claim in flight, so the atomic's round trip overlaps a
  // token's work instead of stalling the copy issue.
  unsigned long long* claim = a.claim;
  unsigned long long claimed = 0;
  if (claim != nullptr && lane == 0) claimed = atomicAdd(claim, 1ull);
  auto next_token = [&]() -> long long {
    if (claim != nullptr) {
      const unsigned long long v = __shfl_sync(0xffffffffu, claimed, 0);
      if (lane == 0) claimed = atomicAdd(claim, 1ull);
      return static_cast<long long>(v);
    }
    const long long t = stat_next;
    stat_next += step;
    return t;
  };
  // token of the key unit held in each ring stage (N marks the end)
  long long* tokq = tokq_all + w * NSW;

  const T* gsrc = static_cast<const T*>(a.g);
  const T* qsrc = static_cast<const T*>(a.qdyn);
  // Position of a unit in this warp's sequence, advanced incrementally (no
  // division in the token loop): token row t, unit u within the token, ring
  // stage st and the stage's phase parity ph.
  struct Cursor {
    long long t;
    int u, st;
    uint32_t ph;
  };
  auto advance = [&](Cursor& c) {
    if (++c.u == U1) c.u = 0;
    if (++c.st == NSW) {
      c.st = 0;
      c.ph ^= 1u;
    }
  };
  // Issue the copies of the unit at cursor c: lane 0 posts the byte count,
  // then lane i copies the rows of sources i, i + 32, ... (the whole warp
  // calls this, converged). Each lane forms its sources' value-row pointers
  // once per token, when the token's key unit is issued.
  constexpr int NL = (SMAX + 31) / 32;
  const T* vrow[NL];
#pragma unroll
  for (int i = 0; i < NL; ++i) vrow[i] = nullptr;
  const T* grow = nullptr;  // this token's grad-output row (backward)
  auto issue = [&](const Cursor& c) {
    const long long t = c.t;
    unsigned char* st = ring + static_cast<size_t>(c.st) * L.stage_bytes;
    uint64_t* bar = &wbars[c.st];
    if (c.u == 0) {
      const uint32_t kb = R * sizeof(T);
      if (lane == 0) mbar_arrive_expect_tx(bar, S * kb + (has_qd ? kb : 0));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const int s = lane + 32 * i;
        if (s < S) {
          bulk_g2s(st + s * kb, sk[s] + t * sks[s], kb, bar);
          vrow[i] = sv[s] + t * svs[s];
        }
      }
      if (has_qd && lane == (S & 31)) bulk_g2s(st + S * kb, qsrc + t * R, kb, bar);
      if (BWD) grow = gsrc + t * d;
    } else {
      const int c0 = (c.u - 1) * CW;
      const uint32_t cb = CW * sizeof(T);
      if (lane == 0) mbar_arrive_expect_tx(bar, S * cb + (BWD ? cb : 0));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const int s = lane + 32 * i;
        if (s < S) bulk_g2s(st + s * cb, vrow[i] + c0, cb, bar);
      }
      if (BWD && lane == (S & 31)) bulk_g2s(st + S * cb, grow + c0, cb, bar);
    }
  };

  // key-segment mapping: groups of KL lanes, fixed head per lane
  const int G = 32 / KL;
  const int gidx = lane / KL, kl = lane % KL;
  const int hshift = __ffs(H) - 1;  // H is a power of two
  const int kh = gidx & (H - 1);
  const int kcol = kh * dk + kl * KE;
  const int rounds = (SH + G - 1) / G;

  float qs[KE];
  {
    const T* qp = static_cast<const T*>(a.q);
#pragma unroll
    for (int e = 0; e < KE; ++e) qs[e] = (a.qmode != ATTNRES_QUERY_DYNAMIC) ? load_f(qp + kcol + e) : 0.f;
  }
  const float gate_k = (a.qmode == ATTNRES_QUERY_GATED) ? load_f(static_cast<const T*>(a.gate) + kh) : 0.f;
  float dq_acc[KE];
#pragma unroll
  for (int e = 0; e < KE; ++e) dq_acc[e] = 0.f;
  float dgate_acc = 0.f, dbias0 = 0.f, dbias1 = 0.f;
  float dwp[SMAX];
#pragma unroll
  for (int s = 0; s < SMAX; ++s) dwp[s] = 0.f;
  float q[KE];
#pragma unroll
  for (int e = 0; e < KE; ++e) q[e] = qs[e];
  // 16-bit T: the query also as packed pairs of T for the mixed-precision key
  // dot products (the reference casts the query to the key dtype)
  uint32_t q16[KE / 2];
  auto pack_q16 = [&]() {
    if constexpr (kIs16<T>) {
#pragma unroll
      for (int i = 0; i < KE / 2; ++i)
        q16[i] = static_cast<uint32_t>(Mixed16<T>::bits(q[2 * i])) |
                 (static_cast<uint32_t>(Mixed16<T>::bits(q[2 * i + 1])) << 16);
    }
  };
  pack_q16();

  // Copy issue runs NSW - 1 units ahead of the consumer. Reaching a new token,
  // it records the token in the stage's slot; a token >= N ends the issue.
  Cursor pc{next_token(), 0, 0, 0u};  // next unit to issue
  bool issuing = true;
  long long issued = 0;
  auto issue_next = [&]() {
    if (pc.u == 0) {
      tokq[pc.st] = pc.t;  // every lane writes the same value
      if (pc.t >= N) {
        issuing = false;
        return;
      }
    }
    issue(pc);
    ++issued;
    advance(pc);
    if (pc.u == 0) pc.t = next_token();
  };
  for (int i = 0; i < NSW - 1 && issuing; ++i) issue_next();

  Cursor cc{0, 0, 0, 0u};  // unit being consumed
  long long j = 0;
  int hcnt = 0, hcur = 0;  // chunk position inside the current head
  for (;; ++j, advance(cc)) {
    if (issuing) {
      // the stage of unit j - 1 has been consumed by every lane: refill it
      __syncwarp();
      fence_proxy_async_smem();
      issue_next();
    }
    if (cc.u == 0) {
      cc.t = tokq[cc.st];
      if (cc.t >= N) break;
    }
    if (!mbar_wait_bounded(&wbars[cc.st], cc.ph)) {
      if (lane == 0) atomicOr(&g_warp_status, kStatusFullWaitTimeout);
      break;
    }
    const unsigned char* st = ring + static_cast<size_t>(cc.st) * L.stage_bytes;
    const long long t = cc.t;
    const int u = cc.u;

    if (u == 0) {
      // ---- new token: key rows, logits, softmax ---------------------------
      const T* kt = reinterpret_cast<const T*>(st);
      const T* qdt = kt + S * R;
      if (BWD) {
        // keep the key rows (and query) for the key-gradient phase
        const int npk = (S * R + (has_qd ? R : 0)) / VEC;
        for (int i = lane; i < npk; i += 32)
          *reinterpret_cast<Pack<T, VEC>*>(kcopy + i * VEC) = lds_pack<T, VEC>(kt + i * VEC);
      }
      if (has_qd) {
#pragma unroll
        for (int pk = 0; pk < KP; ++pk) {
          const Pack<T, VEC> qr = lds_pack<T, VEC>(qdt + kcol + pk * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float qd = Elem<T>::to_f(qr.e[e]);
            q[pk * VEC + e] = (a.qmode == ATTNRES_QUERY_DYNAMIC) ? qd : qs[pk * VEC + e] + gate_k * qd;
          }
        }
        pack_q16();
      }
      for (int r = 0; r < rounds; ++r) {
        const int seg = r * G + gidx;  // seg = s * H + h, h == kh
        const int s = seg >> hshift;
        float ss = 0.f, dot = 0.f;
        if (seg < SH) {
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            const Pack<T, VEC> kr = lds_pack<T, VEC>(kt + s * R + kcol + pk * VEC);
            if constexpr (kIs16<T>) {
              const uint32_t* kw = reinterpret_cast<const uint32_t*>(kr.e);
#pragma unroll
              for (int i = 0; i < VEC / 2; ++i) Mixed16<T>::key_step(ss, dot, kw[i], q16[pk * VEC / 2 + i]);
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                const float x = Elem<T>::to_f(kr.e[e]);
                ss = fmaf(x, x, ss);
                dot = fmaf(x, q[pk * VEC + e], dot);
              }
            }
          }
        }
        ss = group_sum(ss, KL);
        dot = group_sum(dot, KL);
        if (seg < SH && kl == 0) {
          const float kinv = a.key_norm ? rsqrtf(ss / dk + a.key_eps) : 1.f;
          const float qk = dot * kinv;
          sm_logit[kh * SP + s] = qk * a.scale + (a.bias ? a.bias[s] : 0.f);
          sm_kinv[kh * SP + s] = kinv;
          sm_qk[kh * SP + s] = qk;
        }
      }
      __syncwarp();
      for (int h = 0; h < H; ++h) {
        const float* lg = sm_logit + h * SP;
        const float l0 = lane < S ? lg[lane] : -INFINITY;
        const float l1 = lane + 32 < S ? lg[lane + 32] : -INFINITY;
        const float m = warp_max(fmaxf(l0, l1));
        const float e0 = lane < S ? expf(l0 - m) : 0.f;
        const float e1 = lane + 32 < S ? expf(l1 - m) : 0.f;
        const float sum = warp_sum(e0 + e1);
        if (lane < S) sm_alpha[h * SP + lane] = e0 / sum;
        if (lane + 32 < S) sm_alpha[h * SP + lane + 32] = e1 / sum;
        if (!BWD) {
          if (a.alpha_out) {
            if (lane < S) a.alpha_out[(t * H + h) * S + lane] = e0 / sum;
            if (lane + 32 < S) a.alpha_out[(t * H + h) * S + lane + 32] = e1 / sum;
          }
          if (a.kinv_out) {
            if (lane < S) a.kinv_out[(t * H + h) * S + lane] = sm_kinv[h * SP + lane];
            if (lane + 32 < S) a.kinv_out[(t * H + h) * S + lane + 32] = sm_kinv[h * SP + lane + 32];
          }
        }
      }
      __syncwarp();
      continue;
    }

    // ---- value chunk c of this token ----------------------------------------
    const int c = u - 1;
    if (c == 0) hcnt = hcur = 0;
    const int h = hcur;
    const int col = c * CW + lane * VEC;
    const T* vt = reinterpret_cast<const T*>(st) + lane * VEC;  // + s * CW
    const float* al = sm_alpha + h * SP;
    if constexpr (!BWD) {
      float acc[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
      // sources in blocks of four: one 16-byte read of their weights, four
      // value packs, then the packed FMAs; the last block is guarded
      int s0 = 0;
      for (; s0 + 4 <= S; s0 += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(al + s0);
        Pack<T, VEC> r4[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) r4[jj] = lds_pack<T, VEC>(vt + (s0 + jj) * CW);
        if constexpr (kIs16<T>) {
          // weights rounded to T (as the reference's PyTorch path casts them),
          // widened inside the FMA with the values: no conversion instructions
          axpy_pack16<T, VEC>(acc, Mixed16<T>::bits(w4.x), r4[0]);
          axpy_pack16<T, VEC>(acc, Mixed16<T>::bits(w4.y), r4[1]);
          axpy_pack16<T, VEC>(acc, Mixed16<T>::bits(w4.z), r4[2]);
          axpy_pack16<T, VEC>(acc, Mixed16<T>::bits(w4.w), r4[3]);
        } else {
          axpy_pack<T, VEC>(acc, w4.x, r4[0]);
          axpy_pack<T, VEC>(acc, w4.y, r4[1]);
          axpy_pack<T, VEC>(acc, w4.z, r4[2]);
          axpy_pack<T, VEC>(acc, w4.w, r4[3]);
        }
      }
      if (s0 < S) {
        const float4 w4 = *reinterpret_cast<const float4*>(al + s0);
        const float wj[4] = {w4.x, w4.y, w4.z, w4.w};
        Pack<T, VEC> r4[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (s0 + jj < S) r4[jj] = lds_pack<T, VEC>(vt + (s0 + jj) * CW);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (s0 + jj < S) {
            if constexpr (kIs16<T>) axpy_pack16<T, VEC>(acc, Mixed16<T>::bits(wj[jj]), r4[jj]);
            else axpy_pack<T, VEC>(acc, wj[jj], r4[jj]);
          }
      }
      store_pack<T, VEC>(static_cast<T*>(a.out) + t * d + col, acc);
      if (++hcnt == cph) {
        hcnt = 0;
        ++hcur;
      }
    } else {
      float gp[VEC];
      const Pack<T, VEC> gr = lds_pack<T, VEC>(reinterpret_cast<const T*>(st) + S * CW + lane * VEC);
#pragma unroll
      for (int e = 0; e < VEC; ++e) gp[e] = Elem<T>::to_f(gr.e[e]);
#pragma unroll
      for (int s0 = 0; s0 < SMAX; s0 += 4) {
        if (s0 < S) {
          Pack<T, VEC> r4[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            if (s0 + jj < S) r4[jj] = lds_pack<T, VEC>(vt + (s0 + jj) * CW);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            if (s0 + jj < S) {
              const float wgt = al[s0 + jj];
              if constexpr (kIs16<T>) dwp[s0 + jj] = dot_pack16<T, VEC>(dwp[s0 + jj], r4[jj], gr);
              else dwp[s0 + jj] = dot_pack<T, VEC>(dwp[s0 + jj], gp, r4[jj]);
              if (sgv[s0 + jj]) {
                float gv[VEC];
#pragma unroll
                for (int e = 0; e < VEC; e += 2) mul2(gv[e], gv[e + 1], wgt, gp[e], gp[e + 1]);
                store_pack<T, VEC>(sgv[s0 + jj] + t * d + col, gv);
              }
            }
          }
        }
      }
      if (++hcnt == cph) {
        hcnt = 0;
        // last chunk of head h: finish dw_s = <g', V_s> over the head
#pragma unroll
        for (int s = 0; s < SMAX; ++s) {
          if (s < S) {
            const float dw = warp_sum(dwp[s]);
            if (lane == 0) sm_dw[h * SP + s] = dw;
          }
          dwp[s] = 0.f;
        }
        ++hcur;
      }
      if (u == C) {
        __syncwarp();
        // ---- dlogit per head (stored over the logits) -------------------------
        for (int hh = 0; hh < H; ++hh) {
          const float* alp = sm_alpha + hh * SP;
          const float* dwh = sm_dw + hh * SP;
          const float a0 = lane < S ? alp[lane] : 0.f, a1 = lane + 32 < S ? alp[lane + 32] : 0.f;
          const float w0 = lane < S ? dwh[lane] : 0.f, w1 = lane + 32 < S ? dwh[lane + 32] : 0.f;
          const float wd = warp_sum(a0 * w0 + a1 * w1);
          const float dl0 = a0 * (w0 - wd), dl1 = a1 * (w1 - wd);
          if (lane < S) sm_logit[hh * SP + lane] = dl0;
          if (lane + 32 < S) sm_logit[hh * SP + lane + 32] = dl1;
          dbias0 += dl0;
          dbias1 += dl1;
        }
        __syncwarp();
        // ---- key phase 2: dK and dq -------------------------------------------
        float dqt[KE];
#pragma unroll
        for (int e = 0; e < KE; ++e) dqt[e] = 0.f;
        for (int r = 0; r < rounds; ++r) {
          const int seg = r * G + gidx;
          const int s = seg >> hshift;
          if (seg < SH) {
            const float c1 = sm_logit[kh * SP + s] * a.scale;
            const float kinv = sm_kinv[kh * SP + s];
            const float c2 = a.key_norm ? c1 * sm_qk[kh * SP + s] / dk : 0.f;
#pragma unroll
            for (int pk = 0; pk < KP; ++pk) {
              const Pack<T, VEC> kr = lds_pack<T, VEC>(kcopy + s * R + kcol + pk * VEC);
              float gk[VEC];
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                const float khat = Elem<T>::to_f(kr.e[e]) * kinv;
                const float g0 = c1 * q[pk * VEC + e];
                gk[e] = a.key_norm ? kinv * (g0 - khat * c2) : g0;
                dqt[pk * VEC + e] = fmaf(c1, khat, dqt[pk * VEC + e]);
              }
              store_pack<T, VEC>(sgk[s] + t * R + kcol + pk * VEC, gk);
            }
          }
        }
        if (a.qmode != ATTNRES_QUERY_STATIC) {
          float qd_now[KE];
          if (a.qmode == ATTNRES_QUERY_GATED) {
#pragma unroll
            for (int pk = 0; pk < KP; ++pk) {
              const Pack<T, VEC> qr = lds_pack<T, VEC>(qcopy + kcol + pk * VEC);
#pragma unroll
              for (int e = 0; e < VEC; ++e) qd_now[pk * VEC + e] = Elem<T>::to_f(qr.e[e]);
            }
          }
#pragma unroll
          for (int e = 0; e < KE; ++e) {
            if (a.qmode == ATTNRES_QUERY_GATED) {
              dq_acc[e] += dqt[e];
              dgate_acc = fmaf(dqt[e], qd_now[e], dgate_acc);
            }
            float v = dqt[e];
            for (int o = KL * H; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            dqt[e] = v;
          }
          if (gidx < H) {
            T* dqp = static_cast<T*>(a.dq_tok) + t * R + kcol;
#pragma unroll
            for (int pk = 0; pk < KP; ++pk) {
              float o8[VEC];
#pragma unroll
              for (int e = 0; e < VEC; ++e)
                o8[e] = (a.qmode == ATTNRES_QUERY_GATED) ? gate_k * dqt[pk * VEC + e] : dqt[pk * VEC + e];
              store_pack<T, VEC>(dqp + pk * VEC, o8);
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < KE; ++e) dq_acc[e] += dqt[e];
        }
        __syncwarp();
      }
    }
  }

  // On a wait timeout, let this warp's copies still in flight land first
  // (after a normal exit j == issued).
  for (long long i = j; i < issued; ++i, advance(cc))
    if (!mbar_wait_bounded(&wbars[cc.st], cc.ph))
      if (lane == 0) atomicOr(&g_warp_status, kStatusDrainTimeout);

  if (claim != nullptr && lane == 0) {
    // the last warp to finish rewinds the counter pair for the next launch
    __threadfence();
    const unsigned long long warps = static_cast<unsigned long long>(gridDim.x) * NW;
    if (atomicAdd(claim + 1, 1ull) == warps - 1) {
      atomicExch(claim, 0ull);
      atomicExch(claim + 1, 0ull);
    }
  }

  if constexpr (BWD) {
    // ---- fixed-order reduction of the parameter gradients -------------------
    if (a.partials == nullptr) return;
    const int PS = R + H + S;
#pragma unroll
    for (int e = 0; e < KE; ++e) {
      float v = dq_acc[e];
      for (int o = KL * H; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      dq_acc[e] = v;
    }
    float gsum = dgate_acc;
    for (int o = KL * H; o < 32; o <<= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, o);
    gsum = group_sum(gsum, KL);
    float* mine = ep + w * PS;
    if (gidx < H) {
#pragma unroll
      for (int e = 0; e < KE; ++e) mine[kcol + e] = dq_acc[e];
      if (kl == 0) mine[R + kh] = gsum;
    }
    if (lane < S) mine[R + H + lane] = dbias0;
    if (lane + 32 < S) mine[R + H + lane + 32] = dbias1;
    __syncthreads();
    float* row = a.partials + static_cast<long long>(blockIdx.x) * a.part_stride;
    for (int e = tid; e < PS; e += blockDim.x) {
      float s = 0.f;
      for (int ww = 0; ww < NW; ++ww) s += ep[ww * PS + e];
      row[e] = s;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using WarpFn = void (*)(LridArgs);

template <typename T, int KP, bool BWD>
static WarpFn pick_stream_s(int S) {
  if (S <= 16) return lrid_stream_kernel<T, KP, 16, BWD>;
  if (S <= 20) return lrid_stream_kernel<T, KP, 20, BWD>;
  if (S <= 24) return lrid_stream_kernel<T, KP, 24, BWD>;
  if (S <= 32) return lrid_stream_kernel<T, KP, 32, BWD>;
  return lrid_stream_kernel<T, KP, 64, BWD>;
}

template <typename T>
static WarpFn pick_stream_t(const LridPlan& p, const TmaLayout& L, bool bwd) {
  if (L.key_packs == 1) return bwd ? pick_stream_s<T, 1, true>(p.S) : pick_stream_s<T, 1, false>(p.S);
  return bwd ? pick_stream_s<T, 4, true>(p.S) : pick_stream_s<T, 4, false>(p.S);
}

static WarpFn pick_stream(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return pick_stream_t<float>(p, L, bwd);
    case ATTNRES_DTYPE_F16: return pick_stream_t<__half>(p, L, bwd);
    default: return pick_stream_t<__nv_bfloat16>(p, L, bwd);
  }
}

static int env_int_w(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

static bool pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Plan of the streaming kernels. Fields of TmaLayout used: stages (ring depth
// per warp), stage_bytes, stage_off (rings), off_y (per-warp scratch start),
// off_qd (per-warp scratch bytes), off_v (key-copy offset inside a warp's
// scratch), key_lanes, key_packs. Not used with output normalisation.
bool lrid_warp_plan(const LridPlan& base, int esz, bool bwd, bool has_y, bool has_qd, int out_norm,
                    TmaLayout* L, int* consumer_warps) {
  const int VEC = 16 / esz;
  const int CW = 32 * VEC;
  if (has_y || out_norm != ATTNRES_NORM_NONE) return false;
  if (base.vec != VEC || base.dv % CW) return false;
  if (!pow2(base.H) || base.dk % VEC) return false;
  const int kp = (base.dk <= 32 * VEC) ? 1 : 4;
  const int ke = kp * VEC;
  if (base.dk % ke) return false;
  const int kl = base.dk / ke;
  if (!pow2(kl) || kl > 32 || (32 / kl) % base.H) return false;
  int dev = 0, cap = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
  const size_t key_unit = static_cast<size_t>(base.S) * base.R * esz + (has_qd ? base.R * esz : 0);
  const size_t chunk_unit = static_cast<size_t>(base.S) * CW * esz + (bwd ? CW * esz : 0);
  const size_t sb = align_up(std::max(key_unit, chunk_unit), 128);
  const size_t kcopy_off = align_up(5 * static_cast<size_t>(base.H) * ((base.S + 3) & ~3) * sizeof(float), 16);
  const size_t wscr = align_up(kcopy_off + (bwd ? key_unit : 0), 128);
  const int nsw = std::max(2, std::min(kStreamMaxStages, env_int_w("ATTNRES_STREAM_STAGES", 2)));
  const int max_warps = bwd ? (base.S > 16 ? kStreamBwdWarpsManySources : kStreamBwdWarps) : 20;
  int nw = std::min(max_warps, std::max(1, env_int_w("ATTNRES_STREAM_WARPS", max_warps)));
  for (; nw >= 1; --nw) {
    size_t off = kStreamMaxWarps * kStreamMaxStages * (sizeof(uint64_t) + sizeof(long long)) +
                 6 * sizeof(void*) * base.S;
    off += sizeof(float) * static_cast<size_t>(nw) * (base.R + base.H + base.S);
    off = align_up(off, 128);
    const size_t wscr_off = off;
    off += nw * wscr;
    off = align_up(off, 128);
    const size_t total = off + static_cast<size_t>(nw) * nsw * sb;
    if (total <= static_cast<size_t>(cap)) {
      L->stages = nsw;
      L->stage_bytes = static_cast<int>(sb);
      L->stage_off = static_cast<int>(off);
      L->off_y = static_cast<int>(wscr_off);
      L->off_qd = static_cast<int>(wscr);
      L->off_v = static_cast<int>(kcopy_off);
      L->off_g = 0;
      L->smem_bytes = static_cast<int>(total);
      L->key_lanes = kl;
      L->key_packs = kp;
      *consumer_warps = nw;
      return nw >= 2;
    }
  }
  return false;
}

static cudaError_t stream_shape(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd, WarpFn* fn,
                                int* grid) {
  *fn = pick_stream(dtype, p, L, bwd);
  cudaError_t e = cudaFuncSetAttribute(*fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_bytes);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  *grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.N, nsm)));
  return cudaSuccess;
}

cudaError_t lrid_warp_workspace(int dtype, const LridPlan& p, const TmaLayout& L, int nw, size_t* bytes) {
  WarpFn fn;
  int grid = 0;
  (void)nw;
  cudaError_t e = stream_shape(dtype, p, L, true, &fn, &grid);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(float) * static_cast<size_t>(grid) * (p.R + p.H + p.S);
  return cudaSuccess;
}

static void fill_stream_common(LridArgs& a, const LridPlan& p, const TmaLayout& L, const LridIO& io) {
  a.p = p;
  a.tma = L;
  for (int s = 0; s < p.S; ++s) {
    a.v[s] = io.values[s];
    a.k[s] = io.keys[s];
    a.vs[s] = io.vstr[s];
    a.ks[s] = io.kstr[s];
  }
  a.qmode = io.qmode;
  a.q = io.q;
  a.gate = io.gate;
  a.qdyn = io.qdyn;
  a.scale = io.scale;
  a.key_norm = io.key_norm;
  a.key_eps = io.key_eps;
  a.bias = io.bias;
  a.out_norm = io.out_norm;
  a.out_eps = io.out_eps;
}

// Counter pairs of the dynamic token schedule, one per launch in a rotation of
// kClaimSlots (zero at module load; each launch leaves its pair at zero). A
// pair is reused kClaimSlots launches later, so launches on concurrent
// streams do not share a pair; a captured graph keeps the pair it was given,
// and replays of one graph are ordered.
constexpr int kClaimSlots = 64;
constexpr int kClaimMaxDevices = 64;
static __device__ unsigned long long g_claim[kClaimSlots * 2];

static cudaError_t claim_slot(unsigned long long** slot) {
  static std::atomic<unsigned long long*> base[kClaimMaxDevices];
  static std::atomic<unsigned> seq{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kClaimMaxDevices) return cudaErrorInvalidDevice;
  unsigned long long* b = base[dev].load();
  if (b == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_claim);
    if (e != cudaSuccess) return e;
    b = static_cast<unsigned long long*>(p);
    base[dev].store(b);
  }
  *slot = b + 2 * (seq.fetch_add(1) % kClaimSlots);
  return cudaSuccess;
}

static bool dynamic_schedule() {
  const char* v = getenv("ATTNRES_STREAM_SCHEDULE");
  return !(v && strcmp(v, "static") == 0);
}

cudaError_t lrid_warp_forward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                     const LridIO& io, cudaStream_t st) {
  LridArgs a{};
  fill_stream_common(a, p, L, io);
  a.out = io.out;
  a.alpha_out = io.alpha_out;
  a.kinv_out = io.kinv_out;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = stream_shape(dtype, p, L, false, &fn, &grid);
  if (e != cudaSuccess) return e;
  if (dynamic_schedule() && (e = claim_slot(&a.claim)) != cudaSuccess) return e;
  fn<<<grid, nw * 32, L.smem_bytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t lrid_warp_backward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                      const LridIO& io, const LridGradIO& gio, cudaStream_t st) {
  LridArgs a{};
  fill_stream_common(a, p, L, io);
  for (int s = 0; s < p.S; ++s) {
    a.gv[s] = gio.grad_values ? gio.grad_values[s] : nullptr;
    a.gk[s] = gio.grad_keys[s];
  }
  a.g = gio.grad_output;
  a.dq_tok = (io.qmode == ATTNRES_QUERY_DYNAMIC) ? gio.grad_query : gio.grad_query_dynamic;
  a.want_bias_grad = gio.grad_bias != nullptr;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = stream_shape(dtype, p, L, true, &fn, &grid);
  if (e != cudaSuccess) return e;
  const int stride = p.R + p.H + p.S;
  const bool need_partials = io.qmode != ATTNRES_QUERY_DYNAMIC || gio.grad_bias != nullptr;
  a.partials = need_partials ? static_cast<float*>(gio.workspace) : nullptr;
  a.part_stride = stride;
  fn<<<grid, nw * 32, L.smem_bytes, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || !need_partials) return e;
  if (io.qmode != ATTNRES_QUERY_DYNAMIC) {
    launch_reduce_partials(a.partials, grid, stride, 0, p.R, static_cast<float*>(gio.grad_query), st);
    if (io.qmode == ATTNRES_QUERY_GATED)
      launch_reduce_partials(a.partials, grid, stride, p.R, p.H, gio.grad_gate, st);
  }
  launch_reduce_partials(a.partials, grid, stride, p.R + p.H, p.S, gio.grad_bias, st);
  return cudaGetLastError();
}

cudaError_t read_warp_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_warp_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_warp_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
