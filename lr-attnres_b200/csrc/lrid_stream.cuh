// LRID block Attention-Residual read, forward and backward: self-fed warps
// streaming one token row at a time through a private bulk-copy ring (the
// kernel template; instantiated by lrid_stream_*.cu, launched by lrid_warp.cu).
//
// Arithmetic and semantics are those of lrid.cu (fp32, the
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
#pragma once

#include "lrid_args.cuh"
#include "tma.cuh"

namespace attnres {


// Status word of the streaming kernels (one copy per translation unit that
// instantiates them; read through the unit's stream_status_* function).
static __device__ unsigned int g_warp_status = 0;

constexpr int kStreamMaxWarps = 20;
constexpr int kStreamMaxStages = 4;

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Backward warps per CTA: up to 16, or 12 above 16 sources, where the larger
// per-source register arrays need more registers per thread (and shared memory
// holds no more warps' rings anyway). The forward runs 20 warps, or 16 with the
// output norm, which holds a token's output row in registers. NORM selects the
// output-norm variant in both directions.
constexpr int kStreamBwdWarps = 16;
constexpr int kStreamBwdWarpsManySources = 12;
constexpr int kStreamFwdWarps = 20;
// Output norm in the forward: the fp32 sums of one norm group (a row, or a
// head's slice of it), up to NORM 512-byte chunks per lane, stay in registers
// until the group's inverse rms is known; wider groups use the other kernel
// families. Fewer warps leave each thread the registers for them.
constexpr int kNormMaxChunks = 8;
constexpr int stream_fwd_warps(int norm_chunks) { return norm_chunks == 0 ? kStreamFwdWarps : norm_chunks <= 4 ? 16 : 12; }

template <bool BWD, int SMAX, int NORM>
constexpr int stream_threads() {
  return BWD ? (SMAX > 16 ? kStreamBwdWarpsManySources : kStreamBwdWarps) * 32 : stream_fwd_warps(NORM) * 32;
}

// NORM: forward, the register capacity for the output norm in 512-byte chunks
// (0 = no norm); backward, nonzero = with the output-norm backward.
template <typename T, int KP, int SMAX, bool BWD, int NORM>
__global__ void __launch_bounds__(stream_threads<BWD, SMAX, NORM>(), 1) lrid_stream_kernel(const __grid_constant__ LridArgs a) {
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
  // backward of the output norm: a per-token unit with the upstream-gradient
  // and normed-output rows precedes the value chunks (<g, y> per norm group)
  constexpr bool has_y = BWD && NORM != 0;
  const bool row_norm = a.out_norm == ATTNRES_NORM_ROW;
  const int SH = S * H;
  const int SP = (S + 3) & ~3;  // per-head row stride of the scratch arrays (16-byte rows)
  const int HSP = H * SP;
  const int C = d / CW, cph = dv / CW;
  constexpr int UY = has_y ? 1 : 0;  // units before the first value chunk, after the key unit
  const int U1 = C + 1 + UY;

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
  // nothing above touched global memory: from here on the previous launch's
  // results are needed
  pdl_wait_then_release();

  // per-warp scratch: logit | alpha | kinv | qk | dw (each [H][S] fp32) | norm
  // terms ([H] mean <g, y>, [H] inverse rms), then (backward) a copy of the
  // token's key rows [S][R] and query [R]
  float* sm_logit = reinterpret_cast<float*>(wscr0 + static_cast<size_t>(w) * L.off_qd);
  float* sm_alpha = sm_logit + HSP;
  float* sm_kinv = sm_alpha + HSP;
  float* sm_qk = sm_kinv + HSP;
  float* sm_dw = sm_qk + HSP;
  float* sm_nrm = sm_dw + HSP;
  T* kcopy = reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(sm_logit) + L.off_v);
  T* qcopy = kcopy + S * R;
  // backward with the output norm: the token's normalised upstream gradient
  // g' = inv_rms * (g - y * mean<g, y>) per norm group, rounded to T (as the
  // reference's PyTorch path holds it: the rms-norm backward returns a T
  // tensor), formed once per token from the g and y rows
  T* gscr = reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(sm_logit) + L.off_g);
  unsigned char* ring = stage0 + static_cast<size_t>(w) * NSW * L.stage_bytes;
  uint64_t* wbars = bars + w * NSW;
  const unsigned long long wait_ns = a.wait_ns;

  // Token schedule. Static: this warp takes tokens first, first + step, ...
  // Dynamic (a.dynamic_tokens): the warp takes the next unclaimed token from
  // the launch's counter each time its copy issue reaches a new token, so
  // warps on faster SMs take more tokens and all warps finish within about
  // one token.
  const long long N = P.N;
  const long long step = static_cast<long long>(NW) * gridDim.x;
  long long stat_next = blockIdx.x + static_cast<long long>(w) * gridDim.x;
  // Lane 0 keeps one claim in flight, so the atomic's round trip overlaps a
  // token's work instead of stalling the copy issue.
  unsigned long long* claim = a.dynamic_tokens ? a.sched : nullptr;
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
  const T* ysrc = static_cast<const T*>(a.y);
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
  const T* yrow = nullptr;  // this token's normed-output row (backward with output norm)
  long long issued = 0;
  const bool withhold_here = a.withhold >= 0 && blockIdx.x == 0 && w == 0;
  auto issue = [&](const Cursor& c) {
    const long long t = c.t;
    unsigned char* st = ring + static_cast<size_t>(c.st) * L.stage_bytes;
    uint64_t* bar = &wbars[c.st];
    const bool go = !(withhold_here && issued == a.withhold);
    if (c.u == 0) {
      const uint32_t kb = R * sizeof(T);
      if (lane == 0) mbar_arrive_expect_tx(bar, S * kb + (has_qd ? kb : 0));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const int s = lane + 32 * i;
        if (s < S) {
          if (go) bulk_g2s(st + s * kb, sk[s] + t * sks[s], kb, bar);
          vrow[i] = sv[s] + t * svs[s];
        }
      }
      if (go && has_qd && lane == (S & 31)) bulk_g2s(st + S * kb, qsrc + t * R, kb, bar);
      if (BWD) {
        grow = gsrc + t * d;
        if (has_y) yrow = ysrc + t * d;
      }
    } else if (c.u <= UY) {
      // full upstream-gradient and normed-output rows
      const uint32_t rb = d * sizeof(T);
      if (lane == 0) mbar_arrive_expect_tx(bar, 2 * rb);
      __syncwarp();
      if (go && lane == 0) bulk_g2s(st, grow, rb, bar);
      if (go && lane == 1) bulk_g2s(st + rb, yrow, rb, bar);
    } else {
      const int c0 = (c.u - 1 - UY) * CW;
      const uint32_t cb = CW * sizeof(T);
      if (lane == 0) mbar_arrive_expect_tx(bar, S * cb + ((BWD && !has_y) ? cb : 0));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const int s = lane + 32 * i;
        if (go && s < S) bulk_g2s(st + s * cb, vrow[i] + c0, cb, bar);
      }
      if (BWD && !has_y && go && lane == (S & 31)) bulk_g2s(st + S * cb, grow + c0, cb, bar);
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

  // Forward output norm: the fp32 output sums of the current norm group (a
  // row, or one head's slice) and this lane's running sum of their squares.
  constexpr int NB = (!BWD && NORM > 0) ? NORM : 1;
  float ybuf[NB][VEC];
  float ysq = 0.f;
  const int ngrp = row_norm ? C : cph;  // chunks per norm group
  const float nwidth = static_cast<float>(row_norm ? d : dv);
  float yinv_next = 0.f;  // backward: the token's saved inverse rms, loaded one unit early

  // Copy issue runs NSW - 1 units ahead of the consumer. Reaching a new token,
  // it records the token in the stage's slot; a token >= N ends the issue.
  Cursor pc{next_token(), 0, 0, 0u};  // next unit to issue
  bool issuing = true;
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
    if (!mbar_wait_bounded(&wbars[cc.st], cc.ph, wait_ns)) {
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
        if (has_y) {
          // consumed by the next unit; the load overlaps this unit's work
          const int nh = row_norm ? 1 : H;
          yinv_next = lane < nh ? __ldg(a.y_inv + t * nh + lane) : 0.f;
        }
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

    if (has_y && u <= UY) {
      // ---- output-norm backward terms: mean <g, y> per norm group ----------
      const T* gt = reinterpret_cast<const T*>(st);
      const T* yt = gt + d;
      const int ppl = dv / VEC;  // packs per head row
      float rowsum = 0.f;
      for (int h = 0; h < H; ++h) {
        float p = 0.f;
        for (int i = lane; i < ppl; i += 32) {
          const Pack<T, VEC> gr = lds_pack<T, VEC>(gt + h * dv + i * VEC);
          const Pack<T, VEC> yr = lds_pack<T, VEC>(yt + h * dv + i * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) p = fmaf(Elem<T>::to_f(gr.e[e]), Elem<T>::to_f(yr.e[e]), p);
        }
        p = warp_sum(p);
        rowsum += p;
        if (!row_norm && lane == 0) sm_nrm[h] = p / nwidth;
      }
      const float yi0 = __shfl_sync(0xffffffffu, yinv_next, 0);
      if (lane < H) {
        if (row_norm) {
          sm_nrm[lane] = rowsum / nwidth;
          sm_nrm[H + lane] = yi0;
        } else {
          sm_nrm[H + lane] = yinv_next;
        }
      }
      __syncwarp();
      // g' for the whole row; lane i writes packs i, i + 32, ..., the packs it
      // reads again in the value chunks
      for (int h = 0; h < H; ++h) {
        const float md = sm_nrm[h], yi = sm_nrm[H + h];
        for (int i = lane; i < ppl; i += 32) {
          const Pack<T, VEC> gr = lds_pack<T, VEC>(gt + h * dv + i * VEC);
          const Pack<T, VEC> yr = lds_pack<T, VEC>(yt + h * dv + i * VEC);
          float o[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = yi * (Elem<T>::to_f(gr.e[e]) - Elem<T>::to_f(yr.e[e]) * md);
          store_pack<T, VEC>(gscr + h * dv + i * VEC, o);
        }
      }
      __syncwarp();
      continue;
    }

    // ---- value chunk c of this token ----------------------------------------
    const int c = u - 1 - UY;
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
      if constexpr (NORM > 0) {
        // RMS norm of the fp32 read output over its group, rounded once, as
        // the reference's fused read kernel normalises its accumulator
        // (attnres_ops.py:435-439): kept until the group's last chunk.
#pragma unroll
        for (int e = 0; e < VEC; ++e) ysq = fmaf(acc[e], acc[e], ysq);
        const int gi = row_norm ? c : hcnt;
#pragma unroll
        for (int i = 0; i < NB; ++i)
          if (i == gi) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) ybuf[i][e] = acc[e];
          }
        if (gi == ngrp - 1) {
          const float inv = rsqrtf(warp_sum(ysq) / nwidth + a.out_eps);
          ysq = 0.f;
          T* orow = static_cast<T*>(a.out) + t * d + (row_norm ? 0 : h * dv) + lane * VEC;
#pragma unroll
          for (int i = 0; i < NB; ++i) {
            if (i < ngrp) {
              float o[VEC];
#pragma unroll
              for (int e = 0; e < VEC; ++e) o[e] = ybuf[i][e] * inv;
              store_pack<T, VEC>(orow + i * CW, o);
            }
          }
          if (a.out_inv && lane == 0) a.out_inv[row_norm ? t : t * H + h] = inv;
        }
      } else {
        store_pack<T, VEC>(static_cast<T*>(a.out) + t * d + col, acc);
      }
      if (++hcnt == cph) {
        hcnt = 0;
        ++hcur;
      }
    } else {
      float gp[VEC];
      // the upstream-gradient chunk, or with the output norm the token's g'
      Pack<T, VEC> gr;
      if constexpr (has_y) gr = lds_pack<T, VEC>(gscr + col);
      else gr = lds_pack<T, VEC>(reinterpret_cast<const T*>(st) + S * CW + lane * VEC);
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
              if constexpr (kIs16<T>) {
                dwp[s0 + jj] = dot_pack16<T, VEC>(dwp[s0 + jj], r4[jj], gr);
              } else {
                dwp[s0 + jj] = dot_pack<T, VEC>(dwp[s0 + jj], gp, r4[jj]);
              }
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
      if (c == C - 1) {
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
    if (!mbar_wait_bounded(&wbars[cc.st], cc.ph, wait_ns))
      if (lane == 0) atomicOr(&g_warp_status, kStatusDrainTimeout);

  if (claim != nullptr && lane == 0) {
    // the last warp to finish rewinds the counters for the slot's next launch
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


using WarpFn = void (*)(LridArgs);


// Instantiations, one translation unit each (built in parallel).
WarpFn stream_kernel_fwd(int dtype, int key_packs, int S, int norm_chunks);  // lrid_stream_fwd.cu
WarpFn stream_kernel_bwd_f32(int key_packs, int S, bool norm);          // lrid_stream_bwd_f32.cu
WarpFn stream_kernel_bwd_f16(int key_packs, int S, bool norm);          // lrid_stream_bwd_f16.cu
WarpFn stream_kernel_bwd_bf16(int key_packs, int S, bool norm);         // lrid_stream_bwd_bf16.cu
cudaError_t stream_status_fwd(unsigned* status, bool reset);
cudaError_t stream_status_bwd_f32(unsigned* status, bool reset);
cudaError_t stream_status_bwd_f16(unsigned* status, bool reset);
cudaError_t stream_status_bwd_bf16(unsigned* status, bool reset);

// Reads (and optionally clears) this translation unit's status word.
static inline cudaError_t read_stream_status_word(const void* symbol, unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, symbol, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(symbol, &zero, sizeof(unsigned));
}

}  // namespace attnres
