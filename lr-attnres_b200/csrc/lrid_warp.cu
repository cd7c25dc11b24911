// LRID block Attention-Residual read, forward and backward: one warp per token
// row, fed by a bulk-copy (TMA) ring of single-token stages.
//
// Arithmetic and semantics are those of lrid.cu / lrid_tma.cu (fp32, the
// reference's _lrid_read_torch_list attnres_ops.py:4195-4232 and the backward
// of _lrid_attnres_list_backward_kernel attnres_ops.py:602-746). The layout:
//   * a persistent CTA per SM: one producer thread and NW consumer warps;
//   * token k of this CTA lands in stage k % NST of a shared-memory ring (its S
//     key rows, S value rows, and in the backward the upstream gradient, the
//     saved output and the per-token query), one cp.async.bulk per row;
//   * consumer warp w handles tokens k = w, w + NW, ...: logits, softmax over
//     sources, the weighted sum (forward) or dV / dw / dlogit / dK / dq
//     (backward) are all warp-local, so there is no CTA-wide barrier in the
//     token loop; the warp releases the stage with one mbarrier arrive.
// Row widths must split into 32-lane chunks per head: (d/H) % (32*VEC) == 0.
// Parameter gradients (static query, gate, logit bias) are summed per lane,
// then across lanes and warps in a fixed order into one partial row per CTA.
#include <algorithm>

#include "lrid_args.cuh"
#include "tma.cuh"

namespace attnres {

static __device__ unsigned int g_warp_status = 0;

constexpr int kWarpMaxStages = 16;

template <typename T, int KP, int SMAX, bool BWD>
__global__ void __launch_bounds__(288, 1) lrid_warp_kernel(const __grid_constant__ LridArgs a) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int KE = KP * VEC;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const LridPlan& P = a.p;
  const TmaLayout& L = a.tma;
  const int S = P.S, H = P.H, dk = P.dk, dv = P.dv, d = P.d, R = P.R;
  const int NST = L.stages;
  const int NW = (blockDim.x >> 5) - 1;  // consumer warps
  const int KL = L.key_lanes;
  const bool has_qd = a.qmode != ATTNRES_QUERY_STATIC;
  const bool has_y = BWD && a.out_norm != ATTNRES_NORM_NONE;
  const int SH = S * H;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kWarpMaxStages;
  const T** sv = reinterpret_cast<const T**>(empty + kWarpMaxStages);
  const T** sk = sv + S;
  long long* svs = reinterpret_cast<long long*>(sk + S);
  long long* sks = svs + S;
  T** sgv = reinterpret_cast<T**>(sks + S);
  T** sgk = sgv + S;
  float* fs = reinterpret_cast<float*>(sgk + S);
  // per-warp scratch: logit | alpha | kinv | qk | dw  (each [H][S])
  float* scratch = fs;
  float* ep_dq = fs + 5 * SH * NW;  // epilogue [NW][R]
  float* ep_gate = ep_dq + NW * R;  // [NW][H]
  float* ep_bias = ep_gate + NW * H;  // [NW][S]
  unsigned char* stage0 = smem_raw + L.stage_off;

  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
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

  // tokens of this CTA: t = blockIdx.x + k * gridDim.x
  const long long ntok_cta =
      (P.N > blockIdx.x) ? (P.N - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

  // ------------------------------------------------------------------------
  // producer
  // ------------------------------------------------------------------------
  const int NT = NW * 32;
  if (tid >= NT) {
    if (tid != NT) return;
    const T* gsrc = static_cast<const T*>(a.g);
    const T* ysrc = static_cast<const T*>(a.y);
    const T* qsrc = static_cast<const T*>(a.qdyn);
    const uint32_t bytes = static_cast<uint32_t>(sizeof(T)) *
                           (S * (R + d) + (BWD ? d : 0) + (has_y ? d : 0) + (has_qd ? R : 0));
    const uint32_t kb = R * sizeof(T), vb = d * sizeof(T);
    long long k = 0;
    bool ok = true;
    for (; k < ntok_cta; ++k) {
      const int st = static_cast<int>(k % NST);
      const uint32_t par = static_cast<uint32_t>((k / NST) & 1);
      if (!mbar_wait_bounded(&empty[st], par ^ 1u)) {
        atomicOr(&g_warp_status, kStatusEmptyWaitTimeout);
        ok = false;
        break;
      }
      const long long t = blockIdx.x + k * gridDim.x;
      mbar_arrive_expect_tx(&full[st], bytes);
      unsigned char* base = stage0 + static_cast<size_t>(st) * L.stage_bytes;
      for (int s = 0; s < S; ++s) {
        bulk_g2s(base + s * kb, sk[s] + t * sks[s], kb, &full[st]);
        bulk_g2s(base + L.off_v + s * vb, sv[s] + t * svs[s], vb, &full[st]);
      }
      if (BWD) bulk_g2s(base + L.off_g, gsrc + t * d, vb, &full[st]);
      if (has_y) bulk_g2s(base + L.off_y, ysrc + t * d, vb, &full[st]);
      if (has_qd) bulk_g2s(base + L.off_qd, qsrc + t * R, kb, &full[st]);
    }
    if (!ok) {
      for (long long j = (k > NST ? k - NST : 0); j < k; ++j)
        if (!mbar_wait_bounded(&full[j % NST], static_cast<uint32_t>((j / NST) & 1)))
          atomicOr(&g_warp_status, kStatusDrainTimeout);
    }
    return;
  }

  // ------------------------------------------------------------------------
  // consumer warps
  // ------------------------------------------------------------------------
  const int lane = tid & 31, w = tid >> 5;
  float* sm_logit = scratch + w * 5 * SH;
  float* sm_alpha = sm_logit + SH;
  float* sm_kinv = sm_alpha + SH;
  float* sm_qk = sm_kinv + SH;
  float* sm_dw = sm_qk + SH;
  const int G = 32 / KL;           // key groups per warp
  const int gidx = lane / KL, kl = lane % KL;
  const int kh = gidx % H;          // fixed head of this lane (G % H == 0)
  const int kcol = kh * dk + kl * KE;
  const int rounds = (SH + G - 1) / G;
  const int chunks = d / (32 * VEC);       // 32-lane chunks of a row
  const int chunks_per_head = dv / (32 * VEC);

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

  for (long long k = w; k < ntok_cta; k += NW) {
    const int st = static_cast<int>(k % NST);
    const uint32_t par = static_cast<uint32_t>((k / NST) & 1);
    const long long t = blockIdx.x + k * gridDim.x;
    float yinv = 0.f;
    if (has_y) yinv = (a.out_norm == ATTNRES_NORM_PER_HEAD) ? a.y_inv[t * H] : a.y_inv[t];
    if (!mbar_wait_bounded(&full[st], par)) {
      if (lane == 0) atomicOr(&g_warp_status, kStatusFullWaitTimeout);
      break;
    }
    const unsigned char* base = stage0 + static_cast<size_t>(st) * L.stage_bytes;
    const T* kt = reinterpret_cast<const T*>(base);              // [S][R]
    const T* vt = reinterpret_cast<const T*>(base + L.off_v);    // [S][d]
    const T* qdt = reinterpret_cast<const T*>(base + L.off_qd);  // [R]

    // per-lane query elements for this token
    float q[KE];
    {
      Pack<T, VEC> qr[KP];
      if (has_qd) {
#pragma unroll
        for (int pk = 0; pk < KP; ++pk) qr[pk] = lds_pack<T, VEC>(qdt + kcol + pk * VEC);
      }
#pragma unroll
      for (int pk = 0; pk < KP; ++pk)
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          float qv = qs[pk * VEC + e];
          if (has_qd) {
            const float qd = Elem<T>::to_f(qr[pk].e[e]);
            qv = (a.qmode == ATTNRES_QUERY_DYNAMIC) ? qd : qv + gate_k * qd;
          }
          q[pk * VEC + e] = qv;
        }
    }

    // ---- key phase: segments (s, h) over lane groups ----------------------
    for (int r = 0; r < rounds; ++r) {
      const int seg = r * G + gidx;  // seg = s * H + h, h == kh
      const int s = seg / H;
      float ss = 0.f, dot = 0.f;
      if (seg < SH) {
#pragma unroll
        for (int pk = 0; pk < KP; ++pk) {
          const Pack<T, VEC> kr = lds_pack<T, VEC>(kt + s * R + kcol + pk * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float x = Elem<T>::to_f(kr.e[e]);
            ss = fmaf(x, x, ss);
            dot = fmaf(x, q[pk * VEC + e], dot);
          }
        }
      }
      ss = group_sum(ss, KL);
      dot = group_sum(dot, KL);
      if (seg < SH && kl == 0) {
        const float kinv = a.key_norm ? rsqrtf(ss / dk + a.key_eps) : 1.f;
        const float qk = dot * kinv;
        sm_logit[kh * S + s] = qk * a.scale + (a.bias ? a.bias[s] : 0.f);
        sm_kinv[kh * S + s] = kinv;
        sm_qk[kh * S + s] = qk;
      }
    }
    __syncwarp();

    // ---- softmax over sources, per head --------------------------------------
    for (int h = 0; h < H; ++h) {
      const float* lg = sm_logit + h * S;
      float* alp = sm_alpha + h * S;
      const float l0 = lane < S ? lg[lane] : -INFINITY;
      const float l1 = lane + 32 < S ? lg[lane + 32] : -INFINITY;
      const float m = warp_max(fmaxf(l0, l1));
      const float e0 = lane < S ? expf(l0 - m) : 0.f;
      const float e1 = lane + 32 < S ? expf(l1 - m) : 0.f;
      const float sum = warp_sum(e0 + e1);
      if (lane < S) alp[lane] = e0 / sum;
      if (lane + 32 < S) alp[lane + 32] = e1 / sum;
      if (!BWD) {
        if (a.alpha_out) {
          if (lane < S) a.alpha_out[(t * H + h) * S + lane] = e0 / sum;
          if (lane + 32 < S) a.alpha_out[(t * H + h) * S + lane + 32] = e1 / sum;
        }
        if (a.kinv_out) {
          if (lane < S) a.kinv_out[(t * H + h) * S + lane] = sm_kinv[h * S + lane];
          if (lane + 32 < S) a.kinv_out[(t * H + h) * S + lane + 32] = sm_kinv[h * S + lane + 32];
        }
      }
    }
    __syncwarp();

    if constexpr (!BWD) {
      // ---- out = sum_s alpha_s V_s ------------------------------------------
      T* outp = static_cast<T*>(a.out) + t * d;
      const bool norm = a.out_norm != ATTNRES_NORM_NONE;
      float inv = 1.f;
      for (int pass = 0; pass < (norm ? 2 : 1); ++pass) {
        float ssq = 0.f;
        for (int c = 0; c < chunks; ++c) {
          const int col = (c * 32 + lane) * VEC;
          const float* al = sm_alpha + (c / chunks_per_head) * S;
          float acc[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
          int s = 0;
          for (; s + 4 <= S; s += 4) {
            Pack<T, VEC> r4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) r4[j] = lds_pack<T, VEC>(vt + (s + j) * d + col);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float wgt = al[s + j];
#pragma unroll
              for (int e = 0; e < VEC; ++e) acc[e] = fmaf(wgt, Elem<T>::to_f(r4[j].e[e]), acc[e]);
            }
          }
          for (; s < S; ++s) {
            const Pack<T, VEC> r1 = lds_pack<T, VEC>(vt + s * d + col);
            const float wgt = al[s];
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] = fmaf(wgt, Elem<T>::to_f(r1.e[e]), acc[e]);
          }
          if (norm && pass == 0) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) ssq = fmaf(acc[e], acc[e], ssq);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] *= inv;
            store_pack<T, VEC>(outp + col, acc);
          }
        }
        if (norm && pass == 0) {
          inv = rsqrtf(warp_sum(ssq) / d + a.out_eps);
          if (a.out_inv && lane == 0) a.out_inv[t] = inv;  // per-head with H == 1, or row
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    } else {
      const T* gt = reinterpret_cast<const T*>(base + L.off_g);
      const T* yt = reinterpret_cast<const T*>(base + L.off_y);
      // output-norm backward needs <g, y> over the row first
      float mdot = 0.f;
      if (has_y) {
        float gy = 0.f;
        for (int c = 0; c < chunks; ++c) {
          const int col = (c * 32 + lane) * VEC;
          const Pack<T, VEC> gr = lds_pack<T, VEC>(gt + col);
          const Pack<T, VEC> yr = lds_pack<T, VEC>(yt + col);
#pragma unroll
          for (int e = 0; e < VEC; ++e) gy = fmaf(Elem<T>::to_f(gr.e[e]), Elem<T>::to_f(yr.e[e]), gy);
        }
        mdot = warp_sum(gy) / d;
      }
      // ---- dV_s = alpha_s g', dw_s = <g', V_s> per head ----------------------
      for (int h = 0; h < H; ++h) {
        const float* al = sm_alpha + h * S;
        float dwp[SMAX];
#pragma unroll
        for (int s = 0; s < SMAX; ++s) dwp[s] = 0.f;
        for (int cc = 0; cc < chunks_per_head; ++cc) {
          const int col = ((h * chunks_per_head + cc) * 32 + lane) * VEC;
          float gp[VEC];
          const Pack<T, VEC> gr = lds_pack<T, VEC>(gt + col);
          if (has_y) {
            const Pack<T, VEC> yr = lds_pack<T, VEC>(yt + col);
#pragma unroll
            for (int e = 0; e < VEC; ++e)
              gp[e] = yinv * (Elem<T>::to_f(gr.e[e]) - Elem<T>::to_f(yr.e[e]) * mdot);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) gp[e] = Elem<T>::to_f(gr.e[e]);
          }
#pragma unroll
          for (int s0 = 0; s0 < SMAX; s0 += 4) {
            if (s0 < S) {
              Pack<T, VEC> r4[4];
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (s0 + j < S) r4[j] = lds_pack<T, VEC>(vt + (s0 + j) * d + col);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (s0 + j < S) {
                  const float wgt = al[s0 + j];
                  float gv[VEC];
#pragma unroll
                  for (int e = 0; e < VEC; ++e) {
                    dwp[s0 + j] = fmaf(gp[e], Elem<T>::to_f(r4[j].e[e]), dwp[s0 + j]);
                    gv[e] = wgt * gp[e];
                  }
                  store_pack<T, VEC>(sgv[s0 + j] + t * d + col, gv);
                }
              }
            }
          }
        }
#pragma unroll
        for (int s = 0; s < SMAX; ++s) {
          if (s < S) {
            const float dw = warp_sum(dwp[s]);
            if (lane == 0) sm_dw[h * S + s] = dw;
          }
        }
      }
      __syncwarp();
      // ---- dlogit per head (stored over the logits) ---------------------------
      for (int h = 0; h < H; ++h) {
        const float* alp = sm_alpha + h * S;
        const float* dwh = sm_dw + h * S;
        const float a0 = lane < S ? alp[lane] : 0.f, a1 = lane + 32 < S ? alp[lane + 32] : 0.f;
        const float w0 = lane < S ? dwh[lane] : 0.f, w1 = lane + 32 < S ? dwh[lane + 32] : 0.f;
        const float wd = warp_sum(a0 * w0 + a1 * w1);
        const float dl0 = a0 * (w0 - wd), dl1 = a1 * (w1 - wd);
        if (lane < S) sm_logit[h * S + lane] = dl0;
        if (lane + 32 < S) sm_logit[h * S + lane + 32] = dl1;
        dbias0 += dl0;
        dbias1 += dl1;
      }
      __syncwarp();
      // ---- key phase 2: dK and dq ------------------------------------------
      float dqt[KE];
#pragma unroll
      for (int e = 0; e < KE; ++e) dqt[e] = 0.f;
      for (int r = 0; r < rounds; ++r) {
        const int seg = r * G + gidx;
        const int s = seg / H;
        if (seg < SH) {
          const float c1 = sm_logit[kh * S + s] * a.scale;
          const float kinv = sm_kinv[kh * S + s];
          const float c2 = a.key_norm ? c1 * sm_qk[kh * S + s] / dk : 0.f;
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            const Pack<T, VEC> kr = lds_pack<T, VEC>(kt + s * R + kcol + pk * VEC);
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
      // per-token query gradient: sum this lane's partial over the groups that
      // share its head (xor over the group bits above the head bits)
      if (a.qmode != ATTNRES_QUERY_STATIC) {
        float qd_now[KE];
        if (a.qmode == ATTNRES_QUERY_GATED) {
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            const Pack<T, VEC> qr = lds_pack<T, VEC>(qdt + kcol + pk * VEC);
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
          float outv[KE];
#pragma unroll
          for (int e = 0; e < KE; ++e) outv[e] = (a.qmode == ATTNRES_QUERY_GATED) ? gate_k * dqt[e] : dqt[e];
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            float o8[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) o8[e] = outv[pk * VEC + e];
            store_pack<T, VEC>(dqp + pk * VEC, o8);
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < KE; ++e) dq_acc[e] += dqt[e];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }

  if constexpr (BWD) {
    // ---- fixed-order reduction of the parameter gradients -----------------
    if (a.partials == nullptr) return;
    // lanes -> one value per (head, key column): xor over the groups sharing a head
#pragma unroll
    for (int e = 0; e < KE; ++e) {
      float v = dq_acc[e];
      for (int o = KL * H; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      dq_acc[e] = v;
    }
    float gsum = dgate_acc;
    for (int o = KL * H; o < 32; o <<= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, o);
    gsum = group_sum(gsum, KL);
    if (gidx < H) {
#pragma unroll
      for (int e = 0; e < KE; ++e) ep_dq[w * R + kcol + e] = dq_acc[e];
      if (kl == 0) ep_gate[w * H + kh] = gsum;
    }
    if (lane < S) ep_bias[w * S + lane] = dbias0;
    if (lane + 32 < S) ep_bias[w * S + lane + 32] = dbias1;
    consumer_sync(NT);
    float* row = a.partials + static_cast<long long>(blockIdx.x) * a.part_stride;
    for (int e = tid; e < R; e += NT) {
      float s = 0.f;
      for (int ww = 0; ww < NW; ++ww) s += ep_dq[ww * R + e];
      row[e] = s;
    }
    for (int h = tid; h < H; h += NT) {
      float s = 0.f;
      for (int ww = 0; ww < NW; ++ww) s += ep_gate[ww * H + h];
      row[R + h] = s;
    }
    for (int s2 = tid; s2 < S; s2 += NT) {
      float s = 0.f;
      for (int ww = 0; ww < NW; ++ww) s += ep_bias[ww * S + s2];
      row[R + H + s2] = s;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using WarpFn = void (*)(LridArgs);

template <typename T, int KP, bool BWD>
static WarpFn pick_warp_s(int S) {
  if (S <= 16) return lrid_warp_kernel<T, KP, 16, BWD>;
  if (S <= 32) return lrid_warp_kernel<T, KP, 32, BWD>;
  return lrid_warp_kernel<T, KP, 64, BWD>;
}

template <typename T>
static WarpFn pick_warp_t(const LridPlan& p, const TmaLayout& L, bool bwd) {
  if (L.key_packs == 1) return bwd ? pick_warp_s<T, 1, true>(p.S) : pick_warp_s<T, 1, false>(p.S);
  return bwd ? pick_warp_s<T, 4, true>(p.S) : pick_warp_s<T, 4, false>(p.S);
}

static WarpFn pick_warp(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return pick_warp_t<float>(p, L, bwd);
    case ATTNRES_DTYPE_F16: return pick_warp_t<__half>(p, L, bwd);
    default: return pick_warp_t<__nv_bfloat16>(p, L, bwd);
  }
}

static int env_int_w(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

static bool pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }

bool lrid_warp_plan(const LridPlan& base, int esz, bool bwd, bool has_y, bool has_qd, int out_norm,
                    TmaLayout* L, int* consumer_warps) {
  const int VEC = 16 / esz;
  if (base.vec != VEC || base.dv % (32 * VEC)) return false;
  if (out_norm == ATTNRES_NORM_PER_HEAD && base.H != 1) return false;
  if (!pow2(base.H) || base.dk % VEC) return false;
  const int kp = (base.dk <= 32 * VEC) ? 1 : 4;
  const int ke = kp * VEC;
  if (base.dk % ke) return false;
  const int kl = base.dk / ke;
  if (!pow2(kl) || kl > 32 || (32 / kl) % base.H) return false;
  int dev = 0, cap = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
  int nw = env_int_w("ATTNRES_WARP_CONSUMERS", 8);
  nw = std::max(1, std::min(8, nw));
  const size_t SH = static_cast<size_t>(base.S) * base.H;
  size_t off = 2 * kWarpMaxStages * sizeof(uint64_t) + 6 * sizeof(void*) * base.S;
  off += sizeof(float) * (5 * SH * nw + static_cast<size_t>(nw) * (base.R + base.H + base.S));
  off = (off + 127) & ~static_cast<size_t>(127);
  size_t sb = static_cast<size_t>(base.S) * base.R * esz;
  const int off_v = static_cast<int>(sb);
  sb += static_cast<size_t>(base.S) * base.d * esz;
  const int off_g = static_cast<int>(sb);
  if (bwd) sb += static_cast<size_t>(base.d) * esz;
  const int off_y = static_cast<int>(sb);
  if (has_y) sb += static_cast<size_t>(base.d) * esz;
  const int off_qd = static_cast<int>(sb);
  if (has_qd) sb += static_cast<size_t>(base.R) * esz;
  sb = (sb + 127) & ~static_cast<size_t>(127);
  if (off + 2 * sb > static_cast<size_t>(cap)) return false;
  int stages = static_cast<int>((cap - off) / sb);
  stages = std::min(stages, std::min(kWarpMaxStages, env_int_w("ATTNRES_WARP_MAX_STAGES", kWarpMaxStages)));
  // A consumer warp may only wait on a stage whose previous occupant has been
  // filled, or the mbarrier parity would alias two phases: never more
  // consumer warps than stages.
  nw = std::min(nw, stages);
  L->stages = stages;
  L->stage_bytes = static_cast<int>(sb);
  L->off_v = off_v;
  L->off_g = off_g;
  L->off_y = off_y;
  L->off_qd = off_qd;
  L->stage_off = static_cast<int>(off);
  L->smem_bytes = static_cast<int>(off + stages * sb);
  L->key_lanes = kl;
  L->key_packs = kp;
  *consumer_warps = nw;
  return true;
}

static cudaError_t warp_shape(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd, int nw,
                              WarpFn* fn, int* grid) {
  *fn = pick_warp(dtype, p, L, bwd);
  cudaError_t e = cudaFuncSetAttribute(*fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_bytes);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  (void)nw;
  *grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.N, nsm)));
  return cudaSuccess;
}

cudaError_t lrid_warp_workspace(int dtype, const LridPlan& p, const TmaLayout& L, int nw, size_t* bytes) {
  WarpFn fn;
  int grid = 0;
  cudaError_t e = warp_shape(dtype, p, L, true, nw, &fn, &grid);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(float) * static_cast<size_t>(grid) * (p.R + p.H + p.S);
  return cudaSuccess;
}

static void fill_warp_common(LridArgs& a, const LridPlan& p, const TmaLayout& L, const LridIO& io) {
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

cudaError_t lrid_warp_forward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                     const LridIO& io, cudaStream_t st) {
  LridArgs a{};
  fill_warp_common(a, p, L, io);
  a.out = io.out;
  a.out_inv = io.out_inv;
  a.alpha_out = io.alpha_out;
  a.kinv_out = io.kinv_out;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = warp_shape(dtype, p, L, false, nw, &fn, &grid);
  if (e != cudaSuccess) return e;
  fn<<<grid, (nw + 1) * 32, L.smem_bytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t lrid_warp_backward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                      const LridIO& io, const LridGradIO& gio, cudaStream_t st) {
  LridArgs a{};
  fill_warp_common(a, p, L, io);
  for (int s = 0; s < p.S; ++s) {
    a.gv[s] = gio.grad_values[s];
    a.gk[s] = gio.grad_keys[s];
  }
  a.g = gio.grad_output;
  a.y = gio.normed_output;
  a.y_inv = gio.output_inv_rms;
  a.dq_tok = (io.qmode == ATTNRES_QUERY_DYNAMIC) ? gio.grad_query : gio.grad_query_dynamic;
  a.want_bias_grad = gio.grad_bias != nullptr;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = warp_shape(dtype, p, L, true, nw, &fn, &grid);
  if (e != cudaSuccess) return e;
  const int stride = p.R + p.H + p.S;
  const bool need_partials = io.qmode != ATTNRES_QUERY_DYNAMIC || gio.grad_bias != nullptr;
  a.partials = need_partials ? static_cast<float*>(gio.workspace) : nullptr;
  a.part_stride = stride;
  fn<<<grid, (nw + 1) * 32, L.smem_bytes, st>>>(a);
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
