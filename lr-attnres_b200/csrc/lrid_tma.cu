// LRID block Attention-Residual read, forward and backward, with the source
// rows streamed into shared memory by the bulk-copy (TMA) engine.
//
// Same arithmetic as lrid.cu (fp32 throughout, reference semantics of
// _lrid_read_torch_list attnres_ops.py:4195-4232 and the backward formulas of
// _lrid_attnres_list_backward_kernel attnres_ops.py:602-746). What differs is
// the data movement:
//   * one producer warp (one elected thread) walks this CTA's token tiles and,
//     per tile, issues cp.async.bulk copies of every source's key and value
//     rows (plus the upstream gradient / saved output / per-token query) into a
//     ring of `stages` shared-memory buffers, completing on a per-stage
//     mbarrier (full). A source whose rows are dense moves as one copy per tile.
//   * `tpc * tpt` consumer threads wait on the full barrier, compute the read
//     from shared memory, write the outputs to global memory with 16-byte
//     stores, and release the stage (empty barrier, one arrive per warp).
// So the HBM reads of the next stages are in flight while a tile is computed,
// and no thread ever waits on a global load in the critical path.
// Every mbarrier wait is bounded (~2 s); on timeout the kernel records a bit in
// the device status word and returns.
#include <algorithm>

#include "lrid_args.cuh"
#include "tma.cuh"

namespace attnres {

// Device status word of this library (bits: DeviceStatusBits).
static __device__ unsigned int g_device_status = 0;

constexpr int kMaxStages = 8;

template <typename T>
__device__ __forceinline__ void copy_rows(T* dst, const T* src, long long stride, int width, int nrows,
                                          uint64_t* bar) {
  const uint32_t row_bytes = static_cast<uint32_t>(width) * sizeof(T);
  if (stride == width) {
    bulk_g2s(dst, src, row_bytes * nrows, bar);
  } else {
    for (int r = 0; r < nrows; ++r) bulk_g2s(dst + r * width, src + r * stride, row_bytes, bar);
  }
}

// Group sum over consumer threads (see block_group_sum in lrid.cu); the
// barrier is the consumers' named barrier, not __syncthreads.
__device__ __forceinline__ float consumer_group_sum(float v, int gsz, float* red, int nthreads) {
  if (gsz <= 32) return group_sum(v, gsz);
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  consumer_sync(nthreads);
  const int nw = gsz >> 5;
  const int w0 = (threadIdx.x / gsz) * nw;
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w0 + w];
  consumer_sync(nthreads);
  return tot;
}

// Key-segment work of one tile: a segment is one (token slot, source, head)
// key row slice of dk elements, handled by a group of `key_lanes` lanes that
// each own `KP * VEC` consecutive elements (16-byte shared loads). All
// consumer warps share the segments, so the logits of a tile take one or two
// short rounds instead of a serial loop per token.
template <typename T, int KP, bool BWD>
__global__ void __launch_bounds__(288, 2) lrid_tma_kernel(const __grid_constant__ LridArgs a) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int KE = KP * VEC;  // key elements per lane
  constexpr int MAXP = 4;       // (token, key column) pairs per thread in the dq reduction
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const LridPlan& P = a.p;
  const TmaLayout& L = a.tma;
  const int S = P.S, H = P.H, dk = P.dk, dv = P.dv, d = P.d, R = P.R;
  const int tpt = P.tpt, tpc = P.tpc, tph = P.tph;
  const int nvh = P.nvh, wph = P.wph;
  const int NT = tpc * tpt;
  const int STAGES = L.stages;
  const int KL = L.key_lanes;
  const bool has_qd = a.qmode != ATTNRES_QUERY_STATIC;
  const bool has_y = BWD && a.out_norm != ATTNRES_NORM_NONE;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kMaxStages;
  const T** sv = reinterpret_cast<const T**>(empty + kMaxStages);
  const T** sk = sv + S;
  long long* svs = reinterpret_cast<long long*>(sk + S);
  long long* sks = svs + S;
  T** sgv = reinterpret_cast<T**>(sks + S);
  T** sgk = sgv + S;
  float* fs = reinterpret_cast<float*>(sgk + S);
  const int A = tpc * H * S;
  float* sm_logit = fs;           // logits, then dlogits (backward)
  float* sm_alpha = fs + A;
  float* sm_kinv = fs + 2 * A;
  float* sm_qk = fs + 3 * A;      // <q, khat>
  float* sm_dwp = fs + 4 * A;     // backward: per-warp partial <g', v_s>
  float* sm_red = sm_dwp + A * wph;
  float* sm_dqc = sm_red + (NT >> 5);        // backward: [tpc][S][R] dq contributions
  float* sm_dqe = sm_dqc + tpc * S * R;      // [tpc * R] epilogue
  unsigned char* stage0 = smem_raw + L.stage_off;

  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NT >> 5);
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

  // ------------------------------------------------------------------------
  // producer: one thread of the last warp
  // ------------------------------------------------------------------------
  if (tid >= NT) {
    if (tid != NT) return;
    const T* gsrc = static_cast<const T*>(a.g);
    const T* ysrc = static_cast<const T*>(a.y);
    const T* qsrc = static_cast<const T*>(a.qdyn);
    const uint32_t per_row = static_cast<uint32_t>(sizeof(T)) *
                             (S * (R + d) + (BWD ? d : 0) + (has_y ? d : 0) + (has_qd ? R : 0));
    int k = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; tile < P.ntiles; tile += gridDim.x, ++k) {
      const int st = k % STAGES;
      const uint32_t par = (k / STAGES) & 1;
      if (!mbar_wait_bounded(&empty[st], par ^ 1u)) {
        atomicOr(&g_device_status, kStatusEmptyWaitTimeout);
        ok = false;
        break;
      }
      const long long t0 = tile * tpc;
      const int nr = static_cast<int>(min(static_cast<long long>(tpc), P.N - t0));
      mbar_arrive_expect_tx(&full[st], per_row * nr);
      unsigned char* base = stage0 + static_cast<size_t>(st) * L.stage_bytes;
      T* kdst = reinterpret_cast<T*>(base);
      T* vdst = reinterpret_cast<T*>(base + L.off_v);
      for (int s = 0; s < S; ++s) {
        copy_rows(kdst + s * tpc * R, sk[s] + t0 * sks[s], sks[s], R, nr, &full[st]);
        copy_rows(vdst + s * tpc * d, sv[s] + t0 * svs[s], svs[s], d, nr, &full[st]);
      }
      if (BWD) copy_rows(reinterpret_cast<T*>(base + L.off_g), gsrc + t0 * d, d, d, nr, &full[st]);
      if (has_y) copy_rows(reinterpret_cast<T*>(base + L.off_y), ysrc + t0 * d, d, d, nr, &full[st]);
      if (has_qd) copy_rows(reinterpret_cast<T*>(base + L.off_qd), qsrc + t0 * R, R, R, nr, &full[st]);
    }
    if (!ok) {
      // make sure no copy issued by this CTA is still landing when it exits
      for (int j = max(0, k - STAGES); j < k; ++j)
        if (!mbar_wait_bounded(&full[j % STAGES], (j / STAGES) & 1))
          atomicOr(&g_device_status, kStatusDrainTimeout);
    }
    return;
  }

  // ------------------------------------------------------------------------
  // consumers
  // ------------------------------------------------------------------------
  const int lane = tid & 31, warp = tid >> 5, nwarps = NT >> 5;
  const int slot = tid / tpt, it = tid % tpt;
  const int vh = it / tph, vj = it % tph;
  const bool vvalid = vh < H && vj < nvh;
  const int hgrp = P.out_norm_group;
  const int width = (a.out_norm == ATTNRES_NORM_ROW) ? d : dv;
  const int col = (vvalid ? vh * dv + vj * VEC : 0);
  // key-segment mapping (fixed head per thread: the group count is a multiple of H)
  const int ngroups = NT / KL;
  const int grp = tid / KL, kl = tid % KL;
  const int kh = grp % H;
  const int kcol = kh * dk + kl * KE;        // first key column of this lane
  const bool klane = kl * KE < dk;
  const int nseg = tpc * S * H;
  const int rounds = (nseg + ngroups - 1) / ngroups;

  float qs[KE];
  {
    const T* qp = static_cast<const T*>(a.q);
#pragma unroll
    for (int e = 0; e < KE; ++e)
      qs[e] = (a.qmode != ATTNRES_QUERY_DYNAMIC && klane) ? load_f(qp + kcol + e) : 0.f;
  }
  const float gate_k = (a.qmode == ATTNRES_QUERY_GATED) ? load_f(static_cast<const T*>(a.gate) + kh) : 0.f;
  // backward accumulators for the (token slot, key column) pairs this thread reduces
  float dq_acc[MAXP], dgate_acc[MAXP];
#pragma unroll
  for (int i = 0; i < MAXP; ++i) dq_acc[i] = dgate_acc[i] = 0.f;
  float dbias_acc = 0.f;

  int k = 0;
  for (long long tile = blockIdx.x; tile < P.ntiles; tile += gridDim.x, ++k) {
    const int st = k % STAGES;
    const uint32_t par = (k / STAGES) & 1;
    const long long t = tile * tpc + slot;
    const bool tv = t < P.N;
    float yinv = 0.f;
    if (has_y && tv && vh < H)
      yinv = (a.out_norm == ATTNRES_NORM_PER_HEAD) ? a.y_inv[t * H + vh] : a.y_inv[t];

    const bool landed = mbar_wait_bounded(&full[st], par);
    if constexpr (BWD) {
      if (consumer_sync_or(NT, !landed)) {
        if (tid == 0) atomicOr(&g_device_status, kStatusFullWaitTimeout);
        break;
      }
    }
    // forward: logits / key inv-rms double-buffered by tile parity, so the
    // key-phase barrier is the only CTA barrier of a tile
    float* lg_t = BWD ? sm_logit : sm_logit + (k & 1) * A;
    float* ki_t = BWD ? sm_kinv : fs + 2 * A + (k & 1) * A;
    const unsigned char* base = stage0 + static_cast<size_t>(st) * L.stage_bytes;
    const T* kt = reinterpret_cast<const T*>(base);                       // [S][tpc][R]
    const T* vt = reinterpret_cast<const T*>(base + L.off_v) + slot * d;  // + s*tpc*d
    const T* qdt = reinterpret_cast<const T*>(base + L.off_qd);           // [tpc][R]

    // ---- key phase: key rms-norm and logits, all warps -----------------
    for (int r = 0; r < rounds; ++r) {
      const int seg = grp + r * ngroups;
      const int sl = seg / (S * H);
      const int s = (seg / H) % S;
      const bool ok = landed && seg < nseg && tile * tpc + sl < P.N && klane;
      float ss = 0.f, dot = 0.f;
      if (ok) {
        const T* kp = kt + (s * tpc + sl) * R + kcol;
#pragma unroll
        for (int pk = 0; pk < KP; ++pk) {
          const Pack<T, VEC> kr = lds_pack<T, VEC>(kp + pk * VEC);
          Pack<T, VEC> qr;
          if (has_qd) qr = lds_pack<T, VEC>(qdt + sl * R + kcol + pk * VEC);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const float x = Elem<T>::to_f(kr.e[e]);
            float qv = qs[pk * VEC + e];
            if (has_qd) {
              const float qd = Elem<T>::to_f(qr.e[e]);
              qv = (a.qmode == ATTNRES_QUERY_DYNAMIC) ? qd : qv + gate_k * qd;
            }
            ss = fmaf(x, x, ss);
            dot = fmaf(x, qv, dot);
          }
        }
      }
      ss = group_sum(ss, KL);
      dot = group_sum(dot, KL);
      if (seg < nseg && kl == 0) {
        const float kinv = a.key_norm ? rsqrtf(ss / dk + a.key_eps) : 1.f;
        const float qk = dot * kinv;
        const int idx = (sl * H + kh) * S + s;
        lg_t[idx] = qk * a.scale + (a.bias ? a.bias[s] : 0.f);
        ki_t[idx] = kinv;
        if (BWD) sm_qk[idx] = qk;
      }
    }
    if constexpr (BWD) {
      consumer_sync(NT);
    } else {
      if (consumer_sync_or(NT, !landed)) {
        if (tid == 0) atomicOr(&g_device_status, kStatusFullWaitTimeout);
        break;
      }
    }

    // ---- softmax over sources ---------------------------------------------
    // forward: every warp computes the softmax of its own token into private
    // scratch (no barrier); backward: one warp per (token, head), shared.
    const float* al;
    if constexpr (!BWD) {
      float* wal = sm_red + (NT >> 5) + warp * H * S;  // after the reduction slots
      const int ws = (warp * 32) / tpt;  // token slot of this warp
      const long long tw = tile * tpc + ws;
      // heads read by this warp's value threads (one head when tph >= 32)
      const int it0 = (warp * 32) % tpt;
      const int h_lo = it0 / tph;
      const int h_hi = min(H - 1, (it0 + 31) / tph);
      for (int h = h_lo; h <= h_hi; ++h) {
        const bool writer = h * tph >= it0 && h * tph < it0 + 32;  // warp holding the head's first thread
        const float* lg = lg_t + (ws * H + h) * S;
        const float l0 = lane < S ? lg[lane] : -INFINITY;
        const float l1 = lane + 32 < S ? lg[lane + 32] : -INFINITY;
        const float m = warp_max(fmaxf(l0, l1));
        const float e0 = lane < S ? expf(l0 - m) : 0.f;
        const float e1 = lane + 32 < S ? expf(l1 - m) : 0.f;
        const float sum = warp_sum(e0 + e1);
        if (lane < S) wal[h * S + lane] = e0 / sum;
        if (lane + 32 < S) wal[h * S + lane + 32] = e1 / sum;
        if (writer && tw < P.N) {
          const float* kv = ki_t + (ws * H + h) * S;
          for (int s = lane; s < S; s += 32) {
            if (a.alpha_out) a.alpha_out[(tw * H + h) * S + s] = s < 32 ? e0 / sum : e1 / sum;
            if (a.kinv_out) a.kinv_out[(tw * H + h) * S + s] = kv[s];
          }
        }
      }
      __syncwarp();
      al = wal + (vh < H ? vh : 0) * S;
    } else {
    for (int pair = warp; pair < tpc * H; pair += nwarps) {
      const int b = pair * S;
      const long long tp = tile * tpc + pair / H;
      const int h = pair % H;
      float m = -INFINITY;
      for (int s = lane; s < S; s += 32) m = fmaxf(m, sm_logit[b + s]);
      m = warp_max(m);
      float sum = 0.f;
      for (int s = lane; s < S; s += 32) {
        const float e = expf(sm_logit[b + s] - m);
        sm_alpha[b + s] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      for (int s = lane; s < S; s += 32) {
        const float al = sm_alpha[b + s] / sum;
        sm_alpha[b + s] = al;
        if (!BWD && tp < P.N) {
          if (a.alpha_out) a.alpha_out[(tp * H + h) * S + s] = al;
          if (a.kinv_out) a.kinv_out[(tp * H + h) * S + s] = sm_kinv[b + s];
        }
      }
    }
    consumer_sync(NT);
    al = sm_alpha + (slot * H + (vh < H ? vh : 0)) * S;
    }

    if constexpr (!BWD) {
      // ---- out = sum_s alpha_s V_s (shared -> registers -> global) ---------
      float acc[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
      if (vvalid && tv) {
        int s = 0;
        for (; s + 4 <= S; s += 4) {
          Pack<T, VEC> r[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) r[j] = lds_pack<T, VEC>(vt + (s + j) * tpc * d + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float w = al[s + j];
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] = fmaf(w, Elem<T>::to_f(r[j].e[e]), acc[e]);
          }
        }
        for (; s < S; ++s) {
          const Pack<T, VEC> r = lds_pack<T, VEC>(vt + s * tpc * d + col);
          const float w = al[s];
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] = fmaf(w, Elem<T>::to_f(r.e[e]), acc[e]);
        }
      }
      // this warp is done with the stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      T* outp = static_cast<T*>(a.out);
      if (a.out_norm == ATTNRES_NORM_NONE) {
        if (vvalid && tv) store_pack<T, VEC>(outp + t * d + col, acc);
      } else {
        float ssq = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) ssq = fmaf(acc[e], acc[e], ssq);
        const float tot = consumer_group_sum((vvalid && tv) ? ssq : 0.f, hgrp, sm_red, NT);
        const float inv = rsqrtf(tot / width + a.out_eps);
        if (vvalid && tv) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] *= inv;
          store_pack<T, VEC>(outp + t * d + col, acc);
        }
        if (a.out_inv && tv && vh < H && vj == 0) {
          if (a.out_norm == ATTNRES_NORM_PER_HEAD) a.out_inv[t * H + vh] = inv;
          else if (vh == 0) a.out_inv[t] = inv;
        }
      }
    } else {
      // ---- backward: g' (output-norm backward), dV_s = alpha_s g', dw_s ----
      const T* gt = reinterpret_cast<const T*>(base + L.off_g) + slot * d;
      float gp[VEC], yv[VEC];
      float gy = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) gp[e] = yv[e] = 0.f;
      if (vvalid && tv) {
        const Pack<T, VEC> gr = lds_pack<T, VEC>(gt + col);
#pragma unroll
        for (int e = 0; e < VEC; ++e) gp[e] = Elem<T>::to_f(gr.e[e]);
        if (has_y) {
          const T* yt = reinterpret_cast<const T*>(base + L.off_y) + slot * d;
          const Pack<T, VEC> yr = lds_pack<T, VEC>(yt + col);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            yv[e] = Elem<T>::to_f(yr.e[e]);
            gy = fmaf(gp[e], yv[e], gy);
          }
        }
      }
      if (has_y) {
        const float tot = consumer_group_sum(gy, hgrp, sm_red, NT);
        const float mdot = tot / width;
#pragma unroll
        for (int e = 0; e < VEC; ++e) gp[e] = yinv * (gp[e] - yv[e] * mdot);
      }
      const int rg = tph < 32 ? tph : 32;
      for (int s0 = 0; s0 < S; s0 += 4) {
        Pack<T, VEC> r[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (s0 + j < S && vvalid && tv) r[j] = lds_pack<T, VEC>(vt + (s0 + j) * tpc * d + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (s0 + j < S) {
            const int s = s0 + j;
            float dwp = 0.f;
            if (vvalid && tv) {
              const float w = al[s];
              float gvv[VEC];
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                dwp = fmaf(gp[e], Elem<T>::to_f(r[j].e[e]), dwp);
                gvv[e] = w * gp[e];
              }
              if (sgv[s]) store_pack<T, VEC>(sgv[s] + t * d + col, gvv);
            }
            dwp = group_sum(dwp, rg);
            if ((vj & 31) == 0 && vh < H) sm_dwp[((slot * H + vh) * S + s) * wph + (vj >> 5)] = dwp;
          }
        }
      }
      consumer_sync(NT);

      // ---- dlogit_s = alpha_s (dw_s - sum_r alpha_r dw_r) -------------------
      for (int pair = warp; pair < tpc * H; pair += nwarps) {
        const int b = pair * S;
        const long long tp = tile * tpc + pair / H;
        float part = 0.f;
        for (int s = lane; s < S; s += 32) {
          float dw = 0.f;
          for (int w = 0; w < wph; ++w) dw += sm_dwp[(b + s) * wph + w];
          sm_dwp[(b + s) * wph] = dw;
          part = fmaf(sm_alpha[b + s], dw, part);
        }
        const float wd = warp_sum(part);
        for (int s = lane; s < S; s += 32)
          sm_logit[b + s] = (tp < P.N) ? sm_alpha[b + s] * (sm_dwp[(b + s) * wph] - wd) : 0.f;
      }
      consumer_sync(NT);
      if (a.want_bias_grad && tid < S)
        for (int pair = 0; pair < tpc * H; ++pair) dbias_acc += sm_logit[pair * S + tid];

      // ---- key phase 2: dK (global) and dq contributions (shared) -----------
      for (int r = 0; r < rounds; ++r) {
        const int seg = grp + r * ngroups;
        const int sl = seg / (S * H);
        const int s = (seg / H) % S;
        const long long ts = tile * tpc + sl;
        if (seg < nseg && ts < P.N && klane) {
          const int idx = (sl * H + kh) * S + s;
          const float c1 = sm_logit[idx] * a.scale;
          const float kinv = sm_kinv[idx];
          const float c2 = a.key_norm ? c1 * sm_qk[idx] / dk : 0.f;
          const T* kp = kt + (s * tpc + sl) * R + kcol;
          float* dqc = sm_dqc + (sl * S + s) * R + kcol;
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            const Pack<T, VEC> kr = lds_pack<T, VEC>(kp + pk * VEC);
            Pack<T, VEC> qr;
            if (has_qd) qr = lds_pack<T, VEC>(qdt + sl * R + kcol + pk * VEC);
            float gk[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              float qv = qs[pk * VEC + e];
              if (has_qd) {
                const float qd = Elem<T>::to_f(qr.e[e]);
                qv = (a.qmode == ATTNRES_QUERY_DYNAMIC) ? qd : qv + gate_k * qd;
              }
              const float khat = Elem<T>::to_f(kr.e[e]) * kinv;
              const float g0 = c1 * qv;
              gk[e] = a.key_norm ? kinv * (g0 - khat * c2) : g0;
              dqc[pk * VEC + e] = c1 * khat;
            }
            store_pack<T, VEC>(sgk[s] + ts * R + kcol + pk * VEC, gk);
          }
        }
      }
      consumer_sync(NT);

      // ---- dq: sum the contributions over sources in a fixed order ----------
      T* dqp = static_cast<T*>(a.dq_tok);
#pragma unroll
      for (int i = 0; i < MAXP; ++i) {
        const int pidx = tid + i * NT;
        if (pidx < tpc * R) {
          const int sl = pidx / R, e = pidx % R;
          const long long ts = tile * tpc + sl;
          if (ts < P.N) {
            float dq = 0.f;
            for (int s = 0; s < S; ++s) dq += sm_dqc[(sl * S + s) * R + e];
            if (a.qmode == ATTNRES_QUERY_STATIC) {
              dq_acc[i] += dq;
            } else if (a.qmode == ATTNRES_QUERY_DYNAMIC) {
              dqp[ts * R + e] = Elem<T>::from_f(dq);
            } else {
              const int h = e / dk;
              const float gte = load_f(static_cast<const T*>(a.gate) + h);
              const float qd = Elem<T>::to_f(qdt[sl * R + e]);
              dqp[ts * R + e] = Elem<T>::from_f(gte * dq);
              dq_acc[i] += dq;
              dgate_acc[i] = fmaf(dq, qd, dgate_acc[i]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      consumer_sync(NT);
    }
  }

  if constexpr (BWD) {
    // ---- per-CTA partial sums of the parameter gradients, fixed order -------
    if (a.partials == nullptr) return;
    float* gsm = sm_dqc;  // reuse: [tpc * R] dgate partials
#pragma unroll
    for (int i = 0; i < MAXP; ++i) {
      const int pidx = tid + i * NT;
      if (pidx < tpc * R) {
        sm_dqe[pidx] = dq_acc[i];
        gsm[pidx] = dgate_acc[i];
      }
    }
    consumer_sync(NT);
    float* row = a.partials + static_cast<long long>(blockIdx.x) * a.part_stride;
    for (int e = tid; e < R; e += NT) {
      float s = 0.f;
      for (int sl = 0; sl < tpc; ++sl) s += sm_dqe[sl * R + e];
      row[e] = s;
    }
    for (int h = tid; h < H; h += NT) {
      float s = 0.f;
      for (int sl = 0; sl < tpc; ++sl)
        for (int e = h * dk; e < (h + 1) * dk; ++e) s += gsm[sl * R + e];
      row[R + h] = s;
    }
    if (tid < S) row[R + H + tid] = dbias_acc;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using TmaFn = void (*)(LridArgs);

template <typename T>
static TmaFn pick_tma_t(const TmaLayout& L, bool bwd) {
  if (L.key_packs == 1) return bwd ? lrid_tma_kernel<T, 1, true> : lrid_tma_kernel<T, 1, false>;
  return bwd ? lrid_tma_kernel<T, 4, true> : lrid_tma_kernel<T, 4, false>;
}

static TmaFn pick_tma(int dtype, const TmaLayout& L, bool bwd) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return pick_tma_t<float>(L, bwd);
    case ATTNRES_DTYPE_F16: return pick_tma_t<__half>(L, bwd);
    default: return pick_tma_t<__nv_bfloat16>(L, bwd);
  }
}

static int max_smem_optin() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
  return v;
}

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

static bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }

// Pipeline plan for the bulk-copy kernels: token rows per tile, key-lane
// mapping and the shared-memory ring. False when the geometry is outside what
// these kernels handle (the caller then uses the register-streaming kernels).
bool lrid_tma_plan(const LridPlan& base, int esz, bool bwd, bool has_y, bool has_qd, LridPlan* out,
                   TmaLayout* L) {
  const int VEC = 16 / esz;
  if (base.vec != VEC || base.cph != 1 || base.tpt > 256) return false;
  if (!is_pow2(base.H) || base.dk % VEC) return false;
  const int kp = (base.dk <= 32 * VEC) ? 1 : 4;
  const int ke = kp * VEC;
  if (base.dk % ke) return false;
  const int kl = base.dk / ke;
  if (!is_pow2(kl) || kl > 32) return false;
  LridPlan p = base;
  int tpc = 256 / p.tpt;
  const int want = env_int("ATTNRES_TMA_TPC", 0);
  if (want > 0 && want <= tpc && is_pow2(want)) tpc = want;
  p.tpc = tpc;
  p.ntiles = (p.N + tpc - 1) / tpc;
  const int NT = tpc * p.tpt;
  if ((NT / kl) % p.H) return false;
  if (tpc * p.R > 4 * NT) return false;
  size_t off = 0;
  off += 2 * kMaxStages * sizeof(uint64_t);
  off += 6 * sizeof(void*) * p.S;
  const size_t A = static_cast<size_t>(tpc) * p.H * p.S;
  off += sizeof(float) * (4 * A + A * p.wph + NT / 32);
  if (bwd) off += sizeof(float) * (static_cast<size_t>(tpc) * p.S * p.R + static_cast<size_t>(tpc) * p.R);
  else off += sizeof(float) * (static_cast<size_t>(NT / 32) * p.H * p.S);  // per-warp softmax
  off = (off + 127) & ~static_cast<size_t>(127);
  size_t sb = static_cast<size_t>(p.S) * tpc * p.R * esz;
  const int off_v = static_cast<int>(sb);
  sb += static_cast<size_t>(p.S) * tpc * p.d * esz;
  const int off_g = static_cast<int>(sb);
  if (bwd) sb += static_cast<size_t>(tpc) * p.d * esz;
  const int off_y = static_cast<int>(sb);
  if (has_y) sb += static_cast<size_t>(tpc) * p.d * esz;
  const int off_qd = static_cast<int>(sb);
  if (has_qd) sb += static_cast<size_t>(tpc) * p.R * esz;
  sb = (sb + 127) & ~static_cast<size_t>(127);
  const size_t cap = static_cast<size_t>(max_smem_optin());
  if (cap == 0 || off + 2 * sb > cap) return false;
  // Shared memory is split between `ctas` co-resident CTAs per SM (each keeps
  // at least two stages); each CTA takes as deep a ring as its share allows.
  int ctas = env_int("ATTNRES_TMA_CTAS", 2);
  if (ctas < 1) ctas = 1;
  size_t budget = cap;
  for (; ctas > 1; --ctas) {
    const size_t share = (cap + 1024) / ctas - 1024;
    if (off + 2 * sb <= share) {
      budget = share;
      break;
    }
  }
  int stages = static_cast<int>((budget - off) / sb);
  stages = std::min(stages, std::min(kMaxStages, env_int("ATTNRES_TMA_MAX_STAGES", kMaxStages)));
  if (stages < 2) stages = 2;
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
  *out = p;
  return true;
}

struct TmaShape {
  TmaFn fn;
  int block, grid;
};

static cudaError_t tma_shape(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd, TmaShape* ts) {
  ts->fn = pick_tma(dtype, L, bwd);
  ts->block = p.tpc * p.tpt + 32;
  cudaError_t e = cudaFuncSetAttribute(ts->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem_bytes);
  if (e != cudaSuccess) return e;
  int per_sm = 0, dev = 0, nsm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ts->fn, ts->block, L.smem_bytes);
  if (e != cudaSuccess) return e;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  const long long cap = static_cast<long long>(nsm) * per_sm;
  ts->grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.ntiles, cap)));
  return cudaSuccess;
}

cudaError_t lrid_tma_workspace(int dtype, const LridPlan& p, const TmaLayout& L, size_t* bytes) {
  TmaShape ts;
  cudaError_t e = tma_shape(dtype, p, L, true, &ts);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(float) * static_cast<size_t>(ts.grid) * (p.R + p.H + p.S);
  return cudaSuccess;
}

static void fill_common(LridArgs& a, const LridPlan& p, const TmaLayout& L, const LridIO& io) {
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

cudaError_t lrid_tma_forward_launch(int dtype, const LridPlan& p, const TmaLayout& L, const LridIO& io,
                                    cudaStream_t st) {
  LridArgs a{};
  fill_common(a, p, L, io);
  a.out = io.out;
  a.out_inv = io.out_inv;
  a.alpha_out = io.alpha_out;
  a.kinv_out = io.kinv_out;
  TmaShape ts;
  cudaError_t e = tma_shape(dtype, p, L, false, &ts);
  if (e != cudaSuccess) return e;
  ts.fn<<<ts.grid, ts.block, L.smem_bytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t lrid_tma_backward_launch(int dtype, const LridPlan& p, const TmaLayout& L, const LridIO& io,
                                     const LridGradIO& gio, cudaStream_t st) {
  LridArgs a{};
  fill_common(a, p, L, io);
  for (int s = 0; s < p.S; ++s) {
    a.gv[s] = gio.grad_values ? gio.grad_values[s] : nullptr;
    a.gk[s] = gio.grad_keys[s];
  }
  a.g = gio.grad_output;
  a.y = gio.normed_output;
  a.y_inv = gio.output_inv_rms;
  a.dq_tok = (io.qmode == ATTNRES_QUERY_DYNAMIC) ? gio.grad_query : gio.grad_query_dynamic;
  a.want_bias_grad = gio.grad_bias != nullptr;
  TmaShape ts;
  cudaError_t e = tma_shape(dtype, p, L, true, &ts);
  if (e != cudaSuccess) return e;
  const int stride = p.R + p.H + p.S;
  const bool need_partials = io.qmode != ATTNRES_QUERY_DYNAMIC || gio.grad_bias != nullptr;
  a.partials = need_partials ? static_cast<float*>(gio.workspace) : nullptr;
  a.part_stride = stride;
  ts.fn<<<ts.grid, ts.block, L.smem_bytes, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || !need_partials) return e;
  if (io.qmode != ATTNRES_QUERY_DYNAMIC) {
    launch_reduce_partials(a.partials, ts.grid, stride, 0, p.R, static_cast<float*>(gio.grad_query), st);
    if (io.qmode == ATTNRES_QUERY_GATED)
      launch_reduce_partials(a.partials, ts.grid, stride, p.R, p.H, gio.grad_gate, st);
  }
  launch_reduce_partials(a.partials, ts.grid, stride, p.R + p.H, p.S, gio.grad_bias, st);
  return cudaGetLastError();
}

cudaError_t read_device_status(unsigned* status, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned));
  if (e != cudaSuccess || !reset) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned));
}

}  // namespace attnres
