// Host side of the streaming LRID read kernels (lrid_stream.cuh): launch
// plans, per-launch counter slots, programmatic dependent launches, and the
// parameter-gradient summation.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "lrid_stream.cuh"
#include "launch_cache.h"

namespace attnres {

// Fixed-order sum of the per-CTA parameter-gradient rows [dq R | dgate H |
// dbias S] into their outputs (null outputs skipped): one CTA per column,
// thread i takes rows i, i + 256, ..., then a fixed tree. Launched as a
// programmatic dependent of the backward: it waits for the backward's rows
// with griddepcontrol.wait.
__global__ void __launch_bounds__(256) stream_param_sum_kernel(const float* __restrict__ partials, int nrows,
                                                               int stride, int R, int H, float* dq,
                                                               float* dgate, float* dbias) {
  __shared__ float red[256];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int c = blockIdx.x;
  float* base = c < R ? dq : c < R + H ? dgate : dbias;
  if (base == nullptr) return;
  float* out = base + (c < R ? c : c < R + H ? c - R : c - R - H);
  float s = 0.f;
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) s += partials[static_cast<long long>(r) * stride + c];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = red[0];
}

// 512-byte chunks per lane of one output-norm group (0: no norm)
static int norm_chunks(const LridPlan& p, int esz, int out_norm) {
  if (out_norm == ATTNRES_NORM_NONE) return 0;
  const int cw = 32 * (16 / esz);
  return (out_norm == ATTNRES_NORM_ROW ? p.d : p.dv) / cw;
}

static WarpFn pick_stream(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd, int out_norm) {
  const int esz = dtype == ATTNRES_DTYPE_F32 ? 4 : 2;
  const bool norm = out_norm != ATTNRES_NORM_NONE;
  if (!bwd) return stream_kernel_fwd(dtype, L.key_packs, p.S, norm_chunks(p, esz, out_norm));
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return stream_kernel_bwd_f32(L.key_packs, p.S, norm);
    case ATTNRES_DTYPE_F16: return stream_kernel_bwd_f16(L.key_packs, p.S, norm);
    default: return stream_kernel_bwd_bf16(L.key_packs, p.S, norm);
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
// scratch), key_lanes, key_packs. With output normalisation the forward keeps
// a norm group of at most kNormMaxChunks 512-byte chunks per lane in
// registers; the backward adds a unit carrying the token's upstream-gradient
// and normed-output rows.
bool lrid_warp_plan(const LridPlan& base, int esz, bool bwd, bool has_y, bool has_qd, int out_norm,
                    TmaLayout* L, int* consumer_warps) {
  const int VEC = 16 / esz;
  const int CW = 32 * VEC;
  const bool norm = out_norm != ATTNRES_NORM_NONE;
  if (bwd && norm != has_y) return false;
  if (base.vec != VEC || base.dv % CW) return false;
  if (!pow2(base.H) || base.dk % VEC) return false;
  if (norm && !bwd && (out_norm == ATTNRES_NORM_ROW ? base.d : base.dv) > kNormMaxChunks * CW) return false;
  const int kp = (base.dk <= 32 * VEC) ? 1 : 4;
  const int ke = kp * VEC;
  if (base.dk % ke) return false;
  const int kl = base.dk / ke;
  if (!pow2(kl) || kl > 32 || (32 / kl) % base.H) return false;
  int cap = 0;
  if (cached_smem_optin(&cap) != cudaSuccess) return false;
  const size_t key_unit = static_cast<size_t>(base.S) * base.R * esz + (has_qd ? base.R * esz : 0);
  // value chunks carry the g chunk in the backward, except with the output
  // norm, where g' is formed once per token into the warp's scratch
  const size_t chunk_unit = static_cast<size_t>(base.S) * CW * esz + ((bwd && !has_y) ? CW * esz : 0);
  const size_t row_unit = (bwd && has_y) ? 2 * static_cast<size_t>(base.d) * esz : 0;
  const size_t sb = align_up(std::max(std::max(key_unit, chunk_unit), row_unit), 128);
  const size_t kcopy_off = align_up(6 * static_cast<size_t>(base.H) * ((base.S + 3) & ~3) * sizeof(float), 16);
  const size_t gscr_off = align_up(kcopy_off + (bwd ? key_unit : 0), 16);
  const size_t wscr = align_up(gscr_off + ((bwd && has_y) ? static_cast<size_t>(base.d) * esz : 0), 128);
  const int nsw = std::max(2, std::min(kStreamMaxStages, env_int_w("ATTNRES_STREAM_STAGES", 2)));
  const int nchunks = norm ? (out_norm == ATTNRES_NORM_ROW ? base.d : base.dv) / CW : 0;
  const int max_warps = bwd ? (base.S > 16 ? kStreamBwdWarpsManySources : kStreamBwdWarps)
                            : stream_fwd_warps(nchunks <= 4 ? nchunks : kNormMaxChunks);
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
      L->off_g = static_cast<int>(gscr_off);
      L->smem_bytes = static_cast<int>(total);
      L->key_lanes = kl;
      L->key_packs = kp;
      *consumer_warps = nw;
      return nw >= 2;
    }
  }
  return false;
}

static cudaError_t stream_shape(int dtype, const LridPlan& p, const TmaLayout& L, bool bwd, int out_norm,
                                WarpFn* fn, int* grid) {
  *fn = pick_stream(dtype, p, L, bwd, out_norm);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(*fn), L.smem_bytes);
  if (e != cudaSuccess) return e;
  int nsm = 0;
  e = cached_sm_count(&nsm);
  if (e != cudaSuccess) return e;
  *grid = static_cast<int>(std::max<long long>(1, std::min<long long>(p.N, nsm)));
  return cudaSuccess;
}

cudaError_t lrid_warp_workspace(int dtype, const LridPlan& p, const TmaLayout& L, int nw, size_t* bytes) {
  WarpFn fn;
  int grid = 0;
  (void)nw;
  cudaError_t e = stream_shape(dtype, p, L, true, ATTNRES_NORM_NONE, &fn, &grid);
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
  a.withhold = -1;
  a.wait_ns = kWaitLimitNs;
  // Test hook for the bounded waits: ATTNRES_TEST_WITHHOLD_COPY=<unit> makes
  // CTA 0 / warp 0 skip the copies of its <unit>-th unit while still waiting
  // for them; each such wait gives up after 20 ms and sets a status bit.
  const char* wh = getenv("ATTNRES_TEST_WITHHOLD_COPY");
  if (wh && *wh) {
    a.withhold = atoll(wh);
    a.wait_ns = 20000000ull;
  }
}

// Counter slots {next token, finished warps} of the streaming forward. Every launch leaves its slot at zero. Eager launches
// rotate through kEagerSlots slots, so launches on concurrent streams get
// different ones. A launch recorded into a CUDA graph gets a slot of its own
// for the life of the process (kGraphSlots per device): replays of different
// graphs, and eager launches, never share it. Replays of one graph that
// overlap in time share it, as they share every other buffer of that graph,
// and race. When the graph slots run out, captured launches take the static
// token schedule, which needs no slot.
constexpr int kSlotWords = 2;
constexpr int kEagerSlots = 64;
constexpr int kGraphSlots = 4096;
constexpr int kSlotMaxDevices = 64;
static __device__ unsigned long long g_sched[(kEagerSlots + kGraphSlots) * kSlotWords];

// The address is cached per device ordinal, assuming the device's primary
// context lives as long as the process (no cudaDeviceReset in between).
static cudaError_t sched_slot(cudaStream_t st, unsigned long long** slot) {
  static std::atomic<unsigned long long*> base[kSlotMaxDevices];
  static std::atomic<unsigned> eager_seq[kSlotMaxDevices];
  static std::atomic<unsigned> graph_seq[kSlotMaxDevices];
  *slot = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kSlotMaxDevices) return cudaErrorInvalidDevice;
  unsigned long long* b = base[dev].load();
  if (b == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sched);
    if (e != cudaSuccess) return e;
    b = static_cast<unsigned long long*>(p);
    base[dev].store(b);
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return e;
  if (cap == cudaStreamCaptureStatusActive) {
    const unsigned i = graph_seq[dev].fetch_add(1);
    if (i < static_cast<unsigned>(kGraphSlots)) *slot = b + kSlotWords * (kEagerSlots + i);
    return cudaSuccess;
  }
  *slot = b + kSlotWords * (eager_seq[dev].fetch_add(1) % kEagerSlots);
  return cudaSuccess;
}

static bool dynamic_schedule() {
  const char* v = getenv("ATTNRES_STREAM_SCHEDULE");
  return !(v && strcmp(v, "static") == 0);
}

// Launch with programmatic stream serialization (the kernel waits for its
// predecessor's results with griddepcontrol.wait before touching global
// memory), so its CTAs launch while the previous kernel drains.
// ATTNRES_PDL=0 launches it plainly.
static cudaError_t launch_stream(WarpFn fn, int grid, int threads, int smem, cudaStream_t st, const LridArgs& a) {
  static const bool pdl = env_int_w("ATTNRES_PDL", 1) != 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

cudaError_t lrid_warp_forward_launch(int dtype, const LridPlan& p, const TmaLayout& L, int nw,
                                     const LridIO& io, cudaStream_t st) {
  LridArgs a{};
  fill_stream_common(a, p, L, io);
  a.out = io.out;
  a.out_inv = io.out_inv;
  a.alpha_out = io.alpha_out;
  a.kinv_out = io.kinv_out;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = stream_shape(dtype, p, L, false, io.out_norm, &fn, &grid);
  if (e != cudaSuccess) return e;
  if (dynamic_schedule()) {
    if ((e = sched_slot(st, &a.sched)) != cudaSuccess) return e;
    a.dynamic_tokens = a.sched != nullptr;
  }
  e = launch_stream(fn, grid, nw * 32, L.smem_bytes, st, a);
  return e != cudaSuccess ? e : cudaGetLastError();
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
  a.y = gio.normed_output;
  a.y_inv = gio.output_inv_rms;
  a.dq_tok = (io.qmode == ATTNRES_QUERY_DYNAMIC) ? gio.grad_query : gio.grad_query_dynamic;
  a.want_bias_grad = gio.grad_bias != nullptr;
  WarpFn fn;
  int grid = 0;
  cudaError_t e = stream_shape(dtype, p, L, true, io.out_norm, &fn, &grid);
  if (e != cudaSuccess) return e;
  const int stride = p.R + p.H + p.S;
  const bool need_partials = io.qmode != ATTNRES_QUERY_DYNAMIC || gio.grad_bias != nullptr;
  a.partials = need_partials ? static_cast<float*>(gio.workspace) : nullptr;
  a.part_stride = stride;
  e = launch_stream(fn, grid, nw * 32, L.smem_bytes, st, a);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess || !need_partials) return e;
  // One summation launch for every parameter gradient, started while the
  // backward drains. (Summing in the backward's last CTA instead measured
  // slower: that CTA's serial tail outlasts this launch.)
  float* dq = io.qmode != ATTNRES_QUERY_DYNAMIC ? static_cast<float*>(gio.grad_query) : nullptr;
  float* dgate = io.qmode == ATTNRES_QUERY_GATED ? gio.grad_gate : nullptr;
  int ncols = gio.grad_bias ? stride : dgate ? p.R + p.H : p.R;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ncols);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = env_int_w("ATTNRES_PDL", 1) != 0 ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, stream_param_sum_kernel, static_cast<const float*>(a.partials), grid, stride, p.R,
                         p.H, dq, dgate, gio.grad_bias);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t read_warp_status(unsigned* status, bool reset) {
  unsigned s = 0, x = 0;
  cudaError_t e = stream_status_fwd(&x, reset);
  s |= x;
  if (e == cudaSuccess) e = stream_status_bwd_f32(&x, reset), s |= x;
  if (e == cudaSuccess) e = stream_status_bwd_f16(&x, reset), s |= x;
  if (e == cudaSuccess) e = stream_status_bwd_bf16(&x, reset), s |= x;
  *status = s;
  return e;
}

}  // namespace attnres
