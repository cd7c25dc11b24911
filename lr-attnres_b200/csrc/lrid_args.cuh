// Kernel-parameter block shared by the LRID read kernels (passed by value as a
// __grid_constant__ parameter; about 3.3 KB for 64 sources).
#pragma once

#include "common.cuh"
#include "plan.h"

namespace attnres {


struct LridArgs {
  LridPlan p;
  const void* v[kMaxSources];
  const void* k[kMaxSources];
  long long vs[kMaxSources];
  long long ks[kMaxSources];
  void* gv[kMaxSources];
  void* gk[kMaxSources];
  int qmode;
  const void* q;
  const void* gate;
  const void* qdyn;
  float scale;
  int key_norm;
  float key_eps;
  const float* bias;
  int out_norm;
  float out_eps;
  void* out;
  float* out_inv;
  float* alpha_out;
  float* kinv_out;
  const void* g;
  const void* y;
  const float* y_inv;
  void* dq_tok;
  float* partials;
  int part_stride;
  int want_bias_grad;
  // Streaming forward: this launch's counter slot {next token, finished
  // warps}; null selects the static round-robin token schedule.
  unsigned long long* sched;
  int dynamic_tokens;  // take tokens from sched[0]
  // Test hook: CTA 0 / warp 0 posts the byte count of its `withhold`-th unit
  // but issues no copy, so its wait runs out after wait_ns (-1: off).
  long long withhold;
  unsigned long long wait_ns;
  TmaLayout tma;
};

}  // namespace attnres
