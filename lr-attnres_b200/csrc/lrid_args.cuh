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
  // Streaming kernels: {next token, finished warps} counter pair for the
  // dynamic token schedule; null selects the static round-robin schedule.
  unsigned long long* claim;
  TmaLayout tma;
};

}  // namespace attnres
