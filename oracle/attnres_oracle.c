/*
 * attnres_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement, in double precision, of the block Attention-Residual
 * depth-routing read of jon123boss/LR-AttnRes. It is the parity checker for the
 * CUDA kernels (tests, __graft_entry__.smoke, bench.py's cpu_baseline and
 * reference arm) and is never linked into, or called by, the product library.
 *
 * Forward semantics restate the reference's unfused PyTorch path:
 *   LRID read  : _lrid_read_torch_list      attnres_ops.py:4195-4232
 *                (keys rms-normed per head :4217, logits*scale :4221-4224,
 *                 bias :4225-4226, softmax over sources in fp32 :4229,
 *                 weighted sum :4230-4232)
 *                gated hybrid query         model.py:2104-2110
 *                output norm                attnres_ops.py:4985 (_norm of the output)
 *   base read  : _attnres_read_torch_list   attnres_ops.py:2193-2214
 * Backward semantics are the analytic gradients of those expressions, the same
 * formulas the reference's Triton backward kernels use:
 *   LRID       : _lrid_attnres_list_backward_kernel  attnres_ops.py:602-746
 *   base       : _attnres_list_backward_kernel       attnres_ops.py:448-535
 * with the output-norm backward of attnres_ops.py:651-659 / :487-491.
 *
 * Layout: every source tensor is passed stacked and dense: values [S][N][d],
 * keys [S][N][R]; per-token query [N][H][dk]. Outputs are double.
 * Parallel over tokens with OpenMP; parameter gradients are summed per thread
 * and then combined in thread order.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { Q_STATIC = 0, Q_DYNAMIC = 1, Q_GATED = 2 };
enum { NORM_NONE = 0, NORM_PER_HEAD = 1, NORM_ROW = 2 };

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* Per-token forward state of the LRID read, kept for the backward. */
typedef struct {
  double* q;      /* [H][dk] query used for this token */
  double* logit;  /* [H][S] */
  double* alpha;  /* [H][S] */
  double* kinv;   /* [H][S] */
  double* qk;     /* [H][S]  <q, khat> */
  double* acc;    /* [d]     un-normalised read */
  double* inv;    /* [H] or [1] output-norm inverse rms */
} lrid_tok;

static void lrid_token_forward(int S, long long N, int d, int R, int H, const float* values,
                               const float* keys, int qmode, const float* q, const float* gate,
                               const float* qdyn, double scale, int key_norm, double key_eps,
                               const float* bias, int out_norm, double out_eps, long long n,
                               lrid_tok* st) {
  const int dk = R / H, dv = d / H;
  for (int h = 0; h < H; ++h)
    for (int e = 0; e < dk; ++e) {
      double qv;
      if (qmode == Q_STATIC) qv = q[h * dk + e];
      else if (qmode == Q_DYNAMIC) qv = qdyn[n * R + h * dk + e];
      else qv = (double)q[h * dk + e] + (double)gate[h] * (double)qdyn[n * R + h * dk + e];
      st->q[h * dk + e] = qv;
    }
  for (int h = 0; h < H; ++h) {
    double m = -INFINITY;
    for (int s = 0; s < S; ++s) {
      const float* k = keys + ((long long)s * N + n) * R + h * dk;
      double ss = 0.0, dot = 0.0;
      for (int e = 0; e < dk; ++e) {
        ss += (double)k[e] * k[e];
        dot += (double)k[e] * st->q[h * dk + e];
      }
      const double kinv = key_norm ? 1.0 / sqrt(ss / dk + key_eps) : 1.0;
      st->kinv[h * S + s] = kinv;
      st->qk[h * S + s] = dot * kinv;
      st->logit[h * S + s] = dot * kinv * scale + (bias ? (double)bias[s] : 0.0);
      if (st->logit[h * S + s] > m) m = st->logit[h * S + s];
    }
    double sum = 0.0;
    for (int s = 0; s < S; ++s) {
      st->alpha[h * S + s] = exp(st->logit[h * S + s] - m);
      sum += st->alpha[h * S + s];
    }
    for (int s = 0; s < S; ++s) st->alpha[h * S + s] /= sum;
    for (int e = 0; e < dv; ++e) {
      double a = 0.0;
      for (int s = 0; s < S; ++s)
        a += st->alpha[h * S + s] * values[((long long)s * N + n) * d + h * dv + e];
      st->acc[h * dv + e] = a;
    }
  }
  if (out_norm == NORM_PER_HEAD) {
    for (int h = 0; h < H; ++h) {
      double ss = 0.0;
      for (int e = 0; e < dv; ++e) ss += st->acc[h * dv + e] * st->acc[h * dv + e];
      st->inv[h] = 1.0 / sqrt(ss / dv + out_eps);
    }
  } else if (out_norm == NORM_ROW) {
    double ss = 0.0;
    for (int e = 0; e < d; ++e) ss += st->acc[e] * st->acc[e];
    st->inv[0] = 1.0 / sqrt(ss / d + out_eps);
  }
}

static lrid_tok lrid_tok_alloc(int S, int d, int R, int H) {
  lrid_tok st;
  st.q = (double*)malloc(sizeof(double) * R);
  st.logit = (double*)malloc(sizeof(double) * H * S);
  st.alpha = (double*)malloc(sizeof(double) * H * S);
  st.kinv = (double*)malloc(sizeof(double) * H * S);
  st.qk = (double*)malloc(sizeof(double) * H * S);
  st.acc = (double*)malloc(sizeof(double) * d);
  st.inv = (double*)malloc(sizeof(double) * (H > 0 ? H : 1));
  return st;
}

static void lrid_tok_free(lrid_tok* st) {
  free(st->q); free(st->logit); free(st->alpha); free(st->kinv); free(st->qk);
  free(st->acc); free(st->inv);
}

static double norm_inv(const lrid_tok* st, int out_norm, int h) {
  if (out_norm == NORM_PER_HEAD) return st->inv[h];
  if (out_norm == NORM_ROW) return st->inv[0];
  return 1.0;
}

/* LRID read forward. out [N][d]; out_inv [N][H] (PER_HEAD) / [N] (ROW) or NULL;
 * alpha, kinv_out [N][H][S] or NULL. */
void oracle_lrid_forward(int S, long long N, int d, int R, int H, const float* values,
                         const float* keys, int qmode, const float* q, const float* gate,
                         const float* qdyn, double scale, int key_norm, double key_eps,
                         const float* bias, int out_norm, double out_eps, double* out,
                         double* out_inv, double* alpha, double* kinv_out) {
  const int dv = d / H;
#pragma omp parallel
  {
    lrid_tok st = lrid_tok_alloc(S, d, R, H);
#pragma omp for schedule(static)
    for (long long n = 0; n < N; ++n) {
      lrid_token_forward(S, N, d, R, H, values, keys, qmode, q, gate, qdyn, scale, key_norm,
                         key_eps, bias, out_norm, out_eps, n, &st);
      for (int h = 0; h < H; ++h) {
        const double inv = norm_inv(&st, out_norm, h);
        for (int e = 0; e < dv; ++e) out[n * d + h * dv + e] = st.acc[h * dv + e] * inv;
        for (int s = 0; s < S; ++s) {
          if (alpha) alpha[(n * H + h) * S + s] = st.alpha[h * S + s];
          if (kinv_out) kinv_out[(n * H + h) * S + s] = st.kinv[h * S + s];
        }
      }
      if (out_inv) {
        if (out_norm == NORM_PER_HEAD)
          for (int h = 0; h < H; ++h) out_inv[n * H + h] = st.inv[h];
        else if (out_norm == NORM_ROW)
          out_inv[n] = st.inv[0];
      }
    }
    lrid_tok_free(&st);
  }
}

/* LRID read backward (recomputes the forward).
 * dV [S][N][d], dK [S][N][R];
 * dq: STATIC/GATED [H][dk] summed over tokens; DYNAMIC [N][H][dk] per token;
 * dgate [H] and dqdyn [N][H][dk] for GATED (else may be NULL); dbias [S] or NULL. */
void oracle_lrid_backward(int S, long long N, int d, int R, int H, const float* values,
                          const float* keys, int qmode, const float* q, const float* gate,
                          const float* qdyn, double scale, int key_norm, double key_eps,
                          const float* bias, int out_norm, double out_eps,
                          const float* grad_output, double* dV, double* dK, double* dq,
                          double* dgate, double* dqdyn, double* dbias) {
  const int dv = d / H, dk = R / H;
  const int nthr = oracle_num_threads();
  double* red = (double*)calloc((size_t)nthr * (R + H + S), sizeof(double));
#pragma omp parallel
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    double* my = red + (size_t)tid * (R + H + S);
    lrid_tok st = lrid_tok_alloc(S, d, R, H);
    double* gp = (double*)malloc(sizeof(double) * d);
    double* dw = (double*)malloc(sizeof(double) * S);
    double* dqt = (double*)malloc(sizeof(double) * R);
#pragma omp for schedule(static)
    for (long long n = 0; n < N; ++n) {
      lrid_token_forward(S, N, d, R, H, values, keys, qmode, q, gate, qdyn, scale, key_norm,
                         key_eps, bias, out_norm, out_eps, n, &st);
      /* output-norm backward: g' = inv * (g - y * mean(g*y)), y = acc*inv */
      for (int e = 0; e < d; ++e) gp[e] = grad_output[n * d + e];
      if (out_norm == NORM_PER_HEAD) {
        for (int h = 0; h < H; ++h) {
          const double inv = st.inv[h];
          double gy = 0.0;
          for (int e = 0; e < dv; ++e) gy += gp[h * dv + e] * st.acc[h * dv + e] * inv;
          for (int e = 0; e < dv; ++e)
            gp[h * dv + e] = inv * (gp[h * dv + e] - st.acc[h * dv + e] * inv * gy / dv);
        }
      } else if (out_norm == NORM_ROW) {
        const double inv = st.inv[0];
        double gy = 0.0;
        for (int e = 0; e < d; ++e) gy += gp[e] * st.acc[e] * inv;
        for (int e = 0; e < d; ++e) gp[e] = inv * (gp[e] - st.acc[e] * inv * gy / d);
      }
      for (int e = 0; e < R; ++e) dqt[e] = 0.0;
      for (int h = 0; h < H; ++h) {
        double wd = 0.0;
        for (int s = 0; s < S; ++s) {
          const float* v = values + ((long long)s * N + n) * d + h * dv;
          double acc = 0.0;
          for (int e = 0; e < dv; ++e) acc += gp[h * dv + e] * v[e];
          dw[s] = acc;
          wd += st.alpha[h * S + s] * acc;
        }
        for (int s = 0; s < S; ++s) {
          const double al = st.alpha[h * S + s];
          const double dl = al * (dw[s] - wd);
          double* dvp = dV + ((long long)s * N + n) * d + h * dv;
          for (int e = 0; e < dv; ++e) dvp[e] = al * gp[h * dv + e];
          if (dbias) my[R + H + s] += dl;
          const float* k = keys + ((long long)s * N + n) * R + h * dk;
          double* dkp = dK + ((long long)s * N + n) * R + h * dk;
          const double kinv = st.kinv[h * S + s];
          const double c1 = dl * scale;
          for (int e = 0; e < dk; ++e) {
            const double khat = k[e] * kinv;
            const double gk = c1 * st.q[h * dk + e];
            dkp[e] = key_norm ? kinv * (gk - khat * c1 * st.qk[h * S + s] / dk) : gk;
            dqt[h * dk + e] += c1 * khat;
          }
        }
      }
      if (qmode == Q_DYNAMIC) {
        for (int e = 0; e < R; ++e) dq[n * R + e] = dqt[e];
      } else {
        for (int e = 0; e < R; ++e) my[e] += dqt[e];
        if (qmode == Q_GATED) {
          for (int h = 0; h < H; ++h)
            for (int e = 0; e < dk; ++e) {
              dqdyn[n * R + h * dk + e] = (double)gate[h] * dqt[h * dk + e];
              my[R + h] += dqt[h * dk + e] * (double)qdyn[n * R + h * dk + e];
            }
        }
      }
    }
    lrid_tok_free(&st);
    free(gp); free(dw); free(dqt);
  }
  if (qmode != Q_DYNAMIC)
    for (int e = 0; e < R; ++e) {
      double s = 0.0;
      for (int t = 0; t < nthr; ++t) s += red[(size_t)t * (R + H + S) + e];
      dq[e] = s;
    }
  if (qmode == Q_GATED && dgate)
    for (int h = 0; h < H; ++h) {
      double s = 0.0;
      for (int t = 0; t < nthr; ++t) s += red[(size_t)t * (R + H + S) + R + h];
      dgate[h] = s;
    }
  if (dbias)
    for (int s2 = 0; s2 < S; ++s2) {
      double s = 0.0;
      for (int t = 0; t < nthr; ++t) s += red[(size_t)t * (R + H + S) + R + H + s2];
      dbias[s2] = s;
    }
  free(red);
}

/* ---- base AttnRes read (keys = rms-normed values, query [d]) ------------- */

static void base_token(int S, long long N, int d, const float* values, const float* q,
                       int key_norm, double key_eps, const float* bias, long long n,
                       double* kinv, double* qk, double* alpha, double* acc) {
  double m = -INFINITY;
  for (int s = 0; s < S; ++s) {
    const float* v = values + ((long long)s * N + n) * d;
    double ss = 0.0, dot = 0.0;
    for (int e = 0; e < d; ++e) {
      ss += (double)v[e] * v[e];
      dot += (double)v[e] * q[e];
    }
    kinv[s] = key_norm ? 1.0 / sqrt(ss / d + key_eps) : 1.0;
    qk[s] = dot * kinv[s];
    alpha[s] = qk[s] + (bias ? (double)bias[s] : 0.0);
    if (alpha[s] > m) m = alpha[s];
  }
  double sum = 0.0;
  for (int s = 0; s < S; ++s) {
    alpha[s] = exp(alpha[s] - m);
    sum += alpha[s];
  }
  for (int s = 0; s < S; ++s) alpha[s] /= sum;
  for (int e = 0; e < d; ++e) {
    double a = 0.0;
    for (int s = 0; s < S; ++s) a += alpha[s] * values[((long long)s * N + n) * d + e];
    acc[e] = a;
  }
}

void oracle_base_forward(int S, long long N, int d, const float* values, const float* q,
                         int key_norm, double key_eps, const float* bias, int out_norm,
                         double out_eps, double* out, double* out_inv) {
#pragma omp parallel
  {
    double* kinv = (double*)malloc(sizeof(double) * S);
    double* qk = (double*)malloc(sizeof(double) * S);
    double* alpha = (double*)malloc(sizeof(double) * S);
    double* acc = (double*)malloc(sizeof(double) * d);
#pragma omp for schedule(static)
    for (long long n = 0; n < N; ++n) {
      base_token(S, N, d, values, q, key_norm, key_eps, bias, n, kinv, qk, alpha, acc);
      double inv = 1.0;
      if (out_norm != NORM_NONE) {
        double ss = 0.0;
        for (int e = 0; e < d; ++e) ss += acc[e] * acc[e];
        inv = 1.0 / sqrt(ss / d + out_eps);
        if (out_inv) out_inv[n] = inv;
      }
      for (int e = 0; e < d; ++e) out[n * d + e] = acc[e] * inv;
    }
    free(kinv); free(qk); free(alpha); free(acc);
  }
}

void oracle_base_backward(int S, long long N, int d, const float* values, const float* q,
                          int key_norm, double key_eps, const float* bias, int out_norm,
                          double out_eps, const float* grad_output, double* dV, double* dq,
                          double* dbias) {
  const int nthr = oracle_num_threads();
  double* red = (double*)calloc((size_t)nthr * (d + S), sizeof(double));
#pragma omp parallel
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    double* my = red + (size_t)tid * (d + S);
    double* kinv = (double*)malloc(sizeof(double) * S);
    double* qk = (double*)malloc(sizeof(double) * S);
    double* alpha = (double*)malloc(sizeof(double) * S);
    double* dw = (double*)malloc(sizeof(double) * S);
    double* acc = (double*)malloc(sizeof(double) * d);
    double* gp = (double*)malloc(sizeof(double) * d);
#pragma omp for schedule(static)
    for (long long n = 0; n < N; ++n) {
      base_token(S, N, d, values, q, key_norm, key_eps, bias, n, kinv, qk, alpha, acc);
      for (int e = 0; e < d; ++e) gp[e] = grad_output[n * d + e];
      if (out_norm != NORM_NONE) {
        double ss = 0.0;
        for (int e = 0; e < d; ++e) ss += acc[e] * acc[e];
        const double inv = 1.0 / sqrt(ss / d + out_eps);
        double gy = 0.0;
        for (int e = 0; e < d; ++e) gy += gp[e] * acc[e] * inv;
        for (int e = 0; e < d; ++e) gp[e] = inv * (gp[e] - acc[e] * inv * gy / d);
      }
      double wd = 0.0;
      for (int s = 0; s < S; ++s) {
        const float* v = values + ((long long)s * N + n) * d;
        double a = 0.0;
        for (int e = 0; e < d; ++e) a += gp[e] * v[e];
        dw[s] = a;
        wd += alpha[s] * a;
      }
      for (int s = 0; s < S; ++s) {
        const double dl = alpha[s] * (dw[s] - wd);
        if (dbias) my[d + s] += dl;
        const float* v = values + ((long long)s * N + n) * d;
        double* dvp = dV + ((long long)s * N + n) * d;
        for (int e = 0; e < d; ++e) {
          const double khat = v[e] * kinv[s];
          const double gk = key_norm ? kinv[s] * (dl * q[e] - khat * dl * qk[s] / d) : dl * q[e];
          dvp[e] = alpha[s] * gp[e] + gk;
          my[e] += dl * khat;
        }
      }
    }
    free(kinv); free(qk); free(alpha); free(dw); free(acc); free(gp);
  }
  for (int e = 0; e < d; ++e) {
    double s = 0.0;
    for (int t = 0; t < nthr; ++t) s += red[(size_t)t * (d + S) + e];
    dq[e] = s;
  }
  if (dbias)
    for (int s2 = 0; s2 < S; ++s2) {
      double s = 0.0;
      for (int t = 0; t < nthr; ++t) s += red[(size_t)t * (d + S) + d + s2];
      dbias[s2] = s;
    }
  free(red);
}
