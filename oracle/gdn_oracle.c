/*
 * gdn_oracle.c -- CPU restatement of the reference's per-token Gated DeltaNet
 * recurrence and gates, in plain C with OpenMP.  TEST INFRASTRUCTURE: the
 * checker and the timed CPU baseline ("port") of the decode / verify path.
 * The product never links it.
 *
 * Parity status: pinned through gdn_oracle.py (tests/test_oracle_c.py checks
 * this file against the numpy oracle, which is pinned to golden vectors made
 * from the reference's own python/qwen35.py).
 *
 * Per step and state row v (delta::run_reference, cpp/src/delta.cpp:175-204):
 *     kS   = sum_dk k[dk] * S[v,dk]
 *     S    = a * (S - b * (kS * k)) + b * (v * k)
 *     o[v] = sum_dk q[dk] * S[v,dk]
 * Gates (cpp/src/model.cpp:608-612): beta = sigmoid(b),
 * alpha = exp(-exp(A_log) * softplus(a + dt_bias)), softplus = logaddexp(0,x).
 */
#include <math.h>
#include <stddef.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float softplus_c(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }

void oracle_gates(const float* a, const float* b, const float* A_log, const float* dt_bias,
                  float* alpha, float* beta, long long n_tok, int Hv) {
  for (long long t = 0; t < n_tok; ++t)
    for (int h = 0; h < Hv; ++h) {
      const long long i = t * Hv + h;
      alpha[i] = expf(-(expf(A_log[h]) * softplus_c(a[i] + dt_bias[h])));
      beta[i] = 1.f / (1.f + expf(-b[i]));
    }
}

/* q, k (B,T,Hk,D) fp32; v (B,T,Hv,D); alpha, beta (B,T,Hv); S_in (B,Hv,D,D) or
 * NULL; S_out (B,Hv,D,D) (may equal S_in); o (B,T,Hv,D); states (B,Hv,T,D,D)
 * or NULL.  Key head i serves value heads i*r .. i*r+r-1, r = Hv/Hk. */
void oracle_recurrent(const float* q, const float* k, const float* v, const float* alpha,
                      const float* beta, const float* S_in, float* S_out, float* o,
                      float* states, int B, int T, int Hk, int Hv, int D, int nthreads) {
  const int rep = Hv / Hk;
  const size_t DD = (size_t)D * D;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (long long bh = 0; bh < (long long)B * Hv; ++bh) {
    const int b = (int)(bh / Hv), h = (int)(bh % Hv), kh = h / rep;
    float* S = S_out + bh * DD;
    if (S_in && S_in != S_out) memcpy(S, S_in + bh * DD, DD * sizeof(float));
    if (!S_in) memset(S, 0, DD * sizeof(float));
    for (int t = 0; t < T; ++t) {
      const size_t tok = (size_t)b * T + t;
      const float* kt = k + (tok * Hk + kh) * D;
      const float* qt = q + (tok * Hk + kh) * D;
      const float* vt = v + (tok * Hv + h) * D;
      const float a = alpha[tok * Hv + h], bb = beta[tok * Hv + h];
      for (int r = 0; r < D; ++r) {
        float* row = S + (size_t)r * D;
        float kS = 0.f;
        for (int c = 0; c < D; ++c) kS += kt[c] * row[c];
        const float bk = bb * kS, bv = bb * vt[r];
        float ov = 0.f;
        for (int c = 0; c < D; ++c) {
          row[c] = a * (row[c] - bk * kt[c]) + bv * kt[c];
          ov += qt[c] * row[c];
        }
        o[(tok * Hv + h) * D + r] = ov;
      }
      if (states) memcpy(states + ((size_t)bh * T + t) * DD, S, DD * sizeof(float));
    }
  }
}
