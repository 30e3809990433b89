/*
 * householder.c -- plain-C restatement of the reference's fixed-order Householder
 * thin QR (TEST INFRASTRUCTURE ONLY; used by tests as an independent checker).
 *
 * Follows src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:447-549 of
 * pkhairkh/gfst-hmb-public (gfst_local_qr_fixed_order_compact_kernel and
 * gfst_local_qr_fixed_order_explicit_q_kernel): per column k the norm is taken
 * over rows k..m-1 including the diagonal, beta = -sign(alpha) * norm,
 * tau = (beta - alpha) / beta, v = [1; x / (alpha - beta)], trailing columns
 * updated with w = tau * (a_kj + sum_{i>k} v_i a_ij); the explicit Q is then
 * accumulated backward from the identity over all n columns.  The reference
 * builds that kernel with --fmad=false, so this file is compiled with
 * -ffp-contract=off.  The sign rule of gfst.py:35-46 (first significant entry)
 * or sign(diag R) is applied afterwards.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void qr_one(const float* in, float* q, int m, int n, float eps_sign, int sign_mode, float* work,
                   float* tau) {
  float* f = work; /* compact factors, row-major m x n */
  memcpy(f, in, sizeof(float) * (size_t)m * n);
  const int kt = m < n ? m : n;
  for (int k = 0; k < kt; ++k) {
    float norm_sq = 0.0f;
    for (int row = k; row < m; ++row) {
      const float v = f[row * n + k];
      norm_sq += v * v;
    }
    const float norm = sqrtf(norm_sq);
    if (norm == 0.0f) {
      tau[k] = 0.0f;
      continue;
    }
    const float alpha = f[k * n + k];
    const float sign = alpha < 0.0f ? -1.0f : 1.0f;
    const float beta = -sign * norm;
    const float denom = alpha - beta;
    if (fabsf(denom) <= 0.0f) {
      tau[k] = 0.0f;
      continue;
    }
    const float tv = (beta - alpha) / beta;
    f[k * n + k] = beta;
    for (int row = k + 1; row < m; ++row) f[row * n + k] /= denom;
    for (int col = k + 1; col < n; ++col) {
      float dot = f[k * n + col];
      for (int row = k + 1; row < m; ++row) dot += f[row * n + k] * f[row * n + col];
      const float w = tv * dot;
      f[k * n + col] -= w;
      for (int row = k + 1; row < m; ++row) f[row * n + col] -= f[row * n + k] * w;
    }
    tau[k] = tv;
  }
  for (int row = 0; row < m; ++row)
    for (int col = 0; col < n; ++col) q[row * n + col] = row == col ? 1.0f : 0.0f;
  for (int k = kt - 1; k >= 0; --k) {
    const float tv = tau[k];
    if (tv == 0.0f) continue;
    for (int col = 0; col < n; ++col) {
      float dot = q[k * n + col];
      for (int row = k + 1; row < m; ++row) dot += f[row * n + k] * q[row * n + col];
      const float w = tv * dot;
      q[k * n + col] -= w;
      for (int row = k + 1; row < m; ++row) q[row * n + col] -= f[row * n + k] * w;
    }
  }
  for (int col = 0; col < n; ++col) {
    int flip = 0;
    if (sign_mode == 1) {
      flip = col < kt && f[col * n + col] < 0.0f;
    } else {
      for (int row = 0; row < m; ++row) {
        const float v = q[row * n + col];
        if (fabsf(v) > eps_sign) {
          flip = v < 0.0f;
          break;
        }
      }
    }
    if (flip)
      for (int row = 0; row < m; ++row) q[row * n + col] = -q[row * n + col];
  }
}

/* Batched: in/out are [batch, m, n] row-major float32.  Returns 0, or -1 on a
 * bad argument. */
int gfst_oracle_qr_fixed_order(const float* in, float* out, int64_t batch, int m, int n, float eps_sign,
                               int sign_mode) {
  if (!in || !out || batch < 0 || m < 1 || n < 1 || n > m) return -1;
  float* work = (float*)malloc(sizeof(float) * ((size_t)m * n + (size_t)n));
  if (!work) return -1;
  for (int64_t b = 0; b < batch; ++b) {
    qr_one(in + b * (int64_t)m * n, out + b * (int64_t)m * n, m, n, eps_sign, sign_mode, work,
           work + (size_t)m * n);
  }
  free(work);
  return 0;
}
