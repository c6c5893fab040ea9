/*
 * CPU restatement of the reference's conv/norm kernels -- TEST
 * INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load this library, and only as the checker.
 *
 * Each function follows one reference kernel, in double precision:
 *   oracle_group_norm  <- group_norm_kernel, src/cuda/group_norm.cu:40-104
 *   oracle_dwconv1d    <- conv1d_kernel, amd_tuned_torch/_vendor/
 *                         flashfftconv_depthwise_conv1d/conv1d_bhl.cu:53-98
 *                         (with the batch stride of the K == 3 branch,
 *                         :84-86, for every K -- the generic branch's
 *                         b * L_out * D input offset at :89 is a known
 *                         reference bug, not behaviour to reproduce)
 *   oracle_conv3d      <- conv3d_fp32_kernel, src/cuda/conv3d_fp32.cu:33-149
 * Parity is pinned by tests/golden/*.npz, produced by the reference package
 * itself (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>

/* x, y: [N, C, S]; gamma, beta: [C] or NULL.  Two passes per (n, g) as in
 * the reference: mean and var = E[x^2] - mean^2 (group_norm.cu:55-94), here
 * accumulated in double so the cancellation is harmless. */
void oracle_group_norm(const float* x, const float* gamma, const float* beta, float* y,
                       int64_t N, int64_t C, int64_t S, int64_t G, double eps) {
  const int64_t Cg = C / G, M = Cg * S;
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t g = 0; g < G; ++g) {
      const float* xg = x + (n * C + g * Cg) * S;
      float* yg = y + (n * C + g * Cg) * S;
      double sum = 0.0, sumsq = 0.0;
      for (int64_t i = 0; i < M; ++i) {
        sum += xg[i];
        sumsq += (double)xg[i] * xg[i];
      }
      const double mean = sum / (double)M;
      double var = sumsq / (double)M - mean * mean;
      if (var < 0.0) var = 0.0;
      const double rstd = 1.0 / sqrt(var + eps);
      for (int64_t i = 0; i < M; ++i) {
        const int64_t c = g * Cg + i / S;
        double v = ((double)xg[i] - mean) * rstd;
        if (gamma) v *= gamma[c];
        if (beta) v += beta[c];
        yg[i] = (float)v;
      }
    }
  }
}

/* x [B, C, L], w [C, K], bias [C] or NULL -> y [B, C, L_out],
 * L_out = L + 2*pad - K + 1, zero padding. */
void oracle_dwconv1d(const float* x, const float* w, const float* bias, float* y, int64_t B,
                     int64_t C, int64_t L, int64_t K, int64_t pad) {
  const int64_t Lout = L + 2 * pad - K + 1;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t c = 0; c < C; ++c) {
      const float* xr = x + (b * C + c) * L;
      float* yr = y + (b * C + c) * Lout;
      for (int64_t l = 0; l < Lout; ++l) {
        double acc = bias ? bias[c] : 0.0;
        for (int64_t k = 0; k < K; ++k) {
          const int64_t idx = l - pad + k;
          if (idx >= 0 && idx < L) acc += (double)w[c * K + k] * xr[idx];
        }
        yr[l] = (float)acc;
      }
    }
}

/* x [N, Cin, D, H, W], w [Cout, Cin, KD, KH, KW], bias [Cout] or NULL;
 * p = {stride d,h,w, pad d,h,w, dil d,h,w}. */
void oracle_conv3d(const float* x, const float* w, const float* bias, float* y, int64_t N,
                   int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout, int64_t KD,
                   int64_t KH, int64_t KW, const int64_t* p) {
  const int64_t Do = (D + 2 * p[3] - p[6] * (KD - 1) - 1) / p[0] + 1;
  const int64_t Ho = (H + 2 * p[4] - p[7] * (KH - 1) - 1) / p[1] + 1;
  const int64_t Wo = (W + 2 * p[5] - p[8] * (KW - 1) - 1) / p[2] + 1;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t co = 0; co < Cout; ++co)
      for (int64_t od = 0; od < Do; ++od)
        for (int64_t oh = 0; oh < Ho; ++oh)
          for (int64_t ow = 0; ow < Wo; ++ow) {
            double acc = bias ? bias[co] : 0.0;
            for (int64_t ci = 0; ci < Cin; ++ci)
              for (int64_t kd = 0; kd < KD; ++kd) {
                const int64_t id = od * p[0] - p[3] + kd * p[6];
                if (id < 0 || id >= D) continue;
                for (int64_t kh = 0; kh < KH; ++kh) {
                  const int64_t ih = oh * p[1] - p[4] + kh * p[7];
                  if (ih < 0 || ih >= H) continue;
                  for (int64_t kw = 0; kw < KW; ++kw) {
                    const int64_t iw = ow * p[2] - p[5] + kw * p[8];
                    if (iw < 0 || iw >= W) continue;
                    acc += (double)x[(((n * Cin + ci) * D + id) * H + ih) * W + iw] *
                           w[(((co * Cin + ci) * KD + kd) * KH + kh) * KW + kw];
                  }
                }
              }
            y[(((n * Cout + co) * Do + od) * Ho + oh) * Wo + ow] = (float)acc;
          }
}
