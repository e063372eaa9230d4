/*
 * mednext_oracle.c — CPU restatement (fp64, plain loops) of the arithmetic on
 * the MedNeXt block's hot path.  TEST INFRASTRUCTURE ONLY: the checker that
 * the sm_100a kernels are compared against; nothing in the product links it.
 *
 * Reference algorithms restated (paths inside nanaHa1003/mednext-accel,
 * src/mednext_accel/):
 *   depthwise conv, stride 1, pad k/2 ... ops/_triton/depthwise.py:549-563 (F.conv3d fwd),
 *                                         159-203 (dX gather form), 13-83 (dW partial+finish)
 *   depthwise conv, stride 2 ............ ops/_triton/depthwise.py:654-666 (fwd), 206-268 (dX)
 *   depthwise conv-transpose, stride 2 .. ops/_triton/depthwise.py:768-781 (fwd), 86-156 (dW)
 *   GroupNorm(C, C) ..................... models/blocks.py:74 (torch.nn.GroupNorm, biased variance)
 *   exact GELU .......................... models/blocks.py:32-41 (F.gelu approximate="none")
 *   1x1x1 convolution ................... ops/adaptive.py:174-188 (per-sample W @ X + b)
 *   Global Response Norm (v2) ........... ops/grn.py:16-29 (forward formula),
 *                                         ops/_triton/grn.py:150-232 (backward: channel coupling)
 * All tensors are contiguous NCDHW double arrays; sums are plain sequential
 * loops in fp64.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

typedef int64_t i64;

static inline i64 idx5(i64 n, i64 c, i64 d, i64 h, i64 w, i64 C, i64 D, i64 H, i64 W) {
  return (((n * C + c) * D + d) * H + h) * W + w;
}

/* y[n,c,o] = b[c] + sum_t x[n,c,o+t-p] * w[c,t]  (stride 1, zero padding p = k/2) */
void oracle_dw_fwd(const double* x, const double* wt, const double* b, double* y, i64 N, i64 C, i64 D, i64 H,
                   i64 W, int k) {
  const int p = k / 2;
  for (i64 n = 0; n < N; ++n)
    for (i64 c = 0; c < C; ++c)
      for (i64 od = 0; od < D; ++od)
        for (i64 oh = 0; oh < H; ++oh)
          for (i64 ow = 0; ow < W; ++ow) {
            double acc = b ? b[c] : 0.0;
            for (int kd = 0; kd < k; ++kd) {
              const i64 id = od + kd - p;
              if (id < 0 || id >= D) continue;
              for (int kh = 0; kh < k; ++kh) {
                const i64 ih = oh + kh - p;
                if (ih < 0 || ih >= H) continue;
                for (int kw = 0; kw < k; ++kw) {
                  const i64 iw = ow + kw - p;
                  if (iw < 0 || iw >= W) continue;
                  acc += x[idx5(n, c, id, ih, iw, C, D, H, W)] * wt[((c * k + kd) * k + kh) * k + kw];
                }
              }
            }
            y[idx5(n, c, od, oh, ow, C, D, H, W)] = acc;
          }
}

/* dx[n,c,i] = sum_t dy[n,c,i-t+p] * w[c,t]  (gather form of the stride-1 input grad) */
void oracle_dw_dgrad(const double* dy, const double* wt, double* dx, i64 N, i64 C, i64 D, i64 H, i64 W, int k) {
  const int p = k / 2;
  for (i64 n = 0; n < N; ++n)
    for (i64 c = 0; c < C; ++c)
      for (i64 id = 0; id < D; ++id)
        for (i64 ih = 0; ih < H; ++ih)
          for (i64 iw = 0; iw < W; ++iw) {
            double acc = 0.0;
            for (int kd = 0; kd < k; ++kd) {
              const i64 od = id - kd + p;
              if (od < 0 || od >= D) continue;
              for (int kh = 0; kh < k; ++kh) {
                const i64 oh = ih - kh + p;
                if (oh < 0 || oh >= H) continue;
                for (int kw = 0; kw < k; ++kw) {
                  const i64 ow = iw - kw + p;
                  if (ow < 0 || ow >= W) continue;
                  acc += dy[idx5(n, c, od, oh, ow, C, D, H, W)] * wt[((c * k + kd) * k + kh) * k + kw];
                }
              }
            }
            dx[idx5(n, c, id, ih, iw, C, D, H, W)] = acc;
          }
}

/* dw[c,t] = sum_{n,o} x[n,c,o+t-p] * dy[n,c,o];  db[c] = sum dy */
void oracle_dw_wgrad(const double* x, const double* dy, double* dw, double* db, i64 N, i64 C, i64 D, i64 H, i64 W,
                     int k) {
  const int p = k / 2;
  const int k3 = k * k * k;
  for (i64 c = 0; c < C; ++c) {
    for (int t = 0; t < k3; ++t) {
      const int kd = t / (k * k), kh = (t / k) % k, kw = t % k;
      double acc = 0.0;
      for (i64 n = 0; n < N; ++n)
        for (i64 od = 0; od < D; ++od) {
          const i64 id = od + kd - p;
          if (id < 0 || id >= D) continue;
          for (i64 oh = 0; oh < H; ++oh) {
            const i64 ih = oh + kh - p;
            if (ih < 0 || ih >= H) continue;
            for (i64 ow = 0; ow < W; ++ow) {
              const i64 iw = ow + kw - p;
              if (iw < 0 || iw >= W) continue;
              acc += x[idx5(n, c, id, ih, iw, C, D, H, W)] * dy[idx5(n, c, od, oh, ow, C, D, H, W)];
            }
          }
        }
      dw[c * k3 + t] = acc;
    }
    if (db) {
      double s = 0.0;
      for (i64 n = 0; n < N; ++n)
        for (i64 v = 0; v < D * H * W; ++v) s += dy[(n * C + c) * D * H * W + v];
      db[c] = s;
    }
  }
}

/* ---- stride-2 pair: big grid (B) and small grid (S = ceil(B/2)) or B = 2S-1 ---- */

/* small[m] = bias + sum_t big[2m - p + t] * w[t] */
void oracle_s2_gather(const double* big, const double* wt, const double* b, double* small, i64 N, i64 C, i64 Db,
                      i64 Hb, i64 Wb, i64 Ds, i64 Hs, i64 Ws, int k) {
  const int p = k / 2;
  for (i64 n = 0; n < N; ++n)
    for (i64 c = 0; c < C; ++c)
      for (i64 md = 0; md < Ds; ++md)
        for (i64 mh = 0; mh < Hs; ++mh)
          for (i64 mw = 0; mw < Ws; ++mw) {
            double acc = b ? b[c] : 0.0;
            for (int kd = 0; kd < k; ++kd) {
              const i64 id = 2 * md - p + kd;
              if (id < 0 || id >= Db) continue;
              for (int kh = 0; kh < k; ++kh) {
                const i64 ih = 2 * mh - p + kh;
                if (ih < 0 || ih >= Hb) continue;
                for (int kw = 0; kw < k; ++kw) {
                  const i64 iw = 2 * mw - p + kw;
                  if (iw < 0 || iw >= Wb) continue;
                  acc += big[idx5(n, c, id, ih, iw, C, Db, Hb, Wb)] * wt[((c * k + kd) * k + kh) * k + kw];
                }
              }
            }
            small[idx5(n, c, md, mh, mw, C, Ds, Hs, Ws)] = acc;
          }
}

/* big[i] = bias + sum over (m, t) with i = 2m - p + t of small[m] * w[t]  (scatter form) */
void oracle_s2_scatter(const double* small, const double* wt, const double* b, double* big, i64 N, i64 C, i64 Db,
                       i64 Hb, i64 Wb, i64 Ds, i64 Hs, i64 Ws, int k) {
  const int p = k / 2;
  const i64 bvol = Db * Hb * Wb;
  for (i64 n = 0; n < N; ++n)
    for (i64 c = 0; c < C; ++c) {
      double* out = big + (n * C + c) * bvol;
      for (i64 v = 0; v < bvol; ++v) out[v] = b ? b[c] : 0.0;
      for (i64 md = 0; md < Ds; ++md)
        for (i64 mh = 0; mh < Hs; ++mh)
          for (i64 mw = 0; mw < Ws; ++mw) {
            const double s = small[idx5(n, c, md, mh, mw, C, Ds, Hs, Ws)];
            for (int kd = 0; kd < k; ++kd) {
              const i64 id = 2 * md - p + kd;
              if (id < 0 || id >= Db) continue;
              for (int kh = 0; kh < k; ++kh) {
                const i64 ih = 2 * mh - p + kh;
                if (ih < 0 || ih >= Hb) continue;
                for (int kw = 0; kw < k; ++kw) {
                  const i64 iw = 2 * mw - p + kw;
                  if (iw < 0 || iw >= Wb) continue;
                  out[(id * Hb + ih) * Wb + iw] += s * wt[((c * k + kd) * k + kh) * k + kw];
                }
              }
            }
          }
    }
}

/* dw[c,t] = sum_m big[2m - p + t] * small[m] */
void oracle_s2_wgrad(const double* big, const double* small, double* dw, i64 N, i64 C, i64 Db, i64 Hb, i64 Wb,
                     i64 Ds, i64 Hs, i64 Ws, int k) {
  const int p = k / 2;
  const int k3 = k * k * k;
  for (i64 c = 0; c < C; ++c)
    for (int t = 0; t < k3; ++t) {
      const int kd = t / (k * k), kh = (t / k) % k, kw = t % k;
      double acc = 0.0;
      for (i64 n = 0; n < N; ++n)
        for (i64 md = 0; md < Ds; ++md) {
          const i64 id = 2 * md - p + kd;
          if (id < 0 || id >= Db) continue;
          for (i64 mh = 0; mh < Hs; ++mh) {
            const i64 ih = 2 * mh - p + kh;
            if (ih < 0 || ih >= Hb) continue;
            for (i64 mw = 0; mw < Ws; ++mw) {
              const i64 iw = 2 * mw - p + kw;
              if (iw < 0 || iw >= Wb) continue;
              acc += big[idx5(n, c, id, ih, iw, C, Db, Hb, Wb)] * small[idx5(n, c, md, mh, mw, C, Ds, Hs, Ws)];
            }
          }
        }
      dw[c * k3 + t] = acc;
    }
}

/* per-(n,c) sum of a volume, summed over n: the bias gradient */
void oracle_channel_sum(const double* x, double* out, i64 N, i64 C, i64 vol) {
  for (i64 c = 0; c < C; ++c) {
    double s = 0.0;
    for (i64 n = 0; n < N; ++n)
      for (i64 v = 0; v < vol; ++v) s += x[(n * C + c) * vol + v];
    out[c] = s;
  }
}

/* GroupNorm(C, C): mean/biased variance per (n, c); y = (x-mean)*rstd*gamma + beta */
void oracle_groupnorm_fwd(const double* x, const double* gamma, const double* beta, double eps, double* y,
                          double* mean, double* rstd, i64 N, i64 C, i64 vol) {
  for (i64 nc = 0; nc < N * C; ++nc) {
    const i64 c = nc % C;
    const double* xs = x + nc * vol;
    double m = 0.0;
    for (i64 v = 0; v < vol; ++v) m += xs[v];
    m /= (double)vol;
    double var = 0.0;
    for (i64 v = 0; v < vol; ++v) var += (xs[v] - m) * (xs[v] - m);
    var /= (double)vol;
    const double r = 1.0 / sqrt(var + eps);
    mean[nc] = m;
    rstd[nc] = r;
    for (i64 v = 0; v < vol; ++v) y[nc * vol + v] = (xs[v] - m) * r * (gamma ? gamma[c] : 1.0) + (beta ? beta[c] : 0.0);
  }
}

/* GroupNorm backward from dy = dL/dy; writes dx and the affine grads */
void oracle_groupnorm_bwd(const double* dy, const double* x, const double* mean, const double* rstd,
                          const double* gamma, double* dx, double* dgamma, double* dbeta, i64 N, i64 C, i64 vol) {
  for (i64 c = 0; c < C; ++c) {
    dgamma[c] = 0.0;
    dbeta[c] = 0.0;
  }
  for (i64 nc = 0; nc < N * C; ++nc) {
    const i64 c = nc % C;
    const double g = gamma ? gamma[c] : 1.0;
    double s1 = 0.0, s2 = 0.0;
    for (i64 v = 0; v < vol; ++v) {
      const double xh = (x[nc * vol + v] - mean[nc]) * rstd[nc];
      s1 += dy[nc * vol + v];
      s2 += dy[nc * vol + v] * xh;
    }
    dgamma[c] += s2;
    dbeta[c] += s1;
    for (i64 v = 0; v < vol; ++v) {
      const double xh = (x[nc * vol + v] - mean[nc]) * rstd[nc];
      dx[nc * vol + v] = rstd[nc] * g * (dy[nc * vol + v] - s1 / (double)vol - xh * s2 / (double)vol);
    }
  }
}

/* exact GELU x * Phi(x) and its derivative Phi(x) + x * phi(x) */
void oracle_gelu(const double* x, double* y, i64 n) {
  for (i64 i = 0; i < n; ++i) y[i] = 0.5 * x[i] * (1.0 + erf(x[i] / sqrt(2.0)));
}
void oracle_gelu_grad(const double* x, double* g, i64 n) {
  const double inv_sqrt_2pi = 0.3989422804014327;
  for (i64 i = 0; i < n; ++i) g[i] = 0.5 * (1.0 + erf(x[i] / sqrt(2.0))) + x[i] * inv_sqrt_2pi * exp(-0.5 * x[i] * x[i]);
}

/* y[n,j,v] = b[j] + sum_k w[j,k] x[n,k,v] */
void oracle_pointwise_fwd(const double* x, const double* wt, const double* b, double* y, i64 N, i64 Cin, i64 Cout,
                          i64 vol) {
  for (i64 n = 0; n < N; ++n)
    for (i64 j = 0; j < Cout; ++j)
      for (i64 v = 0; v < vol; ++v) {
        double acc = b ? b[j] : 0.0;
        for (i64 k = 0; k < Cin; ++k) acc += wt[j * Cin + k] * x[(n * Cin + k) * vol + v];
        y[(n * Cout + j) * vol + v] = acc;
      }
}
/* dx[n,k,v] = sum_j w[j,k] dy[n,j,v];  dw[j,k] = sum_{n,v} dy[n,j,v] x[n,k,v];  db[j] = sum dy */
void oracle_pointwise_bwd(const double* dy, const double* x, const double* wt, double* dx, double* dw, double* db,
                          i64 N, i64 Cin, i64 Cout, i64 vol) {
  for (i64 n = 0; n < N; ++n)
    for (i64 k = 0; k < Cin; ++k)
      for (i64 v = 0; v < vol; ++v) {
        double acc = 0.0;
        for (i64 j = 0; j < Cout; ++j) acc += wt[j * Cin + k] * dy[(n * Cout + j) * vol + v];
        dx[(n * Cin + k) * vol + v] = acc;
      }
  for (i64 j = 0; j < Cout; ++j) {
    for (i64 k = 0; k < Cin; ++k) {
      double acc = 0.0;
      for (i64 n = 0; n < N; ++n)
        for (i64 v = 0; v < vol; ++v) acc += dy[(n * Cout + j) * vol + v] * x[(n * Cin + k) * vol + v];
      dw[j * Cin + k] = acc;
    }
    if (db) {
      double s = 0.0;
      for (i64 n = 0; n < N; ++n)
        for (i64 v = 0; v < vol; ++v) s += dy[(n * Cout + j) * vol + v];
      db[j] = s;
    }
  }
}

/* MedNeXt v2 GRN forward, ops/grn.py:16-29:
 *   norm[n,c] = ||x[n,c,:]||_2,  den[n] = sum_c norm[n,c] + eps,
 *   y = x + gamma[c] * x * (norm[n,c] / den[n]) + beta[c].
 * norm and den are also returned (the saved statistics of the backward). */
void oracle_grn_fwd(const double* x, const double* gamma, const double* beta, double* y, double* norm, double* den,
                    i64 N, i64 C, i64 V, double eps) {
  for (i64 n = 0; n < N; ++n) {
    double total = 0.0;
    for (i64 c = 0; c < C; ++c) {
      const double* row = x + (n * C + c) * V;
      double ss = 0.0;
      for (i64 v = 0; v < V; ++v) ss += row[v] * row[v];
      norm[n * C + c] = sqrt(ss);
      total += norm[n * C + c];
    }
    den[n] = total + eps;
    for (i64 c = 0; c < C; ++c) {
      const double r = norm[n * C + c] / den[n];
      const double* row = x + (n * C + c) * V;
      double* out = y + (n * C + c) * V;
      for (i64 v = 0; v < V; ++v) out[v] = row[v] + gamma[c] * row[v] * r + beta[c];
    }
  }
}

/* GRN backward (the derivative of oracle_grn_fwd; the reference's split form is
 * ops/_triton/grn.py:150-232):
 *   qx[c] = sum_v dy x,  q[c] = sum_v dy,  h[c] = gamma[c] qx[c],
 *   dnorm[c] = (h[c] - sum_j h[j] norm[j] / den) / den,
 *   dx = dy (1 + gamma[c] norm[c] / den) + (norm[c] > 0 ? x / norm[c] : 0) dnorm[c],
 *   dgamma[c] = sum_n qx[n,c] norm[n,c] / den[n],  dbeta[c] = sum_n q[n,c]. */
void oracle_grn_bwd(const double* dy, const double* x, const double* gamma, const double* norm, const double* den,
                    double* dx, double* dgamma, double* dbeta, i64 N, i64 C, i64 V) {
  for (i64 c = 0; c < C; ++c) dgamma[c] = dbeta[c] = 0.0;
  for (i64 n = 0; n < N; ++n) {
    double coupled = 0.0;
    for (i64 c = 0; c < C; ++c) {
      const double* xr = x + (n * C + c) * V;
      const double* gr = dy + (n * C + c) * V;
      double qx = 0.0, q = 0.0;
      for (i64 v = 0; v < V; ++v) {
        qx += gr[v] * xr[v];
        q += gr[v];
      }
      const double r = norm[n * C + c] / den[n];
      coupled += gamma[c] * qx * r;
      dgamma[c] += qx * r;
      dbeta[c] += q;
    }
    for (i64 c = 0; c < C; ++c) {
      const double* xr = x + (n * C + c) * V;
      const double* gr = dy + (n * C + c) * V;
      double qx = 0.0;
      for (i64 v = 0; v < V; ++v) qx += gr[v] * xr[v];
      const double g = norm[n * C + c];
      const double dnorm = (gamma[c] * qx - coupled) / den[n];
      const double scale = 1.0 + gamma[c] * (g / den[n]);
      double* out = dx + (n * C + c) * V;
      for (i64 v = 0; v < V; ++v) out[v] = gr[v] * scale + (g > 0.0 ? xr[v] / g : 0.0) * dnorm;
    }
  }
}
