/*
 * gl_oracle.c — CPU oracle for the B200 sparse-pooling hot path.
 *
 * TEST INFRASTRUCTURE, NOT THE PRODUCT.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load this library, and only as the checker
 * or the timed CPU baseline; the product path (granulelayer_b200) never calls it.
 *
 * Plain-C restatement of the reference's algorithm, accumulating in double:
 *   forward   z[t,g,s] = b[f] + sum_k w[8f+k] * x[t, idx[8f+k]]      (f = g*NB*8 + s)
 *             sparse_pooling/reference/pytorch_reference.py:29-47 (Mode A: 43-46)
 *             pre[t,g] = sum_{s < n_g} act(z) / n_g  (mean)            pytorch_reference.py:78-79
 *             pre[t,g] = sum_{s < n_g} act(z)        (sum extension)
 *             act: config.py:33, pytorch_reference.py:19-26 (GELU = exact erf form)
 *   backward  the gradient torch autograd takes through the above (pytorch_reference.py
 *             plus autograd), equivalently kernels/ops.py:242-249 + triton_fused.py:402-445:
 *             c1 = gpre / n_g (mean) or gpre (sum); dz = c1 * act'(z) on valid slots;
 *             dx[t, idx] += dz * w ; dw[8f+k] = sum_t dz * x[t, idx] ; db[f] = sum_t dz
 *   adam      sparse_pooling/optim.py:39-42 (fp32 params, fp32 moments, fused zero_grad :53)
 *
 * Build: make -C oracle  (gcc -O2 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static double act_d(double z, int act) {
  if (act == 0) return z;
  if (act == 1) return z > 0 ? z : 0;
  return 0.5 * z * (1.0 + erf(z * 0.70710678118654752440));
}

static double dact_d(double z, int act) {
  if (act == 0) return 1.0;
  if (act == 1) return z > 0 ? 1.0 : 0.0;
  double cdf = 0.5 * (1.0 + erf(z * 0.70710678118654752440));
  double pdf = 0.39894228040143267794 * exp(-0.5 * z * z);
  return cdf + z * pdf;
}

static int check(int64_t B, int64_t D, int64_t G, int64_t NB) {
  return (B < 0 || D < 1 || G < 0 || NB < 1) ? -2 : 0;
}

static double zval(const float* xr, const int16_t* ir, const float* wr, float bias) {
  double z = bias;
  for (int k = 0; k < 8; ++k) z += (double)wr[k] * (double)xr[ir[k]];
  return z;
}

/* pre[t*G + g] for groups [0, G) of the parameter arrays. */
int glo_fwd(const float* x, int64_t B, int64_t D, int64_t ldx, const int16_t* idx, const float* w, const float* b,
            const int32_t* counts, int64_t G, int64_t NB, int pool, int act, double* pre, int nthreads) {
  if (check(B, D, G, NB)) return -2;
  const int64_t slots = NB * 8;
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t g = 0; g < G; ++g) {
    for (int64_t t = 0; t < B; ++t) {
      const int64_t ng = counts[g] < slots ? counts[g] : slots;
      const float* xr = x + t * ldx;
      double s = 0;
      for (int64_t j = 0; j < ng; ++j) {
        const int64_t f = g * slots + j;
        s += act_d(zval(xr, idx + f * 8, w + f * 8, b[f]), act);
      }
      pre[t * G + g] = pool == 0 ? s / (double)ng : s;
    }
  }
  return 0;
}

/* Overwrites dx [B, D], dw [G*NB*8*8], db [G*NB*8] (padding slots get 0).
 *
 * Optional slack outputs (NULL = skip), same shapes as dx/dw/db: ReLU's derivative
 * jumps at z = 0, and an fp32 evaluation of z can take either side when
 * |z| <= 1e-6 * (|b| + sum_k |w_k x_k|) (twice the worst-case error, 8 * 2^-24 of the
 * term magnitudes, of an fp32 fused multiply-add chain).  For
 * such (token, neuron) pairs the slack arrays receive the magnitude of that pair's
 * contribution (|c1| |w_k| to dx, |c1| |x_k| to dw, |c1| to db), so a checker can
 * accept either side of the jump and nothing else. */
int glo_bwd(const float* x, int64_t B, int64_t D, int64_t ldx, const int16_t* idx, const float* w, const float* b,
            const int32_t* counts, int64_t G, int64_t NB, int pool, int act, const double* gpre, double* dx,
            double* dw, double* db, int nthreads, double* sdx, double* sdw, double* sdb) {
  if (check(B, D, G, NB)) return -2;
  const int64_t slots = NB * 8;
  int nt = nthreads > 0 ? nthreads : 1;
  memset(dw, 0, sizeof(double) * G * slots * 8);
  memset(db, 0, sizeof(double) * G * slots);
  const int slack = sdx != NULL && act == 1;
  if (sdx) memset(sdx, 0, sizeof(double) * B * D);
  if (sdw) memset(sdw, 0, sizeof(double) * G * slots * 8);
  if (sdb) memset(sdb, 0, sizeof(double) * G * slots);
  double* priv = (double*)calloc((size_t)nt * B * D * (slack ? 2 : 1), sizeof(double));
  if (!priv) return -8;
#pragma omp parallel num_threads(nt)
  {
    int me = 0;
#ifdef _OPENMP
    me = omp_get_thread_num();
#endif
    double* mydx = priv + (size_t)me * B * D;
    double* mysdx = slack ? priv + (size_t)(nt + me) * B * D : NULL;
    /* work items: (group, chunk of 256 slots); each owns its slots' dw/db */
    const int64_t chunks = (slots + 255) / 256;
#pragma omp for schedule(dynamic, 1)
    for (int64_t item = 0; item < G * chunks; ++item) {
      const int64_t g = item / chunks, c = item % chunks;
      const int64_t ng = counts[g] < slots ? counts[g] : slots;
      const int64_t jend = (c + 1) * 256 < ng ? (c + 1) * 256 : ng;
      for (int64_t j = c * 256; j < jend; ++j) {
        const int64_t f = g * slots + j;
        const int16_t* ir = idx + f * 8;
        const float* wr = w + f * 8;
        double dwl[8] = {0, 0, 0, 0, 0, 0, 0, 0}, dbl = 0;
        double swl[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sbl = 0;
        for (int64_t t = 0; t < B; ++t) {
          const float* xr = x + t * ldx;
          double c1 = gpre[t * G + g];
          if (pool == 0) c1 /= (double)ng;
          const double z = zval(xr, ir, wr, b[f]);
          const double dz = c1 * dact_d(z, act);
          dbl += dz;
          for (int k = 0; k < 8; ++k) {
            dwl[k] += dz * (double)xr[ir[k]];
            mydx[t * D + ir[k]] += dz * (double)wr[k];
          }
          if (slack) {
            double mag = fabs((double)b[f]);
            for (int k = 0; k < 8; ++k) mag += fabs((double)wr[k] * (double)xr[ir[k]]);
            if (fabs(z) <= 1e-6 * mag) {
              const double a1 = fabs(c1);
              sbl += a1;
              for (int k = 0; k < 8; ++k) {
                swl[k] += a1 * fabs((double)xr[ir[k]]);
                mysdx[t * D + ir[k]] += a1 * fabs((double)wr[k]);
              }
            }
          }
        }
        for (int k = 0; k < 8; ++k) dw[f * 8 + k] = dwl[k];
        db[f] = dbl;
        if (slack) {
          if (sdw)
            for (int k = 0; k < 8; ++k) sdw[f * 8 + k] = swl[k];
          if (sdb) sdb[f] = sbl;
        }
      }
    }
  }
  for (int64_t e = 0; e < B * D; ++e) {
    double s = 0, sl = 0;
    for (int i = 0; i < nt; ++i) s += priv[(size_t)i * B * D + e];
    dx[e] = s;
    if (slack) {
      for (int i = 0; i < nt; ++i) sl += priv[(size_t)(nt + i) * B * D + e];
      sdx[e] = sl;
    }
  }
  free(priv);
  return 0;
}

/* One Adam(W) step in double over double state (p, m, v updated; g read). */
int glo_adam(double* p, const double* g, double* m, double* v, int64_t n, double lr, double b1, double b2,
             double eps, double wd, int64_t step) {
  const double bc1 = 1.0 - pow(b1, (double)step), bc2 = 1.0 - pow(b2, (double)step);
  for (int64_t i = 0; i < n; ++i) {
    m[i] = b1 * m[i] + (1.0 - b1) * g[i];
    v[i] = b2 * v[i] + (1.0 - b2) * g[i] * g[i];
    const double upd = (m[i] / bc1) / (sqrt(v[i] / bc2) + eps);
    p[i] = p[i] * (1.0 - lr * wd) - lr * upd;
  }
  return 0;
}

int glo_version(void) { return 1; }
