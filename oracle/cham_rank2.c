/*
 * cham_rank2.c -- TEST INFRASTRUCTURE ONLY: the parity checker's fast CHAM scan.
 *
 * The same function as ``cham_scan_rank2`` in verace_oracle.py (which states the
 * mathematics and is the readable definition), in fp64 C with OpenMP so that sequences
 * of thousands of tokens at D = 1024 check in seconds.  Nothing in the product package
 * links or calls this file.
 *
 * Reference: the Woodbury form of the exact Cayley factor of the reference's Triton CHAM
 * kernel (verace_v1/serving/triton_kernels.py:152-306), with the eager path's semantics
 * (verace_v1/modules/cham_memory.py:211-243): H_t = U_t H_{t-1} with
 * U_t = (I - iG/2)^-1 (I + iG/2), G = g (k v^T + v k^T), so U_t H = H + W (M Z) with
 * W = [k v], Z = W^T H and the 2x2 complex M = B + K (I + Gam B), B = (i g / 2) J,
 * J = [[0, 1], [1, 0]], Gam = W^T W, K = (I - B Gam)^-1 B.  A non-finite M leaves the
 * state unchanged (cham_memory.py:76-96).  Readout rec_t = Re(H_t y_t) with y_t = p q_t
 * for a caller-supplied complex matrix p (the Newton-Schulz polynomial of H_0^H H_0), or
 * y_t = q_t when p is NULL.
 *
 * Layout: q, k, v [b][s][D]; gamma [b][s]; Hr, Hi [b][D][D] (in: H_0, out: H_s);
 * pr, pi [b][D][D] or NULL; rec [b][s][D].  All fp64, row-major.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct { double re, im; } cplx;

static cplx cmul(cplx a, cplx b) { cplx r = {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re}; return r; }
static cplx cadd(cplx a, cplx b) { cplx r = {a.re + b.re, a.im + b.im}; return r; }

/* 2x2 complex M for one token; returns 0 if not finite */
static int factor(const double* k, const double* v, double g, int D, cplx M[2][2]) {
  double kk = 0, kv = 0, vv = 0;
  for (int i = 0; i < D; ++i) { kk += k[i] * k[i]; kv += k[i] * v[i]; vv += v[i] * v[i]; }
  const double Gam[2][2] = {{kk, kv}, {kv, vv}};
  cplx B[2][2] = {{{0, 0}, {0, 0.5 * g}}, {{0, 0.5 * g}, {0, 0}}};
  /* X = I - B Gam */
  cplx X[2][2];
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c) {
      cplx a = {r == c ? 1.0 : 0.0, 0.0};
      for (int m = 0; m < 2; ++m) {
        cplx p = {B[r][m].re * Gam[m][c], B[r][m].im * Gam[m][c]};
        a.re -= p.re; a.im -= p.im;
      }
      X[r][c] = a;
    }
  /* K = X^-1 B */
  cplx det = cadd(cmul(X[0][0], X[1][1]), (cplx){-cmul(X[0][1], X[1][0]).re, -cmul(X[0][1], X[1][0]).im});
  double dn = det.re * det.re + det.im * det.im;
  if (!(dn > 0) || !isfinite(dn)) return 0;
  cplx inv_det = {det.re / dn, -det.im / dn};
  cplx Xi[2][2] = {{cmul(X[1][1], inv_det), cmul((cplx){-X[0][1].re, -X[0][1].im}, inv_det)},
                   {cmul((cplx){-X[1][0].re, -X[1][0].im}, inv_det), cmul(X[0][0], inv_det)}};
  cplx K[2][2];
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c) K[r][c] = cadd(cmul(Xi[r][0], B[0][c]), cmul(Xi[r][1], B[1][c]));
  /* M = B + K (I + Gam B) */
  cplx Y[2][2];
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c) {
      cplx a = {r == c ? 1.0 : 0.0, 0.0};
      for (int m = 0; m < 2; ++m) { a.re += Gam[r][m] * B[m][c].re; a.im += Gam[r][m] * B[m][c].im; }
      Y[r][c] = a;
    }
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c) {
      M[r][c] = cadd(B[r][c], cadd(cmul(K[r][0], Y[0][c]), cmul(K[r][1], Y[1][c])));
      if (!isfinite(M[r][c].re) || !isfinite(M[r][c].im)) return 0;
    }
  return 1;
}

void cham_rank2_scan(int b, int s, int D, const double* q, const double* k, const double* v,
                     const double* gamma, double* Hr, double* Hi, const double* pr, const double* pi,
                     double* rec) {
  double* Z = (double*)malloc(sizeof(double) * 4 * D);   /* Zk re, Zk im, Zv re, Zv im */
  double* X = (double*)malloc(sizeof(double) * 4 * D);
  double* y = (double*)malloc(sizeof(double) * 2 * D);
  for (int it = 0; it < b; ++it) {
    double* hr = Hr + (size_t)it * D * D;
    double* hi = Hi + (size_t)it * D * D;
    for (int t = 0; t < s; ++t) {
      const double* kt = k + ((size_t)it * s + t) * D;
      const double* vt = v + ((size_t)it * s + t) * D;
      const double* qt = q + ((size_t)it * s + t) * D;
      cplx M[2][2];
      if (factor(kt, vt, gamma[(size_t)it * s + t], D, M)) {
        /* Z = W^T H (parallel over blocks of 64 columns, rows streamed in order) */
#pragma omp parallel for schedule(static)
        for (int j0 = 0; j0 < D; j0 += 64) {
          const int nj = D - j0 < 64 ? D - j0 : 64;
          double a[64] = {0}, bb[64] = {0}, c[64] = {0}, d[64] = {0};
          for (int i = 0; i < D; ++i) {
            const double* r = hr + (size_t)i * D + j0;
            const double* m = hi + (size_t)i * D + j0;
            const double ki = kt[i], vi = vt[i];
            for (int j = 0; j < nj; ++j) { a[j] += ki * r[j]; bb[j] += ki * m[j]; c[j] += vi * r[j]; d[j] += vi * m[j]; }
          }
          for (int j = 0; j < nj; ++j) { Z[j0 + j] = a[j]; Z[D + j0 + j] = bb[j]; Z[2 * D + j0 + j] = c[j]; Z[3 * D + j0 + j] = d[j]; }
        }
        /* X = M Z */
        for (int j = 0; j < D; ++j) {
          cplx zk = {Z[j], Z[D + j]}, zv = {Z[2 * D + j], Z[3 * D + j]};
          cplx x0 = cadd(cmul(M[0][0], zk), cmul(M[0][1], zv));
          cplx x1 = cadd(cmul(M[1][0], zk), cmul(M[1][1], zv));
          X[j] = x0.re; X[D + j] = x0.im; X[2 * D + j] = x1.re; X[3 * D + j] = x1.im;
        }
        /* H += k X0 + v X1 (row-parallel) */
#pragma omp parallel for schedule(static)
        for (int i = 0; i < D; ++i) {
          double* r = hr + (size_t)i * D;
          double* m = hi + (size_t)i * D;
          const double a = kt[i], c = vt[i];
          for (int j = 0; j < D; ++j) {
            r[j] += a * X[j] + c * X[2 * D + j];
            m[j] += a * X[D + j] + c * X[3 * D + j];
          }
        }
      }
      /* y = p q (or q) */
      if (pr) {
        const double* par = pr + (size_t)it * D * D;
        const double* pai = pi + (size_t)it * D * D;
#pragma omp parallel for schedule(static)
        for (int i = 0; i < D; ++i) {
          double a = 0, c = 0;
          for (int j = 0; j < D; ++j) { a += par[(size_t)i * D + j] * qt[j]; c += pai[(size_t)i * D + j] * qt[j]; }
          y[i] = a; y[D + i] = c;
        }
      } else {
        for (int i = 0; i < D; ++i) { y[i] = qt[i]; y[D + i] = 0.0; }
      }
      /* rec = Re(H y) */
      double* rt = rec + ((size_t)it * s + t) * D;
#pragma omp parallel for schedule(static)
      for (int i = 0; i < D; ++i) {
        const double* r = hr + (size_t)i * D;
        const double* m = hi + (size_t)i * D;
        double a = 0;
        for (int j = 0; j < D; ++j) a += r[j] * y[j] - m[j] * y[D + j];
        rt[i] = a;
      }
    }
  }
  free(Z);
  free(X);
  free(y);
}
