/*
 * CPU oracle for the torchwarp differentiable-alignment dynamic programs.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C, float64 restatement of
 * the reference algorithms (hibana2077/torchwarp, paths relative to the
 * project root).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it, and only as the checker / the timed CPU
 * baseline.  The product (torchwarp_b200) never calls it.
 *
 * Layouts are natural and row-major: cost [B, N, M], JEANIE cost
 * [B, K1, K2, T, U].  Every loop is a straight restatement of the recurrence;
 * nothing here is optimised.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_INF INFINITY

static inline double dmin2(double a, double b) { return a < b ? a : b; }

/* ------------------------------------------------------------------------
 * uDTW / soft-DTW on a precomputed cost and penalty.
 * Forward: src/torchwarp/udtw/_torch_dp.py:14-42.
 *   R_ij = C_ij + softmin_gamma(R_{i-1,j-1}, R_{i-1,j}, R_{i,j-1})
 *   P_ij = Q_ij + sum_k softmax(-R_k/gamma) P_k
 *   unreachable (all predecessors +inf) or outside the Sakoe-Chiba band
 *   (|i-j| > band when band > 0): R = +inf, P = 0.
 * R and P are written in natural layout [B, N, M] (may be NULL).
 * ---------------------------------------------------------------------- */
void orc_udtw_forward(const double* C, const double* Q, int B, int N, int M,
                      double gamma, double band, double* out_r, double* out_p,
                      double* R, double* P) {
  double* Rp = (double*)malloc(sizeof(double) * (size_t)(N + 1) * (M + 1));
  double* Pp = (double*)malloc(sizeof(double) * (size_t)(N + 1) * (M + 1));
  const int W = M + 1;
  for (int b = 0; b < B; ++b) {
    const double* c = C + (size_t)b * N * M;
    const double* q = Q ? Q + (size_t)b * N * M : NULL;
    for (int k = 0; k < (N + 1) * W; ++k) { Rp[k] = ORC_INF; Pp[k] = 0.0; }
    Rp[0] = 0.0;  /* virtual cell (-1,-1) */
    for (int i = 0; i < N; ++i) {
      for (int j = 0; j < M; ++j) {
        const double rd = Rp[i * W + j], ru = Rp[i * W + j + 1], rl = Rp[(i + 1) * W + j];
        const double m = dmin2(rd, dmin2(ru, rl));
        double r = ORC_INF, p = 0.0;
        if (m != ORC_INF) {
          const double ed = exp((m - rd) / gamma), eu = exp((m - ru) / gamma),
                       el = exp((m - rl) / gamma);
          const double s = ed + eu + el;
          r = c[i * M + j] + m - gamma * log(s);
          p = (q ? q[i * M + j] : 0.0) +
              (ed * Pp[i * W + j] + eu * Pp[i * W + j + 1] + el * Pp[(i + 1) * W + j]) / s;
        }
        int ok = isfinite(r);
        if (band > 0 && fabs((double)(i - j)) > band) ok = 0;
        Rp[(i + 1) * W + j + 1] = ok ? r : ORC_INF;
        Pp[(i + 1) * W + j + 1] = ok ? p : 0.0;
      }
    }
    out_r[b] = Rp[N * W + M];
    if (out_p) out_p[b] = Pp[N * W + M];
    if (R) for (int i = 0; i < N; ++i) for (int j = 0; j < M; ++j)
      R[(size_t)b * N * M + i * M + j] = Rp[(i + 1) * W + j + 1];
    if (P) for (int i = 0; i < N; ++i) for (int j = 0; j < M; ++j)
      P[(size_t)b * N * M + i * M + j] = Pp[(i + 1) * W + j + 1];
  }
  free(Rp);
  free(Pp);
}

/* ------------------------------------------------------------------------
 * uDTW backward: src/torchwarp/udtw/_torch_dp.py:45-76.
 * For L = grad_r * R_NM + grad_p * P_NM, with E_s = R_s - C_s and
 * A_s = P_s - Q_s at the successors s of cell k:
 *   w = exp((E_s - R_k) / gamma)
 *   Rbar_k = sum_s w [Rbar_s - Pbar_s (P_k - A_s) / gamma]
 *   Pbar_k = sum_s w Pbar_s
 * dC = Rbar, dQ = Pbar.  R, P in natural layout.
 * ---------------------------------------------------------------------- */
void orc_udtw_backward(const double* C, const double* Q, const double* R, const double* P,
                       const double* grad_r, const double* grad_p, int B, int N, int M,
                       double gamma, double* dC, double* dQ) {
  const int W = M + 1;
  const size_t sz = (size_t)(N + 1) * W;
  double* G = (double*)malloc(sizeof(double) * sz);
  double* H = (double*)malloc(sizeof(double) * sz);
  double* E = (double*)malloc(sizeof(double) * sz);
  double* A = (double*)malloc(sizeof(double) * sz);
  for (int b = 0; b < B; ++b) {
    const size_t o = (size_t)b * N * M;
    const double *c = C + o, *r = R + o, *p = P + o;
    const double* q = Q ? Q + o : NULL;
    for (size_t k = 0; k < sz; ++k) { G[k] = 0; H[k] = 0; E[k] = -ORC_INF; A[k] = 0; }
    const int last = (N - 1) * W + (M - 1);
    G[last] = grad_r[b];
    H[last] = grad_p ? grad_p[b] : 0.0;
    E[last] = r[(N - 1) * M + M - 1] - c[(N - 1) * M + M - 1];
    A[last] = p[(N - 1) * M + M - 1] - (q ? q[(N - 1) * M + M - 1] : 0.0);
    for (int i = N - 1; i >= 0; --i) {
      for (int j = M - 1; j >= 0; --j) {
        if (i == N - 1 && j == M - 1) continue;
        const double rk = r[i * M + j], pk = p[i * M + j];
        const int succ[3] = {(i + 1) * W + j, i * W + j + 1, (i + 1) * W + j + 1};
        double g = 0, h = 0;
        for (int s = 0; s < 3; ++s) {
          const double w = exp((E[succ[s]] - rk) / gamma);
          g += w * (G[succ[s]] - H[succ[s]] * (pk - A[succ[s]]) / gamma);
          h += w * H[succ[s]];
        }
        G[i * W + j] = g;
        H[i * W + j] = h;
        E[i * W + j] = isfinite(rk) ? rk - c[i * M + j] : -ORC_INF;
        A[i * W + j] = pk - (q ? q[i * M + j] : 0.0);
      }
    }
    for (int i = 0; i < N; ++i) for (int j = 0; j < M; ++j) {
      dC[o + i * M + j] = G[i * W + j];
      if (dQ) dQ[o + i * M + j] = H[i * W + j];
    }
  }
  free(G); free(H); free(E); free(A);
}

/* ------------------------------------------------------------------------
 * JEANIE on a cost [B, K1, K2, T, U]: src/torchwarp/jeanie/_torch_dp.py:14-38.
 *   R[n,0,0] = C[n,0,0]
 *   R[n,t,u] = C[n,t,u] + softmin_gamma{ R[n',t',u'] : |n1'-n1| <= s1,
 *              |n2'-n2| <= s2, (t',u') in {(t-1,u), (t,u-1), (t-1,u-1)} }
 *   out = softmin_gamma over n of R[n, T-1, U-1]
 * Out-of-range predecessors are +inf (excluded).  R natural layout.
 * ---------------------------------------------------------------------- */
static double lse_neg(const double* v, int n, double gamma) {
  /* -gamma * logsumexp(-v / gamma) over n values (+inf entries excluded) */
  double m = ORC_INF;
  for (int k = 0; k < n; ++k) m = dmin2(m, v[k]);
  if (m == ORC_INF) return ORC_INF;
  double s = 0;
  for (int k = 0; k < n; ++k) s += exp((m - v[k]) / gamma);
  return m - gamma * log(s);
}

void orc_jeanie_forward(const double* C, int B, int K1, int K2, int T, int U, int s1, int s2,
                        double gamma, double* out, double* R) {
  const int K = K1 * K2;
  const size_t cells = (size_t)K * T * U;
  double* buf = (double*)malloc(sizeof(double) * (size_t)(2 * s1 + 1) * (2 * s2 + 1) * 3 + 8);
  double* fin = (double*)malloc(sizeof(double) * K);
  for (int b = 0; b < B; ++b) {
    const double* c = C + b * cells;
    double* r = R + b * cells;
    for (int t = 0; t < T; ++t) {
      for (int u = 0; u < U; ++u) {
        for (int n1 = 0; n1 < K1; ++n1) for (int n2 = 0; n2 < K2; ++n2) {
          const size_t idx = (((size_t)n1 * K2 + n2) * T + t) * U + u;
          if (t == 0 && u == 0) { r[idx] = c[idx]; continue; }
          int cnt = 0;
          for (int a1 = n1 - s1; a1 <= n1 + s1; ++a1) {
            if (a1 < 0 || a1 >= K1) continue;
            for (int a2 = n2 - s2; a2 <= n2 + s2; ++a2) {
              if (a2 < 0 || a2 >= K2) continue;
              const size_t base = ((size_t)a1 * K2 + a2) * T;
              if (t > 0) buf[cnt++] = r[(base + t - 1) * U + u];
              if (u > 0) buf[cnt++] = r[(base + t) * U + u - 1];
              if (t > 0 && u > 0) buf[cnt++] = r[(base + t - 1) * U + u - 1];
            }
          }
          r[idx] = c[idx] + lse_neg(buf, cnt, gamma);
        }
      }
    }
    for (int n = 0; n < K; ++n) fin[n] = r[((size_t)n * T + T - 1) * U + U - 1];
    out[b] = lse_neg(fin, K, gamma);
  }
  free(buf);
  free(fin);
}

/* ------------------------------------------------------------------------
 * JEANIE backward: src/torchwarp/jeanie/_torch_dp.py:41-75.
 * L = sum_b grad_out[b] out[b] + <grad_R, R>.  With E_s = R_s - C_s:
 *   Rbar_k = sum_s exp((E_s - R_k)/gamma) Rbar_s (+ grad_R[k])
 * seeded with Rbar[n,T-1,U-1] = grad_out * softmax_n(-R[n,T-1,U-1]/gamma)
 * (+ grad_R there).  dC = Rbar.  grad_R may be NULL.
 * ---------------------------------------------------------------------- */
void orc_jeanie_backward(const double* C, const double* R, const double* grad_out,
                         const double* grad_R, int B, int K1, int K2, int T, int U, int s1,
                         int s2, double gamma, double* dC) {
  const int K = K1 * K2;
  const size_t cells = (size_t)K * T * U;
  for (int b = 0; b < B; ++b) {
    const double* c = C + b * cells;
    const double* r = R + b * cells;
    const double* gR = grad_R ? grad_R + b * cells : NULL;
    double* g = dC + b * cells;
    /* final soft-min weights */
    double m = ORC_INF;
    for (int n = 0; n < K; ++n) m = dmin2(m, r[((size_t)n * T + T - 1) * U + U - 1]);
    double s = 0;
    for (int n = 0; n < K; ++n) s += exp((m - r[((size_t)n * T + T - 1) * U + U - 1]) / gamma);
    for (int t = T - 1; t >= 0; --t) {
      for (int u = U - 1; u >= 0; --u) {
        for (int n1 = 0; n1 < K1; ++n1) for (int n2 = 0; n2 < K2; ++n2) {
          const size_t idx = (((size_t)n1 * K2 + n2) * T + t) * U + u;
          double acc;
          if (t == T - 1 && u == U - 1) {
            acc = grad_out[b] * exp((m - r[idx]) / gamma) / s;
          } else {
            acc = 0;
            for (int a1 = n1 - s1; a1 <= n1 + s1; ++a1) {
              if (a1 < 0 || a1 >= K1) continue;
              for (int a2 = n2 - s2; a2 <= n2 + s2; ++a2) {
                if (a2 < 0 || a2 >= K2) continue;
                const size_t base = ((size_t)a1 * K2 + a2) * T;
                size_t sidx[3];
                int ns = 0;
                if (t + 1 < T) sidx[ns++] = (base + t + 1) * U + u;
                if (u + 1 < U) sidx[ns++] = (base + t) * U + u + 1;
                if (t + 1 < T && u + 1 < U) sidx[ns++] = (base + t + 1) * U + u + 1;
                for (int k = 0; k < ns; ++k) {
                  const double Es = r[sidx[k]] - c[sidx[k]];
                  acc += exp((Es - r[idx]) / gamma) * g[sidx[k]];
                }
              }
            }
          }
          if (gR) acc += gR[idx];
          g[idx] = acc;
        }
      }
    }
  }
}

/* ------------------------------------------------------------------------
 * Hard alignment path (gamma -> 0) with back-pointers:
 * src/torchwarp/paths.py:85-117 (_optimal_3d).  D is [K, T, U] float64.
 * Tie-break: viewpoint kk ascending, then predecessors (t-1,u-1), (t-1,u),
 * (t,u-1), strict '<'; end viewpoint = first minimum.  start_view < 0 means
 * free start.  Writes the path as (t, u, k) triples from (0,0) to
 * (T-1,U-1) into `path` (capacity 3*(T+U)); returns its length.
 * ---------------------------------------------------------------------- */
int orc_optimal_path(const double* D, int K, int T, int U, int max_shift, int start_view,
                     int* path) {
  const size_t cells = (size_t)K * T * U;
  double* r = (double*)malloc(sizeof(double) * cells);
  int* back = (int*)malloc(sizeof(int) * cells * 3);
  for (size_t k = 0; k < cells; ++k) { r[k] = ORC_INF; back[3 * k] = back[3 * k + 1] = back[3 * k + 2] = 0; }
#define IDX(k, t, u) (((size_t)(k) * T + (t)) * U + (u))
  for (int k = 0; k < K; ++k) r[IDX(k, 0, 0)] = D[IDX(k, 0, 0)];
  if (start_view >= 0) {
    for (int k = 0; k < K; ++k) r[IDX(k, 0, 0)] = ORC_INF;
    r[IDX(start_view, 0, 0)] = D[IDX(start_view, 0, 0)];
  }
  for (int t = 0; t < T; ++t) {
    for (int u = 0; u < U; ++u) {
      if (t == 0 && u == 0) continue;
      for (int k = 0; k < K; ++k) {
        double best = ORC_INF;
        int found = 0, bk = 0, bt = 0, bu = 0;
        const int lo = k - max_shift < 0 ? 0 : k - max_shift;
        const int hi = k + max_shift + 1 > K ? K : k + max_shift + 1;
        for (int kk = lo; kk < hi; ++kk) {
          const int cand[3][2] = {{t - 1, u - 1}, {t - 1, u}, {t, u - 1}};
          for (int c = 0; c < 3; ++c) {
            const int a = cand[c][0], bb = cand[c][1];
            if (a >= 0 && bb >= 0 && r[IDX(kk, a, bb)] < best) {
              best = r[IDX(kk, a, bb)];
              found = 1; bk = kk; bt = a; bu = bb;
            }
          }
        }
        if (found) {
          r[IDX(k, t, u)] = D[IDX(k, t, u)] + best;
          back[3 * IDX(k, t, u)] = bk;
          back[3 * IDX(k, t, u) + 1] = bt;
          back[3 * IDX(k, t, u) + 2] = bu;
        }
      }
    }
  }
  int k = 0;
  double bestv = r[IDX(0, T - 1, U - 1)];
  for (int kk = 1; kk < K; ++kk) if (r[IDX(kk, T - 1, U - 1)] < bestv) { bestv = r[IDX(kk, T - 1, U - 1)]; k = kk; }
  int t = T - 1, u = U - 1, n = 0;
  /* collect backwards, then reverse */
  int* tmp = (int*)malloc(sizeof(int) * 3 * (size_t)(T + U + 2));
  tmp[3 * n] = t; tmp[3 * n + 1] = u; tmp[3 * n + 2] = k; ++n;
  while (!(t == 0 && u == 0)) {
    const size_t id = IDX(k, t, u);
    const int nk = back[3 * id], nt = back[3 * id + 1], nu = back[3 * id + 2];
    k = nk; t = nt; u = nu;
    tmp[3 * n] = t; tmp[3 * n + 1] = u; tmp[3 * n + 2] = k; ++n;
  }
  for (int i = 0; i < n; ++i) {
    path[3 * i] = tmp[3 * (n - 1 - i)];
    path[3 * i + 1] = tmp[3 * (n - 1 - i) + 1];
    path[3 * i + 2] = tmp[3 * (n - 1 - i) + 2];
  }
#undef IDX
  free(tmp);
  free(r);
  free(back);
  return n;
}
