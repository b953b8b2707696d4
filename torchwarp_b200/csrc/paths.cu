// Hard (gamma -> 0) alignment path of a [K, T, U] float64 cost, with the
// tie-break of hibana2077/torchwarp src/torchwarp/paths.py:85-117:
//   r[k,0,0] = D[k,0,0] (only k = start_view when one is given)
//   r[k,t,u] = D[k,t,u] + min over kk in [k - s, k + s] (ascending) and
//              predecessors (t-1,u-1), (t-1,u), (t,u-1) in that order, first
//              strict minimum wins; the end viewpoint is the first argmin.
// One CTA per pair sweeps the (t, u) anti-diagonals with every viewpoint of
// a diagonal in parallel (a cell's value depends only on earlier diagonals,
// and its candidate order is fixed, so the result is bit-identical to the
// sequential loop); thread 0 then follows the back-pointers.
#include "common.cuh"

namespace tw {
namespace {

constexpr int PT = 256;

__global__ void __launch_bounds__(PT) optimal_path_kernel(const double* __restrict__ Dc, int K,
                                                          int T, int U, int max_shift,
                                                          int start_view, double* __restrict__ r,
                                                          int* __restrict__ back,
                                                          int* __restrict__ path,
                                                          int* __restrict__ length) {
  const int b = blockIdx.x;
  const long long cells = (long long)K * T * U;
  const double* Db = Dc + b * cells;
  double* rb = r + b * cells;
  int* bk = back + b * cells;
  const int TU = T * U;
  const double inf = __longlong_as_double(0x7ff0000000000000LL);
  for (int d = 0; d < T + U - 1; ++d) {
    const int tlo = max(0, d - U + 1), thi = min(T - 1, d);
    const int n_cells = (thi - tlo + 1) * K;
    for (int i = threadIdx.x; i < n_cells; i += PT) {
      const int t = tlo + i / K, k = i - (i / K) * K;
      const int u = d - t;
      const long long o = (long long)k * TU + t * U + u;
      if (d == 0) {
        rb[o] = (start_view < 0 || k == start_view) ? Db[o] : inf;
        bk[o] = 0;
        continue;
      }
      double best = inf;
      int arg = -1;
      const int lo = k - max_shift < 0 ? 0 : k - max_shift;
      const int hi = k + max_shift + 1 > K ? K : k + max_shift + 1;
      for (int kk = lo; kk < hi; ++kk) {
        const long long base = (long long)kk * TU;
        if (t >= 1 && u >= 1) {
          const double v = rb[base + (t - 1) * U + u - 1];
          if (v < best) { best = v; arg = (kk * 3 + 0); }
        }
        if (t >= 1) {
          const double v = rb[base + (t - 1) * U + u];
          if (v < best) { best = v; arg = (kk * 3 + 1); }
        }
        if (u >= 1) {
          const double v = rb[base + t * U + u - 1];
          if (v < best) { best = v; arg = (kk * 3 + 2); }
        }
      }
      rb[o] = arg >= 0 ? __dadd_rn(Db[o], best) : inf;
      bk[o] = arg;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int k = 0;
    double bv = rb[(long long)0 * TU + TU - 1];
    for (int kk = 1; kk < K; ++kk) {
      const double v = rb[(long long)kk * TU + TU - 1];
      if (v < bv) { bv = v; k = kk; }
    }
    int t = T - 1, u = U - 1, n = 0;
    const int maxlen = T + U - 1;
    int* pb = path + (long long)b * maxlen * 3;
    // walk back, writing from the end of the buffer, then shift to the front
    int pos = maxlen - 1;
    pb[3 * pos] = t; pb[3 * pos + 1] = u; pb[3 * pos + 2] = k;
    ++n;
    while (!(t == 0 && u == 0) && n < maxlen) {
      const int a = bk[(long long)k * TU + t * U + u];
      if (a < 0) break;  // unreachable cell: stop (cannot happen on finite costs)
      const int kk = a / 3, mv = a - kk * 3;
      if (mv == 0) { --t; --u; } else if (mv == 1) { --t; } else { --u; }
      k = kk;
      --pos;
      pb[3 * pos] = t; pb[3 * pos + 1] = u; pb[3 * pos + 2] = k;
      ++n;
    }
    for (int i = 0; i < n; ++i) {
      pb[3 * i] = pb[3 * (pos + i)];
      pb[3 * i + 1] = pb[3 * (pos + i) + 1];
      pb[3 * i + 2] = pb[3 * (pos + i) + 2];
    }
    length[b] = n;
  }
}

}  // namespace

int optimal_path(const double* D, int B, int K, int T, int U, int max_shift, int start_view,
                 double* r_ws, int* back_ws, int* path, int* length, cudaStream_t st) {
  if (B == 0) return kOk;
  optimal_path_kernel<<<B, PT, 0, st>>>(D, K, T, U, max_shift, start_view, r_ws, back_ws, path,
                                        length);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "optimal path launch: %s", cudaGetErrorString(e));
  return kOk;
}

}  // namespace tw
