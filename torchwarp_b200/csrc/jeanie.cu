// JEANIE (joint temporal + viewpoint soft-min DP), FVM viewpoint soft-min and
// the query/support cost builders, sm_100a.
//
// JEANIE recurrence (hibana2077/torchwarp src/torchwarp/csrc/jeanie_cuda.cu:13-23,
// src/torchwarp/jeanie/_torch_dp.py:14-75), in the log2 domain R' = R log2(e)/gamma:
//   R[n,0,0] = C[n,0,0]
//   R[n,t,u] = C[n,t,u] + softmin{ R[n',t',u'] : |n1'-n1| <= s1, |n2'-n2| <= s2,
//                                  (t',u') in {(t-1,u), (t,u-1), (t-1,u-1)} }
//   out      = softmin_n R[n, T-1, U-1]
// Backward (pull form): Rbar_k = sum over successors s of 2^(E_s - R_k) Rbar_s
// with E_s = R_s - C_s, seeded with Rbar[n,T-1,U-1] = g_out * softmax_n and
// dL/dR added everywhere when the accumulator itself feeds the loss.
//
// One CTA per pair sweeps the (t, u) anti-diagonals; the cells of a diagonal
// (all rows t on it, all K viewpoints) are independent and spread over the
// threads.  R is the pair's saved state and the accumulator output at once
// (natural layout [K1, K2, T, U], in natural units); predecessors are read
// back from it through L1 after the per-diagonal barrier.
#include "common.cuh"

namespace tw {

// tensor-core cost and chain rule (tc_gemm.cu)
bool tc_cost_eligible(const float* X, const float* Y, const float* vx, const float* vy, int N,
                      int M, int D, const float* C, const float* Q);
int tc_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B, int N,
                int M, int D, double beta, double eps, float* C, float* Q, uint32_t* mask,
                cudaStream_t st);
int tc_qs_grad_f32(const float* Q, const float* Sp, const float* C, const float* dC, int B,
                   int R, int U, int D, int sqrt_cost, float* dQ, float* dSp, cudaStream_t st);

namespace {

struct JGrid {
  int K1, K2, K, T, U, s1, s2;
};

constexpr int JT = 256;  // threads per CTA

template <typename T>
__device__ __forceinline__ T jmin(T a, T b) { return a < b ? a : b; }

// log2-domain soft-min over the (2 s1 + 1)(2 s2 + 1) x 3 predecessors of
// (n, t, u); Rb points at the pair's R (natural units), kap = log2(e)/gamma.
template <typename T>
__device__ __forceinline__ T pred_softmin(const T* Rb, const JGrid& g, int n, int t, int u, T kap) {
  const int n1 = n / g.K2, n2 = n - n1 * g.K2;
  const int a1 = max(0, n1 - g.s1), b1 = min(g.K1 - 1, n1 + g.s1);
  const int a2 = max(0, n2 - g.s2), b2 = min(g.K2 - 1, n2 + g.s2);
  const int TU = g.T * g.U;
  T m = Big<T>::value;
  for (int x1 = a1; x1 <= b1; ++x1)
    for (int x2 = a2; x2 <= b2; ++x2) {
      const T* r = Rb + (long long)(x1 * g.K2 + x2) * TU;
      if (t > 0) m = jmin(m, r[(t - 1) * g.U + u] * kap);
      if (u > 0) m = jmin(m, r[t * g.U + u - 1] * kap);
      if (t > 0 && u > 0) m = jmin(m, r[(t - 1) * g.U + u - 1] * kap);
    }
  T s = T(0);
  for (int x1 = a1; x1 <= b1; ++x1)
    for (int x2 = a2; x2 <= b2; ++x2) {
      const T* r = Rb + (long long)(x1 * g.K2 + x2) * TU;
      if (t > 0) s += ex2(m - r[(t - 1) * g.U + u] * kap);
      if (u > 0) s += ex2(m - r[t * g.U + u - 1] * kap);
      if (t > 0 && u > 0) s += ex2(m - r[(t - 1) * g.U + u - 1] * kap);
    }
  return m - lg2(s);
}

template <typename T>
__device__ __forceinline__ T final_softmin(const T* Rb, const JGrid& g, T kap) {
  const int TU = g.T * g.U, last = TU - 1;
  T m = Big<T>::value;
  for (int n = 0; n < g.K; ++n) m = jmin(m, Rb[(long long)n * TU + last] * kap);
  T s = T(0);
  for (int n = 0; n < g.K; ++n) s += ex2(m - Rb[(long long)n * TU + last] * kap);
  return m - lg2(s);
}

template <typename T>
__global__ void __launch_bounds__(JT) jeanie_fwd_kernel(const T* __restrict__ C, T* __restrict__ R,
                                                        T* __restrict__ out, JGrid g, T kap,
                                                        T inv_kap) {
  const int b = blockIdx.x;
  const long long cells = (long long)g.K * g.T * g.U;
  const T* Cb = C + b * cells;
  T* Rb = R + b * cells;
  const int TU = g.T * g.U;
  for (int d = 0; d < g.T + g.U - 1; ++d) {
    const int tlo = max(0, d - g.U + 1), thi = min(g.T - 1, d);
    const int n_cells = (thi - tlo + 1) * g.K;
    for (int i = threadIdx.x; i < n_cells; i += JT) {
      const int t = tlo + i / g.K, n = i - (i / g.K) * g.K;
      const int u = d - t;
      const long long o = (long long)n * TU + t * g.U + u;
      T r = Cb[o];
      if (d > 0) r += pred_softmin(Rb, g, n, t, u, kap) * inv_kap;
      Rb[o] = r;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[b] = final_softmin(Rb, g, kap) * inv_kap;
}

template <typename T>
__global__ void __launch_bounds__(JT) jeanie_bwd_kernel(const T* __restrict__ C,
                                                        const T* __restrict__ R,
                                                        const T* __restrict__ g_out,
                                                        const T* __restrict__ g_R,
                                                        T* __restrict__ dC, JGrid g, T kap) {
  const int b = blockIdx.x;
  const long long cells = (long long)g.K * g.T * g.U;
  const T* Cb = C + b * cells;
  const T* Rb = R + b * cells;
  const T* gRb = g_R ? g_R + b * cells : nullptr;
  T* Gb = dC + b * cells;  // Rbar, written diagonal by diagonal
  const int TU = g.T * g.U, last = TU - 1;
  const T fin = final_softmin(Rb, g, kap);
  const T go = g_out[b];
  for (int d = g.T + g.U - 2; d >= 0; --d) {
    const int tlo = max(0, d - g.U + 1), thi = min(g.T - 1, d);
    const int n_cells = (thi - tlo + 1) * g.K;
    for (int i = threadIdx.x; i < n_cells; i += JT) {
      const int t = tlo + i / g.K, n = i - (i / g.K) * g.K;
      const int u = d - t;
      const long long o = (long long)n * TU + t * g.U + u;
      const T rk = Rb[o] * kap;
      T acc = T(0);
      if (t == g.T - 1 && u == g.U - 1) {
        acc = go * ex2(fin - rk);
      } else {
        const int n1 = n / g.K2, n2 = n - n1 * g.K2;
        const int a1 = max(0, n1 - g.s1), b1 = min(g.K1 - 1, n1 + g.s1);
        const int a2 = max(0, n2 - g.s2), b2 = min(g.K2 - 1, n2 + g.s2);
        for (int x1 = a1; x1 <= b1; ++x1)
          for (int x2 = a2; x2 <= b2; ++x2) {
            const long long base = (long long)(x1 * g.K2 + x2) * TU;
            if (t + 1 < g.T) {
              const long long so = base + (t + 1) * g.U + u;
              acc += ex2((Rb[so] - Cb[so]) * kap - rk) * Gb[so];
            }
            if (u + 1 < g.U) {
              const long long so = base + t * g.U + u + 1;
              acc += ex2((Rb[so] - Cb[so]) * kap - rk) * Gb[so];
            }
            if (t + 1 < g.T && u + 1 < g.U) {
              const long long so = base + (t + 1) * g.U + u + 1;
              acc += ex2((Rb[so] - Cb[so]) * kap - rk) * Gb[so];
            }
          }
      }
      if (gRb) acc += gRb[o];
      Gb[o] = acc;
    }
    __syncthreads();
  }
  (void)last;
}

// ---------------------------------------------------------------- costs
// query rows r = (n, t) of q [B, R, D], support rows u of s [B, U, D]:
//   sq_raw = |q_r|^2 + |s_u|^2 - 2 q_r.s_u, sq = max(sq_raw, 0)
//   cost   = sq (metric 0) or sqrt(sq) with zero gradient at 0 (metric 1)
// (jeanie/distances.py:25-38, jeanie/_ops.py:179-185).  A chunk of CU
// support frames sits in shared memory; each thread owns query rows, streams
// them once per chunk and keeps CU dot products in registers.

constexpr int CU = 16;   // support frames per chunk (cost kernel)
constexpr int GU = 64;   // support frames per launch (gradient kernel)

template <typename T>
__global__ void __launch_bounds__(JT) qs_cost_kernel(const T* __restrict__ q,
                                                     const T* __restrict__ s, int Rr, int U, int D,
                                                     int metric, T* __restrict__ cost) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ss = reinterpret_cast<T*>(smem_raw);  // [CU][D]
  T* s2 = ss + CU * D;                     // [CU]
  const int b = blockIdx.y;
  const T* qb = q + (long long)b * Rr * D;
  const T* sb = s + (long long)b * U * D;
  for (int u0 = 0; u0 < U; u0 += CU) {
    const int nu = min(CU, U - u0);
    __syncthreads();
    for (int e = threadIdx.x; e < CU * D; e += JT)
      ss[e] = e < nu * D ? sb[(long long)u0 * D + e] : T(0);
    __syncthreads();
    for (int u = threadIdx.x; u < CU; u += JT) {
      T a = T(0);
      for (int d = 0; d < D; ++d) a += ss[u * D + d] * ss[u * D + d];
      s2[u] = a;
    }
    __syncthreads();
    for (int r = blockIdx.x * JT + threadIdx.x; r < Rr; r += gridDim.x * JT) {
      const T* qr = qb + (long long)r * D;
      T acc[CU];
#pragma unroll
      for (int u = 0; u < CU; ++u) acc[u] = T(0);
      T q2 = T(0);
      for (int d = 0; d < D; ++d) {
        const T v = qr[d];
        q2 += v * v;
#pragma unroll
        for (int u = 0; u < CU; ++u) acc[u] += v * ss[u * D + d];
      }
      T* cr = cost + ((long long)b * Rr + r) * U + u0;
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        if (u >= nu) break;
        const T raw = (q2 + s2[u]) - T(2) * acc[u];
        const T sq = raw > T(0) ? raw : T(0);
        cr[u] = metric == 1 ? (raw > T(0) ? sqrt(sq) : T(0)) : sq;
      }
    }
  }
}

// Gradient of the cost with respect to q and s for support frames
// [u0, u0 + nu) (nu <= GU):
//   dsq = dcost (metric 0) or dcost / (2 cost) (metric 1), 0 where cost == 0
//         (sq_raw <= 0, the torch.clamp_min / sqrt-at-0 convention)
//   dq_r += 2 q_r sum_u dsq_ru - 2 sum_u dsq_ru s_u
//   ds_u  = 2 s_u sum_r dsq_ru - 2 sum_r dsq_ru q_r
// A CTA owns one pair and GF features; thread (feature, row lane) walks the
// query rows, so every q row is read once per launch and ds is reduced over
// the row lanes in a fixed order (no atomics: bitwise reproducible).
constexpr int GF = 32;  // features per CTA
constexpr int GR = 8;   // row lanes per feature

template <typename T>
__global__ void __launch_bounds__(GF * GR) qs_grad_kernel(const T* __restrict__ q,
                                                          const T* __restrict__ s,
                                                          const T* __restrict__ cost,
                                                          const T* __restrict__ dcost, int Rr,
                                                          int U, int D, int metric, int u0,
                                                          int nu, int accumulate,
                                                          T* __restrict__ dq, T* __restrict__ ds) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* dsq = reinterpret_cast<T*>(smem_raw);  // [GR][GU] dsq of the rows in flight
  T* ssv = dsq + GR * GU;                   // [GU][GF] support values of this feature chunk
  T* part = ssv + GU * GF;                  // [GR][GU][GF] partial sum_r dsq q
  T* csum = part + (size_t)GR * GU * GF;    // [GU] column sums of dsq
  const int b = blockIdx.y;
  const int f = threadIdx.x % GF;
  const int d = blockIdx.x * GF + f;
  const int lr = threadIdx.x / GF;
  const bool dv = d < D;
  const T* qb = q + (long long)b * Rr * D;
  const T* sb = s + (long long)b * U * D;
  for (int e = threadIdx.x; e < GU * GF; e += GF * GR) {
    const int u = e / GF, ff = e % GF;
    ssv[e] = (u < nu && blockIdx.x * GF + ff < D) ? sb[(long long)(u0 + u) * D + blockIdx.x * GF + ff]
                                                 : T(0);
  }
  for (int e = threadIdx.x; e < GR * GU * GF; e += GF * GR) part[e] = T(0);
  for (int u = threadIdx.x; u < GU; u += GF * GR) csum[u] = T(0);
  for (int r0 = 0; r0 < Rr; r0 += GR) {
    __syncthreads();
    {
      const int r = r0 + lr;
      for (int u = f; u < GU; u += GF) {
        T g = T(0);
        if (r < Rr && u < nu) {
          const long long o = ((long long)b * Rr + r) * U + u0 + u;
          const T c = cost[o], dc = dcost[o];
          g = c > T(0) ? (metric == 1 ? dc * T(0.5) / c : dc) : T(0);
        }
        dsq[lr * GU + u] = g;
      }
    }
    __syncthreads();
    if (threadIdx.x < GU) {  // column sums, in row order
      T c = csum[threadIdx.x];
      for (int k = 0; k < GR; ++k) c += dsq[k * GU + threadIdx.x];
      csum[threadIdx.x] = c;
    }
    const int r = r0 + lr;
    if (r < Rr && dv) {
      T rs = T(0), acc = T(0);
      const T qv = qb[(long long)r * D + d];
      for (int u = 0; u < nu; ++u) {
        const T g = dsq[lr * GU + u];
        rs += g;
        acc += g * ssv[u * GF + f];
        part[((size_t)lr * GU + u) * GF + f] += g * qv;
      }
      T* dqp = dq + ((long long)b * Rr + r) * D + d;
      const T v = T(2) * qv * rs - T(2) * acc;
      *dqp = accumulate ? *dqp + v : v;
    }
  }
  __syncthreads();
  if (lr == 0 && dv) {
    for (int u = 0; u < nu; ++u) {
      T a = T(0);
      for (int k = 0; k < GR; ++k) a += part[((size_t)k * GU + u) * GF + f];
      ds[((long long)b * U + u0 + u) * D + d] = T(2) * ssv[u * GF + f] * csum[u] - T(2) * a;
    }
  }
}

// FVM viewpoint soft-min (jeanie/fvm.py:36-37): temporal[t,u] =
// -gamma logsumexp_n(-cost[n,t,u]/gamma); backward dcost = softmax_n * dtemporal.
template <typename T>
__global__ void fvm_softmin_kernel(const T* __restrict__ cost, int Kf, int TU, T kap, T inv_kap,
                                   T* __restrict__ temporal) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (i >= TU) return;
  const T* c = cost + (long long)b * Kf * TU + i;
  T m = Big<T>::value;
  for (int n = 0; n < Kf; ++n) m = jmin(m, c[(long long)n * TU] * kap);
  T s = T(0);
  for (int n = 0; n < Kf; ++n) s += ex2(m - c[(long long)n * TU] * kap);
  temporal[(long long)b * TU + i] = (m - lg2(s)) * inv_kap;
}

template <typename T>
__global__ void fvm_softmin_bwd_kernel(const T* __restrict__ cost, const T* __restrict__ dtemp,
                                       int Kf, int TU, T kap, T* __restrict__ dcost) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (i >= TU) return;
  const T* c = cost + (long long)b * Kf * TU + i;
  T m = Big<T>::value;
  for (int n = 0; n < Kf; ++n) m = jmin(m, c[(long long)n * TU] * kap);
  T s = T(0);
  for (int n = 0; n < Kf; ++n) s += ex2(m - c[(long long)n * TU] * kap);
  const T g = dtemp[(long long)b * TU + i] * rcp(s);
  T* dc = dcost + (long long)b * Kf * TU + i;
  for (int n = 0; n < Kf; ++n) dc[(long long)n * TU] = g * ex2(m - c[(long long)n * TU] * kap);
}

// ---------------------------------------------------------------------------
// Warp-per-row forms of the query/support cost and its chain rule for fp32,
// U <= 16 support frames and D <= 256 features (the JEANIE / FVM shapes).
// Lanes split the features (4 per lane per 128-feature chunk), so every q row
// is read with coalesced 16-byte loads; the pair's support rows (and, in the
// backward, the partial ds accumulators) stay in registers, and the U dot
// products of a row meet in a shuffle butterfly.  Row sums and the ds
// partials of the warps are combined in a fixed order: results are
// bitwise reproducible.

constexpr int QW = 4;  // warps per CTA

template <int CU>
__device__ __forceinline__ void warp_allreduce(float (&v)[CU]) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
    for (int u = 0; u < CU; ++u) v[u] += __shfl_xor_sync(0xffffffffu, v[u], m);
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

template <int NCH, int CU>
__global__ void __launch_bounds__(32 * QW) qs_cost_fast_kernel(const float* __restrict__ q,
                                                                const float* __restrict__ s,
                                                                int Rr, int U, int D, int metric,
                                                                float* __restrict__ cost) {
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* sb = s + (long long)b * U * D;
  const float* qb = q + (long long)b * Rr * D;
  float4 sv[NCH][CU];
  float s2[CU];
#pragma unroll
  for (int u = 0; u < CU; ++u) {
    s2[u] = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int d = c * 128 + 4 * lane;
      sv[c][u] = (u < U && d < D) ? __ldg(reinterpret_cast<const float4*>(sb + (long long)u * D + d))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      s2[u] += dot4(sv[c][u], sv[c][u]);
    }
  }
  warp_allreduce<CU>(s2);
  float s2u = s2[0];
#pragma unroll
  for (int u = 1; u < CU; ++u) s2u = lane == u ? s2[u] : s2u;
  // two rows per iteration (r and r + step): independent loads and butterflies
  const int step = gridDim.x * QW;
  for (int r = blockIdx.x * QW + warp; r < Rr; r += 2 * step) {
    const int r2 = r + step;
    const bool has2 = r2 < Rr;
    float acc[2][CU + 1];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int u = 0; u <= CU; ++u) acc[h][u] = 0.f;
    float4 qv[2][NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int d = c * 128 + 4 * lane;
      qv[0][c] = d < D ? __ldg(reinterpret_cast<const float4*>(qb + (long long)r * D + d))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      qv[1][c] = (d < D && has2)
                     ? __ldg(reinterpret_cast<const float4*>(qb + (long long)r2 * D + d))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[h][CU] += dot4(qv[h][c], qv[h][c]);
#pragma unroll
        for (int u = 0; u < CU; ++u) acc[h][u] += dot4(qv[h][c], sv[c][u]);
      }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
      for (int u = 0; u <= CU; ++u) {
        acc[0][u] += __shfl_xor_sync(0xffffffffu, acc[0][u], m);
        acc[1][u] += __shfl_xor_sync(0xffffffffu, acc[1][u], m);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // lane u writes column u
      float mine = acc[h][0];
#pragma unroll
      for (int u = 1; u < CU; ++u) mine = lane == u ? acc[h][u] : mine;
      const int rr = h == 0 ? r : r2;
      if (lane < U && (h == 0 || has2)) {
        const float raw = (acc[h][CU] + s2u) - 2.f * mine;
        const float sq = raw > 0.f ? raw : 0.f;
        cost[((long long)b * Rr + rr) * U + lane] =
            metric == 1 ? (raw > 0.f ? sqrtf(sq) : 0.f) : sq;
      }
    }
  }
}

template <int NCH, int CU>
__global__ void __launch_bounds__(32 * QW) qs_grad_fast_kernel(
    const float* __restrict__ q, const float* __restrict__ s, const float* __restrict__ cost,
    const float* __restrict__ dcost, int Rr, int U, int D, int metric, float* __restrict__ dq,
    float* __restrict__ ds) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float4* part = reinterpret_cast<float4*>(smem_raw);  // [QW][NCH][CU][32] ds partials
  float* csum = reinterpret_cast<float*>(part + QW * NCH * CU * 32);  // [QW][CU]
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* sb = s + (long long)b * U * D;
  const float* qb = q + (long long)b * Rr * D;
  float4 sv[NCH][CU], acc[NCH][CU];
#pragma unroll
  for (int u = 0; u < CU; ++u)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int d = c * 128 + 4 * lane;
      sv[c][u] = (u < U && d < D) ? __ldg(reinterpret_cast<const float4*>(sb + (long long)u * D + d))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      acc[c][u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  float cs[CU];
#pragma unroll
  for (int u = 0; u < CU; ++u) cs[u] = 0.f;
  // the next row's cost / dcost / q are loaded one iteration ahead
  float cn = 0.f, dcn = 0.f;
  float4 qn[NCH];
  auto fetch = [&](int r) {
    if (r < Rr) {
      if (lane < U) {
        const long long o = ((long long)b * Rr + r) * U + lane;
        cn = __ldg(cost + o);
        dcn = __ldg(dcost + o);
      }
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int d = c * 128 + 4 * lane;
        qn[c] = d < D ? __ldg(reinterpret_cast<const float4*>(qb + (long long)r * D + d))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  fetch(warp);
  for (int r = warp; r < Rr; r += QW) {
    const float c0 = cn, dc0 = dcn;
    float4 qcur[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) qcur[c] = qn[c];
    fetch(r + QW);
    // dsq of the row: dcost (metric 0) or dcost / (2 cost) (metric 1), 0
    // where the cost is 0 (the clamp_min / sqrt-at-0 convention)
    float gl = 0.f;
    if (lane < U) gl = c0 > 0.f ? (metric == 1 ? dc0 * 0.5f / c0 : dc0) : 0.f;
    float gu[CU];
    float rs = 0.f;
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      gu[u] = __shfl_sync(0xffffffffu, gl, u);
      rs += gu[u];
      cs[u] += gu[u];
    }
    float* dqr = dq + ((long long)b * Rr + r) * D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int d = c * 128 + 4 * lane;
      if (d >= D) continue;
      const float4 qv = qcur[c];
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        t.x = fmaf(gu[u], sv[c][u].x, t.x);
        t.y = fmaf(gu[u], sv[c][u].y, t.y);
        t.z = fmaf(gu[u], sv[c][u].z, t.z);
        t.w = fmaf(gu[u], sv[c][u].w, t.w);
        acc[c][u].x = fmaf(gu[u], qv.x, acc[c][u].x);
        acc[c][u].y = fmaf(gu[u], qv.y, acc[c][u].y);
        acc[c][u].z = fmaf(gu[u], qv.z, acc[c][u].z);
        acc[c][u].w = fmaf(gu[u], qv.w, acc[c][u].w);
      }
      float4 o;
      o.x = 2.f * qv.x * rs - 2.f * t.x;
      o.y = 2.f * qv.y * rs - 2.f * t.y;
      o.z = 2.f * qv.z * rs - 2.f * t.z;
      o.w = 2.f * qv.w * rs - 2.f * t.w;
      *reinterpret_cast<float4*>(dqr + d) = o;
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int u = 0; u < CU; ++u) part[((warp * NCH + c) * CU + u) * 32 + lane] = acc[c][u];
  if (lane == 0)
#pragma unroll
    for (int u = 0; u < CU; ++u) csum[warp * CU + u] = cs[u];
  __syncthreads();
  // ds[u][d] = 2 s_u[d] colsum_u - 2 sum_r dsq_ru q_r[d], warps summed in order
  for (int e = threadIdx.x; e < NCH * CU * 32; e += 32 * QW) {
    const int l = e & 31, cu = e >> 5, u = cu % CU, c = cu / CU;
    const int d = c * 128 + 4 * l;
    if (u >= U || d >= D) continue;
    float4 a = part[(0 * NCH * CU + cu) * 32 + l];
    float col = csum[u];
#pragma unroll
    for (int w = 1; w < QW; ++w) {
      const float4 p = part[(w * NCH * CU + cu) * 32 + l];
      a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
      col += csum[w * CU + u];
    }
    const float4 sd = __ldg(reinterpret_cast<const float4*>(sb + (long long)u * D + d));
    float4 o;
    o.x = 2.f * sd.x * col - 2.f * a.x;
    o.y = 2.f * sd.y * col - 2.f * a.y;
    o.z = 2.f * sd.z * col - 2.f * a.z;
    o.w = 2.f * sd.w * col - 2.f * a.w;
    *reinterpret_cast<float4*>(ds + ((long long)b * U + u) * D + d) = o;
  }
}

template <int NCH, int CU>
int qs_fast_launch(const float* q, const float* s, const float* cost, const float* dcost, int B,
                   int Rr, int U, int D, int metric, float* out_cost, float* dq, float* ds,
                   cudaStream_t st) {
  if (out_cost != nullptr) {
    int gx = (Rr + 32 * QW - 1) / (32 * QW);  // about 32 rows per warp: the support load amortises
    dim3 grid(gx, B);
    qs_cost_fast_kernel<NCH, CU><<<grid, 32 * QW, 0, st>>>(q, s, Rr, U, D, metric, out_cost);
  } else {
    const size_t smem = (size_t)QW * NCH * CU * 32 * sizeof(float4) + (size_t)QW * CU * sizeof(float);
    auto kern = qs_grad_fast_kernel<NCH, CU>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return set_error(kLaunch, "qs grad: shared memory");
    kern<<<B, 32 * QW, smem, st>>>(q, s, cost, dcost, Rr, U, D, metric, dq, ds);
  }
  return kOk;
}

// Dispatch to the warp-per-row kernels when they apply; kUnsupported otherwise.
int qs_fast(const float* q, const float* s, const float* cost, const float* dcost, int B, int Rr,
            int U, int D, int metric, float* out_cost, float* dq, float* ds, cudaStream_t st) {
  if (D % 4 != 0 || D > 256 || U > 16 || U < 1 || ((uintptr_t)q & 15u) || ((uintptr_t)s & 15u) ||
      (dq && ((uintptr_t)dq & 15u)) || (ds && ((uintptr_t)ds & 15u)))
    return kUnsupported;
  const int nch = D > 128 ? 2 : 1;
  const int cu = U <= 4 ? 4 : (U <= 8 ? 8 : (U <= 12 ? 12 : 16));
#define TW_QS(NC, C)                                                                             \
  if (nch == NC && cu == C)                                                                      \
    return qs_fast_launch<NC, C>(q, s, cost, dcost, B, Rr, U, D, metric, out_cost, dq, ds, st);
  TW_QS(1, 4) TW_QS(1, 8) TW_QS(1, 12) TW_QS(1, 16)
  TW_QS(2, 4) TW_QS(2, 8) TW_QS(2, 12) TW_QS(2, 16)
#undef TW_QS
  return kUnsupported;
}

template <typename T>
int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "%s launch: %s", what, cudaGetErrorString(e));
  return kOk;
}

}  // namespace

template <typename T>
int jeanie_forward(const T* C, int B, int K1, int K2, int Tn, int U, int s1, int s2, double gamma,
                   T* out, T* R, cudaStream_t st) {
  if (B == 0) return kOk;
  JGrid g{K1, K2, K1 * K2, Tn, U, s1, s2};
  const double kap = 1.4426950408889634 / gamma;
  jeanie_fwd_kernel<T><<<B, JT, 0, st>>>(C, R, out, g, (T)kap, (T)(1.0 / kap));
  return check_launch<T>("jeanie forward");
}

template <typename T>
int jeanie_backward(const T* C, const T* R, const T* g_out, const T* g_R, int B, int K1, int K2,
                    int Tn, int U, int s1, int s2, double gamma, T* dC, cudaStream_t st) {
  if (B == 0) return kOk;
  JGrid g{K1, K2, K1 * K2, Tn, U, s1, s2};
  const double kap = 1.4426950408889634 / gamma;
  jeanie_bwd_kernel<T><<<B, JT, 0, st>>>(C, R, g_out, g_R, dC, g, (T)kap);
  return check_launch<T>("jeanie backward");
}

// The Euclidean cost from the clamped squared one, in place (n a multiple of 4,
// 16-byte aligned).
__global__ void sqrt_inplace_kernel(float4* __restrict__ c, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 v = c[i];
    v.x = sqrtf(v.x);
    v.y = sqrtf(v.y);
    v.z = sqrtf(v.z);
    v.w = sqrtf(v.w);
    c[i] = v;
  }
}

// The tensor-core route of the query/support cost and its chain rule (fp32):
// a real contraction (64 <= D <= 256) over enough rows and support frames to
// fill the 128 x 128 tiles, with the uDTW cost kernel's alignment rules.
inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

bool qs_tc_eligible(const float* q, const float* s, const float* c, int Rr, int U, int D) {
  return Rr >= 64 && U >= 32 && D <= 256 &&
         tc_cost_eligible(q, s, nullptr, nullptr, Rr, U, D, c, nullptr);
}

template <typename T>
int qs_cost(const T* q, const T* s, int B, int Rr, int U, int D, int metric, T* cost,
            cudaStream_t st) {
  if (B == 0 || Rr == 0) return kOk;
  if constexpr (sizeof(T) == 4) {
    if (qs_tc_eligible(q, s, cost, Rr, U, D)) {
      int rc = tc_cost_f32(q, s, nullptr, nullptr, B, Rr, U, D, 0.0, 1e-8, cost, nullptr,
                           nullptr, st);
      if (rc != kOk || metric != 1) return rc;
      const long long n4 = (long long)B * Rr * U / 4;
      const int grid = (int)(n4 / 256 + 1 < 4 * 148 ? n4 / 256 + 1 : 4 * 148);
      sqrt_inplace_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<float4*>(cost), n4);
      return check_launch<T>("euclidean cost");
    }
    if (qs_fast(q, s, nullptr, nullptr, B, Rr, U, D, metric, cost, nullptr, nullptr, st) == kOk)
      return check_launch<T>("query/support cost");
  }
  const size_t smem = (size_t)(CU * D + CU) * sizeof(T);
  if (smem > 200 * 1024) return set_error(kUnsupported, "feature dimension %d too large", D);
  auto kern = qs_cost_kernel<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return set_error(kLaunch, "qs cost: shared memory");
  int gx = (Rr + JT - 1) / JT;
  gx = gx > 64 ? 64 : gx;
  dim3 grid(gx, B);
  kern<<<grid, JT, smem, st>>>(q, s, Rr, U, D, metric, cost);
  return check_launch<T>("query/support cost");
}

template <typename T>
int qs_grad(const T* q, const T* s, const T* cost, const T* dcost, int B, int Rr, int U, int D,
            int metric, T* dq, T* ds, cudaStream_t st) {
  if (B == 0 || Rr == 0) return kOk;
  if constexpr (sizeof(T) == 4) {
    if (qs_tc_eligible(q, s, cost, Rr, U, D) && al16(dcost) && al16(dq) && al16(ds))
      return tc_qs_grad_f32(q, s, cost, dcost, B, Rr, U, D, metric == 1 ? 1 : 0, dq, ds, st);
    if (qs_fast(q, s, cost, dcost, B, Rr, U, D, metric, nullptr, dq, ds, st) == kOk)
      return check_launch<T>("query/support gradient");
  }
  const size_t smem = ((size_t)GR * GU + (size_t)GU * GF + (size_t)GR * GU * GF + GU) * sizeof(T);
  auto kern = qs_grad_kernel<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return set_error(kLaunch, "qs grad: shared memory");
  dim3 grid((D + GF - 1) / GF, B);
  for (int u0 = 0; u0 < U; u0 += GU) {
    const int nu = U - u0 < GU ? U - u0 : GU;
    kern<<<grid, GF * GR, smem, st>>>(q, s, cost, dcost, Rr, U, D, metric, u0, nu, u0 > 0, dq, ds);
  }
  return check_launch<T>("query/support gradient");
}

// ------------------------------------------------------------ rbf cost
// cost_ru = sum_d [2 - 2 exp(-sigma (q_rd - s_ud)^2)] (jeanie/distances.py:41-51),
// computed without the [R, U, D] difference tensor the PyTorch form builds.
// Each dimension adds -2 expm1(-sigma delta^2), which is 2 - 2 e^(-sigma delta^2)
// without cancellation for close frames.  Same chunking as qs_cost_kernel: CU
// support frames in shared memory, one query row per thread.
template <typename T>
__global__ void __launch_bounds__(JT) qs_rbf_cost_kernel(const T* __restrict__ q,
                                                         const T* __restrict__ s, int Rr, int U,
                                                         int D, T sigma, T* __restrict__ cost) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ss = reinterpret_cast<T*>(smem_raw);  // [CU][D]
  const int b = blockIdx.y;
  const T* qb = q + (long long)b * Rr * D;
  const T* sb = s + (long long)b * U * D;
  for (int u0 = 0; u0 < U; u0 += CU) {
    const int nu = min(CU, U - u0);
    __syncthreads();
    for (int e = threadIdx.x; e < CU * D; e += JT)
      ss[e] = e < nu * D ? sb[(long long)u0 * D + e] : T(0);
    __syncthreads();
    for (int r = blockIdx.x * JT + threadIdx.x; r < Rr; r += gridDim.x * JT) {
      const T* qr = qb + (long long)r * D;
      T acc[CU];
#pragma unroll
      for (int u = 0; u < CU; ++u) acc[u] = T(0);
      for (int d = 0; d < D; ++d) {
        const T v = qr[d];
#pragma unroll
        for (int u = 0; u < CU; ++u) {
          const T dl = v - ss[u * D + d];
          acc[u] -= expm1(-sigma * dl * dl);
        }
      }
      T* cr = cost + ((long long)b * Rr + r) * U + u0;
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        if (u >= nu) break;
        cr[u] = T(2) * acc[u];
      }
    }
  }
}

// d_cost -> d_query: dq_rd = 4 sigma sum_u dcost_ru (q_rd - s_ud) e^(-sigma (q_rd - s_ud)^2).
// One thread per (pair, row, feature), features fastest (coalesced q, s, dq;
// the row's dcost values are shared by the warp).
template <typename T>
__global__ void __launch_bounds__(256) qs_rbf_dq_kernel(const T* __restrict__ q,
                                                        const T* __restrict__ s,
                                                        const T* __restrict__ dcost, int B,
                                                        int Rr, int U, int D, T sigma,
                                                        T* __restrict__ dq) {
  const long long n = (long long)B * Rr * D;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
    const int d = (int)(i % D);
    const long long br = i / D;  // b * Rr + r
    const int b = (int)(br / Rr);
    const T v = q[i];
    const T* g = dcost + br * U;
    const T* sb = s + (long long)b * U * D + d;
    T acc = T(0);
    for (int u = 0; u < U; ++u) {
      const T dl = v - sb[(long long)u * D];
      acc += g[u] * dl * exp(-sigma * dl * dl);
    }
    dq[i] = T(4) * sigma * acc;
  }
}

// d_cost -> d_support: ds_ud = -4 sigma sum_r dcost_ru (q_rd - s_ud) e^(-sigma (q_rd - s_ud)^2),
// one thread per (pair, support frame, feature), rows summed in order.
template <typename T>
__global__ void __launch_bounds__(256) qs_rbf_ds_kernel(const T* __restrict__ q,
                                                        const T* __restrict__ s,
                                                        const T* __restrict__ dcost, int B,
                                                        int Rr, int U, int D, T sigma,
                                                        T* __restrict__ ds) {
  const long long n = (long long)B * U * D;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
    const int d = (int)(i % D);
    const long long bu = i / D;  // b * U + u
    const int b = (int)(bu / U);
    const int u = (int)(bu - (long long)b * U);
    const T sv = s[i];
    const T* qb = q + (long long)b * Rr * D + d;
    const T* g = dcost + (long long)b * Rr * U + u;
    T acc = T(0);
    for (int r = 0; r < Rr; ++r) {
      const T dl = qb[(long long)r * D] - sv;
      acc += g[(long long)r * U] * dl * exp(-sigma * dl * dl);
    }
    ds[i] = -T(4) * sigma * acc;
  }
}

template <typename T>
int qs_rbf_cost(const T* q, const T* s, int B, int Rr, int U, int D, double sigma, T* cost,
                cudaStream_t st) {
  if (B == 0 || Rr == 0 || U == 0) return kOk;
  const size_t smem = (size_t)CU * D * sizeof(T);
  if (smem > 200 * 1024) return set_error(kUnsupported, "feature dimension %d too large", D);
  auto kern = qs_rbf_cost_kernel<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return set_error(kLaunch, "rbf cost: shared memory");
  int gx = (Rr + JT - 1) / JT;
  gx = gx > 64 ? 64 : gx;
  dim3 grid(gx, B);
  kern<<<grid, JT, smem, st>>>(q, s, Rr, U, D, (T)sigma, cost);
  return check_launch<T>("rbf cost");
}

template <typename T>
int qs_rbf_grad(const T* q, const T* s, const T* dcost, int B, int Rr, int U, int D,
                double sigma, T* dq, T* ds, cudaStream_t st) {
  if (B == 0) return kOk;
  auto blocks = [](long long n) {
    long long g = (n + 255) / 256;
    return (int)(g < 1 ? 1 : (g > 148 * 32 ? 148 * 32 : g));
  };
  const long long nq = (long long)B * Rr * D, ns = (long long)B * U * D;
  if (nq > 0) qs_rbf_dq_kernel<T><<<blocks(nq), 256, 0, st>>>(q, s, dcost, B, Rr, U, D, (T)sigma, dq);
  if (ns > 0) qs_rbf_ds_kernel<T><<<blocks(ns), 256, 0, st>>>(q, s, dcost, B, Rr, U, D, (T)sigma, ds);
  return check_launch<T>("rbf cost gradient");
}

template <typename T>
int fvm_softmin(const T* cost, int B, int Kf, int TU, double gamma, T* temporal, cudaStream_t st) {
  if (B == 0 || TU == 0) return kOk;
  const double kap = 1.4426950408889634 / gamma;
  dim3 grid((TU + 255) / 256, B);
  fvm_softmin_kernel<T><<<grid, 256, 0, st>>>(cost, Kf, TU, (T)kap, (T)(1.0 / kap), temporal);
  return check_launch<T>("fvm soft-min");
}

template <typename T>
int fvm_softmin_bwd(const T* cost, const T* dtemp, int B, int Kf, int TU, double gamma, T* dcost,
                    cudaStream_t st) {
  if (B == 0 || TU == 0) return kOk;
  const double kap = 1.4426950408889634 / gamma;
  dim3 grid((TU + 255) / 256, B);
  fvm_softmin_bwd_kernel<T><<<grid, 256, 0, st>>>(cost, dtemp, Kf, TU, (T)kap, dcost);
  return check_launch<T>("fvm soft-min backward");
}

#define TW_INST(T)                                                                               \
  template int jeanie_forward<T>(const T*, int, int, int, int, int, int, int, double, T*, T*,   \
                                 cudaStream_t);                                                  \
  template int jeanie_backward<T>(const T*, const T*, const T*, const T*, int, int, int, int,  \
                                  int, int, int, double, T*, cudaStream_t);                     \
  template int qs_cost<T>(const T*, const T*, int, int, int, int, int, T*, cudaStream_t);      \
  template int qs_grad<T>(const T*, const T*, const T*, const T*, int, int, int, int, int, T*, \
                          T*, cudaStream_t);                                                     \
  template int qs_rbf_cost<T>(const T*, const T*, int, int, int, int, double, T*,             \
                              cudaStream_t);                                                     \
  template int qs_rbf_grad<T>(const T*, const T*, const T*, int, int, int, int, double, T*, T*, \
                              cudaStream_t);                                                     \
  template int fvm_softmin<T>(const T*, int, int, int, double, T*, cudaStream_t);              \
  template int fvm_softmin_bwd<T>(const T*, const T*, int, int, int, double, T*, cudaStream_t);
TW_INST(float)
TW_INST(double)
#undef TW_INST

}  // namespace tw
