// Pairwise uDTW / soft-DTW cost from features and its chain rule, SIMT tiles.
//
// Cost (hibana2077/torchwarp src/torchwarp/csrc/udtw_cuda.cu:379-387 and
// src/torchwarp/udtw/_autograd.py:24-29):
//   sq = max(|x_i|^2 + |y_j|^2 - 2 x_i.y_j, 0), var = max(0.5 (vx_i + vy_j), eps)
//   C = sq / var, Q = beta * log(var)
// Chain rule (udtw_cuda.cu:557-568, udtw/_ops.py:179-183, 200-211):
//   dsq = dC / var  where sq_raw > 0 (equivalently C > 0), else 0
//   dvar = (beta dQ - dC C) / var  where var_raw > eps, else 0
//   dX = -2 dsq Y + 2 X rowsum(dsq), dY = -2 dsq^T X + 2 Y colsum(dsq)
//   dvx = 0.5 rowsum(dvar), dvy = 0.5 colsum(dvar)
// One CTA owns a 64 x 64 tile of (i, j) cells (cost) or a 64-row / 64-column
// strip (gradients); no atomics, so every result is bitwise reproducible.
// fp32 with D >= 64 goes to the tensor-core kernels of tc_gemm.cu instead.
#include "common.cuh"

namespace tw {
namespace {

constexpr int TM = 64;   // tile edge (cells)
constexpr int KC = 32;   // feature chunk

template <typename T>
__global__ void __launch_bounds__(256) udtw_cost_kernel(const T* __restrict__ X,
                                                        const T* __restrict__ Y,
                                                        const T* __restrict__ vx,
                                                        const T* __restrict__ vy, int N, int M,
                                                        int D, T beta, T eps, T* __restrict__ C,
                                                        T* __restrict__ Q,
                                                        uint32_t* __restrict__ mask) {
  __shared__ T Xs[TM][KC + 1];
  __shared__ T Ys[TM][KC + 1];
  __shared__ uint32_t pos[TM][TM / 32];  // positivity bits of the tile's cells
  const int b = blockIdx.z;
  const int i0 = blockIdx.y * TM, j0 = blockIdx.x * TM;
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const T* Xb = X + (long long)b * N * D;
  const T* Yb = Y + (long long)b * M * D;
  T acc[4][4] = {};
  T x2[4] = {}, y2[4] = {};
  for (int d0 = 0; d0 < D; d0 += KC) {
    for (int e = tid; e < TM * KC; e += 256) {
      const int r = e / KC, d = e % KC;
      const int gi = i0 + r, gj = j0 + r, gd = d0 + d;
      Xs[r][d] = (gi < N && gd < D) ? Xb[(long long)gi * D + gd] : T(0);
      Ys[r][d] = (gj < M && gd < D) ? Yb[(long long)gj * D + gd] : T(0);
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < KC; ++d) {
      T xa[4], yb[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xa[a] = Xs[ty * 4 + a][d];
#pragma unroll
      for (int c = 0; c < 4; ++c) yb[c] = Ys[tx * 4 + c][d];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        x2[a] += xa[a] * xa[a];
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] += xa[a] * yb[c];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) y2[c] += yb[c] * yb[c];
    }
    __syncthreads();
  }
  if (mask != nullptr) {
    if (tid < TM * TM / 32) pos[tid >> 1][tid & 1] = 0u;
    __syncthreads();
  }
  for (int a = 0; a < 4; ++a) {
    const int i = i0 + ty * 4 + a;
    if (i >= N) continue;
    for (int c = 0; c < 4; ++c) {
      const int j = j0 + tx * 4 + c;
      if (j >= M) continue;
      T sq = (x2[a] + y2[c]) - T(2) * acc[a][c];
      if (mask != nullptr && sq > T(0))
        atomicOr(&pos[ty * 4 + a][(tx * 4 + c) >> 5], 1u << ((tx * 4 + c) & 31));
      sq = sq > T(0) ? sq : T(0);
      T var = T(1);
      if (vx != nullptr) {
        var = T(0.5) * (vx[(long long)b * N + i] + vy[(long long)b * M + j]);
        var = var > eps ? var : eps;
      }
      const long long o = ((long long)b * N + i) * M + j;
      C[o] = sq / var;
      if (Q != nullptr) Q[o] = beta * log(var);
    }
  }
  if (mask != nullptr) {
    // words [b][j0/32 + w][i] (rows padded to NP = 4 ceil(N/4), padding rows
    // zero): j0 is a multiple of 64, so each tile owns 2 words per row
    __syncthreads();
    const int MW = (M + 31) >> 5, NP = (N + 3) & ~3;
    if (tid < TM * TM / 32) {
      const int r = tid >> 1, w = tid & 1;
      const int i = i0 + r, jw = (j0 >> 5) + w;
      if (i < NP && jw < MW) mask[((long long)b * MW + jw) * NP + i] = pos[r][w];
    }
  }
}

// One side of the chain rule: a CTA owns a strip of 64 rows of the gradient
// (rows of X for SIDE 0, rows of Y for SIDE 1) and 64 features, sweeping the
// summed index (j for SIDE 0, i for SIDE 1) in chunks of 32 cells.
template <typename T, int SIDE>
__global__ void __launch_bounds__(256) udtw_grad_strip_kernel(
    const T* __restrict__ A, const T* __restrict__ Bf, const T* __restrict__ va,
    const T* __restrict__ vb, const T* __restrict__ C, const T* __restrict__ dC,
    const T* __restrict__ dQ, int N, int M, int D, T beta, T eps, T* __restrict__ dA,
    T* __restrict__ dva, const uint32_t* __restrict__ mask) {
  constexpr int TS = 32;
  __shared__ T Gs[TM][TS + 1];   // dsq [strip row][summed index]
  __shared__ T Bs[TS][TM + 1];   // other side's features [summed index][feature]
  __shared__ T rs[TM];
  const int b = blockIdx.z;
  const int r0 = blockIdx.y * TM;   // strip rows
  const int f0 = blockIdx.x * TM;   // feature chunk
  const int R = SIDE == 0 ? N : M;  // strip extent
  const int S = SIDE == 0 ? M : N;  // summed extent
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int rr = tid >> 2, cq = tid & 3;
  const T* Ab = A + (long long)b * R * D;
  const T* Bb = Bf + (long long)b * S * D;
  T acc[4][4] = {};
  T rsum = T(0), vsum = T(0);
  for (int s0 = 0; s0 < S; s0 += TS) {
#pragma unroll
    for (int c = 0; c < TS / 4; ++c) {
      const int ss = cq * (TS / 4) + c;
      const int gr = r0 + rr, gs = s0 + ss;
      T g = T(0);
      if (gr < R && gs < S) {
        const int i = SIDE == 0 ? gr : gs, j = SIDE == 0 ? gs : gr;
        const long long o = ((long long)b * N + i) * M + j;
        T var = T(1), var_raw = T(1);
        if (va != nullptr) {
          const T vi = SIDE == 0 ? va[(long long)b * N + i] : vb[(long long)b * N + i];
          const T vj = SIDE == 0 ? vb[(long long)b * M + j] : va[(long long)b * M + j];
          var_raw = T(0.5) * (vi + vj);
          var = var_raw > eps ? var_raw : eps;
        }
        const T dc = dC[o];
        bool positive;
        T cc = T(0);
        if (mask != nullptr) {
          const int MW = (M + 31) >> 5, NP = (N + 3) & ~3;
          positive = (mask[((long long)b * MW + (j >> 5)) * NP + i] >> (j & 31)) & 1u;
        } else if (C != nullptr) {
          cc = C[o];
          positive = cc > T(0);
        } else {
          positive = true;  // dC already carries the positivity mask
        }
        g = positive ? dc / var : T(0);
        if (va != nullptr && var_raw > eps) {
          const T dq = dQ != nullptr ? dQ[o] : T(0);
          vsum += (beta * dq - dc * cc) / var;
        }
      }
      Gs[rr][ss] = g;
      rsum += g;
    }
    for (int e = tid; e < TS * TM; e += 256) {
      const int ss = e / TM, ff = e % TM;
      const int gs = s0 + ss, gf = f0 + ff;
      Bs[ss][ff] = (gs < S && gf < D) ? Bb[(long long)gs * D + gf] : T(0);
    }
    __syncthreads();
#pragma unroll 4
    for (int ss = 0; ss < TS; ++ss) {
      T ga[4], bf[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) ga[a] = Gs[ty * 4 + a][ss];
#pragma unroll
      for (int c = 0; c < 4; ++c) bf[c] = Bs[ss][tx * 4 + c];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] += ga[a] * bf[c];
    }
    __syncthreads();
  }
  // the four threads of a strip row are adjacent lanes: combine their sums
  rsum += __shfl_xor_sync(0xffffffffu, rsum, 1);
  rsum += __shfl_xor_sync(0xffffffffu, rsum, 2);
  vsum += __shfl_xor_sync(0xffffffffu, vsum, 1);
  vsum += __shfl_xor_sync(0xffffffffu, vsum, 2);
  if (cq == 0) rs[rr] = rsum;
  if (cq == 0 && blockIdx.x == 0 && dva != nullptr && r0 + rr < R)
    dva[(long long)b * R + r0 + rr] = T(0.5) * vsum;
  __syncthreads();
  for (int a = 0; a < 4; ++a) {
    const int gr = r0 + ty * 4 + a;
    if (gr >= R) continue;
    for (int c = 0; c < 4; ++c) {
      const int gf = f0 + tx * 4 + c;
      if (gf >= D) continue;
      const long long o = ((long long)b * R + gr) * D + gf;
      dA[o] = T(-2) * acc[a][c] + T(2) * Ab[(long long)gr * D + gf] * rs[ty * 4 + a];
    }
  }
}

template <typename T>
int cost_launch(const T* X, const T* Y, const T* vx, const T* vy, int B, int N, int M, int D,
                double beta, double eps, T* C, T* Q, cudaStream_t st, uint32_t* mask = nullptr) {
  if (B == 0 || N == 0 || M == 0) return kOk;
  dim3 grid((M + TM - 1) / TM, (N + TM - 1) / TM, B);
  udtw_cost_kernel<T><<<grid, 256, 0, st>>>(X, Y, vx, vy, N, M, D, (T)beta, (T)eps, C, Q, mask);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "udtw cost launch: %s", cudaGetErrorString(e));
  return kOk;
}

template <typename T>
int grad_launch(const T* X, const T* Y, const T* vx, const T* vy, const T* C, const T* dC,
                const T* dQ, int B, int N, int M, int D, double beta, double eps, T* dX, T* dY,
                T* dvx, T* dvy, cudaStream_t st, const uint32_t* mask = nullptr) {
  if (B == 0 || N == 0 || M == 0) return kOk;
  const int fch = (D + TM - 1) / TM;
  dim3 gx(fch, (N + TM - 1) / TM, B), gy(fch, (M + TM - 1) / TM, B);
  udtw_grad_strip_kernel<T, 0><<<gx, 256, 0, st>>>(X, Y, vx, vy, C, dC, dQ, N, M, D, (T)beta,
                                                    (T)eps, dX, vx ? dvx : nullptr, mask);
  udtw_grad_strip_kernel<T, 1><<<gy, 256, 0, st>>>(Y, X, vy, vx, C, dC, dQ, N, M, D, (T)beta,
                                                    (T)eps, dY, vx ? dvy : nullptr, mask);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "udtw grad launch: %s", cudaGetErrorString(e));
  return kOk;
}

}  // namespace

// Tensor-core forms (tc_gemm.cu), used for fp32 when they apply.
bool tc_cost_eligible(const float* X, const float* Y, const float* vx, const float* vy, int N,
                      int M, int D, const float* C, const float* Q);
int tc_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B, int N,
                int M, int D, double beta, double eps, float* C, float* Q, uint32_t* mask,
                cudaStream_t st);
int tc_sq_grad_f32(const float* X, const float* Y, const uint32_t* mask, const float* dC, int B,
                   int N, int M, int D, float* dX, float* dY, cudaStream_t st,
                   const uint8_t* tf_rows = nullptr, const uint8_t* tf_cols = nullptr);
bool tc_grad_eligible(const float* X, const float* Y, const float* C, const float* dC,
                      const float* dQ, const float* dX, const float* dY, int M, int D);
int tc_grad_f32(const float* X, const float* Y, const float* vx, const float* vy, const float* C,
                const float* dC, const float* dQ, int B, int N, int M, int D, double beta,
                double eps, float* dX, float* dY, float* dvx, float* dvy, cudaStream_t st,
                const uint8_t* tf_rows = nullptr, const uint8_t* tf_cols = nullptr);

int udtw_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B, int N,
                  int M, int D, double beta, double eps, float* C, float* Q, cudaStream_t st) {
  if (tc_cost_eligible(X, Y, vx, vy, N, M, D, C, Q))
    return tc_cost_f32(X, Y, vx, vy, B, N, M, D, beta, eps, C, Q, nullptr, st);
  return cost_launch(X, Y, vx, vy, B, N, M, D, beta, eps, C, Q, st);
}
int udtw_cost_f64(const double* X, const double* Y, const double* vx, const double* vy, int B,
                  int N, int M, int D, double beta, double eps, double* C, double* Q,
                  cudaStream_t st) {
  return cost_launch(X, Y, vx, vy, B, N, M, D, beta, eps, C, Q, st);
}
int udtw_grad_f32(const float* X, const float* Y, const float* vx, const float* vy, const float* C,
                  const float* dC, const float* dQ, int B, int N, int M, int D, double beta,
                  double eps, float* dX, float* dY, float* dvx, float* dvy, cudaStream_t st,
                  const uint8_t* tf_rows, const uint8_t* tf_cols) {
  if (tc_grad_eligible(X, Y, C, dC, dQ, dX, dY, M, D))
    return tc_grad_f32(X, Y, vx, vy, C, dC, dQ, B, N, M, D, beta, eps, dX, dY, dvx, dvy, st,
                       tf_rows, tf_cols);
  return grad_launch(X, Y, vx, vy, C, dC, dQ, B, N, M, D, beta, eps, dX, dY, dvx, dvy, st);
}
int udtw_grad_f64(const double* X, const double* Y, const double* vx, const double* vy,
                  const double* C, const double* dC, const double* dQ, int B, int N, int M, int D,
                  double beta, double eps, double* dX, double* dY, double* dvx, double* dvy,
                  cudaStream_t st) {
  return grad_launch(X, Y, vx, vy, C, dC, dQ, B, N, M, D, beta, eps, dX, dY, dvx, dvy, st);
}

// Squared-Euclidean cost with its positivity mask (bit j & 31 of word
// [b][j >> 5][i] set where sq_raw > 0; rows padded to 4 ceil(N/4)), and the
// chain rule that takes the mask in place of the cost.
int sq_cost_f32(const float* X, const float* Y, int B, int N, int M, int D, float* C,
                uint32_t* mask, cudaStream_t st) {
  if (tc_cost_eligible(X, Y, nullptr, nullptr, N, M, D, C, nullptr))
    return tc_cost_f32(X, Y, nullptr, nullptr, B, N, M, D, 0.0, 1e-8, C, nullptr, mask, st);
  return cost_launch<float>(X, Y, nullptr, nullptr, B, N, M, D, 0.0, 1e-8, C, nullptr, st, mask);
}
int sq_cost_f64(const double* X, const double* Y, int B, int N, int M, int D, double* C,
                uint32_t* mask, cudaStream_t st) {
  return cost_launch<double>(X, Y, nullptr, nullptr, B, N, M, D, 0.0, 1e-8, C, nullptr, st, mask);
}
int sq_grad_f32(const float* X, const float* Y, const uint32_t* mask, const float* dC, int B,
                int N, int M, int D, float* dX, float* dY, cudaStream_t st) {
  if (tc_grad_eligible(X, Y, dC, dC, nullptr, dX, dY, M, D))
    return tc_sq_grad_f32(X, Y, mask, dC, B, N, M, D, dX, dY, st);
  return grad_launch<float>(X, Y, nullptr, nullptr, nullptr, dC, nullptr, B, N, M, D, 0.0, 1e-8,
                            dX, dY, nullptr, nullptr, st, mask);
}
// The soft-DTW chain rule after tw_sdtw_backward_masked (S = dC): true when
// it runs on tensor cores, which then skip the chunks of dC that the DP
// backward flagged as all zero (tf_rows / tf_cols, see tc_sq_grad_f32).
bool sq_grad_flagged_eligible(const float* X, const float* Y, const float* dC, const float* dX,
                              const float* dY, int M, int D) {
  return tc_grad_eligible(X, Y, dC, dC, nullptr, dX, dY, M, D);
}
// mask: null (S = dC), or the mask of the cells of dC that hold S (the others
// are 0 whatever dC holds there, e.g. dC written sparsely by the backward).
int sq_grad_flagged_f32(const float* X, const float* Y, const uint32_t* mask, const float* dC,
                        int B, int N, int M, int D, float* dX, float* dY,
                        const uint8_t* tf_rows, const uint8_t* tf_cols, cudaStream_t st) {
  if (sq_grad_flagged_eligible(X, Y, dC, dX, dY, M, D))
    return tc_sq_grad_f32(X, Y, mask, dC, B, N, M, D, dX, dY, st, tf_rows, tf_cols);
  return grad_launch<float>(X, Y, nullptr, nullptr, nullptr, dC, nullptr, B, N, M, D, 0.0, 1e-8,
                            dX, dY, nullptr, nullptr, st, mask);
}
int sq_grad_f64(const double* X, const double* Y, const uint32_t* mask, const double* dC, int B,
                int N, int M, int D, double* dX, double* dY, cudaStream_t st) {
  return grad_launch<double>(X, Y, nullptr, nullptr, nullptr, dC, nullptr, B, N, M, D, 0.0, 1e-8,
                             dX, dY, nullptr, nullptr, st, mask);
}

}  // namespace tw
