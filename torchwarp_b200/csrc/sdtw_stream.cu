// Warp-stream soft-DTW / uDTW forward and backward kernels; see sdtw_stream.cuh.
//
// Recurrences (hibana2077/torchwarp src/torchwarp/csrc/udtw_cuda.cu:13-21,
// src/torchwarp/udtw/_torch_dp.py:14-76), written here in the log2 domain
// R' = R * log2(e)/gamma, C' = C * log2(e)/gamma:
//   forward : R'_s = C'_s + m - log2(1 + 2^(m - o1) + 2^(m - o2)),
//             m = min of the three predecessor R', o1, o2 the other two;
//             P_s  = Q_s + sum_p w_p P_p,  w = softmax over predecessors.
//   backward (push form): cell s hands w_p * (Rbar_s - Pbar_s (P_p - A_s)/gamma)
//             to each predecessor p (A_s = sum_p w_p P_p), and w_p * Pbar_s to
//             its Pbar; w_p is recomputed from the saved R' of the predecessors.
#include <climits>

#include "sdtw_stream.cuh"

namespace tw {
namespace {

template <typename T> struct RingStride;
// Row stride (elements) of the per-lane cost rings: lane l reads column
// (t - l) of row l, so the bank of its word is (l*(S-1) + t) mod 32; S-1 odd
// (and S*elem a multiple of 16 bytes for cp.async) makes the read conflict-free.
template <> struct RingStride<float> { static constexpr int value = 68; };
template <> struct RingStride<double> { static constexpr int value = 66; };

constexpr int RING = 64;   // stream columns a lane row can hold
constexpr int TILE = 8;    // columns per copy tile / flush tile
constexpr int LEAD = 3;    // forward: cost tiles issued ahead of use
constexpr int SROWS = 32;  // backward: saved-stream rows staged in shared memory

__device__ __forceinline__ int floor_div(int a, int b) {
  const int q = a / b;
  return (a % b != 0 && a < 0) ? q - 1 : q;
}
__device__ __forceinline__ int pos_mod(int a, int b) {
  const int r = a % b;
  return r < 0 ? r + b : r;
}

struct WarpInfo {
  int w, wib, lane, npairs, p0, Q, Tw;
};

__device__ __forceinline__ bool warp_setup(const StreamPlan& p, int KS, WarpInfo& wi) {
  wi.lane = threadIdx.x & 31;
  wi.wib = threadIdx.x >> 5;
  wi.w = blockIdx.x * (blockDim.x >> 5) + wi.wib;
  if (wi.w >= p.warps) return false;
  wi.npairs = p.base + (wi.w < p.rem ? 1 : 0);
  if (wi.npairs == 0) return false;
  wi.p0 = wi.w * p.base + min(wi.w, p.rem);
  wi.Q = wi.npairs * p.NB;
  wi.Tw = wi.Q * p.L + 32 * KS - 1;
  return true;
}

// ---------------------------------------------------------------- forward

// Copy the 8 stream columns [8u, 8u+8) of this lane's row of sub-band k into
// its ring row (cp.async, zero-filled outside the data).
template <typename T, int KS>
__device__ __forceinline__ void load_row_tile(const T* __restrict__ src_base, T* ring_row, int u,
                                              int k, const StreamPlan& p, const WarpInfo& wi,
                                              int vec) {
  if (u < 0) return;
  const int sc0 = u * TILE;
  const int q = sc0 / p.L;
  if (q >= wi.Q) return;
  const int j0 = sc0 - q * p.L;
  if (j0 >= p.M) return;  // all padding: patched, never read from memory
  const int pq = q / p.NB;
  const int band = q - pq * p.NB;
  const int row = band * 32 * KS + 32 * k + wi.lane;
  const bool rv = row < p.N;
  T* dst = ring_row + (sc0 & (RING - 1));
  const T* src = src_base + ((long long)(wi.p0 + pq) * p.N + (rv ? row : 0)) * p.M;
  if (vec) {
    constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
    for (int h = 0; h < TILE / PER; ++h) {
      const int j = j0 + h * PER;
      int cnt = rv ? min(PER, p.M - j) : 0;
      cnt = cnt < 0 ? 0 : cnt;
      cp_async16(dst + h * PER, cnt > 0 ? (const void*)(src + j) : (const void*)src_base,
                 cnt * (int)sizeof(T));
    }
  } else {
#pragma unroll
    for (int h = 0; h < TILE; ++h) {
      const int j = j0 + h;
      const bool v = rv && j < p.M;
      cp_async_elem<sizeof(T)>(dst + h, v ? (const void*)(src + j) : (const void*)src_base,
                               v ? (int)sizeof(T) : 0);
    }
  }
}

// Padding columns j >= M of a landed tile get the raw cost Big/kappa.
template <typename T>
__device__ __forceinline__ void patch_row_tile(T* ring_row, int u, const StreamPlan& p,
                                               const WarpInfo& wi, T padv) {
  if (u < 0) return;
  const int sc0 = u * TILE;
  const int q = sc0 / p.L;
  if (q >= wi.Q) return;
  const int j0 = sc0 - q * p.L;
  if (j0 + TILE <= p.M) return;
  T* dst = ring_row + (sc0 & (RING - 1));
  for (int h = max(0, p.M - j0); h < TILE; ++h) dst[h] = padv;
}

// Value of "row -1" that lane 0 of sub-band 0 sees at stream column sc:
// the previous band's bottom row (delay line), +Big above a pair's first
// band, and 0 at the last column of a pass that precedes a first band (it is
// the diagonal predecessor of cell (0,0), R(-1,-1) = 0).  For P: 0 / delay line.
template <typename T>
__device__ __forceinline__ T row_above(const T* dl, int sc, const StreamPlan& p,
                                       const WarpInfo& wi, T first_value) {
  const int q = floor_div(sc, p.L);
  const int j = sc - q * p.L;
  const bool first = q < 0 || q >= wi.Q || pos_mod(q, p.NB) == 0;
  T v = first ? first_value : dl[j];
  if (j == p.L - 1 && pos_mod(q + 1, p.NB) == 0) v = T(0);
  return v;
}

template <typename T, bool HAS_P>
__device__ __forceinline__ void cell_forward(T c, T qv, T left, T up, T dg, T Pl, T Pu, T Pd,
                                             T& r, T& pv) {
  const T m1 = fmin(left, up), M1 = fmax(left, up);
  const T m = fmin(m1, dg), Mx = fmax(m1, dg);
  const T e1 = ex2(add_rn(m, -M1));
  const T e2 = ex2(add_rn(m, -Mx));
  const T s = add_rn(add_rn(T(1), e1), e2);
  r = add_rn(c, add_rn(m, -lg2(s)));
  if constexpr (HAS_P) {
    const bool p1 = left <= up;
    const bool p2 = m1 <= dg;
    const T wm1 = p2 ? T(1) : e2;
    const T wd = p2 ? e2 : T(1);
    const T wl = p1 ? wm1 : e1;
    const T wu = p1 ? e1 : wm1;
    pv = qv + (wl * Pl + wu * Pu + wd * Pd) * rcp(s);
  } else {
    pv = T(0);
  }
}

template <typename T, int KS, bool HAS_P, bool HAS_BAND>
__global__ void __launch_bounds__(128) sdtw_fwd_kernel(const SdtwArgs<T> a) {
  constexpr int S = RingStride<T>::value;
  constexpr int RW = KS * 32 * S;  // ring elements per operand per warp
  const StreamPlan& p = a.p;
  WarpInfo wi;
  if (!warp_setup(p, KS, wi)) return;
  const int lane = wi.lane;
  const T big = Big<T>::value;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* ringC = reinterpret_cast<T*>(smem_raw) + (size_t)wi.wib * RW * (HAS_P ? 2 : 1);
  T* ringQ = ringC + RW;
  for (int i = lane; i < RW; i += 32) {
    ringC[i] = a.pad_raw;
    if (HAS_P) ringQ[i] = T(0);
  }
  __syncwarp();
  T* myC = ringC + lane * S;
  T* myQ = ringQ + lane * S;

#pragma unroll 1
  for (int pb = -LEAD; pb < 0; ++pb) {
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      load_row_tile<T, KS>(a.C, myC + k * 32 * S, pb - 4 * k + LEAD, k, p, wi, a.vec);
      if (HAS_P) load_row_tile<T, KS>(a.Q, myQ + k * 32 * S, pb - 4 * k + LEAD, k, p, wi, a.vec);
    }
    cp_async_commit();
  }

  T left[KS], up[KS], dg[KS], Pl[KS], Pu[KS], Pd[KS];
  int jk[KS], rowk[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    left[k] = up[k] = dg[k] = big;
    Pl[k] = Pu[k] = Pd[k] = T(0);
    if (HAS_BAND) {
      const int sc = -32 * k - lane;
      const int q = floor_div(sc, p.L);
      jk[k] = sc - q * p.L;
      rowk[k] = pos_mod(q, p.NB) * 32 * KS + 32 * k + lane;
    }
  }
  if (lane == 0) dg[0] = T(0);

  const T* dlR = a.dlR + (long long)wi.w * p.L;
  const T* dlP = HAS_P ? a.dlP + (long long)wi.w * p.L : nullptr;
  T* dlRw = a.dlR + (long long)wi.w * p.L;
  T* dlPw = HAS_P ? a.dlP + (long long)wi.w * p.L : nullptr;
  T rbR = row_above(dlR, lane, p, wi, big), rbRn = row_above(dlR, 32 + lane, p, wi, big);
  T rbP = T(0), rbPn = T(0);
  if (HAS_P) {
    rbP = row_above(dlP, lane, p, wi, T(0));
    rbPn = row_above(dlP, 32 + lane, p, wi, T(0));
  }
  T wbR = T(0), wbP = T(0);

  const int rows = 32 * KS;
  const int kstar = ((p.N - 1) % rows) / 32, lstar = (p.N - 1) % 32;
  const long long NBL = (long long)p.NB * p.L;
  long long cap_t = (long long)((p.N - 1) / rows) * p.L + (p.M - 1) + 32 * kstar + lstar;
  int cap_i = 0;

  T* sR = a.sR + (long long)wi.w * p.tmax * KS * 32 + lane;
  T* sP = HAS_P ? a.sP + (long long)wi.w * p.tmax * KS * 32 + lane : nullptr;
  const T kap = a.kappa;

#pragma unroll 1
  for (int t0 = 0; t0 < wi.Tw; t0 += TILE) {
    cp_async_wait<LEAD - 1>();
#pragma unroll
    for (int k = 0; k < KS; ++k) patch_row_tile(myC + k * 32 * S, t0 / TILE - 4 * k, p, wi, a.pad_raw);
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      load_row_tile<T, KS>(a.C, myC + k * 32 * S, t0 / TILE - 4 * k + LEAD, k, p, wi, a.vec);
      if (HAS_P) load_row_tile<T, KS>(a.Q, myQ + k * 32 * S, t0 / TILE - 4 * k + LEAD, k, p, wi, a.vec);
    }
    cp_async_commit();

#pragma unroll
    for (int s = 0; s < TILE; ++s) {
      const int t = t0 + s;
      const int ia = (t - lane) & (RING - 1);
      T Rn[KS], Pn[KS];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const int off = k * 32 * S + ((k & 1) ? (ia ^ 32) : ia);
        const T c = myC[off] * kap;
        const T qv = HAS_P ? myQ[off] : T(0);
        cell_forward<T, HAS_P>(c, qv, left[k], up[k], dg[k], Pl[k], Pu[k], Pd[k], Rn[k], Pn[k]);
        if constexpr (HAS_BAND) {
          if (fabs((T)(rowk[k] - jk[k])) > a.band) {
            Rn[k] = big;
            Pn[k] = T(0);
          }
          if (++jk[k] == p.L) {
            jk[k] = 0;
            rowk[k] += rows;
            if (rowk[k] >= p.NB * rows) rowk[k] -= p.NB * rows;
          }
        }
        sR[((long long)t * KS + k) * 32] = Rn[k];
        if (HAS_P) sP[((long long)t * KS + k) * 32] = Pn[k];
      }

      if (t == cap_t) {
        T v = Rn[0], vp = Pn[0];
#pragma unroll
        for (int k = 1; k < KS; ++k)
          if (k == kstar) { v = Rn[k]; vp = Pn[k]; }
        if (lane == lstar) {
          a.out_r[wi.p0 + cap_i] = v >= big * T(0.5) ? T(INFINITY) : v * a.inv_kappa;
          if (HAS_P) a.out_p[wi.p0 + cap_i] = vp;
        }
        ++cap_i;
        cap_t = cap_i < wi.npairs ? cap_t + NBL : LLONG_MAX;
      }

      {  // bottom row of the band -> delay line (gathered 32 columns at a time)
        const int scb = t - 32 * (KS - 1) - 31;
        const T v = shfl(Rn[KS - 1], 31);
        const T vp = HAS_P ? shfl(Pn[KS - 1], 31) : T(0);
        if ((scb & 31) == lane) { wbR = v; wbP = vp; }
        if ((scb & 31) == 31) {
          const int scx = scb - 31 + lane;
          if (scx >= 0) {
            const int j = scx - (scx / p.L) * p.L;
            dlRw[j] = wbR;
            if (HAS_P) dlPw[j] = wbP;
          }
          __syncwarp();
        }
      }

      if (((t + 1) & 31) == 0) {
        rbR = rbRn;
        rbRn = row_above(dlR, t + 33 + lane, p, wi, big);
        if (HAS_P) {
          rbP = rbPn;
          rbPn = row_above(dlP, t + 33 + lane, p, wi, T(0));
        }
      }
      const T bv = shfl(rbR, (t + 1) & 31);
      const T bp = HAS_P ? shfl(rbP, (t + 1) & 31) : T(0);

#pragma unroll
      for (int k = 0; k < KS; ++k) {
        dg[k] = up[k];
        left[k] = Rn[k];
        if (HAS_P) { Pd[k] = Pu[k]; Pl[k] = Pn[k]; }
      }
#pragma unroll
      for (int k = KS - 1; k >= 1; --k) {
        up[k] = shfl_up1_rot(lane == 31 ? Rn[k - 1] : Rn[k]);
        if (HAS_P) Pu[k] = shfl_up1_rot(lane == 31 ? Pn[k - 1] : Pn[k]);
      }
      up[0] = shfl_up1_rot(lane == 31 ? bv : Rn[0]);
      if (HAS_P) Pu[0] = shfl_up1_rot(lane == 31 ? bp : Pn[0]);
    }
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------- backward

// Copy saved rows [8c, 8c+8) (contiguous: 8*KS*32 elements) into slot c&3.
template <typename T, int KS>
__device__ __forceinline__ void load_saved_chunk(const T* __restrict__ src_warp, T* ring, int c,
                                                 int lane) {
  if (c < 0) return;
  constexpr int ELEMS = TILE * KS * 32;
  constexpr int PER = 16 / (int)sizeof(T);
  const T* src = src_warp + (long long)c * ELEMS;
  T* dst = ring + (c & 3) * ELEMS;
#pragma unroll
  for (int i = lane; i < ELEMS / PER; i += 32) cp_async16(dst + i * PER, src + i * PER, 16);
}

template <typename T, int KS>
__device__ __forceinline__ T saved_at(const T* ring, int row, int k, int lane, T big) {
  constexpr int ELEMS = TILE * KS * 32;
  if (row < 0) return big;
  return ring[((row >> 3) & 3) * ELEMS + ((row & 7) * KS + k) * 32 + lane];
}

// Row -1 value lane 0 of sub-band 0 used at stream column sc in the forward
// sweep, re-read from the saved stream (bottom row of the previous band).
template <typename T, int KS>
__device__ __forceinline__ T row_above_saved(const T* s_warp, int sc, const StreamPlan& p,
                                             const WarpInfo& wi, T first_value) {
  const int q = floor_div(sc, p.L);
  const int j = sc - q * p.L;
  const bool first = q < 0 || q >= wi.Q || pos_mod(q, p.NB) == 0;
  T v = first_value;
  if (!first) v = s_warp[((long long)(sc - p.L + 32 * KS - 1) * KS + (KS - 1)) * 32 + 31];
  if (j == p.L - 1 && pos_mod(q + 1, p.NB) == 0) v = T(0);
  return v;
}

// Adjoint pushed into the bottom row of the band at stream column sc from the
// next band's top row (delay line); zero when the next band starts a new pair.
template <typename T>
__device__ __forceinline__ T push_from_below(const T* dl, int sc, const StreamPlan& p,
                                             const WarpInfo& wi) {
  if (sc < 0) return T(0);
  const int q = sc / p.L;
  const int j = sc - q * p.L;
  if (q + 1 >= wi.Q || (q + 1) % p.NB == 0) return T(0);
  return dl[j];
}

template <typename T, bool HAS_P>
__device__ __forceinline__ void cell_backward(T Rl, T Ru, T Rd, T Pl, T Pu, T Pd, T rbar, T pbar,
                                              T inv_gamma, T& pl, T& pu, T& pd, T& ql, T& qu,
                                              T& qd) {
  const T m1 = fmin(Rl, Ru), M1 = fmax(Rl, Ru);
  const T m = fmin(m1, Rd), Mx = fmax(m1, Rd);
  const T e1 = ex2(add_rn(m, -M1));
  const T e2 = ex2(add_rn(m, -Mx));
  const T inv = rcp(add_rn(add_rn(T(1), e1), e2));
  const bool p1 = Rl <= Ru;
  const bool p2 = m1 <= Rd;
  const T wm1 = p2 ? T(1) : e2;
  const T wd = (p2 ? e2 : T(1)) * inv;
  const T wl = (p1 ? wm1 : e1) * inv;
  const T wu = (p1 ? e1 : wm1) * inv;
  if constexpr (HAS_P) {
    const T A = wl * Pl + wu * Pu + wd * Pd;
    const T pg = pbar * inv_gamma;
    pl = wl * (rbar - pg * (Pl - A));
    pu = wu * (rbar - pg * (Pu - A));
    pd = wd * (rbar - pg * (Pd - A));
    ql = wl * pbar;
    qu = wu * pbar;
    qd = wd * pbar;
  } else {
    pl = wl * rbar;
    pu = wu * rbar;
    pd = wd * rbar;
    ql = qu = qd = T(0);
  }
}

// Write this lane's row of flush tile u (8 stream columns) from the staging
// ring to dC (natural layout), data columns only.
template <typename T, int KS>
__device__ __forceinline__ void flush_row_tile(T* __restrict__ dst_base, const T* ring_row, int u,
                                               int k, const StreamPlan& p, const WarpInfo& wi,
                                               int vec) {
  if (u < 0) return;
  const int sc0 = u * TILE;
  const int q = sc0 / p.L;
  if (q >= wi.Q) return;
  const int j0 = sc0 - q * p.L;
  if (j0 >= p.M) return;
  const int pq = q / p.NB;
  const int band = q - pq * p.NB;
  const int row = band * 32 * KS + 32 * k + wi.lane;
  if (row >= p.N) return;
  const T* src = ring_row + (sc0 & (RING - 1));
  T* dst = dst_base + ((long long)(wi.p0 + pq) * p.N + row) * p.M + j0;
  if (vec && j0 + TILE <= p.M) {
    constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
    for (int h = 0; h < TILE / PER; ++h)
      *reinterpret_cast<int4*>(dst + h * PER) = *reinterpret_cast<const int4*>(src + h * PER);
  } else {
    const int n = min(TILE, p.M - j0);
    for (int h = 0; h < n; ++h) dst[h] = src[h];
  }
}

template <typename T, int KS, bool HAS_P>
__global__ void __launch_bounds__(128) sdtw_bwd_kernel(const SdtwArgs<T> a) {
  constexpr int S = RingStride<T>::value;
  constexpr int RW = KS * 32 * S;
  constexpr int SW = 4 * TILE * KS * 32;  // saved staging per operand
  const StreamPlan& p = a.p;
  WarpInfo wi;
  if (!warp_setup(p, KS, wi)) return;
  const int lane = wi.lane;
  const T big = Big<T>::value;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* base = reinterpret_cast<T*>(smem_raw) + (size_t)wi.wib * (RW + SW) * (HAS_P ? 2 : 1);
  T* outC = base;
  T* outQ = base + RW;
  T* stR = base + RW * (HAS_P ? 2 : 1);
  T* stP = stR + SW;
  T* myC = outC + lane * S;
  T* myQ = outQ + lane * S;

  const long long woff = (long long)wi.w * p.tmax * KS * 32;
  const T* sRw = a.sR + woff;
  const T* sPw = HAS_P ? a.sP + woff : nullptr;
  const int Tend = (wi.Tw + TILE - 1) / TILE * TILE;
  const int btop = Tend / TILE - 1;

#pragma unroll 1
  for (int c = btop; c > btop - 3; --c) {
    load_saved_chunk<T, KS>(sRw, stR, c, lane);
    if (HAS_P) load_saved_chunk<T, KS>(sPw, stP, c, lane);
    cp_async_commit();
  }

  T* dlR = a.dlR + (long long)wi.w * p.L;
  T* dlP = HAS_P ? a.dlP + (long long)wi.w * p.L : nullptr;

  // iteration state
  T accL[KS], accB[KS], dgp[KS], Qacc[KS], QaccB[KS], dgq[KS];
  T cur[KS], Xc[KS], Pcur[KS], PXc[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    accL[k] = accB[k] = dgp[k] = Qacc[k] = QaccB[k] = dgq[k] = T(0);
  }

  // rows t-1 and X(t) for t = Tend - 1 need the chunk btop landed
  cp_async_wait<2>();
  __syncwarp();
  const int t_first = Tend - 1;
  // boundary windows (values of row -1 for lane 0 / sub-band 0), keyed by stream column
  // A window holds 32 consecutive stream columns [32m, 32m+32), one per lane;
  // the loop moves to the next lower window when its column hits 32m+31.  If
  // the first column is already such a top, start one window higher.
  const int c_b = t_first - 1;  // first column needing a row -1 value
  int bw = floor_div(c_b, 32) + (pos_mod(c_b, 32) == 31 ? 1 : 0);
  T bR = row_above_saved<T, KS>(sRw, 32 * bw + lane, p, wi, big);
  T bRn = row_above_saved<T, KS>(sRw, 32 * (bw - 1) + lane, p, wi, big);
  T bP = T(0), bPn = T(0);
  if (HAS_P) {
    bP = row_above_saved<T, KS>(sPw, 32 * bw + lane, p, wi, T(0));
    bPn = row_above_saved<T, KS>(sPw, 32 * (bw - 1) + lane, p, wi, T(0));
  }
  // push windows (adjoint from the band below), keyed by the bottom row's column
  const int c_d = t_first - 1 - 32 * (KS - 1) - 31;
  int dwin = floor_div(c_d, 32) + (pos_mod(c_d, 32) == 31 ? 1 : 0);
  T dR = push_from_below(dlR, 32 * dwin + lane, p, wi);
  T dRn = push_from_below(dlR, 32 * (dwin - 1) + lane, p, wi);
  T dP = T(0), dPn = T(0);
  if (HAS_P) {
    dP = push_from_below(dlP, 32 * dwin + lane, p, wi);
    dPn = push_from_below(dlP, 32 * (dwin - 1) + lane, p, wi);
  }
  T wdR = T(0), wdP = T(0);

  {  // cur = saved row t_first - 1, Xc = X(t_first)
    const T b0 = row_above_saved<T, KS>(sRw, t_first, p, wi, big);
    const T b0p = HAS_P ? row_above_saved<T, KS>(sPw, t_first, p, wi, T(0)) : T(0);
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      cur[k] = saved_at<T, KS>(stR, t_first - 1, k, lane, big);
      Pcur[k] = HAS_P ? saved_at<T, KS>(stP, t_first - 1, k, lane, T(0)) : T(0);
    }
#pragma unroll
    for (int k = KS - 1; k >= 1; --k) {
      Xc[k] = shfl_up1_rot(lane == 31 ? cur[k - 1] : cur[k]);
      if (HAS_P) PXc[k] = shfl_up1_rot(lane == 31 ? Pcur[k - 1] : Pcur[k]);
    }
    Xc[0] = shfl_up1_rot(lane == 31 ? b0 : cur[0]);
    PXc[0] = HAS_P ? shfl_up1_rot(lane == 31 ? b0p : Pcur[0]) : T(0);
  }

  const int rows = 32 * KS;
  const int kstar = ((p.N - 1) % rows) / 32, lstar = (p.N - 1) % 32;
  const long long NBL = (long long)p.NB * p.L;
  int cap_i = wi.npairs - 1;
  long long cap_t = (long long)cap_i * NBL + (long long)((p.N - 1) / rows) * p.L + (p.M - 1) +
                    32 * kstar + lstar;

#pragma unroll 1
  for (int b = btop; b >= 0; --b) {
    load_saved_chunk<T, KS>(sRw, stR, b - 3, lane);
    if (HAS_P) load_saved_chunk<T, KS>(sPw, stP, b - 3, lane);
    cp_async_commit();
    cp_async_wait<2>();
    __syncwarp();

#pragma unroll
    for (int s = TILE - 1; s >= 0; --s) {
      const int t = b * TILE + s;
      if (t == cap_t) {
        const int pi = wi.p0 + cap_i;
        const T gr = a.grad_r[pi];
        const T gp = HAS_P ? a.grad_p[pi] : T(0);
        if (lane == lstar) {
#pragma unroll
          for (int k = 0; k < KS; ++k)
            if (k == kstar) { accL[k] += gr; if (HAS_P) Qacc[k] += gp; }
        }
        --cap_i;
        cap_t = cap_i >= 0 ? cap_t - NBL : -1;
      }
      // next predecessor rows: saved row t-2 and X(t-1)
      if ((pos_mod(t - 1, 32)) == 31) {
        bR = bRn;
        bRn = row_above_saved<T, KS>(sRw, t - 1 - 63 + lane, p, wi, big);
        if (HAS_P) {
          bP = bPn;
          bPn = row_above_saved<T, KS>(sPw, t - 1 - 63 + lane, p, wi, T(0));
        }
      }
      const T bv = shfl(bR, pos_mod(t - 1, 32));
      const T bvp = HAS_P ? shfl(bP, pos_mod(t - 1, 32)) : T(0);
      T nxt[KS], Pnxt[KS], Xn[KS], PXn[KS];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        nxt[k] = saved_at<T, KS>(stR, t - 2, k, lane, big);
        Pnxt[k] = HAS_P ? saved_at<T, KS>(stP, t - 2, k, lane, T(0)) : T(0);
      }
#pragma unroll
      for (int k = KS - 1; k >= 1; --k) {
        Xn[k] = shfl_up1_rot(lane == 31 ? nxt[k - 1] : nxt[k]);
        PXn[k] = HAS_P ? shfl_up1_rot(lane == 31 ? Pnxt[k - 1] : Pnxt[k]) : T(0);
      }
      Xn[0] = shfl_up1_rot(lane == 31 ? bv : nxt[0]);
      PXn[0] = HAS_P ? shfl_up1_rot(lane == 31 ? bvp : Pnxt[0]) : T(0);

      const int ia = (t - lane) & (RING - 1);
      T send[KS], sendq[KS];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const T rbar = accL[k] + accB[k];
        const T pbar = HAS_P ? Qacc[k] + QaccB[k] : T(0);
        const int off = k * 32 * S + ((k & 1) ? (ia ^ 32) : ia);
        myC[off] = rbar;
        if (HAS_P) myQ[off] = pbar;
        T pl, pu, pd, ql, qu, qd;
        cell_backward<T, HAS_P>(cur[k], Xc[k], Xn[k], Pcur[k], PXc[k], PXn[k], rbar, pbar,
                                a.inv_gamma, pl, pu, pd, ql, qu, qd);
        accL[k] = pl;
        send[k] = pu + dgp[k];
        dgp[k] = pd;
        if (HAS_P) {
          Qacc[k] = ql;
          sendq[k] = qu + dgq[k];
          dgq[k] = qd;
        }
      }

      {  // top row of the band -> delay line (adjoint for the band above)
        const T v = shfl(send[0], 0);
        const T vq = HAS_P ? shfl(sendq[0], 0) : T(0);
        if ((t & 31) == lane) { wdR = v; wdP = vq; }
        if ((t & 31) == 0) {
          const int scx = t + lane;
          const int j = scx - (scx / p.L) * p.L;
          dlR[j] = wdR;
          if (HAS_P) dlP[j] = wdP;
          __syncwarp();
        }
      }
      // adjoint arriving at the bottom row (lane 31, sub-band KS-1) at t-1
      const int scd = t - 1 - 32 * (KS - 1) - 31;
      if (pos_mod(scd, 32) == 31) {
        dR = dRn;
        dRn = push_from_below(dlR, scd - 63 + lane, p, wi);
        if (HAS_P) {
          dP = dPn;
          dPn = push_from_below(dlP, scd - 63 + lane, p, wi);
        }
      }
      const T dv = shfl(dR, pos_mod(scd, 32));
      const T dvq = HAS_P ? shfl(dP, pos_mod(scd, 32)) : T(0);
#pragma unroll
      for (int k = 0; k < KS - 1; ++k) {
        accB[k] = shfl_dn1_rot(lane == 0 ? send[k + 1] : send[k]);
        if (HAS_P) QaccB[k] = shfl_dn1_rot(lane == 0 ? sendq[k + 1] : sendq[k]);
      }
      accB[KS - 1] = shfl_dn1_rot(lane == 0 ? dv : send[KS - 1]);
      if (HAS_P) QaccB[KS - 1] = shfl_dn1_rot(lane == 0 ? dvq : sendq[KS - 1]);

#pragma unroll
      for (int k = 0; k < KS; ++k) {
        cur[k] = nxt[k];
        Xc[k] = Xn[k];
        if (HAS_P) { Pcur[k] = Pnxt[k]; PXc[k] = PXn[k]; }
      }
    }
    // tiles completed in this block: u = b - 4k - lane/8
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      flush_row_tile<T, KS>(a.dC, myC + k * 32 * S, b - 4 * k - (lane >> 3), k, p, wi, a.vec);
      if (HAS_P) flush_row_tile<T, KS>(a.dQ, myQ + k * 32 * S, b - 4 * k - (lane >> 3), k, p, wi, a.vec);
    }
  }
  cp_async_wait<0>();
}

template <typename T, int KS, bool HAS_P, bool HAS_BAND>
int launch_fwd(const SdtwArgs<T>& a, cudaStream_t st) {
  auto kern = sdtw_fwd_kernel<T, KS, HAS_P, HAS_BAND>;
  const size_t smem = a.p.smem_fwd;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_error(kLaunch, "sdtw forward: cannot reserve %zu bytes of shared memory", smem);
  const int grid = (a.p.warps + a.p.wpc - 1) / a.p.wpc;
  kern<<<grid, 32 * a.p.wpc, smem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "sdtw forward launch: %s", cudaGetErrorString(e));
  return kOk;
}

template <typename T, int KS, bool HAS_P>
int launch_bwd(const SdtwArgs<T>& a, cudaStream_t st) {
  auto kern = sdtw_bwd_kernel<T, KS, HAS_P>;
  const size_t smem = a.p.smem_bwd;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_error(kLaunch, "sdtw backward: cannot reserve %zu bytes of shared memory", smem);
  const int grid = (a.p.warps + a.p.wpc - 1) / a.p.wpc;
  kern<<<grid, 32 * a.p.wpc, smem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "sdtw backward launch: %s", cudaGetErrorString(e));
  return kOk;
}

template <typename T, int KS>
int fwd_ks(const SdtwArgs<T>& a, bool has_p, bool has_band, cudaStream_t st) {
  if (has_p) return has_band ? launch_fwd<T, KS, true, true>(a, st) : launch_fwd<T, KS, true, false>(a, st);
  return has_band ? launch_fwd<T, KS, false, true>(a, st) : launch_fwd<T, KS, false, false>(a, st);
}

template <typename T, int KS>
int bwd_ks(const SdtwArgs<T>& a, bool has_p, cudaStream_t st) {
  return has_p ? launch_bwd<T, KS, true>(a, st) : launch_bwd<T, KS, false>(a, st);
}

}  // namespace

StreamPlan make_stream_plan(int B, int N, int M, int eb, bool has_p, int sms) {
  StreamPlan p;
  p.B = B;
  p.N = N;
  p.M = M;
  p.KS = N <= 32 ? 1 : (N <= 64 ? 2 : 4);
  const int rows = 32 * p.KS;
  p.NB = (N + rows - 1) / rows;
  const int L = M + 1 > rows + 128 ? M + 1 : rows + 128;
  p.L = (L + TILE - 1) / TILE * TILE;
  const int S = eb == 4 ? RingStride<float>::value : RingStride<double>::value;
  const size_t ring = (size_t)p.KS * 32 * S * eb;
  const size_t stage = (size_t)4 * TILE * p.KS * 32 * eb;
  const size_t fwd_w = ring * (has_p ? 2 : 1);
  const size_t bwd_w = (ring + stage) * (has_p ? 2 : 1);
  const size_t per_w = fwd_w > bwd_w ? fwd_w : bwd_w;
  int wps = (int)((size_t)(200 * 1024) / per_w);
  wps = wps < 1 ? 1 : (wps > 16 ? 16 : wps);
  p.wpc = wps < 4 ? wps : 4;
  const int cps = wps / p.wpc > 0 ? wps / p.wpc : 1;
  const int maxw = sms * cps * p.wpc;
  p.warps = B < maxw ? B : maxw;
  if (p.warps < 1) p.warps = 1;
  p.base = B / p.warps;
  p.rem = B % p.warps;
  const long long maxpairs = p.base + (p.rem ? 1 : 0);
  const long long Tw = maxpairs * p.NB * p.L + 32 * p.KS - 1;
  p.tmax = (Tw + TILE - 1) / TILE * TILE;
  p.smem_fwd = fwd_w * p.wpc;
  p.smem_bwd = bwd_w * p.wpc;
  return p;
}

template <typename T>
int sdtw_stream_forward(const SdtwArgs<T>& a, bool has_p, bool has_band, cudaStream_t st) {
  switch (a.p.KS) {
    case 1: return fwd_ks<T, 1>(a, has_p, has_band, st);
    case 2: return fwd_ks<T, 2>(a, has_p, has_band, st);
    case 4: return fwd_ks<T, 4>(a, has_p, has_band, st);
    default: return set_error(kUnsupported, "sdtw forward: unsupported sub-band count %d", a.p.KS);
  }
}

template <typename T>
int sdtw_stream_backward(const SdtwArgs<T>& a, bool has_p, bool /*has_band*/, cudaStream_t st) {
  switch (a.p.KS) {
    case 1: return bwd_ks<T, 1>(a, has_p, st);
    case 2: return bwd_ks<T, 2>(a, has_p, st);
    case 4: return bwd_ks<T, 4>(a, has_p, st);
    default: return set_error(kUnsupported, "sdtw backward: unsupported sub-band count %d", a.p.KS);
  }
}

template int sdtw_stream_forward<float>(const SdtwArgs<float>&, bool, bool, cudaStream_t);
template int sdtw_stream_forward<double>(const SdtwArgs<double>&, bool, bool, cudaStream_t);
template int sdtw_stream_backward<float>(const SdtwArgs<float>&, bool, bool, cudaStream_t);
template int sdtw_stream_backward<double>(const SdtwArgs<double>&, bool, bool, cudaStream_t);

}  // namespace tw
