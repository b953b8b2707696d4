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
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "sdtw_stream.cuh"
#include "tc_common.cuh"

namespace tw {

__device__ int g_dp_error;

namespace {

template <typename T> struct RingStride;
// Row stride (elements) of the per-lane rings: lane l reads column (t - l)
// of row l, so the bank of its word is (l*(S-1) + t) mod 32; S-1 odd (and
// S*elem a multiple of 16 bytes for cp.async) makes the access conflict-free.
template <> struct RingStride<float> { static constexpr int value = 36; };
template <> struct RingStride<double> { static constexpr int value = 34; };

// Each lane streams its own row: at block u it works in tiles cur-1 and cur
// (cur = u - 4k - lane/8) and has tiles cur+1 .. cur+LEAD in flight, so a
// ring of LEAD + 2 tiles per lane row suffices.
constexpr int RING = 32;   // stream columns a lane row can hold
constexpr int TILE = 8;    // columns per copy tile / flush tile
constexpr int LEAD = 2;    // forward: cost tiles issued ahead of use
static_assert(TILE * (LEAD + 2) <= RING, "ring too small for the lead");

// Shared memory of one warp, in elements: the per-lane rings (cost / penalty
// in the forward, adjoint staging in the backward), 64 slots for band-edge
// collection, and the 64-column circular buffers of row -1 values (both
// sweeps) and of adjoints arriving from the band below (backward), one set
// for R and one for P.
__host__ __device__ constexpr int warp_smem_elems(int KS, int S, bool has_p) {
  return KS * 32 * S * (has_p ? 2 : 1) + 64 + (has_p ? 256 : 128);
}

// n / v.d for 0 <= n < 2^31 (see Divisor).
__device__ __forceinline__ int udiv(int n, const Divisor& v) {
  return (int)((__umulhi((unsigned)n, v.m) + (unsigned)n) >> v.l);
}
// floor(n / v.d) and the non-negative remainder, for any sign of n.
__device__ __forceinline__ int fl_div(int n, const Divisor& v) {
  const int q = udiv(n >= 0 ? n : -n - 1, v);
  return n >= 0 ? q : -q - 1;
}
__device__ __forceinline__ int p_mod(int n, const Divisor& v) { return n - fl_div(n, v) * v.d; }

__device__ __forceinline__ int floor_div(int a, int b) {
  const int q = a / b;
  return (a % b != 0 && a < 0) ? q - 1 : q;
}
__device__ __forceinline__ int pos_mod(int a, int b) {
  const int r = a % b;
  return r < 0 ? r + b : r;
}

// Group size and bands per warp stream: compile-time 1 and NB in the kernels
// without band groups, so their code is the single-warp stream's.
template <bool GRP>
__device__ __forceinline__ int grp_G(const StreamPlan& p) { return GRP ? p.G : 1; }
template <bool GRP>
__device__ __forceinline__ int grp_NBg(const StreamPlan& p) { return GRP ? p.NBg : p.NB; }
template <bool GRP>
__device__ __forceinline__ const Divisor& grp_dNBg(const StreamPlan& p) {
  return GRP ? p.dNBg : p.dNB;
}

// g: warp within its band group; off = g * D, the shift of this warp's own
// stream (local column = step - off); Q: local passes (npairs * NB / G); Tw:
// steps every warp of the group runs (the group's stream length).
// wprev / wnext: warps of the bands above / below this warp's bands.
struct WarpInfo {
  int w, wib, lane, npairs, p0, Q, Tw, g, off, wprev, wnext;
};

// Pair ranges are handed out per band group in slot order s = (group in
// CTA) * CTAs + CTA, so the groups that get one extra pair are spread over
// all SMs.  Every warp of a group gets the same answer.
template <bool GRP>
__device__ __forceinline__ bool warp_setup(const StreamPlan& p, int KS, WarpInfo& wi) {
  wi.lane = threadIdx.x & 31;
  wi.wib = threadIdx.x >> 5;
  wi.w = blockIdx.x * (blockDim.x >> 5) + wi.wib;
  if (wi.w >= p.warps) return false;
  const int gib = wi.wib / grp_G<GRP>(p);
  wi.g = wi.wib - gib * grp_G<GRP>(p);
  const int slot = gib * gridDim.x + blockIdx.x;
  wi.npairs = p.base + (slot < p.rem ? 1 : 0);
  if (wi.npairs == 0) return false;
  wi.p0 = slot * p.base + min(slot, p.rem);
  wi.Q = wi.npairs * grp_NBg<GRP>(p);
  wi.Tw = wi.Q * p.L + 32 * KS - 1 + (grp_G<GRP>(p) - 1) * p.D;
  wi.off = wi.g * p.D;
  wi.wprev = wi.g > 0 ? wi.w - 1 : wi.w + grp_G<GRP>(p) - 1;
  wi.wnext = wi.g < grp_G<GRP>(p) - 1 ? wi.w + 1 : wi.w - (grp_G<GRP>(p) - 1);
  return true;
}

// Band of this warp's local pass q (any q, also outside [0, Q)).
template <bool GRP>
__device__ __forceinline__ int band_of(int q, const StreamPlan& p, const WarpInfo& wi) {
  return wi.g + grp_G<GRP>(p) * pos_mod(q, grp_NBg<GRP>(p));
}
template <bool GRP>
__device__ __forceinline__ bool first_band(int q, const StreamPlan& p, const WarpInfo& wi) {
  return wi.g == 0 && p_mod(q, grp_dNBg<GRP>(p)) == 0;
}
template <bool GRP>
__device__ __forceinline__ bool last_band(int q, const StreamPlan& p, const WarpInfo& wi) {
  return wi.g == grp_G<GRP>(p) - 1 && p_mod(q + 1, grp_dNBg<GRP>(p)) == 0;
}

// One step of a band group's lockstep: every lane arrives on the group's
// mbarrier (release) and waits for the phase to complete (acquire), so the
// delay-line writes of every warp before it are visible to every warp after
// it.  The wait is bounded; a warp whose wait runs out records kTimeout and
// stops waiting (it keeps arriving, so the others are not held up), and the
// sweep runs to its end with its results marked invalid by the error word.
__device__ __forceinline__ void group_step(uint64_t* bar, unsigned& phase, bool& dead) {
  tc::mbar_arrive(bar);
  if (!dead) {
    bool ok = false;
    for (unsigned n = 0; n < tc::kSpinLimit; ++n)
      if (tc::mbar_try_wait(bar, phase)) { ok = true; break; }
    if (!ok) {
      dead = true;
      atomicExch(&g_dp_error, kTimeout);
    }
  }
  phase ^= 1u;
}

// The groups' mbarriers (one per group of the CTA, 32 G arrivals), at `area`
// after the warps' regions, set up before any warp leaves; a no-op without
// band groups.
template <bool GRP>
__device__ __forceinline__ uint64_t* group_barrier_init(const StreamPlan& p,
                                                        unsigned char* area) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(area);
  if (grp_G<GRP>(p) > 1) {
    const int groups = (blockDim.x >> 5) / grp_G<GRP>(p);
    if ((int)threadIdx.x < groups) tc::mbar_init(&bars[threadIdx.x], 32u * grp_G<GRP>(p));
    __syncthreads();
  }
  return bars + (threadIdx.x >> 5) / grp_G<GRP>(p);
}

// Position of stream tile u (the 8 columns [8u, 8u+8)) in (pass, column)
// space.  Kernels step cursors by one tile per 8-step block, so the hot loop
// never divides by the runtime L or NB.
struct Cursor {
  int u;     // tile index in step time (local tile + off / 8): its ring slot
  int q;     // pass (nothing to do when < 0 or >= Q)
  int j0;    // first column of the tile within the pass (L is a multiple of 8)
  int band;  // q mod NB
  int pq;    // q div NB: pair index within the warp
};

// u is a tile of the warp's local stream.  Local pass q is band
// g + G (q mod NB/G) of the pair q div (NB/G), so stepping a pass moves the
// band by G.  The ring slot of a tile follows the step at which it is used,
// so c.u counts in steps (shifted by off), not in local columns.
template <bool GRP>
__device__ __forceinline__ Cursor cursor_at(int u, const StreamPlan& p, const WarpInfo& wi) {
  Cursor c;
  c.u = u + wi.off / TILE;
  c.q = floor_div(u * TILE, p.L);
  c.j0 = u * TILE - c.q * p.L;
  c.pq = floor_div(c.q, grp_NBg<GRP>(p));
  c.band = wi.g + grp_G<GRP>(p) * (c.q - c.pq * grp_NBg<GRP>(p));
  return c;
}
template <bool GRP>
__device__ __forceinline__ void cursor_next(Cursor& c, const StreamPlan& p) {
  ++c.u;
  c.j0 += TILE;
  if (c.j0 >= p.L) {
    c.j0 = 0;
    ++c.q;
    c.band += grp_G<GRP>(p);
    if (c.band >= p.NB) { c.band -= p.NB; ++c.pq; }
  }
}
template <bool GRP>
__device__ __forceinline__ void cursor_prev(Cursor& c, const StreamPlan& p) {
  --c.u;
  c.j0 -= TILE;
  if (c.j0 < 0) {
    c.j0 = p.L - TILE;
    --c.q;
    c.band -= grp_G<GRP>(p);
    if (c.band < 0) { c.band += p.NB; --c.pq; }
  }
}

// ---------------------------------------------------------------- forward

// What a lane does for the tiles of cursor c's pass in sub-band k: 0 nothing
// (no pass), 1 zero-fill (a row past N), 2 copy its row, whose element offset
// in the cost / penalty is `off`.  Recomputed only when a pass begins.
template <int KS>
__device__ __forceinline__ int row_mode(const Cursor& c, int k, const StreamPlan& p,
                                        const WarpInfo& wi, long long& off) {
  off = 0;
  if (c.q < 0 || c.q >= wi.Q) return 0;
  const int row = c.band * 32 * KS + 32 * k + wi.lane;
  if (row >= p.N) return 1;
  off = ((long long)(wi.p0 + c.pq) * p.N + row) * p.M;
  return 2;
}

// Copy the 8 stream columns of tile c of this lane's row into its ring row
// (cp.async, zero-filled outside the data); `mode` and `off` from row_mode.
template <typename T>
__device__ __forceinline__ void load_row_tile(const T* __restrict__ src_base, T* ring_row,
                                              const Cursor& c, int mode, long long off,
                                              const StreamPlan& p, int vec) {
  if (mode == 0 || c.j0 >= p.M) return;  // nothing, or all padding
  const int j0 = c.j0;
  T* dst = ring_row + ((c.u * TILE) & (RING - 1));
  const T* src = src_base + off;
  if (vec) {
    constexpr int PER = 16 / (int)sizeof(T);
    if (mode == 2 && j0 + TILE <= p.M) {  // a whole tile of data
#pragma unroll
      for (int h = 0; h < TILE / PER; ++h) cp_async16(dst + h * PER, src + j0 + h * PER, 16);
    } else {
#pragma unroll
      for (int h = 0; h < TILE / PER; ++h) {
        const int j = j0 + h * PER;
        int cnt = mode == 2 ? min(PER, p.M - j) : 0;
        cnt = cnt < 0 ? 0 : cnt;
        cp_async16(dst + h * PER, cnt > 0 ? (const void*)(src + j) : (const void*)src_base,
                   cnt * (int)sizeof(T));
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < TILE; ++h) {
      const int j = j0 + h;
      const bool v = mode == 2 && j < p.M;
      cp_async_elem<sizeof(T)>(dst + h, v ? (const void*)(src + j) : (const void*)src_base,
                               v ? (int)sizeof(T) : 0);
    }
  }
}

// Padding columns j >= M of a landed tile get the raw cost Big/kappa.
template <typename T>
__device__ __forceinline__ void patch_row_tile(T* ring_row, const Cursor& c, const StreamPlan& p,
                                               const WarpInfo& wi, T padv) {
  if (c.q < 0 || c.q >= wi.Q || c.j0 + TILE <= p.M) return;
  T* dst = ring_row + ((c.u * TILE) & (RING - 1));
  for (int h = max(0, p.M - c.j0); h < TILE; ++h) dst[h] = padv;
}

// Value of "row -1" that lane 0 of sub-band 0 sees at local stream column
// sc: the previous band's bottom row (the delay line `dl` of the warp that
// computed it), +Big above a pair's first band, and 0 at the last column of a
// pass that precedes a first band in this warp's stream (it is the diagonal
// predecessor of cell (0,0), R(-1,-1) = 0).  For P: 0 / delay line.
template <bool GRP, typename T>
__device__ __forceinline__ T row_above(const T* dl, int sc, const StreamPlan& p,
                                       const WarpInfo& wi, T first_value) {
  const int q = fl_div(sc, p.dL);
  const int j = sc - q * p.L;
  const bool first = q < 0 || q >= wi.Q || first_band<GRP>(q, p, wi);
  T v = first ? first_value : dl[j];
  if (j == p.L - 1 && first_band<GRP>(q + 1, p, wi)) v = T(0);
  return v;
}

// c is the raw cost; kap = log2(e) / gamma scales it into the log2 domain
// inside the final fused multiply-add.
template <typename T, bool HAS_P>
__device__ __forceinline__ void cell_forward(T c, T kap, T qv, T left, T up, T dg, T Pl, T Pu,
                                             T Pd, T& r, T& pv) {
  const T m1 = fmin(left, up), M1 = fmax(left, up);
  const T m = fmin(m1, dg), Mx = fmax(m1, dg);
  const T e1 = ex2(add_rn(m, -M1));
  const T e2 = ex2(add_rn(m, -Mx));
  const T s = add_rn(add_rn(T(1), e1), e2);
  r = fma(c, kap, add_rn(m, -lg2(s)));
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

template <typename T, int KS, bool HAS_P, bool HAS_BAND, bool GRP>
__global__ void __launch_bounds__(128) sdtw_fwd_kernel(const SdtwArgs<T> a) {
  constexpr int S = RingStride<T>::value;
  constexpr int RW = KS * 32 * S;  // ring elements per operand per warp
  const StreamPlan& p = a.p;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int WE = warp_smem_elems(KS, S, HAS_P);
  uint64_t* gbar =
      group_barrier_init<GRP>(p, smem_raw + (blockDim.x >> 5) * WE * sizeof(T));
  WarpInfo wi;
  if (!warp_setup<GRP>(p, KS, wi)) return;
  const int lane = wi.lane;
  const T big = Big<T>::value;
  T* ringC = reinterpret_cast<T*>(smem_raw) + (size_t)wi.wib * WE;
  T* ringQ = ringC + RW;
  // bottom-row values of the current 32-step window: R at [0, 32), P at [32, 64)
  T* coll = ringC + RW * (HAS_P ? 2 : 1);
  // row -1 values (lane 0 / sub-band 0) by stream column mod 64: the window
  // of the current step and the next one
  T* fb = coll + 64;
  T* fbp = fb + 64;
  for (int i = lane; i < RW; i += 32) {
    ringC[i] = a.pad_raw;
    if (HAS_P) ringQ[i] = T(0);
  }
  __syncwarp();
  T* myC = ringC + lane * S;
  T* myQ = ringQ + lane * S;

  Cursor ld[KS], pt[KS];  // next tile to load / to patch, per sub-band (lane-dependent)
  int lmode[KS];           // row_mode of ld's pass
  long long loff[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    ld[k] = cursor_at<GRP>(-4 * k - (lane >> 3) - wi.off / TILE, p, wi);
    pt[k] = ld[k];
    lmode[k] = row_mode<KS>(ld[k], k, p, wi, loff[k]);
  }
#pragma unroll 1
  for (int pb = -LEAD; pb < 0; ++pb) {
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      load_row_tile<T>(a.C, myC + k * 32 * S, ld[k], lmode[k], loff[k], p, a.vec);
      if (HAS_P) load_row_tile<T>(a.Q, myQ + k * 32 * S, ld[k], lmode[k], loff[k], p, a.vec);
      cursor_next<GRP>(ld[k], p);
      if (ld[k].j0 == 0) lmode[k] = row_mode<KS>(ld[k], k, p, wi, loff[k]);
    }
    cp_async_commit();
  }

  T left[KS], up[KS], dg[KS], Pl[KS], Pu[KS], Pd[KS];
  int jk[KS], rowk[KS];
  const int rows = 32 * KS;
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    left[k] = up[k] = dg[k] = big;
    Pl[k] = Pu[k] = Pd[k] = T(0);
    if (HAS_BAND) {
      const int sc = -32 * k - lane - wi.off;
      const int q = floor_div(sc, p.L);
      jk[k] = sc - q * p.L;
      rowk[k] = band_of<GRP>(q, p, wi) * rows + 32 * k + lane;
    }
  }
  if (lane == 0) dg[0] = T(0);

  // own delay line (written) and that of the warp of the band above (read)
  T* dlR = a.dlR + (long long)wi.w * p.L;
  T* dlP = HAS_P ? a.dlP + (long long)wi.w * p.L : nullptr;
  const T* dlRa = a.dlR + (long long)wi.wprev * p.L;
  const T* dlPa = HAS_P ? a.dlP + (long long)wi.wprev * p.L : nullptr;
  fb[lane] = row_above<GRP>(dlRa, lane - wi.off, p, wi, big);
  fb[32 + lane] = row_above<GRP>(dlRa, 32 + lane - wi.off, p, wi, big);
  if (HAS_P) {
    fbp[lane] = row_above<GRP>(dlPa, lane - wi.off, p, wi, T(0));
    fbp[32 + lane] = row_above<GRP>(dlPa, 32 + lane - wi.off, p, wi, T(0));
  }
  __syncwarp();
  unsigned gphase = 0;
  bool gdead = false;
  const int ql = wi.Q * p.L;  // local columns of the warp's passes

  const long long woff = p.saved_offset(wi.w);
  const long long eoff = p.edge_offset(wi.w);
  const T kap = a.kappa;
  // rows below the stream start read as +Big (R) / 0 (P) in the backward
#pragma unroll 1
  for (int r = -StreamPlan::kPreRows; r < 0; ++r)
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      a.sR[woff + ((long long)r * KS + k) * 32 + lane] = big;
      if (HAS_P) a.sP[woff + ((long long)r * KS + k) * 32 + lane] = T(0);
    }

  // The 8 steps of a block are straight-line code; every rare event (cost
  // tiles, delay-line flush, window change) happens between blocks.
#pragma unroll 1
  for (int t0 = 0; t0 < wi.Tw; t0 += TILE) {
    cp_async_wait<LEAD - 1>();
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      patch_row_tile(myC + k * 32 * S, pt[k], p, wi, a.pad_raw);
      cursor_next<GRP>(pt[k], p);
    }
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      load_row_tile<T>(a.C, myC + k * 32 * S, ld[k], lmode[k], loff[k], p, a.vec);
      if (HAS_P) load_row_tile<T>(a.Q, myQ + k * 32 * S, ld[k], lmode[k], loff[k], p, a.vec);
      cursor_next<GRP>(ld[k], p);
      if (ld[k].j0 == 0) lmode[k] = row_mode<KS>(ld[k], k, p, wi, loff[k]);  // a new pass
    }
    cp_async_commit();

    const bool wrapw = ((t0 + TILE) & 31) == 0;  // column t0+8 opens the next window
    T* coll8 = coll + (t0 & 24);                 // slot of step t0 + s is coll8[s]
    T* srow = a.sR + woff + lane + (long long)t0 * KS * 32;
    T* prow = HAS_P ? a.sP + woff + lane + (long long)t0 * KS * 32 : nullptr;
    const int c0 = (t0 - lane) & (RING - 1);
    // row -1 values of columns t0 + s + 1, read before the block's stores
    T fbv[TILE], fbpv[TILE];
    {
      const T* fbs = fb + ((t0 + 1) & 63);
      const T* fbps = fbp + ((t0 + 1) & 63);
      const int c7 = (t0 + TILE) & 63;
#pragma unroll
      for (int s = 0; s < TILE; ++s) {
        fbv[s] = s == TILE - 1 ? fb[c7] : fbs[s];
        if (HAS_P) fbpv[s] = s == TILE - 1 ? fbp[c7] : fbps[s];
      }
    }
#pragma unroll
    for (int s = 0; s < TILE; ++s) {
      const int ia = (c0 + s) & (RING - 1);
      T Rn[KS], Pn[KS];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const int off = k * 32 * S + ia;  // column t - 32k - lane of sub-band k
        const T qv = HAS_P ? myQ[off] : T(0);
        cell_forward<T, HAS_P>(myC[off], kap, qv, left[k], up[k], dg[k], Pl[k], Pu[k], Pd[k],
                               Rn[k], Pn[k]);
        if constexpr (HAS_BAND) {
          const bool ok = fabs((T)(rowk[k] - jk[k])) <= a.band;
          Rn[k] = ok ? Rn[k] : big;
          Pn[k] = ok ? Pn[k] : T(0);
          const int jn = jk[k] + 1;
          const bool wrap = jn == p.L;
          int rn = rowk[k] + grp_G<GRP>(p) * rows;
          rn = rn >= p.NB * rows ? rn - p.NB * rows : rn;
          jk[k] = wrap ? 0 : jn;
          rowk[k] = wrap ? rn : rowk[k];
        }
        srow[(s * KS + k) * 32] = Rn[k];
        if (HAS_P) prow[(s * KS + k) * 32] = Pn[k];
      }
      // bottom row (column t - 32 KS + 1): lane 31 files it under step t mod 32
      if (lane == 31) {
        coll8[s] = Rn[KS - 1];
        if (HAS_P) coll8[32 + s] = Pn[KS - 1];
      }
      // row -1 value for the next step (column t + 1)
      const T bv = fbv[s];
      const T bp = HAS_P ? fbpv[s] : T(0);
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

    if (wrapw) {
      // lane l takes the bottom row of step l of the window: column
      // t0 - 23 - 32 KS + lane
      __syncwarp();
      const T wbR = coll[lane];
      const T wbP = HAS_P ? coll[32 + lane] : T(0);
      // the window's bottom-row values (steps t0 - 24 .. t0 + 7) to the edge stream
      a.sR[eoff + t0 - 24 + lane] = wbR;
      if (HAS_P) a.sP[eoff + t0 - 24 + lane] = wbP;
      const int scx = t0 - 23 - 32 * KS + lane - wi.off;
      if (scx >= 0 && (!GRP || scx < ql)) {
        const int j = scx - udiv(scx, p.dL) * p.L;
        dlR[j] = wbR;
        if (HAS_P) dlP[j] = wbP;
      }
      if constexpr (GRP) group_step(gbar, gphase, gdead);
      else __syncwarp();
      // the window that just ended makes room for the one after next (the
      // delay line was written D >= 32 KS + 128 steps earlier, so these loads
      // hit L2)
      const int cn = t0 + TILE + 32 + lane;
      fb[cn & 63] = row_above<GRP>(dlRa, cn - wi.off, p, wi, big);
      if (HAS_P) fbp[cn & 63] = row_above<GRP>(dlPa, cn - wi.off, p, wi, T(0));
      __syncwarp();
    }
  }
  cp_async_wait<0>();

  // R[N-1, M-1] of each pair, read back from the saved stream of the lane
  // (and warp of the group) that computed it
  const int kstar = ((p.N - 1) % rows) / 32, lstar = (p.N - 1) % 32;
  const int bstar = (p.N - 1) / rows;
  if (lane == lstar && bstar % grp_G<GRP>(p) == wi.g) {
    for (int i = 0; i < wi.npairs; ++i) {
      const long long ct = (long long)(i * grp_NBg<GRP>(p) + bstar / grp_G<GRP>(p)) * p.L +
                           (p.M - 1) + 32 * kstar + lstar + wi.off;
      const T v = a.sR[woff + (ct * KS + kstar) * 32 + lane];
      a.out_r[wi.p0 + i] = v >= big * T(0.5) ? T(INFINITY) : v * a.inv_kappa;
      if (HAS_P) a.out_p[wi.p0 + i] = a.sP[woff + (ct * KS + kstar) * 32 + lane];
    }
  }
}

// ---------------------------------------------------------------- backward

// This lane's saved values of stream row r (one per sub-band).  Rows down to
// -kPreRows exist (the forward fills them with +Big / 0), so no guard.
template <typename T, int KS>
__device__ __forceinline__ void load_saved_row(const T* __restrict__ s_lane, int r, T (&out)[KS]) {
#pragma unroll
  for (int k = 0; k < KS; ++k) out[k] = s_lane[((long long)r * KS + k) * 32];
}

// Row -1 value lane 0 of sub-band 0 used at step sc in the forward sweep,
// re-read from the edge stream `e_above` of the warp of the band above (its
// bottom row, which that warp computed D - 32 KS + 1 steps earlier).  Lanes
// read consecutive steps: one coalesced load per window.
template <typename T, int KS, bool GRP>
__device__ __forceinline__ T row_above_saved(const T* e_above, int sc, const StreamPlan& p,
                                             const WarpInfo& wi, T first_value) {
  if constexpr (!GRP) {  // one warp per pair: the band above is this warp's previous pass
    const int q = fl_div(sc, p.dL);
    const int j = sc - q * p.L;
    const bool first = q < 0 || q >= wi.Q || p_mod(q, p.dNB) == 0;
    T v = first_value;
    if (!first) v = e_above[sc - p.L + 32 * KS - 1];
    if (j == p.L - 1 && p_mod(q + 1, p.dNB) == 0) v = T(0);
    return v;
  }
  const int sl = sc - wi.off;
  const int q = fl_div(sl, p.dL);
  const int j = sl - q * p.L;
  const bool first = q < 0 || q >= wi.Q || first_band<GRP>(q, p, wi);
  T v = first_value;
  if (!first) v = e_above[sc - p.D + 32 * KS - 1];
  if (j == p.L - 1 && first_band<GRP>(q + 1, p, wi)) v = T(0);
  return v;
}

// Adjoint pushed into the bottom row of the band at stream column sc from the
// next band's top row (delay line); zero when the next band starts a new pair,
// and zero on padding columns (j >= M), which carry no adjoint.  (The top row
// of a pair's first band hands the adjoint of its virtual corner R(-1,-1) one
// column back, into the previous pass's last padding column; it must stop there.)
// SEEDB (N a multiple of the band height): the bottom row of a pair's last
// band is row N-1, so the pair's seed dL/dR enters here, at column M-1.
// sc is a step; `dl` is the delay line of the warp of the band below.
template <typename T, bool SEEDB, bool GRP>
__device__ __forceinline__ T push_from_below(const T* dl, int sc, const StreamPlan& p,
                                             const WarpInfo& wi, const T* grad) {
  if constexpr (!GRP) {  // one warp per pair: the band below is this warp's next pass
    if (sc < 0) return T(0);
    const int q = udiv(sc, p.dL);
    const int j = sc - q * p.L;
    if (j >= p.M || q >= wi.Q) return T(0);
    const int pq = udiv(q + 1, p.dNB);
    if (pq * p.NB == q + 1) return (SEEDB && j == p.M - 1) ? grad[wi.p0 + pq - 1] : T(0);
    return dl[j];
  }
  const int sl = sc - wi.off;
  if (sl < 0) return T(0);
  const int q = udiv(sl, p.dL);
  const int j = sl - q * p.L;
  if (j >= p.M || q >= wi.Q) return T(0);
  if (last_band<GRP>(q, p, wi))
    return (SEEDB && j == p.M - 1) ? grad[wi.p0 + udiv(q, grp_dNBg<GRP>(p))] : T(0);
  return dl[j];
}

template <typename T, bool HAS_P>
__device__ __forceinline__ void cell_backward(T Rl, T Ru, T Rd, T Pl, T Pu, T Pd, T rbar, T pbar,
                                              T inv_gamma, T& pl, T& pu, T& pd, T& ql, T& qu,
                                              T& qd) {
  // unnormalised soft-min weights of the left / up / diagonal predecessors
  // (the smallest R' gets exactly 1) and the reciprocal of their sum
  T ul, uu, ud, inv;
  if constexpr (sizeof(T) == 4) {
    // three exponentials and no selects: fewer issue slots than sorting
    const T m = fmin(fmin(Rl, Ru), Rd);
    ul = ex2(add_rn(m, -Rl));
    uu = ex2(add_rn(m, -Ru));
    ud = ex2(add_rn(m, -Rd));
    inv = rcp(add_rn(add_rn(ul, uu), ud));
  } else {
    // double: exp2 is a long sequence, so evaluate two and place the 1
    const T m1 = fmin(Rl, Ru), M1 = fmax(Rl, Ru);
    const T m = fmin(m1, Rd), Mx = fmax(m1, Rd);
    const T e1 = ex2(add_rn(m, -M1));
    const T e2 = ex2(add_rn(m, -Mx));
    inv = rcp(add_rn(add_rn(T(1), e1), e2));
    const bool p1 = Rl <= Ru;
    const bool p2 = m1 <= Rd;
    const T wm1 = p2 ? T(1) : e2;
    ud = p2 ? e2 : T(1);
    ul = p1 ? wm1 : e1;
    uu = p1 ? e1 : wm1;
  }
  if constexpr (HAS_P) {
    const T wd = ud * inv, wl = ul * inv, wu = uu * inv;
    const T A = wl * Pl + wu * Pu + wd * Pd;
    const T pg = pbar * inv_gamma;
    pl = wl * (rbar - pg * (Pl - A));
    pu = wu * (rbar - pg * (Pu - A));
    pd = wd * (rbar - pg * (Pd - A));
    ql = wl * pbar;
    qu = wu * pbar;
    qd = wd * pbar;
  } else {
    const T ri = rbar * inv;  // adjoint over the soft-min normaliser
    pl = ul * ri;
    pu = uu * ri;
    pd = ud * ri;
    ql = qu = qd = T(0);
  }
}

// Positivity-mask words of this lane's row in the pass of cursor c: word jw
// of the row is at [jw * np].  Outside the data (no pass, or a padding row)
// it points at the mask's first row instead, so that every load stays in
// bounds; the flush writes nothing there.
template <int KS>
__device__ __forceinline__ const uint32_t* mask_row(const uint32_t* mask, int np, const Cursor& c,
                                                    int k, const StreamPlan& p,
                                                    const WarpInfo& wi) {
  const int row = c.band * 32 * KS + 32 * k + wi.lane;
  if (c.q < 0 || c.q >= wi.Q || row >= p.N) return mask;
  const int mw = (p.M + 31) >> 5;
  return mask + (long long)(wi.p0 + c.pq) * mw * np + row;
}

// Write this lane's row of flush tile c (8 stream columns) from the staging
// ring to dC (natural layout), data columns only; `mode` and `off` come from
// row_mode for the tile's pass.  With `masked`, columns whose bit in `word` is
// clear are written as 0.  Returns nonzero when a written value is nonzero;
// with `sparse`, the bit mask of the tile's nonzero values (bit e: column
// j0 + e), and a whole tile of zeros is not written at all.
template <typename T>
__device__ __forceinline__ uint32_t flush_row_tile(T* __restrict__ dst_base, const T* ring_row,
                                                   const Cursor& c, int mode, long long off,
                                                   const StreamPlan& p, int vec, bool masked,
                                                   uint32_t word, bool sparse,
                                                   bool known_zero) {
  if (mode != 2 || c.j0 >= p.M) return 0u;
  const int j0 = c.j0;
  const T* src = ring_row + ((c.u * TILE) & (RING - 1));
  T* dst = dst_base + off + j0;
  if (known_zero) {  // every step of the tile was in a dead block
    if (!sparse) {
      if (vec && j0 + TILE <= p.M) {
        constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
        for (int h = 0; h < TILE / PER; ++h)
          *reinterpret_cast<int4*>(dst + h * PER) = make_int4(0, 0, 0, 0);
      } else {
        const int n = min(TILE, p.M - j0);
        for (int h = 0; h < n; ++h) dst[h] = T(0);
      }
    }
    return 0u;
  }
  if (vec && j0 + TILE <= p.M) {
    constexpr int PER = 16 / (int)sizeof(T);
    union {
      int4 i;
      T v[PER];
    } u[TILE / PER];
    int any = 0;  // OR of the staged words (float: magnitude bits only)
#pragma unroll
    for (int h = 0; h < TILE / PER; ++h) {
      u[h].i = *reinterpret_cast<const int4*>(src + h * PER);
      if constexpr (sizeof(T) == 4) {
        any |= (u[h].i.x | u[h].i.y | u[h].i.z | u[h].i.w);
      } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) any |= u[h].v[e] != T(0) ? 1 : 0;
      }
    }
    const bool nz = sizeof(T) == 4 ? (any & 0x7fffffff) != 0 : any != 0;
    uint32_t nzb = nz ? 1u : 0u;
    // An all-zero tile needs no mask, so it does not wait for the mask word
    // (loaded a block earlier; dead blocks are short).
    if (nz && (masked || sparse)) {
      const uint32_t mb = masked ? word >> (j0 & 31) : 0xffu;
      nzb = 0u;
#pragma unroll
      for (int h = 0; h < TILE / PER; ++h) {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          if (!((mb >> (h * PER + e)) & 1u)) u[h].v[e] = T(0);
          nzb |= (u[h].v[e] != T(0) ? 1u : 0u) << (h * PER + e);
        }
      }
    }
    if (!sparse || nzb != 0u) {
#pragma unroll
      for (int h = 0; h < TILE / PER; ++h) *reinterpret_cast<int4*>(dst + h * PER) = u[h].i;
    }
    return nzb;
  }
  const uint32_t bits = masked ? word >> (j0 & 31) : 0xffu;
  const int n = min(TILE, p.M - j0);
  uint32_t nzb = 0u;
  for (int h = 0; h < n; ++h) {
    const T v = ((bits >> h) & 1u) ? src[h] : T(0);
    dst[h] = v;
    nzb |= (v != T(0) ? 1u : 0u) << h;
  }
  return nzb;
}

template <typename T, int KS, bool HAS_P, bool SEEDB, bool GRP>
__global__ void __launch_bounds__(128) sdtw_bwd_kernel(const SdtwArgs<T> a) {
  constexpr int S = RingStride<T>::value;
  constexpr int RW = KS * 32 * S;
  const StreamPlan& p = a.p;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int WE = warp_smem_elems(KS, S, HAS_P);
  uint64_t* gbar =
      group_barrier_init<GRP>(p, smem_raw + (blockDim.x >> 5) * WE * sizeof(T));
  WarpInfo wi;
  if (!warp_setup<GRP>(p, KS, wi)) return;
  const int lane = wi.lane;
  const T big = Big<T>::value;
  T* base = reinterpret_cast<T*>(smem_raw) + (size_t)wi.wib * WE;
  T* outC = base;
  T* outQ = base + RW;
  // top-row sends of the current 32-step window: R at [0, 32), P at [32, 64)
  T* coll = base + RW * (HAS_P ? 2 : 1);
  // by stream column mod 64 (two 32-column windows each): row -1 values of
  // lane 0 / sub-band 0 (sb, sbp), and adjoints arriving at lane 31 of
  // sub-band KS-1 from the band below (sd, sdp)
  T* sb = coll + 64;
  T* sbp = sb + 64;
  T* sd = sb + (HAS_P ? 128 : 64);
  T* sdp = sd + 64;
  T* myC = outC + lane * S;
  T* myQ = outQ + lane * S;

  const long long woff = p.saved_offset(wi.w);
  const T* sRw = a.sR + woff;
  const T* sPw = HAS_P ? a.sP + woff : nullptr;
  // edge stream of the warp of the band above (row -1 values)
  const T* eRa = a.sR + p.edge_offset(wi.wprev);
  const T* ePa = HAS_P ? a.sP + p.edge_offset(wi.wprev) : nullptr;
  const int Tend = (wi.Tw + TILE - 1) / TILE * TILE;
  const int btop = Tend / TILE - 1;
  const T* sRl = sRw + lane;
  const T* sPl = HAS_P ? sPw + lane : nullptr;

  // Two register sets of saved rows, F and G: a block reads saved row t-2 of
  // iteration t = 8b + s from one set (index s) and, at its start, loads the
  // next block's rows into the other, so every load has 8 to 15 steps to
  // land.  The block loop is unrolled by two so the sets swap roles without
  // copies.
  T F[TILE][KS], FP[TILE][KS], G[TILE][KS], GP[TILE][KS];
#pragma unroll
  for (int s = 0; s < TILE; ++s) {
    load_saved_row<T, KS>(sRl, TILE * btop - 2 + s, F[s]);
    if (HAS_P) load_saved_row<T, KS>(sPl, TILE * btop - 2 + s, FP[s]);
  }

  // own delay line (top-row sends, written) and that of the warp of the band
  // below (read)
  T* dlR = a.dlR + (long long)wi.w * p.L;
  T* dlP = HAS_P ? a.dlP + (long long)wi.w * p.L : nullptr;
  const T* dlRb = a.dlR + (long long)wi.wnext * p.L;
  const T* dlPb = HAS_P ? a.dlP + (long long)wi.wnext * p.L : nullptr;

  T accL[KS], accB[KS], dgp[KS], Qacc[KS], QaccB[KS], dgq[KS];
  T cur[KS], Xc[KS], Pcur[KS], PXc[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    accL[k] = accB[k] = dgp[k] = Qacc[k] = QaccB[k] = dgq[k] = T(0);
  }

  const int t_first = Tend - 1;
  // Row -1 values by stream column: iteration t reads column t-1, so the
  // first block needs the windows of t_first-1 and the one below.
  {
    const int bw = (t_first - 1) >> 5;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 32 * (bw - h) + lane;
      sb[c & 63] = row_above_saved<T, KS, GRP>(eRa, c, p, wi, big);
      if (HAS_P) sbp[c & 63] = row_above_saved<T, KS, GRP>(ePa, c, p, wi, T(0));
    }
  }
  // Adjoint from the band below, by the bottom row's column t - 32 KS at
  // iteration t (used one iteration later); a block never straddles windows.
  int dw = (TILE * btop - 32 * KS) >> 5;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = 32 * (dw - h) + lane;
    sd[c & 63] = push_from_below<T, SEEDB, GRP>(dlRb, c, p, wi, a.grad_r);
    if (HAS_P) sdp[c & 63] = push_from_below<T, SEEDB, GRP>(dlPb, c, p, wi, a.grad_p);
  }
  __syncwarp();

  {  // cur = saved row t_first - 1, Xc = X(t_first)
    const T b0 = row_above_saved<T, KS, GRP>(eRa, t_first, p, wi, big);
    const T b0p = HAS_P ? row_above_saved<T, KS, GRP>(ePa, t_first, p, wi, T(0)) : T(0);
    load_saved_row<T, KS>(sRl, t_first - 1, cur);
#pragma unroll
    for (int k = 0; k < KS; ++k) Pcur[k] = T(0);
    if (HAS_P) load_saved_row<T, KS>(sPl, t_first - 1, Pcur);
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
  const int bstar = (p.N - 1) / rows;
  const int NBL = grp_NBg<GRP>(p) * p.L;  // local steps per pair
  // the end cell of each pair lies in band bstar, in the stream of warp
  // bstar mod G of the group; the other warps have no seed
  const bool has_end = bstar % grp_G<GRP>(p) == wi.g;
  int cap_i = has_end ? wi.npairs - 1 : -1;
  int cap_t = has_end ? cap_i * NBL + (bstar / grp_G<GRP>(p)) * p.L + (p.M - 1) + 32 * kstar +
                            lstar + wi.off
                      : -1;
  // adjoint seeds dL/dR (dL/dP) of the current pair's end cell, held by the
  // lane and sub-band that own it
  const bool seed_lane = lane == lstar;
  T sdR[KS], sdP[KS];
  {
    const T sr = cap_i >= 0 ? a.grad_r[wi.p0 + cap_i] : T(0);
    const T sp = HAS_P && cap_i >= 0 ? a.grad_p[wi.p0 + cap_i] : T(0);
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      sdR[k] = (seed_lane && k == kstar) ? sr : T(0);
      sdP[k] = (seed_lane && k == kstar) ? sp : T(0);
    }
  }

  // tile completed by this lane in block b: u = b - 4k - lane/8; with a
  // positivity mask, its word is loaded a block before the flush
  Cursor fl[KS];
  int fmode[KS];     // row_mode of fl's pass
  long long foff[KS];
  uint32_t mwd[KS];
  const uint32_t* mrow[KS];
  const bool masked = a.mask != nullptr;
  const int mwl = ((p.M + 31) >> 5) - 1;  // last word of a mask row
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    fl[k] = cursor_at<GRP>(btop - 4 * k - (lane >> 3) - wi.off / TILE, p, wi);
    fmode[k] = row_mode<KS>(fl[k], k, p, wi, foff[k]);
    mrow[k] = masked ? mask_row<KS>(a.mask, a.mask_np, fl[k], k, p, wi) : nullptr;
    mwd[k] = masked ? mrow[k][min(fl[k].j0 >> 5, mwl) * a.mask_np] : 0u;
  }

  // The 8 steps of block b, reading saved rows from Fc and loading the next
  // block's rows into Fn.  A pair's seed enters at step s_inj (-1: none).
  //
  // An adjoint enters the block's cells only from the warp's carried
  // adjoints, the band below (dvs) or a seed.  When all of them are zero,
  // every cell of the block has a zero adjoint and hands zero to each
  // predecessor, so the soft-min weights need not be formed: such a dead
  // block only stages zeros for dC and files zero top-row sends.  The test
  // is exact (NaN is not zero) and warp-uniform.  The predecessor registers
  // (cur, Xc) are not carried through dead blocks (`stale`): a dead block
  // loads no saved row unless the next block is live, and then loads that
  // block's rows and, into cur, the row it starts from; the live block
  // forms Xc from it.  (Loading each dead block's first row to carry cur and
  // Xc through, or deferring that consumption, measured slower: every dead
  // block then waits on a DRAM load issued one short block earlier.)
  bool stale = false;
  // liveness of the block just run and of the one before it (the start
  // counts as live, so the first tiles are flushed from the ring)
  bool cur_live = true, prev_live = true;
  // the next block is proved dead (set by a dead block)
  bool next_dead = false;
  // window zw_idx of adjoints from below holds a nonzero value (zw_any)
  int zw_idx = INT_MIN;
  bool zw_any = true;
  auto run_block = [&](const int t0, T (&Fc)[TILE][KS], T (&FPc)[TILE][KS], T (&Fn)[TILE][KS],
                       T (&FPn)[TILE][KS]) {
    const int s_inj = (!SEEDB && cap_t >= t0 && cap_t < t0 + TILE) ? cap_t - t0 : -1;
    T* coll8 = coll + (t0 & 24);  // slot of step t0 + s is coll8[s]
    // adjoints arriving at the bottom row from the band below (column t - 32 KS)
    T dvs[TILE], dvqs[TILE];
    // a block that the dead block before it proved dead needs no test
    bool blk_live = false;
    if (!next_dead) {
      const T* sdb = sd + ((t0 - 32 * KS) & 63);
      const T* sdpb = sdp + ((t0 - 32 * KS) & 63);
#pragma unroll
      for (int s = 0; s < TILE; ++s) {
        dvs[s] = sdb[s];
        if (HAS_P) dvqs[s] = sdpb[s];
      }
      bool live = a.all_blocks != 0 || (!SEEDB && s_inj >= 0);
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        live = live || accL[k] != T(0) || accB[k] != T(0) || dgp[k] != T(0);
        if (HAS_P) live = live || Qacc[k] != T(0) || QaccB[k] != T(0) || dgq[k] != T(0);
      }
#pragma unroll
      for (int s = 0; s < TILE; ++s) {
        live = live || dvs[s] != T(0);
        if (HAS_P) live = live || dvqs[s] != T(0);
      }
      blk_live = __any_sync(0xffffffffu, live);
    }
    if (!blk_live) {
      // The next block is as surely dead when no seed enters it and the
      // adjoints it receives from below (already in shared memory: a window
      // is stored at least one block before this test reads it) are zero.
      // The test reads the 32-column window of the next block's adjoints
      // from below once (lane l its column l) and keeps the answer for the
      // window's four blocks.
      const int wn = (t0 - TILE - 32 * KS) >> 5;
      if (wn != zw_idx) {
        const int c = (32 * wn + lane) & 63;
        const bool nzw = sd[c] != T(0) || (HAS_P && sdp[c] != T(0));
        zw_any = __any_sync(0xffffffffu, nzw);
        zw_idx = wn;
      }
      const bool nxt_live = zw_any || (!SEEDB && cap_t >= t0 - TILE && cap_t < t0);
      next_dead = !nxt_live;
      if (nxt_live) {
        // the next block is live: its rows, and in cur the saved row it
        // starts from (t0 - 2, this block's first row)
#pragma unroll
        for (int s = 0; s < TILE; ++s) {
          load_saved_row<T, KS>(sRl, t0 - TILE - 2 + s, Fn[s]);
          if (HAS_P) load_saved_row<T, KS>(sPl, t0 - TILE - 2 + s, FPn[s]);
        }
        load_saved_row<T, KS>(sRl, t0 - 2, cur);
        if (HAS_P) load_saved_row<T, KS>(sPl, t0 - 2, Pcur);
      }
      // zeros in the ring only where a flushed tile also holds cells of a
      // live block: the tiles flushed after this block and after the next
      // one share their steps with the block before and the block after
      const bool stage = prev_live || nxt_live;
#pragma unroll
      for (int s = 0; s < TILE; ++s) {
        if (stage) {
          const int ia = (t0 + s - lane) & (RING - 1);
#pragma unroll
          for (int k = 0; k < KS; ++k) {
            myC[k * 32 * S + ia] = T(0);
            if (HAS_P) myQ[k * 32 * S + ia] = T(0);
          }
        }
      }
      if (lane == 0) {  // zero top-row sends: 16-byte stores (coll8 is 32-byte aligned)
        constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
        for (int h = 0; h < TILE / PER; ++h) {
          reinterpret_cast<int4*>(coll8)[h] = make_int4(0, 0, 0, 0);
          if (HAS_P) reinterpret_cast<int4*>(coll8 + 32)[h] = make_int4(0, 0, 0, 0);
        }
      }
      cur_live = false;
      stale = true;
      return;
    }
    cur_live = true;
    next_dead = false;
    if (stale) {
      // after dead blocks: cur holds saved row t0 + 6, loaded by the block
      // before; Xc = X(t0 + 7) with the row -1 value of column t0 + 7 (in
      // this block's window of sb)
      const T b7 = sb[(t0 + 7) & 63];
      const T b7p = HAS_P ? sbp[(t0 + 7) & 63] : T(0);
#pragma unroll
      for (int k = KS - 1; k >= 1; --k) {
        Xc[k] = shfl_up1_rot(lane == 31 ? cur[k - 1] : cur[k]);
        if (HAS_P) PXc[k] = shfl_up1_rot(lane == 31 ? Pcur[k - 1] : Pcur[k]);
      }
      Xc[0] = shfl_up1_rot(lane == 31 ? b7 : cur[0]);
      if (HAS_P) PXc[0] = shfl_up1_rot(lane == 31 ? b7p : Pcur[0]);
      stale = false;
    }
#pragma unroll
    for (int s = 0; s < TILE; ++s) {
      load_saved_row<T, KS>(sRl, t0 - TILE - 2 + s, Fn[s]);
      if (HAS_P) load_saved_row<T, KS>(sPl, t0 - TILE - 2 + s, FPn[s]);
    }
    // The block's row -1 values (column t-1), read into registers before the
    // block's first shared-memory store so that no step waits on a shared load.
    T bvs[TILE], bvps[TILE];
    {
      const int cb0 = (t0 - 1) & 63;
      const T* sb1 = sb + (t0 & 63);
      const T* sbp1 = sbp + (t0 & 63);
#pragma unroll
      for (int s = 0; s < TILE; ++s) {
        bvs[s] = s == 0 ? sb[cb0] : sb1[s - 1];
        if (HAS_P) bvps[s] = s == 0 ? sbp[cb0] : sbp1[s - 1];
      }
    }
#pragma unroll
    for (int s = TILE - 1; s >= 0; --s) {
      const int t = t0 + s;
      // the end cell of a pair receives dL/dR (and dL/dP) as its adjoint
      if (!SEEDB && s == s_inj) {
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          accL[k] += sdR[k];
          if (HAS_P) Qacc[k] += sdP[k];
        }
      }
      // predecessor rows: saved row t-2 and X(t-1)
      const T bv = bvs[s];
      const T bvp = HAS_P ? bvps[s] : T(0);
      T nxt[KS], Pnxt[KS], Xn[KS], PXn[KS];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        nxt[k] = Fc[s][k];
        Pnxt[k] = HAS_P ? FPc[s][k] : T(0);
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
        const int off = k * 32 * S + ia;
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
      // top row's send (column t): lane 0 files it under step t mod 32
      if (lane == 0) {
        coll8[s] = send[0];
        if (HAS_P) coll8[32 + s] = sendq[0];
      }
      // adjoint arriving at the bottom row (lane 31, sub-band KS-1) at t-1
      const T dv = dvs[s];
      const T dvq = HAS_P ? dvqs[s] : T(0);
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
  };

  unsigned gphase = 0;
  bool gdead = false;
  const int ql = wi.Q * p.L;  // local columns of the warp's passes
  int pend_b = 0, pend_d = 0;  // refills waiting for their shared-memory store: blocks to go
  int pbc = 0, pdc = 0;
  T pbv = T(0), pbpv = T(0), pdv = T(0), pdpv = T(0);
  // Work between block t0 and block t0 - 8.
  auto between = [&](const int t0) {
    const bool seedhere = !SEEDB && cap_t >= t0 && cap_t < t0 + TILE;
    // the tiles flushed here have their cells in this block and the one
    // before it; when both were dead they are zero and the ring is not read
    const bool zero_tiles = !cur_live && !prev_live;
    prev_live = cur_live;

    // ---- between blocks
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      const uint32_t nzb = flush_row_tile<T>(a.dC, myC + k * 32 * S, fl[k], fmode[k], foff[k],
                                             p, a.vec, masked, mwd[k], a.nzm != nullptr,
                                             zero_tiles);
      // a chunk is flagged where dC or (uDTW) dQ holds a nonzero value
      uint32_t nzf = nzb;
      if (HAS_P)
        nzf |= flush_row_tile<T>(a.dQ, myQ + k * 32 * S, fl[k], fmode[k], foff[k], p, a.vec, false,
                                 0u, false, zero_tiles);
      if (nzf != 0u && (a.tf_rows != nullptr || a.nzm != nullptr)) {
        // this lane's 8 columns lie in one 32-column and one 128-column block
        const int row = fl[k].band * 32 * KS + 32 * k + lane;
        const long long b = wi.p0 + fl[k].pq;
        const int j0 = fl[k].j0;
        if (a.tf_rows != nullptr) {
          a.tf_rows[(b * ((p.N + 127) >> 7) + (row >> 7)) * a.tf_kr + (j0 >> 5)] = 1;
          a.tf_cols[(b * ((p.M + 127) >> 7) + (j0 >> 7)) * a.tf_kc + (row >> 5)] = 1;
        }
        if (a.nzm != nullptr && nzb != 0u)  // byte (j0 & 31) / 8 of word [b][j0 / 32][row]
          a.nzm[((b * ((p.M + 31) >> 5) + (j0 >> 5)) * a.mask_np + row) * 4 + ((j0 & 31) >> 3)] =
              (uint8_t)nzb;
      }
      const int oq = fl[k].q;
      cursor_prev<GRP>(fl[k], p);
      if (fl[k].q != oq) {  // a new pass
        fmode[k] = row_mode<KS>(fl[k], k, p, wi, foff[k]);
        if (masked) mrow[k] = mask_row<KS>(a.mask, a.mask_np, fl[k], k, p, wi);
      }
      // the word is for the next flush; when the next block is proved dead
      // that flush reads nothing (this block is dead too)
      if (masked && !next_dead) mwd[k] = mrow[k][min(fl[k].j0 >> 5, mwl) * a.mask_np];
    }
    if (seedhere) {
      --cap_i;
      cap_t = cap_i >= 0 ? cap_t - NBL : -1;
      if (cap_i >= 0) {
        const T sr = a.grad_r[wi.p0 + cap_i];
        const T sp = HAS_P ? a.grad_p[wi.p0 + cap_i] : T(0);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          sdR[k] = (seed_lane && k == kstar) ? sr : T(0);
          sdP[k] = (seed_lane && k == kstar) ? sp : T(0);
        }
      }
    }
    // Window refills are loaded from global memory at the end of one block
    // and stored to shared memory three blocks later, so no warp waits for
    // the load even when the blocks between are dead (short); the slots they
    // fill are first read four blocks after the load (by the dead-block test
    // of the next block's adjoints from below, at the start of the fourth).
    if (pend_b > 0 && --pend_b == 0) {
      __syncwarp();
      sb[pbc & 63] = pbv;
      if (HAS_P) sbp[pbc & 63] = pbpv;
      __syncwarp();
    }
    if (pend_d > 0 && --pend_d == 0) {
      __syncwarp();
      sd[pdc & 63] = pdv;
      if (HAS_P) sdp[pdc & 63] = pdpv;
      __syncwarp();
    }
    if ((t0 & 31) == 0) {
      // the window [t0, t0+32) of top-row sends is complete: lane l takes
      // the send of step t0 + l
      __syncwarp();
      const T wdR = coll[lane];
      const T wdP = HAS_P ? coll[32 + lane] : T(0);
      if constexpr (!GRP) {
        const int j = (t0 + lane) - udiv(t0 + lane, p.dL) * p.L;
        dlR[j] = wdR;
        if (HAS_P) dlP[j] = wdP;
      } else {
        const int sl = t0 + lane - wi.off;
        if (sl >= 0 && sl < ql) {
          const int j = sl - udiv(sl, p.dL) * p.L;
          dlR[j] = wdR;
          if (HAS_P) dlP[j] = wdP;
        }
      }
      if constexpr (GRP) group_step(gbar, gphase, gdead);
      else __syncwarp();
      // row -1 values two windows down replace the window just finished
      pbc = t0 - 64 + lane;
      pbv = row_above_saved<T, KS, GRP>(eRa, pbc, p, wi, big);
      if (HAS_P) pbpv = row_above_saved<T, KS, GRP>(ePa, pbc, p, wi, T(0));
      pend_b = 3;
    }
    // the next block (t0 - 8) may open a new window of bottom-row columns
    const int dwn = (t0 - TILE - 32 * KS) >> 5;
    if (dwn != dw) {
      dw = dwn;
      pdc = 32 * (dw - 1) + lane;
      pdv = push_from_below<T, SEEDB, GRP>(dlRb, pdc, p, wi, a.grad_r);
      if (HAS_P) pdpv = push_from_below<T, SEEDB, GRP>(dlPb, pdc, p, wi, a.grad_p);
      pend_d = 3;
    }
  };

#pragma unroll 1
  for (int b = btop; b >= 0; b -= 2) {
    run_block(TILE * b, F, FP, G, GP);
    between(TILE * b);
    if (b == 0) break;
    run_block(TILE * (b - 1), G, GP, F, FP);
    between(TILE * (b - 1));
  }
}

template <typename T, int KS, bool HAS_P, bool HAS_BAND>
int launch_fwd(const SdtwArgs<T>& a, cudaStream_t st) {
  auto kern = a.p.G > 1 ? sdtw_fwd_kernel<T, KS, HAS_P, HAS_BAND, true>
                        : sdtw_fwd_kernel<T, KS, HAS_P, HAS_BAND, false>;
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
  // a pair's end cell is the last lane of the last sub-band when N is a
  // multiple of the band height: its seed then needs no per-step test
  const bool seedb = (a.p.N % (32 * KS)) == 0;
  auto kern = a.p.G > 1 ? (seedb ? sdtw_bwd_kernel<T, KS, HAS_P, true, true>
                                 : sdtw_bwd_kernel<T, KS, HAS_P, false, true>)
                        : (seedb ? sdtw_bwd_kernel<T, KS, HAS_P, true, false>
                                 : sdtw_bwd_kernel<T, KS, HAS_P, false, false>);
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

// Blocks of `wpc` warps per SM that both sweeps of a plan can keep resident
// with `smem` bytes each (registers and shared memory), or -1 when the
// device cannot be asked (no GPU: the shared-memory bound alone is used).
// GRP: the kernels with band groups.
template <typename T, int KS, bool HAS_P, bool GRP>
int resident_blocks(int wpc, size_t smem) {
  const void* kerns[4] = {(const void*)sdtw_fwd_kernel<T, KS, HAS_P, false, GRP>,
                          (const void*)sdtw_fwd_kernel<T, KS, HAS_P, true, GRP>,
                          (const void*)sdtw_bwd_kernel<T, KS, HAS_P, false, GRP>,
                          (const void*)sdtw_bwd_kernel<T, KS, HAS_P, true, GRP>};
  int best = INT_MAX;
  for (const void* k : kerns) {
    int n = 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, 32 * wpc, smem) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    best = n < best ? n : best;
  }
  return best;
}

int resident_blocks_any(int eb, int KS, bool has_p, bool grp, int wpc, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, bool, bool, int, size_t>, int> cache;
  const auto key = std::make_tuple(eb, KS, has_p, grp, wpc, smem);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = -1;
#define TW_RB(TT, K)                                                                          \
  n = has_p ? (grp ? resident_blocks<TT, K, true, true>(wpc, smem)                             \
                   : resident_blocks<TT, K, true, false>(wpc, smem))                           \
            : (grp ? resident_blocks<TT, K, false, true>(wpc, smem)                            \
                   : resident_blocks<TT, K, false, false>(wpc, smem))
  if (eb == 4) {
    if (KS == 1) TW_RB(float, 1);
    else if (KS == 2) TW_RB(float, 2);
    else if (KS == 3) TW_RB(float, 3);
    else TW_RB(float, 4);
  } else {
    if (KS == 1) TW_RB(double, 1);
    else if (KS == 2) TW_RB(double, 2);
    else if (KS == 3) TW_RB(double, 3);
    else TW_RB(double, 4);
  }
#undef TW_RB
  if (n >= 0) {
    std::lock_guard<std::mutex> g(mu);
    cache[key] = n;
  }
  return n;
}

}  // namespace

#ifndef SLICE_ALIGN
#define SLICE_ALIGN(x) (x)
#endif

static int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : fallback;
}

StreamPlan make_stream_plan(int B, int N, int M, int eb, bool has_p, int sms) {
  StreamPlan p;
  p.B = B;
  p.N = N;
  p.M = M;
  // Sub-bands per warp: ILP inside a warp.  Thread-level parallelism (warps
  // per SM) is what hides the soft-min's latency, and every sub-band costs a
  // ring of shared memory, so two sub-bands by default; one with the uDTW
  // penalty, whose second stream doubles the registers and shared memory of
  // a sub-band (cfg5 uDTW: 68.2 ms per step at one, 71.8 at two).
  //
  // Small batches (a batch sharded over 4 or 8 GPUs, or fewer than 12 pairs
  // per SM on one) give too few warps to hide the latency.  Band groups put
  // G warps on each pair: G is the smallest of 2 and 4 that brings B * G to
  // 12 warps per SM (or the largest that applies), with G dividing NB and the
  // lag L / G >= 32 KS + 128 met without widening L.  N=M=1024, fp32 soft-DTW
  // fwd+bwd on the cost: B=32 4.56 ms (best sub-band count, one warp per
  // pair) -> 1.71 ms (G = 4), B=512 5.77 -> 3.80 ms (G = 4), B=1024 7.58 ->
  // 6.81 ms (G = 2), B=2048 13.1 ms at G = 1 vs 13.3 at G = 2; uDTW B=512
  // 10.4 -> 7.7 ms, fp64 B=512 28.0 -> 17.4 (G = 2) / 18.7 ms (G = 4).  With
  // groups, more sub-bands per warp lose: B=512 4 sub-bands and G = 2
  // 4.23 ms, B=1024 4 and G = 2 8.13 ms.  TW_STREAM_KS and TW_STREAM_G force
  // either choice.
  const int ks_def = (N <= 32 || has_p) ? 1 : 2;
  const int ks_env = env_int("TW_STREAM_KS", 0);
  int ks = ks_env > 0 ? ks_env : ks_def;
  ks = ks >= 4 ? 4 : (ks < 1 ? 1 : ks);
  auto group_fits = [&](int g, int k) {
    const int r = 32 * k;
    const int nb = (N + r - 1) / r;
    return nb % g == 0 && M + 1 >= g * (r + 128);
  };
  int G = env_int("TW_STREAM_G", 0);
  if (G <= 0) {
    G = 1;
    const long long want = 12LL * sms;
    if ((long long)B < want) {
      for (int g : {2, 4}) {
        if (!group_fits(g, ks)) continue;
        G = g;
        if ((long long)B * g >= want) break;
      }
    }
  }
  p.KS = ks;
  const int rows = 32 * p.KS;
  p.NB = (N + rows - 1) / rows;
  // G warps share a group's pairs, one band in G each; G divides NB.
  G = G >= 4 ? 4 : (G >= 2 ? 2 : 1);
  while (G > 1 && p.NB % G != 0) G /= 2;
  p.G = G;
  p.NBg = p.NB / G;
  p.dNB = make_divisor(p.NB);
  p.dNBg = make_divisor(p.NBg);
  // The band-to-band delay line needs a lag D >= 32*KS + 128 between the
  // starts of consecutive passes (see row_above); D = L / G, so L >= G (32 KS
  // + 128), a multiple of 8 G.  A single-band pair has no delay line and only
  // needs the padding column.
  int L = M + 1;
  if (p.NB > 1 && L < G * (rows + 128)) L = G * (rows + 128);
  p.L = (L + TILE * G - 1) / (TILE * G) * (TILE * G);
  p.D = p.L / G;
  p.dL = make_divisor(p.L);
  const int S = eb == 4 ? RingStride<float>::value : RingStride<double>::value;
  const size_t per_w = (size_t)warp_smem_elems(p.KS, S, has_p) * eb;
  // the groups' mbarriers; none without groups, where 64 bytes more per CTA
  // would push cfg5's backward (8 CTAs of 19968 + 1024 bytes = 164 KB exactly)
  // to the next shared-memory carveout and cost it 32 KB of L1
  const size_t hdr = G > 1 ? StreamPlan::kSmemHeader : 0;
  // Warps per SM: bounded by shared memory (the per-lane rings), by the
  // registers of the heavier of the two sweeps, and by 32.
  int wps = (int)((size_t)(216 * 1024) / per_w);
  wps = wps < 1 ? 1 : (wps > 32 ? 32 : wps);
  const int cap = env_int("TW_STREAM_WPS", 0);
  if (cap > 0 && cap < wps) wps = cap;
  // Warps per CTA (4, 2 or 1; a multiple of G) and pairs per group.  Every
  // group carries whole pairs and every CTA is resident from the start, so a
  // sweep lasts about (pairs per group) x (warps on the fullest SM)
  // warp-steps of issue.  Take the CTA size that minimises that product
  // (ties: the larger CTA).  Small CTAs spread the warps evenly: 2048 warps
  // in 4-warp CTAs put 16 warps on some SMs, in 2-warp CTAs at most 14.
  int wpc = G;
  long long per_group = 1, groups_needed = 1, best_cost = LLONG_MAX;
  for (int c : {4, 2, 1}) {
    if (c > wps || c % G != 0) continue;
    int n = wps / c;
    const int resident = resident_blocks_any(eb, p.KS, has_p, G > 1, c, per_w * c + hdr);
    if (resident >= 0 && resident < n) n = resident;
    if (n < 1) continue;
    const int gpc = c / G;
    const long long capg = (long long)sms * n * gpc;
    const long long pg = B > 0 ? (B + capg - 1) / capg : 1;
    const long long gn = B > 0 ? (B + pg - 1) / pg : 1;
    const long long ctas_c = (gn + gpc - 1) / gpc;
    const long long fullest = c * ((ctas_c + sms - 1) / sms);
    const long long cost = pg * fullest;
    if (cost < best_cost) {
      best_cost = cost;
      wpc = c;
      per_group = pg;
      groups_needed = gn;
    }
  }
  if (best_cost == LLONG_MAX) {  // nothing fits the residency estimate: one group per CTA
    wpc = G;
    per_group = B > 0 ? (B + sms - 1) / sms : 1;
    groups_needed = B > 0 ? (B + per_group - 1) / per_group : 1;
  }
  const int gpc = wpc / G;
  int ctas = (int)((groups_needed + gpc - 1) / gpc);
  if (ctas < 1) ctas = 1;
  p.wpc = wpc;
  p.warps = ctas * wpc;
  const int groups = p.warps / G;
  p.base = B / groups;
  p.rem = B % groups;
  const long long maxpairs = p.base + (p.rem ? 1 : 0);
  const long long Tw = maxpairs * p.NBg * p.L + 32 * p.KS - 1 + (long long)(G - 1) * p.D;
  p.tmax = (Tw + TILE - 1) / TILE * TILE;
  p.tstride = SLICE_ALIGN(p.tmax + StreamPlan::kPreRows);
  p.smem_fwd = per_w * p.wpc + hdr;
  p.smem_bwd = per_w * p.wpc + hdr;
  return p;
}

Divisor make_divisor(int d) {
  Divisor v;
  v.d = d < 1 ? 1 : d;
  int l = 0;
  while ((1ll << l) < v.d) ++l;
  v.l = l;
  v.m = (uint32_t)((((unsigned __int128)1 << 32) * (((unsigned __int128)1 << l) - v.d)) / v.d + 1);
  return v;
}

int dp_take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dp_error, sizeof(int)) != cudaSuccess) return kLaunch;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_dp_error, &zero, sizeof(int));
  }
  return v;
}

template <typename T>
int sdtw_stream_forward(const SdtwArgs<T>& a, bool has_p, bool has_band, cudaStream_t st) {
  switch (a.p.KS) {
    case 1: return fwd_ks<T, 1>(a, has_p, has_band, st);
    case 2: return fwd_ks<T, 2>(a, has_p, has_band, st);
    case 3: return fwd_ks<T, 3>(a, has_p, has_band, st);
    case 4: return fwd_ks<T, 4>(a, has_p, has_band, st);
    default: return set_error(kUnsupported, "sdtw forward: unsupported sub-band count %d", a.p.KS);
  }
}

template <typename T>
int sdtw_stream_backward(const SdtwArgs<T>& a, bool has_p, bool /*has_band*/, cudaStream_t st) {
  switch (a.p.KS) {
    case 1: return bwd_ks<T, 1>(a, has_p, st);
    case 2: return bwd_ks<T, 2>(a, has_p, st);
    case 3: return bwd_ks<T, 3>(a, has_p, st);
    case 4: return bwd_ks<T, 4>(a, has_p, st);
    default: return set_error(kUnsupported, "sdtw backward: unsupported sub-band count %d", a.p.KS);
  }
}

template int sdtw_stream_forward<float>(const SdtwArgs<float>&, bool, bool, cudaStream_t);
template int sdtw_stream_forward<double>(const SdtwArgs<double>&, bool, bool, cudaStream_t);
template int sdtw_stream_backward<float>(const SdtwArgs<float>&, bool, bool, cudaStream_t);
template int sdtw_stream_backward<double>(const SdtwArgs<double>&, bool, bool, cudaStream_t);

}  // namespace tw
