// Fused JEANIE and FVM for float32 (sm_100a): one CTA per (query, support)
// pair builds the pair's query/support cost from the features, runs the
// viewpoint soft-min (FVM) and the temporal soft-min DP in shared memory, and
// in the backward runs the DP adjoint and the chain rule back to the features.
//
// Reference: hibana2077/torchwarp src/torchwarp/csrc/jeanie_cuda.cu:309-503
// (jeanie_fused_forward_kernel / jeanie_fused_backward_kernel: the cost from
// the Gram matrix inside the sweep) and src/torchwarp/jeanie/fvm.py:15-67
// (viewpoint soft-min, then soft-DTW).  Recurrences as jeanie.cu.
//
// Layout and roles.
//   * The CTA has W = ceil(D / 128) warps; warp w owns features
//     [128 w, 128 w + 128) of every query row and support frame (four per
//     lane).  Each warp streams all K*T query rows of the pair (its feature
//     slice, 512 contiguous bytes per row, JF_PF rows in flight), keeps its slice
//     of the U support frames in registers, and reduces the U dot products
//     and |q|^2 of a row across its lanes by recursive halving (16 values in
//     16 shuffles).  The W partial sums of a row meet in shared memory in a
//     fixed order (deterministic).
//   * The cost [K, T, U] stays in shared memory; JEANIE's DP runs on it,
//     FVM first reduces it over the viewpoints to [T, U] and runs the DP on
//     that.  HBM sees the features once per direction plus small saved state
//     (the cost, the DP values and per-diagonal minima).
//   * The DP is a warp-level anti-diagonal wavefront (warp 0, __syncwarp
//     between diagonals); a diagonal's cells (every t on it, every
//     viewpoint) are spread over the lanes.
//
// Precision.  Along a diagonal d = t + u, R grows with d (about d times a
// typical cost), so float32 R loses the resolution of the soft-min weights
// exp(-(R_p - m)/gamma) as d grows; the reference's own float32 has that
// error.  Here every diagonal is stored relative to its own base, the sum of
// the minima of the diagonals before it: r = R - base[d], with
// base[d+1] = base[d] + min(r on d).  A predecessor on diagonal d-1 then
// enters as r_p - mn[d-1], one on d-2 as r_p - mn[d-2] - mn[d-1], so the
// values compared by the soft-min are of the size of a few costs, not of R.
// The natural R (the accumulator output) is r + base, formed in double.
#include "common.cuh"

namespace tw {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int JF_SLOT = 16;   // values reduced per query row: U dots (slots < 15), |q|^2 (slot 15)
constexpr int JF_ROWS = 32;   // query rows per shared-memory reduction chunk
constexpr int JF_PF = 8;      // query rows in flight per warp (registers)
static_assert(JF_ROWS % JF_PF == 0, "chunk must hold whole prefetch groups");

struct JFGeom {
  int K1, K2, K, T, U, D, s1, s2, metric;
  int R;        // K * T query rows
  float kap;    // log2(e) / gamma
  float ikap;   // gamma ln 2
};

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fminf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

// Sum of v[0..15] over the 32 lanes by recursive halving: after the step
// with offset o the lane keeps the half of its values selected by lane bit
// o and adds its partner's copy of that half.  Returns the full sum of slot
// jf_slot(lane) (each slot ends up in two lanes, l and l ^ 1).
__device__ __forceinline__ float reduce16(float (&v)[JF_SLOT], int lane) {
#pragma unroll
  for (int h = 8, o = 16; h >= 1; h >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? v[i] : v[i + h];
      const float keep = up ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(FULL, send, o);
    }
  }
  return v[0] + __shfl_xor_sync(FULL, v[0], 1);
}
__device__ __forceinline__ int jf_slot(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

__device__ __forceinline__ float4 ld_row4(const float* p, bool ok) {
  return ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}
__device__ __forceinline__ void fma4(float4& acc, float w, float4 v) {
  acc.x = fmaf(w, v.x, acc.x);
  acc.y = fmaf(w, v.y, acc.y);
  acc.z = fmaf(w, v.z, acc.z);
  acc.w = fmaf(w, v.w, acc.w);
}

// ------------------------------------------------------------ the DP
// Grid [K1][K2][T][U] (natural layout), viewpoint window |n1'-n1| <= s1,
// |n2'-n2| <= s2; one warp.

// Forward: rw = R - base[t+u]; mn[d] = min of rw on diagonal d; base[d] in
// double (only for the natural accumulator and the output).
__device__ void dp_forward_warp(const float* Cw, float* rw, float* mn, double* base, int K1,
                                int K2, int T, int U, int s1, int s2, float kap, float ikap,
                                int lane) {
  const int K = K1 * K2, TU = T * U, ND = T + U - 1;
  double acc = 0.0;
  for (int d = 0; d < ND; ++d) {
    if (lane == 0) base[d] = acc;
    const int tlo = max(0, d - U + 1), thi = min(T - 1, d);
    const int nc = (thi - tlo + 1) * K;
    const float m1 = d >= 1 ? mn[d - 1] : 0.f;
    const float m2 = d >= 2 ? mn[d - 2] + mn[d - 1] : 0.f;
    float lmin = INFINITY;
    for (int i = lane; i < nc; i += 32) {
      const int tt = i / K, n = i - tt * K, t = tlo + tt, u = d - t;
      const int o = n * TU + t * U + u;
      float r = Cw[o];
      if (d > 0) {
        const int n1 = n / K2, n2 = n - n1 * K2;
        const int a1 = max(0, n1 - s1), b1 = min(K1 - 1, n1 + s1);
        const int a2 = max(0, n2 - s2), b2 = min(K2 - 1, n2 + s2);
        float m = INFINITY;
        for (int x1 = a1; x1 <= b1; ++x1)
          for (int x2 = a2; x2 <= b2; ++x2) {
            const float* rp = rw + (x1 * K2 + x2) * TU;
            if (t > 0) m = fminf(m, rp[(t - 1) * U + u] - m1);
            if (u > 0) m = fminf(m, rp[t * U + u - 1] - m1);
            if (t > 0 && u > 0) m = fminf(m, rp[(t - 1) * U + u - 1] - m2);
          }
        float s = 0.f;
        for (int x1 = a1; x1 <= b1; ++x1)
          for (int x2 = a2; x2 <= b2; ++x2) {
            const float* rp = rw + (x1 * K2 + x2) * TU;
            if (t > 0) s += ex2((m - (rp[(t - 1) * U + u] - m1)) * kap);
            if (u > 0) s += ex2((m - (rp[t * U + u - 1] - m1)) * kap);
            if (t > 0 && u > 0) s += ex2((m - (rp[(t - 1) * U + u - 1] - m2)) * kap);
          }
        r += m - lg2(s) * ikap;
      }
      rw[o] = r;
      lmin = fminf(lmin, r);
    }
    lmin = warp_min(lmin);
    if (lane == 0) mn[d] = lmin;
    acc += (double)lmin;
    __syncwarp();
  }
}

// Soft-min over the viewpoints of the end cells (relative to base[ND-1]).
__device__ float dp_final(const float* rw, int K, int TU, float kap, float ikap, int lane) {
  float m = INFINITY;
  for (int n = lane; n < K; n += 32) m = fminf(m, rw[n * TU + TU - 1]);
  m = warp_min(m);
  float s = 0.f;
  for (int n = lane; n < K; n += 32) s += ex2((m - rw[n * TU + TU - 1]) * kap);
  s = warp_sum(s);
  return m - lg2(s) * ikap;
}

// Backward (pull form): Gw = dL/dR for L = g_out * out + <g_R, R>.  The
// weight of successor s of cell k is 2^((R_s - C_s - R_k) kap), with
// R_s - R_k = r_s - r_k + mn[d] (s on d+1) or + mn[d] + mn[d+1] (s on d+2).
__device__ void dp_backward_warp(const float* Cw, const float* rw, const float* mn, float* Gw,
                                 float g_out, const float* gR, int K1, int K2, int T, int U,
                                 int s1, int s2, float kap, float ikap, int lane) {
  const int K = K1 * K2, TU = T * U, ND = T + U - 1;
  const float fin = dp_final(rw, K, TU, kap, ikap, lane);
  for (int d = ND - 1; d >= 0; --d) {
    const int tlo = max(0, d - U + 1), thi = min(T - 1, d);
    const int nc = (thi - tlo + 1) * K;
    const float e1 = d + 1 < ND ? mn[d] : 0.f;
    const float e2 = d + 2 < ND ? mn[d] + mn[d + 1] : 0.f;
    for (int i = lane; i < nc; i += 32) {
      const int tt = i / K, n = i - tt * K, t = tlo + tt, u = d - t;
      const int o = n * TU + t * U + u;
      const float rk = rw[o];
      float acc = 0.f;
      if (t == T - 1 && u == U - 1) {
        acc = g_out * ex2((fin - rk) * kap);
      } else {
        const int n1 = n / K2, n2 = n - n1 * K2;
        const int a1 = max(0, n1 - s1), b1 = min(K1 - 1, n1 + s1);
        const int a2 = max(0, n2 - s2), b2 = min(K2 - 1, n2 + s2);
        const float k1 = e1 - rk, k2 = e2 - rk;
        for (int x1 = a1; x1 <= b1; ++x1)
          for (int x2 = a2; x2 <= b2; ++x2) {
            const int p = (x1 * K2 + x2) * TU;
            if (t + 1 < T) {
              const int so = p + (t + 1) * U + u;
              acc += ex2(((rw[so] - Cw[so]) + k1) * kap) * Gw[so];
            }
            if (u + 1 < U) {
              const int so = p + t * U + u + 1;
              acc += ex2(((rw[so] - Cw[so]) + k1) * kap) * Gw[so];
            }
            if (t + 1 < T && u + 1 < U) {
              const int so = p + (t + 1) * U + u + 1;
              acc += ex2(((rw[so] - Cw[so]) + k2) * kap) * Gw[so];
            }
          }
      }
      if (gR != nullptr) acc += gR[o];
      Gw[o] = acc;
    }
    __syncwarp();
  }
}

// ------------------------------------------------------ shared memory

struct JFSmem {
  float* mn;    // [ND] per-diagonal minima
  double* base; // [ND] per-diagonal bases
  float* s2;    // [16] support norms
  float* C;     // [K T U] cost (FVM backward: dC, then dsq, in place)
  float* tmp;   // FVM: [T U] viewpoint soft-min
  float* r;     // [dpn] relative DP values
  float* G;     // [dpn] adjoint
  float* part;  // [W][JF_ROWS][16] partial row sums (forward, features)
  float* Sp;    // [K T][16] dL/dsq per query row, zero past U (backward, features)
  float* rs;    // [K T] row sums of Sp
  float* cs;    // [16] column sums of Sp
};

__host__ __device__ inline size_t jf_align16(size_t n) { return (n + 15) & ~size_t(15); }

// Byte offsets of the shared-memory regions (same on host and device).
__host__ __device__ inline size_t jf_smem_layout(int K, int T, int U, int W, bool fvm, bool fwd,
                                                 bool feat, size_t* off) {
  const int R = K * T;
  const bool chain = !fwd && feat;
  const int KTU = K * T * U, TU = T * U, ND = T + U - 1, dpn = fvm ? TU : KTU;
  size_t o = 0;
  off[0] = o; o = jf_align16(o + sizeof(double) * ND);   // base
  off[1] = o; o = jf_align16(o + sizeof(float) * ND);    // mn
  off[2] = o; o = jf_align16(o + sizeof(float) * 16);    // s2
  off[3] = o; o = jf_align16(o + sizeof(float) * KTU);   // C
  off[4] = o; o = jf_align16(o + sizeof(float) * (fvm ? TU : 0));   // tmp
  off[5] = o; o = jf_align16(o + sizeof(float) * dpn);   // r
  off[6] = o; o = jf_align16(o + sizeof(float) * (fwd ? 0 : dpn));  // G
  off[7] = o; o = jf_align16(o + sizeof(float) * ((fwd && feat) ? W * JF_ROWS * JF_SLOT : 0));
  off[8] = o; o = jf_align16(o + sizeof(float) * (chain ? R * JF_SLOT : 0));
  off[9] = o; o = jf_align16(o + sizeof(float) * (chain ? R : 0));
  off[10] = o; o = jf_align16(o + sizeof(float) * (chain ? JF_SLOT : 0));
  return o;
}

__device__ inline JFSmem jf_carve(unsigned char* smem, int K, int T, int U, int W, bool fvm,
                                  bool fwd, bool feat) {
  size_t off[11];
  jf_smem_layout(K, T, U, W, fvm, fwd, feat, off);
  JFSmem s;
  s.base = reinterpret_cast<double*>(smem + off[0]);
  s.mn = reinterpret_cast<float*>(smem + off[1]);
  s.s2 = reinterpret_cast<float*>(smem + off[2]);
  s.C = reinterpret_cast<float*>(smem + off[3]);
  s.tmp = reinterpret_cast<float*>(smem + off[4]);
  s.r = reinterpret_cast<float*>(smem + off[5]);
  s.G = reinterpret_cast<float*>(smem + off[6]);
  s.part = reinterpret_cast<float*>(smem + off[7]);
  s.Sp = reinterpret_cast<float*>(smem + off[8]);
  s.rs = reinterpret_cast<float*>(smem + off[9]);
  s.cs = reinterpret_cast<float*>(smem + off[10]);
  return s;
}

// Saved state per pair (floats): [cost K T U (features only)] [r dpn]
// [tmp T U (FVM)] [mn ND], each section 16-byte aligned over the batch.
struct JFSaved {
  size_t c, r, t, m, total;  // byte offsets of the sections and the total
};
__host__ __device__ inline JFSaved jf_saved_layout(int B, int K, int T, int U, bool fvm,
                                                   bool feat) {
  const size_t KTU = (size_t)K * T * U, TU = (size_t)T * U, ND = T + U - 1;
  const size_t dpn = fvm ? TU : KTU;
  JFSaved s;
  size_t o = 0;
  s.c = o; o = jf_align16(o + sizeof(float) * (feat ? KTU * B : 0));
  s.r = o; o = jf_align16(o + sizeof(float) * dpn * B);
  s.t = o; o = jf_align16(o + sizeof(float) * (fvm ? TU * B : 0));
  s.m = o; o = jf_align16(o + sizeof(float) * ND * B);
  s.total = o;
  return s;
}

struct JFArgs {
  const float* q;      // [B, K T, D] query rows in (n, t) order (features)
  const float* s;      // [B, U, D] support frames (features)
  const float* cost;   // [B, K, T, U] cost input (no features), or null
  unsigned char* saved;
  float* out;          // [B]
  float* Rnat;         // [B, K, T, U] natural accumulator (JEANIE, optional)
  const float* g_out;  // [B]
  const float* g_R;    // [B, K, T, U] or null
  float* dq;           // [B, K T, D]
  float* ds;           // [B, U, D]
  float* dC;           // [B, K, T, U] (no features)
  int B, W;
  JFGeom g;
  JFSaved sv;
};

// Load this warp's slice of the support frames and write the frames' |s|^2
// (all warps' partials, fixed order) to s2[0..U).
template <int CU>
__device__ __forceinline__ void load_support(const JFArgs& a, int b, int warp, int lane, int d0,
                                             bool dv, float4 (&sv)[CU], float* part,
                                             float* s2) {
  const JFGeom& g = a.g;
  const float* sb = a.s + (long long)b * g.U * g.D + d0;
  float v[JF_SLOT];
#pragma unroll
  for (int u = 0; u < JF_SLOT; ++u) v[u] = 0.f;
#pragma unroll
  for (int u = 0; u < CU; ++u) {
    sv[u] = ld_row4(sb + (long long)u * g.D, dv && u < g.U);
    v[u] = dot4(sv[u], sv[u]);
  }
  const float red = reduce16(v, lane);
  if (!(lane & 1)) part[warp * JF_SLOT + jf_slot(lane)] = red;
  __syncthreads();
  if ((int)threadIdx.x < g.U) {
    float t = 0.f;
    for (int w = 0; w < a.W; ++w) t += part[w * JF_SLOT + threadIdx.x];
    s2[threadIdx.x] = t;
  }
  __syncthreads();
}

// The pair's cost [K T, U] into C (shared memory) from the features.
template <int CU>
__device__ void build_cost(const JFArgs& a, int b, const JFSmem& sm, float4 (&sv)[CU]) {
  const JFGeom& g = a.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d0 = 128 * warp + 4 * lane;
  const bool dv = d0 < g.D;
  load_support<CU>(a, b, warp, lane, d0, dv, sv, sm.part, sm.s2);
  const float* qb = a.q + (long long)b * g.R * g.D + d0;
  float4 pf[JF_PF];
#pragma unroll
  for (int p = 0; p < JF_PF; ++p) pf[p] = ld_row4(qb + (long long)p * g.D, dv && p < g.R);
  for (int r0 = 0; r0 < g.R; r0 += JF_ROWS) {
#pragma unroll 1
    for (int k = 0; k < JF_ROWS; k += JF_PF) {
#pragma unroll
      for (int p = 0; p < JF_PF; ++p) {
        const int r = r0 + k + p;
        const float4 qv = pf[p];
        const int rn = r + JF_PF;
        pf[p] = ld_row4(qb + (long long)rn * g.D, dv && rn < g.R);
        if (r < g.R) {
          float v[JF_SLOT];
#pragma unroll
          for (int u = 0; u < JF_SLOT; ++u) v[u] = 0.f;
#pragma unroll
          for (int u = 0; u < CU; ++u) v[u] = dot4(qv, sv[u]);
          v[JF_SLOT - 1] = dot4(qv, qv);
          const float red = reduce16(v, lane);
          if (!(lane & 1)) sm.part[(warp * JF_ROWS + k + p) * JF_SLOT + jf_slot(lane)] = red;
        }
      }
    }
    __syncthreads();
    const int nr = min(JF_ROWS, g.R - r0);
    for (int i = threadIdx.x; i < nr * g.U; i += blockDim.x) {
      const int rr = i / g.U, u = i - rr * g.U;
      float dot = 0.f, q2 = 0.f;
      for (int w = 0; w < a.W; ++w) {
        dot += sm.part[(w * JF_ROWS + rr) * JF_SLOT + u];
        q2 += sm.part[(w * JF_ROWS + rr) * JF_SLOT + JF_SLOT - 1];
      }
      const float raw = (q2 + sm.s2[u]) - 2.f * dot;
      const float sq = raw > 0.f ? raw : 0.f;
      sm.C[(r0 + rr) * g.U + u] = g.metric == 1 ? sqrtf(sq) : sq;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ kernels

template <int CU, bool FVM, bool FEAT>
__global__ void __launch_bounds__(128) jf_forward_kernel(const JFArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const JFGeom& g = a.g;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const JFSmem sm = jf_carve(smem_raw, g.K, g.T, g.U, a.W, FVM, true, FEAT);
  const int KTU = g.K * g.T * g.U, TU = g.T * g.U, ND = g.T + g.U - 1;
  const int dpn = FVM ? TU : KTU;
  if constexpr (FEAT) {
    float4 sv[CU];
    build_cost<CU>(a, b, sm, sv);
    float* Cs = reinterpret_cast<float*>(a.saved + a.sv.c) + (long long)b * KTU;
    for (int i = threadIdx.x; i < KTU; i += blockDim.x) Cs[i] = sm.C[i];
  } else {
    const float* Cb = a.cost + (long long)b * KTU;
    for (int i = threadIdx.x; i < KTU; i += blockDim.x) sm.C[i] = __ldg(Cb + i);
    __syncthreads();
  }
  if constexpr (FVM) {
    // temporal[t, u] = soft-min over the viewpoints of C[n, t, u]
    for (int i = threadIdx.x; i < TU; i += blockDim.x) {
      float m = INFINITY;
      for (int n = 0; n < g.K; ++n) m = fminf(m, sm.C[n * TU + i]);
      float s = 0.f;
      for (int n = 0; n < g.K; ++n) s += ex2((m - sm.C[n * TU + i]) * g.kap);
      sm.tmp[i] = m - lg2(s) * g.ikap;
    }
    __syncthreads();
  }
  if (warp == 0) {
    if constexpr (FVM)
      dp_forward_warp(sm.tmp, sm.r, sm.mn, sm.base, 1, 1, g.T, g.U, 0, 0, g.kap, g.ikap, lane);
    else
      dp_forward_warp(sm.C, sm.r, sm.mn, sm.base, g.K1, g.K2, g.T, g.U, g.s1, g.s2, g.kap,
                      g.ikap, lane);
    const float fin = dp_final(sm.r, FVM ? 1 : g.K, TU, g.kap, g.ikap, lane);
    if (lane == 0) a.out[b] = (float)(sm.base[ND - 1] + (double)fin);
  }
  __syncthreads();
  float* rs = reinterpret_cast<float*>(a.saved + a.sv.r) + (long long)b * dpn;
  for (int i = threadIdx.x; i < dpn; i += blockDim.x) rs[i] = sm.r[i];
  float* ms = reinterpret_cast<float*>(a.saved + a.sv.m) + (long long)b * ND;
  for (int i = threadIdx.x; i < ND; i += blockDim.x) ms[i] = sm.mn[i];
  if constexpr (FVM) {
    float* ts = reinterpret_cast<float*>(a.saved + a.sv.t) + (long long)b * TU;
    for (int i = threadIdx.x; i < TU; i += blockDim.x) ts[i] = sm.tmp[i];
  } else {
    if (a.Rnat != nullptr) {
      float* Rb = a.Rnat + (long long)b * KTU;
      for (int i = threadIdx.x; i < KTU; i += blockDim.x) {
        const int tu = i % TU, t = tu / g.U, u = tu - t * g.U;
        Rb[i] = (float)(sm.base[t + u] + (double)sm.r[i]);
      }
    }
  }
}

template <int CU, bool FVM, bool FEAT>
__global__ void __launch_bounds__(128) jf_backward_kernel(const JFArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const JFGeom& g = a.g;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const JFSmem sm = jf_carve(smem_raw, g.K, g.T, g.U, a.W, FVM, false, FEAT);
  const int KTU = g.K * g.T * g.U, TU = g.T * g.U, ND = g.T + g.U - 1;
  const int dpn = FVM ? TU : KTU;
  const float* Cb = FEAT ? reinterpret_cast<const float*>(a.saved + a.sv.c) + (long long)b * KTU
                         : a.cost + (long long)b * KTU;
  for (int i = threadIdx.x; i < KTU; i += blockDim.x) sm.C[i] = __ldg(Cb + i);
  const float* rs = reinterpret_cast<const float*>(a.saved + a.sv.r) + (long long)b * dpn;
  for (int i = threadIdx.x; i < dpn; i += blockDim.x) sm.r[i] = __ldg(rs + i);
  const float* ms = reinterpret_cast<const float*>(a.saved + a.sv.m) + (long long)b * ND;
  for (int i = threadIdx.x; i < ND; i += blockDim.x) sm.mn[i] = __ldg(ms + i);
  if constexpr (FVM) {
    const float* ts = reinterpret_cast<const float*>(a.saved + a.sv.t) + (long long)b * TU;
    for (int i = threadIdx.x; i < TU; i += blockDim.x) sm.tmp[i] = __ldg(ts + i);
  }
  __syncthreads();
  if (warp == 0) {
    const float go = __ldg(a.g_out + b);
    if constexpr (FVM)
      dp_backward_warp(sm.tmp, sm.r, sm.mn, sm.G, go, nullptr, 1, 1, g.T, g.U, 0, 0, g.kap,
                       g.ikap, lane);
    else
      dp_backward_warp(sm.C, sm.r, sm.mn, sm.G, go,
                       a.g_R != nullptr ? a.g_R + (long long)b * KTU : nullptr, g.K1, g.K2, g.T,
                       g.U, g.s1, g.s2, g.kap, g.ikap, lane);
  }
  __syncthreads();
  // dL/dC per cell; with features, dL/dsq per query row (Sp, padded to 16
  // columns with zeros) and its row and column sums: the clamp passes dL/dC
  // where the cost is > 0, the Euclidean root divides by 2 cost (no gradient
  // at cost 0, jeanie/distances.py:34-38)
  auto dcost = [&](int i) {
    if constexpr (FVM) {
      const int tu = i % TU;
      return ex2((sm.tmp[tu] - sm.C[i]) * g.kap) * sm.G[tu];  // viewpoint weight x dtemporal
    } else {
      return sm.G[i];
    }
  };
  if constexpr (!FEAT) {
    for (int i = threadIdx.x; i < KTU; i += blockDim.x) a.dC[(long long)b * KTU + i] = dcost(i);
  } else {
    for (int i = threadIdx.x; i < g.R * JF_SLOT; i += blockDim.x) {
      const int r = i >> 4, u = i & 15;
      float v = 0.f;
      if (u < g.U) {
        const int o = r * g.U + u;
        const float c = sm.C[o], dc = dcost(o);
        v = c > 0.f ? (g.metric == 1 ? dc * (0.5f / c) : dc) : 0.f;
      }
      sm.Sp[i] = v;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < g.R; r += blockDim.x) {
      float t = 0.f;
      for (int u = 0; u < g.U; ++u) t += sm.Sp[r * JF_SLOT + u];
      sm.rs[r] = t;
    }
    if ((int)threadIdx.x < JF_SLOT) {
      float t = 0.f;
      for (int r = 0; r < g.R; ++r) t += sm.Sp[r * JF_SLOT + threadIdx.x];
      sm.cs[threadIdx.x] = t;
    }
    __syncthreads();
    // dq_r = 2 (q_r rowsum_r - sum_u S_ru s_u); ds_u = 2 (s_u colsum_u - sum_r S_ru q_r)
    const int d0 = 128 * warp + 4 * lane;
    const bool dv = d0 < g.D;
    const float* sb = a.s + (long long)b * g.U * g.D + d0;
    float4 sv[CU], acc[CU];
#pragma unroll
    for (int u = 0; u < CU; ++u) {
      sv[u] = ld_row4(sb + (long long)u * g.D, dv && u < g.U);
      acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float* qb = a.q + (long long)b * g.R * g.D + d0;
    float* dqb = a.dq + (long long)b * g.R * g.D + d0;
    float4 pf[JF_PF];
#pragma unroll
    for (int p = 0; p < JF_PF; ++p) pf[p] = ld_row4(qb + (long long)p * g.D, dv && p < g.R);
    for (int r0 = 0; r0 < g.R; r0 += JF_PF) {
#pragma unroll
      for (int p = 0; p < JF_PF; ++p) {
        const int r = r0 + p;
        const float4 qv = pf[p];
        const int rn = r + JF_PF;
        pf[p] = ld_row4(qb + (long long)rn * g.D, dv && rn < g.R);
        if (r < g.R) {
          float w[16];
          const float4* srow = reinterpret_cast<const float4*>(sm.Sp + r * JF_SLOT);
#pragma unroll
          for (int k = 0; k < (CU + 3) / 4; ++k) {
            const float4 t4 = srow[k];
            w[4 * k] = t4.x;
            w[4 * k + 1] = t4.y;
            w[4 * k + 2] = t4.z;
            w[4 * k + 3] = t4.w;
          }
          float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int u = 0; u < CU; ++u) {
            fma4(t, w[u], sv[u]);
            fma4(acc[u], w[u], qv);
          }
          if (dv) {
            const float rsum = sm.rs[r];
            float4 o;
            o.x = 2.f * fmaf(qv.x, rsum, -t.x);
            o.y = 2.f * fmaf(qv.y, rsum, -t.y);
            o.z = 2.f * fmaf(qv.z, rsum, -t.z);
            o.w = 2.f * fmaf(qv.w, rsum, -t.w);
            *reinterpret_cast<float4*>(dqb + (long long)r * g.D) = o;
          }
        }
      }
    }
    if (dv) {
      float* dsb = a.ds + (long long)b * g.U * g.D + d0;
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        if (u < g.U) {
          const float cu = sm.cs[u];
          float4 o;
          o.x = 2.f * fmaf(sv[u].x, cu, -acc[u].x);
          o.y = 2.f * fmaf(sv[u].y, cu, -acc[u].y);
          o.z = 2.f * fmaf(sv[u].z, cu, -acc[u].z);
          o.w = 2.f * fmaf(sv[u].w, cu, -acc[u].w);
          *reinterpret_cast<float4*>(dsb + (long long)u * g.D) = o;
        }
      }
    }
  }
}

template <int CU, bool FVM, bool FEAT>
int jf_launch(const JFArgs& a, bool fwd, cudaStream_t st) {
  size_t off[11];
  const size_t smem = jf_smem_layout(a.g.K, a.g.T, a.g.U, a.W, FVM, fwd, FEAT, off);
  auto kern = fwd ? jf_forward_kernel<CU, FVM, FEAT> : jf_backward_kernel<CU, FVM, FEAT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return set_error(kLaunch, "fused JEANIE: shared memory attribute");
  kern<<<a.B, 32 * a.W, smem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "fused JEANIE launch: %s", cudaGetErrorString(e));
  return kOk;
}

// CU: support frames held in registers (the smallest instance >= U)
template <bool FVM, bool FEAT>
int jf_dispatch(const JFArgs& a, bool fwd, cudaStream_t st) {
  if (!FEAT || a.g.U <= 4) return jf_launch<4, FVM, FEAT>(a, fwd, st);
  if (a.g.U <= 8) return jf_launch<8, FVM, FEAT>(a, fwd, st);
  if (a.g.U <= 12) return jf_launch<12, FVM, FEAT>(a, fwd, st);
  return jf_launch<15, FVM, FEAT>(a, fwd, st);
}

constexpr size_t JF_SMEM_MAX = 96 * 1024;

}  // namespace

// Whether the fused kernels take this shape: float32, features with D <= 256
// a multiple of 4 and at most 15 support frames (or a cost input), and a
// pair's shared-memory state within JF_SMEM_MAX.
bool jf_supported(int K, int T, int U, int D, bool fvm, bool feat) {
  if (K <= 0 || T <= 0 || U <= 0) return false;
  if (feat && (D <= 0 || D > 256 || (D & 3) || U > 15)) return false;
  if ((long long)K * T * U > (1 << 15)) return false;
  const int W = feat ? (D + 127) / 128 : 1;
  size_t off[11];
  const size_t fw = jf_smem_layout(K, T, U, W, fvm, true, feat, off);
  const size_t bw = jf_smem_layout(K, T, U, W, fvm, false, feat, off);
  return fw <= JF_SMEM_MAX && bw <= JF_SMEM_MAX;
}

size_t jf_saved_bytes(int B, int K, int T, int U, bool fvm, bool feat) {
  return jf_saved_layout(B, K, T, U, fvm, feat).total;
}

int jf_run(const float* q, const float* s, const float* cost, int B, int K1, int K2, int T, int U,
           int D, int s1, int s2, int metric, bool fvm, double gamma, bool fwd, float* out,
           float* Rnat, void* saved, size_t saved_bytes, const float* g_out, const float* g_R,
           float* dq, float* ds, float* dC, cudaStream_t st) {
  const bool feat = q != nullptr;
  const int K = K1 * K2;
  if (!jf_supported(K, T, U, D, fvm, feat))
    return set_error(kUnsupported, "fused JEANIE: shape K=%d T=%d U=%d D=%d not supported", K, T,
                     U, D);
  const JFSaved sv = jf_saved_layout(B, K, T, U, fvm, feat);
  if (saved_bytes < sv.total)
    return set_error(kWorkspace, "fused JEANIE: saved needs %zu bytes", sv.total);
  if (feat && ((((uintptr_t)q | (uintptr_t)s) & 15u) ||
               (!fwd && (((uintptr_t)dq | (uintptr_t)ds) & 15u))))
    return set_error(kUnsupported, "fused JEANIE: features must be 16-byte aligned");
  if ((uintptr_t)saved & 15u) return set_error(kInvalid, "fused JEANIE: saved not 16-byte aligned");
  if (B == 0) return kOk;
  JFArgs a{};
  a.q = q;
  a.s = s;
  a.cost = cost;
  a.saved = static_cast<unsigned char*>(saved);
  a.out = out;
  a.Rnat = Rnat;
  a.g_out = g_out;
  a.g_R = g_R;
  a.dq = dq;
  a.ds = ds;
  a.dC = dC;
  a.B = B;
  a.W = feat ? (D + 127) / 128 : 1;
  const double kap = 1.4426950408889634 / gamma;
  a.g = JFGeom{K1, K2, K, T, U, D, s1, s2, metric, K * T, (float)kap, (float)(1.0 / kap)};
  a.sv = sv;
  if (fvm) return feat ? jf_dispatch<true, true>(a, fwd, st) : jf_dispatch<true, false>(a, fwd, st);
  return feat ? jf_dispatch<false, true>(a, fwd, st) : jf_dispatch<false, false>(a, fwd, st);
}

}  // namespace tw
