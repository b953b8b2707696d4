// Tensor-core (tcgen05, 3xTF32, fp32 accumulate in TMEM) forms of the
// pairwise cost and of its feature chain rule, for fp32 features with
// D >= 64 (the contraction is then worth a tensor core; smaller D stays on
// the SIMT kernels of cost_simt.cu).
//
// Cost (hibana2077/torchwarp src/torchwarp/csrc/udtw_cuda.cu:379-387,
// src/torchwarp/udtw/_autograd.py:24-29, jeanie/distances.py:15-27):
//   G = X Y^T on tensor cores, sq = max(|x_i|^2 + |y_j|^2 - 2 G_ij, 0),
//   var = max(0.5 (vx_i + vy_j), eps), C = sq / var, Q = beta log(var).
//
// Each CTA is persistent (one per SM) and walks output tiles of 128 x 128
// cells.  Warp roles:
//   warps 0-3, 10-13  epilogue: TMEM -> registers -> cost -> swizzled smem ->
//              TMA store (two warps per TMEM lane quadrant, each half of the
//              tile's columns)
//   warps 4-7  split:    fp32 tile -> (hi, lo) TF32 pair in place, row norms
//   warp  8    TMA producer of the X / Y feature chunks (32 features each)
//   warp  9    MMA issuer: per 8-feature step an N = 256 MMA A_hi [B_hi; B_lo]
//              and an N = 128 MMA A_lo B_hi (the three 3xTF32 products)
// Two TMEM accumulators (2 x 256 columns) let the epilogue of one tile
// overlap the MMAs of the next.  No atomics: results are reproducible.
#include <cstdlib>
#include <mutex>

#include "tc_common.cuh"

namespace tw {

namespace {

__device__ int g_tc_error;

using namespace tc;

constexpr int BM = 128;            // rows (i) per tile
constexpr int BN = 128;            // columns (j) per tile
constexpr int KC = 32;             // features per chunk: one 128-byte swizzle line
constexpr int STAGES = 2;  // streaming form (D > 128); the X-resident form has its own ring
constexpr int TILE_A = BM * KC * 4;                       // 16 KB
constexpr int TILE_B = BN * KC * 4;                       // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_B;      // hi and lo of A and B
constexpr int STG_BYTES = BM * 32 * 4;                    // one 128 x 32 output chunk
// Warps 0-3 and 10-13 epilogue (warp w reads TMEM lanes 32 (w % 4) ..; warps
// 0-3 take the tile's columns [0, BN/2), warps 10-13 [BN/2, BN)), 4-7 split,
// 8 TMA producer, 9 MMA issuer.
constexpr int COST_THREADS = 448;
// Per tile a 128 x 2BN accumulator: columns [0, BN) take A * B_hi products,
// [BN, 2BN) A * B_lo (B_hi and B_lo are contiguous in shared memory, so one
// N = 256 MMA covers both); two tiles in flight fill all 512 columns.
constexpr uint32_t COST_ACC_COLS = 2 * BN;
constexpr uint32_t COST_TMEM_COLS = 2 * COST_ACC_COLS;

struct CostShared {
  float x2[2][BM];
  float y2[2][BN];
  float vyt[2][BN];  // uDTW: the tile's column variances
  uint64_t full[STAGES], empty[STAGES], conv[STAGES];
  uint64_t accf[2], acce[2], nfull[2], nempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t COST_SMEM = (size_t)STAGES * STAGE_BYTES + 2 * STG_BYTES + sizeof(CostShared);

__device__ __forceinline__ void record_timeout(volatile int* abort) {
  *abort = 1;
  atomicExch(&g_tc_error, kTimeout);
}

struct TileCoord {
  int b, ib, jb;
};

__device__ __forceinline__ TileCoord tile_of(int t, int nI, int nJ) {
  const int per = nI * nJ;
  TileCoord c;
  c.b = t / per;
  const int r = t - c.b * per;
  c.ib = r / nJ;
  c.jb = r - c.ib * nJ;
  return c;
}

// Splits one 128-byte line (32 fp32) of a swizzled box in place into its
// TF32 hi part, writing the lo part at the same offset of `lo_base`.
// Returns the sum of squares of the original values.
__device__ __forceinline__ float split_line(uint8_t* hi_base, uint8_t* lo_base, int line) {
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t off = sw128_chunk(line, q);
    float4 v = *reinterpret_cast<float4*>(hi_base + off);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hi_base + off) = h;
    *reinterpret_cast<float4*>(lo_base + off) = l;
  }
  return ss;
}

// Epilogue of one half (h) of a 128 x BN cost tile (accumulator a): TMEM ->
// registers -> cost (and penalty, positivity mask) -> swizzled staging -> TMA
// store.  Called by the four epilogue warps of half h, each half with its
// own staging buffer and named barrier; `si` counts staging-buffer uses.
template <bool VAR>
__device__ __forceinline__ void cost_epilogue_tile(
    const TileCoord& c, int a, uint32_t tmem, int warp, int row, int h, const float* x2s,
    const float* y2s, const float* vys, uint64_t* acce, uint64_t* nempty, uint8_t* stg_base,
    const CUtensorMap* mapC, const CUtensorMap* mapQ, const float* __restrict__ vx,
    const float* __restrict__ vy, int N, int M, float beta, float eps, int write_q,
    uint32_t* __restrict__ mask, int& si) {
  tc_fence_after();
  const int i = c.ib * BM + row;
  const float x2 = x2s[row];
  float vxi = 0.f;
  if (VAR) vxi = i < N ? vx[(long long)c.b * N + i] : 1.f;
  const float beta_ln2 = beta * 0.693147180559945309f;
  constexpr int CPH = BN / 64;  // 32-column chunks per half
#pragma unroll 1
  for (int cc = CPH * h; cc < CPH * (h + 1); ++cc) {
    float v[32], w[32];
    const uint32_t tcol =
        tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(a * COST_ACC_COLS + 32 * cc);
    tmem_ld32(tcol, v);
    tmem_ld32(tcol + BN, w);
    if (cc == CPH * (h + 1) - 1) {
      tc_fence_before();
      mbar_arrive(acce);
    }
#pragma unroll
    for (int q = 0; q < 32; ++q) v[q] += w[q];  // (hi.hi + lo.hi) + hi.lo
    const int j0 = c.jb * BN + 32 * cc;
    float qv[32];
    uint32_t pos = 0;  // bit q: sq_raw > 0 at column j0 + q
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      float sq = (x2 + y2s[32 * cc + q]) - 2.f * v[q];
      pos |= (sq > 0.f ? 1u : 0u) << q;
      sq = sq > 0.f ? sq : 0.f;
      if (VAR) {
        // var = max((vx_i + vy_j) / 2, eps); cost = sq / var through the
        // hardware reciprocal (relative error ~2^-22, like the division's
        // fp32 rounding); penalty = beta ln(var) from log2
        float var = 0.5f * (vxi + vys[32 * cc + q]);
        var = var > eps ? var : eps;
        v[q] = sq * rcp(var);
        qv[q] = beta_ln2 * lg2(var);
      } else {
        v[q] = sq;
      }
    }
    if (cc == CPH * (h + 1) - 1) mbar_arrive(nempty);
    if (mask != nullptr && j0 < M) {
      // words [b][j >> 5][i] with the row count padded to NP = 4 ceil(N/4)
      const int NP = (N + 3) & ~3;
      if (i < NP) {
        const int left = M - j0;
        const uint32_t valid = left >= 32 ? 0xFFFFFFFFu : ((1u << left) - 1u);
        const int MW = (M + 31) >> 5;
        mask[((long long)c.b * MW + (j0 >> 5)) * NP + i] = i < N ? (pos & valid) : 0u;
      }
    }
    // C chunk (and Q chunk) through the two staging buffers
#pragma unroll
    for (int which = 0; which < (VAR ? 2 : 1); ++which) {
      if (which == 1 && !write_q) break;
      uint8_t* buf = stg_base + (size_t)h * STG_BYTES;
      if (row == 0) bulk_wait_read<0>();  // this half's previous store has read the buffer
      named_bar(1 + h, 128);
      const float* src = which == 0 ? v : qv;
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4)
        *reinterpret_cast<float4*>(buf + sw128_chunk(row, q4)) =
            make_float4(src[4 * q4], src[4 * q4 + 1], src[4 * q4 + 2], src[4 * q4 + 3]);
      fence_async_smem();
      named_bar(1 + h, 128);
      if (row == 0) {
        tma_store_3d(which == 0 ? mapC : mapQ, buf, j0, c.ib * BM, c.b);
        bulk_commit();
      }
      ++si;
    }
  }
}

template <bool VAR>
__global__ void __launch_bounds__(COST_THREADS, 1)
    tc_cost_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapY,
                   const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapQ,
                   const float* __restrict__ vx, const float* __restrict__ vy, int B, int N, int M,
                   int D, float beta, float eps, int write_q, uint32_t* __restrict__ mask) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stage_base = smem;
  uint8_t* stg_base = smem + (size_t)STAGES * STAGE_BYTES;
  CostShared& sh = *reinterpret_cast<CostShared*>(stg_base + 2 * STG_BYTES);
  volatile int* abort = &sh.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nI = (N + BM - 1) / BM, nJ = (M + BN - 1) / BN, nK = (D + KC - 1) / KC;
  const int total = B * nI * nJ;

  if (tid == 0) {
    if ((smem_u32(smem) & 1023u) != 0) {
      atomicExch(&g_tc_error, kLaunch);
      sh.abort = 1;
    } else {
      sh.abort = 0;
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
      mbar_init(&sh.conv[s], 128);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.accf[a], 1);
      mbar_init(&sh.acce[a], 256);
      mbar_init(&sh.nfull[a], 128);
      mbar_init(&sh.nempty[a], 256);
    }
    mbar_init(&sh.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    prefetch_map(&mapX);
    prefetch_map(&mapY);
    prefetch_map(&mapC);
    if (VAR) prefetch_map(&mapQ);
  }
  if (warp == 9) tmem_alloc(&sh.tmem_base, COST_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const bool dead = sh.abort != 0;

  if (!dead && warp == 8 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileCoord c = tile_of(t, nI, nJ);
      for (int kc = 0; kc < nK; ++kc, ++it) {
        const int s = it % STAGES;
        const unsigned ph = (unsigned)(it / STAGES) & 1u;
        if (!mbar_wait(&sh.empty[s], ph ^ 1u, abort)) { record_timeout(abort); goto producer_drain; }
        uint8_t* st = stage_base + (size_t)s * STAGE_BYTES;
        mbar_arrive_expect_tx(&sh.full[s], TILE_A + TILE_B);
        tma_load_3d(st, &mapX, &sh.full[s], kc * KC, c.ib * BM, c.b);
        tma_load_3d(st + 2 * TILE_A, &mapY, &sh.full[s], kc * KC, c.jb * BN, c.b);
      }
    }
  producer_drain:
    // every load issued lands before the CTA exits
    for (int k = (it > STAGES ? it - STAGES : 0); k < it; ++k) {
      const int s = k % STAGES;
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.full[s], (unsigned)(k / STAGES) & 1u)) break;
    }
  } else if (!dead && warp >= 4 && warp < 8) {
    // ------------------------------------------------ TF32 split + norms
    const int ct = tid - 128;
    int it = 0, ti = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
      float sa = 0.f, sb = 0.f;
      for (int kc = 0; kc < nK; ++kc, ++it) {
        const int s = it % STAGES;
        const unsigned ph = (unsigned)(it / STAGES) & 1u;
        if (!mbar_wait(&sh.full[s], ph, abort)) { record_timeout(abort); goto split_done; }
        uint8_t* st = stage_base + (size_t)s * STAGE_BYTES;
        sa += split_line(st, st + TILE_A, ct);
        sb += split_line(st + 2 * TILE_A, st + 2 * TILE_A + TILE_B, ct);
        fence_async_smem();
        mbar_arrive(&sh.conv[s]);
      }
      const int a = ti & 1;
      if (!mbar_wait(&sh.nempty[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
        record_timeout(abort);
        goto split_done;
      }
      sh.x2[a][ct] = sa;
      sh.y2[a][ct] = sb;
      if (VAR) {
        const TileCoord c = tile_of(t, nI, nJ);
        const int j = c.jb * BN + ct;
        sh.vyt[a][ct] = j < M ? vy[(long long)c.b * M + j] : 1.f;
      }
      mbar_arrive(&sh.nfull[a]);
    }
  split_done:;
  } else if (!dead && warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_tf32(BM, 2 * BN, 0, 0);
      // X_lo x Y_hi over the first BN columns only (X_lo x Y_lo is below fp32
      // resolution)
      constexpr uint32_t IDESC_LO = idesc_tf32(BM, BN, 0, 0);
      int it = 0, ti = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
        const int a = ti & 1;
        if (!mbar_wait(&sh.acce[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
          record_timeout(abort);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(a * COST_ACC_COLS);
        bool ok = true;
        for (int kc = 0; kc < nK; ++kc, ++it) {
          const int s = it % STAGES;
          const unsigned ph = (unsigned)(it / STAGES) & 1u;
          if (!mbar_wait(&sh.conv[s], ph, abort)) { record_timeout(abort); ok = false; break; }
          tc_fence_after();
          const uint32_t ah = smem_u32(stage_base + (size_t)s * STAGE_BYTES);
          const uint32_t al = ah + TILE_A, bh = ah + 2 * TILE_A;
#pragma unroll
          for (int kk = 0; kk < KC / 8; ++kk) {
            // B = [B_hi; B_lo] (256 rows): A_hi B -> hi.hi | hi.lo; A_lo B_hi -> lo.hi
            const uint64_t dah = smem_desc_sw128(ah + kk * 32, 16, 1024);
            const uint64_t dal = smem_desc_sw128(al + kk * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(bh + kk * 32, 16, 1024);
            mma_tf32(d_tmem, dah, db, IDESC, (kc | kk) != 0);
            mma_tf32(d_tmem, dal, db, IDESC_LO, 1);
          }
          mma_commit(&sh.empty[s]);
        }
        if (!ok) break;
        mma_commit(&sh.accf[a]);
      }
      // every MMA issued has finished before TMEM is released
      mma_commit(&sh.mma_done);
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.mma_done, 0)) break;
    }
    __syncwarp();
  } else if (!dead && (warp < 4 || warp >= 10)) {
    // ------------------------------------------------ epilogue
    const int row = 32 * (warp & 3) + lane;  // TMEM lane == tile row
    const int h = warp >= 10 ? 1 : 0;       // column half of the tile
    int ti = 0, si = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
      const TileCoord c = tile_of(t, nI, nJ);
      const int a = ti & 1;
      const unsigned ph = (unsigned)(ti >> 1) & 1u;
      const bool ok = mbar_wait(&sh.accf[a], ph, abort) && mbar_wait(&sh.nfull[a], ph, abort);
      if (!ok) record_timeout(abort);
      if (named_bar_or(3, 256, !ok)) break;  // the eight warps stop together
      cost_epilogue_tile<VAR>(c, a, tmem, warp, row, h, sh.x2[a], sh.y2[a], sh.vyt[a],
                              &sh.acce[a], &sh.nempty[a], stg_base, &mapC, &mapQ, vx, vy, N, M,
                              beta, eps, write_q, mask, si);
    }
    if (row == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, COST_TMEM_COLS);
}

// ----------------------------------------------------------------------
// Cost with the X row block resident: a work unit is one pair's 128 rows
// (b, ib) against all its column tiles.  The X chunks of the unit are loaded
// and split into TF32 (hi, lo) once (XB buffers, so the next unit's X loads
// while this one is in use) and serve every column tile; only Y streams
// through the YS-deep ring.  Same roles, tiles and epilogue as
// tc_cost_kernel.
constexpr int XR_MAX_YS = 4;
constexpr int XR_CHUNK = 2 * TILE_A;   // hi + lo of one 128 x 32 chunk (32 KB)

struct CostXRShared {
  float x2[2][BM];
  float y2[2][BN];
  float vyt[2][BN];  // uDTW: the tile's column variances
  uint64_t full[XR_MAX_YS], empty[XR_MAX_YS], conv[XR_MAX_YS];
  uint64_t xfull[2], xempty[2], xconv[2];
  uint64_t accf[2], acce[2], nfull[2], nempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

struct CostXRGeom {
  int nK;   // 32-feature chunks
  int XB;   // X buffers (1 or 2)
  int YS;   // Y stages
};

template <bool VAR>
__global__ void __launch_bounds__(COST_THREADS, 1)
    tc_cost_xr_kernel(const __grid_constant__ CUtensorMap mapX,
                      const __grid_constant__ CUtensorMap mapY,
                      const __grid_constant__ CUtensorMap mapC,
                      const __grid_constant__ CUtensorMap mapQ, const float* __restrict__ vx,
                      const float* __restrict__ vy, int B, int N, int M, int D, float beta,
                      float eps, int write_q, uint32_t* __restrict__ mask, CostXRGeom g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nK = g.nK, XB = g.XB, YS = g.YS;
  uint8_t* x_base = smem;                                        // XB x nK chunks
  uint8_t* y_base = smem + (size_t)XB * nK * XR_CHUNK;            // YS chunks
  uint8_t* stg_base = y_base + (size_t)YS * XR_CHUNK;
  CostXRShared& sh = *reinterpret_cast<CostXRShared*>(stg_base + 2 * STG_BYTES);
  volatile int* abort = &sh.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nI = (N + BM - 1) / BM, nJ = (M + BN - 1) / BN;
  const int units = B * nI;

  if (tid == 0) {
    if ((smem_u32(smem) & 1023u) != 0) {
      atomicExch(&g_tc_error, kLaunch);
      sh.abort = 1;
    } else {
      sh.abort = 0;
    }
    for (int s = 0; s < YS; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
      mbar_init(&sh.conv[s], 128);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.xfull[a], 1);
      mbar_init(&sh.xempty[a], 1);
      mbar_init(&sh.xconv[a], 128);
      mbar_init(&sh.accf[a], 1);
      mbar_init(&sh.acce[a], 256);
      mbar_init(&sh.nfull[a], 128);
      mbar_init(&sh.nempty[a], 256);
    }
    mbar_init(&sh.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    prefetch_map(&mapX);
    prefetch_map(&mapY);
    prefetch_map(&mapC);
    if (VAR) prefetch_map(&mapQ);
  }
  if (warp == 9) tmem_alloc(&sh.tmem_base, COST_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const bool dead = sh.abort != 0;

  if (!dead && warp == 8 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int it = 0, ui = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++ui) {
      const int b = u / nI, ib = u - b * nI;
      const int xb = ui % XB;
      if (!mbar_wait(&sh.xempty[xb], ((unsigned)(ui / XB) & 1u) ^ 1u, abort)) {
        record_timeout(abort);
        goto producer_drain;
      }
      mbar_arrive_expect_tx(&sh.xfull[xb], nK * TILE_A);
      for (int kc = 0; kc < nK; ++kc)
        tma_load_3d(x_base + (size_t)(xb * nK + kc) * XR_CHUNK, &mapX, &sh.xfull[xb], kc * KC,
                    ib * BM, b);
      for (int jb = 0; jb < nJ; ++jb) {
        for (int kc = 0; kc < nK; ++kc, ++it) {
          const int s = it % YS;
          if (!mbar_wait(&sh.empty[s], ((unsigned)(it / YS) & 1u) ^ 1u, abort)) {
            record_timeout(abort);
            goto producer_drain;
          }
          mbar_arrive_expect_tx(&sh.full[s], TILE_B);
          tma_load_3d(y_base + (size_t)s * XR_CHUNK, &mapY, &sh.full[s], kc * KC, jb * BN, b);
        }
      }
    }
  producer_drain:
    // every load issued lands before the CTA exits
    for (int k = (it > YS ? it - YS : 0); k < it; ++k) {
      const int s = k % YS;
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.full[s], (unsigned)(k / YS) & 1u)) break;
    }
    for (int k = (ui > XB ? ui - XB : 0); k < ui; ++k) {
      const int xb = k % XB;
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.xfull[xb], (unsigned)(k / XB) & 1u)) break;
    }
  } else if (!dead && warp >= 4 && warp < 8) {
    // ------------------------------------------------ TF32 split + norms
    const int ct = tid - 128;
    int it = 0, ti = 0, ui = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++ui) {
      const int xb = ui % XB;
      if (!mbar_wait(&sh.xfull[xb], (unsigned)(ui / XB) & 1u, abort)) {
        record_timeout(abort);
        goto split_done;
      }
      float sa = 0.f;
      for (int kc = 0; kc < nK; ++kc) {
        uint8_t* xc = x_base + (size_t)(xb * nK + kc) * XR_CHUNK;
        sa += split_line(xc, xc + TILE_A, ct);
      }
      fence_async_smem();
      mbar_arrive(&sh.xconv[xb]);
      for (int jb = 0; jb < nJ; ++jb, ++ti) {
        float sb = 0.f;
        for (int kc = 0; kc < nK; ++kc, ++it) {
          const int s = it % YS;
          if (!mbar_wait(&sh.full[s], (unsigned)(it / YS) & 1u, abort)) {
            record_timeout(abort);
            goto split_done;
          }
          uint8_t* yc = y_base + (size_t)s * XR_CHUNK;
          sb += split_line(yc, yc + TILE_B, ct);
          fence_async_smem();
          mbar_arrive(&sh.conv[s]);
        }
        const int a = ti & 1;
        if (!mbar_wait(&sh.nempty[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
          record_timeout(abort);
          goto split_done;
        }
        sh.x2[a][ct] = sa;
        sh.y2[a][ct] = sb;
        if (VAR) {
          const int j = jb * BN + ct;
          sh.vyt[a][ct] = j < M ? vy[(long long)(u / nI) * M + j] : 1.f;
        }
        mbar_arrive(&sh.nfull[a]);
      }
    }
  split_done:;
  } else if (!dead && warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_tf32(BM, 2 * BN, 0, 0);
      // X_lo x Y_hi over the first BN columns only (X_lo x Y_lo is below fp32
      // resolution)
      constexpr uint32_t IDESC_LO = idesc_tf32(BM, BN, 0, 0);
      int it = 0, ti = 0, ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ui) {
        const int xb = ui % XB;
        if (!mbar_wait(&sh.xconv[xb], (unsigned)(ui / XB) & 1u, abort)) {
          record_timeout(abort);
          break;
        }
        tc_fence_after();
        for (int jb = 0; jb < nJ && ok; ++jb, ++ti) {
          const int a = ti & 1;
          if (!mbar_wait(&sh.acce[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
            record_timeout(abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(a * COST_ACC_COLS);
          for (int kc = 0; kc < nK; ++kc, ++it) {
            const int s = it % YS;
            if (!mbar_wait(&sh.conv[s], (unsigned)(it / YS) & 1u, abort)) {
              record_timeout(abort);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ah = smem_u32(x_base + (size_t)(xb * nK + kc) * XR_CHUNK);
            const uint32_t al = ah + TILE_A;
            const uint32_t bh = smem_u32(y_base + (size_t)s * XR_CHUNK);
#pragma unroll
            for (int kk = 0; kk < KC / 8; ++kk) {
              // B = [B_hi; B_lo] (256 rows): A_hi B -> hi.hi | hi.lo; A_lo B_hi -> lo.hi
              const uint64_t dah = smem_desc_sw128(ah + kk * 32, 16, 1024);
              const uint64_t dal = smem_desc_sw128(al + kk * 32, 16, 1024);
              const uint64_t db = smem_desc_sw128(bh + kk * 32, 16, 1024);
              mma_tf32(d_tmem, dah, db, IDESC, (kc | kk) != 0);
              mma_tf32(d_tmem, dal, db, IDESC_LO, 1);
            }
            mma_commit(&sh.empty[s]);
          }
          if (!ok) break;
          mma_commit(&sh.accf[a]);
        }
        if (!ok) break;
        mma_commit(&sh.xempty[xb]);   // this unit's X chunks are free once its MMAs finish
      }
      // every MMA issued has finished before TMEM is released
      mma_commit(&sh.mma_done);
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.mma_done, 0)) break;
    }
    __syncwarp();
  } else if (!dead && (warp < 4 || warp >= 10)) {
    // ------------------------------------------------ epilogue
    const int row = 32 * (warp & 3) + lane;  // TMEM lane == tile row
    const int h = warp >= 10 ? 1 : 0;       // column half of the tile
    int ti = 0, si = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int b = u / nI, ib = u - b * nI;
      for (int jb = 0; jb < nJ; ++jb, ++ti) {
        TileCoord c;
        c.b = b;
        c.ib = ib;
        c.jb = jb;
        const int a = ti & 1;
        const unsigned ph = (unsigned)(ti >> 1) & 1u;
        const bool good = mbar_wait(&sh.accf[a], ph, abort) && mbar_wait(&sh.nfull[a], ph, abort);
        if (!good) record_timeout(abort);
        if (named_bar_or(3, 256, !good)) {  // the eight warps stop together
          ok = false;
          break;
        }
        cost_epilogue_tile<VAR>(c, a, tmem, warp, row, h, sh.x2[a], sh.y2[a], sh.vyt[a],
                                &sh.acce[a], &sh.nempty[a], stg_base, &mapC, &mapQ, vx, vy, N,
                                M, beta, eps, write_q, mask, si);
      }
    }
    if (row == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, COST_TMEM_COLS);
}

// ----------------------------------------------------------------------
// Chain rule of the cost on tensor cores (udtw_cuda.cu:557-568,
// udtw/_ops.py:179-183):
//   S = dsq = dC / var where sq_raw > 0 (C > 0, or the cost's positivity
//       mask), else 0
//   dX = -2 S Y + 2 X rowsum(S)        (SIDE 0: unit = 128 rows i of a pair,
//                                        K = j in chunks of 32)
//   dY = -2 S^T X + 2 Y colsum(S)      (SIDE 1: unit = 128 rows j of a pair,
//                                        K = i in chunks of 32)
//   dvx = 0.5 rowsum(dvar), dvy = 0.5 colsum(dvar),
//   dvar = (beta dQ - dC C) / var where var_raw > eps.
// Two rings of shared memory: a deep landing ring that TMA fills with raw
// chunks (dC [, C] [, dQ], the other side's 32 feature rows, the mask words;
// with PRE only dC and the features) so that enough bytes are in flight to
// cover HBM latency, and a ring of converted operands: the split warps read a
// landing chunk, write S (to TMEM, or to shared memory for wide D) and the
// features as TF32 (hi, lo) pairs into a converted slot (same swizzled
// positions) and release the landing slot at once.  The MMA
// contracts S (K-major for SIDE 0, MN-major for SIDE 1) with the features
// (MN-major) into a 128 x BD TMEM accumulator; the epilogue adds 2 A rowsum
// and stores through TMA.  MN-major TF32 operands are only valid in the
// 32-byte-granule swizzle (a standard 128-byte-swizzle MN-major descriptor
// yields no product), so those boxes are loaded with that swizzle.

// Warp roles: 0-3 epilogue (TMEM lanes 32 w ..), 4-11 split, 12 TMA, 13 MMA.
constexpr int GRAD_CONV = 256;            // split threads
constexpr int GRAD_PROD_WARP = 4 + GRAD_CONV / 32;
constexpr int GRAD_MMA_WARP = GRAD_PROD_WARP + 1;
constexpr int GRAD_THREADS = 32 * (GRAD_MMA_WARP + 1);
constexpr int GRAD_MAX_LAND = 6;
constexpr int GRAD_MAX_CONV = 4;
constexpr int SBOX = 128 * 32 * 4;  // one 16 KB chunk of dC / C / dQ

struct GradShared {
  float rs[2][128];
  float red[8][128];  // partial row / column sums of the split threads
  float redv[8][128];
  uint64_t lfull[GRAD_MAX_LAND], lempty[GRAD_MAX_LAND];
  uint64_t cfull[GRAD_MAX_CONV], cempty[GRAD_MAX_CONV];
  uint64_t accf[2], acce[2], nfull[2], nempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int linfo[GRAD_MAX_LAND];  // chunk of each landing slot (index | kLastChunk)
  int cinfo[GRAD_MAX_CONV];  // the same for each converted slot
};

// Chunk schedule of a chain-rule unit.  Without flags every 32-wide chunk of
// the summed extent is processed.  With flags (one byte per chunk of the
// unit, nonzero where the DP backward wrote a nonzero value of S into it)
// only the flagged chunks and chunk 0 are: a chunk of S that is all zero adds
// exactly zero to the products and to the row sums, and chunk 0 always runs
// so that every unit writes its accumulator.  The producer walks the
// schedule and files each landing slot's chunk in linfo; the consumers read
// it from there, so all roles agree.
constexpr int kLastChunk = 1 << 30;

__device__ __forceinline__ uint32_t nz_bytes(uint32_t w) {
  return (uint32_t)((w & 0xffu) != 0u) | ((uint32_t)((w & 0xff00u) != 0u) << 1) |
         ((uint32_t)((w & 0xff0000u) != 0u) << 2) | ((uint32_t)((w >> 24) != 0u) << 3);
}

struct ChunkSched {
  const uint8_t* fr;  // the unit's flag row (16-byte aligned, padded to 16), or null
  int nK;
  int w0;             // first chunk of the 64-chunk window in m
  uint64_t m;
  // first chunk >= c to process, or nK
  __device__ __forceinline__ int next(int c) {
    if (fr == nullptr) return c;
    while (c < nK) {
      if (c - w0 >= 64) {
        w0 = c & ~63;
        m = 0;
#pragma unroll
        for (int v = 0; v < 4; ++v)
          if (w0 + 16 * v < nK) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(fr + w0 + 16 * v));
            const uint32_t b16 = nz_bytes(q.x) | (nz_bytes(q.y) << 4) | (nz_bytes(q.z) << 8) |
                                 (nz_bytes(q.w) << 12);
            m |= (uint64_t)b16 << (16 * v);
          }
      }
      const uint64_t rest = m >> (c - w0);
      if (rest != 0) return c + __ffsll((long long)rest) - 1;
      c = w0 + 64;
    }
    return nK;
  }
};

struct GradGeom {
  int nF;           // 32-feature boxes (BD = 32 nF)
  int mw;           // positivity-mask words per row: ceil(M / 32)
  int np;           // mask row count, padded: 4 ceil(N / 4)
  int lstages, cstages;
  int l_c, l_dq, l_f, l_mask, l_bytes;  // landing slot layout (dC at 0)
  int c_bytes;      // converted slot (shared memory)
  int c_fh, c_fl;   // features hi / lo in a converted slot (S hi / lo at 0 / SBOX unless in TMEM)
  int tx_fixed;     // landing bytes per chunk other than the mask
  uint32_t tmem_cols;
  uint32_t a_col0;  // S in TMEM: first column of the (hi 32 | lo 32) x cstages ring
};

__device__ __forceinline__ float4 split4(float4 v, float4& lo) {
  float4 hi;
  split_tf32(v.x, hi.x, lo.x);
  split_tf32(v.y, hi.y, lo.y);
  split_tf32(v.z, hi.z, lo.z);
  split_tf32(v.w, hi.w, lo.w);
  return hi;
}

// S of a cell whose cost c the chain rule reads (no variance, no mask): the
// clamp's derivative passes dC where c > 0; with sqrt_cost, c is a Euclidean
// cost sqrt(sq) and dsq = dC / (2 c) (zero gradient at c = 0, as
// jeanie/distances.py:34-38).
__device__ __forceinline__ float s_of_cost(float g, float c, int sqrt_cost) {
  return c > 0.f ? (sqrt_cost ? g * (0.5f * rcp(c)) : g) : 0.f;
}

// PRE: dC already carries the positivity mask (S = dC), so neither the cost
// nor mask words are loaded and the split warps skip the mask test.
template <int SIDE, bool VAR, bool MASKED, bool TA, bool WIDE, bool PRE = false>
__global__ void __launch_bounds__(GRAD_THREADS, 1)
    tc_grad_kernel(const __grid_constant__ CUtensorMap mapDC, const __grid_constant__ CUtensorMap mapC,
                   const __grid_constant__ CUtensorMap mapDQ, const __grid_constant__ CUtensorMap mapF,
                   const __grid_constant__ CUtensorMap mapOut, const float* __restrict__ A,
                   const float* __restrict__ va, const float* __restrict__ vb,
                   float* __restrict__ dva, int B, int N, int M, int D, float beta, float eps,
                   int has_dq, GradGeom g, const uint32_t* __restrict__ mask, int sqrt_cost,
                   const uint8_t* __restrict__ tflags, int tf_k) {
  static_assert(!(PRE && (VAR || MASKED)), "PRE is the plain soft-DTW chain rule");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* land_base = smem;
  uint8_t* conv_base = smem + (size_t)g.lstages * g.l_bytes;
  uint8_t* stg_base = conv_base + (size_t)g.cstages * g.c_bytes;  // one staging buffer
  GradShared& sh = *reinterpret_cast<GradShared*>(stg_base + STG_BYTES);
  volatile int* abort = &sh.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int R = SIDE == 0 ? N : M;   // rows of the gradient (own side)
  const int S = SIDE == 0 ? M : N;   // summed extent
  const int nBlk = (R + 127) / 128, nK = (S + 31) / 32;
  const int total = B * nBlk;
  const int BD = 32 * g.nF;
  const int LS = g.lstages, CS = g.cstages;

  if (tid == 0) {
    if ((smem_u32(smem) & 1023u) != 0) {
      atomicExch(&g_tc_error, kLaunch);
      sh.abort = 1;
    } else {
      sh.abort = 0;
    }
    for (int s = 0; s < LS; ++s) {
      mbar_init(&sh.lfull[s], 1);
      mbar_init(&sh.lempty[s], GRAD_CONV);
    }
    for (int s = 0; s < CS; ++s) {
      mbar_init(&sh.cfull[s], GRAD_CONV);
      mbar_init(&sh.cempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.accf[a], 1);
      mbar_init(&sh.acce[a], 128);
      mbar_init(&sh.nfull[a], 128);
      mbar_init(&sh.nempty[a], 128);
    }
    mbar_init(&sh.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == GRAD_PROD_WARP && lane == 0) {
    prefetch_map(&mapDC);
    if (!MASKED) prefetch_map(&mapC);
    if (VAR && has_dq) prefetch_map(&mapDQ);
    prefetch_map(&mapF);
    prefetch_map(&mapOut);
  }
  if (warp == GRAD_MMA_WARP) tmem_alloc(&sh.tmem_base, g.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const bool dead = sh.abort != 0;

  if (!dead && warp == GRAD_PROD_WARP && lane == 0) {
    // ------------------------------------------------ TMA producer
    int it = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int b = u / nBlk, blk = u - b * nBlk;
      ChunkSched sched{tflags != nullptr ? tflags + ((long long)b * nBlk + blk) * tf_k : nullptr,
                       nK, -64, 0ull};
      for (int kc = 0; kc < nK; ++it) {
        const int nx = sched.next(kc + 1);
        const int s = it % LS;
        const unsigned ph = (unsigned)(it / LS) & 1u;
        if (!mbar_wait(&sh.lempty[s], ph ^ 1u, abort)) { record_timeout(abort); goto producer_drain; }
        sh.linfo[s] = kc | (nx >= nK ? kLastChunk : 0);
        uint8_t* st = land_base + (size_t)s * g.l_bytes;
        unsigned tx = g.tx_fixed;
        const uint32_t* msrc[4] = {nullptr, nullptr, nullptr, nullptr};
        unsigned mbytes[4] = {0, 0, 0, 0};
        if (MASKED) {
          // SIDE 0: word row kc, rows blk*128 ..; SIDE 1: word rows blk*4 + q, rows kc*32 ..
          if (SIDE == 0) {
            const int r0 = blk * 128, n = min(128, g.np - r0);
            msrc[0] = mask + ((long long)b * g.mw + kc) * g.np + r0;
            mbytes[0] = (unsigned)n * 4u;
          } else {
            const int r0 = kc * 32, n = min(32, g.np - r0);
            for (int q = 0; q < 4; ++q) {
              const int jw = blk * 4 + q;
              if (jw < g.mw) {
                msrc[q] = mask + ((long long)b * g.mw + jw) * g.np + r0;
                mbytes[q] = (unsigned)n * 4u;
              }
            }
          }
          tx += mbytes[0] + mbytes[1] + mbytes[2] + mbytes[3];
        }
        mbar_arrive_expect_tx(&sh.lfull[s], tx);
        if (MASKED) {
          for (int q = 0; q < 4; ++q)
            if (mbytes[q]) bulk_load(st + g.l_mask + q * 128, msrc[q], mbytes[q], &sh.lfull[s]);
        }
        if (SIDE == 0) {
          // S chunk: 128 rows i x 32 columns j
          tma_load_3d(st, &mapDC, &sh.lfull[s], kc * 32, blk * 128, b);
          if (!MASKED && !PRE) tma_load_3d(st + g.l_c, &mapC, &sh.lfull[s], kc * 32, blk * 128, b);
          if (VAR && has_dq) tma_load_3d(st + g.l_dq, &mapDQ, &sh.lfull[s], kc * 32, blk * 128, b);
        } else {
          // S chunk: 32 rows i x 128 columns j, as four 32 x 32 boxes
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int x = blk * 128 + 32 * q;
            tma_load_3d(st + q * 4096, &mapDC, &sh.lfull[s], x, kc * 32, b);
            if (!MASKED && !PRE)
              tma_load_3d(st + g.l_c + q * 4096, &mapC, &sh.lfull[s], x, kc * 32, b);
            if (VAR && has_dq)
              tma_load_3d(st + g.l_dq + q * 4096, &mapDQ, &sh.lfull[s], x, kc * 32, b);
          }
        }
        // the other side's features: 32 summed rows x BD features
        for (int f = 0; f < g.nF; ++f)
          tma_load_3d(st + g.l_f + f * 4096, &mapF, &sh.lfull[s], 32 * f, kc * 32, b);
        kc = nx;
      }
    }
  producer_drain:
    // every load issued lands before the CTA exits
    for (int k = (it > LS ? it - LS : 0); k < it; ++k) {
      const int s = k % LS;
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.lfull[s], (unsigned)(k / LS) & 1u)) break;
    }
  } else if (TA && !dead && warp >= 4 && warp < GRAD_PROD_WARP) {
    // ------------------------------------------- S = dsq, split into TMEM, sums
    // S goes to TMEM as the MMA's A operand (lane = own row, column = summed
    // index), so neither its hi / lo halves nor the MMA's A reads touch
    // shared memory.  Warp w writes TMEM lanes 32 (w % 4) ..; thread ct owns
    // own-row ct & 127 and the 16 summed columns 16 hh .. of each chunk.
    const int ct = tid - 128;
    const int own = ct & 127, hh = ct >> 7;
    const int sub = warp & 3;
    const uint32_t lane_base = (uint32_t)(32 * sub) << 16;
    int it = 0, ti = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++ti) {
      const int b = u / nBlk, blk = u - b * nBlk;
      const int r = blk * 128 + own;
      const float va_r = VAR ? (r < R ? va[(long long)b * R + r] : 1.f) : 0.f;
      const float* vb_b = VAR ? vb + (long long)b * S : nullptr;
      float rsum = 0.f, vsum = 0.f;
      for (bool more = true; more && ok; ++it) {
        const int s = it % LS, cs = it % CS;
        if (!mbar_wait(&sh.lfull[s], (unsigned)(it / LS) & 1u, abort) ||
            !mbar_wait(&sh.cempty[cs], ((unsigned)(it / CS) & 1u) ^ 1u, abort)) {
          record_timeout(abort);
          ok = false;
          break;
        }
        const int info = sh.linfo[s];
        const int kc = info & (kLastChunk - 1);
        more = (info & kLastChunk) == 0;
        if (ct == 0) sh.cinfo[cs] = info;
        tc_fence_after();  // the MMAs that read this TMEM slot have completed
        const uint8_t* ld = land_base + (size_t)s * g.l_bytes;
        uint8_t* cv = conv_base + (size_t)cs * g.c_bytes;
        // uDTW: lane l holds the other side's variance at summed index kc*32 + l
        float vbl = 1.f;
        if (VAR) {
          const int idx = kc * 32 + lane;
          vbl = idx < S ? __ldg(vb_b + idx) : 1.f;
        }
        // the other side's features of this chunk (at most 3 float4 per
        // thread: TA runs for D <= 96), read first so that their latency
        // overlaps the split of S
        float4 fv[3];
        {
          const float4* fr = reinterpret_cast<const float4*>(ld + g.l_f);
#pragma unroll
          for (int q = 0; q < 3; ++q)
            if (q < g.nF) fv[q] = fr[ct + GRAD_CONV * q];
        }
        float sv[16];
        if (SIDE == 0) {
          const uint32_t mword =
              MASKED ? reinterpret_cast<const uint32_t*>(ld + g.l_mask)[own] : 0u;
          float4 g4[4], c4[4], q4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t off = sw128_chunk(own, 4 * hh + k);
            g4[k] = *reinterpret_cast<const float4*>(ld + off);
            if (!MASKED && !PRE) c4[k] = *reinterpret_cast<const float4*>(ld + g.l_c + off);
            q4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VAR && has_dq) q4[k] = *reinterpret_cast<const float4*>(ld + g.l_dq + off);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float ge[4] = {g4[k].x, g4[k].y, g4[k].z, g4[k].w};
            const float qe[4] = {q4[k].x, q4[k].y, q4[k].z, q4[k].w};
            float ce[4] = {1.f, 1.f, 1.f, 1.f};
            if (!MASKED && !PRE) { ce[0] = c4[k].x; ce[1] = c4[k].y; ce[2] = c4[k].z; ce[3] = c4[k].w; }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int jj = 16 * hh + 4 * k + e;  // summed column within the chunk
              if (MASKED) ce[e] = (mword >> jj) & 1u ? 1.f : 0.f;
              float inv = 1.f, var_raw = 1.f;
              if (VAR) {
                var_raw = 0.5f * (va_r + __shfl_sync(0xffffffffu, vbl, jj));
                inv = rcp(var_raw > eps ? var_raw : eps);
              }
              const float v = PRE ? ge[e]
                            : (VAR ? (ce[e] > 0.f ? ge[e] * inv : 0.f)
                                   : s_of_cost(ge[e], ce[e], sqrt_cost));
              rsum += v;
              if (VAR && var_raw > eps) vsum += (beta * qe[e] - ge[e] * ce[e]) * inv;
              sv[4 * k + e] = v;
            }
          }
        } else {
          // own column j = blk*128 + 32 sub + lane: box `sub`, element `lane`
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int rr = 16 * hh + k;
            const uint32_t off = sub * 4096 + sw128b32_elem(rr, lane);
            const float gv = *reinterpret_cast<const float*>(ld + off);
            float cvv = 1.f;
            if (MASKED) {
              const int jw = blk * 4 + sub;
              const uint32_t w =
                  jw < g.mw ? reinterpret_cast<const uint32_t*>(ld + g.l_mask)[sub * 32 + rr] : 0u;
              cvv = (w >> lane) & 1u ? 1.f : 0.f;
            } else if (!PRE) {
              cvv = *reinterpret_cast<const float*>(ld + g.l_c + off);
            }
            const float qv = (VAR && has_dq) ? *reinterpret_cast<const float*>(ld + g.l_dq + off)
                                             : 0.f;
            float inv = 1.f, var_raw = 1.f;
            if (VAR) {
              var_raw = 0.5f * (__shfl_sync(0xffffffffu, vbl, rr) + va_r);
              inv = rcp(var_raw > eps ? var_raw : eps);
            }
            const float v = PRE ? gv
                            : (VAR ? (cvv > 0.f ? gv * inv : 0.f) : s_of_cost(gv, cvv, sqrt_cost));
            rsum += v;
            if (VAR && var_raw > eps) vsum += (beta * qv - gv * cvv) * inv;
            sv[k] = v;
          }
        }
        {
          float hi[16], lo[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) split_tf32(sv[k], hi[k], lo[k]);
          const uint32_t a_hi = tmem + lane_base + g.a_col0 + (uint32_t)(cs * 64 + 16 * hh);
          tmem_st16(a_hi, hi);
          tmem_st16(a_hi + 32, lo);
        }
        // the other side's features: elementwise split into shared memory
        {
          float4* fh = reinterpret_cast<float4*>(cv + g.c_fh);
          float4* fl = reinterpret_cast<float4*>(cv + g.c_fl);
#pragma unroll
          for (int q = 0; q < 3; ++q)
            if (q < g.nF) {
              float4 lo;
              fh[ct + GRAD_CONV * q] = split4(fv[q], lo);
              fl[ct + GRAD_CONV * q] = lo;
            }
        }
        tmem_st_wait();
        mbar_arrive(&sh.lempty[s]);
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&sh.cfull[cs]);
      }
      if (named_bar_or(2, GRAD_CONV, !ok)) break;
      const int a = ti & 1;
      sh.red[hh][own] = rsum;
      if (VAR) sh.redv[hh][own] = vsum;
      named_bar(2, GRAD_CONV);
      if (ct < 128) {
        const float rfin = sh.red[0][ct] + sh.red[1][ct];
        const float vfin = VAR ? sh.redv[0][ct] + sh.redv[1][ct] : 0.f;
        const int rr = blk * 128 + ct;
        if (VAR && dva != nullptr && rr < R) dva[(long long)b * R + rr] = 0.5f * vfin;
        if (mbar_wait(&sh.nempty[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
          sh.rs[a][ct] = rfin;
          mbar_arrive(&sh.nfull[a]);
        } else {
          record_timeout(abort);
          ok = false;
        }
      }
      named_bar(2, GRAD_CONV);
    }
  } else if (!TA && !dead && warp >= 4 && warp < GRAD_PROD_WARP) {
    // ------------------------------------------------ S = dsq, split, sums
    // SIDE 0: thread ct owns row (ct & 127) of the 128-row chunk, 16-byte
    // pieces 4h .. 4h+3 of its 128-byte line (h = ct >> 7).
    // SIDE 1: thread ct owns the 4 columns 4 cq .. 4 cq + 3 (cq = ct & 31) of
    // the chunk rows 4 rg .. 4 rg + 3 (rg = ct >> 5).
    // Partial sums meet in shared memory at the end of a unit; thread
    // ct < 128 then holds the sums of gradient row ct.
    const int ct = tid - 128;
    const int h = ct >> 7, row = ct & 127;
    const int rg = ct >> 5, cq = ct & 31;
    int it = 0, ti = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++ti) {
      const int b = u / nBlk, blk = u - b * nBlk;
      float va_r[4] = {0.f, 0.f, 0.f, 0.f};
      const float* vb_b = VAR ? vb + (long long)b * S : nullptr;
      if (VAR) {
        if (SIDE == 0) {
          const int r = blk * 128 + row;
          va_r[0] = r < R ? va[(long long)b * R + r] : 1.f;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = blk * 128 + 4 * cq + e;
            va_r[e] = j < R ? va[(long long)b * R + j] : 1.f;
          }
        }
      }
      float rsum[4] = {0.f, 0.f, 0.f, 0.f}, vsum[4] = {0.f, 0.f, 0.f, 0.f};
      for (bool more = true; more && ok; ++it) {
        const int s = it % LS, cs = it % CS;
        if (!mbar_wait(&sh.lfull[s], (unsigned)(it / LS) & 1u, abort) ||
            !mbar_wait(&sh.cempty[cs], ((unsigned)(it / CS) & 1u) ^ 1u, abort)) {
          record_timeout(abort);
          ok = false;
          break;
        }
        const int info = sh.linfo[s];
        const int kc = info & (kLastChunk - 1);
        more = (info & kLastChunk) == 0;
        if (ct == 0) sh.cinfo[cs] = info;
        const uint8_t* ld = land_base + (size_t)s * g.l_bytes;
        uint8_t* cv = conv_base + (size_t)cs * g.c_bytes;
        if (SIDE == 0) {
          const uint32_t mword =
              MASKED ? reinterpret_cast<const uint32_t*>(ld + g.l_mask)[row] : 0u;
          float4 g4[4], c4[4], q4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t off = sw128_chunk(row, 4 * h + k);
            g4[k] = *reinterpret_cast<const float4*>(ld + off);
            if (!MASKED && !PRE) c4[k] = *reinterpret_cast<const float4*>(ld + g.l_c + off);
            q4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VAR && has_dq) q4[k] = *reinterpret_cast<const float4*>(ld + g.l_dq + off);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int q = 4 * h + k;
            const uint32_t off = sw128_chunk(row, q);
            float ce[4] = {1.f, 1.f, 1.f, 1.f};
            if (MASKED) {
#pragma unroll
              for (int e = 0; e < 4; ++e) ce[e] = (mword >> (4 * q + e)) & 1u ? 1.f : 0.f;
            } else if (!PRE) {
              ce[0] = c4[k].x; ce[1] = c4[k].y; ce[2] = c4[k].z; ce[3] = c4[k].w;
            }
            const float ge[4] = {g4[k].x, g4[k].y, g4[k].z, g4[k].w};
            const float qe[4] = {q4[k].x, q4[k].y, q4[k].z, q4[k].w};
            float sv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float var = 1.f, var_raw = 1.f;
              if (VAR) {
                const int j = kc * 32 + 4 * q + e;
                var_raw = 0.5f * (va_r[0] + (j < S ? __ldg(vb_b + j) : 1.f));
                var = var_raw > eps ? var_raw : eps;
              }
              const float rv = VAR ? rcp(var) : 1.f;
              sv[e] = PRE ? ge[e]
                      : (VAR ? (ce[e] > 0.f ? ge[e] * rv : 0.f) : s_of_cost(ge[e], ce[e], sqrt_cost));
              rsum[0] += sv[e];
              if (VAR && var_raw > eps) vsum[0] += (beta * qe[e] - ge[e] * ce[e]) * rv;
            }
            float4 lo;
            const float4 hi = split4(make_float4(sv[0], sv[1], sv[2], sv[3]), lo);
            *reinterpret_cast<float4*>(cv + off) = hi;
            *reinterpret_cast<float4*>(cv + SBOX + off) = lo;
          }
        } else {
          // 4 columns (one 16-byte piece of a 32-byte granule) of 4 rows
          const int box = cq >> 3, gq = (cq & 7) >> 1, half = cq & 1;
          const int jw = blk * 4 + box;
          float4 g4[4], c4[4], q4[4];
          uint32_t mw4[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int rr = rg * 4 + k;
            const uint32_t off =
                box * 4096 + rr * 128 + (uint32_t)(((gq ^ (rr & 3)) << 5) + half * 16);
            g4[k] = *reinterpret_cast<const float4*>(ld + off);
            if (!MASKED && !PRE) c4[k] = *reinterpret_cast<const float4*>(ld + g.l_c + off);
            q4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VAR && has_dq) q4[k] = *reinterpret_cast<const float4*>(ld + g.l_dq + off);
            mw4[k] = (MASKED && jw < g.mw)
                         ? reinterpret_cast<const uint32_t*>(ld + g.l_mask)[box * 32 + rr]
                         : 0u;
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int rr = rg * 4 + k;
            const uint32_t off =
                box * 4096 + rr * 128 + (uint32_t)(((gq ^ (rr & 3)) << 5) + half * 16);
            float ce[4] = {1.f, 1.f, 1.f, 1.f};
            if (MASKED) {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                ce[e] = (mw4[k] >> (4 * (cq & 7) + e)) & 1u ? 1.f : 0.f;
            } else if (!PRE) {
              ce[0] = c4[k].x; ce[1] = c4[k].y; ce[2] = c4[k].z; ce[3] = c4[k].w;
            }
            const float ge[4] = {g4[k].x, g4[k].y, g4[k].z, g4[k].w};
            const float qe[4] = {q4[k].x, q4[k].y, q4[k].z, q4[k].w};
            float vbi = 0.f;
            if (VAR) {
              const int i = kc * 32 + rr;
              vbi = i < S ? __ldg(vb_b + i) : 1.f;
            }
            float sv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float var = 1.f, var_raw = 1.f;
              if (VAR) {
                var_raw = 0.5f * (vbi + va_r[e]);
                var = var_raw > eps ? var_raw : eps;
              }
              const float rv = VAR ? rcp(var) : 1.f;
              sv[e] = PRE ? ge[e]
                      : (VAR ? (ce[e] > 0.f ? ge[e] * rv : 0.f) : s_of_cost(ge[e], ce[e], sqrt_cost));
              rsum[e] += sv[e];
              if (VAR && var_raw > eps) vsum[e] += (beta * qe[e] - ge[e] * ce[e]) * rv;
            }
            float4 lo;
            const float4 hi = split4(make_float4(sv[0], sv[1], sv[2], sv[3]), lo);
            *reinterpret_cast<float4*>(cv + off) = hi;
            *reinterpret_cast<float4*>(cv + SBOX + off) = lo;
          }
        }
        // the other side's features: elementwise split of the whole slab
        {
          const float4* fr = reinterpret_cast<const float4*>(ld + g.l_f);
          float4* fh = reinterpret_cast<float4*>(cv + g.c_fh);
          float4* fl = reinterpret_cast<float4*>(cv + g.c_fl);
          const int n4 = g.nF * 256;
#pragma unroll 2
          for (int k = ct; k < n4; k += GRAD_CONV) {
            float4 lo;
            fh[k] = split4(fr[k], lo);
            fl[k] = lo;
          }
        }
        mbar_arrive(&sh.lempty[s]);   // landing slot read completely
        fence_async_smem();
        mbar_arrive(&sh.cfull[cs]);
      }
      // the eight split warps decide together whether to go on
      if (named_bar_or(2, GRAD_CONV, !ok)) break;
      const int a = ti & 1;
      if (SIDE == 0) {
        sh.red[h][row] = rsum[0];
        if (VAR) sh.redv[h][row] = vsum[0];
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sh.red[rg][4 * cq + e] = rsum[e];
          if (VAR) sh.redv[rg][4 * cq + e] = vsum[e];
        }
      }
      named_bar(2, GRAD_CONV);
      if (ct < 128) {
        float rfin, vfin = 0.f;
        if (SIDE == 0) {
          rfin = sh.red[0][ct] + sh.red[1][ct];
          if (VAR) vfin = sh.redv[0][ct] + sh.redv[1][ct];
        } else {
          rfin = ((sh.red[0][ct] + sh.red[1][ct]) + (sh.red[2][ct] + sh.red[3][ct])) +
                 ((sh.red[4][ct] + sh.red[5][ct]) + (sh.red[6][ct] + sh.red[7][ct]));
          if (VAR)
            vfin = ((sh.redv[0][ct] + sh.redv[1][ct]) + (sh.redv[2][ct] + sh.redv[3][ct])) +
                   ((sh.redv[4][ct] + sh.redv[5][ct]) + (sh.redv[6][ct] + sh.redv[7][ct]));
        }
        const int r = blk * 128 + ct;
        if (VAR && dva != nullptr && r < R) dva[(long long)b * R + r] = 0.5f * vfin;
        if (mbar_wait(&sh.nempty[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
          sh.rs[a][ct] = rfin;
          mbar_arrive(&sh.nfull[a]);
        } else {
          record_timeout(abort);
          ok = false;
        }
      }
      named_bar(2, GRAD_CONV);  // red[] is free for the next unit
    }
  } else if (!dead && warp == GRAD_MMA_WARP) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      // WIDE: B = [F_hi | F_lo] along N (2 BD columns), two MMAs per K step:
      // S_hi x [F_hi | F_lo] over 2 BD columns and S_lo x F_hi over the first
      // BD (the S_lo x F_lo term is below fp32 resolution and is skipped)
      const int ACC = WIDE ? 2 * BD : BD;
      const uint32_t idesc = idesc_tf32(128, ACC, (SIDE == 1 && !TA) ? 1 : 0, 1);
      const uint32_t idesc_lo = idesc_tf32(128, BD, (SIDE == 1 && !TA) ? 1 : 0, 1);
      int it = 0, ti = 0;
      for (int u = blockIdx.x; u < total; u += gridDim.x, ++ti) {
        const int a = ti & 1;
        if (!mbar_wait(&sh.acce[a], ((unsigned)(ti >> 1) & 1u) ^ 1u, abort)) {
          record_timeout(abort);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(a * ACC);
        bool ok = true;
        for (bool more = true; more; ++it) {
          const int cs = it % CS;
          if (!mbar_wait(&sh.cfull[cs], (unsigned)(it / CS) & 1u, abort)) {
            record_timeout(abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const int info = sh.cinfo[cs];
          const int kc = info & (kLastChunk - 1);
          more = (info & kLastChunk) == 0;
          const uint32_t st = smem_u32(conv_base + (size_t)cs * g.c_bytes);
          const uint32_t ah = st, al = st + SBOX, fh = st + g.c_fh, fl = st + g.c_fl;
          if constexpr (TA) {
            const uint32_t ta = tmem + g.a_col0 + (uint32_t)(cs * 64);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t dbh = smem_desc(fh + kk * 1024, 4096, 512, kLayoutSW128Base32);
              if (WIDE) {
                mma_tf32_ts(d_tmem, ta + 8 * kk, dbh, idesc, (kc | kk) != 0);
                mma_tf32_ts(d_tmem, ta + 32 + 8 * kk, dbh, idesc_lo, 1);
              } else {
                const uint64_t dbl = smem_desc(fl + kk * 1024, 4096, 512, kLayoutSW128Base32);
                mma_tf32_ts(d_tmem, ta + 32 + 8 * kk, dbh, idesc, (kc | kk) != 0);
                mma_tf32_ts(d_tmem, ta + 8 * kk, dbl, idesc, 1);
                mma_tf32_ts(d_tmem, ta + 8 * kk, dbh, idesc, 1);
              }
            }
            mma_commit(&sh.cempty[cs]);
          } else {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint64_t dah, dal;
            if (SIDE == 0) {
              dah = smem_desc_sw128(ah + kk * 32, 16, 1024);
              dal = smem_desc_sw128(al + kk * 32, 16, 1024);
            } else {
              dah = smem_desc(ah + kk * 1024, 4096, 512, kLayoutSW128Base32);
              dal = smem_desc(al + kk * 1024, 4096, 512, kLayoutSW128Base32);
            }
            const uint64_t dbh = smem_desc(fh + kk * 1024, 4096, 512, kLayoutSW128Base32);
            if (WIDE) {
              mma_tf32(d_tmem, dah, dbh, idesc, (kc | kk) != 0);
              mma_tf32(d_tmem, dal, dbh, idesc_lo, 1);
            } else {
              const uint64_t dbl = smem_desc(fl + kk * 1024, 4096, 512, kLayoutSW128Base32);
              mma_tf32(d_tmem, dal, dbh, idesc, (kc | kk) != 0);
              mma_tf32(d_tmem, dah, dbl, idesc, 1);
              mma_tf32(d_tmem, dah, dbh, idesc, 1);
            }
          }
          mma_commit(&sh.cempty[cs]);
          }
        }
        if (!ok) break;
        mma_commit(&sh.accf[a]);
      }
      mma_commit(&sh.mma_done);
      for (unsigned n = 0; n < kSpinLimit; ++n)
        if (mbar_try_wait(&sh.mma_done, 0)) break;
    }
    __syncwarp();
  } else if (!dead && warp < 4) {
    // ------------------------------------------------ epilogue
    int ti = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++ti) {
      const int b = u / nBlk, blk = u - b * nBlk;
      const int a = ti & 1;
      const unsigned ph = (unsigned)(ti >> 1) & 1u;
      const bool ok = mbar_wait(&sh.accf[a], ph, abort) && mbar_wait(&sh.nfull[a], ph, abort);
      if (!ok) record_timeout(abort);
      if (named_bar_or(1, 128, !ok)) break;
      tc_fence_after();
      const int r = blk * 128 + tid;
      const float rs2 = 2.f * sh.rs[a][tid];
      const float* Ar = A + ((long long)b * R + (r < R ? r : 0)) * D;
#pragma unroll 1
      for (int cc = 0; cc < g.nF; ++cc) {
        float v[32];
        const uint32_t tcol =
            tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(a * (WIDE ? 2 * BD : BD) + 32 * cc);
        tmem_ld32(tcol, v);
        if (WIDE) {
          float w[32];
          tmem_ld32(tcol + BD, w);
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] += w[q];  // (hi.hi + lo.hi) + hi.lo
        }
        if (cc == g.nF - 1) {
          tc_fence_before();
          mbar_arrive(&sh.acce[a]);
          mbar_arrive(&sh.nempty[a]);
        }
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const int d = 32 * cc + 4 * q4;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (r < R && d < D) x = __ldg(reinterpret_cast<const float4*>(Ar + d));
          v[4 * q4] = -2.f * v[4 * q4] + x.x * rs2;
          v[4 * q4 + 1] = -2.f * v[4 * q4 + 1] + x.y * rs2;
          v[4 * q4 + 2] = -2.f * v[4 * q4 + 2] + x.z * rs2;
          v[4 * q4 + 3] = -2.f * v[4 * q4 + 3] + x.w * rs2;
        }
        uint8_t* buf = stg_base;
        if (tid == 0) bulk_wait_read<0>();   // the previous store has read the buffer
        named_bar(1, 128);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<float4*>(buf + sw128_chunk(tid, q4)) =
              make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        fence_async_smem();
        named_bar(1, 128);
        if (tid == 0) {
          tma_store_3d(&mapOut, buf, 32 * cc, blk * 128, b);
          bulk_commit();
        }
      }
    }
    if (tid == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == GRAD_MMA_WARP) tmem_dealloc(tmem, g.tmem_cols);
}

int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  });
  return n;
}

bool aligned16(const void* p) { return p == nullptr || ((uintptr_t)p & 15u) == 0; }

}  // namespace

// ------------------------------------------------------------------ host

int make_map_3d_f32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t dim2, uint32_t box0, uint32_t box1, bool granule32) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<EncodeFn>(fn);
  });
  if (encode == nullptr) return set_error(kUnsupported, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {dim0, dim1, dim2};
  const cuuint64_t strides[2] = {dim0 * 4, dim0 * dim1 * 4};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            granule32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                      : CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kUnsupported, "tensor map rejected (CUresult %d)", (int)r);
  return kOk;
}

int tc_take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return kLaunch;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
  }
  return v;
}

// True when the tensor-core cost path applies: fp32 features with D >= 64,
// 16-byte aligned rows (D, M multiples of 4) and base pointers.  The
// TW_COST_SIMT environment variable (any value but "0") forces the SIMT path.
bool tc_cost_eligible(const float* X, const float* Y, const float* vx, const float* vy, int N,
                      int M, int D, const float* C, const float* Q) {
  const char* env = std::getenv("TW_COST_SIMT");
  if (env != nullptr && env[0] != '\0' && env[0] != '0') return false;
  (void)vx;
  (void)vy;
  (void)N;
  return D >= 64 && D % 4 == 0 && M % 4 == 0 && aligned16(X) && aligned16(Y) && aligned16(C) &&
         aligned16(Q);
}

int tc_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B, int N,
                int M, int D, double beta, double eps, float* C, float* Q, uint32_t* mask,
                cudaStream_t st) {
  if (B == 0 || N == 0 || M == 0) return kOk;
  CUtensorMap mX, mY, mC, mQ;
  int rc;
  if ((rc = make_map_3d_f32(&mX, X, D, N, B, KC, BM)) != kOk) return rc;
  if ((rc = make_map_3d_f32(&mY, Y, D, M, B, KC, BN)) != kOk) return rc;
  if ((rc = make_map_3d_f32(&mC, C, M, N, B, 32, BM)) != kOk) return rc;
  mQ = mC;
  if (Q != nullptr && (rc = make_map_3d_f32(&mQ, Q, M, N, B, 32, BM)) != kOk) return rc;
  const bool var = vx != nullptr;
  // X-resident form while one row block's X chunks and at least two Y stages
  // fit in shared memory (D <= 128); otherwise every tile streams X and Y.
  const int nK = (D + KC - 1) / KC;
  const int budget = 232448 - 2 * STG_BYTES - (int)sizeof(CostXRShared);
  for (int XB = 2; XB >= 1; --XB) {
    int YS = (budget - XB * nK * XR_CHUNK) / XR_CHUNK;
    if (YS > XR_MAX_YS) YS = XR_MAX_YS;
    if (YS < 2) continue;
    const CostXRGeom g{nK, XB, YS};
    const size_t smem =
        (size_t)(XB * nK + YS) * XR_CHUNK + 2 * STG_BYTES + sizeof(CostXRShared);
    const long long units = (long long)B * ((N + BM - 1) / BM);
    const int grid = (int)(units < sm_count() ? units : sm_count());
    auto kern = var ? tc_cost_xr_kernel<true> : tc_cost_xr_kernel<false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, COST_THREADS, smem, st>>>(mX, mY, mC, mQ, vx, vy, B, N, M, D, (float)beta,
                                           (float)eps, Q != nullptr ? 1 : 0, mask, g);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(kLaunch, "tc cost launch: %s", cudaGetErrorString(e));
    return kOk;
  }
  const long long tiles = (long long)B * ((N + BM - 1) / BM) * ((M + BN - 1) / BN);
  const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
  auto kern = var ? tc_cost_kernel<true> : tc_cost_kernel<false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)COST_SMEM);
  kern<<<grid, COST_THREADS, COST_SMEM, st>>>(mX, mY, mC, mQ, vx, vy, B, N, M, D, (float)beta,
                                              (float)eps, Q != nullptr ? 1 : 0, mask);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "tc cost launch: %s", cudaGetErrorString(e));
  return kOk;
}

namespace {

template <int SIDE, bool VAR, bool MASKED, bool TA, bool WIDE, bool PRE>
int grad_side_impl(const float* A, const float* F, const float* va, const float* vb,
                   const float* C, const float* dC, const float* dQ, int B, int N, int M, int D,
                   double beta, double eps, float* dA, float* dva, cudaStream_t st,
                   const uint32_t* mask, int sqrt_cost, const uint8_t* tflags) {
  const int R = SIDE == 0 ? N : M, S = SIDE == 0 ? M : N;
  if (((uintptr_t)tflags & 15u) != 0)
    return set_error(kUnsupported, "tc grad: chunk flags not 16-byte aligned");
  CUtensorMap mDC, mC, mDQ, mF, mOut;
  int rc;
  // SIDE 0 reads S as a K-major operand (16-byte granules), SIDE 1 as an
  // MN-major one (32-byte granules); the features are always MN-major.
  const uint32_t sbox_rows = SIDE == 0 ? 128 : 32;
  const bool s_g32 = SIDE == 1;
  if ((rc = make_map_3d_f32(&mDC, dC, M, N, B, 32, sbox_rows, s_g32)) != kOk) return rc;
  mC = mDC;  // C is not read when the positivity mask replaces it (or is already applied)
  if (!MASKED && !PRE && (rc = make_map_3d_f32(&mC, C, M, N, B, 32, sbox_rows, s_g32)) != kOk)
    return rc;
  mDQ = mC;
  const bool has_dq = VAR && dQ != nullptr;
  if (has_dq && (rc = make_map_3d_f32(&mDQ, dQ, M, N, B, 32, sbox_rows, s_g32)) != kOk) return rc;
  if ((rc = make_map_3d_f32(&mF, F, D, S, B, 32, 32, true)) != kOk) return rc;
  if ((rc = make_map_3d_f32(&mOut, dA, D, R, B, 32, 128)) != kOk) return rc;
  GradGeom g;
  g.nF = (D + 31) / 32;
  g.mw = (M + 31) / 32;
  g.np = (N + 3) & ~3;
  if (MASKED && ((uintptr_t)mask & 15u) != 0)
    return set_error(kUnsupported, "tc grad: mask not 16-byte aligned");
  int off = SBOX;                       // dC at 0
  g.l_c = (MASKED || PRE) ? -1 : off;
  if (!MASKED && !PRE) off += SBOX;
  g.l_dq = has_dq ? off : -1;
  if (has_dq) off += SBOX;
  g.l_f = off;
  off += g.nF * 4096;
  g.l_mask = off;
  if (MASKED) off += 512;
  g.l_bytes = (off + 1023) & ~1023;
  g.tx_fixed = SBOX * ((MASKED || PRE) ? 1 : 2) + (has_dq ? SBOX : 0) + g.nF * 4096;
  const int BD = 32 * g.nF;
  const int budget = 232448 - STG_BYTES - (int)sizeof(GradShared);
  if (TA) {
    // S in TMEM after the two accumulators: (hi 32 | lo 32) columns per slot
    g.c_fh = 0;
    g.c_fl = g.nF * 4096;
    g.c_bytes = 2 * g.nF * 4096;
    g.a_col0 = (uint32_t)(2 * (WIDE ? 2 * BD : BD));
    g.cstages = (512 - (int)g.a_col0) / 64;
    if (g.cstages > GRAD_MAX_CONV) g.cstages = GRAD_MAX_CONV;
    if (g.cstages < 1) return set_error(kUnsupported, "tc grad: D=%d too wide for S in TMEM", D);
    g.lstages = (budget - g.cstages * g.c_bytes) / g.l_bytes;
  } else {
    g.c_fh = 2 * SBOX;
    g.c_fl = 2 * SBOX + g.nF * 4096;
    g.c_bytes = 2 * SBOX + 2 * g.nF * 4096;
    g.a_col0 = 0;
    g.cstages = 2;
    g.lstages = (budget - g.cstages * g.c_bytes) / g.l_bytes;
    if (g.lstages < 2) {
      g.cstages = 1;
      g.lstages = (budget - g.c_bytes) / g.l_bytes;
    }
  }
  if (g.lstages > GRAD_MAX_LAND) g.lstages = GRAD_MAX_LAND;
  if (g.lstages < 1) return set_error(kUnsupported, "tc grad: D=%d needs too much shared memory", D);
  uint32_t need = (uint32_t)(2 * (WIDE ? 2 * BD : BD)) + (TA ? (uint32_t)(64 * g.cstages) : 0u);
  if (need > 512) return set_error(kUnsupported, "tc grad: D=%d needs %u TMEM columns", D, need);
  uint32_t cols = 32;
  while (cols < need) cols <<= 1;
  g.tmem_cols = cols;
  const size_t smem = (size_t)g.lstages * g.l_bytes + (size_t)g.cstages * g.c_bytes +
                      STG_BYTES + sizeof(GradShared);
  const long long units = (long long)B * ((R + 127) / 128);
  const int grid = (int)(units < sm_count() ? units : sm_count());
  auto kern = tc_grad_kernel<SIDE, VAR, MASKED, TA, WIDE, PRE>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int tf_k = ((S + 31) / 32 + 15) & ~15;  // flag row: one byte per chunk, padded to 16
  kern<<<grid, GRAD_THREADS, smem, st>>>(mDC, mC, mDQ, mF, mOut, A, va, vb, dva, B, N, M, D,
                                         (float)beta, (float)eps, has_dq ? 1 : 0, g, mask,
                                         sqrt_cost, tflags, tf_k);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kLaunch, "tc grad launch: %s", cudaGetErrorString(e));
  return kOk;
}

// S goes to TMEM (no shared-memory traffic for it) whenever the two
// accumulators leave room for it.  TW_GRAD_SMEM_S=1 keeps S in shared
// memory (for comparisons).
template <int SIDE, bool VAR, bool MASKED = false, bool PRE = false>
int grad_side(const float* A, const float* F, const float* va, const float* vb, const float* C,
              const float* dC, const float* dQ, int B, int N, int M, int D, double beta,
              double eps, float* dA, float* dva, cudaStream_t st,
              const uint32_t* mask = nullptr, int sqrt_cost = 0,
              const uint8_t* tflags = nullptr) {
  const char* env = std::getenv("TW_GRAD_SMEM_S");
  const bool smem_s = env != nullptr && env[0] != '\0' && env[0] != '0';
  const int BD = 32 * ((D + 31) / 32);
  // S in TMEM with wide MMAs while 2 x 2BD accumulator columns + one S slot
  // fit in 512 (D <= 96); wide MMAs with S in shared memory up to D = 128.
  if (!smem_s && 4 * BD + 64 <= 512)
    return grad_side_impl<SIDE, VAR, MASKED, true, true, PRE>(
        A, F, va, vb, C, dC, dQ, B, N, M, D, beta, eps, dA, dva, st, mask, sqrt_cost, tflags);
  if (2 * BD <= 256)
    return grad_side_impl<SIDE, VAR, MASKED, false, true, PRE>(
        A, F, va, vb, C, dC, dQ, B, N, M, D, beta, eps, dA, dva, st, mask, sqrt_cost, tflags);
  return grad_side_impl<SIDE, VAR, MASKED, false, false, PRE>(
      A, F, va, vb, C, dC, dQ, B, N, M, D, beta, eps, dA, dva, st, mask, sqrt_cost, tflags);
}

}  // namespace

// True when the tensor-core chain-rule path applies (same conditions as the
// cost path, and D <= 256 so a 128 x D accumulator pair fits in TMEM).
bool tc_grad_eligible(const float* X, const float* Y, const float* C, const float* dC,
                      const float* dQ, const float* dX, const float* dY, int M, int D) {
  return tc_cost_eligible(X, Y, nullptr, nullptr, 0, M, D, C, dC) && D <= 256 && aligned16(dQ) &&
         aligned16(dX) && aligned16(dY);
}

// tf_rows / tf_cols: optional chunk flags of dC and dQ (see tc_sq_grad_f32).
int tc_grad_f32(const float* X, const float* Y, const float* vx, const float* vy, const float* C,
                const float* dC, const float* dQ, int B, int N, int M, int D, double beta,
                double eps, float* dX, float* dY, float* dvx, float* dvy, cudaStream_t st,
                const uint8_t* tf_rows, const uint8_t* tf_cols) {
  if (B == 0 || N == 0 || M == 0) return kOk;
  int rc;
  if (vx != nullptr) {
    if ((rc = grad_side<0, true>(X, Y, vx, vy, C, dC, dQ, B, N, M, D, beta, eps, dX, dvx, st,
                                 nullptr, 0, tf_rows)))
      return rc;
    return grad_side<1, true>(Y, X, vy, vx, C, dC, dQ, B, N, M, D, beta, eps, dY, dvy, st,
                              nullptr, 0, tf_cols);
  }
  if ((rc = grad_side<0, false>(X, Y, nullptr, nullptr, C, dC, nullptr, B, N, M, D, beta, eps, dX,
                                nullptr, st, nullptr, 0, tf_rows)))
    return rc;
  return grad_side<1, false>(Y, X, nullptr, nullptr, C, dC, nullptr, B, N, M, D, beta, eps, dY,
                             nullptr, st, nullptr, 0, tf_cols);
}

// Chain rule of a query/support cost built by tc_cost_f32 (no variance):
// S = dC where cost > 0, or dC / (2 cost) for the Euclidean cost (sqrt_cost).
int tc_qs_grad_f32(const float* Q, const float* Sp, const float* C, const float* dC, int B,
                   int R, int U, int D, int sqrt_cost, float* dQ, float* dSp, cudaStream_t st) {
  if (B == 0 || R == 0 || U == 0) return kOk;
  int rc;
  if ((rc = grad_side<0, false>(Q, Sp, nullptr, nullptr, C, dC, nullptr, B, R, U, D, 0.0, 1e-8,
                                dQ, nullptr, st, nullptr, sqrt_cost)))
    return rc;
  return grad_side<1, false>(Sp, Q, nullptr, nullptr, C, dC, nullptr, B, R, U, D, 0.0, 1e-8, dSp,
                             nullptr, st, nullptr, sqrt_cost);
}

// Squared-Euclidean chain rule with the positivity mask of the cost kernel in
// place of the cost: S = dC where sq_raw > 0; with mask == nullptr, dC
// already carries the mask (S = dC).  tf_rows / tf_cols (optional) are the DP
// backward's nonzero-chunk flags of dC:
// [B][ceil(N/128)][KR] and [B][ceil(M/128)][KC] bytes, KR = 16 ceil(ceil(M/32)/16),
// KC = 16 ceil(ceil(N/32)/16); chunks flagged 0 are all zero and skipped.
int tc_sq_grad_f32(const float* X, const float* Y, const uint32_t* mask, const float* dC, int B,
                   int N, int M, int D, float* dX, float* dY, cudaStream_t st,
                   const uint8_t* tf_rows, const uint8_t* tf_cols) {
  if (B == 0 || N == 0 || M == 0) return kOk;
  int rc;
  if (mask == nullptr) {
    if ((rc = grad_side<0, false, false, true>(X, Y, nullptr, nullptr, nullptr, dC, nullptr, B, N,
                                               M, D, 0.0, 1e-8, dX, nullptr, st, nullptr, 0,
                                               tf_rows)))
      return rc;
    return grad_side<1, false, false, true>(Y, X, nullptr, nullptr, nullptr, dC, nullptr, B, N, M,
                                            D, 0.0, 1e-8, dY, nullptr, st, nullptr, 0, tf_cols);
  }
  if ((rc = grad_side<0, false, true>(X, Y, nullptr, nullptr, nullptr, dC, nullptr, B, N, M, D,
                                      0.0, 1e-8, dX, nullptr, st, mask, 0, tf_rows)))
    return rc;
  return grad_side<1, false, true>(Y, X, nullptr, nullptr, nullptr, dC, nullptr, B, N, M, D, 0.0,
                                   1e-8, dY, nullptr, st, mask, 0, tf_cols);
}

}  // namespace tw
