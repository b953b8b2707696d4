// Warp-stream soft-min dynamic program for soft-DTW / uDTW (sm_100a).
//
// Work decomposition (host plan, StreamPlan):
//   * One warp owns the pairs [p0, p0 + npairs).  A pair's N rows are cut into
//     NB bands of 32*KS rows; a band is one "pass" over L >= M + 1 stream
//     columns (column j < M is data, j >= M is padding with cost +Big).
//   * Inside a band, lane l owns rows 32k + l of the KS sub-bands k.  Sub-band
//     k lags sub-band k-1 by 32 steps and lane l lags lane l-1 by one step, so
//     at warp step t every lane works on stream column t - 32k - l: all KS
//     cells of a lane lie on one anti-diagonal and are independent (ILP = KS).
//   * Passes follow each other without a gap: after a lane finishes column
//     L-1 of one band it starts column 0 of the next band (or the next pair),
//     so the warp never drains between bands or pairs.
//   * Row i-1 -> row i hand-off is one rotating __shfl per sub-band (lane 31 of
//     sub-band k-1 feeds lane 0 of sub-band k); band b -> band b+1 goes through
//     a per-warp delay line of L values in global scratch.
//   * Band groups (G > 1, for batches too small to fill the SMs): G warps of
//     one CTA share a group's pairs, warp g taking bands g, g+G, g+2G, ...
//     Pass q of the group starts D = L/G steps after pass q-1, so warp g runs
//     its own stream shifted by g*D steps, reads band b-1's bottom row from
//     the delay line of the warp that computed it, and the G warps stay in
//     step through one bounded mbarrier wait per 32-step window.  G = 1 is
//     the single-warp stream above.
//
// Saved state: R (and P for uDTW) of every cell, in stream order
// [warp][t][k][lane] (one coalesced 128-byte row per sub-band and step), in
// the log2 domain R' = R * log2(e) / gamma, and each warp's band-bottom row
// again as a compact edge stream [warp][t].  The backward sweep replays the
// stream in reverse and needs nothing else: the soft-min weights of a cell's
// three predecessors are recomputed from their saved R', so neither the cost
// nor the penalty is read again.
#pragma once

#include "common.cuh"

namespace tw {

// Division by a divisor fixed for a launch (Granlund & Montgomery, "Division
// by invariant integers using multiplication", PLDI 1994: the round-up
// multiplier with the add-back step).  With l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(m, n) + n) >> l exactly
// for 0 <= n < 2^31.
struct Divisor {
  uint32_t m = 1;
  int l = 0;
  int d = 1;
};
Divisor make_divisor(int d);

struct StreamPlan {
  int B = 0, N = 0, M = 0;
  int KS = 1;        // sub-bands per warp
  int NB = 1;        // bands per pair
  int L = 0;         // stream columns per band pass (multiple of 8 G)
  int G = 1;         // warps per band group (divides NB and wpc)
  int NBg = 1;       // NB / G: bands of a pair in one warp's stream
  Divisor dL, dNB, dNBg;   // L, NB and NBg as invariant divisors
  int D = 0;         // L / G: steps between the starts of consecutive passes
  int warps = 0;     // warps launched (a multiple of G)
  int wpc = 4;       // warps per CTA
  int base = 0, rem = 0;   // group s: base + (s < rem) pairs from s*base + min(s, rem)
  long long tmax = 0;      // saved rows per warp (multiple of 8)
  size_t smem_fwd = 0, smem_bwd = 0;   // dynamic shared memory per CTA

  // Each warp's saved stream starts with kPreRows rows of +Big (R) / 0 (P),
  // so the backward sweep reloads rows below the stream start unguarded.
  // Warp slices are `tstride` rows apart (>= tmax + kPreRows).
  static constexpr int kPreRows = 16;
  long long tstride = 0;
  // Each of the R and P blocks of the saved buffer is the stream of every
  // warp followed by its edge stream: the value of lane 31 of sub-band KS-1
  // (the band's bottom row) at every step, tstride values per warp, which
  // the backward reads as the row above the next band.
  long long saved_elems() const {
    return (long long)warps * tstride * KS * 32 + (long long)warps * tstride;
  }
  // offset of warp w's stream row 0
  __host__ __device__ long long saved_offset(int w) const {
    return ((long long)w * tstride + kPreRows) * KS * 32;
  }
  // offset of warp w's edge value of step 0
  __host__ __device__ long long edge_offset(int w) const {
    return (long long)warps * tstride * KS * 32 + (long long)w * tstride + kPreRows;
  }
  long long delay_elems() const { return (long long)warps * L; }
  // dynamic shared memory after the warps' regions: the groups' mbarriers
  // (reserved only when G > 1)
  static constexpr int kSmemHeader = 64;
};

// elem_bytes: 4 or 8.  has_p: uDTW penalty accumulator.  sms: SM count.
StreamPlan make_stream_plan(int B, int N, int M, int elem_bytes, bool has_p, int sms);

template <typename T>
struct SdtwArgs {
  // forward inputs / outputs
  const T* C = nullptr;      // cost [B,N,M]
  const T* Q = nullptr;      // penalty [B,N,M] (uDTW) or null
  T* out_r = nullptr;        // [B]
  T* out_p = nullptr;        // [B] (uDTW) or null
  // saved stream (written by forward, read by backward)
  T* sR = nullptr;
  T* sP = nullptr;
  // per-warp delay lines (global scratch)
  T* dlR = nullptr;
  T* dlP = nullptr;
  // backward
  const T* grad_r = nullptr;  // [B]
  const T* grad_p = nullptr;  // [B] or null
  T* dC = nullptr;            // [B,N,M]
  T* dQ = nullptr;            // [B,N,M] or null
  // positivity mask of the squared-Euclidean cost, uint32 words
  // [B][ceil(M/32)][mask_np]: dC is written as dC * bit (null: no mask)
  const uint32_t* mask = nullptr;
  int mask_np = 0;
  // Nonzero-chunk flags of dC for the chain rule (optional; the caller zeroes
  // them first): byte [b][i/128][j/32] of tf_rows (row stride tf_kr) and
  // byte [b][j/128][i/32] of tf_cols (row stride tf_kc) are set to 1 where a
  // written dC value of that 128 x 32 (32 x 128) chunk is nonzero.
  uint8_t* tf_rows = nullptr;
  uint8_t* tf_cols = nullptr;
  int tf_kr = 0, tf_kc = 0;
  // backward: 1 = evaluate every block, also those whose adjoints are all
  // zero (for comparisons; the result is the same)
  int all_blocks = 0;
  // Sparse dC (optional, with `mask`): 8-column tiles of a row that hold only
  // zeros are not written, and nzm (uint32 words in the positivity mask's
  // layout, zeroed by the caller) gets the bits of the nonzero values; cells
  // whose bit is clear may hold anything.
  uint8_t* nzm = nullptr;
  // scalars
  T kappa = 1;      // log2(e) / gamma
  T inv_kappa = 1;  // gamma * ln 2
  T inv_gamma = 1;
  T pad_raw = 0;    // Big / kappa: raw cost of a padding column
  T band = 0;       // Sakoe-Chiba band (> 0 active)
  int vec = 0;      // 16-byte global accesses allowed for C/Q/dC/dQ
  StreamPlan p;
};

// Reads and clears the device-side error word of the stream kernels (a band
// group's window wait that ran out: kTimeout).
int dp_take_device_error();

template <typename T>
int sdtw_stream_forward(const SdtwArgs<T>& a, bool has_p, bool has_band, cudaStream_t st);
template <typename T>
int sdtw_stream_backward(const SdtwArgs<T>& a, bool has_p, bool has_band, cudaStream_t st);

}  // namespace tw
