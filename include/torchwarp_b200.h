/*
 * torchwarp_b200 — C ABI of the B200 (sm_100a) differentiable-alignment kernels.
 *
 * Contract for every entry point:
 *   - All tensor pointers are device pointers to contiguous row-major arrays
 *     of the stated dtype (f32 = float, f64 = double).  The library never
 *     allocates or frees memory: the caller passes outputs, the saved state
 *     of a forward call (size from *_saved_bytes) and scratch workspace (size
 *     from *_workspace_bytes).
 *   - `stream` is a cudaStream_t (passed as void*); the work is enqueued on
 *     it and the call returns without synchronising.  The device is the
 *     caller's current device.
 *   - Return value: TW_OK (0) or a TW_ERR_* code; tw_last_error() returns a
 *     thread-local message for the last failure.  No exception crosses the ABI.
 *   - A forward and its backward must see the same (B, N, M, dtype) and run on
 *     the same device: the saved state is laid out by a plan derived from
 *     those and the device's SM count.
 *
 * Reference interfaces replaced (hibana2077/torchwarp, path:line):
 *   tw_sdtw_forward_*   <- udtw_forward()  src/torchwarp/csrc/udtw_cuda.cu:624-660
 *                          and jeanie_forward() with K=1 (soft_dtw_from_cost)
 *                          src/torchwarp/csrc/jeanie_cuda.cu:564-588
 *   tw_sdtw_backward_*  <- udtw_backward() src/torchwarp/csrc/udtw_cuda.cu:662-697
 *                          and jeanie_backward() with K=1 (jeanie_cuda.cu:590-619)
 *   tw_udtw_cost_*      <- the cost/penalty construction inside
 *                          udtw_fused_forward_kernel (udtw_cuda.cu:298-422) and
 *                          torch.bmm in udtw/_ops.py:164-165
 *   tw_udtw_features_grad_* <- udtw_fused_backward's chain rule
 *                          (udtw_cuda.cu:557-568) plus _features_grads
 *                          (udtw/_ops.py:179-183)
 */
#ifndef TORCHWARP_B200_H_
#define TORCHWARP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TW_OK 0
#define TW_ERR_INVALID 1
#define TW_ERR_UNSUPPORTED 2
#define TW_ERR_LAUNCH 3
#define TW_ERR_TIMEOUT 4
#define TW_ERR_WORKSPACE 5

/* Library version (major*10000 + minor*100 + patch). */
int tw_version(void);
/* Message of the last error on this host thread ("" if none). */
const char* tw_last_error(void);
/* Reads and clears the device-side error words of the tensor-core kernels
 * and of the DP sweeps (0: none; TW_ERR_TIMEOUT: a bounded pipeline wait, or
 * a band group's window wait, ran out; TW_ERR_LAUNCH: unaligned shared
 * memory).  Synchronises with the device.  No counterpart in the reference,
 * whose kernels have no device-side waits. */
int tw_device_error(void);

/* ---------------------------------------------------------------------
 * Soft-min DP on a precomputed cost (soft-DTW / uDTW), natural layout.
 *   cost, penalty: [B, N, M]; penalty may be NULL (soft-DTW: no P output).
 *   gamma > 0; bandwidth > 0 enables the Sakoe-Chiba band |i - j| <= band.
 *   out_r [B]: R[N-1, M-1] (+inf if the band makes it unreachable);
 *   out_p [B]: P[N-1, M-1] (only when penalty != NULL).
 *   saved: tw_sdtw_saved_bytes() bytes, written here, read by the backward.
 *   workspace: tw_sdtw_workspace_bytes() bytes of scratch.
 * ------------------------------------------------------------------- */
size_t tw_sdtw_saved_bytes(int B, int N, int M, int dtype_bytes, int has_penalty);
size_t tw_sdtw_workspace_bytes(int B, int N, int M, int dtype_bytes, int has_penalty);

int tw_sdtw_forward_f32(const float* cost, const float* penalty, int B, int N, int M,
                        double gamma, double bandwidth, float* out_r, float* out_p,
                        void* saved, size_t saved_bytes, void* workspace, size_t ws_bytes,
                        void* stream);
int tw_sdtw_forward_f64(const double* cost, const double* penalty, int B, int N, int M,
                        double gamma, double bandwidth, double* out_r, double* out_p,
                        void* saved, size_t saved_bytes, void* workspace, size_t ws_bytes,
                        void* stream);

/* Allocation-free variant of tw_sdtw_forward_f32 (no counterpart in the
 * reference; an addition of this library).  For callers that own every device
 * allocation and can pass only inputs and outputs: the forward's scratch comes
 * from a static 4 MiB device buffer inside the library instead of `workspace`.
 * Same arguments and results as tw_sdtw_forward_f32 minus the workspace;
 * `saved` is still the caller's (it is an output consumed by the backward).
 * Limits: shapes whose scratch (tw_sdtw_workspace_bytes) exceeds 4 MiB are
 * rejected with TW_ERR_WORKSPACE; every call shares the one buffer, so calls
 * that overlap on the GPU race and must be serialised by the caller.  Each
 * call looks up the buffer's device address on the current device (so a
 * device reset between calls is harmless); the first call on a device also
 * loads the library's device code there and should come before any stream
 * capture. */
int tw_sdtw_forward_noalloc_f32(const float* cost, const float* penalty, int B, int N, int M,
                                double gamma, double bandwidth, float* out_r, float* out_p,
                                void* saved, size_t saved_bytes, void* stream);

/* Backward of the call above for L = sum_b grad_r[b]*out_r[b] + grad_p[b]*out_p[b].
 *   d_cost, d_penalty: [B, N, M] outputs (d_penalty only when has_penalty). */
int tw_sdtw_backward_f32(const float* grad_r, const float* grad_p, int B, int N, int M,
                         double gamma, int has_penalty, const void* saved, size_t saved_bytes,
                         float* d_cost, float* d_penalty, void* workspace, size_t ws_bytes,
                         void* stream);
int tw_sdtw_backward_f64(const double* grad_r, const double* grad_p, int B, int N, int M,
                         double gamma, int has_penalty, const void* saved, size_t saved_bytes,
                         double* d_cost, double* d_penalty, void* workspace, size_t ws_bytes,
                         void* stream);

/* tw_sdtw_backward_f32 that also flags, in `flags` (layout of
 * tw_sdtw_backward_masked_flags_f32, zeroed here; NULL: none), the chunks
 * where d_cost or d_penalty holds a nonzero value, for
 * tw_udtw_features_grad_flagged_f32. */
int tw_sdtw_backward_flags_f32(const float* grad_r, const float* grad_p, int B, int N, int M,
                               double gamma, int has_penalty, const void* saved,
                               size_t saved_bytes, float* d_cost, float* d_penalty,
                               uint8_t* flags, size_t flags_bytes, void* workspace,
                               size_t ws_bytes, void* stream);

/* soft-DTW backward that also applies the positivity mask of
 * tw_sqeuclid_cost_* (no penalty): writes d_cost[b,i,j] = dL/dcost[b,i,j] where
 * the mask bit of (b,i,j) is set, else 0 -- the S operand of the squared-
 * Euclidean chain rule, which tw_sqeuclid_grad_* then takes with mask = NULL.
 * Same saved state, workspace and results as tw_sdtw_backward_* otherwise.
 * Mask layout: see tw_sqeuclid_cost_f32.  (The reference multiplies by the
 * clamp's derivative inside its chain rule, udtw_cuda.cu:557-568.) */
int tw_sdtw_backward_masked_f32(const float* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                float* d_cost, void* workspace, size_t ws_bytes, void* stream);
int tw_sdtw_backward_masked_f64(const double* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                double* d_cost, void* workspace, size_t ws_bytes, void* stream);

/* The masked soft-DTW backward above (fp32), also flagging the chunks of
 * d_cost it writes a nonzero value into, for tw_sqeuclid_grad_flagged_f32.
 * flags: tw_sdtw_chunk_flags_bytes(B, N, M) bytes (zeroed and filled here):
 * one byte per 128 x 32 chunk [B][ceil(N/128)][KR], then one per 32 x 128
 * chunk [B][ceil(M/128)][KC], each part 256-byte aligned, KR and KC the
 * chunk counts ceil(M/32) and ceil(N/32) rounded up to multiples of 16.
 * flags = NULL: no flags (same as tw_sdtw_backward_masked_f32). */
size_t tw_sdtw_chunk_flags_bytes(int B, int N, int M);
int tw_sdtw_backward_masked_flags_f32(const float* grad_r, int B, int N, int M, double gamma,
                                      const void* saved, size_t saved_bytes,
                                      const uint32_t* mask, float* d_cost, uint8_t* flags,
                                      size_t flags_bytes, void* workspace, size_t ws_bytes,
                                      void* stream);

/* The fastest fp32 pair for soft-DTW on features.  The masked backward
 * above with the chunk flags, writing d_cost sparsely: an 8-column tile of a
 * row that holds only zeros is not written, and nz_mask (uint32 words in the
 * positivity mask's layout [B][ceil(M/32)][4 ceil(N/4)],
 * tw_sdtw_nonzero_mask_bytes(B, N, M) bytes, zeroed and filled here) gets a
 * set bit for every nonzero value.  Cells of d_cost whose bit is clear may
 * hold anything; pass nz_mask along with it.  mask, nz_mask and flags are
 * required.  (The reference writes every cell of its cost gradient.) */
size_t tw_sdtw_nonzero_mask_bytes(int B, int N, int M);
int tw_sdtw_backward_sparse_f32(const float* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                float* d_cost, uint32_t* nz_mask, uint8_t* flags,
                                size_t flags_bytes, void* workspace, size_t ws_bytes,
                                void* stream);

/* soft-DTW backward on features for the squared-Euclidean cost of
 * tw_sqeuclid_cost_* (the backward half of the reference's fused soft-DTW on
 * features: udtw_fused_backward with unit variance, src/torchwarp/udtw/_ops.py:179-183,
 * csrc/udtw_cuda.cu:557-568): the masked DP backward, then the chain rule
 *   dX = -2 S Y + 2 X rowsum(S), dY = -2 S^T X + 2 Y colsum(S),  S = dL/dcost.
 * X [B,N,D], Y [B,M,D], mask and saved from tw_sqeuclid_cost_* and
 * tw_sdtw_forward_*; dX, dY outputs.  workspace: at least
 * tw_sdtw_features_workspace_bytes(B, N, M, dtype_bytes) bytes (dL/dcost,
 * the DP's delay lines and, for fp32, the chunk flags and the nonzero mask).
 * fp32 runs tw_sdtw_backward_sparse_f32 then tw_sqeuclid_grad_sparse_f32. */
size_t tw_sdtw_features_workspace_bytes(int B, int N, int M, int dtype_bytes);
int tw_sdtw_features_backward_f32(const float* X, const float* Y, const uint32_t* mask,
                                  const float* grad_r, int B, int N, int M, int D, double gamma,
                                  const void* saved, size_t saved_bytes, float* dX, float* dY,
                                  void* workspace, size_t ws_bytes, void* stream);
int tw_sdtw_features_backward_f64(const double* X, const double* Y, const uint32_t* mask,
                                  const double* grad_r, int B, int N, int M, int D, double gamma,
                                  const void* saved, size_t saved_bytes, double* dX, double* dY,
                                  void* workspace, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------
 * uDTW / soft-DTW cost from features (uDTW Eqs. 8, 16):
 *   sq_ij  = max(|x_i|^2 + |y_j|^2 - 2 x_i.y_j, 0)
 *   var_ij = max(0.5 (vx_i + vy_j), eps)
 *   cost_ij = sq_ij / var_ij,  penalty_ij = beta * log(var_ij)
 * X [B,N,D], Y [B,M,D], vx [B,N], vy [B,M] (vx/vy NULL: variance 1, no penalty).
 * cost, penalty: [B,N,M] outputs (penalty may be NULL).
 * fp32 with D >= 64, D and M multiples of 4 and 16-byte aligned pointers runs
 * the x.y contraction on tcgen05 tensor cores (3xTF32, fp32 accumulate);
 * other shapes, and fp64, use SIMT kernels.  Setting the environment
 * variable TW_COST_SIMT=1 forces the SIMT kernels (for testing). */
int tw_udtw_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B,
                     int N, int M, int D, double beta, double eps, float* cost, float* penalty,
                     void* stream);
int tw_udtw_cost_f64(const double* X, const double* Y, const double* vx, const double* vy, int B,
                     int N, int M, int D, double beta, double eps, double* cost, double* penalty,
                     void* stream);

/* Chain rule of the cost above: given d_cost, d_penalty [B,N,M] (d_penalty may
 * be NULL), the cost [B,N,M] it was built with, and the inputs, writes
 *   dX [B,N,D], dY [B,M,D], dvx [B,N], dvy [B,M]  (dvx/dvy may be NULL).
 * Zero-gradient conventions of torch.clamp_min: none through sq <= 0 or
 * var_raw <= eps. */
int tw_udtw_features_grad_f32(const float* X, const float* Y, const float* vx, const float* vy,
                              const float* cost, const float* d_cost, const float* d_penalty,
                              int B, int N, int M, int D, double beta, double eps, float* dX,
                              float* dY, float* dvx, float* dvy, void* stream);
int tw_udtw_features_grad_f64(const double* X, const double* Y, const double* vx,
                              const double* vy, const double* cost, const double* d_cost,
                              const double* d_penalty, int B, int N, int M, int D, double beta,
                              double eps, double* dX, double* dY, double* dvx, double* dvy,
                              void* stream);
/* tw_udtw_features_grad_f32 given the chunk flags of tw_sdtw_backward_flags_f32
 * (NULL: none): on the tensor-core path it reads only the chunks where d_cost
 * or d_penalty is nonzero; the others add exactly zero to every output.
 * TW_GRAD_DENSE=1 reads every chunk. */
int tw_udtw_features_grad_flagged_f32(const float* X, const float* Y, const float* vx,
                                      const float* vy, const float* cost, const float* d_cost,
                                      const float* d_penalty, const uint8_t* flags, int B, int N,
                                      int M, int D, double beta, double eps, float* dX, float* dY,
                                      float* dvx, float* dvy, void* stream);

/* ---------------------------------------------------------------------
 * soft-DTW's squared-Euclidean cost with a positivity mask in place of the
 * cost for the chain rule (cost path of sdtw.py:78-84, chain rule of
 * udtw_cuda.cu:557-568 with unit variance):
 *   cost_ij = max(|x_i|^2 + |y_j|^2 - 2 x_i.y_j, 0)   [B,N,M]
 *   mask: uint32 words [B][ceil(M/32)][NP], NP = 4 ceil(N/4); bit (j & 31)
 *         of word [b][j>>5][i] is set where the unclamped value is > 0 (bits
 *         for j >= M and words of rows i >= N are 0).
 * The chain rule reads the mask instead of the cost (1 bit instead of 4 or 8
 * bytes per cell), so the cost can be freed after the DP forward:
 *   dX = -2 S Y + 2 X rowsum(S), dY = -2 S^T X + 2 Y colsum(S),
 *   S = d_cost where the mask bit is set, else 0; with mask = NULL, S = d_cost
 *   (the mask was already applied, e.g. by tw_sdtw_backward_masked_*).
 * fp32 with D >= 64 (D, M multiples of 4, 16-byte aligned) runs on tcgen05
 * tensor cores (3xTF32); other shapes and fp64 on SIMT kernels. */
int tw_sqeuclid_cost_f32(const float* X, const float* Y, int B, int N, int M, int D, float* cost,
                         uint32_t* mask, void* stream);
int tw_sqeuclid_cost_f64(const double* X, const double* Y, int B, int N, int M, int D,
                         double* cost, uint32_t* mask, void* stream);
int tw_sqeuclid_grad_f32(const float* X, const float* Y, const uint32_t* mask,
                         const float* d_cost, int B, int N, int M, int D, float* dX, float* dY,
                         void* stream);
int tw_sqeuclid_grad_f64(const double* X, const double* Y, const uint32_t* mask,
                         const double* d_cost, int B, int N, int M, int D, double* dX,
                         double* dY, void* stream);
/* tw_sqeuclid_grad_f32 with mask = NULL (S = d_cost), given the chunk flags
 * of tw_sdtw_backward_masked_flags_f32 (NULL: none).  On the tensor-core path
 * it reads only the flagged chunks of d_cost and the first chunk of each
 * 128-row (128-column) unit: a chunk flagged zero holds only zeros and adds
 * exactly zero, so the result is that of the dense product.  The
 * environment variable TW_GRAD_DENSE=1 makes it read every chunk. */
int tw_sqeuclid_grad_flagged_f32(const float* X, const float* Y, const float* d_cost,
                                 const uint8_t* flags, int B, int N, int M, int D, float* dX,
                                 float* dY, void* stream);
/* The chain rule after tw_sdtw_backward_sparse_f32: S = d_cost where the
 * nz_mask bit is set, else 0 (whatever d_cost holds there), reading only the
 * flagged chunks on the tensor-core path.  Same result as the dense d_cost of
 * tw_sdtw_backward_masked_f32 through tw_sqeuclid_grad_f32. */
int tw_sqeuclid_grad_sparse_f32(const float* X, const float* Y, const uint32_t* nz_mask,
                                const float* d_cost, const uint8_t* flags, int B, int N, int M,
                                int D, float* dX, float* dY, void* stream);

/* ---------------------------------------------------------------------
 * JEANIE on a cost [B, K1, K2, T, U] (one viewpoint axis: K2 = 1).
 *   s1, s2: viewpoint shifts (already clamped to K-1 by the caller).
 *   out [B]: soft-min over viewpoints of R[:, T-1, U-1];
 *   R [B, K1, K2, T, U]: the accumulator (saved state of the backward).
 * Replaces jeanie_forward() src/torchwarp/csrc/jeanie_cuda.cu:564-588 (and
 * the diagonal-major relayout of jeanie/_ops.py:68-79: layouts are natural).
 * ------------------------------------------------------------------- */
int tw_jeanie_forward_f32(const float* cost, int B, int K1, int K2, int T, int U, int s1, int s2,
                          double gamma, float* out, float* R, void* stream);
int tw_jeanie_forward_f64(const double* cost, int B, int K1, int K2, int T, int U, int s1, int s2,
                          double gamma, double* out, double* R, void* stream);
/* Backward for L = sum_b grad_out[b] out[b] + <grad_R, R> (grad_R may be NULL).
 * Replaces jeanie_backward() src/torchwarp/csrc/jeanie_cuda.cu:590-619. */
int tw_jeanie_backward_f32(const float* cost, const float* R, const float* grad_out,
                           const float* grad_R, int B, int K1, int K2, int T, int U, int s1,
                           int s2, double gamma, float* d_cost, void* stream);
int tw_jeanie_backward_f64(const double* cost, const double* R, const double* grad_out,
                           const double* grad_R, int B, int K1, int K2, int T, int U, int s1,
                           int s2, double gamma, double* d_cost, void* stream);

/* Query/support base cost: query [B, R, D] (R = K*T rows in (n, t) order),
 * support [B, U, D] -> cost [B, R, U]; metric 0 = squared Euclidean
 * (clamped at 0), 1 = Euclidean.  Replaces the bmm + relayout of
 * jeanie/_ops.py:159-167 feeding jeanie_fused_forward (jeanie_cuda.cu:621-648)
 * and the torch cost of jeanie/distances.py:25-38. */
int tw_qs_cost_f32(const float* query, const float* support, int B, int R, int U, int D,
                   int metric, float* cost, void* stream);
int tw_qs_cost_f64(const double* query, const double* support, int B, int R, int U, int D,
                   int metric, double* cost, void* stream);
/* Gradient of that cost given d_cost [B, R, U]: d_query [B, R, D],
 * d_support [B, U, D] (no gradient through sq <= 0, as torch.clamp_min /
 * sqrt at 0).  Replaces jeanie_fused_backward's chain rule + bmm
 * (jeanie_cuda.cu:650-683, jeanie/_ops.py:208-215); deterministic. */
int tw_qs_cost_grad_f32(const float* query, const float* support, const float* cost,
                        const float* d_cost, int B, int R, int U, int D, int metric,
                        float* d_query, float* d_support, void* stream);
int tw_qs_cost_grad_f64(const double* query, const double* support, const double* cost,
                        const double* d_cost, int B, int R, int U, int D, int metric,
                        double* d_query, double* d_support, void* stream);

/* RBF base cost: query [B, R, D], support [B, U, D] -> cost [B, R, U] with
 * cost_ru = sum_d [2 - 2 exp(-sigma (q_rd - s_ud)^2)], sigma > 0.  Replaces
 * the PyTorch rbf_cost of jeanie/distances.py:41-51, which materialises the
 * [.., R, U, D] difference tensor. */
int tw_qs_rbf_cost_f32(const float* query, const float* support, int B, int R, int U, int D,
                       double sigma, float* cost, void* stream);
int tw_qs_rbf_cost_f64(const double* query, const double* support, int B, int R, int U, int D,
                       double sigma, double* cost, void* stream);
/* Its gradient given d_cost [B, R, U]: d_query [B, R, D] and d_support
 * [B, U, D], written (not accumulated); deterministic (no atomics).  Replaces
 * autograd through the same expression. */
int tw_qs_rbf_cost_grad_f32(const float* query, const float* support, const float* d_cost,
                            int B, int R, int U, int D, double sigma, float* d_query,
                            float* d_support, void* stream);
int tw_qs_rbf_cost_grad_f64(const double* query, const double* support, const double* d_cost,
                            int B, int R, int U, int D, double sigma, double* d_query,
                            double* d_support, void* stream);

/* FVM viewpoint soft-min: cost [B, Kf, TU] -> temporal [B, TU] =
 * -gamma logsumexp_n(-cost / gamma), and its backward d_cost = softmax_n *
 * d_temporal.  Replaces jeanie/fvm.py:36-37 (torch logsumexp). */
int tw_fvm_softmin_f32(const float* cost, int B, int Kf, int TU, double gamma, float* temporal,
                       void* stream);
int tw_fvm_softmin_f64(const double* cost, int B, int Kf, int TU, double gamma,
                       double* temporal, void* stream);
int tw_fvm_softmin_backward_f32(const float* cost, const float* d_temporal, int B, int Kf,
                                int TU, double gamma, float* d_cost, void* stream);
int tw_fvm_softmin_backward_f64(const double* cost, const double* d_temporal, int B, int Kf,
                                int TU, double gamma, double* d_cost, void* stream);

/* ---------------------------------------------------------------------
 * Fused JEANIE and FVM, float32: one call per direction builds each pair's
 * query/support cost from the features (or takes a cost), runs FVM's
 * viewpoint soft-min and the temporal soft-min DP on chip, and in the
 * backward the DP adjoint and the chain rule back to the features.
 *   features: query [B, K1*K2*T, D] (rows in (viewpoint, t) order), support
 *             [B, U, D], cost = NULL; metric 0 squared Euclidean (clamped at
 *             0), 1 Euclidean (no gradient at distance 0).
 *   cost:     query = support = NULL, cost [B, K1, K2, T, U].
 *   fvm = 0:  JEANIE with viewpoint shifts s1, s2 (clamped to K-1 by the
 *             caller); out [B] = soft-min over the viewpoints of the end
 *             cells; R [B, K1, K2, T, U] (may be NULL) = the accumulator.
 *   fvm = 1:  FVM (K2 = 1, K1 = all viewpoints): soft-min over the
 *             viewpoints at every (t, u), then soft-DTW; R must be NULL.
 *   saved:    tw_jeanie_fused_saved_bytes() bytes, 16-byte aligned, written
 *             by the forward and read by the backward (with the same cost
 *             pointer for a cost input).
 *   Backward for L = sum_b grad_out[b] out[b] + <grad_R, R> (grad_R NULL for
 *   none; always NULL for FVM): d_query [B, K T, D], d_support [B, U, D]
 *   with features, d_cost [B, K1, K2, T, U] with a cost; written, not
 *   accumulated.
 * tw_jeanie_fused_supported says whether a shape runs here (even D <= 256,
 * U <= 15 with features, a pair's state within 96 KB of shared memory);
 * other shapes use tw_qs_cost_* + tw_jeanie_* / tw_fvm_softmin_*.
 * Replaces jeanie_fused_forward / jeanie_fused_backward
 * (src/torchwarp/csrc/jeanie_cuda.cu:621-683, with jeanie/_ops.py:155-230)
 * and FVM's logsumexp + soft-DTW (src/torchwarp/jeanie/fvm.py:15-67). */
int tw_jeanie_fused_supported(int K, int T, int U, int D, int fvm, int features);
size_t tw_jeanie_fused_saved_bytes(int B, int K, int T, int U, int fvm, int features);
int tw_jeanie_fused_forward_f32(const float* query, const float* support, const float* cost,
                                int B, int K1, int K2, int T, int U, int D, int s1, int s2,
                                int metric, int fvm, double gamma, float* out, float* R,
                                void* saved, size_t saved_bytes, void* stream);
int tw_jeanie_fused_backward_f32(const float* query, const float* support, const float* cost,
                                 const float* grad_out, const float* grad_R, int B, int K1, int K2,
                                 int T, int U, int D, int s1, int s2, int metric, int fvm,
                                 double gamma, const void* saved, size_t saved_bytes,
                                 float* d_query, float* d_support, float* d_cost, void* stream);

/* Hard alignment path (gamma -> 0) of cost [B, K, T, U] (float64), with the
 * tie-break of src/torchwarp/paths.py:85-117 (viewpoint ascending, then
 * (t-1,u-1), (t-1,u), (t,u-1), strict <; end viewpoint = first argmin);
 * start_view < 0 means a free start.  Workspaces r_ws (double) and back_ws
 * (int) hold B*K*T*U each; path [B, T+U-1, 3] gets (t, u, k) from (0,0) to
 * (T-1,U-1) and length [B] its number of cells.  Replaces _optimal_3d. */
int tw_optimal_path_f64(const double* cost, int B, int K, int T, int U, int max_shift,
                        int start_view, double* r_ws, int* back_ws, int* path, int* length,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TORCHWARP_B200_H_ */
