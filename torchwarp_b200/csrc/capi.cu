// extern "C" entry points of libtorchwarp_b200.so; see include/torchwarp_b200.h.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/torchwarp_b200.h"
#include "common.cuh"
#include "sdtw_stream.cuh"

namespace tw {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// SM count of the current device, read once per device.
static int device_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

static bool dims_ok(int B, int N, int M) { return B >= 0 && N > 0 && M > 0; }

static int check_dims(const char* who, int B, int N, int M) {
  if (!dims_ok(B, N, M))
    return set_error(kInvalid, "%s: invalid sizes B=%d N=%d M=%d (need B >= 0, N, M > 0)", who, B,
                     N, M);
  const long long steps = ((long long)B * ((N + 127) / 128)) * (long long)(M + 256);
  if (steps > (1LL << 30))
    return set_error(kUnsupported, "%s: problem too large for one launch (B=%d N=%d M=%d)", who,
                     B, N, M);
  return kOk;
}

template <typename T>
int sdtw_fwd(const T* cost, const T* pen, int B, int N, int M, double gamma, double band,
                    T* out_r, T* out_p, void* saved, size_t saved_bytes, void* ws, size_t ws_bytes,
                    cudaStream_t st) {
  g_err[0] = 0;
  if (int e = check_dims("tw_sdtw_forward", B, N, M)) return e;
  if (!(gamma > 0)) return set_error(kInvalid, "tw_sdtw_forward: gamma must be > 0");
  if (B == 0) return kOk;
  if (!cost || !out_r || !saved || !ws || (pen && !out_p))
    return set_error(kInvalid, "tw_sdtw_forward: null pointer argument");
  const bool has_p = pen != nullptr;
  StreamPlan p = make_stream_plan(B, N, M, sizeof(T), has_p, device_sms());
  const size_t sb = align256(p.saved_elems() * sizeof(T)) * (has_p ? 2 : 1);
  const size_t wb = align256(p.delay_elems() * sizeof(T)) * (has_p ? 2 : 1);
  if (saved_bytes < sb) return set_error(kWorkspace, "tw_sdtw_forward: saved needs %zu bytes", sb);
  if (ws_bytes < wb) return set_error(kWorkspace, "tw_sdtw_forward: workspace needs %zu bytes", wb);
  SdtwArgs<T> a;
  a.C = cost;
  a.Q = pen;
  a.out_r = out_r;
  a.out_p = out_p;
  a.sR = static_cast<T*>(saved);
  a.sP = has_p ? reinterpret_cast<T*>(static_cast<char*>(saved) + sb / 2) : nullptr;
  a.dlR = static_cast<T*>(ws);
  a.dlP = has_p ? reinterpret_cast<T*>(static_cast<char*>(ws) + wb / 2) : nullptr;
  const double kappa = 1.4426950408889634 / gamma;
  a.kappa = (T)kappa;
  a.inv_kappa = (T)(1.0 / kappa);
  a.inv_gamma = (T)(1.0 / gamma);
  a.pad_raw = (T)((double)Big<T>::value / kappa);
  if (!std::isfinite((double)a.pad_raw)) a.pad_raw = (T)(Big<T>::value);
  a.band = (T)band;
  a.vec = ((M * sizeof(T)) % 16 == 0) && ((uintptr_t)cost % 16 == 0) &&
          (!pen || (uintptr_t)pen % 16 == 0);
  a.p = p;
  return sdtw_stream_forward<T>(a, has_p, band > 0, st);
}

template <typename T>
static int sdtw_bwd(const T* grad_r, const T* grad_p, int B, int N, int M, double gamma,
                    int has_pen, const void* saved, size_t saved_bytes, T* d_cost, T* d_pen,
                    void* ws, size_t ws_bytes, cudaStream_t st, const uint32_t* mask = nullptr,
                    uint8_t* tf_rows = nullptr, uint8_t* tf_cols = nullptr,
                    uint8_t* nzm = nullptr) {
  g_err[0] = 0;
  if (int e = check_dims("tw_sdtw_backward", B, N, M)) return e;
  if (!(gamma > 0)) return set_error(kInvalid, "tw_sdtw_backward: gamma must be > 0");
  if (B == 0) return kOk;
  const bool has_p = has_pen != 0;
  if (!grad_r || !saved || !d_cost || !ws || (has_p && (!grad_p || !d_pen)))
    return set_error(kInvalid, "tw_sdtw_backward: null pointer argument");
  StreamPlan p = make_stream_plan(B, N, M, sizeof(T), has_p, device_sms());
  const size_t sb = align256(p.saved_elems() * sizeof(T)) * (has_p ? 2 : 1);
  const size_t wb = align256(p.delay_elems() * sizeof(T)) * (has_p ? 2 : 1);
  if (saved_bytes < sb) return set_error(kWorkspace, "tw_sdtw_backward: saved needs %zu bytes", sb);
  if (ws_bytes < wb) return set_error(kWorkspace, "tw_sdtw_backward: workspace needs %zu bytes", wb);
  SdtwArgs<T> a;
  a.sR = const_cast<T*>(static_cast<const T*>(saved));
  a.sP = has_p ? reinterpret_cast<T*>(const_cast<char*>(static_cast<const char*>(saved)) + sb / 2)
               : nullptr;
  a.dlR = static_cast<T*>(ws);
  a.dlP = has_p ? reinterpret_cast<T*>(static_cast<char*>(ws) + wb / 2) : nullptr;
  a.grad_r = grad_r;
  a.grad_p = grad_p;
  a.dC = d_cost;
  a.dQ = d_pen;
  const double kappa = 1.4426950408889634 / gamma;
  a.kappa = (T)kappa;
  a.inv_kappa = (T)(1.0 / kappa);
  a.inv_gamma = (T)(1.0 / gamma);
  a.vec = ((M * sizeof(T)) % 16 == 0) && ((uintptr_t)d_cost % 16 == 0) &&
          (!d_pen || (uintptr_t)d_pen % 16 == 0);
  a.mask = mask;
  a.mask_np = (N + 3) & ~3;
  a.tf_rows = tf_rows;
  a.tf_cols = tf_cols;
  a.nzm = nzm;
  {
    // TW_DP_ALL_BLOCKS=1: no shortcut for blocks whose adjoints are all zero
    const char* env = std::getenv("TW_DP_ALL_BLOCKS");
    a.all_blocks = env != nullptr && env[0] != '\0' && env[0] != '0';
  }
  a.tf_kr = (((M + 31) >> 5) + 15) & ~15;
  a.tf_kc = (((N + 31) >> 5) + 15) & ~15;
  a.p = p;
  return sdtw_stream_backward<T>(a, has_p, false, st);
}

template int sdtw_fwd<float>(const float*, const float*, int, int, int, double, double, float*,
                             float*, void*, size_t, void*, size_t, cudaStream_t);

int tc_take_device_error();
int udtw_cost_f32(const float*, const float*, const float*, const float*, int, int, int, int,
                  double, double, float*, float*, cudaStream_t);
int udtw_cost_f64(const double*, const double*, const double*, const double*, int, int, int, int,
                  double, double, double*, double*, cudaStream_t);
int udtw_grad_f32(const float*, const float*, const float*, const float*, const float*,
                  const float*, const float*, int, int, int, int, double, double, float*, float*,
                  float*, float*, cudaStream_t, const uint8_t* = nullptr,
                  const uint8_t* = nullptr);
int udtw_grad_f64(const double*, const double*, const double*, const double*, const double*,
                  const double*, const double*, int, int, int, int, double, double, double*,
                  double*, double*, double*, cudaStream_t);
int sq_cost_f32(const float*, const float*, int, int, int, int, float*, uint32_t*, cudaStream_t);
int sq_cost_f64(const double*, const double*, int, int, int, int, double*, uint32_t*,
                cudaStream_t);
int sq_grad_f32(const float*, const float*, const uint32_t*, const float*, int, int, int, int,
                float*, float*, cudaStream_t);
int sq_grad_f64(const double*, const double*, const uint32_t*, const double*, int, int, int, int,
                double*, double*, cudaStream_t);
bool sq_grad_flagged_eligible(const float*, const float*, const float*, const float*,
                              const float*, int, int);
int sq_grad_flagged_f32(const float*, const float*, const uint32_t*, const float*, int, int, int,
                        int, float*, float*, const uint8_t*, const uint8_t*, cudaStream_t);

template <typename T>
int jeanie_forward(const T*, int, int, int, int, int, int, int, double, T*, T*, cudaStream_t);
template <typename T>
int jeanie_backward(const T*, const T*, const T*, const T*, int, int, int, int, int, int, int,
                    double, T*, cudaStream_t);
template <typename T>
int qs_cost(const T*, const T*, int, int, int, int, int, T*, cudaStream_t);
template <typename T>
int qs_grad(const T*, const T*, const T*, const T*, int, int, int, int, int, T*, T*, cudaStream_t);
template <typename T>
int qs_rbf_cost(const T*, const T*, int, int, int, int, double, T*, cudaStream_t);
template <typename T>
int qs_rbf_grad(const T*, const T*, const T*, int, int, int, int, double, T*, T*, cudaStream_t);
template <typename T>
int fvm_softmin(const T*, int, int, int, double, T*, cudaStream_t);
template <typename T>
int fvm_softmin_bwd(const T*, const T*, int, int, int, double, T*, cudaStream_t);
int optimal_path(const double*, int, int, int, int, int, int, double*, int*, int*, int*,
                 cudaStream_t);
bool jf_supported(int K, int T, int U, int D, bool fvm, bool feat);
size_t jf_saved_bytes(int B, int K, int T, int U, bool fvm, bool feat);
int jf_run(const float* q, const float* s, const float* cost, int B, int K1, int K2, int T, int U,
           int D, int s1, int s2, int metric, bool fvm, double gamma, bool fwd, float* out,
           float* Rnat, void* saved, size_t saved_bytes, const float* g_out, const float* g_R,
           float* dq, float* ds, float* dC, cudaStream_t st);

static int check_jeanie(const char* who, int B, int K1, int K2, int T, int U, int s1, int s2,
                        double gamma) {
  if (B < 0 || K1 <= 0 || K2 <= 0 || T <= 0 || U <= 0 || s1 < 0 || s2 < 0 || !(gamma > 0))
    return set_error(kInvalid, "%s: invalid arguments (B=%d K1=%d K2=%d T=%d U=%d s=%d,%d)", who,
                     B, K1, K2, T, U, s1, s2);
  return kOk;
}

}  // namespace tw

using namespace tw;

extern "C" {

int tw_version(void) { return 100; }

const char* tw_last_error(void) { return g_err; }

int tw_device_error(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return set_error(kLaunch, "device synchronize failed");
  const int tc_err = tc_take_device_error();
  const int dp_err = dp_take_device_error();
  return tc_err != 0 ? tc_err : dp_err;
}

size_t tw_sdtw_saved_bytes(int B, int N, int M, int dtype_bytes, int has_penalty) {
  if (!dims_ok(B, N, M) || B == 0 || (dtype_bytes != 4 && dtype_bytes != 8)) return 0;
  StreamPlan p = make_stream_plan(B, N, M, dtype_bytes, has_penalty != 0, device_sms());
  return align256(p.saved_elems() * dtype_bytes) * (has_penalty ? 2 : 1);
}

size_t tw_sdtw_workspace_bytes(int B, int N, int M, int dtype_bytes, int has_penalty) {
  if (!dims_ok(B, N, M) || B == 0 || (dtype_bytes != 4 && dtype_bytes != 8)) return 0;
  StreamPlan p = make_stream_plan(B, N, M, dtype_bytes, has_penalty != 0, device_sms());
  return align256(p.delay_elems() * dtype_bytes) * (has_penalty ? 2 : 1);
}

int tw_sdtw_forward_f32(const float* cost, const float* penalty, int B, int N, int M,
                        double gamma, double bandwidth, float* out_r, float* out_p, void* saved,
                        size_t saved_bytes, void* workspace, size_t ws_bytes, void* stream) {
  return sdtw_fwd<float>(cost, penalty, B, N, M, gamma, bandwidth, out_r, out_p, saved,
                         saved_bytes, workspace, ws_bytes, (cudaStream_t)stream);
}
int tw_sdtw_forward_f64(const double* cost, const double* penalty, int B, int N, int M,
                        double gamma, double bandwidth, double* out_r, double* out_p, void* saved,
                        size_t saved_bytes, void* workspace, size_t ws_bytes, void* stream) {
  return sdtw_fwd<double>(cost, penalty, B, N, M, gamma, bandwidth, out_r, out_p, saved,
                          saved_bytes, workspace, ws_bytes, (cudaStream_t)stream);
}

int tw_sdtw_backward_f32(const float* grad_r, const float* grad_p, int B, int N, int M,
                         double gamma, int has_penalty, const void* saved, size_t saved_bytes,
                         float* d_cost, float* d_penalty, void* workspace, size_t ws_bytes,
                         void* stream) {
  return sdtw_bwd<float>(grad_r, grad_p, B, N, M, gamma, has_penalty, saved, saved_bytes, d_cost,
                         d_penalty, workspace, ws_bytes, (cudaStream_t)stream);
}
int tw_sdtw_backward_f64(const double* grad_r, const double* grad_p, int B, int N, int M,
                         double gamma, int has_penalty, const void* saved, size_t saved_bytes,
                         double* d_cost, double* d_penalty, void* workspace, size_t ws_bytes,
                         void* stream) {
  return sdtw_bwd<double>(grad_r, grad_p, B, N, M, gamma, has_penalty, saved, saved_bytes,
                          d_cost, d_penalty, workspace, ws_bytes, (cudaStream_t)stream);
}

int tw_sdtw_backward_masked_f32(const float* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                float* d_cost, void* workspace, size_t ws_bytes, void* stream) {
  if (B > 0 && mask == nullptr) return set_error(kInvalid, "tw_sdtw_backward_masked: null mask");
  return sdtw_bwd<float>(grad_r, nullptr, B, N, M, gamma, 0, saved, saved_bytes, d_cost, nullptr,
                         workspace, ws_bytes, (cudaStream_t)stream, mask);
}
int tw_sdtw_backward_masked_f64(const double* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                double* d_cost, void* workspace, size_t ws_bytes, void* stream) {
  if (B > 0 && mask == nullptr) return set_error(kInvalid, "tw_sdtw_backward_masked: null mask");
  return sdtw_bwd<double>(grad_r, nullptr, B, N, M, gamma, 0, saved, saved_bytes, d_cost, nullptr,
                          workspace, ws_bytes, (cudaStream_t)stream, mask);
}

// Nonzero-chunk flags of dL/dcost (fp32): rows part [B][ceil(N/128)][KR],
// then the cols part [B][ceil(M/128)][KC], each 256-byte aligned;
// KR = 16 ceil(ceil(M/32)/16), KC = 16 ceil(ceil(N/32)/16).
struct FlagLayout {
  size_t rows, cols;
};
static FlagLayout flag_layout(int B, int N, int M) {
  FlagLayout f;
  f.rows = align256((size_t)B * ((N + 127) / 128) * ((((M + 31) >> 5) + 15) & ~15));
  f.cols = align256((size_t)B * ((M + 127) / 128) * ((((N + 31) >> 5) + 15) & ~15));
  return f;
}

size_t tw_sdtw_chunk_flags_bytes(int B, int N, int M) {
  if (!dims_ok(B, N, M) || B == 0) return 0;
  const FlagLayout f = flag_layout(B, N, M);
  return f.rows + f.cols;
}

int tw_sdtw_backward_masked_flags_f32(const float* grad_r, int B, int N, int M, double gamma,
                                      const void* saved, size_t saved_bytes,
                                      const uint32_t* mask, float* d_cost, uint8_t* flags,
                                      size_t flags_bytes, void* workspace, size_t ws_bytes,
                                      void* stream) {
  if (B > 0 && mask == nullptr) return set_error(kInvalid, "tw_sdtw_backward_masked: null mask");
  uint8_t* rows = nullptr;
  uint8_t* cols = nullptr;
  if (B > 0 && dims_ok(B, N, M) && flags != nullptr) {
    const FlagLayout f = flag_layout(B, N, M);
    if (flags_bytes < f.rows + f.cols)
      return set_error(kWorkspace, "tw_sdtw_backward_masked_flags: flags need %zu bytes",
                       f.rows + f.cols);
    const cudaError_t e = cudaMemsetAsync(flags, 0, f.rows + f.cols, (cudaStream_t)stream);
    if (e != cudaSuccess)
      return set_error(kLaunch, "tw_sdtw_backward_masked_flags: %s", cudaGetErrorString(e));
    rows = flags;
    cols = flags + f.rows;
  }
  return sdtw_bwd<float>(grad_r, nullptr, B, N, M, gamma, 0, saved, saved_bytes, d_cost, nullptr,
                         workspace, ws_bytes, (cudaStream_t)stream, mask, rows, cols);
}

// TW_GRAD_DENSE=1 makes the chain rule read every chunk of dL/dcost (for
// comparisons); by default it skips the chunks the DP backward flagged zero.
static bool grad_dense() {
  const char* env = std::getenv("TW_GRAD_DENSE");
  return env != nullptr && env[0] != '\0' && env[0] != '0';
}

int tw_sqeuclid_grad_flagged_f32(const float* X, const float* Y, const float* d_cost,
                                 const uint8_t* flags, int B, int N, int M, int D, float* dX,
                                 float* dY, void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || (B && (!X || !Y || !d_cost || !dX || !dY)))
    return set_error(kInvalid, "tw_sqeuclid_grad_flagged: invalid arguments");
  const uint8_t* rows = nullptr;
  const uint8_t* cols = nullptr;
  if (B > 0 && flags != nullptr && !grad_dense()) {
    rows = flags;
    cols = flags + flag_layout(B, N, M).rows;
  }
  return sq_grad_flagged_f32(X, Y, nullptr, d_cost, B, N, M, D, dX, dY, rows, cols,
                             (cudaStream_t)stream);
}

int tw_sdtw_backward_flags_f32(const float* grad_r, const float* grad_p, int B, int N, int M,
                               double gamma, int has_penalty, const void* saved,
                               size_t saved_bytes, float* d_cost, float* d_penalty,
                               uint8_t* flags, size_t flags_bytes, void* workspace,
                               size_t ws_bytes, void* stream) {
  uint8_t* rows = nullptr;
  uint8_t* cols = nullptr;
  if (B > 0 && dims_ok(B, N, M) && flags != nullptr) {
    const FlagLayout f = flag_layout(B, N, M);
    if (flags_bytes < f.rows + f.cols)
      return set_error(kWorkspace, "tw_sdtw_backward_flags: flags need %zu bytes",
                       f.rows + f.cols);
    const cudaError_t e = cudaMemsetAsync(flags, 0, f.rows + f.cols, (cudaStream_t)stream);
    if (e != cudaSuccess)
      return set_error(kLaunch, "tw_sdtw_backward_flags: %s", cudaGetErrorString(e));
    rows = flags;
    cols = flags + f.rows;
  }
  return sdtw_bwd<float>(grad_r, grad_p, B, N, M, gamma, has_penalty, saved, saved_bytes, d_cost,
                         d_penalty, workspace, ws_bytes, (cudaStream_t)stream, nullptr, rows,
                         cols);
}

int tw_udtw_features_grad_flagged_f32(const float* X, const float* Y, const float* vx,
                                      const float* vy, const float* cost, const float* d_cost,
                                      const float* d_penalty, const uint8_t* flags, int B, int N,
                                      int M, int D, double beta, double eps, float* dX, float* dY,
                                      float* dvx, float* dvy, void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || !X || !Y || !cost || !d_cost || !dX || !dY ||
      ((vx == nullptr) != (vy == nullptr)))
    return set_error(kInvalid, "tw_udtw_features_grad_flagged: invalid arguments");
  const uint8_t* rows = nullptr;
  const uint8_t* cols = nullptr;
  if (B > 0 && flags != nullptr && !grad_dense()) {
    rows = flags;
    cols = flags + flag_layout(B, N, M).rows;
  }
  return udtw_grad_f32(X, Y, vx, vy, cost, d_cost, d_penalty, B, N, M, D, beta, eps, dX, dY, dvx,
                       dvy, (cudaStream_t)stream, rows, cols);
}

size_t tw_sdtw_nonzero_mask_bytes(int B, int N, int M) {
  if (!dims_ok(B, N, M) || B == 0) return 0;
  return (size_t)B * ((M + 31) / 32) * ((N + 3) & ~3) * 4;
}

int tw_sdtw_backward_sparse_f32(const float* grad_r, int B, int N, int M, double gamma,
                                const void* saved, size_t saved_bytes, const uint32_t* mask,
                                float* d_cost, uint32_t* nz_mask, uint8_t* flags,
                                size_t flags_bytes, void* workspace, size_t ws_bytes,
                                void* stream) {
  g_err[0] = 0;
  if (int e = check_dims("tw_sdtw_backward_sparse", B, N, M)) return e;
  if (B == 0) return kOk;
  if (!mask || !nz_mask || !flags)
    return set_error(kInvalid, "tw_sdtw_backward_sparse: null mask, nz_mask or flags");
  const FlagLayout f = flag_layout(B, N, M);
  if (flags_bytes < f.rows + f.cols)
    return set_error(kWorkspace, "tw_sdtw_backward_sparse: flags need %zu bytes", f.rows + f.cols);
  cudaError_t e = cudaMemsetAsync(flags, 0, f.rows + f.cols, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(nz_mask, 0, tw_sdtw_nonzero_mask_bytes(B, N, M), (cudaStream_t)stream);
  if (e != cudaSuccess)
    return set_error(kLaunch, "tw_sdtw_backward_sparse: %s", cudaGetErrorString(e));
  return sdtw_bwd<float>(grad_r, nullptr, B, N, M, gamma, 0, saved, saved_bytes, d_cost, nullptr,
                         workspace, ws_bytes, (cudaStream_t)stream, mask, flags, flags + f.rows,
                         reinterpret_cast<uint8_t*>(nz_mask));
}

int tw_sqeuclid_grad_sparse_f32(const float* X, const float* Y, const uint32_t* nz_mask,
                                const float* d_cost, const uint8_t* flags, int B, int N, int M,
                                int D, float* dX, float* dY, void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 ||
      (B && (!X || !Y || !nz_mask || !d_cost || !flags || !dX || !dY)))
    return set_error(kInvalid, "tw_sqeuclid_grad_sparse: invalid arguments");
  const uint8_t* rows = nullptr;
  const uint8_t* cols = nullptr;
  if (B > 0 && !grad_dense()) {
    rows = flags;
    cols = flags + flag_layout(B, N, M).rows;
  }
  return sq_grad_flagged_f32(X, Y, nz_mask, d_cost, B, N, M, D, dX, dY, rows, cols,
                             (cudaStream_t)stream);
}

// Workspace of tw_sdtw_features_backward_*: dL/dcost, the DP's delay lines
// and (fp32) the chunk flags.
struct FeatWs {
  size_t dc, dp, fl, nz;
  size_t total() const { return dc + dp + fl + nz; }
};
static FeatWs feat_ws(int B, int N, int M, int dtype_bytes) {
  FeatWs w{0, 0, 0, 0};
  if (!dims_ok(B, N, M) || B == 0 || (dtype_bytes != 4 && dtype_bytes != 8)) return w;
  w.dc = align256((size_t)B * N * M * dtype_bytes);
  w.dp = tw_sdtw_workspace_bytes(B, N, M, dtype_bytes, 0);
  if (dtype_bytes == 4) {
    w.fl = tw_sdtw_chunk_flags_bytes(B, N, M);
    w.nz = align256(tw_sdtw_nonzero_mask_bytes(B, N, M));
  }
  return w;
}

size_t tw_sdtw_features_workspace_bytes(int B, int N, int M, int dtype_bytes) {
  return feat_ws(B, N, M, dtype_bytes).total();
}

}  // extern "C"

template <typename T>
static int sdtw_feat_bwd(const T* X, const T* Y, const uint32_t* mask, const T* grad_r, int B,
                         int N, int M, int D, double gamma, const void* saved, size_t saved_bytes,
                         T* dX, T* dY, void* ws, size_t ws_bytes, cudaStream_t st) {
  g_err[0] = 0;
  if (int e = check_dims("tw_sdtw_features_backward", B, N, M)) return e;
  if (D <= 0) return set_error(kInvalid, "tw_sdtw_features_backward: D must be > 0");
  if (B == 0) return kOk;
  if (!X || !Y || !mask || !dX || !dY || !ws)
    return set_error(kInvalid, "tw_sdtw_features_backward: null pointer argument");
  const FeatWs w = feat_ws(B, N, M, (int)sizeof(T));
  if (ws_bytes < w.total())
    return set_error(kWorkspace, "tw_sdtw_features_backward: workspace needs %zu bytes", w.total());
  char* base = static_cast<char*>(ws);
  T* dC = reinterpret_cast<T*>(base);
  void* dpws = base + w.dc;
  if constexpr (sizeof(T) == 4) {
    uint8_t* flags = reinterpret_cast<uint8_t*>(base + w.dc + w.dp);
    uint32_t* nzm = reinterpret_cast<uint32_t*>(base + w.dc + w.dp + w.fl);
    if (int rc = tw_sdtw_backward_sparse_f32(grad_r, B, N, M, gamma, saved, saved_bytes, mask, dC,
                                             nzm, flags, w.fl, dpws, w.dp, st))
      return rc;
    return tw_sqeuclid_grad_sparse_f32(X, Y, nzm, dC, flags, B, N, M, D, dX, dY, st);
  } else {
    if (int rc = sdtw_bwd<T>(grad_r, nullptr, B, N, M, gamma, 0, saved, saved_bytes, dC, nullptr,
                             dpws, w.dp, st, mask))
      return rc;
    return sq_grad_f64(X, Y, nullptr, dC, B, N, M, D, dX, dY, st);
  }
}

extern "C" {

int tw_sdtw_features_backward_f32(const float* X, const float* Y, const uint32_t* mask,
                                  const float* grad_r, int B, int N, int M, int D, double gamma,
                                  const void* saved, size_t saved_bytes, float* dX, float* dY,
                                  void* workspace, size_t ws_bytes, void* stream) {
  return sdtw_feat_bwd<float>(X, Y, mask, grad_r, B, N, M, D, gamma, saved, saved_bytes, dX, dY,
                              workspace, ws_bytes, (cudaStream_t)stream);
}
int tw_sdtw_features_backward_f64(const double* X, const double* Y, const uint32_t* mask,
                                  const double* grad_r, int B, int N, int M, int D, double gamma,
                                  const void* saved, size_t saved_bytes, double* dX, double* dY,
                                  void* workspace, size_t ws_bytes, void* stream) {
  return sdtw_feat_bwd<double>(X, Y, mask, grad_r, B, N, M, D, gamma, saved, saved_bytes, dX, dY,
                               workspace, ws_bytes, (cudaStream_t)stream);
}

int tw_udtw_cost_f32(const float* X, const float* Y, const float* vx, const float* vy, int B,
                     int N, int M, int D, double beta, double eps, float* cost, float* penalty,
                     void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || !X || !Y || !cost || ((vx == nullptr) != (vy == nullptr)))
    return set_error(kInvalid, "tw_udtw_cost: invalid arguments");
  return udtw_cost_f32(X, Y, vx, vy, B, N, M, D, beta, eps, cost, penalty, (cudaStream_t)stream);
}
int tw_udtw_cost_f64(const double* X, const double* Y, const double* vx, const double* vy, int B,
                     int N, int M, int D, double beta, double eps, double* cost, double* penalty,
                     void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || !X || !Y || !cost || ((vx == nullptr) != (vy == nullptr)))
    return set_error(kInvalid, "tw_udtw_cost: invalid arguments");
  return udtw_cost_f64(X, Y, vx, vy, B, N, M, D, beta, eps, cost, penalty, (cudaStream_t)stream);
}

int tw_udtw_features_grad_f32(const float* X, const float* Y, const float* vx, const float* vy,
                              const float* cost, const float* d_cost, const float* d_penalty,
                              int B, int N, int M, int D, double beta, double eps, float* dX,
                              float* dY, float* dvx, float* dvy, void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || !X || !Y || !cost || !d_cost || !dX || !dY ||
      ((vx == nullptr) != (vy == nullptr)))
    return set_error(kInvalid, "tw_udtw_features_grad: invalid arguments");
  return udtw_grad_f32(X, Y, vx, vy, cost, d_cost, d_penalty, B, N, M, D, beta, eps, dX, dY, dvx,
                       dvy, (cudaStream_t)stream);
}
#define TW_SQ_ENTRIES(SUF, T)                                                                    \
  int tw_sqeuclid_cost_##SUF(const T* X, const T* Y, int B, int N, int M, int D, T* cost,       \
                             uint32_t* mask, void* stream) {                                     \
    g_err[0] = 0;                                                                               \
    if (B < 0 || N <= 0 || M <= 0 || D <= 0 || (B && (!X || !Y || !cost || !mask)))             \
      return set_error(kInvalid, "tw_sqeuclid_cost: invalid arguments");                        \
    return sq_cost_##SUF(X, Y, B, N, M, D, cost, mask, (cudaStream_t)stream);                   \
  }                                                                                             \
  int tw_sqeuclid_grad_##SUF(const T* X, const T* Y, const uint32_t* mask, const T* d_cost,     \
                             int B, int N, int M, int D, T* dX, T* dY, void* stream) {          \
    g_err[0] = 0;                                                                               \
    if (B < 0 || N <= 0 || M <= 0 || D <= 0 ||                                                  \
        (B && (!X || !Y || !d_cost || !dX || !dY)))                                             \
      return set_error(kInvalid, "tw_sqeuclid_grad: invalid arguments");                        \
    return sq_grad_##SUF(X, Y, mask, d_cost, B, N, M, D, dX, dY, (cudaStream_t)stream);         \
  }

TW_SQ_ENTRIES(f32, float)
TW_SQ_ENTRIES(f64, double)

int tw_udtw_features_grad_f64(const double* X, const double* Y, const double* vx,
                              const double* vy, const double* cost, const double* d_cost,
                              const double* d_penalty, int B, int N, int M, int D, double beta,
                              double eps, double* dX, double* dY, double* dvx, double* dvy,
                              void* stream) {
  g_err[0] = 0;
  if (B < 0 || N <= 0 || M <= 0 || D <= 0 || !X || !Y || !cost || !d_cost || !dX || !dY ||
      ((vx == nullptr) != (vy == nullptr)))
    return set_error(kInvalid, "tw_udtw_features_grad: invalid arguments");
  return udtw_grad_f64(X, Y, vx, vy, cost, d_cost, d_penalty, B, N, M, D, beta, eps, dX, dY, dvx,
                       dvy, (cudaStream_t)stream);
}


#define TW_JEANIE_ENTRIES(SUF, T)                                                                \
  int tw_jeanie_forward_##SUF(const T* cost, int B, int K1, int K2, int Tn, int U, int s1,      \
                              int s2, double gamma, T* out, T* R, void* stream) {               \
    g_err[0] = 0;                                                                               \
    if (int e = check_jeanie("tw_jeanie_forward", B, K1, K2, Tn, U, s1, s2, gamma)) return e;   \
    if (B && (!cost || !out || !R)) return set_error(kInvalid, "tw_jeanie_forward: null pointer"); \
    return jeanie_forward<T>(cost, B, K1, K2, Tn, U, s1, s2, gamma, out, R,                    \
                             (cudaStream_t)stream);                                              \
  }                                                                                             \
  int tw_jeanie_backward_##SUF(const T* cost, const T* R, const T* grad_out, const T* grad_R,   \
                               int B, int K1, int K2, int Tn, int U, int s1, int s2,            \
                               double gamma, T* d_cost, void* stream) {                         \
    g_err[0] = 0;                                                                               \
    if (int e = check_jeanie("tw_jeanie_backward", B, K1, K2, Tn, U, s1, s2, gamma)) return e;  \
    if (B && (!cost || !R || !grad_out || !d_cost))                                              \
      return set_error(kInvalid, "tw_jeanie_backward: null pointer");                          \
    return jeanie_backward<T>(cost, R, grad_out, grad_R, B, K1, K2, Tn, U, s1, s2, gamma, d_cost, \
                              (cudaStream_t)stream);                                             \
  }                                                                                             \
  int tw_qs_cost_##SUF(const T* query, const T* support, int B, int R, int U, int D,           \
                       int metric, T* cost, void* stream) {                                     \
    g_err[0] = 0;                                                                               \
    if (B < 0 || R <= 0 || U <= 0 || D <= 0 || (metric != 0 && metric != 1))                  \
      return set_error(kInvalid, "tw_qs_cost: invalid arguments");                             \
    if (B && (!query || !support || !cost)) return set_error(kInvalid, "tw_qs_cost: null pointer"); \
    return qs_cost<T>(query, support, B, R, U, D, metric, cost, (cudaStream_t)stream);         \
  }                                                                                             \
  int tw_qs_cost_grad_##SUF(const T* query, const T* support, const T* cost, const T* d_cost,  \
                            int B, int R, int U, int D, int metric, T* d_query, T* d_support,   \
                            void* stream) {                                                     \
    g_err[0] = 0;                                                                               \
    if (B < 0 || R <= 0 || U <= 0 || D <= 0 || (metric != 0 && metric != 1))                  \
      return set_error(kInvalid, "tw_qs_cost_grad: invalid arguments");                        \
    if (B && (!query || !support || !cost || !d_cost || !d_query || !d_support))              \
      return set_error(kInvalid, "tw_qs_cost_grad: null pointer");                             \
    return qs_grad<T>(query, support, cost, d_cost, B, R, U, D, metric, d_query, d_support,    \
                      (cudaStream_t)stream);                                                     \
  }                                                                                             \
  int tw_qs_rbf_cost_##SUF(const T* query, const T* support, int B, int R, int U, int D,       \
                           double sigma, T* cost, void* stream) {                               \
    g_err[0] = 0;                                                                               \
    if (B < 0 || R <= 0 || U <= 0 || D <= 0 || !(sigma > 0))                                   \
      return set_error(kInvalid, "tw_qs_rbf_cost: invalid arguments");                         \
    if (B && (!query || !support || !cost))                                                     \
      return set_error(kInvalid, "tw_qs_rbf_cost: null pointer");                              \
    return qs_rbf_cost<T>(query, support, B, R, U, D, sigma, cost, (cudaStream_t)stream);      \
  }                                                                                             \
  int tw_qs_rbf_cost_grad_##SUF(const T* query, const T* support, const T* d_cost, int B,      \
                                int R, int U, int D, double sigma, T* d_query, T* d_support,    \
                                void* stream) {                                                 \
    g_err[0] = 0;                                                                               \
    if (B < 0 || R <= 0 || U <= 0 || D <= 0 || !(sigma > 0))                                   \
      return set_error(kInvalid, "tw_qs_rbf_cost_grad: invalid arguments");                    \
    if (B && (!query || !support || !d_cost || !d_query || !d_support))                        \
      return set_error(kInvalid, "tw_qs_rbf_cost_grad: null pointer");                         \
    return qs_rbf_grad<T>(query, support, d_cost, B, R, U, D, sigma, d_query, d_support,       \
                          (cudaStream_t)stream);                                                 \
  }                                                                                             \
  int tw_fvm_softmin_##SUF(const T* cost, int B, int Kf, int TU, double gamma, T* temporal,    \
                           void* stream) {                                                      \
    g_err[0] = 0;                                                                               \
    if (B < 0 || Kf <= 0 || TU <= 0 || !(gamma > 0))                                           \
      return set_error(kInvalid, "tw_fvm_softmin: invalid arguments");                         \
    return fvm_softmin<T>(cost, B, Kf, TU, gamma, temporal, (cudaStream_t)stream);             \
  }                                                                                             \
  int tw_fvm_softmin_backward_##SUF(const T* cost, const T* d_temporal, int B, int Kf, int TU, \
                                    double gamma, T* d_cost, void* stream) {                    \
    g_err[0] = 0;                                                                               \
    if (B < 0 || Kf <= 0 || TU <= 0 || !(gamma > 0))                                           \
      return set_error(kInvalid, "tw_fvm_softmin_backward: invalid arguments");                \
    return fvm_softmin_bwd<T>(cost, d_temporal, B, Kf, TU, gamma, d_cost, (cudaStream_t)stream); \
  }

TW_JEANIE_ENTRIES(f32, float)
TW_JEANIE_ENTRIES(f64, double)
#undef TW_JEANIE_ENTRIES

int tw_jeanie_fused_supported(int K, int T, int U, int D, int fvm, int features) {
  return jf_supported(K, T, U, D, fvm != 0, features != 0) ? 1 : 0;
}

size_t tw_jeanie_fused_saved_bytes(int B, int K, int T, int U, int fvm, int features) {
  if (B < 0 || K <= 0 || T <= 0 || U <= 0) return 0;
  return jf_saved_bytes(B, K, T, U, fvm != 0, features != 0);
}

static int check_fused(const char* who, const float* query, const float* support,
                       const float* cost, int B, int K1, int K2, int T, int U, int D, int s1,
                       int s2, int metric, int fvm, double gamma) {
  if (B < 0 || K1 <= 0 || K2 <= 0 || T <= 0 || U <= 0 || s1 < 0 || s2 < 0 || !(gamma > 0) ||
      (metric != 0 && metric != 1) || (fvm && K2 != 1))
    return set_error(kInvalid, "%s: invalid arguments (B=%d K1=%d K2=%d T=%d U=%d D=%d)", who, B,
                     K1, K2, T, U, D);
  const bool feat = query != nullptr;
  if (B && (feat ? (support == nullptr || cost != nullptr || D <= 0) : cost == nullptr))
    return set_error(kInvalid, "%s: pass query and support (and no cost), or a cost", who);
  return kOk;
}

int tw_jeanie_fused_forward_f32(const float* query, const float* support, const float* cost,
                                int B, int K1, int K2, int T, int U, int D, int s1, int s2,
                                int metric, int fvm, double gamma, float* out, float* R,
                                void* saved, size_t saved_bytes, void* stream) {
  g_err[0] = 0;
  if (int e = check_fused("tw_jeanie_fused_forward", query, support, cost, B, K1, K2, T, U, D, s1,
                          s2, metric, fvm, gamma))
    return e;
  if (B && (!out || !saved)) return set_error(kInvalid, "tw_jeanie_fused_forward: null pointer");
  return jf_run(query, support, cost, B, K1, K2, T, U, D, s1, s2, metric, fvm != 0, gamma, true,
                out, fvm ? nullptr : R, saved, saved_bytes, nullptr, nullptr, nullptr, nullptr,
                nullptr, (cudaStream_t)stream);
}

int tw_jeanie_fused_backward_f32(const float* query, const float* support, const float* cost,
                                 const float* grad_out, const float* grad_R, int B, int K1, int K2,
                                 int T, int U, int D, int s1, int s2, int metric, int fvm,
                                 double gamma, const void* saved, size_t saved_bytes,
                                 float* d_query, float* d_support, float* d_cost, void* stream) {
  g_err[0] = 0;
  if (int e = check_fused("tw_jeanie_fused_backward", query, support, cost, B, K1, K2, T, U, D,
                          s1, s2, metric, fvm, gamma))
    return e;
  const bool feat = query != nullptr;
  if (B && (!grad_out || !saved || (feat ? (!d_query || !d_support) : !d_cost)))
    return set_error(kInvalid, "tw_jeanie_fused_backward: null pointer");
  if (fvm && grad_R != nullptr)
    return set_error(kInvalid, "tw_jeanie_fused_backward: FVM has no accumulator gradient");
  return jf_run(query, support, cost, B, K1, K2, T, U, D, s1, s2, metric, fvm != 0, gamma, false,
                nullptr, nullptr, const_cast<void*>(saved), saved_bytes, grad_out, grad_R,
                d_query, d_support, d_cost, (cudaStream_t)stream);
}

int tw_optimal_path_f64(const double* cost, int B, int K, int T, int U, int max_shift,
                        int start_view, double* r_ws, int* back_ws, int* path, int* length,
                        void* stream) {
  g_err[0] = 0;
  if (B < 0 || K <= 0 || T <= 0 || U <= 0 || max_shift < 0 || start_view >= K)
    return set_error(kInvalid, "tw_optimal_path: invalid arguments");
  if (B && (!cost || !r_ws || !back_ws || !path || !length))
    return set_error(kInvalid, "tw_optimal_path: null pointer");
  return optimal_path(cost, B, K, T, U, max_shift, start_view, r_ws, back_ws, path, length,
                      (cudaStream_t)stream);
}

}  // extern "C"
