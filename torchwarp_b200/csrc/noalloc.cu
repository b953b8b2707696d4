// Allocation-free variant of the soft-DTW / uDTW forward DP.
//
// Some callers own every device allocation themselves and hand a library
// only their input and output buffers: plugin hosts and serving runtimes
// that budget device memory up front, or run with no allocator they can
// lend.  They can pass the cost, the outputs and the saved state, but not
// the forward's scratch (the per-warp delay lines that carry one band's
// bottom row to the next band).  tw_sdtw_forward_noalloc_f32 takes its
// scratch from the static array below instead, so it never allocates.
//
// The array is a fixed kStaticScratchBytes (4 MiB) in every GPU's memory
// for as long as the library stays loaded.  All calls share it, so calls
// that overlap on the GPU (several streams, several host threads) race and
// must be serialised by the caller.  The kernel writes every scratch word
// before it reads it, so the contents left by an earlier call never matter
// and nothing is cleared.
#include <cuda_runtime.h>

#include "../../include/torchwarp_b200.h"
#include "common.cuh"

namespace tw {

template <typename T>
int sdtw_fwd(const T* cost, const T* pen, int B, int N, int M, double gamma, double band,
             T* out_r, T* out_p, void* saved, size_t saved_bytes, void* ws, size_t ws_bytes,
             cudaStream_t st);

namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_sdtw_scratch[kStaticScratchBytes];

// Device address of g_sdtw_scratch on the current device.  In host code the
// symbol's name is only a host-side handle, so the address is looked up with
// the caller's device current.  The lookup runs on every call and is not
// cached: it is not a stream operation and costs little, and a cached address
// would go stale if the caller reset the device (cudaDeviceReset) or its
// primary context was torn down and created again, which can place the
// module's globals elsewhere.  The first lookup on a device loads the module
// there (lazy loading), which is why the first call should come before any
// stream capture.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess)
    return set_error(kLaunch, "tw_sdtw_forward_noalloc_f32: no current CUDA device");
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_sdtw_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(kLaunch, "tw_sdtw_forward_noalloc_f32: cudaGetSymbolAddress failed: %s",
                     cudaGetErrorString(e));
  *out = p;
  return kOk;
}

}  // namespace
}  // namespace tw

extern "C" int tw_sdtw_forward_noalloc_f32(const float* cost, const float* penalty, int B, int N,
                                           int M, double gamma, double bandwidth, float* out_r,
                                           float* out_p, void* saved, size_t saved_bytes,
                                           void* stream) {
  using namespace tw;
  if (B > 0 && N > 0 && M > 0) {
    const size_t need = tw_sdtw_workspace_bytes(B, N, M, 4, penalty != nullptr);
    if (need > kStaticScratchBytes)
      return set_error(kWorkspace,
                       "tw_sdtw_forward_noalloc_f32: this shape needs %zu bytes of scratch, "
                       "more than the %zu-byte static buffer; use tw_sdtw_forward_f32 with a "
                       "caller-provided workspace",
                       need, kStaticScratchBytes);
  }
  void* ws = nullptr;
  if (int e = scratch_address(&ws)) return e;
  return sdtw_fwd<float>(cost, penalty, B, N, M, gamma, bandwidth, out_r, out_p, saved,
                         saved_bytes, ws, kStaticScratchBytes, (cudaStream_t)stream);
}
