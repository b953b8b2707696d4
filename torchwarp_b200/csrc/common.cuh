// Shared device/host helpers for the torchwarp_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#ifndef __CUDA_ARCH__
#define TW_HOST_ONLY 1
#endif

namespace tw {

// Status codes shared with include/torchwarp_b200.h.
enum Status : int {
  kOk = 0,
  kInvalid = 1,       // bad argument (null pointer, negative size, ...)
  kUnsupported = 2,   // a shape or dtype this build does not handle
  kLaunch = 3,        // a CUDA launch or runtime call failed
  kTimeout = 4,       // a bounded device-side wait gave up
  kWorkspace = 5,     // caller-provided workspace too small
};

// Sets the thread-local message returned by tw_last_error().
int set_error(int code, const char* fmt, ...);

// Unreachable-cell sentinel of the soft-min dynamic programs, in the scaled
// (log2) domain.  A finite sentinel keeps every difference of two
// sentinels finite, so no inf - inf ever reaches exp2 or the adjoint sweep.
template <typename T> struct Big;
template <> struct Big<float> { static constexpr float value = 1e30f; };
template <> struct Big<double> { static constexpr double value = 1e300; };

// exp2 / log2 / reciprocal.  float uses the MUFU instructions directly
// (PTX ex2.approx / lg2.approx / rcp.approx: relative error around 2^-22);
// double calls CUDA's exp2 / log2 and an IEEE division.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ double ex2(double x) { return exp2(x); }
__device__ __forceinline__ double lg2(double x) { return log2(x); }
__device__ __forceinline__ double rcp(double x) { return 1.0 / x; }

// Round-to-nearest adds/multiplies that the compiler may not contract into
// FMAs, so the forward sweep and its replay in the backward sweep produce
// identical bits.
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }

template <typename T>
__device__ __forceinline__ T shfl(T v, int src) {
  return __shfl_sync(0xffffffffu, v, src);
}
template <typename T>
__device__ __forceinline__ T shfl_up1_rot(T v) {  // lane l reads lane (l-1) mod 32
  return __shfl_sync(0xffffffffu, v, (threadIdx.x + 31) & 31);
}
template <typename T>
__device__ __forceinline__ T shfl_dn1_rot(T v) {  // lane l reads lane (l+1) mod 32
  return __shfl_sync(0xffffffffu, v, (threadIdx.x + 1) & 31);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// cp.async of 16 bytes (src_bytes valid, rest zero-filled), L2-only.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)),
               "l"(src), "r"(src_bytes));
}
// cp.async of one 4- or 8-byte element (zero-filled when src_bytes == 0).
template <int BYTES>
__device__ __forceinline__ void cp_async_elem(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;\n" ::"r"(smem_u32(dst)),
               "l"(src), "n"(BYTES), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

}  // namespace tw
