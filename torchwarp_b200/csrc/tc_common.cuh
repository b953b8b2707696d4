// Blackwell (sm_100a) building blocks for the tensor-core contractions:
// mbarriers with bounded waits, TMA tensor-map copies (no cluster
// broadcast: every CTA fetches its own tiles), tcgen05 MMA / TMEM access,
// UMMA shared-memory and instruction descriptors, and the 3xTF32 split.
//
// Operand tiles live in shared memory in the 128-byte swizzled layout that a
// TMA box of 32 fp32 (128 B) per line produces: line r of a box sits at
// r * 128 B and its 16-byte chunk c at chunk c ^ (r % 8).  Such a box is a
// K-major UMMA operand when a line holds 32 consecutive K values (8-line
// groups 1024 B apart, SBO = 1024) and an MN-major operand when a line holds
// 32 consecutive M/N values of one K index (32-wide MN atoms LBO apart).
#pragma once

#include <cuda.h>
#include <cstdint>

#include "common.cuh"

namespace tw {
namespace tc {

// Spin limit of every mbarrier wait.  A correct pipeline never comes close;
// a wait that runs out sets the kernel's error word and the caller unwinds.
constexpr unsigned kSpinLimit = 1u << 26;

// ------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of the given parity to complete; false if the spin
// limit ran out or another role already gave up (*abort set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, volatile int* abort) {
  for (unsigned n = 0; n < kSpinLimit; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 1023u) == 1023u && *abort) return false;
  }
  *abort = 1;
  return false;
}

// ------------------------------------------------------------------ TMA

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Plain bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on an mbarrier like the tensor loads.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes become visible to the async proxy
// (TMA stores, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also returns the OR of `pred` over the participating
// threads, so a group of warps takes one decision (e.g. to stop) together.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
  unsigned r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((unsigned)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, unsigned cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, unsigned cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], kind::tf32, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::tf32: A's M rows in TMEM lanes, its
// K values in consecutive columns starting at a_tmem.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes, one lane per
// thread; tmem_st_wait() makes the stores complete before they are signalled.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// The mbarrier completes one arrival once every tcgen05 op this thread issued
// before has finished (operand reads included).
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes, one lane per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// --------------------------------------------------------- descriptors

// Shared-memory matrix descriptor.  lbo/sbo in bytes.  K-major operands use
// the 128-byte swizzle with 16-byte granules (layout 2: SBO = 1024, the
// stride of 8-line groups; LBO unused).  MN-major 32-bit (TF32) operands
// must use the 128-byte swizzle with 32-byte granules (layout 1): a line of
// 128 B holds 32 M/N values of one K index, its granule g sits at
// g ^ (line % 4); LBO = stride between 32-wide M/N atoms, SBO = stride
// between 4-line K groups.
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Base32 = 1;

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  d |= (uint64_t)layout << 61;
  return d;
}

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return smem_desc(saddr, lbo, sbo, kLayoutSW128);
}

// Instruction descriptor: tf32 x tf32 -> fp32, M x N tile, operand majors
// (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------- 3xTF32

// x = hi + lo exactly, hi with the 13 low mantissa bits cleared (a TF32
// value whatever rounding the tensor core applies to its inputs); the three
// products hi*hi + hi*lo + lo*hi carry the fp32 product to ~2^-22.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// Byte offset of the 16-byte chunk `c` of line `r` in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c) {
  return (uint32_t)r * 128u + (uint32_t)((c ^ (r & 7)) << 4);
}

// Byte offset of fp32 element `w` (0..31) of line `r` in a box loaded with
// the 128-byte / 32-byte-granule swizzle.
__device__ __forceinline__ uint32_t sw128b32_elem(int r, int w) {
  return (uint32_t)r * 128u + (uint32_t)((((w >> 3) ^ (r & 3)) << 5) + ((w & 7) << 2));
}

}  // namespace tc

// Host side: 3-D fp32 tensor map over a [dim2][dim1][dim0] row-major array
// (dim0 contiguous) with a box of box0 x box1 x 1 and the 128-byte swizzle
// (16-byte granules, or 32-byte granules when `granule32`, the layout of
// MN-major TF32 operands).  Returns kOk, or kUnsupported with tw_last_error
// set when the driver rejects the layout (alignment, strides).
int make_map_3d_f32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                    uint64_t dim2, uint32_t box0, uint32_t box1, bool granule32 = false);

// Reads and clears the device error word set by a tensor-core kernel whose
// bounded wait ran out (0 = none).
int tc_take_device_error();

}  // namespace tw
