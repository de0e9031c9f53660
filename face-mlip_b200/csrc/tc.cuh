// tcgen05 (5th-generation tensor core) primitives for sm_100a, written as inline PTX.
//
// Operands live in shared memory in the K-major, no-swizzle canonical layout: a "core matrix" is 8 rows x 16 bytes
// stored as 128 contiguous bytes; core matrices of consecutive 8-row groups are SBO bytes apart and the two 16-byte
// K chunks that one MMA step consumes are LBO bytes apart. kmajor_off() below places element (row, k) of an fp32
// operand with R rows so that SBO = 128 and LBO = R * 16, which also makes one warp's 32 consecutive rows a
// contiguous, bank-conflict-free 512-byte store for each 4-float chunk.
//
// fp32 accuracy on the tf32 datapath uses the three-term split x = hi + lo (hi = tf32(x), lo = tf32(x - hi)):
// A.B ~= Ahi.Bhi + Ahi.Blo + Alo.Bhi, dropping only the Alo.Blo term (relative size 2^-22). Where an operand is
// fed to the tensor core as raw fp32, hi is the truncation the hardware applies and lo = tf32(x - trunc(x))
// (dropped term 2^-21).
//
// Every wait here is bounded: a wait that runs out sets a status bit in g_tc_status (read and cleared through
// facek_tc_status) and returns false; callers then skip the remaining work and release their tensor memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace facek {
namespace tc {

// bit 0: an mbarrier wait ran out. One copy per translation unit (no relocatable device code); each unit that
// launches tcgen05 kernels reports its copy through facek_tc_status.
static __device__ int g_tc_status = 0;

constexpr uint32_t kWaitLimit = 1u << 22;   // try_wait rounds (each suspends up to a hardware time slice)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of element (row, k) of an R-row fp32 K-major operand (R a multiple of 8)
__host__ __device__ constexpr uint32_t kmajor_off(uint32_t row, uint32_t k, uint32_t R) {
  return (k >> 2) * (R * 16u) + (row >> 3) * 128u + (row & 7u) * 16u + (k & 3u) * 4u;
}

// shared-memory matrix descriptor, K-major, no swizzle (fields per the sm_100 UMMA descriptor format:
// start>>4 in [0,14), LBO>>4 in [16,30), SBO>>4 in [32,46), version 1 in [46,48), layout 0 in [61,64))
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// instruction descriptor, kind::tf32: D fp32, A and B tf32, both K-major, dense
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T, issued by one thread
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// arrive once on mbar when every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(mbar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// non-blocking check of the phase with the given parity
__device__ __forceinline__ bool mbar_test(uint64_t* mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(mbar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait for the phase with the given parity; on running out (or when *abort is already set by a sibling
// thread) returns false and sets *abort and the device status.  A phase that is already complete is seen by the
// non-blocking test (measured ~2x quicker than try_wait on sm_100 in a pipeline that mostly finds its barriers
// complete); try_wait, which may suspend the thread until the phase completes, runs only when it is not.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, volatile int* abort) {
  if (mbar_test(mbar, parity)) return true;
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    if (mbar_try_wait(mbar, parity)) return true;
    if (*abort) return false;
  }
  *abort = 1;
  atomicOr(&g_tc_status, 1);
  return false;
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// named barrier over `count` threads
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// tensor-memory allocation: one full warp; writes the base address to *slot
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32*(w%4) .. +31)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// 8 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 8 consecutive fp32 columns of this thread's TMEM lane <- v (TMEM as a parking place for values that would
// otherwise stay live in registers across an MMA round)
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// round to tf32 (nearest, ties away from zero), kept in an fp32 register with the low 13 mantissa bits zero.
// Integer form: adding half of the dropped range to the magnitude bits and masking rounds the magnitude
// half-up, the same result as cvt.rna.tf32.f32 for finite values, on the integer ALU instead of the
// conversion pipe.
__device__ __forceinline__ float to_tf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
// the tf32 value the tensor core reads from an fp32 bit pattern (the low 13 mantissa bits ignored)
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// store 4 consecutive-k values of one row as (hi, lo) into two operand planes
__device__ __forceinline__ void store_split4(unsigned char* hi_plane, unsigned char* lo_plane, uint32_t off,
                                             float a, float b, float c, float d) {
  const float ah = to_tf32(a), bh = to_tf32(b), ch = to_tf32(c), dh = to_tf32(d);
  *reinterpret_cast<float4*>(hi_plane + off) = make_float4(ah, bh, ch, dh);
  *reinterpret_cast<float4*>(lo_plane + off) =
      make_float4(to_tf32(a - ah), to_tf32(b - bh), to_tf32(c - ch), to_tf32(d - dh));
}

}  // namespace tc
}  // namespace facek
