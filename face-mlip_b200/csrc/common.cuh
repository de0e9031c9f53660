// Shared helpers for libfacek.so (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <type_traits>

#include "../../include/facek.h"

namespace facek {

void set_error(const char* fmt, ...);
int launch_status(const char* what);      // FACEK_OK or FACEK_ELAUNCH with the CUDA error recorded
int sm_count();                           // multiprocessors of the current device (cached per device)
int max_smem_optin();                     // opt-in shared memory per block (bytes)

// tensor-core radial MLP (radial_tc.cu), fp32 only
bool radial_tc_supported(int n_el, int nb, int H, int B);
int radial_tc_fwd(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
                  int nb, int H, int B, const void* w1, const void* b1, const void* pair, const void* w2,
                  const void* b2, const void* w3, const void* b3, void* phi, void* dphidr, int64_t E, void* stream);
// tensor-core density forward, fp32 B=16 K=32, component-major planes (density_tc.cu) and its status word
int density_tc_xm_fwd(const float* phi, const float* msg, const float* Y, float* D, int64_t N,
                      const int32_t* row_ptr, void* stream);
int density_tc_status(int clear);
// message part of dY accumulated into dY (edge.cu)
int edge_msg_dy(int dtype, const int32_t* ei, const int32_t* ej, const void* TJ, const void* TI, const void* dmsg,
                int nc, int K, int64_t N, int64_t E, void* dY, void* stream);
// bounded-wait status word of the tensor-core GEMM unit (gemm_tc.cu); -1 when it cannot be read
int gemm_tc_status(int clear);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
__host__ __device__ inline T ceil_div(T a, T b) { return (a + b - 1) / b; }

// grid of `per_sm` blocks per SM, capped by the work (persistent-style loops use grid-stride indexing)
inline int grid_for(int64_t work_blocks, int per_sm) {
  int64_t g = (int64_t)sm_count() * per_sm;
  if (work_blocks < g) g = work_blocks;
  return (int)(g < 1 ? 1 : g);
}

// d0 += a0 * b0, d1 += a1 * b1 as one paired fp32 FMA (fma.rn.f32x2, sm_100): two round-to-nearest fp32 FMAs,
// bit-identical to two scalar fmaf calls, in one issue slot
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// ---- asynchronous global->shared copies (cp.async, 16-byte chunks; both addresses 16-byte aligned)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// copy n elements of T from global to shared: cp.async in 16-byte chunks when both ends are 16-byte aligned
// and n*sizeof(T) is a multiple of 16, else plain loads (caller syncs)
template <typename T>
__device__ __forceinline__ void stage(T* dst, const T* src, int n, int tid, int nthr) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0 &&
                   ((n * (int)sizeof(T)) & 15) == 0;
  if (vec) {
    const int nv = n * (int)sizeof(T) / 16;
    for (int q = tid; q < nv; q += nthr) cp_async16(reinterpret_cast<char*>(dst) + 16 * q,
                                                    reinterpret_cast<const char*>(src) + 16 * q);
  } else {
    for (int q = tid; q < n; q += nthr) dst[q] = src[q];
  }
}

}  // namespace facek

#define FACEK_CHECK_ARG(cond, ...)          \
  do {                                      \
    if (!(cond)) {                          \
      facek::set_error(__VA_ARGS__);        \
      return FACEK_EINVAL;                  \
    }                                       \
  } while (0)

// dispatch a templated launcher on the dtype tag
#define FACEK_DISPATCH(dtype, FN, ...)                                              \
  ((dtype) == FACEK_F32   ? FN<float>(__VA_ARGS__)                                 \
   : (dtype) == FACEK_F64 ? FN<double>(__VA_ARGS__)                                \
                          : (facek::set_error("unknown dtype tag %d", (int)(dtype)), FACEK_EINVAL))
