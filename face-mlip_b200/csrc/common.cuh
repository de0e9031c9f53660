// Shared helpers for libfacek.so (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdarg>
#include <cstdio>

#include "../../include/facek.h"

namespace facek {

void set_error(const char* fmt, ...);
int launch_status(const char* what);      // FACEK_OK or FACEK_ELAUNCH with the CUDA error recorded
int sm_count();                           // multiprocessors of the current device (cached per device)
int max_smem_optin();                     // opt-in shared memory per block (bytes)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
__host__ __device__ inline T ceil_div(T a, T b) { return (a + b - 1) / b; }

// grid of `per_sm` blocks per SM, capped by the work (persistent-style loops use grid-stride indexing)
inline int grid_for(int64_t work_blocks, int per_sm) {
  int64_t g = (int64_t)sm_count() * per_sm;
  if (work_blocks < g) g = work_blocks;
  return (int)(g < 1 ? 1 : g);
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
