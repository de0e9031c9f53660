// Element math shared by the SIMT and tensor-core radial kernels: the polynomial envelope and the SiLU gate.
#pragma once
#include <cuda_runtime.h>

namespace facek {

template <typename T>
__device__ __forceinline__ T sigmoid(T z) {
  return T(1) / (T(1) + exp(-z));
}
// fp32 sigmoid with the reciprocal as __frcp_rn: the correctly rounded 1/x, i.e. the same value as the IEEE division
// above, in fewer instructions
__device__ __forceinline__ float sigmoid_f(float z) { return __frcp_rn(1.f + expf(-z)); }

// polynomial envelope p = 6 (face/model.py:34-37) and its r-derivative
template <typename T>
__device__ __forceinline__ void envelope(T r, T rc, T& env, T& denv) {
  const T x = r / rc;
  if (x >= T(1)) {
    env = 0;
    denv = 0;
    return;
  }
  const T x2 = x * x, x5 = x2 * x2 * x, x6 = x5 * x, x7 = x6 * x, x8 = x7 * x;
  env = T(1) - T(28) * x6 + T(48) * x7 - T(21) * x8;
  denv = (T(-168) * x5 + T(336) * x6 - T(168) * x7) / rc;
}

}  // namespace facek
