// Node-level elementwise kernels of the readout (face/model.py:331-339): LayerNorm over the 9C invariants of an atom
// (nn.LayerNorm, affine, biased variance) and the SiLU activations of the readout MLP, forward and adjoint.
//
// LayerNorm: one warp per row, the row held in registers (W <= 32 * LN_MAXPER), two-pass mean / variance in the
// model dtype as torch computes them, then y = (x - mean) * rstd * w + b.  The forward stores mean and rstd per row
// for the adjoint  dx = rstd * (gw - mean(gw) - xhat * mean(gw * xhat)),  gw = g * w  (weights are constants here).
#include "common.cuh"

namespace facek {
namespace {

constexpr int LN_MAXPER = 24;       // up to 768 features per row

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void ln_fwd_k(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b, T eps,
                         int64_t N, int W, T* __restrict__ y, T* __restrict__ mean, T* __restrict__ rstd) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < N; r += warps) {
    const T* xr = x + r * W;
    T v[LN_MAXPER];
    T s = 0;
#pragma unroll
    for (int k = 0; k < LN_MAXPER; k++) {
      const int c = lane + 32 * k;
      v[k] = c < W ? xr[c] : T(0);
      s += v[k];
    }
    const T mu = warp_sum(s) / T(W);
    T q = 0;
#pragma unroll
    for (int k = 0; k < LN_MAXPER; k++) {
      const int c = lane + 32 * k;
      const T d = c < W ? v[k] - mu : T(0);
      q += d * d;
    }
    const T rs = T(1) / sqrt(warp_sum(q) / T(W) + eps);
    T* yr = y + r * W;
#pragma unroll
    for (int k = 0; k < LN_MAXPER; k++) {
      const int c = lane + 32 * k;
      if (c < W) yr[c] = (v[k] - mu) * rs * w[c] + b[c];
    }
    if (lane == 0) {
      mean[r] = mu;
      rstd[r] = rs;
    }
  }
}

template <typename T>
__global__ void ln_bwd_k(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ g,
                         const T* __restrict__ mean, const T* __restrict__ rstd, int64_t N, int W,
                         T* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < N; r += warps) {
    const T mu = mean[r], rs = rstd[r];
    T xh[LN_MAXPER], gw[LN_MAXPER];
    T s1 = 0, s2 = 0;
#pragma unroll
    for (int k = 0; k < LN_MAXPER; k++) {
      const int c = lane + 32 * k;
      xh[k] = c < W ? (x[r * W + c] - mu) * rs : T(0);
      gw[k] = c < W ? g[r * W + c] * w[c] : T(0);
      s1 += gw[k];
      s2 += gw[k] * xh[k];
    }
    const T m1 = warp_sum(s1) / T(W), m2 = warp_sum(s2) / T(W);
#pragma unroll
    for (int k = 0; k < LN_MAXPER; k++) {
      const int c = lane + 32 * k;
      if (c < W) dx[r * W + c] = rs * (gw[k] - m1 - xh[k] * m2);
    }
  }
}

template <typename T>
__device__ __forceinline__ T sig(T z) {
  return T(1) / (T(1) + exp(-z));
}

template <typename T>
__global__ void silu_fwd_k(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    const T v = x[k];
    y[k] = v * sig(v);
  }
}

template <typename T>
__global__ void silu_bwd_k(const T* __restrict__ x, const T* __restrict__ g, T* __restrict__ dx, int64_t n) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    const T v = x[k], s = sig(v);
    dx[k] = g[k] * s * (T(1) + v * (T(1) - s));
  }
}

inline int warp_rows_grid(int64_t rows) { return grid_for(ceil_div<int64_t>(rows, 8), 8); }
inline int elem_blocks(int64_t n) { return grid_for(ceil_div<int64_t>(n, 256), 8); }

template <typename T>
int ln_fwd(const void* x, const void* w, const void* b, double eps, int64_t N, int W, void* y, void* mean, void* rstd,
           void* stream) {
  if (N == 0) return FACEK_OK;
  ln_fwd_k<T><<<warp_rows_grid(N), 256, 0, as_stream(stream)>>>((const T*)x, (const T*)w, (const T*)b, (T)eps, N, W,
                                                                (T*)y, (T*)mean, (T*)rstd);
  return launch_status("facek_layer_norm_fwd");
}
template <typename T>
int ln_bwd(const void* x, const void* w, const void* g, const void* mean, const void* rstd, int64_t N, int W,
           void* dx, void* stream) {
  if (N == 0) return FACEK_OK;
  ln_bwd_k<T><<<warp_rows_grid(N), 256, 0, as_stream(stream)>>>((const T*)x, (const T*)w, (const T*)g,
                                                                (const T*)mean, (const T*)rstd, N, W, (T*)dx);
  return launch_status("facek_layer_norm_bwd");
}
template <typename T>
int silu_fwd(const void* x, void* y, int64_t n, void* stream) {
  if (n == 0) return FACEK_OK;
  silu_fwd_k<T><<<elem_blocks(n), 256, 0, as_stream(stream)>>>((const T*)x, (T*)y, n);
  return launch_status("facek_silu_fwd");
}
template <typename T>
int silu_bwd(const void* x, const void* g, void* dx, int64_t n, void* stream) {
  if (n == 0) return FACEK_OK;
  silu_bwd_k<T><<<elem_blocks(n), 256, 0, as_stream(stream)>>>((const T*)x, (const T*)g, (T*)dx, n);
  return launch_status("facek_silu_bwd");
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_layer_norm_fwd(int dtype, const void* x, const void* w, const void* b, double eps, int64_t N,
                                    int32_t W, void* y, void* mean, void* rstd, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && W > 0 && W <= 32 * LN_MAXPER && eps >= 0 && (N == 0 || (x && w && b && y && mean && rstd)),
                  "facek_layer_norm_fwd: bad arguments (W=%d, at most %d)", W, 32 * LN_MAXPER);
  return FACEK_DISPATCH(dtype, ln_fwd, x, w, b, eps, N, W, y, mean, rstd, stream);
}
extern "C" int facek_layer_norm_bwd(int dtype, const void* x, const void* w, const void* g, const void* mean,
                                    const void* rstd, int64_t N, int32_t W, void* dx, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && W > 0 && W <= 32 * LN_MAXPER && (N == 0 || (x && w && g && mean && rstd && dx)),
                  "facek_layer_norm_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, ln_bwd, x, w, g, mean, rstd, N, W, dx, stream);
}
extern "C" int facek_silu_fwd(int dtype, const void* x, void* y, int64_t n, void* stream) {
  FACEK_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "facek_silu_fwd: bad arguments");
  return FACEK_DISPATCH(dtype, silu_fwd, x, y, n, stream);
}
extern "C" int facek_silu_bwd(int dtype, const void* x, const void* g, void* dx, int64_t n, void* stream) {
  FACEK_CHECK_ARG(n >= 0 && (n == 0 || (x && g && dx)), "facek_silu_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, silu_bwd, x, g, dx, n, stream);
}
