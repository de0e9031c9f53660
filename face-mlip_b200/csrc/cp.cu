// Per-channel Cartesian density of the CP factorised form (face/model.py:496-502, cp=True) and of the
// non-factorised MomentBlock (face/model.py:160-187):
//
//   D[x, i, c] = sum_{e in row i} Y[e, x] R[e, l(x), c] m[e, c]        x < 20, l(x) the rank of component x
//
// R = the per-(rank, channel) radial functions (envelope included) at column offset r_off of a row of stride ldr,
// m = the per-edge channel message (CP: msg(h)_j plus the directional term; MomentBlock: h_j plus the directional
// term).  D is component-major (20, N, C) so each rank block is one contiguous operand.  CSR rows, no atomics.
// The reference computes the same sums as one bmm over all 4 x 20 (rank, component) pairs and keeps the
// rank-diagonal blocks (face/model.py:498-502).
//
// Adjoint, with G = dL/dD:
//   S_l[e, c]  = sum_{x in rank l} Y[e, x] G[x, i, c]
//   dR[e,l,c]  = m[e, c] S_l[e, c],     dm[e, c] = sum_l R[e, l, c] S_l[e, c]
//   dY[e, x]   = sum_c R[e, l(x), c] m[e, c] G[x, i, c]        (a reduction over channels: one warp per edge)
#include "common.cuh"

namespace facek {
namespace {

constexpr int NX = 20;

__host__ __device__ constexpr int rank_of(int x) { return x < 1 ? 0 : (x < 4 ? 1 : (x < 10 ? 2 : 3)); }

// one block per row (grid-stride), one thread per channel
template <typename T>
__global__ void cp_fwd_k(const T* __restrict__ Y, const T* __restrict__ R, int64_t ldr, int r_off,
                         const T* __restrict__ m, const int32_t* __restrict__ row_ptr, int64_t N, int C,
                         T* __restrict__ D) {
  const int c = threadIdx.x;
  if (c >= C) return;
  const int64_t plane = N * (int64_t)C;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    T acc[NX];
#pragma unroll
    for (int x = 0; x < NX; x++) acc[x] = 0;
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T* re = R + (int64_t)e * ldr + r_off + c;
      const T me = m[(int64_t)e * C + c];
      T rm[4];
#pragma unroll
      for (int l = 0; l < 4; l++) rm[l] = re[l * C] * me;
      const T* ye = Y + (int64_t)e * NX;
#pragma unroll
      for (int x = 0; x < NX; x++) acc[x] += __ldg(ye + x) * rm[rank_of(x)];
    }
#pragma unroll
    for (int x = 0; x < NX; x++) D[x * plane + i * C + c] = acc[x];
  }
}

template <typename T>
__global__ void cp_bwd_k(const T* __restrict__ Y, const T* __restrict__ R, int64_t ldr, int r_off,
                         const T* __restrict__ m, const T* __restrict__ G, const int32_t* __restrict__ row_ptr,
                         int64_t N, int C, T* __restrict__ dR, T* __restrict__ dm) {
  const int c = threadIdx.x;
  if (c >= C) return;
  const int64_t plane = N * (int64_t)C;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    T g[NX];
#pragma unroll
    for (int x = 0; x < NX; x++) g[x] = G[x * plane + i * C + c];
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T* ye = Y + (int64_t)e * NX;
      T S[4] = {0, 0, 0, 0};
#pragma unroll
      for (int x = 0; x < NX; x++) S[rank_of(x)] += __ldg(ye + x) * g[x];
      const T* re = R + (int64_t)e * ldr + r_off + c;
      T* dre = dR + (int64_t)e * ldr + r_off + c;
      const T me = m[(int64_t)e * C + c];
      T s = 0;
#pragma unroll
      for (int l = 0; l < 4; l++) {
        dre[l * C] = me * S[l];
        s += re[l * C] * S[l];
      }
      dm[(int64_t)e * C + c] = s;
    }
  }
}

// one warp per edge: dY[e, x] = sum_c R[e, l(x), c] m[e, c] G[x, ei[e], c]
template <typename T>
__global__ void cp_dy_k(const T* __restrict__ R, int64_t ldr, int r_off, const T* __restrict__ m,
                        const T* __restrict__ G, const int32_t* __restrict__ ei, int64_t N, int64_t E, int C,
                        T* __restrict__ dY) {
  const int lane = threadIdx.x & 31;
  const int64_t plane = N * (int64_t)C;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t e = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < E; e += warps) {
    const int64_t i = ei[e];
    T acc[NX];
#pragma unroll
    for (int x = 0; x < NX; x++) acc[x] = 0;
    for (int c = lane; c < C; c += 32) {
      const T me = m[e * C + c];
      const T* re = R + e * ldr + r_off + c;
      T rm[4];
#pragma unroll
      for (int l = 0; l < 4; l++) rm[l] = re[l * C] * me;
#pragma unroll
      for (int x = 0; x < NX; x++) acc[x] += rm[rank_of(x)] * G[x * plane + i * C + c];
    }
#pragma unroll
    for (int x = 0; x < NX; x++) {
      T v = acc[x];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[x] = v;
    }
    if (lane == 0) {
#pragma unroll
      for (int x = 0; x < NX; x++) dY[e * NX + x] = acc[x];
    }
  }
}

inline int threads_for(int C) { return ((C + 31) / 32) * 32; }

template <typename T>
int cp_fwd(const void* Y, const void* R, int64_t ldr, int r_off, const void* m, const int32_t* row_ptr, int64_t N,
           int C, void* D, void* stream) {
  if (N == 0) return FACEK_OK;
  cp_fwd_k<T><<<grid_for(N, 8), threads_for(C), 0, as_stream(stream)>>>((const T*)Y, (const T*)R, ldr, r_off,
                                                                        (const T*)m, row_ptr, N, C, (T*)D);
  return launch_status("facek_cp_density_fwd");
}

template <typename T>
int cp_bwd(const void* Y, const void* R, int64_t ldr, int r_off, const void* m, const void* G, const int32_t* ei,
           const int32_t* row_ptr, int64_t N, int64_t E, int C, void* dR, void* dm, void* dY, void* stream) {
  if (N == 0) return FACEK_OK;
  cp_bwd_k<T><<<grid_for(N, 8), threads_for(C), 0, as_stream(stream)>>>((const T*)Y, (const T*)R, ldr, r_off,
                                                                        (const T*)m, (const T*)G, row_ptr, N, C,
                                                                        (T*)dR, (T*)dm);
  int st = launch_status("facek_cp_density_bwd");
  if (st || E == 0) return st;
  cp_dy_k<T><<<grid_for(ceil_div<int64_t>(E, 8), 8), 256, 0, as_stream(stream)>>>(
      (const T*)R, ldr, r_off, (const T*)m, (const T*)G, ei, N, E, C, (T*)dY);
  return launch_status("facek_cp_density_bwd(dY)");
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_cp_density_fwd(int dtype, const void* Y, const void* R, int64_t ldr, int32_t r_off,
                                    const void* m, const int32_t* row_ptr, int64_t N, int32_t C, void* D,
                                    void* stream) {
  FACEK_CHECK_ARG(N >= 0 && C > 0 && C <= 1024 && r_off >= 0 && ldr >= r_off + 4 * (int64_t)C &&
                      (N == 0 || (Y && R && m && row_ptr && D)),
                  "facek_cp_density_fwd: bad arguments");
  return FACEK_DISPATCH(dtype, cp_fwd, Y, R, ldr, r_off, m, row_ptr, N, C, D, stream);
}

extern "C" int facek_cp_density_bwd(int dtype, const void* Y, const void* R, int64_t ldr, int32_t r_off,
                                    const void* m, const void* G, const int32_t* ei, const int32_t* row_ptr,
                                    int64_t N, int64_t E, int32_t C, void* dR, void* dm, void* dY, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && E >= 0 && C > 0 && C <= 1024 && r_off >= 0 && ldr >= r_off + 4 * (int64_t)C &&
                      (N == 0 || (Y && R && m && G && ei && row_ptr && dR && dm && dY)),
                  "facek_cp_density_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, cp_bwd, Y, R, ldr, r_off, m, G, ei, row_ptr, N, E, C, dR, dm, dY, stream);
}
