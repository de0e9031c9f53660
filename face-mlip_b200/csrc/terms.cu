// Pair physics terms of FACE, per CSR row (centre atom) over a symmetric neighbour list, forward and adjoint:
//   ZBL        universal screened nuclear repulsion switched off between r_in and r_out (face/model.py:538-554)
//   dispersion environment-dependent C6 / (r^6 + R0^6) with a smooth switch to zero at r_long over a long-range
//              pair list (face/dispersion.py:13-48)
// Each row sums its own edges (no atomics); the adjoints write per-edge dE/dvec for the row's own term and per-atom
// charge-like gradients that join both rows of a pair, as the Coulomb real-space kernels do.
#include "common.cuh"

namespace facek {
namespace {

// universal ZBL screening function phi(x) = sum_k c_k exp(-d_k x) and its x-derivative
template <typename T>
__device__ __forceinline__ void zbl_screen(T x, T& f, T& df) {
  const T c[4] = {T(0.18175), T(0.50986), T(0.28022), T(0.02817)};
  const T d[4] = {T(3.19980), T(0.94229), T(0.40290), T(0.20162)};
  f = 0;
  df = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const T ex = c[k] * exp(-d[k] * x);
    f += ex;
    df -= d[k] * ex;
  }
}

// smooth step s = 1 - t^3 (10 - 15 t + 6 t^2), t = clamp((r - r0) / w, 0, 1), and ds/dr (zero where t is clamped)
template <typename T>
__device__ __forceinline__ void smooth_off(T r, T r0, T w, T& s, T& ds) {
  T t = (r - r0) / w;
  if (t <= T(0)) {
    s = 1;
    ds = 0;
  } else if (t >= T(1)) {
    s = 0;
    ds = 0;
  } else {
    s = T(1) - t * t * t * (T(10) - T(15) * t + T(6) * t * t);
    ds = -T(30) * t * t * (T(1) - t) * (T(1) - t) / w;
  }
}

// pair energy E(r) = KE Zi Zj / r phi(r / a) s(r) and dE/dr
template <typename T>
__device__ __forceinline__ void zbl_pair(T r, T zi, T zj, T r_in, T r_out, T& E, T& dE) {
  const T a = T(0.46850) / (pow(zi, T(0.23)) + pow(zj, T(0.23)));
  T f, df, s, ds;
  zbl_screen(r / a, f, df);
  smooth_off(r, r_in, r_out - r_in, s, ds);
  const T pre = T(14.399645) * zi * zj;
  E = pre / r * f * s;
  dE = pre * ((-f / (r * r) + df / (a * r)) * s + f / r * ds);
}

template <typename T>
__global__ void zbl_fwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                          const int32_t* __restrict__ ej, const int32_t* __restrict__ Z, T r_in, T r_out, int64_t N,
                          T* __restrict__ e_row) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const T zi = (T)Z[i];
    T s = 0;
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T r = sqrt(vx * vx + vy * vy + vz * vz);
      if (r >= r_out) continue;                    // switched off
      T E, dE;
      zbl_pair(r, zi, (T)Z[ej[e]], r_in, r_out, E, dE);
      s += E;
    }
    e_row[i] = T(0.5) * s;
  }
}

// dvec[e] (+)= g_row[i] / 2 dE/dr u for the edges of row i
template <typename T>
__global__ void zbl_bwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                          const int32_t* __restrict__ ej, const int32_t* __restrict__ Z, T r_in, T r_out,
                          const T* __restrict__ g_row, int64_t N, T* __restrict__ dvec, int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const T zi = (T)Z[i], gi = g_row[i];
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T r = sqrt(vx * vx + vy * vy + vz * vz);
      T E = 0, dE = 0;
      if (r < r_out) zbl_pair(r, zi, (T)Z[ej[e]], r_in, r_out, E, dE);
      const T c = T(0.5) * gi * dE / r;
      if (acc) {
        dvec[(int64_t)e * 3] += c * vx; dvec[(int64_t)e * 3 + 1] += c * vy; dvec[(int64_t)e * 3 + 2] += c * vz;
      } else {
        dvec[(int64_t)e * 3] = c * vx; dvec[(int64_t)e * 3 + 1] = c * vy; dvec[(int64_t)e * 3 + 2] = c * vz;
      }
    }
  }
}

// dispersion pair term e = -1/2 C6ij / (d^6 + R0^6) s(d), C6ij = sqrt(C6i C6j), R0 = A1 (r0i + r0j) / 2 + A2;
// returns e and de/dd
template <typename T>
__device__ __forceinline__ void disp_pair(T d, T c6ij, T R0, T r_long, T& e, T& de) {
  T s, ds;
  smooth_off(d, r_long - T(2), T(2), s, ds);
  const T d2 = d * d, d6 = d2 * d2 * d2, R2 = R0 * R0, den = d6 + R2 * R2 * R2;
  e = T(-0.5) * c6ij / den * s;
  de = T(-0.5) * c6ij * (ds / den - T(6) * d6 / d / (den * den) * s);
}

template <typename T>
__global__ void disp_fwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                           const int32_t* __restrict__ ej, const T* __restrict__ C6, const T* __restrict__ r0,
                           const T* __restrict__ A, T r_long, int64_t N, T* __restrict__ e_row) {
  const T A1 = A[0], A2 = A[1];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const T ci = C6[i], ri = r0[i];
    T s = 0;
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const int j = ej[e];
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T d = sqrt(vx * vx + vy * vy + vz * vz);
      T pe, de;
      disp_pair(d, sqrt(ci * C6[j]), A1 * T(0.5) * (ri + r0[j]) + A2, r_long, pe, de);
      s += pe;
    }
    e_row[i] = s;
  }
}

// dC6[i] = sum_{e in row i} (g_i + g_j) e_ij / (2 C6_i)   (both rows of a pair depend on C6_i)
// dvec[e] (+)= g_i de/dd u
template <typename T>
__global__ void disp_bwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                           const int32_t* __restrict__ ej, const T* __restrict__ C6, const T* __restrict__ r0,
                           const T* __restrict__ A, T r_long, const T* __restrict__ g_row, int64_t N,
                           T* __restrict__ dvec, int acc, T* __restrict__ dC6) {
  const T A1 = A[0], A2 = A[1];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const T ci = C6[i], ri = r0[i], gi = g_row[i];
    T sc = 0;
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const int j = ej[e];
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T d = sqrt(vx * vx + vy * vy + vz * vz);
      T pe, de;
      disp_pair(d, sqrt(ci * C6[j]), A1 * T(0.5) * (ri + r0[j]) + A2, r_long, pe, de);
      sc += (gi + g_row[j]) * pe;
      const T c = gi * de / d;
      if (acc) {
        dvec[(int64_t)e * 3] += c * vx; dvec[(int64_t)e * 3 + 1] += c * vy; dvec[(int64_t)e * 3 + 2] += c * vz;
      } else {
        dvec[(int64_t)e * 3] = c * vx; dvec[(int64_t)e * 3 + 1] = c * vy; dvec[(int64_t)e * 3 + 2] = c * vz;
      }
    }
    dC6[i] = sc / (T(2) * ci);
  }
}

inline int row_grid(int64_t n) { return grid_for(ceil_div<int64_t>(n, 128), 16); }

template <typename T>
int zbl_fwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z, double r_in, double r_out,
            int64_t N, void* e_row, void* stream) {
  if (N == 0) return FACEK_OK;
  zbl_fwd_k<T><<<row_grid(N), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, Z, (T)r_in, (T)r_out, N,
                                                           (T*)e_row);
  return launch_status("facek_zbl_fwd");
}
template <typename T>
int zbl_bwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z, double r_in, double r_out,
            const void* g_row, int64_t N, void* dvec, int acc, void* stream) {
  if (N == 0) return FACEK_OK;
  zbl_bwd_k<T><<<row_grid(N), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, Z, (T)r_in, (T)r_out,
                                                           (const T*)g_row, N, (T*)dvec, acc);
  return launch_status("facek_zbl_bwd");
}
template <typename T>
int disp_fwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6, const void* r0,
             const void* A, double r_long, int64_t N, void* e_row, void* stream) {
  if (N == 0) return FACEK_OK;
  disp_fwd_k<T><<<row_grid(N), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, (const T*)C6, (const T*)r0,
                                                            (const T*)A, (T)r_long, N, (T*)e_row);
  return launch_status("facek_disp_fwd");
}
template <typename T>
int disp_bwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6, const void* r0,
             const void* A, double r_long, const void* g_row, int64_t N, void* dvec, int acc, void* dC6,
             void* stream) {
  if (N == 0) return FACEK_OK;
  disp_bwd_k<T><<<row_grid(N), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, (const T*)C6, (const T*)r0,
                                                            (const T*)A, (T)r_long, (const T*)g_row, N, (T*)dvec,
                                                            acc, (T*)dC6);
  return launch_status("facek_disp_bwd");
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_zbl_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z,
                             double r_in, double r_out, int64_t N, void* e_row, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && r_out > r_in && (N == 0 || (vec && row_ptr && ej && Z && e_row)),
                  "facek_zbl_fwd: bad arguments");
  return FACEK_DISPATCH(dtype, zbl_fwd, vec, row_ptr, ej, Z, r_in, r_out, N, e_row, stream);
}
extern "C" int facek_zbl_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z,
                             double r_in, double r_out, const void* g_row, int64_t N, void* dvec, int32_t accumulate,
                             void* stream) {
  FACEK_CHECK_ARG(N >= 0 && r_out > r_in && (N == 0 || (vec && row_ptr && ej && Z && g_row && dvec)),
                  "facek_zbl_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, zbl_bwd, vec, row_ptr, ej, Z, r_in, r_out, g_row, N, dvec, accumulate, stream);
}
extern "C" int facek_disp_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6,
                              const void* r0, const void* A, double r_long, int64_t N, void* e_row, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && r_long > 2 && (N == 0 || (vec && row_ptr && ej && C6 && r0 && A && e_row)),
                  "facek_disp_fwd: bad arguments");
  return FACEK_DISPATCH(dtype, disp_fwd, vec, row_ptr, ej, C6, r0, A, r_long, N, e_row, stream);
}
extern "C" int facek_disp_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6,
                              const void* r0, const void* A, double r_long, const void* g_row, int64_t N, void* dvec,
                              int32_t accumulate, void* dC6, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && r_long > 2 && (N == 0 || (vec && row_ptr && ej && C6 && r0 && A && g_row && dvec && dC6)),
                  "facek_disp_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, disp_bwd, vec, row_ptr, ej, C6, r0, A, r_long, g_row, N, dvec, accumulate, dC6,
                        stream);
}
