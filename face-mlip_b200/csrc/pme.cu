// Smooth particle-mesh Ewald pieces of face-mlip's latent-charge Coulomb term
// (face/electrostatics.py:34-77 pme_recip_energy, :91-92 and :125-127 real-space Gaussian kernel).
//   spread : Q[(base - k) mod n] += q * w_k0(f0) w_k1(f1) w_k2(f2), order-4 cardinal B-spline, u = (pos @ inv) * n
//   green  : E = 1/(2V) sum_m G(k) B(m) |F(m)|^2 over the full spectrum, from the rfft half spectrum;
//            conv = G B F * (n0 n1 n2 / V) so that irfftn(conv) = dE/dQ on the mesh
//   gather : dE/dq_i = sum W phi, dE/dpos_i = q_i sum (dW/du) (du/dpos) phi (autograd of the reference, :60-68)
//   real   : e_i = 1/2 sum_{e in row i} q_i q_j (erf(r/gamma) - erf(r/gp)) / r and its adjoint
#include <limits>

#include "common.cuh"

namespace facek {
namespace {

template <typename T>
__device__ __forceinline__ void bspline4(T f, T w[4], T dw[4]) {
  // weights for grid offsets 0, -1, -2, -3 (face/electrostatics.py:34-41) and their derivatives in f
  const T f2 = f * f, f3 = f2 * f, g = T(1) - f;
  w[0] = f3 / T(6);
  w[1] = (T(-3) * f3 + T(3) * f2 + T(3) * f + T(1)) / T(6);
  w[2] = (T(3) * f3 - T(6) * f2 + T(4)) / T(6);
  w[3] = g * g * g / T(6);
  dw[0] = f2 / T(2);
  dw[1] = (T(-9) * f2 + T(6) * f + T(3)) / T(6);
  dw[2] = (T(9) * f2 - T(12) * f) / T(6);
  dw[3] = -g * g / T(2);
}

struct Mesh {
  double inv[9];
  int n[3];
};

template <typename T>
__device__ __forceinline__ void grid_coords(const T* p, const Mesh& m, int base[3], T f[3]) {
#pragma unroll
  for (int d = 0; d < 3; d++) {
    const T fr = p[0] * (T)m.inv[d] + p[1] * (T)m.inv[3 + d] + p[2] * (T)m.inv[6 + d];
    const T u = fr * (T)m.n[d];
    const T b = floor(u);
    f[d] = u - b;
    int bi = (int)b % m.n[d];
    if (bi < 0) bi += m.n[d];
    base[d] = bi;
  }
}

template <typename T>
__global__ void spread_k(const T* __restrict__ pos, const T* __restrict__ q, int64_t N, Mesh m, T* __restrict__ mesh) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    int base[3];
    T f[3], w[3][4], dw[4];
    grid_coords(pos + i * 3, m, base, f);
#pragma unroll
    for (int d = 0; d < 3; d++) bspline4(f[d], w[d], dw);
    const T qi = q[i];
#pragma unroll
    for (int a = 0; a < 4; a++) {
      const int i0 = (base[0] - a + m.n[0]) % m.n[0];
      const T wa = qi * w[0][a];
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i1 = (base[1] - b + m.n[1]) % m.n[1];
        const T wab = wa * w[1][b];
        T* row = mesh + ((int64_t)i0 * m.n[1] + i1) * m.n[2];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int i2 = (base[2] - c + m.n[2]) % m.n[2];
          atomicAdd(row + i2, wab * w[2][c]);
        }
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ int fftfreq(int k, int n) { return k <= (n - 1) / 2 ? k : k - n; }

template <typename T>
__global__ void green_k(const T* __restrict__ spec, int n0, int n1, int n2, Mesh m, T gp, T vol,
                        const T* __restrict__ bmod, double* __restrict__ energy, T* __restrict__ conv) {
  const int nh = n2 / 2 + 1;
  const int64_t total = (int64_t)n0 * n1 * nh;
  const T two_pi = T(6.283185307179586476925286766559);
  const T scale = T((double)n0 * n1 * n2) / vol;
  double local = 0;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int k2 = (int)(q % nh);
    const int64_t r = q / nh;
    const int k1 = (int)(r % n1), k0 = (int)(r / n1);
    const T m0 = (T)fftfreq<T>(k0, n0), m1 = (T)fftfreq<T>(k1, n1), m2 = (T)fftfreq<T>(k2, n2);
    // k = 2 pi m . inv^T  (face/electrostatics.py:72)
    T kx = two_pi * (m0 * (T)m.inv[0] + m1 * (T)m.inv[1] + m2 * (T)m.inv[2]);
    T ky = two_pi * (m0 * (T)m.inv[3] + m1 * (T)m.inv[4] + m2 * (T)m.inv[5]);
    T kz = two_pi * (m0 * (T)m.inv[6] + m1 * (T)m.inv[7] + m2 * (T)m.inv[8]);
    const T ksq = kx * kx + ky * ky + kz * kz;
    T G = 0;
    if (ksq > T(1e-12)) G = T(4) * T(3.14159265358979323846) / ksq * exp(-gp * gp * ksq / T(4));
    const T Bm = bmod[k0] * bmod[n0 + k1] * bmod[n0 + n1 + k2];
    const T re = spec[2 * q], im = spec[2 * q + 1];
    const T gb = G * Bm;
    const double wz = (k2 == 0 || (n2 % 2 == 0 && k2 == n2 / 2)) ? 1.0 : 2.0;
    local += wz * (double)gb * ((double)re * re + (double)im * im);
    conv[2 * q] = gb * re * scale;
    conv[2 * q + 1] = gb * im * scale;
  }
  // block reduction in double
  __shared__ double red[32];
  for (int off = 16; off > 0; off >>= 1) local += __shfl_xor_sync(0xffffffffu, local, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) atomicAdd(energy, 0.5 * v / (double)vol);
  }
}

template <typename T>
__global__ void gather_k(const T* __restrict__ pos, const T* __restrict__ q, int64_t N, Mesh m,
                         const T* __restrict__ pot, T scale, T* __restrict__ dq, T* __restrict__ dpos) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    int base[3];
    T f[3], w[3][4], dw[3][4];
    grid_coords(pos + i * 3, m, base, f);
#pragma unroll
    for (int d = 0; d < 3; d++) bspline4(f[d], w[d], dw[d]);
    T s = 0, g0 = 0, g1 = 0, g2 = 0;
#pragma unroll
    for (int a = 0; a < 4; a++) {
      const int i0 = (base[0] - a + m.n[0]) % m.n[0];
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i1 = (base[1] - b + m.n[1]) % m.n[1];
        const T* row = pot + ((int64_t)i0 * m.n[1] + i1) * m.n[2];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int i2 = (base[2] - c + m.n[2]) % m.n[2];
          const T ph = row[i2];
          s += w[0][a] * w[1][b] * w[2][c] * ph;
          g0 += dw[0][a] * w[1][b] * w[2][c] * ph;
          g1 += w[0][a] * dw[1][b] * w[2][c] * ph;
          g2 += w[0][a] * w[1][b] * dw[2][c] * ph;
        }
      }
    }
    dq[i] = scale * s;
    // du_d / dpos_e = n_d inv[e][d]
    const T qi = scale * q[i];
    const T gu[3] = {g0 * (T)m.n[0], g1 * (T)m.n[1], g2 * (T)m.n[2]};
#pragma unroll
    for (int e = 0; e < 3; e++)
      dpos[i * 3 + e] = qi * (gu[0] * (T)m.inv[e * 3] + gu[1] * (T)m.inv[e * 3 + 1] + gu[2] * (T)m.inv[e * 3 + 2]);
  }
}

template <typename T>
__device__ __forceinline__ void gauss_kernel(T r, T gamma, T gp, T& K, T& dK) {
  const T c = T(1.1283791670955125738961589031215);     // 2 / sqrt(pi)
  K = (erf(r / gamma) - erf(r / gp)) / r;
  dK = (c * (exp(-(r / gamma) * (r / gamma)) / gamma - exp(-(r / gp) * (r / gp)) / gp) - K) / r;
}

template <typename T>
__global__ void real_fwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                           const int32_t* __restrict__ ej, const T* __restrict__ q, T gamma, T gp, T rcut, int64_t N,
                           T* __restrict__ e_row) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    T s = 0;
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T r = sqrt(vx * vx + vy * vy + vz * vz);
      if (r >= rcut) continue;                        // skin edges of a reused neighbour list
      T K, dK;
      gauss_kernel(r, gamma, gp, K, dK);
      s += q[ej[e]] * K;
    }
    e_row[i] = T(0.5) * q[i] * s;
  }
}

// g_row: per-row upstream dL/de_row.  With the symmetric list, edge (i,j) in row i and its reverse in row j give
// dq_i = sum_{e in row i} (g_i + g_j)/2 q_j K(r);  dvec[e] (+)= g_i q_i q_j K'(r) u / 2
template <typename T>
__global__ void real_bwd_k(const T* __restrict__ vec, const int32_t* __restrict__ row_ptr,
                           const int32_t* __restrict__ ej, const T* __restrict__ q, T gamma, T gp, T rcut,
                           const T* __restrict__ g_row, int64_t N, T* __restrict__ dvec, int acc, T* __restrict__ dq) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    T s = 0;
    const T qi = q[i], gi = g_row[i];
    for (int e = row_ptr[i]; e < row_ptr[i + 1]; e++) {
      const T vx = vec[(int64_t)e * 3], vy = vec[(int64_t)e * 3 + 1], vz = vec[(int64_t)e * 3 + 2];
      const T r = sqrt(vx * vx + vy * vy + vz * vz);
      T K = 0, dK = 0;
      if (r < rcut) gauss_kernel(r, gamma, gp, K, dK);   // beyond the cut the edge contributes zero
      const int j = ej[e];
      const T qj = q[j];
      s += T(0.5) * (gi + g_row[j]) * qj * K;
      const T c = gi * T(0.5) * qi * qj * dK / r;
      if (acc) {
        dvec[(int64_t)e * 3] += c * vx; dvec[(int64_t)e * 3 + 1] += c * vy; dvec[(int64_t)e * 3 + 2] += c * vz;
      } else {
        dvec[(int64_t)e * 3] = c * vx; dvec[(int64_t)e * 3 + 1] = c * vy; dvec[(int64_t)e * 3 + 2] = c * vz;
      }
    }
    dq[i] = s;
  }
}

// real-space cut: r_cut <= 0 keeps every edge of the list (the reference's behaviour: the pair list is the model's)
template <typename T>
T cut_value(double rcut) {
  return rcut > 0 ? (T)rcut : std::numeric_limits<T>::infinity();
}

Mesh make_mesh(const double* inv, int n0, int n1, int n2) {
  Mesh m;
  for (int k = 0; k < 9; k++) m.inv[k] = inv[k];
  m.n[0] = n0; m.n[1] = n1; m.n[2] = n2;
  return m;
}
inline int ew_grid(int64_t n, int threads) { return grid_for(ceil_div<int64_t>(n, threads), 16); }

template <typename T>
int spread(const void* pos, const void* q, int64_t N, const double* inv, int n0, int n1, int n2, void* mesh,
           void* stream) {
  if (N == 0) return FACEK_OK;
  spread_k<T><<<ew_grid(N, 128), 128, 0, as_stream(stream)>>>((const T*)pos, (const T*)q, N,
                                                              make_mesh(inv, n0, n1, n2), (T*)mesh);
  return launch_status("facek_pme_spread");
}
template <typename T>
int green(const void* spec, int n0, int n1, int n2, const double* inv, double gp, double vol, const void* bmod,
          double* energy, void* conv, void* stream) {
  const int64_t total = (int64_t)n0 * n1 * (n2 / 2 + 1);
  green_k<T><<<ew_grid(total, 256), 256, 0, as_stream(stream)>>>((const T*)spec, n0, n1, n2,
                                                                 make_mesh(inv, n0, n1, n2), (T)gp, (T)vol,
                                                                 (const T*)bmod, energy, (T*)conv);
  return launch_status("facek_pme_green");
}
template <typename T>
int gather(const void* pos, const void* q, int64_t N, const double* inv, int n0, int n1, int n2, const void* pot,
           double scale, void* dq, void* dpos, void* stream) {
  if (N == 0) return FACEK_OK;
  gather_k<T><<<ew_grid(N, 128), 128, 0, as_stream(stream)>>>((const T*)pos, (const T*)q, N,
                                                              make_mesh(inv, n0, n1, n2), (const T*)pot, (T)scale,
                                                              (T*)dq, (T*)dpos);
  return launch_status("facek_pme_gather");
}
template <typename T>
int real_fwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* q, double gamma, double gp,
             double rcut, int64_t N, void* e_row, void* stream) {
  if (N == 0) return FACEK_OK;
  real_fwd_k<T><<<ew_grid(N, 128), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, (const T*)q, (T)gamma,
                                                                (T)gp, cut_value<T>(rcut), N, (T*)e_row);
  return launch_status("facek_coulomb_real_fwd");
}
template <typename T>
int real_bwd(const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* q, double gamma, double gp,
             double rcut, const void* g, int64_t N, void* dvec, int acc, void* dq, void* stream) {
  if (N == 0) return FACEK_OK;
  real_bwd_k<T><<<ew_grid(N, 128), 128, 0, as_stream(stream)>>>((const T*)vec, row_ptr, ej, (const T*)q, (T)gamma,
                                                                (T)gp, cut_value<T>(rcut), (const T*)g, N, (T*)dvec,
                                                                acc, (T*)dq);
  return launch_status("facek_coulomb_real_bwd");
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_pme_spread(int dtype, const void* pos, const void* q, int64_t N, const double* inv, int32_t n0,
                                int32_t n1, int32_t n2, void* mesh, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && n0 >= 4 && n1 >= 4 && n2 >= 4 && inv && mesh && (N == 0 || (pos && q)),
                  "facek_pme_spread: bad arguments (mesh dims must be >= 4)");
  return FACEK_DISPATCH(dtype, spread, pos, q, N, inv, n0, n1, n2, mesh, stream);
}
extern "C" int facek_pme_green(int dtype, const void* spectrum, int32_t n0, int32_t n1, int32_t n2, const double* inv,
                               double gp, double volume, const void* bmod, double* energy, void* conv, void* stream) {
  FACEK_CHECK_ARG(spectrum && inv && bmod && energy && conv && n0 > 0 && n1 > 0 && n2 > 0 && volume > 0 && gp > 0,
                  "facek_pme_green: bad arguments");
  return FACEK_DISPATCH(dtype, green, spectrum, n0, n1, n2, inv, gp, volume, bmod, energy, conv, stream);
}
extern "C" int facek_pme_gather(int dtype, const void* pos, const void* q, int64_t N, const double* inv, int32_t n0,
                                int32_t n1, int32_t n2, const void* potential, double scale, void* dq, void* dpos,
                                void* stream) {
  FACEK_CHECK_ARG(N >= 0 && inv && potential && (N == 0 || (pos && q && dq && dpos)), "facek_pme_gather: bad args");
  return FACEK_DISPATCH(dtype, gather, pos, q, N, inv, n0, n1, n2, potential, scale, dq, dpos, stream);
}
extern "C" int facek_coulomb_real_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej,
                                      const void* q, double gamma, double gp, double r_cut, int64_t N, void* e_row,
                                      void* stream) {
  FACEK_CHECK_ARG(N >= 0 && gamma > 0 && gp > 0 && (N == 0 || (vec && row_ptr && ej && q && e_row)),
                  "facek_coulomb_real_fwd: bad arguments");
  return FACEK_DISPATCH(dtype, real_fwd, vec, row_ptr, ej, q, gamma, gp, r_cut, N, e_row, stream);
}
extern "C" int facek_coulomb_real_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej,
                                      const void* q, double gamma, double gp, double r_cut, const void* g_row,
                                      int64_t N, void* dvec, int32_t accumulate, void* dq, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && gamma > 0 && gp > 0 && (N == 0 || (vec && row_ptr && ej && q && g_row && dvec && dq)),
                  "facek_coulomb_real_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, real_bwd, vec, row_ptr, ej, q, gamma, gp, r_cut, g_row, N, dvec, accumulate, dq,
                        stream);
}
