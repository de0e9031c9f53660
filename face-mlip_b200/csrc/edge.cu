// Edge-level kernels of the FACE engine (face-mlip face/model.py:665-679, :460-534):
//   edge vectors and the force gather, symmetric monomials Y(u), the radial basis x radial MLP with
//   forward-mode dphi/dr (or the cubic Hermite spline), directional edge messages, transport sums.
// All scatter-to-neighbour adjoints use the reverse-edge index of the symmetric neighbour list (gathers,
// no atomics, deterministic).
#include "common.cuh"
#include "radial.cuh"

namespace facek {
namespace {

constexpr int NX = 20;

// ------------------------------------------------------------------------------------------ geometry
template <typename T>
__global__ void edge_vec_k(const T* __restrict__ pos, const int32_t* __restrict__ ei, const int32_t* __restrict__ ej,
                           const T* __restrict__ shift, T* __restrict__ vec, int64_t E) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = ei[e], j = ej[e];
#pragma unroll
    for (int d = 0; d < 3; d++) vec[e * 3 + d] = (pos[j * 3 + d] - pos[i * 3 + d]) + shift[e * 3 + d];
  }
}

// dpos[k] = sum_{e in row k} (dvec[rev e] - dvec[e])
template <typename T>
__global__ void edge_vec_bwd_k(const T* __restrict__ dvec, const int32_t* __restrict__ row_ptr,
                               const int32_t* __restrict__ rev, int64_t N, T* __restrict__ dpos) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < N; k += (int64_t)gridDim.x * blockDim.x) {
    T g0 = 0, g1 = 0, g2 = 0;
    for (int e = row_ptr[k]; e < row_ptr[k + 1]; e++) {
      const int64_t r = rev[e];
      g0 += dvec[r * 3 + 0] - dvec[(int64_t)e * 3 + 0];
      g1 += dvec[r * 3 + 1] - dvec[(int64_t)e * 3 + 1];
      g2 += dvec[r * 3 + 2] - dvec[(int64_t)e * 3 + 2];
    }
    dpos[k * 3 + 0] = g0;
    dpos[k * 3 + 1] = g1;
    dpos[k * 3 + 2] = g2;
  }
}

template <typename T>
__device__ __forceinline__ void monomials(T x, T y, T z, T* Y) {
  Y[0] = T(1); Y[1] = x; Y[2] = y; Y[3] = z;
  Y[4] = x * x; Y[5] = y * y; Y[6] = z * z; Y[7] = x * y; Y[8] = x * z; Y[9] = y * z;
  Y[10] = x * x * x; Y[11] = y * y * y; Y[12] = z * z * z; Y[13] = x * x * y; Y[14] = x * x * z;
  Y[15] = x * y * y; Y[16] = y * y * z; Y[17] = x * z * z; Y[18] = y * z * z; Y[19] = x * y * z;
}

// gradient of the 20 monomials w.r.t. u
template <typename T>
__device__ __forceinline__ void monomials_bwd(T x, T y, T z, const T* g, T& ux, T& uy, T& uz) {
  ux = g[1] + 2 * x * g[4] + y * g[7] + z * g[8] + 3 * x * x * g[10] + 2 * x * y * g[13] + 2 * x * z * g[14] +
       y * y * g[15] + z * z * g[17] + y * z * g[19];
  uy = g[2] + 2 * y * g[5] + x * g[7] + z * g[9] + 3 * y * y * g[11] + x * x * g[13] + 2 * x * y * g[15] +
       2 * y * z * g[16] + z * z * g[18] + x * z * g[19];
  uz = g[3] + 2 * z * g[6] + x * g[8] + y * g[9] + 3 * z * z * g[12] + x * x * g[14] + y * y * g[16] +
       2 * x * z * g[17] + 2 * y * z * g[18] + x * y * g[19];
}

// du -> dvec for u = vec / |vec|
template <typename T>
__device__ __forceinline__ void unit_bwd(T ux, T uy, T uz, T r, T gx, T gy, T gz, T& dx, T& dy, T& dz) {
  const T ud = ux * gx + uy * gy + uz * gz;
  dx = (gx - ux * ud) / r;
  dy = (gy - uy * ud) / r;
  dz = (gz - uz * ud) / r;
}

template <typename T>
__global__ void edge_sym_k(const T* __restrict__ vec, T* __restrict__ Y, int64_t E) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    T y[NX];
    monomials(vx / r, vy / r, vz / r, y);
#pragma unroll
    for (int x = 0; x < NX; x++) Y[e * NX + x] = y[x];
  }
}

// fp32: five lanes per edge, each storing one 16-byte piece (monomials 4q .. 4q+3) of the edge's 80-byte row, so a
// warp's stores are contiguous (a thread per edge wrote 20 scalars at an 80-byte lane stride).  Each lane evaluates
// all 20 monomials (a few dozen multiplies) and picks its piece with static indices.
__global__ void edge_sym5_k(const float* __restrict__ vec, float4* __restrict__ Y, int64_t total) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / 5;
    const int q = (int)(t - e * 5);
    const float vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const float r = sqrtf(vx * vx + vy * vy + vz * vz);
    float y[NX];
    monomials(vx / r, vy / r, vz / r, y);
    float4 o;
    switch (q) {
      case 0: o = make_float4(y[0], y[1], y[2], y[3]); break;
      case 1: o = make_float4(y[4], y[5], y[6], y[7]); break;
      case 2: o = make_float4(y[8], y[9], y[10], y[11]); break;
      case 3: o = make_float4(y[12], y[13], y[14], y[15]); break;
      default: o = make_float4(y[16], y[17], y[18], y[19]); break;
    }
    Y[t] = o;
  }
}

template <typename T>
__global__ void edge_sym_bwd_k(const T* __restrict__ vec, const T* __restrict__ dY, T* __restrict__ dvec, int acc,
                               int64_t E) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    const T ux = vx / r, uy = vy / r, uz = vz / r;
    T g[NX];
#pragma unroll
    for (int x = 0; x < NX; x++) g[x] = dY[e * NX + x];
    T gx, gy, gz, dx, dy, dz;
    monomials_bwd(ux, uy, uz, g, gx, gy, gz);
    unit_bwd(ux, uy, uz, r, gx, gy, gz, dx, dy, dz);
    if (acc) {
      dvec[e * 3] += dx; dvec[e * 3 + 1] += dy; dvec[e * 3 + 2] += dz;
    } else {
      dvec[e * 3] = dx; dvec[e * 3 + 1] = dy; dvec[e * 3 + 2] = dz;
    }
  }
}

// ------------------------------------------------------------------------------------------ radial
template <typename T, int NBMAX, int HMAX, int BMAX>
__global__ void __launch_bounds__(128) radial_mlp_k(const T* __restrict__ vec, const int32_t* __restrict__ ei,
                                                    const int32_t* __restrict__ ej, const int32_t* __restrict__ zidx,
                                                    int n_el, T rc, int nb, int H, int B, const T* __restrict__ w1,
                                                    const T* __restrict__ b1, const T* __restrict__ pair,
                                                    const T* __restrict__ w2, const T* __restrict__ b2,
                                                    const T* __restrict__ w3, const T* __restrict__ b3,
                                                    T* __restrict__ phi, T* __restrict__ dphidr, int64_t E) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sW1 = reinterpret_cast<T*>(smem_raw);   // H x nb
  T* sB1 = sW1 + H * nb;                      // H
  T* sPair = sB1 + H;                         // n_el^2 x H
  T* sW2 = sPair + n_el * n_el * H;           // H x H
  T* sB2 = sW2 + H * H;                       // H
  T* sW3 = sB2 + H;                           // B x H
  T* sB3 = sW3 + B * H;                       // B
  for (int q = threadIdx.x; q < H * nb; q += blockDim.x) sW1[q] = w1[q];
  for (int q = threadIdx.x; q < H; q += blockDim.x) { sB1[q] = b1[q]; sB2[q] = b2[q]; }
  for (int q = threadIdx.x; q < n_el * n_el * H; q += blockDim.x) sPair[q] = pair[q];
  for (int q = threadIdx.x; q < H * H; q += blockDim.x) sW2[q] = w2[q];
  for (int q = threadIdx.x; q < B * H; q += blockDim.x) sW3[q] = w3[q];
  for (int q = threadIdx.x; q < B; q += blockDim.x) sB3[q] = b3[q];
  __syncthreads();
  const T c = sqrt(T(2) / rc);
  const T pi = T(3.14159265358979323846);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    T env, denv;
    envelope(r, rc, env, denv);
    T rb[NBMAX], drb[NBMAX];
#pragma unroll
    for (int n = 0; n < NBMAX; n++) {
      if (n < nb) {
        const T f = T(n + 1) * pi / rc;
        T s, co;
        s = sin(f * r);
        co = cos(f * r);
        const T bes = s / r * c;
        const T dbes = (f * co / r - s / (r * r)) * c;
        rb[n] = bes * env;
        drb[n] = dbes * env + bes * denv;
      } else {
        rb[n] = 0;
        drb[n] = 0;
      }
    }
    const T* prow = sPair + (zidx[ei[e]] * n_el + zidx[ej[e]]) * H;
    T a1[HMAX], da1[HMAX];
#pragma unroll
    for (int h = 0; h < HMAX; h++) {
      if (h < H) {
        T z = sB1[h] + prow[h], dz = 0;
#pragma unroll
        for (int n = 0; n < NBMAX; n++)
          if (n < nb) {
            z += sW1[h * nb + n] * rb[n];
            dz += sW1[h * nb + n] * drb[n];
          }
        const T s = sigmoid(z);
        a1[h] = z * s;
        da1[h] = s * (T(1) + z * (T(1) - s)) * dz;
      } else {
        a1[h] = 0;
        da1[h] = 0;
      }
    }
    T z3[BMAX], dz3[BMAX];
#pragma unroll
    for (int b = 0; b < BMAX; b++) { z3[b] = 0; dz3[b] = 0; }
    // layer 2 four output neurons at a time: 8 independent FMA chains, weights read as broadcasts
    for (int o0 = 0; o0 < H; o0 += 4) {
      T z[4], dz[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        z[j] = (o0 + j < H) ? sB2[o0 + j] : T(0);
        dz[j] = 0;
      }
#pragma unroll
      for (int h = 0; h < HMAX; h++)
        if (h < H) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const T w = (o0 + j < H) ? sW2[(o0 + j) * H + h] : T(0);
            z[j] += w * a1[h];
            dz[j] += w * da1[h];
          }
        }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        if (o0 + j < H) {
          const T sg = sigmoid(z[j]);
          const T a2 = z[j] * sg, da2 = sg * (T(1) + z[j] * (T(1) - sg)) * dz[j];
#pragma unroll
          for (int b = 0; b < BMAX; b++)
            if (b < B) {
              z3[b] += sW3[b * H + o0 + j] * a2;
              dz3[b] += sW3[b * H + o0 + j] * da2;
            }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < BMAX; b++)
      if (b < B) {
        const T v = z3[b] + sB3[b];
        phi[e * B + b] = v * env;
        dphidr[e * B + b] = dz3[b] * env + v * denv;
      }
  }
}

// Wide output layer (B > 32: the CP form's B + 4C radial functions, face/model.py:449, and the non-factorised
// block's 4C or 8C, face/model.py:130): both hidden layers and their r-tangents stay in registers, and the output
// rows of W3 are read as warp-uniform broadcasts from global memory (L1-resident) one output at a time.
template <typename T, int NBMAX, int HMAX>
__global__ void __launch_bounds__(128) radial_wide_k(const T* __restrict__ vec, const int32_t* __restrict__ ei,
                                                     const int32_t* __restrict__ ej, const int32_t* __restrict__ zidx,
                                                     int n_el, T rc, int nb, int H, int B, const T* __restrict__ w1,
                                                     const T* __restrict__ b1, const T* __restrict__ pair,
                                                     const T* __restrict__ w2, const T* __restrict__ b2,
                                                     const T* __restrict__ w3, const T* __restrict__ b3,
                                                     T* __restrict__ phi, T* __restrict__ dphidr, int64_t E) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sW1 = reinterpret_cast<T*>(smem_raw);   // H x nb
  T* sB1 = sW1 + H * nb;                      // H
  T* sPair = sB1 + H;                         // n_el^2 x H
  T* sW2 = sPair + n_el * n_el * H;           // H x H
  T* sB2 = sW2 + H * H;                       // H
  for (int q = threadIdx.x; q < H * nb; q += blockDim.x) sW1[q] = w1[q];
  for (int q = threadIdx.x; q < H; q += blockDim.x) { sB1[q] = b1[q]; sB2[q] = b2[q]; }
  for (int q = threadIdx.x; q < n_el * n_el * H; q += blockDim.x) sPair[q] = pair[q];
  for (int q = threadIdx.x; q < H * H; q += blockDim.x) sW2[q] = w2[q];
  __syncthreads();
  const T c = sqrt(T(2) / rc);
  const T pi = T(3.14159265358979323846);
  // every thread runs the same number of loop trips so the output loop's W3 reads stay warp-uniform
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e0 = (int64_t)blockIdx.x * blockDim.x; e0 < E; e0 += stride) {
    const int64_t e = e0 + threadIdx.x;
    const bool live = e < E;
    const int64_t ee = live ? e : E - 1;
    const T vx = vec[ee * 3], vy = vec[ee * 3 + 1], vz = vec[ee * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    T env, denv;
    envelope(r, rc, env, denv);
    T rb[NBMAX], drb[NBMAX];
#pragma unroll
    for (int n = 0; n < NBMAX; n++) {
      rb[n] = 0;
      drb[n] = 0;
      if (n < nb) {
        const T f = T(n + 1) * pi / rc;
        const T s = sin(f * r), co = cos(f * r);
        const T bes = s / r * c;
        const T dbes = (f * co / r - s / (r * r)) * c;
        rb[n] = bes * env;
        drb[n] = dbes * env + bes * denv;
      }
    }
    const T* prow = sPair + (zidx[ei[ee]] * n_el + zidx[ej[ee]]) * H;
    T a1[HMAX], da1[HMAX];
#pragma unroll
    for (int h = 0; h < HMAX; h++) {
      a1[h] = 0;
      da1[h] = 0;
      if (h < H) {
        T z = sB1[h] + prow[h], dz = 0;
#pragma unroll
        for (int n = 0; n < NBMAX; n++)
          if (n < nb) {
            z += sW1[h * nb + n] * rb[n];
            dz += sW1[h * nb + n] * drb[n];
          }
        const T sg = sigmoid(z);
        a1[h] = z * sg;
        da1[h] = sg * (T(1) + z * (T(1) - sg)) * dz;
      }
    }
    T a2[HMAX], da2[HMAX];
#pragma unroll
    for (int o = 0; o < HMAX; o++) {
      a2[o] = 0;
      da2[o] = 0;
      if (o < H) {
        T z = sB2[o], dz = 0;
#pragma unroll
        for (int h = 0; h < HMAX; h++)
          if (h < H) {
            z += sW2[o * H + h] * a1[h];
            dz += sW2[o * H + h] * da1[h];
          }
        const T sg = sigmoid(z);
        a2[o] = z * sg;
        da2[o] = sg * (T(1) + z * (T(1) - sg)) * dz;
      }
    }
#pragma unroll 1
    for (int b = 0; b < B; b++) {
      const T* wrow = w3 + (int64_t)b * H;
      T z = __ldg(b3 + b), dz = 0;
#pragma unroll
      for (int h = 0; h < HMAX; h++)
        if (h < H) {
          const T w = __ldg(wrow + h);
          z += w * a2[h];
          dz += w * da2[h];
        }
      if (live) {
        phi[e * B + b] = z * env;
        dphidr[e * B + b] = dz * env + z * denv;
      }
    }
  }
}

template <typename T, int BMAX>
__global__ void radial_spline_k(const T* __restrict__ vec, const int32_t* __restrict__ ei,
                                const int32_t* __restrict__ ej, const int32_t* __restrict__ zidx, int n_el, T rc,
                                int G, T dr, int B, const T* __restrict__ Tab, const T* __restrict__ dTab,
                                T* __restrict__ phi, T* __restrict__ dphidr, int64_t E) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    T env, denv;
    envelope(r, rc, env, denv);
    T x = r / dr;
    T dxdr = T(1) / dr;
    if (x < T(0)) { x = 0; dxdr = 0; }
    if (x > T(G - 1)) { x = T(G - 1); dxdr = 0; }
    int i = (int)floor(x);
    if (i > G - 2) i = G - 2;
    const T t = x - T(i), t2 = t * t, t3 = t2 * t;
    const T h00 = 2 * t3 - 3 * t2 + 1, h10 = t3 - 2 * t2 + t, h01 = -2 * t3 + 3 * t2, h11 = t3 - t2;
    const T g00 = 6 * t2 - 6 * t, g10 = 3 * t2 - 4 * t + 1, g01 = -6 * t2 + 6 * t, g11 = 3 * t2 - 2 * t;
    const int64_t base = ((int64_t)(zidx[ei[e]] * n_el + zidx[ej[e]]) * G + i) * B;
    for (int b = 0; b < B; b++) {
      const T p0 = Tab[base + b], p1 = Tab[base + B + b];
      const T m0 = dTab[base + b] * dr, m1 = dTab[base + B + b] * dr;
      const T v = h00 * p0 + h10 * m0 + h01 * p1 + h11 * m1;
      const T dv = (g00 * p0 + g10 * m0 + g01 * p1 + g11 * m1) * dxdr;
      phi[e * B + b] = v * env;
      dphidr[e * B + b] = dv * env + v * denv;
    }
  }
}

// fp32, B % 4 == 0: the same interpolation with one thread per (edge, 4 consecutive basis functions), so that
// consecutive lanes read consecutive 16-byte pieces of the two grid rows of T and dT and write phi, dphi/dr as fully
// coalesced 16-byte vectors (the scalar kernel above gives each thread a whole edge: 4 B strided stores per lane).
// The B/4 threads of an edge recompute r and the envelope, which costs a few FLOPs against 32 B of output each.
__global__ void radial_spline4_k(const float* __restrict__ vec, const int32_t* __restrict__ ei,
                                 const int32_t* __restrict__ ej, const int32_t* __restrict__ zidx, int n_el, float rc,
                                 int G, float dr, int B4, const float4* __restrict__ Tab,
                                 const float4* __restrict__ dTab, float4* __restrict__ phi,
                                 float4* __restrict__ dphidr, int64_t EB4) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < EB4; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / B4;
    const int q = (int)(t - e * B4);
    const float vx = __ldg(vec + e * 3), vy = __ldg(vec + e * 3 + 1), vz = __ldg(vec + e * 3 + 2);
    const float r = sqrtf(vx * vx + vy * vy + vz * vz);
    float env, denv;
    envelope(r, rc, env, denv);
    float x = r / dr;
    float dxdr = 1.f / dr;
    if (x < 0.f) { x = 0.f; dxdr = 0.f; }
    if (x > float(G - 1)) { x = float(G - 1); dxdr = 0.f; }
    int i = (int)floorf(x);
    if (i > G - 2) i = G - 2;
    const float u = x - float(i), u2 = u * u, u3 = u2 * u;
    const float h00 = 2 * u3 - 3 * u2 + 1, h10 = u3 - 2 * u2 + u, h01 = -2 * u3 + 3 * u2, h11 = u3 - u2;
    const float g00 = 6 * u2 - 6 * u, g10 = 3 * u2 - 4 * u + 1, g01 = -6 * u2 + 6 * u, g11 = 3 * u2 - 2 * u;
    const int64_t base = ((int64_t)(__ldg(zidx + __ldg(ei + e)) * n_el + __ldg(zidx + __ldg(ej + e))) * G + i) * B4 + q;
    const float4 p0 = __ldg(Tab + base), p1 = __ldg(Tab + base + B4);
    const float4 d0 = __ldg(dTab + base), d1 = __ldg(dTab + base + B4);
    const float a0[4] = {p0.x, p0.y, p0.z, p0.w}, a1[4] = {p1.x, p1.y, p1.z, p1.w};
    const float b0[4] = {d0.x, d0.y, d0.z, d0.w}, b1[4] = {d1.x, d1.y, d1.z, d1.w};
    float o[4], od[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float m0 = b0[k] * dr, m1 = b1[k] * dr;
      const float v = h00 * a0[k] + h10 * m0 + h01 * a1[k] + h11 * m1;
      const float dv = (g00 * a0[k] + g10 * m0 + g01 * a1[k] + g11 * m1) * dxdr;
      o[k] = v * env;
      od[k] = dv * env + v * denv;
    }
    phi[t] = make_float4(o[0], o[1], o[2], o[3]);
    dphidr[t] = make_float4(od[0], od[1], od[2], od[3]);
  }
}

template <typename T>
__global__ void radial_bwd_k(const T* __restrict__ vec, const T* __restrict__ dphi, const T* __restrict__ dphidr,
                             int B, T* __restrict__ dvec, int acc, int64_t E) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
    const T r = sqrt(vx * vx + vy * vy + vz * vz);
    T s = 0;
    for (int b = 0; b < B; b++) s += dphi[e * B + b] * dphidr[e * B + b];
    const T gx = s * vx / r, gy = s * vy / r, gz = s * vz / r;
    if (acc) {
      dvec[e * 3] += gx; dvec[e * 3 + 1] += gy; dvec[e * 3 + 2] += gz;
    } else {
      dvec[e * 3] = gx; dvec[e * 3 + 1] = gy; dvec[e * 3 + 2] = gz;
    }
  }
}

// fp32, B/4 a power of two: B/4 consecutive lanes per edge, each a 16-byte piece of dphi and dphi/dr (a warp reads
// contiguous 512-byte spans), the partial dot products joined by shuffles within the lane group.  Groups never
// straddle a warp or the end of the range: the total E*B/4, the block size and the grid stride are all multiples of
// the group size, so every lane a shuffle names is active.
__global__ void radial_bwd4_k(const float* __restrict__ vec, const float4* __restrict__ dphi,
                              const float4* __restrict__ dphidr, int B4, float* __restrict__ dvec, int acc,
                              int64_t total) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(dphi + t), b = __ldg(dphidr + t);
    float s = fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
    const unsigned m = __activemask();
    for (int o = 1; o < B4; o <<= 1) s += __shfl_xor_sync(m, s, o);
    if ((t & (B4 - 1)) == 0) {
      const int64_t e = t / B4;
      const float vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
      const float r = sqrtf(vx * vx + vy * vy + vz * vz);
      const float gx = s * vx / r, gy = s * vy / r, gz = s * vz / r;
      if (acc) {
        dvec[e * 3] += gx; dvec[e * 3 + 1] += gy; dvec[e * 3 + 2] += gz;
      } else {
        dvec[e * 3] = gx; dvec[e * 3 + 1] = gy; dvec[e * 3 + 2] = gz;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------ messages
template <typename T>
__global__ void edge_msg_k(const T* __restrict__ Y, const int32_t* __restrict__ ei, const int32_t* __restrict__ ej,
                           const T* __restrict__ TJ, const T* __restrict__ TI, int nc, int K, int64_t N,
                           T* __restrict__ msg, int64_t EK) {
  const int64_t NK = N * K;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < EK; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = q / K;
    const int k = (int)(q - e * K);
    const T* tj = TJ + (int64_t)ej[e] * K + k;
    T s = 0;
    if (TI) {
      const T* ti = TI + (int64_t)ei[e] * K + k;
      for (int c = 0; c < nc; c++) s += Y[e * NX + c] * (tj[c * NK] + ti[c * NK]);
    } else {
      for (int c = 0; c < nc; c++) s += Y[e * NX + c] * tj[c * NK];
    }
    msg[q] = s;
  }
}

// fp32, K = 32, nc <= 10: eight lanes per edge (a float4 of k each), four edges per warp; the component loop is
// unrolled so that all of an edge's table rows are requested at once, and no index division is needed
__global__ void __launch_bounds__(256) edge_msg32_k(const float* __restrict__ Y, const int32_t* __restrict__ ei,
                                                    const int32_t* __restrict__ ej, const float4* __restrict__ TJ,
                                                    const float4* __restrict__ TI, int nc, int64_t N,
                                                    float4* __restrict__ msg, int64_t E) {
  const int64_t NK4 = N * 8;                                   // one component plane, in float4
  const int sub = threadIdx.x & 7;
  for (int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 3; e < E;
       e += ((int64_t)gridDim.x * blockDim.x) >> 3) {
    const float4* tj = TJ + (int64_t)ej[e] * 8 + sub;
    const float4* ti = TI ? TI + (int64_t)ei[e] * 8 + sub : nullptr;
    const float* y = Y + e * NX;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 10; c++) {
      if (c < nc) {
        float4 t = __ldg(tj + c * NK4);
        if (ti) {
          const float4 u = __ldg(ti + c * NK4);
          t.x += u.x;
          t.y += u.y;
          t.z += u.z;
          t.w += u.w;
        }
        const float yc = __ldg(y + c);
        s.x += yc * t.x;
        s.y += yc * t.y;
        s.z += yc * t.z;
        s.w += yc * t.w;
      }
    }
    msg[e * 8 + sub] = s;
  }
}

// dY[e, c<nc] (+)= sum_k dmsg[e,k] (TJ[ej,c,k] + TI[ei,c,k]); one warp per edge
template <typename T>
__global__ void edge_msg_bwd_dy_k(const int32_t* __restrict__ ei, const int32_t* __restrict__ ej,
                                  const T* __restrict__ TJ, const T* __restrict__ TI, const T* __restrict__ dmsg,
                                  int nc, int K, int64_t N, T* __restrict__ dY, int acc, int64_t E) {
  const int64_t NK = N * K;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t e = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); e < E; e += warps) {
    T part[10];
#pragma unroll
    for (int c = 0; c < 10; c++) part[c] = 0;
    const T* tj = TJ + (int64_t)ej[e] * K;
    const T* ti = TI ? TI + (int64_t)ei[e] * K : nullptr;
    for (int k = lane; k < K; k += 32) {
      const T g = dmsg[e * K + k];
#pragma unroll
      for (int c = 0; c < 10; c++)
        if (c < nc) part[c] += g * (tj[c * NK + k] + (ti ? ti[c * NK + k] : T(0)));
    }
#pragma unroll
    for (int c = 0; c < 10; c++) {
      T v = part[c];
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      part[c] = v;
    }
    if (lane < nc) {
      T v = 0;
#pragma unroll
      for (int c = 0; c < 10; c++)
        if (c == lane) v = part[c];
      if (acc)
        dY[e * NX + lane] += v;
      else
        dY[e * NX + lane] = v;
    }
    if (!acc && lane >= nc && lane < NX) dY[e * NX + lane] = 0;
  }
}

// dTJ[c,a,k] = sum_{e in row a} Y[rev e, c] dmsg[rev e, k];  dTI[c,a,k] = sum_{e in row a} Y[e, c] dmsg[e, k]
template <typename T>
__global__ void edge_msg_bwd_tables_k(const T* __restrict__ Y, const T* __restrict__ dmsg,
                                      const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ rev, int nc,
                                      int K, T* __restrict__ dTJ, T* __restrict__ dTI, int64_t NK) {
  // q = a*K + k indexes (atom, channel); plane c of a (nc, N, K) table starts at c*NK
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < NK; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t a = q / K;
    const int k = (int)(q - a * K);
    T sj[10], si[10];
#pragma unroll
    for (int c = 0; c < 10; c++) { sj[c] = 0; si[c] = 0; }
    const int e1 = row_ptr[a + 1];
#pragma unroll 2
    for (int e = row_ptr[a]; e < e1; e++) {
      const int64_t r = rev[e];
      const T gr = dmsg[r * K + k];
      const T ge = dmsg[(int64_t)e * K + k];
      T yr[10], ye[10];
      if constexpr (sizeof(T) == 4) {          // Y rows are 80 B (16-byte aligned): the first ten as 4 + 4 + 2
        const float4* r4 = reinterpret_cast<const float4*>(Y + r * NX);
        const float4* e4 = reinterpret_cast<const float4*>(Y + (int64_t)e * NX);
        const float4 ra = __ldg(r4), rb = __ldg(r4 + 1), ea = __ldg(e4), eb = __ldg(e4 + 1);
        const float2 rc = __ldg(reinterpret_cast<const float2*>(r4 + 2));
        const float2 ec = __ldg(reinterpret_cast<const float2*>(e4 + 2));
        yr[0] = ra.x; yr[1] = ra.y; yr[2] = ra.z; yr[3] = ra.w; yr[4] = rb.x; yr[5] = rb.y; yr[6] = rb.z;
        yr[7] = rb.w; yr[8] = rc.x; yr[9] = rc.y;
        ye[0] = ea.x; ye[1] = ea.y; ye[2] = ea.z; ye[3] = ea.w; ye[4] = eb.x; ye[5] = eb.y; ye[6] = eb.z;
        ye[7] = eb.w; ye[8] = ec.x; ye[9] = ec.y;
      } else {
#pragma unroll
        for (int c = 0; c < 10; c++) {
          yr[c] = Y[r * NX + c];
          ye[c] = Y[(int64_t)e * NX + c];
        }
      }
#pragma unroll
      for (int c = 0; c < 10; c++)
        if (c < nc) {
          sj[c] += yr[c] * gr;
          si[c] += ye[c] * ge;
        }
    }
#pragma unroll
    for (int c = 0; c < 10; c++)
      if (c < nc) {
        dTJ[c * NK + q] = sj[c];
        if (dTI) dTI[c * NK + q] = si[c];
      }
  }
}

// ------------------------------------------------------------------------------------------ transport
// storage row of transport output o (see facek.h): V_a -> 2a, (M u)_a -> 2a+1, M_s -> 6+2s, sym(uV)_s -> 7+2s
__host__ __device__ constexpr int trow(int o) {
  return o < 3 ? 2 * o : (o < 6 ? 2 * (o - 3) + 1 : (o < 12 ? 6 + 2 * (o - 6) : 7 + 2 * (o - 12)));
}
__host__ __device__ constexpr int s2i(int a, int b) { return a == b ? a : 2 + a + b; }
__host__ __device__ constexpr int pair_p(int s) { return s < 3 ? s : (s == 5 ? 1 : 0); }
__host__ __device__ constexpr int pair_q(int s) { return s < 3 ? s : (s == 3 ? 1 : 2); }

template <typename T>
__device__ __forceinline__ void transport_f(T ux, T uy, T uz, const T g[9], T f[18]) {
  const T u[3] = {ux, uy, uz};
#pragma unroll
  for (int a = 0; a < 3; a++) f[a] = g[a];
#pragma unroll
  for (int a = 0; a < 3; a++) {
    T s = 0;
#pragma unroll
    for (int b = 0; b < 3; b++) s += g[3 + s2i(a, b)] * u[b];
    f[3 + a] = s;
  }
#pragma unroll
  for (int s = 0; s < 6; s++) f[6 + s] = g[3 + s];
#pragma unroll
  for (int s = 0; s < 6; s++) {
    const int p = pair_p(s), q = pair_q(s);
    f[12 + s] = p == q ? u[p] * g[p] : T(0.5) * (u[p] * g[q] + u[q] * g[p]);
  }
}

constexpr int TR_TILE = 16;

// storage row r (= trow(o)) of atom i in the two transport planes, as one offset from the start of plane 1:
// plane 1 (3, N, 2, BKd) holds rows 0..5 as (comp r/2, t r%2); plane 2 (6, N, 2, BKd) rows 6..17 likewise
__host__ __device__ inline int64_t plane_off(int r, int64_t i, int64_t N, int BKd) {
  if (r < 6) return (((int64_t)(r >> 1) * N + i) * 2 + (r & 1)) * BKd;
  const int s = r - 6;
  return 6 * N * (int64_t)BKd + (((int64_t)(s >> 1) * N + i) * 2 + (s & 1)) * BKd;
}

// CTA per row; thread (group of BQ b's, kd) accumulates BQ x 18 outputs; edges staged in shared memory
template <typename T, int BQ>
__global__ void __launch_bounds__(256) transport_fwd_k(const T* __restrict__ phi, const T* __restrict__ vec,
                                                       const int32_t* __restrict__ ej, const T* __restrict__ Gt,
                                                       const int32_t* __restrict__ row_ptr, T* __restrict__ DT,
                                                       int64_t N, int B, int Kd) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sP = reinterpret_cast<T*>(smem_raw);   // TR_TILE x B
  T* sF = sP + TR_TILE * B;                  // TR_TILE x Kd x 18
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int nbq = B / BQ;
  const int kd = tid % Kd, bq = tid / Kd;
  const bool active = bq < nbq;
  const int BKd = B * Kd;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    const int64_t e0 = row_ptr[i];
    const int deg = row_ptr[i + 1] - row_ptr[i];
    T acc[BQ][18];
#pragma unroll
    for (int a = 0; a < BQ; a++)
#pragma unroll
      for (int o = 0; o < 18; o++) acc[a][o] = 0;
    for (int t0 = 0; t0 < deg; t0 += TR_TILE) {
      const int nt = min(TR_TILE, deg - t0);
      __syncthreads();
      for (int q = tid; q < nt * B; q += nthr) sP[q] = phi[(e0 + t0) * B + q];
      for (int q = tid; q < nt * Kd; q += nthr) {
        const int t = q / Kd, k = q - t * Kd;
        const int64_t e = e0 + t0 + t;
        const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
        const T r = sqrt(vx * vx + vy * vy + vz * vz);
        const T* gj = Gt + (int64_t)ej[e] * Kd + k;
        T g[9], f[18];
#pragma unroll
        for (int c = 0; c < 9; c++) g[c] = gj[c * N * Kd];
        transport_f(vx / r, vy / r, vz / r, g, f);
        if constexpr (sizeof(T) == 4) {               // 8-byte stores and loads: (t*Kd+k)*18 floats is even
          float2* f2 = reinterpret_cast<float2*>(sF + (t * Kd + k) * 18);
#pragma unroll
          for (int o = 0; o < 9; o++) f2[o] = make_float2(f[2 * o], f[2 * o + 1]);
        } else {
#pragma unroll
          for (int o = 0; o < 18; o++) sF[(t * Kd + k) * 18 + o] = f[o];
        }
      }
      __syncthreads();
      if (active) {
        for (int t = 0; t < nt; t++) {
          T f[18];
          if constexpr (sizeof(T) == 4) {
            const float2* f2 = reinterpret_cast<const float2*>(sF + (t * Kd + kd) * 18);
#pragma unroll
            for (int o = 0; o < 9; o++) {
              const float2 v = f2[o];
              f[2 * o] = v.x;
              f[2 * o + 1] = v.y;
            }
          } else {
#pragma unroll
            for (int o = 0; o < 18; o++) f[o] = sF[(t * Kd + kd) * 18 + o];
          }
#pragma unroll
          for (int a = 0; a < BQ; a++) {
            const T p = sP[t * B + bq * BQ + a];
            if constexpr (sizeof(T) == 4) {
#pragma unroll
              for (int o = 0; o < 18; o += 2) ffma2(acc[a][o], acc[a][o + 1], p, p, f[o], f[o + 1]);
            } else {
#pragma unroll
              for (int o = 0; o < 18; o++) acc[a][o] += p * f[o];
            }
          }
        }
      }
    }
    if (active) {
#pragma unroll
      for (int o = 0; o < 18; o++) {
        T* out = DT + plane_off(trow(o), i, N, BKd);
#pragma unroll
        for (int a = 0; a < BQ; a++) out[(bq * BQ + a) * Kd + kd] = acc[a][o];
      }
    }
  }
}

// CTA per row with the row's 18 gradient rows (dT1/dT2 planes) staged in shared memory by cp.async, the next row
// prefetched into the second buffer; each edge is handled by KQ threads (KDT = 2 kd channels each).
template <typename T, int BMAX>
__global__ void __launch_bounds__(256) transport_bwd_k(const T* __restrict__ phi, const T* __restrict__ vec,
                                                       const int32_t* __restrict__ ej, const T* __restrict__ Gt,
                                                       const T* __restrict__ dT1, const T* __restrict__ dT2,
                                                       const int32_t* __restrict__ row_ptr,
                                                       T* __restrict__ dphi, T* __restrict__ dvec, int acc,
                                                       T* __restrict__ dGe, int64_t N, int B, int Kd, int KQ) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int BKd = B * Kd;
  T* sDb[2] = {reinterpret_cast<T*>(smem_raw), reinterpret_cast<T*>(smem_raw) + 18 * BKd};
  const int kq = tid % KQ, slot = tid / KQ, per_pass = nthr / KQ;
  auto issue = [&](T* sD, int64_t i) {
#pragma unroll 2
    for (int r = 0; r < 18; r++) {
      const int64_t off = plane_off(r, i, N, BKd);
      stage(sD + r * BKd, r < 6 ? dT1 + off : dT2 + (off - 6 * N * (int64_t)BKd), BKd, tid, nthr);
    }
    cp_async_commit();
  };
  int cur = 0;
  if ((int64_t)blockIdx.x < N) issue(sDb[0], blockIdx.x);
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    const int64_t inext = i + gridDim.x;
    if (inext < N) {
      issue(sDb[cur ^ 1], inext);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const T* sD = sDb[cur];
    const int64_t e0 = row_ptr[i];
    const int deg = row_ptr[i + 1] - row_ptr[i];
    for (int t0 = 0; t0 < deg; t0 += per_pass) {
      const int t = t0 + slot;
      const bool live = t < deg;
      const int64_t e = e0 + (live ? t : 0);
      const T vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
      const T r = sqrt(vx * vx + vy * vy + vz * vz);
      const T u[3] = {vx / r, vy / r, vz / r};
      constexpr int KDT = 2;
      T f[KDT][18], Pd[KDT][18];
      const T* gj = Gt + (int64_t)ej[e] * Kd;
#pragma unroll
      for (int q = 0; q < KDT; q++) {
        const int k = kq * KDT + q;
        T g[9];
#pragma unroll
        for (int c = 0; c < 9; c++) g[c] = k < Kd ? gj[c * N * Kd + k] : T(0);
        transport_f(u[0], u[1], u[2], g, f[q]);
#pragma unroll
        for (int o = 0; o < 18; o++) Pd[q][o] = 0;
      }
      // b outer (runtime), the 18 outputs unrolled: phi_b and its gradient stay scalars
      for (int b = 0; b < B; b++) {
        const T pb = live ? phi[e * B + b] : T(0);
        T dpb = 0;
        const T* rowb = sD + b * Kd + kq * KDT;
#pragma unroll
        for (int o = 0; o < 18; o++) {
          const T* row = rowb + (int64_t)trow(o) * BKd;
          T d2[KDT];
#pragma unroll
          for (int q = 0; q < KDT; q++) d2[q] = (kq * KDT + q < Kd) ? row[q] : T(0);
          dpb += d2[0] * f[0][o] + d2[1] * f[1][o];
#pragma unroll
          for (int q = 0; q < KDT; q++) Pd[q][o] += pb * d2[q];
        }
        for (int off = 1; off < KQ; off <<= 1) dpb += __shfl_xor_sync(0xffffffffu, dpb, off);
        if (live && kq == 0) dphi[e * B + b] = dpb;
      }
      // adjoint of f -> dV, dMs (per kd) and du
      T du[3] = {0, 0, 0};
#pragma unroll
      for (int q = 0; q < KDT; q++) {
        T dV[3], dM[6], g[9];
        const int kk = kq * KDT + q;
#pragma unroll
        for (int c = 0; c < 9; c++) g[c] = kk < Kd ? gj[c * N * Kd + kk] : T(0);     // reload (L1/L2 hit)
#pragma unroll
        for (int a = 0; a < 3; a++) dV[a] = Pd[q][a];
#pragma unroll
        for (int s = 0; s < 6; s++) dM[s] = Pd[q][6 + s];
#pragma unroll
        for (int a = 0; a < 3; a++)
#pragma unroll
          for (int b = 0; b < 3; b++) {
            dM[s2i(a, b)] += Pd[q][3 + a] * u[b];
            du[b] += Pd[q][3 + a] * g[3 + s2i(a, b)];
          }
#pragma unroll
        for (int s = 0; s < 6; s++) {
          const int pp = pair_p(s), qq = pair_q(s);
          const T w = Pd[q][12 + s];
          if (pp == qq) {
            du[pp] += w * g[pp];
            dV[pp] += w * u[pp];
          } else {
            du[pp] += T(0.5) * w * g[qq];
            du[qq] += T(0.5) * w * g[pp];
            dV[qq] += T(0.5) * w * u[pp];
            dV[pp] += T(0.5) * w * u[qq];
          }
        }
        const int k = kq * KDT + q;
        if (live && k < Kd) {
          T* dg = dGe + e * 9 * (int64_t)Kd + k;
#pragma unroll
          for (int a = 0; a < 3; a++) dg[a * Kd] = dV[a];
#pragma unroll
          for (int s = 0; s < 6; s++) dg[(3 + s) * Kd] = dM[s];
        }
      }
      for (int off = 1; off < KQ; off <<= 1)
#pragma unroll
        for (int d = 0; d < 3; d++) du[d] += __shfl_xor_sync(0xffffffffu, du[d], off);
      if (live && kq == 0) {
        T dx, dy, dz;
        unit_bwd(u[0], u[1], u[2], r, du[0], du[1], du[2], dx, dy, dz);
        if (acc) {
          dvec[e * 3] += dx; dvec[e * 3 + 1] += dy; dvec[e * 3 + 2] += dz;
        } else {
          dvec[e * 3] = dx; dvec[e * 3 + 1] = dy; dvec[e * 3 + 2] = dz;
        }
      }
    }
    __syncthreads();
    cur ^= 1;
  }
}

// Transport backward, two lanes per edge (fp32, B = BB, Kd a multiple of 8).  A 96-thread CTA takes one row (atom)
// at a time and stages its 18 gradient rows dT[o, i] (BB x Kd each) in shared memory.  Each lane of an edge's pair
// takes half of the kd channels; for each group of KQ = 2 it keeps g = Gt[:, j, kd..kd+1] (9 x 2), walks the 18
// outputs o and for each the BB rows dT[o, i, b, kd..kd+1] (8-byte broadcast reads; groups of 2 rather than 4 keep
// the live set under the 128-register cap of five CTAs per SM and the unrolled walk small enough for the
// instruction cache):
//   dphi[b] += dT . f_o,   P_o = sum_b phi[b] dT   ->   folded at once into dV, dM (per kd) and du
// and the pair adds its dphi and du halves with shuffles.  Same outputs as transport_bwd_k.  96 lanes = 48 edges
// per round (rows with more edges loop).
template <int BB>
__global__ void __launch_bounds__(96, 4) transport_bwd_lane_k(const float* __restrict__ phi,
                                                              const float* __restrict__ vec,
                                                              const int32_t* __restrict__ ej,
                                                              const float* __restrict__ Gt,
                                                              const float* __restrict__ dT1,
                                                              const float* __restrict__ dT2,
                                                              const int32_t* __restrict__ row_ptr,
                                                              float* __restrict__ dphi, float* __restrict__ dvec,
                                                              int acc, float* __restrict__ dGe, int64_t N, int Kd) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sD = reinterpret_cast<float*>(smem_raw);              // [o][b][kd], o in output order
  constexpr int KQ = 2;                                         // kd channels per group
  const int tid = threadIdx.x, half = tid & 1, slot = tid >> 1;
  const int BKd = BB * Kd;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    const int64_t e0 = row_ptr[i];
    const int deg = row_ptr[i + 1] - (int)e0;
    if (deg == 0) continue;
    __syncthreads();                                           // previous row's readers are done with sD
#pragma unroll 2
    for (int o = 0; o < 18; o++) {
      const int64_t off = plane_off(trow(o), i, N, BKd);
      stage(sD + o * BKd, trow(o) < 6 ? dT1 + off : dT2 + (off - 6 * N * (int64_t)BKd), BKd, tid, 96);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int t0 = 0; t0 < deg; t0 += 48) {
      if (t0 + slot >= deg) break;                             // pairs take this branch together
      const int64_t e = e0 + t0 + slot, j = ej[e];
      const float vx = vec[e * 3], vy = vec[e * 3 + 1], vz = vec[e * 3 + 2];
      const float r = sqrtf(vx * vx + vy * vy + vz * vz);
      const float u[3] = {vx / r, vy / r, vz / r};
      float p[BB], dp[BB][2];                                   // dp[b] as two partial sums (paired FMAs)
#pragma unroll
      for (int b = 0; b < BB; b += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(phi + e * BB + b));
        p[b] = v.x;
        p[b + 1] = v.y;
        p[b + 2] = v.z;
        p[b + 3] = v.w;
#pragma unroll
        for (int q = 0; q < 4; q++) dp[b + q][0] = dp[b + q][1] = 0.f;
      }
      float du[3] = {0.f, 0.f, 0.f};
      const int kh = Kd / 2;
#pragma unroll 1
      for (int k0 = half * kh; k0 < half * kh + kh; k0 += KQ) {
        float g[9][KQ], dG[9][KQ];
#pragma unroll
        for (int c = 0; c < 9; c++) {
          const float2 v = __ldg(reinterpret_cast<const float2*>(Gt + ((int64_t)c * N + j) * Kd + k0));
          g[c][0] = v.x;
          g[c][1] = v.y;
          dG[c][0] = dG[c][1] = 0.f;
        }
#pragma unroll
        for (int o = 0; o < 18; o++) {
          float f[KQ];
#pragma unroll
          for (int q = 0; q < KQ; q++) {
            if (o < 3) f[q] = g[o][q];
            else if (o < 6) {
              const int a = o - 3;
              f[q] = g[3 + s2i(a, 0)][q] * u[0] + g[3 + s2i(a, 1)][q] * u[1] + g[3 + s2i(a, 2)][q] * u[2];
            } else if (o < 12) f[q] = g[3 + (o - 6)][q];
            else {
              const int s = o - 12, pp = pair_p(s), qq = pair_q(s);
              f[q] = pp == qq ? u[pp] * g[pp][q] : 0.5f * (u[pp] * g[qq][q] + u[qq] * g[pp][q]);
            }
          }
          const float* rowp = sD + o * BKd + k0;
          float P[KQ] = {0.f, 0.f};
#pragma unroll
          for (int b = 0; b < BB; b++) {
            const float2 d = *reinterpret_cast<const float2*>(rowp + b * Kd);
            ffma2(dp[b][0], dp[b][1], d.x, d.y, f[0], f[1]);
            ffma2(P[0], P[1], p[b], p[b], d.x, d.y);
          }
#pragma unroll
          for (int q = 0; q < KQ; q++) {
            const float w = P[q];
            if (o < 3) dG[o][q] += w;
            else if (o < 6) {
              const int a = o - 3;
#pragma unroll
              for (int bb = 0; bb < 3; bb++) {
                dG[3 + s2i(a, bb)][q] += w * u[bb];
                du[bb] += w * g[3 + s2i(a, bb)][q];
              }
            } else if (o < 12) dG[3 + (o - 6)][q] += w;
            else {
              const int s = o - 12, pp = pair_p(s), qq = pair_q(s);
              if (pp == qq) {
                du[pp] += w * g[pp][q];
                dG[pp][q] += w * u[pp];
              } else {
                du[pp] += 0.5f * w * g[qq][q];
                du[qq] += 0.5f * w * g[pp][q];
                dG[qq][q] += 0.5f * w * u[pp];
                dG[pp][q] += 0.5f * w * u[qq];
              }
            }
          }
        }
        float* dg = dGe + e * 9 * (int64_t)Kd + k0;
#pragma unroll
        for (int c = 0; c < 9; c++) *reinterpret_cast<float2*>(dg + c * Kd) = make_float2(dG[c][0], dG[c][1]);
      }
      const unsigned pm = __activemask();
      float dps[BB];
#pragma unroll
      for (int b = 0; b < BB; b++) {
        dps[b] = dp[b][0] + dp[b][1];
        dps[b] += __shfl_xor_sync(pm, dps[b], 1);
      }
#pragma unroll
      for (int d = 0; d < 3; d++) du[d] += __shfl_xor_sync(pm, du[d], 1);
      if (half) continue;
#pragma unroll
      for (int b = 0; b < BB; b += 4)
        *reinterpret_cast<float4*>(dphi + e * BB + b) = make_float4(dps[b], dps[b + 1], dps[b + 2], dps[b + 3]);
      float dx, dy, dz;
      unit_bwd(u[0], u[1], u[2], r, du[0], du[1], du[2], dx, dy, dz);
      if (acc) {
        dvec[e * 3] += dx;
        dvec[e * 3 + 1] += dy;
        dvec[e * 3 + 2] += dz;
      } else {
        dvec[e * 3] = dx;
        dvec[e * 3 + 1] = dy;
        dvec[e * 3 + 2] = dz;
      }
    }
  }
}

// dGt[c, a, kd] = sum_{e in row a} dGe[rev e, c, kd]   (per-edge scratch (E, 9, Kd) -> planes (9, N, Kd))
template <typename T>
__global__ void gather_rev_k(const T* __restrict__ src, const int32_t* __restrict__ row_ptr,
                             const int32_t* __restrict__ rev, int Kd, int64_t N, T* __restrict__ dst, int64_t total) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = q / (N * Kd);
    const int64_t r = q - c * N * Kd;
    const int64_t a = r / Kd;
    const int kd = (int)(r - a * Kd);
    T s = 0;
    for (int e = row_ptr[a]; e < row_ptr[a + 1]; e++) s += src[((int64_t)rev[e] * 9 + c) * Kd + kd];
    dst[q] = s;
  }
}

// ------------------------------------------------------------------------------------------ launchers
inline int elem_grid(int64_t n, int threads) { return grid_for(ceil_div<int64_t>(n, threads), 16); }

template <typename T>
int edge_vec(const void* pos, const int32_t* ei, const int32_t* ej, const void* shift, void* vec, int64_t E,
             void* stream) {
  if (E == 0) return FACEK_OK;
  edge_vec_k<T><<<elem_grid(E, 256), 256, 0, as_stream(stream)>>>((const T*)pos, ei, ej, (const T*)shift, (T*)vec, E);
  return launch_status("facek_edge_vec");
}
template <typename T>
int edge_vec_bwd(const void* dvec, const int32_t* row_ptr, const int32_t* rev, int64_t N, void* dpos, void* stream) {
  if (N == 0) return FACEK_OK;
  edge_vec_bwd_k<T><<<elem_grid(N, 128), 128, 0, as_stream(stream)>>>((const T*)dvec, row_ptr, rev, N, (T*)dpos);
  return launch_status("facek_edge_vec_bwd");
}
template <typename T>
int edge_sym(const void* vec, void* Y, int64_t E, void* stream) {
  if (E == 0) return FACEK_OK;
  if (std::is_same<T, float>::value && (reinterpret_cast<uintptr_t>(Y) & 15) == 0) {
    const int64_t total = E * 5;                        // NX = 20 floats = five 16-byte pieces per edge
    edge_sym5_k<<<elem_grid(total, 256), 256, 0, as_stream(stream)>>>((const float*)vec, (float4*)Y, total);
    return launch_status("facek_edge_sym");
  }
  edge_sym_k<T><<<elem_grid(E, 256), 256, 0, as_stream(stream)>>>((const T*)vec, (T*)Y, E);
  return launch_status("facek_edge_sym");
}
template <typename T>
int edge_sym_bwd(const void* vec, const void* dY, void* dvec, int acc, int64_t E, void* stream) {
  if (E == 0) return FACEK_OK;
  edge_sym_bwd_k<T><<<elem_grid(E, 256), 256, 0, as_stream(stream)>>>((const T*)vec, (const T*)dY, (T*)dvec, acc, E);
  return launch_status("facek_edge_sym_bwd");
}

template <typename T, int NBMAX, int HMAX, int BMAX>
int radial_launch(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
                  int nb, int H, int B, const void* w1, const void* b1, const void* pair, const void* w2,
                  const void* b2, const void* w3, const void* b3, void* phi, void* dphidr, int64_t E, void* stream) {
  const size_t smem = sizeof(T) * ((size_t)H * nb + 2 * H + (size_t)n_el * n_el * H + (size_t)H * H + (size_t)B * H + B);
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_radial_fwd: weights (%zu B) exceed shared memory", smem);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(radial_mlp_k<T, NBMAX, HMAX, BMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  radial_mlp_k<T, NBMAX, HMAX, BMAX><<<grid_for(ceil_div<int64_t>(E, 128), 4), 128, smem, as_stream(stream)>>>(
      (const T*)vec, ei, ej, zidx, n_el, (T)rc, nb, H, B, (const T*)w1, (const T*)b1, (const T*)pair, (const T*)w2,
      (const T*)b2, (const T*)w3, (const T*)b3, (T*)phi, (T*)dphidr, E);
  return launch_status("facek_radial_fwd");
}

template <typename T, int NBMAX>
int radial_wide_launch(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el,
                       double rc, int nb, int H, int B, const void* w1, const void* b1, const void* pair,
                       const void* w2, const void* b2, const void* w3, const void* b3, void* phi, void* dphidr,
                       int64_t E, void* stream) {
  const size_t smem = sizeof(T) * ((size_t)H * nb + 2 * H + (size_t)n_el * n_el * H + (size_t)H * H);
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_radial_fwd: weights (%zu B) exceed shared memory", smem);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(radial_wide_k<T, NBMAX, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  radial_wide_k<T, NBMAX, 64><<<grid_for(ceil_div<int64_t>(E, 128), 4), 128, smem, as_stream(stream)>>>(
      (const T*)vec, ei, ej, zidx, n_el, (T)rc, nb, H, B, (const T*)w1, (const T*)b1, (const T*)pair, (const T*)w2,
      (const T*)b2, (const T*)w3, (const T*)b3, (T*)phi, (T*)dphidr, E);
  return launch_status("facek_radial_fwd");
}

template <typename T>
int radial_simt(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
                int nb, int H, int B, const void* w1, const void* b1, const void* pair, const void* w2, const void* b2,
                const void* w3, const void* b3, void* phi, void* dphidr, int64_t E, void* stream) {
  if (E == 0) return FACEK_OK;
  FACEK_CHECK_ARG(H <= 64 && nb <= 16, "facek_radial_fwd: H=%d nb=%d exceed 64/16", H, nb);
  if (B > 32) {
    if (nb <= 8)
      return radial_wide_launch<T, 8>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                                      dphidr, E, stream);
    return radial_wide_launch<T, 16>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                                     dphidr, E, stream);
  }
  if (nb <= 8 && B <= 16)
    return radial_launch<T, 8, 64, 16>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                                       dphidr, E, stream);
  if (B <= 16)
    return radial_launch<T, 16, 64, 16>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                                        dphidr, E, stream);
  return radial_launch<T, 16, 64, 32>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                                      dphidr, E, stream);
}

// fp32 with the flagship shapes runs on the tensor cores (radial_tc.cu); fp64 and other shapes on the CUDA cores
template <typename T>
int radial_fwd(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
               int nb, int H, int B, const void* w1, const void* b1, const void* pair, const void* w2, const void* b2,
               const void* w3, const void* b3, void* phi, void* dphidr, int64_t E, void* stream) {
  if (std::is_same<T, float>::value && radial_tc_supported(n_el, nb, H, B))
    return radial_tc_fwd(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi, dphidr, E, stream);
  return radial_simt<T>(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi, dphidr, E, stream);
}

template <typename T>
int radial_spline(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
                  int G, double dr, int B, const void* Tab, const void* dTab, void* phi, void* dphidr, int64_t E,
                  void* stream) {
  if (E == 0) return FACEK_OK;
  const uintptr_t al = reinterpret_cast<uintptr_t>(Tab) | reinterpret_cast<uintptr_t>(dTab) |
                       reinterpret_cast<uintptr_t>(phi) | reinterpret_cast<uintptr_t>(dphidr);
  if (std::is_same<T, float>::value && B % 4 == 0 && (al & 15) == 0) {
    const int64_t EB4 = E * (B / 4);
    radial_spline4_k<<<elem_grid(EB4, 256), 256, 0, as_stream(stream)>>>(
        (const float*)vec, ei, ej, zidx, n_el, (float)rc, G, (float)dr, B / 4, (const float4*)Tab,
        (const float4*)dTab, (float4*)phi, (float4*)dphidr, EB4);
    return launch_status("facek_radial_spline_fwd");
  }
  radial_spline_k<T, 32><<<elem_grid(E, 256), 256, 0, as_stream(stream)>>>(
      (const T*)vec, ei, ej, zidx, n_el, (T)rc, G, (T)dr, B, (const T*)Tab, (const T*)dTab, (T*)phi, (T*)dphidr, E);
  return launch_status("facek_radial_spline_fwd");
}

template <typename T>
int radial_bwd(const void* vec, const void* dphi, const void* dphidr, int B, void* dvec, int acc, int64_t E,
               void* stream) {
  if (E == 0) return FACEK_OK;
  const int B4 = B / 4;
  const uintptr_t al = reinterpret_cast<uintptr_t>(dphi) | reinterpret_cast<uintptr_t>(dphidr);
  if (std::is_same<T, float>::value && B % 4 == 0 && B4 <= 32 && (B4 & (B4 - 1)) == 0 && (al & 15) == 0) {
    const int64_t total = E * B4;
    radial_bwd4_k<<<elem_grid(total, 256), 256, 0, as_stream(stream)>>>(
        (const float*)vec, (const float4*)dphi, (const float4*)dphidr, B4, (float*)dvec, acc, total);
    return launch_status("facek_radial_bwd");
  }
  radial_bwd_k<T><<<elem_grid(E, 256), 256, 0, as_stream(stream)>>>((const T*)vec, (const T*)dphi,
                                                                     (const T*)dphidr, B, (T*)dvec, acc, E);
  return launch_status("facek_radial_bwd");
}

template <typename T>
int msg_fwd(const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ, const void* TI, int nc, int K,
            void* msg, int64_t N, int64_t E, void* stream) {
  if (E == 0) return FACEK_OK;
  const uintptr_t al = reinterpret_cast<uintptr_t>(TJ) | reinterpret_cast<uintptr_t>(TI) | reinterpret_cast<uintptr_t>(msg);
  if (std::is_same<T, float>::value && K == 32 && nc <= 10 && (al & 15) == 0) {
    edge_msg32_k<<<elem_grid(E * 8, 256), 256, 0, as_stream(stream)>>>((const float*)Y, ei, ej, (const float4*)TJ,
                                                                        (const float4*)TI, nc, N, (float4*)msg, E);
    return launch_status("facek_edge_msg_fwd");
  }
  const int64_t EK = E * K;
  edge_msg_k<T><<<elem_grid(EK, 256), 256, 0, as_stream(stream)>>>((const T*)Y, ei, ej, (const T*)TJ, (const T*)TI,
                                                                    nc, K, N, (T*)msg, EK);
  return launch_status("facek_edge_msg_fwd");
}

template <typename T>
int msg_bwd(const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ, const void* TI, const void* dmsg,
            const int32_t* row_ptr, const int32_t* rev, int nc, int K, void* dY, int acc, void* dTJ, void* dTI,
            int64_t N, int64_t E, void* stream) {
  if (E > 0 && dY) {
    edge_msg_bwd_dy_k<T><<<grid_for(ceil_div<int64_t>(E, 8), 16), 256, 0, as_stream(stream)>>>(
        ei, ej, (const T*)TJ, (const T*)TI, (const T*)dmsg, nc, K, N, (T*)dY, acc, E);
    int st = launch_status("facek_edge_msg_bwd(dY)");
    if (st) return st;
  }
  if (N > 0) {
    const int64_t NK = N * K;
    FACEK_CHECK_ARG(E == 0 || (reinterpret_cast<uintptr_t>(Y) & 15) == 0,
                    "facek_edge_msg_bwd: Y must be 16-byte aligned (rows are read as 16-byte vectors)");
    edge_msg_bwd_tables_k<T><<<elem_grid(NK, 128), 128, 0, as_stream(stream)>>>((const T*)Y, (const T*)dmsg, row_ptr,
                                                                                 rev, nc, K, (T*)dTJ, (T*)dTI, NK);
    return launch_status("facek_edge_msg_bwd(tables)");
  }
  return FACEK_OK;
}

template <typename T, int BQ>
void launch_transport_fwd(const void* phi, const void* vec, const int32_t* ej, const void* Gt, const int32_t* row_ptr,
                          void* DT, int64_t N, int B, int Kd, int cps, void* stream) {
  const int threads = ceil_div((B / BQ) * Kd, 32) * 32;
  const size_t smem = sizeof(T) * TR_TILE * ((size_t)B + (size_t)Kd * 18);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(transport_fwd_k<T, BQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  transport_fwd_k<T, BQ><<<grid_for(N, cps), threads, smem, as_stream(stream)>>>(
      (const T*)phi, (const T*)vec, ej, (const T*)Gt, row_ptr, (T*)DT, N, B, Kd);
}

template <typename T>
int transport_fwd(const void* phi, const void* vec, const int32_t* ej, const void* Gt, const int32_t* row_ptr,
                  void* DT, int64_t N, int B, int Kd, void* stream) {
  if (N == 0) return FACEK_OK;
  FACEK_CHECK_ARG(B % 2 == 0, "facek_transport_fwd: B=%d is odd", B);
  // Two b's per thread (72 registers, seven 128-thread CTAs per SM) measured 5.7% faster than four (124 registers,
  // eight 64-thread CTAs) at the alloys' shape B = Kd = 16; four b's remain for shapes with more than 256 threads.
  if ((B / 2) * Kd <= 256) {
    launch_transport_fwd<T, 2>(phi, vec, ej, Gt, row_ptr, DT, N, B, Kd, 6, stream);
  } else {
    FACEK_CHECK_ARG(B % 4 == 0 && (B / 4) * Kd <= 256, "facek_transport_fwd: B=%d, Kd=%d unsupported", B, Kd);
    launch_transport_fwd<T, 4>(phi, vec, ej, Gt, row_ptr, DT, N, B, Kd, 8, stream);
  }
  return launch_status("facek_transport_fwd");
}

template <typename T>
int transport_bwd(const void* phi, const void* vec, const int32_t* ej, const void* Gt, const void* dT1,
                  const void* dT2, const int32_t* row_ptr, const int32_t* rev, void* dphi, void* dvec, int acc,
                  void* dGe, void* dGt, int64_t N, int64_t E, int B, int Kd, void* stream) {
  if (N == 0) return FACEK_OK;
  int KQ = 1;
  while (KQ * 2 < Kd) KQ <<= 1;                   // two kd channels per thread
  FACEK_CHECK_ARG(KQ <= 32, "facek_transport_bwd: Kd=%d too large", Kd);
  const size_t smem = 2 * sizeof(T) * 18 * (size_t)B * Kd;
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_transport_bwd: gradient tiles %zu B exceed shared memory",
                  smem);
  const int threads = KQ * 32 <= 256 ? KQ * 32 : 256;   // 32 edge slots per pass
  if (E > 0) {
    if (std::is_same<T, float>::value && B == 16 && Kd % 8 == 0 && 18 * 16 * Kd * 4 <= 48 * 1024) {
      // flagship shape: lane-per-edge kernel over the row's gradient rows in shared memory
      const size_t smem1 = sizeof(float) * 18 * 16 * (size_t)Kd;
      transport_bwd_lane_k<16><<<grid_for(N, 4), 96, smem1, as_stream(stream)>>>(
          (const float*)phi, (const float*)vec, ej, (const float*)Gt, (const float*)dT1, (const float*)dT2, row_ptr,
          (float*)dphi, (float*)dvec, acc, (float*)dGe, N, Kd);
    } else if (B <= 16) {
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(transport_bwd_k<T, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      transport_bwd_k<T, 16><<<grid_for(N, 2), threads, smem, as_stream(stream)>>>(
          (const T*)phi, (const T*)vec, ej, (const T*)Gt, (const T*)dT1, (const T*)dT2, row_ptr, (T*)dphi, (T*)dvec,
          acc, (T*)dGe, N, B, Kd, KQ);
    } else {
      FACEK_CHECK_ARG(B <= 32, "facek_transport_bwd: B=%d > 32", B);
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(transport_bwd_k<T, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      transport_bwd_k<T, 32><<<grid_for(N, 2), threads, smem, as_stream(stream)>>>(
          (const T*)phi, (const T*)vec, ej, (const T*)Gt, (const T*)dT1, (const T*)dT2, row_ptr, (T*)dphi, (T*)dvec,
          acc, (T*)dGe, N, B, Kd, KQ);
    }
    int st = launch_status("facek_transport_bwd");
    if (st) return st;
  }
  const int64_t total = 9 * N * Kd;
  gather_rev_k<T><<<elem_grid(total, 256), 256, 0, as_stream(stream)>>>((const T*)dGe, row_ptr, rev, Kd, N, (T*)dGt,
                                                                        total);
  return launch_status("facek_transport_bwd(gather)");
}

}  // namespace

// message part of dY only, accumulated into dY (used after a density adjoint that wrote dY)
int edge_msg_dy(int dtype, const int32_t* ei, const int32_t* ej, const void* TJ, const void* TI, const void* dmsg,
                int nc, int K, int64_t N, int64_t E, void* dY, void* stream) {
  if (E == 0) return FACEK_OK;
  if (dtype == FACEK_F32)
    edge_msg_bwd_dy_k<float><<<grid_for(ceil_div<int64_t>(E, 8), 16), 256, 0, as_stream(stream)>>>(
        ei, ej, (const float*)TJ, (const float*)TI, (const float*)dmsg, nc, K, N, (float*)dY, 1, E);
  else
    edge_msg_bwd_dy_k<double><<<grid_for(ceil_div<int64_t>(E, 8), 16), 256, 0, as_stream(stream)>>>(
        ei, ej, (const double*)TJ, (const double*)TI, (const double*)dmsg, nc, K, N, (double*)dY, 1, E);
  return launch_status("facek_density_msg_xm_bwd(message dY)");
}

}  // namespace facek

using namespace facek;

extern "C" int facek_edge_vec(int dtype, const void* pos, const int32_t* ei, const int32_t* ej, const void* shift,
                              void* vec, int64_t E, void* stream) {
  FACEK_CHECK_ARG(E >= 0 && (E == 0 || (pos && ei && ej && shift && vec)), "facek_edge_vec: bad arguments");
  return FACEK_DISPATCH(dtype, edge_vec, pos, ei, ej, shift, vec, E, stream);
}
extern "C" int facek_edge_vec_bwd(int dtype, const void* dvec, const int32_t* row_ptr, const int32_t* rev, int64_t N,
                                  void* dpos, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && (N == 0 || (dvec && row_ptr && rev && dpos)), "facek_edge_vec_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, edge_vec_bwd, dvec, row_ptr, rev, N, dpos, stream);
}
extern "C" int facek_edge_sym(int dtype, const void* vec, void* Y, int64_t E, void* stream) {
  FACEK_CHECK_ARG(E >= 0 && (E == 0 || (vec && Y)), "facek_edge_sym: bad arguments");
  return FACEK_DISPATCH(dtype, edge_sym, vec, Y, E, stream);
}
extern "C" int facek_edge_sym_bwd(int dtype, const void* vec, const void* dY, void* dvec, int32_t accumulate, int64_t E,
                                  void* stream) {
  FACEK_CHECK_ARG(E >= 0 && (E == 0 || (vec && dY && dvec)), "facek_edge_sym_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, edge_sym_bwd, vec, dY, dvec, accumulate, E, stream);
}
extern "C" int facek_radial_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx,
                                int32_t n_el, double rc, int32_t nb, int32_t H, int32_t B, const void* w1,
                                const void* b1, const void* pair, const void* w2, const void* b2, const void* w3,
                                const void* b3, void* phi, void* dphidr, int64_t E, void* stream) {
  FACEK_CHECK_ARG(E >= 0 && n_el > 0 && rc > 0 && nb > 0 && H > 0 && B > 0, "facek_radial_fwd: bad sizes");
  FACEK_CHECK_ARG(E == 0 || (vec && ei && ej && zidx && w1 && b1 && pair && w2 && b2 && w3 && b3 && phi && dphidr),
                  "facek_radial_fwd: null tensor");
  return FACEK_DISPATCH(dtype, radial_fwd, vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                        dphidr, E, stream);
}
extern "C" int facek_radial_simt_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej,
                                     const int32_t* zidx, int32_t n_el, double rc, int32_t nb, int32_t H, int32_t B,
                                     const void* w1, const void* b1, const void* pair, const void* w2, const void* b2,
                                     const void* w3, const void* b3, void* phi, void* dphidr, int64_t E,
                                     void* stream) {
  FACEK_CHECK_ARG(E >= 0 && n_el > 0 && rc > 0 && nb > 0 && H > 0 && B > 0, "facek_radial_simt_fwd: bad sizes");
  FACEK_CHECK_ARG(E == 0 || (vec && ei && ej && zidx && w1 && b1 && pair && w2 && b2 && w3 && b3 && phi && dphidr),
                  "facek_radial_simt_fwd: null tensor");
  return FACEK_DISPATCH(dtype, radial_simt, vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi,
                        dphidr, E, stream);
}
extern "C" int facek_radial_spline_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej,
                                       const int32_t* zidx, int32_t n_el, double rc, int32_t G, double dr, int32_t B,
                                       const void* T, const void* dT, void* phi, void* dphidr, int64_t E,
                                       void* stream) {
  FACEK_CHECK_ARG(E >= 0 && n_el > 0 && G >= 2 && dr > 0 && B > 0, "facek_radial_spline_fwd: bad sizes");
  FACEK_CHECK_ARG(E == 0 || (vec && ei && ej && zidx && T && dT && phi && dphidr), "facek_radial_spline_fwd: null");
  return FACEK_DISPATCH(dtype, radial_spline, vec, ei, ej, zidx, n_el, rc, G, dr, B, T, dT, phi, dphidr, E, stream);
}
extern "C" int facek_radial_bwd(int dtype, const void* vec, const void* dphi, const void* dphidr, int32_t B, void* dvec,
                                int32_t accumulate, int64_t E, void* stream) {
  FACEK_CHECK_ARG(E >= 0 && B > 0 && (E == 0 || (vec && dphi && dphidr && dvec)), "facek_radial_bwd: bad arguments");
  return FACEK_DISPATCH(dtype, radial_bwd, vec, dphi, dphidr, B, dvec, accumulate, E, stream);
}
extern "C" int facek_edge_msg_fwd(int dtype, const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ,
                                  const void* TI, int32_t nc, int32_t K, void* msg, int64_t N, int64_t E,
                                  void* stream) {
  FACEK_CHECK_ARG(E >= 0 && N >= 0 && nc >= 1 && nc <= 10 && K > 0, "facek_edge_msg_fwd: bad sizes nc=%d K=%d", nc,
                  K);
  FACEK_CHECK_ARG(E == 0 || (Y && ei && ej && TJ && msg), "facek_edge_msg_fwd: null tensor");
  return FACEK_DISPATCH(dtype, msg_fwd, Y, ei, ej, TJ, TI, nc, K, msg, N, E, stream);
}
extern "C" int facek_edge_msg_bwd(int dtype, const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ,
                                  const void* TI, const void* dmsg, const int32_t* row_ptr, const int32_t* rev,
                                  int32_t nc, int32_t K, void* dY, int32_t accumulate, void* dTJ, void* dTI, int64_t N,
                                  int64_t E, void* stream) {
  FACEK_CHECK_ARG(E >= 0 && N >= 0 && nc >= 1 && nc <= 10 && K > 0, "facek_edge_msg_bwd: bad sizes");
  FACEK_CHECK_ARG(row_ptr && rev && dTJ && (E == 0 || (Y && ei && ej && TJ && dmsg)), "facek_edge_msg_bwd: null");
  return FACEK_DISPATCH(dtype, msg_bwd, Y, ei, ej, TJ, TI, dmsg, row_ptr, rev, nc, K, dY, accumulate, dTJ, dTI, N, E,
                        stream);
}
extern "C" int facek_transport_fwd(int dtype, const void* phi, const void* vec, const int32_t* ej, const void* Gt,
                                   const int32_t* row_ptr, void* DT, int64_t N, int32_t B, int32_t Kd, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B > 0 && B % 4 == 0 && Kd > 0, "facek_transport_fwd: need B %% 4 == 0 (B=%d)", B);
  FACEK_CHECK_ARG(N == 0 || (phi && vec && ej && Gt && row_ptr && DT), "facek_transport_fwd: null tensor");
  return FACEK_DISPATCH(dtype, transport_fwd, phi, vec, ej, Gt, row_ptr, DT, N, B, Kd, stream);
}
extern "C" int facek_transport_bwd(int dtype, const void* phi, const void* vec, const int32_t* ej, const void* Gt,
                                   const void* dT1, const void* dT2, const int32_t* row_ptr, const int32_t* rev,
                                   void* dphi, void* dvec, int32_t accumulate, void* dGt_edge, void* dGt, int64_t N,
                                   int64_t E, int32_t B, int32_t Kd, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && E >= 0 && B > 0 && Kd > 0, "facek_transport_bwd: bad sizes");
  FACEK_CHECK_ARG(row_ptr && rev && dGt && (E == 0 || (phi && vec && ej && Gt && dT1 && dT2 && dphi && dvec &&
                                                       dGt_edge)),
                  "facek_transport_bwd: null tensor");
  return FACEK_DISPATCH(dtype, transport_bwd, phi, vec, ej, Gt, dT1, dT2, row_ptr, rev, dphi, dvec, accumulate,
                        dGt_edge, dGt, N, E, B, Kd, stream);
}
