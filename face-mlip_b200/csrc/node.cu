// Node invariant algebra: the 8 polynomial invariant families (3-, 4-, 5-body) and the gated equivariant
// products of face-mlip's MomentBlock (face/model.py:252-264 invariants, :288-296 V/Mf products), forward and
// hand-derived first-order backward.  One thread per (atom, channel); every tensor is read through a
// (row, channel, component) stride triple so the same code serves the reference's (N,C,k) tensors
// (face/node_kernel.py:164-209) and the engine's (N,k,3C) projection output without any transpose copy.
//
// HBM-bound: per (atom,channel) the forward reads 47 values and writes 20, the backward reads 67 and writes 47.
#include "common.cuh"

namespace facek {
namespace {

// symmetric-storage index of a full rank-2 / rank-3 Cartesian index (face/cartesian.py:11-17 order)
__host__ __device__ constexpr int sym2(int a, int b) { return a == b ? a : 2 + a + b; }
__host__ __device__ constexpr int sym3(int a, int b, int c) {
  // sort (a,b,c) ascending
  int x = a < b ? a : b, y = a < b ? b : a;
  int z = c;
  if (z < x) { int t = x; x = z; z = y; y = t; }
  else if (z < y) { int t = y; y = z; z = t; }
  const int code = x * 9 + y * 3 + z;
  switch (code) {
    case 0: return 0;            // 000
    case 13: return 1;           // 111
    case 26: return 2;           // 222
    case 1: return 3;            // 001
    case 2: return 4;            // 002
    case 4: return 5;            // 011
    case 14: return 6;           // 112
    case 8: return 7;            // 022
    case 17: return 8;           // 122
    default: return 9;           // 012
  }
}

template <typename T>
struct Acc {                 // element (n, c, k) = p[n*sN + c*sC + k*sK]
  const T* p;
  int64_t sN;
  int64_t sC;
  int64_t sK;
  __device__ T operator()(int64_t n, int c, int k) const { return p[n * sN + (int64_t)c * sC + (int64_t)k * sK]; }
};
template <typename T>
struct Out {
  T* p;
  int64_t sN;
  int64_t sC;
  int64_t sK;
  __device__ void set(int64_t n, int c, int k, T v) const { p[n * sN + (int64_t)c * sC + (int64_t)k * sK] = v; }
};

template <typename T>
struct NodeIO {
  Acc<T> P1, Q1, S1, P2, Q2, S2, P3, Q3;
};

template <typename T>
struct Vals {
  T p1[3], q1[3], s1[3], p2[9], q2[9], s2[9], p3[27], q3[27];
};

template <typename T>
__device__ __forceinline__ void load_vals(const NodeIO<T>& io, int64_t n, int c, Vals<T>& v) {
#pragma unroll
  for (int a = 0; a < 3; a++) {
    v.p1[a] = io.P1(n, c, a);
    v.q1[a] = io.Q1(n, c, a);
    v.s1[a] = io.S1(n, c, a);
  }
  T t2p[6], t2q[6], t2s[6], t3p[10], t3q[10];
#pragma unroll
  for (int s = 0; s < 6; s++) {
    t2p[s] = io.P2(n, c, s);
    t2q[s] = io.Q2(n, c, s);
    t2s[s] = io.S2(n, c, s);
  }
#pragma unroll
  for (int s = 0; s < 10; s++) {
    t3p[s] = io.P3(n, c, s);
    t3q[s] = io.Q3(n, c, s);
  }
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++) {
      v.p2[a * 3 + b] = t2p[sym2(a, b)];
      v.q2[a * 3 + b] = t2q[sym2(a, b)];
      v.s2[a * 3 + b] = t2s[sym2(a, b)];
#pragma unroll
      for (int d = 0; d < 3; d++) {
        v.p3[a * 9 + b * 3 + d] = t3p[sym3(a, b, d)];
        v.q3[a * 9 + b * 3 + d] = t3q[sym3(a, b, d)];
      }
    }
}

// contractions shared by forward and backward
template <typename T>
struct Mid {
  T q2s1[3];   // Q2_ab S1_b
  T p3q2[3];   // P3_abd Q2_bd
  T p2q1[3];   // P2_ab Q1_b
  T pq2[9];    // P2_ab Q2_bd   -> [a][d]
  T p3s1[9];   // P3_adb S1_b   -> [a][d]
  T x33[9];    // P3_abd Q3_abe -> [d][e]
};

template <typename T>
__device__ __forceinline__ void mid(const Vals<T>& v, Mid<T>& m) {
#pragma unroll
  for (int a = 0; a < 3; a++) {
    T x = 0, y = 0, z = 0;
#pragma unroll
    for (int b = 0; b < 3; b++) {
      x += v.q2[a * 3 + b] * v.s1[b];
      z += v.p2[a * 3 + b] * v.q1[b];
#pragma unroll
      for (int d = 0; d < 3; d++) y += v.p3[a * 9 + b * 3 + d] * v.q2[b * 3 + d];
    }
    m.q2s1[a] = x;
    m.p3q2[a] = y;
    m.p2q1[a] = z;
  }
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int d = 0; d < 3; d++) {
      T x = 0, y = 0, w = 0;
#pragma unroll
      for (int b = 0; b < 3; b++) {
        x += v.p2[a * 3 + b] * v.q2[b * 3 + d];
        y += v.p3[a * 9 + d * 3 + b] * v.s1[b];
#pragma unroll
        for (int e = 0; e < 3; e++) w += v.p3[e * 9 + b * 3 + a] * v.q3[e * 9 + b * 3 + d];
      }
      m.pq2[a * 3 + d] = x;
      m.p3s1[a * 3 + d] = y;
      m.x33[a * 3 + d] = w;
    }
}

template <typename T>
__device__ __forceinline__ void invariants(const Vals<T>& v, const Mid<T>& m, T inv[8]) {
  T i1 = 0, i2 = 0, i3 = 0, i4 = 0, i5 = 0, i6 = 0, i7 = 0, i8 = 0;
#pragma unroll
  for (int a = 0; a < 3; a++) {
    i1 += v.p1[a] * v.q1[a];
    i4 += v.p1[a] * m.q2s1[a];
    i6 += m.p3q2[a] * v.s1[a];
  }
#pragma unroll
  for (int k = 0; k < 9; k++) i2 += v.p2[k] * v.q2[k];
#pragma unroll
  for (int k = 0; k < 27; k++) i3 += v.p3[k] * v.q3[k];
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int d = 0; d < 3; d++) {
      i5 += m.pq2[a * 3 + d] * v.s2[d * 3 + a];
      i7 += m.x33[a * 3 + d] * v.s2[a * 3 + d];
    }
#pragma unroll
  for (int a = 0; a < 3; a++) {
    T t = 0;
#pragma unroll
    for (int b = 0; b < 3; b++) {
      T u = 0;
#pragma unroll
      for (int d = 0; d < 3; d++) u += v.p3[a * 9 + b * 3 + d] * v.q1[d];
      t += u * v.s1[b];
    }
    i8 += t * v.q1[a];
  }
  inv[0] = i1; inv[1] = i2; inv[2] = i3; inv[3] = i4; inv[4] = i5; inv[5] = i6; inv[6] = i7; inv[7] = i8;
}

// gradients w.r.t. the FULL tensors; folded to symmetric storage by the caller
template <typename T>
struct Grads {
  T p1[3], q1[3], s1[3], p2[9], q2[9], s2[9], p3[27], q3[27];
  T da[4], db[4];
};

template <typename T>
__device__ __forceinline__ void backward(const Vals<T>& v, const Mid<T>& m, const T g[8], const T gv[3],
                                         const T gm[9], const T av[4], const T bv[4], bool eq, Grads<T>& d) {
#pragma unroll
  for (int a = 0; a < 3; a++) {
    d.p1[a] = g[0] * v.q1[a] + g[3] * m.q2s1[a];
    d.q1[a] = g[0] * v.p1[a];
    d.s1[a] = g[5] * m.p3q2[a];
  }
#pragma unroll
  for (int k = 0; k < 9; k++) {
    d.p2[k] = g[1] * v.q2[k];
    d.q2[k] = g[1] * v.p2[k];
  }
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++) d.s2[a * 3 + b] = g[4] * m.pq2[b * 3 + a] + g[6] * m.x33[a * 3 + b];
#pragma unroll
  for (int k = 0; k < 27; k++) {
    d.p3[k] = g[2] * v.q3[k];
    d.q3[k] = g[2] * v.p3[k];
  }
  // i4 = P1_a Q2_ab S1_b
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++) {
      d.q2[a * 3 + b] += g[3] * v.p1[a] * v.s1[b];
      d.s1[b] += g[3] * v.p1[a] * v.q2[a * 3 + b];
    }
  // i5 = P2_ab Q2_bd S2_da
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++) {
      T x = 0, y = 0;
#pragma unroll
      for (int e = 0; e < 3; e++) {
        x += v.q2[b * 3 + e] * v.s2[e * 3 + a];     // d i5 / d P2_ab
        y += v.s2[b * 3 + e] * v.p2[e * 3 + a];     // d i5 / d Q2_ab = S2_be P2_ea
      }
      d.p2[a * 3 + b] += g[4] * x;
      d.q2[a * 3 + b] += g[4] * y;
    }
  // i6 = P3_abd Q2_bd S1_a ; i7 = P3_abd Q3_abe S2_de ; i8 = P3_abd Q1_d S1_b Q1_a
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++)
#pragma unroll
      for (int e = 0; e < 3; e++) {
        const int k = a * 9 + b * 3 + e;
        T s2q3 = 0, p3s2 = 0;
#pragma unroll
        for (int f = 0; f < 3; f++) {
          s2q3 += v.q3[a * 9 + b * 3 + f] * v.s2[e * 3 + f];
          p3s2 += v.p3[a * 9 + b * 3 + f] * v.s2[f * 3 + e];
        }
        const T pv = v.p3[k];
        d.p3[k] += g[5] * v.q2[b * 3 + e] * v.s1[a] + g[6] * s2q3 + g[7] * v.q1[a] * v.s1[b] * v.q1[e];
        d.q3[k] += g[6] * p3s2;
        d.q2[b * 3 + e] += g[5] * pv * v.s1[a];
        d.q1[e] += g[7] * pv * v.s1[b] * v.q1[a];
        d.q1[a] += g[7] * pv * v.s1[b] * v.q1[e];
        d.s1[b] += g[7] * pv * v.q1[a] * v.q1[e];
      }
#pragma unroll
  for (int k = 0; k < 4; k++) { d.da[k] = 0; d.db[k] = 0; }
  if (!eq) return;
  // V_a = a0 P1_a + a1 Q2_ab S1_b + a2 P3_abd Q2_bd + a3 P2_ab Q1_b
#pragma unroll
  for (int a = 0; a < 3; a++) {
    d.p1[a] += av[0] * gv[a];
    d.da[0] += gv[a] * v.p1[a];
    d.da[1] += gv[a] * m.q2s1[a];
    d.da[2] += gv[a] * m.p3q2[a];
    d.da[3] += gv[a] * m.p2q1[a];
#pragma unroll
    for (int b = 0; b < 3; b++) {
      d.q2[a * 3 + b] += av[1] * gv[a] * v.s1[b];
      d.s1[b] += av[1] * gv[a] * v.q2[a * 3 + b];
      d.p2[a * 3 + b] += av[3] * gv[a] * v.q1[b];
      d.q1[b] += av[3] * gv[a] * v.p2[a * 3 + b];
#pragma unroll
      for (int e = 0; e < 3; e++) {
        d.p3[a * 9 + b * 3 + e] += av[2] * gv[a] * v.q2[b * 3 + e];
        d.q2[b * 3 + e] += av[2] * gv[a] * v.p3[a * 9 + b * 3 + e];
      }
    }
  }
  // Mf_ad = b0 P2_ad + b1 P1_a Q1_d + b2 P2_ab Q2_bd + b3 P3_adb S1_b
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int e = 0; e < 3; e++) {
      const T gg = gm[a * 3 + e];
      d.p2[a * 3 + e] += bv[0] * gg;
      d.p1[a] += bv[1] * gg * v.q1[e];
      d.q1[e] += bv[1] * gg * v.p1[a];
      d.db[0] += gg * v.p2[a * 3 + e];
      d.db[1] += gg * v.p1[a] * v.q1[e];
      d.db[2] += gg * m.pq2[a * 3 + e];
      d.db[3] += gg * m.p3s1[a * 3 + e];
#pragma unroll
      for (int b = 0; b < 3; b++) {
        d.p2[a * 3 + b] += bv[2] * gg * v.q2[b * 3 + e];
        d.q2[b * 3 + e] += bv[2] * gg * v.p2[a * 3 + b];
        d.p3[a * 9 + e * 3 + b] += bv[3] * gg * v.s1[b];
        d.s1[b] += bv[3] * gg * v.p3[a * 9 + e * 3 + b];
      }
    }
}

template <typename T>
__device__ __forceinline__ void fold2(const T full[9], T sym[6]) {
#pragma unroll
  for (int s = 0; s < 6; s++) sym[s] = 0;
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++) sym[sym2(a, b)] += full[a * 3 + b];
}
template <typename T>
__device__ __forceinline__ void fold3(const T full[27], T sym[10]) {
#pragma unroll
  for (int s = 0; s < 10; s++) sym[s] = 0;
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int b = 0; b < 3; b++)
#pragma unroll
      for (int e = 0; e < 3; e++) sym[sym3(a, b, e)] += full[a * 9 + b * 3 + e];
}

template <typename T>
__device__ __forceinline__ void products(const Vals<T>& v, const Mid<T>& m, const T av[4], const T bv[4], T V[3],
                                         T Mf[9]) {
#pragma unroll
  for (int a = 0; a < 3; a++) V[a] = av[0] * v.p1[a] + av[1] * m.q2s1[a] + av[2] * m.p3q2[a] + av[3] * m.p2q1[a];
#pragma unroll
  for (int a = 0; a < 3; a++)
#pragma unroll
    for (int e = 0; e < 3; e++)
      Mf[a * 3 + e] = bv[0] * v.p2[a * 3 + e] + bv[1] * v.p1[a] * v.q1[e] + bv[2] * m.pq2[a * 3 + e] +
                      bv[3] * m.p3s1[a * 3 + e];
}

// ------------------------------------------------------------------------------------------- kernels
// path weights a, b are (4, C) row-major (the parameters vpath/mpath, face/model.py:155-156)
template <typename T>
__global__ void __launch_bounds__(128) node_ref_fwd_k(NodeIO<T> io, const T* __restrict__ av, const T* __restrict__ bv,
                                                      T* __restrict__ inv, T* __restrict__ V, T* __restrict__ Mf,
                                                      int64_t NC, int C, int eq) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= NC) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  Vals<T> v;
  load_vals(io, n, c, v);
  Mid<T> m;
  mid(v, m);
  T iv[8];
  invariants(v, m, iv);
#pragma unroll
  for (int f = 0; f < 8; f++) inv[t * 8 + f] = iv[f];
  if (eq) {
    T a4[4], b4[4], Vv[3], M9[9];
#pragma unroll
    for (int k = 0; k < 4; k++) { a4[k] = av[k * C + c]; b4[k] = bv[k * C + c]; }
    products(v, m, a4, b4, Vv, M9);
#pragma unroll
    for (int a = 0; a < 3; a++) V[t * 3 + a] = Vv[a];
#pragma unroll
    for (int k = 0; k < 9; k++) Mf[t * 9 + k] = M9[k];
  }
}

template <typename T>
__global__ void __launch_bounds__(128) node_ref_bwd_k(NodeIO<T> io, const T* __restrict__ av, const T* __restrict__ bv,
                                                      const T* __restrict__ gI, const T* __restrict__ gV,
                                                      const T* __restrict__ gM, T* dP1, T* dQ1, T* dS1, T* dP2, T* dQ2,
                                                      T* dS2, T* dP3, T* dQ3, T* da, T* db, int64_t NC, int C, int eq) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= NC) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  Vals<T> v;
  load_vals(io, n, c, v);
  Mid<T> m;
  mid(v, m);
  T g[8], gv[3] = {0, 0, 0}, gm[9], a4[4] = {0, 0, 0, 0}, b4[4] = {0, 0, 0, 0};
#pragma unroll
  for (int f = 0; f < 8; f++) g[f] = gI[t * 8 + f];
#pragma unroll
  for (int k = 0; k < 9; k++) gm[k] = 0;
  if (eq) {
#pragma unroll
    for (int k = 0; k < 4; k++) { a4[k] = av[k * C + c]; b4[k] = bv[k * C + c]; }
    if (gV)
#pragma unroll
      for (int a = 0; a < 3; a++) gv[a] = gV[t * 3 + a];
    if (gM)
#pragma unroll
      for (int k = 0; k < 9; k++) gm[k] = gM[t * 9 + k];
  }
  Grads<T> d;
  backward(v, m, g, gv, gm, a4, b4, eq != 0, d);
#pragma unroll
  for (int a = 0; a < 3; a++) { dP1[t * 3 + a] = d.p1[a]; dQ1[t * 3 + a] = d.q1[a]; dS1[t * 3 + a] = d.s1[a]; }
  T s6[6], s10[10];
  fold2(d.p2, s6);
#pragma unroll
  for (int s = 0; s < 6; s++) dP2[t * 6 + s] = s6[s];
  fold2(d.q2, s6);
#pragma unroll
  for (int s = 0; s < 6; s++) dQ2[t * 6 + s] = s6[s];
  fold2(d.s2, s6);
#pragma unroll
  for (int s = 0; s < 6; s++) dS2[t * 6 + s] = s6[s];
  fold3(d.p3, s10);
#pragma unroll
  for (int s = 0; s < 10; s++) dP3[t * 10 + s] = s10[s];
  fold3(d.q3, s10);
#pragma unroll
  for (int s = 0; s < 10; s++) dQ3[t * 10 + s] = s10[s];
  if (eq && da && db) {
#pragma unroll
    for (int k = 0; k < 4; k++) { da[t * 4 + k] = d.da[k]; db[t * 4 + k] = d.db[k]; }
  }
}

// engine layout: y_l (N, k_l, 3C); inv9 (N, 9C) family-major; V (N,3,C); Ms (N,6,C)
__host__ __device__ constexpr int family_body(int f) { return f == 0 ? 2 : (f <= 3 ? 3 : (f <= 7 ? 4 : 5)); }

// engine layout: y_l is (k_l, N, 3C): element (n, c, comp) of P at y_l[(comp*N + n)*3C + c], Q at +C, S at +2C
template <typename T>
__device__ __forceinline__ NodeIO<T> engine_io(const T* y1, const T* y2, const T* y3, int C, int64_t N) {
  NodeIO<T> io;
  const int64_t C3 = 3 * (int64_t)C, pl = N * C3;
  io.P1 = {y1, C3, 1, pl};
  io.Q1 = {y1 + C, C3, 1, pl};
  io.S1 = {y1 + 2 * C, C3, 1, pl};
  io.P2 = {y2, C3, 1, pl};
  io.Q2 = {y2 + C, C3, 1, pl};
  io.S2 = {y2 + 2 * C, C3, 1, pl};
  io.P3 = {y3, C3, 1, pl};
  io.Q3 = {y3 + C, C3, 1, pl};
  return io;
}

template <typename T>
__global__ void __launch_bounds__(128) node_eng_fwd_k(const T* __restrict__ y0, const T* __restrict__ y1,
                                                      const T* __restrict__ y2, const T* __restrict__ y3,
                                                      const T* __restrict__ av, const T* __restrict__ bv,
                                                      T* __restrict__ inv9, T* __restrict__ V, T* __restrict__ Ms,
                                                      int64_t NC, int C, int eq, int max_body) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= NC) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  const int64_t N = NC / C;
  const NodeIO<T> io = engine_io(y1, y2, y3, C, N);
  Vals<T> v;
  load_vals(io, n, c, v);
  Mid<T> m;
  mid(v, m);
  T iv[8];
  invariants(v, m, iv);
  T* o = inv9 + n * 9 * (int64_t)C + c;
  o[0] = family_body(0) <= max_body ? y0[n * 3 * (int64_t)C + c] : T(0);
#pragma unroll
  for (int f = 0; f < 8; f++) o[(int64_t)(f + 1) * C] = family_body(f + 1) <= max_body ? iv[f] : T(0);
  if (eq) {
    T a4[4], b4[4], Vv[3], M9[9];
#pragma unroll
    for (int k = 0; k < 4; k++) { a4[k] = av[k * C + c]; b4[k] = bv[k * C + c]; }
    products(v, m, a4, b4, Vv, M9);
#pragma unroll
    for (int a = 0; a < 3; a++) V[((int64_t)a * N + n) * C + c] = Vv[a];
    // symmetric storage of (Mf + Mf^T)/2, face/model.py:274-276
#pragma unroll
    for (int a = 0; a < 3; a++)
#pragma unroll
      for (int e = a; e < 3; e++)
        Ms[((int64_t)sym2(a, e) * N + n) * C + c] = a == e ? M9[a * 3 + a] : T(0.5) * (M9[a * 3 + e] + M9[e * 3 + a]);
  }
}

template <typename T>
__global__ void __launch_bounds__(128, 4) node_eng_bwd_k(const T* __restrict__ y1, const T* __restrict__ y2,
                                                      const T* __restrict__ y3, const T* __restrict__ av,
                                                      const T* __restrict__ bv, const T* __restrict__ gI9,
                                                      const T* __restrict__ gV, const T* __restrict__ gMs,
                                                      T* __restrict__ dy0, T* __restrict__ dy1, T* __restrict__ dy2,
                                                      T* __restrict__ dy3, int64_t NC, int C, int eq, int max_body) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= NC) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  const int64_t C3 = 3 * (int64_t)C;
  const int64_t N = NC / C;
  const NodeIO<T> io = engine_io(y1, y2, y3, C, N);
  Vals<T> v;
  load_vals(io, n, c, v);
  Mid<T> m;
  mid(v, m);
  const T* gi = gI9 + n * 9 * (int64_t)C + c;
  T g[8], gv[3] = {0, 0, 0}, gm[9], a4[4] = {0, 0, 0, 0}, b4[4] = {0, 0, 0, 0};
#pragma unroll
  for (int f = 0; f < 8; f++) g[f] = family_body(f + 1) <= max_body ? gi[(int64_t)(f + 1) * C] : T(0);
#pragma unroll
  for (int k = 0; k < 9; k++) gm[k] = 0;
  if (eq) {
#pragma unroll
    for (int k = 0; k < 4; k++) { a4[k] = av[k * C + c]; b4[k] = bv[k * C + c]; }
#pragma unroll
    for (int a = 0; a < 3; a++) gv[a] = gV[((int64_t)a * N + n) * C + c];
#pragma unroll
    for (int a = 0; a < 3; a++)
#pragma unroll
      for (int e = 0; e < 3; e++) {
        const T gs = gMs[((int64_t)sym2(a, e) * N + n) * C + c];
        gm[a * 3 + e] = a == e ? gs : T(0.5) * gs;
      }
  }
  Grads<T> d;
  backward(v, m, g, gv, gm, a4, b4, eq != 0, d);
  // rank 0: P0 passes straight through to inv9 family 0; Q0, S0 are unused
  dy0[n * C3 + c] = family_body(0) <= max_body ? gi[0] : T(0);
  dy0[n * C3 + C + c] = 0;
  dy0[n * C3 + 2 * C + c] = 0;
#pragma unroll
  for (int a = 0; a < 3; a++) {
    T* r = dy1 + ((int64_t)a * N + n) * C3 + c;
    r[0] = d.p1[a]; r[C] = d.q1[a]; r[2 * C] = d.s1[a];
  }
  T sp[6], sq[6], ss[6];
  fold2(d.p2, sp); fold2(d.q2, sq); fold2(d.s2, ss);
#pragma unroll
  for (int s = 0; s < 6; s++) {
    T* r = dy2 + ((int64_t)s * N + n) * C3 + c;
    r[0] = sp[s]; r[C] = sq[s]; r[2 * C] = ss[s];
  }
  T tp[10], tq[10];
  fold3(d.p3, tp); fold3(d.q3, tq);
#pragma unroll
  for (int s = 0; s < 10; s++) {
    T* r = dy3 + ((int64_t)s * N + n) * C3 + c;
    r[0] = tp[s]; r[C] = tq[s]; r[2 * C] = 0;
  }
}

template <typename T>
NodeIO<T> ref_io(const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2, const void* S2,
                 const void* P3, const void* Q3, int C) {
  NodeIO<T> io;
  auto mk = [&](const void* p, int k) { return Acc<T>{(const T*)p, (int64_t)C * k, k, 1}; };
  io.P1 = mk(P1, 3); io.Q1 = mk(Q1, 3); io.S1 = mk(S1, 3);
  io.P2 = mk(P2, 6); io.Q2 = mk(Q2, 6); io.S2 = mk(S2, 6);
  io.P3 = mk(P3, 10); io.Q3 = mk(Q3, 10);
  return io;
}

template <typename T>
int ref_fwd(const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2, const void* S2,
            const void* P3, const void* Q3, const void* a, const void* b, void* inv, void* V, void* Mf, int64_t N,
            int C, int eq, void* stream) {
  const int64_t NC = N * C;
  if (NC == 0) return FACEK_OK;
  node_ref_fwd_k<T><<<(unsigned)ceil_div<int64_t>(NC, 128), 128, 0, as_stream(stream)>>>(
      ref_io<T>(P1, Q1, S1, P2, Q2, S2, P3, Q3, C), (const T*)a, (const T*)b, (T*)inv, (T*)V, (T*)Mf, NC, C, eq);
  return launch_status("facek_node_fwd");
}

template <typename T>
int ref_bwd(const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2, const void* S2,
            const void* P3, const void* Q3, const void* a, const void* b, const void* gI, const void* gV,
            const void* gM, void* dP1, void* dQ1, void* dS1, void* dP2, void* dQ2, void* dS2, void* dP3, void* dQ3,
            void* da, void* db, int64_t N, int C, int eq, void* stream) {
  const int64_t NC = N * C;
  if (NC == 0) return FACEK_OK;
  node_ref_bwd_k<T><<<(unsigned)ceil_div<int64_t>(NC, 128), 128, 0, as_stream(stream)>>>(
      ref_io<T>(P1, Q1, S1, P2, Q2, S2, P3, Q3, C), (const T*)a, (const T*)b, (const T*)gI, (const T*)gV,
      (const T*)gM, (T*)dP1, (T*)dQ1, (T*)dS1, (T*)dP2, (T*)dQ2, (T*)dS2, (T*)dP3, (T*)dQ3, (T*)da, (T*)db, NC, C,
      eq);
  return launch_status("facek_node_bwd");
}

template <typename T>
int eng_fwd(const void* y0, const void* y1, const void* y2, const void* y3, const void* a, const void* b, void* inv9,
            void* V, void* Ms, int64_t N, int C, int eq, int max_body, void* stream) {
  const int64_t NC = N * C;
  if (NC == 0) return FACEK_OK;
  node_eng_fwd_k<T><<<(unsigned)ceil_div<int64_t>(NC, 128), 128, 0, as_stream(stream)>>>(
      (const T*)y0, (const T*)y1, (const T*)y2, (const T*)y3, (const T*)a, (const T*)b, (T*)inv9, (T*)V, (T*)Ms, NC,
      C, eq, max_body);
  return launch_status("facek_node_engine_fwd");
}

template <typename T>
int eng_bwd(const void* y1, const void* y2, const void* y3, const void* a, const void* b, const void* gI9,
            const void* gV, const void* gMs, void* dy0, void* dy1, void* dy2, void* dy3, int64_t N, int C, int eq,
            int max_body, void* stream) {
  const int64_t NC = N * C;
  if (NC == 0) return FACEK_OK;
  node_eng_bwd_k<T><<<(unsigned)ceil_div<int64_t>(NC, 128), 128, 0, as_stream(stream)>>>(
      (const T*)y1, (const T*)y2, (const T*)y3, (const T*)a, (const T*)b, (const T*)gI9, (const T*)gV, (const T*)gMs,
      (T*)dy0, (T*)dy1, (T*)dy2, (T*)dy3, NC, C, eq, max_body);
  return launch_status("facek_node_engine_bwd");
}

}  // namespace
}  // namespace facek

using namespace facek;

// ---- per-atom broadcast scaling x[j, n, c] * s[n, c] over the J components of a Cartesian rank
// (face-mlip face/model.py:183-186 and :200-201 moment scaling by the element scale / <neighbours>,
// :277-295 the gates of the equivariant products).  s may be a column slice of a wider row (row stride lds).
// Forward out = x * s; adjoint dx = g * s and, when wanted, ds[n, c] = sum_j g[j, n, c] x[j, n, c].
namespace facek {
namespace {
template <typename T>
__global__ void bcast_mul_k(const T* __restrict__ x, const T* __restrict__ s, T* __restrict__ out, int J, int64_t N,
                            int C, int64_t lds) {
  const int64_t NC = N * C;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < NC; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = q / C;
    const T sv = s[n * lds + (q - n * C)];
    for (int j = 0; j < J; j++) out[j * NC + q] = x[j * NC + q] * sv;
  }
}
// fp32, C % 4 == 0 and 16-byte aligned rows: four channels per thread
__global__ void bcast_mul4_k(const float4* __restrict__ x, const float* __restrict__ s, float4* __restrict__ out,
                             int J, int64_t N, int C4, int64_t lds) {
  const int64_t NC4 = N * C4;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < NC4; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = q / C4;
    const float4 sv = *reinterpret_cast<const float4*>(s + n * lds + 4 * (q - n * C4));
#pragma unroll 2
    for (int j = 0; j < J; j++) {
      const float4 v = x[j * NC4 + q];
      out[j * NC4 + q] = make_float4(v.x * sv.x, v.y * sv.y, v.z * sv.z, v.w * sv.w);
    }
  }
}
template <typename T>
__global__ void bcast_mul_bwd_k(const T* __restrict__ g, const T* __restrict__ x, const T* __restrict__ s,
                                T* __restrict__ dx, T* __restrict__ ds, int J, int64_t N, int C, int64_t lds) {
  const int64_t NC = N * C;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < NC; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = q / C;
    const T sv = s[n * lds + (q - n * C)];
    T acc = 0;
    for (int j = 0; j < J; j++) {
      const T gv = g[j * NC + q];
      dx[j * NC + q] = gv * sv;
      if (ds) acc += gv * x[j * NC + q];
    }
    if (ds) ds[q] = acc;
  }
}
__global__ void bcast_mul_bwd4_k(const float4* __restrict__ g, const float4* __restrict__ x,
                                 const float* __restrict__ s, float4* __restrict__ dx, float4* __restrict__ ds, int J,
                                 int64_t N, int C4, int64_t lds) {
  const int64_t NC4 = N * C4;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < NC4; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = q / C4;
    const float4 sv = *reinterpret_cast<const float4*>(s + n * lds + 4 * (q - n * C4));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < J; j++) {
      const float4 gv = g[j * NC4 + q];
      dx[j * NC4 + q] = make_float4(gv.x * sv.x, gv.y * sv.y, gv.z * sv.z, gv.w * sv.w);
      if (ds) {
        const float4 xv = x[j * NC4 + q];
        acc.x += gv.x * xv.x;
        acc.y += gv.y * xv.y;
        acc.z += gv.z * xv.z;
        acc.w += gv.w * xv.w;
      }
    }
    if (ds) ds[q] = acc;
  }
}
bool vec4_ok(const void* a, const void* b, const void* c, const void* d, int C, int64_t lds) {
  const uintptr_t m = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                      reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(d);
  return (m & 15) == 0 && C % 4 == 0 && lds % 4 == 0;
}
template <typename T>
int bcast_fwd(const void* x, const void* s, void* out, int J, int64_t N, int C, int64_t lds, void* stream) {
  if (std::is_same<T, float>::value && vec4_ok(x, s, out, nullptr, C, lds)) {
    const int64_t n4 = N * (C / 4);
    bcast_mul4_k<<<grid_for(ceil_div<int64_t>(n4, 256), 8), 256, 0, as_stream(stream)>>>(
        (const float4*)x, (const float*)s, (float4*)out, J, N, C / 4, lds);
  } else {
    bcast_mul_k<T><<<grid_for(ceil_div<int64_t>(N * C, 256), 8), 256, 0, as_stream(stream)>>>(
        (const T*)x, (const T*)s, (T*)out, J, N, C, lds);
  }
  return launch_status("facek_bcast_mul_fwd");
}
template <typename T>
int bcast_bwd(const void* g, const void* x, const void* s, void* dx, void* ds, int J, int64_t N, int C, int64_t lds,
              void* stream) {
  if (std::is_same<T, float>::value && vec4_ok(g, s, dx, ds ? x : nullptr, C, lds) &&
      (reinterpret_cast<uintptr_t>(ds) & 15) == 0) {
    const int64_t n4 = N * (C / 4);
    bcast_mul_bwd4_k<<<grid_for(ceil_div<int64_t>(n4, 256), 8), 256, 0, as_stream(stream)>>>(
        (const float4*)g, (const float4*)x, (const float*)s, (float4*)dx, (float4*)ds, J, N, C / 4, lds);
  } else {
    bcast_mul_bwd_k<T><<<grid_for(ceil_div<int64_t>(N * C, 256), 8), 256, 0, as_stream(stream)>>>(
        (const T*)g, (const T*)x, (const T*)s, (T*)dx, (T*)ds, J, N, C, lds);
  }
  return launch_status("facek_bcast_mul_bwd");
}
}  // namespace
}  // namespace facek

extern "C" int facek_node_fwd(int dtype, const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2,
                              const void* S2, const void* P3, const void* Q3, const void* a, const void* b, void* inv,
                              void* V, void* Mf, int64_t N, int32_t C, int32_t eq, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && C > 0, "facek_node_fwd: bad sizes N=%lld C=%d", (long long)N, C);
  FACEK_CHECK_ARG(P1 && Q1 && S1 && P2 && Q2 && S2 && P3 && Q3 && inv, "facek_node_fwd: null tensor");
  FACEK_CHECK_ARG(!eq || (a && b && V && Mf), "facek_node_fwd: eq=1 needs a, b, V, Mf");
  return FACEK_DISPATCH(dtype, ref_fwd, P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, inv, V, Mf, N, C, eq, stream);
}

extern "C" int facek_node_bwd(int dtype, const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2,
                              const void* S2, const void* P3, const void* Q3, const void* a, const void* b,
                              const void* gI, const void* gV, const void* gM, void* dP1, void* dQ1, void* dS1,
                              void* dP2, void* dQ2, void* dS2, void* dP3, void* dQ3, void* da_part, void* db_part,
                              int64_t N, int32_t C, int32_t eq, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && C > 0, "facek_node_bwd: bad sizes N=%lld C=%d", (long long)N, C);
  FACEK_CHECK_ARG(P1 && Q1 && S1 && P2 && Q2 && S2 && P3 && Q3 && gI, "facek_node_bwd: null input");
  FACEK_CHECK_ARG(dP1 && dQ1 && dS1 && dP2 && dQ2 && dS2 && dP3 && dQ3, "facek_node_bwd: null output");
  FACEK_CHECK_ARG(!eq || (a && b), "facek_node_bwd: eq=1 needs a, b");
  return FACEK_DISPATCH(dtype, ref_bwd, P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, gI, gV, gM, dP1, dQ1, dS1, dP2, dQ2,
                        dS2, dP3, dQ3, da_part, db_part, N, C, eq, stream);
}

extern "C" int facek_node_engine_fwd(int dtype, const void* y0, const void* y1, const void* y2, const void* y3,
                                     const void* a, const void* b, void* inv9, void* V, void* Ms, int64_t N, int32_t C,
                                     int32_t eq, int32_t max_body, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && C > 0, "facek_node_engine_fwd: bad sizes N=%lld C=%d", (long long)N, C);
  FACEK_CHECK_ARG(y0 && y1 && y2 && y3 && inv9, "facek_node_engine_fwd: null tensor");
  FACEK_CHECK_ARG(!eq || (a && b && V && Ms), "facek_node_engine_fwd: eq=1 needs a, b, V, Ms");
  return FACEK_DISPATCH(dtype, eng_fwd, y0, y1, y2, y3, a, b, inv9, V, Ms, N, C, eq, max_body, stream);
}

extern "C" int facek_node_engine_bwd(int dtype, const void* y0, const void* y1, const void* y2, const void* y3,
                                     const void* a, const void* b, const void* g_inv9, const void* gV,
                                     const void* gMs, void* dy0, void* dy1, void* dy2, void* dy3, int64_t N, int32_t C,
                                     int32_t eq, int32_t max_body, void* stream) {
  (void)y0;
  FACEK_CHECK_ARG(N >= 0 && C > 0, "facek_node_engine_bwd: bad sizes N=%lld C=%d", (long long)N, C);
  FACEK_CHECK_ARG(y1 && y2 && y3 && g_inv9 && dy0 && dy1 && dy2 && dy3, "facek_node_engine_bwd: null tensor");
  FACEK_CHECK_ARG(!eq || (a && b && gV && gMs), "facek_node_engine_bwd: eq=1 needs a, b, gV, gMs");
  return FACEK_DISPATCH(dtype, eng_bwd, y1, y2, y3, a, b, g_inv9, gV, gMs, dy0, dy1, dy2, dy3, N, C, eq, max_body,
                        stream);
}

extern "C" int facek_bcast_mul_fwd(int dtype, const void* x, const void* s, void* out, int32_t J, int64_t N, int32_t C,
                                   int64_t lds, void* stream) {
  FACEK_CHECK_ARG(J >= 0 && N >= 0 && C > 0 && lds >= C, "facek_bcast_mul_fwd: bad sizes J=%d N=%lld C=%d lds=%lld", J,
                  (long long)N, C, (long long)lds);
  if (J == 0 || N == 0) return FACEK_OK;
  FACEK_CHECK_ARG(x && s && out, "facek_bcast_mul_fwd: null tensor");
  return FACEK_DISPATCH(dtype, bcast_fwd, x, s, out, J, N, C, lds, stream);
}

extern "C" int facek_bcast_mul_bwd(int dtype, const void* g, const void* x, const void* s, void* dx, void* ds,
                                   int32_t J, int64_t N, int32_t C, int64_t lds, void* stream) {
  FACEK_CHECK_ARG(J >= 0 && N >= 0 && C > 0 && lds >= C, "facek_bcast_mul_bwd: bad sizes J=%d N=%lld C=%d lds=%lld", J,
                  (long long)N, C, (long long)lds);
  if (N == 0) return FACEK_OK;
  // J == 0: no components (empty g, x, dx may be null); ds, when wanted, is zeroed
  FACEK_CHECK_ARG(s && ((g && dx) || J == 0), "facek_bcast_mul_bwd: null tensor");
  FACEK_CHECK_ARG(!ds || x || J == 0, "facek_bcast_mul_bwd: ds needs x");
  return FACEK_DISPATCH(dtype, bcast_bwd, g, x, s, dx, ds, J, N, C, lds, stream);
}
