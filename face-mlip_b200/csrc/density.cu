// Factorised Cartesian density of face-mlip's FactorBlock (face/model.py:503-513, face/kernels.py:170-178):
//   D[i, x, b*K + k] = sum_{m in row i} phi[m, b] * msg[m, k] * Y[m, x]      x = 0..19
// and its first-order backward
//   T[m,b,k] = sum_x G[i,x,b,k] Y[m,x];  dphi[m,b] = sum_k msg[m,k] T;  dmsg[m,k] = sum_b phi[m,b] T;
//   dY[m,x] = sum_{b,k} G[i,x,b,k] phi[m,b] msg[m,k].
// Rows are padded (row i = edges i*M .. i*M+M-1, the reference's (N,M,*) tensors) or CSR.
//
// Forward: one CTA per row (segment reduction, no atomics).  Each thread owns a TBxTK block of (b,k)
// channel pairs and all 20 monomials in registers; edge tiles of phi/msg/Y are staged in shared memory and
// read as broadcasts, so each edge costs 20*TB*TK FMAs per thread against ~7 shared loads.
// Backward: one CTA per row with the row's G (20 x B*K) staged in shared memory as [b*K+k][x]; each edge is
// handled by KS threads (a k-chunk each) that walk (b,k) in lockstep, so every G read is a broadcast.  The
// per-edge reductions over k are register-local plus a KS-way shuffle.
#include "common.cuh"

namespace facek {
namespace {

constexpr int NX = 20;
constexpr int FWD_TILE = 32;

// D / G addressing: element (i, x, q) at base[r(x)] + (x - off[r(x)]) * sX + i * sN + q, r(x) the rank of x
// (x in [0,1) [1,4) [4,10) [10,20)).  Reference layout (N,20,BK): one buffer, sN = 20 BK, sX = BK.
// Engine layout: per-rank planes (k_l, N, BK): sN = BK, sX = N BK.
template <typename P>
struct Planes {
  P base[4];
  int64_t sN, sX;
  __device__ __forceinline__ P at(int64_t i, int x) const {
    const int r = x < 1 ? 0 : (x < 4 ? 1 : (x < 10 ? 2 : 3));
    const int o = r == 0 ? 0 : (r == 1 ? 1 : (r == 2 ? 4 : 10));
    return base[r] + (int64_t)(x - o) * sX + i * sN;
  }
};

struct Rows {
  const int32_t* row_ptr;
  int M;
  __device__ __forceinline__ void range(int64_t i, int64_t& s, int& n) const {
    if (row_ptr) {
      s = row_ptr[i];
      n = row_ptr[i + 1] - row_ptr[i];
    } else {
      s = i * (int64_t)M;
      n = M;
    }
  }
};

template <typename T, int TB, int TK>
__global__ void __launch_bounds__(256) dens_fwd_k(const T* __restrict__ phi, const T* __restrict__ msg,
                                                  const T* __restrict__ Y, Planes<T*> D, int64_t N, Rows rows,
                                                  int B, int K) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sY = reinterpret_cast<T*>(smem_raw);        // FWD_TILE * 20
  T* sP = sY + FWD_TILE * NX;                     // FWD_TILE * B
  T* sM = sP + FWD_TILE * B;                      // FWD_TILE * K
  const int nb = B / TB, nk = K / TK;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int tb = tid / nk, tk = tid - (tid / nk) * nk;
  const bool active = tid < nb * nk;
  const int BK = B * K;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    int64_t e0;
    int deg;
    rows.range(i, e0, deg);
    T acc[TB][TK][NX];
#pragma unroll
    for (int a = 0; a < TB; a++)
#pragma unroll
      for (int c = 0; c < TK; c++)
#pragma unroll
        for (int x = 0; x < NX; x++) acc[a][c][x] = T(0);
    for (int t0 = 0; t0 < deg; t0 += FWD_TILE) {
      const int nt = min(FWD_TILE, deg - t0);
      __syncthreads();
      for (int q = tid; q < nt * NX; q += nthr) sY[q] = Y[(e0 + t0) * NX + q];
      for (int q = tid; q < nt * B; q += nthr) sP[q] = phi[(e0 + t0) * B + q];
      for (int q = tid; q < nt * K; q += nthr) sM[q] = msg[(e0 + t0) * K + q];
      __syncthreads();
      if (active) {
        for (int t = 0; t < nt; t++) {
          T y[NX];
#pragma unroll
          for (int x = 0; x < NX; x++) y[x] = sY[t * NX + x];
          T p[TB], m[TK];
#pragma unroll
          for (int a = 0; a < TB; a++) p[a] = sP[t * B + tb + a * nb];
#pragma unroll
          for (int c = 0; c < TK; c++) m[c] = sM[t * K + tk + c * nk];
#pragma unroll
          for (int a = 0; a < TB; a++)
#pragma unroll
            for (int c = 0; c < TK; c++) {
              const T w = p[a] * m[c];
#pragma unroll
              for (int x = 0; x < NX; x++) acc[a][c][x] += w * y[x];
            }
        }
      }
    }
    if (active) {
#pragma unroll
      for (int x = 0; x < NX; x++) {
        T* out = D.at(i, x);
#pragma unroll
        for (int a = 0; a < TB; a++)
#pragma unroll
          for (int c = 0; c < TK; c++) out[(tb + a * nb) * K + tk + c * nk] = acc[a][c][x];
      }
    }
  }
}

template <typename T, int BMAX, int KC>
__global__ void __launch_bounds__(128) dens_bwd_k(const T* __restrict__ phi, const T* __restrict__ msg,
                                                  const T* __restrict__ Y, Planes<const T*> G,
                                                  T* __restrict__ dphi, T* __restrict__ dmsg, T* __restrict__ dY,
                                                  int64_t N, Rows rows, int B, int K, int KS) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sG = reinterpret_cast<T*>(smem_raw);   // (B*K) x 20, x fastest
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int BK = B * K;
  const int kc = tid % KS;                  // this thread's k chunk
  const int slot = tid / KS;                // edge slot within a pass
  const int per_pass = nthr / KS;
  const int k0 = kc * KC;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    int64_t e0;
    int deg;
    rows.range(i, e0, deg);
    __syncthreads();
    for (int q = tid; q < NX * BK; q += nthr) {     // coalesced read of [x][bk], transposed store
      const int x = q / BK, c = q - x * BK;
      sG[c * NX + x] = G.at(i, x)[c];
    }
    __syncthreads();
    for (int t0 = 0; t0 < deg; t0 += per_pass) {
      const int t = t0 + slot;
      const bool live = t < deg && slot < per_pass;
      const int64_t e = e0 + (live ? t : 0);
      T y[NX], dy[NX], p[BMAX], dp[BMAX], m[KC], dm[KC];
#pragma unroll
      for (int x = 0; x < NX; x++) { y[x] = live ? Y[e * NX + x] : T(0); dy[x] = T(0); }
#pragma unroll
      for (int b = 0; b < BMAX; b++) { p[b] = (live && b < B) ? phi[e * B + b] : T(0); dp[b] = T(0); }
#pragma unroll
      for (int c = 0; c < KC; c++) { m[c] = (live && k0 + c < K) ? msg[e * K + k0 + c] : T(0); dm[c] = T(0); }
#pragma unroll
      for (int b = 0; b < BMAX; b++) {
        if (b < B) {
#pragma unroll
          for (int c = 0; c < KC; c++) {
            const int k = k0 + c < K ? k0 + c : K - 1;
            const T* gg = sG + (b * K + k) * NX;
            T gx[NX];
#pragma unroll
            for (int x = 0; x < NX; x++) gx[x] = gg[x];
            T s = 0;
#pragma unroll
            for (int x = 0; x < NX; x++) s += gx[x] * y[x];
            dp[b] += s * m[c];
            dm[c] += s * p[b];
            const T w = p[b] * m[c];
#pragma unroll
            for (int x = 0; x < NX; x++) dy[x] += gx[x] * w;
          }
        }
      }
      // reduce the k-chunk partials of dphi and dY across the KS threads of this edge
      for (int off = 1; off < KS; off <<= 1) {
#pragma unroll
        for (int b = 0; b < BMAX; b++) dp[b] += __shfl_xor_sync(0xffffffffu, dp[b], off);
#pragma unroll
        for (int x = 0; x < NX; x++) dy[x] += __shfl_xor_sync(0xffffffffu, dy[x], off);
      }
      if (live) {
#pragma unroll
        for (int c = 0; c < KC; c++)
          if (k0 + c < K) dmsg[e * K + k0 + c] = dm[c];
        if (kc == 0) {
#pragma unroll
          for (int b = 0; b < BMAX; b++)
            if (b < B) dphi[e * B + b] = dp[b];
#pragma unroll
          for (int x = 0; x < NX; x++) dY[e * NX + x] = dy[x];
        }
      }
    }
  }
}

template <typename T, int TB, int TK>
int launch_fwd(const void* phi, const void* msg, const void* Y, Planes<T*> D, int64_t N, Rows rows, int B, int K,
               void* stream) {
  const int threads = (B / TB) * (K / TK);
  const int threads_r = ceil_div(threads, 32) * 32;
  const size_t smem = sizeof(T) * FWD_TILE * (NX + B + K);
  const int grid = grid_for(N, 8);
  dens_fwd_k<T, TB, TK><<<grid, threads_r, smem, as_stream(stream)>>>((const T*)phi, (const T*)msg, (const T*)Y,
                                                                     D, N, rows, B, K);
  return launch_status("facek_density_fwd");
}

template <typename T>
int density_fwd(const void* phi, const void* msg, const void* Y, Planes<T*> D, int64_t N, int M, int B, int K,
                const int32_t* row_ptr, void* stream) {
  if (N == 0) return FACEK_OK;
  Rows rows{row_ptr, M};
  if constexpr (sizeof(T) == 4) {
    if (B % 2 == 0 && K % 2 == 0 && (B / 2) * (K / 2) <= 256)
      return launch_fwd<T, 2, 2>(phi, msg, Y, D, N, rows, B, K, stream);
  } else {
    if (K % 2 == 0 && B * (K / 2) <= 256) return launch_fwd<T, 1, 2>(phi, msg, Y, D, N, rows, B, K, stream);
  }
  FACEK_CHECK_ARG(B * K <= 256, "facek_density_fwd: B*K=%d unsupported (max 256 with odd B/K, 1024 otherwise)", B * K);
  return launch_fwd<T, 1, 1>(phi, msg, Y, D, N, rows, B, K, stream);
}

template <typename T, int BMAX, int KC>
int launch_bwd(const void* phi, const void* msg, const void* Y, Planes<const T*> G, void* dphi, void* dmsg,
               void* dY, int64_t N, Rows rows, int B, int K, void* stream) {
  int KS = ceil_div(K, KC);
  int ks2 = 1;
  while (ks2 < KS) ks2 <<= 1;                     // shuffle groups are powers of two
  FACEK_CHECK_ARG(ks2 <= 32, "facek_density_bwd: K=%d too large", K);
  const size_t smem = sizeof(T) * (size_t)B * K * NX;
  if (smem > 48 * 1024) {
    FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_density_bwd: G tile %zu B exceeds shared memory", smem);
    cudaFuncSetAttribute(dens_bwd_k<T, BMAX, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  const int grid = grid_for(N, 4);
  dens_bwd_k<T, BMAX, KC><<<grid, 128, smem, as_stream(stream)>>>((const T*)phi, (const T*)msg, (const T*)Y,
                                                                  G, (T*)dphi, (T*)dmsg, (T*)dY, N, rows, B, K, ks2);
  return launch_status("facek_density_bwd");
}

template <typename T>
int density_bwd(const void* phi, const void* msg, const void* Y, Planes<const T*> G, void* dphi, void* dmsg,
                void* dY, int64_t N, int M, int B, int K, const int32_t* row_ptr, void* stream) {
  if (N == 0) return FACEK_OK;
  Rows rows{row_ptr, M};
  FACEK_CHECK_ARG(B <= 32, "facek_density_bwd: B=%d > 32 unsupported", B);
  if constexpr (sizeof(T) == 4) {
    if (B <= 16) return launch_bwd<T, 16, 16>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
    return launch_bwd<T, 32, 8>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
  } else {
    if (B <= 16) return launch_bwd<T, 16, 4>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
    return launch_bwd<T, 32, 4>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
  }
}

template <typename T>
Planes<T*> ref_planes(void* D, int64_t N, int BK) {
  T* b = (T*)D;
  return Planes<T*>{{b, b + BK, b + 4 * (int64_t)BK, b + 10 * (int64_t)BK}, 20 * (int64_t)BK, BK};
}
template <typename T>
Planes<const T*> ref_planes_c(const void* D, int64_t N, int BK) {
  const T* b = (const T*)D;
  return Planes<const T*>{{b, b + BK, b + 4 * (int64_t)BK, b + 10 * (int64_t)BK}, 20 * (int64_t)BK, BK};
}

template <typename T>
int ref_fwd(const void* phi, const void* msg, const void* Y, void* D, int64_t N, int M, int B, int K,
            const int32_t* row_ptr, void* stream) {
  return density_fwd<T>(phi, msg, Y, ref_planes<T>(D, N, B * K), N, M, B, K, row_ptr, stream);
}
template <typename T>
int ref_bwd(const void* phi, const void* msg, const void* Y, const void* G, void* dphi, void* dmsg, void* dY,
            int64_t N, int M, int B, int K, const int32_t* row_ptr, void* stream) {
  return density_bwd<T>(phi, msg, Y, ref_planes_c<T>(G, N, B * K), dphi, dmsg, dY, N, M, B, K, row_ptr, stream);
}
template <typename T>
int xm_fwd(const void* phi, const void* msg, const void* Y, void* D, int64_t N, int B, int K, const int32_t* row_ptr,
           void* stream) {
  T* b = (T*)D;
  const int64_t pl = N * (int64_t)B * K;
  Planes<T*> P{{b, b + pl, b + 4 * pl, b + 10 * pl}, (int64_t)B * K, pl};
  return density_fwd<T>(phi, msg, Y, P, N, 0, B, K, row_ptr, stream);
}
template <typename T>
int xm_bwd(const void* phi, const void* msg, const void* Y, const void* G0, const void* G1, const void* G2,
           const void* G3, void* dphi, void* dmsg, void* dY, int64_t N, int B, int K, const int32_t* row_ptr,
           void* stream) {
  const int64_t pl = N * (int64_t)B * K;
  Planes<const T*> P{{(const T*)G0, (const T*)G1, (const T*)G2, (const T*)G3}, (int64_t)B * K, pl};
  return density_bwd<T>(phi, msg, Y, P, dphi, dmsg, dY, N, 0, B, K, row_ptr, stream);
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_density_fwd(int dtype, const void* phi, const void* msg, const void* Y, void* D, int64_t N,
                                 int32_t M, int32_t B, int32_t K, const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B > 0 && K > 0 && (row_ptr || M >= 0), "facek_density_fwd: bad sizes");
  if (N == 0) return FACEK_OK;
  FACEK_CHECK_ARG(D && (row_ptr || M == 0 || (phi && msg && Y)), "facek_density_fwd: null tensor");
  FACEK_CHECK_ARG(!row_ptr || (phi && msg && Y), "facek_density_fwd: null tensor");
  return FACEK_DISPATCH(dtype, ref_fwd, phi, msg, Y, D, N, M, B, K, row_ptr, stream);
}

extern "C" int facek_density_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G, void* dphi,
                                 void* dmsg, void* dY, int64_t N, int32_t M, int32_t B, int32_t K,
                                 const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B > 0 && K > 0 && (row_ptr || M >= 0), "facek_density_bwd: bad sizes");
  if (N == 0 || (!row_ptr && M == 0)) return FACEK_OK;
  FACEK_CHECK_ARG(phi && msg && Y && G && dphi && dmsg && dY, "facek_density_bwd: null tensor");
  return FACEK_DISPATCH(dtype, ref_bwd, phi, msg, Y, G, dphi, dmsg, dY, N, M, B, K, row_ptr, stream);
}

extern "C" int facek_density_xm_fwd(int dtype, const void* phi, const void* msg, const void* Y, void* D, int64_t N,
                                    int32_t B, int32_t K, const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B > 0 && K > 0 && row_ptr && D, "facek_density_xm_fwd: bad arguments");
  if (N == 0) return FACEK_OK;
  return FACEK_DISPATCH(dtype, xm_fwd, phi, msg, Y, D, N, B, K, row_ptr, stream);
}

extern "C" int facek_density_xm_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G0,
                                    const void* G1, const void* G2, const void* G3, void* dphi, void* dmsg, void* dY,
                                    int64_t N, int32_t B, int32_t K, const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B > 0 && K > 0 && row_ptr && G0 && G1 && G2 && G3, "facek_density_xm_bwd: bad arguments");
  if (N == 0) return FACEK_OK;
  return FACEK_DISPATCH(dtype, xm_bwd, phi, msg, Y, G0, G1, G2, G3, dphi, dmsg, dY, N, B, K, row_ptr, stream);
}
