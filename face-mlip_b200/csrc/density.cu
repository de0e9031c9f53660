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
constexpr int FWD_TILE = 48;                 // one tile per row at the alloys' ~44 neighbours

// D / G addressing: element (i, x, q) at base[r(x)] + (x - off[r(x)]) * sX + i * sN + q, r(x) the rank of x
// (x in [0,1) [1,4) [4,10) [10,20)).  Reference layout (N,20,BK): one buffer, sN = 20 BK, sX = BK.
// Engine layout: per-rank planes (k_l, N, BK): sN = BK, sX = N BK.
template <typename P>
struct Planes {
  P base[4];
  int64_t sN, sX;
  // selects rather than base[rank]: a runtime index into the parameter array would move it to local memory
  __device__ __forceinline__ P at(int64_t i, int x) const {
    const P b = x < 1 ? base[0] : (x < 4 ? base[1] : (x < 10 ? base[2] : base[3]));
    const int o = x < 1 ? 0 : (x < 4 ? 1 : (x < 10 ? 4 : 10));
    return b + (int64_t)(x - o) * sX + i * sN;
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

// Forward.  The CTA walks its rows' edge tiles as one sequence and prefetches tile n+1 (possibly the next row's
// first tile) with cp.async while tile n is consumed, so the staging latency is hidden behind the FMAs.
template <typename T, int TB, int TK>
__global__ void __launch_bounds__(256) dens_fwd_k(const T* __restrict__ phi, const T* __restrict__ msg,
                                                  const T* __restrict__ Y, Planes<T*> D, int64_t N, Rows rows,
                                                  int B, int K) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int tile_elems = FWD_TILE * (NX + B + K);
  // the two tile buffers by offset (a pointer array indexed by the buffer number would live in local memory)
  T* const buf0 = reinterpret_cast<T*>(smem_raw);
  auto buf = [&](int c) { return buf0 + c * tile_elems; };
  const int nb = B / TB, nk = K / TK;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int tb = tid / nk, tk = tid - (tid / nk) * nk;
  const bool active = tid < nb * nk;
  const int BK = B * K;
  auto write_row = [&](int64_t i, T (*acc)[TK][NX]) {
    if (!active) return;
#pragma unroll
    for (int x = 0; x < NX; x++) {
      T* out = D.at(i, x);
#pragma unroll
      for (int a = 0; a < TB; a++)
#pragma unroll
        for (int c = 0; c < TK; c++) out[(tb + a * nb) * K + tk + c * nk] = acc ? acc[a][c][x] : T(0);
    }
  };
  // next (row, tile start) with edges, writing zero rows for empty rows on the way
  auto advance = [&](int64_t& i, int& t0, int64_t& e0, int& deg) {
    t0 += FWD_TILE;
    if (t0 < deg) return;
    t0 = 0;
    for (i += gridDim.x; i < N; i += gridDim.x) {
      rows.range(i, e0, deg);
      if (deg > 0) return;
      write_row(i, nullptr);
    }
  };
  auto issue = [&](T* b, int64_t e0, int t0, int deg) {
    const int nt = min(FWD_TILE, deg - t0);
    T* sY = b;
    T* sP = sY + FWD_TILE * NX;
    T* sM = sP + FWD_TILE * B;
    stage(sY, Y + (e0 + t0) * NX, nt * NX, tid, nthr);
    stage(sP, phi + (e0 + t0) * B, nt * B, tid, nthr);
    stage(sM, msg + (e0 + t0) * K, nt * K, tid, nthr);
    cp_async_commit();
  };
  int64_t i = (int64_t)blockIdx.x - gridDim.x, e0 = 0;
  int t0 = 0, deg = 0;
  advance(i, t0, e0, deg);                      // first non-empty row (t0 = 0)
  if (i < N) issue(buf(0), e0, t0, deg);
  T acc[TB][TK][NX];
#pragma unroll
  for (int a = 0; a < TB; a++)
#pragma unroll
    for (int c = 0; c < TK; c++)
#pragma unroll
      for (int x = 0; x < NX; x++) acc[a][c][x] = T(0);
  int cur = 0;
  while (i < N) {
    int64_t ni = i, ne0 = e0;
    int nt0 = t0, ndeg = deg;
    advance(ni, nt0, ne0, ndeg);
    if (ni < N) {
      issue(buf(cur ^ 1), ne0, nt0, ndeg);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int nt = min(FWD_TILE, deg - t0);
    const T* sY = buf(cur);
    const T* sP = sY + FWD_TILE * NX;
    const T* sM = sP + FWD_TILE * B;
    if (active) {
      for (int t = 0; t < nt; t++) {
        T y[NX];
        if constexpr (sizeof(T) == 4) {                // 5 x 128-bit broadcast loads (80-byte rows)
          const float4* r4 = reinterpret_cast<const float4*>(sY + t * NX);
#pragma unroll
          for (int v = 0; v < NX / 4; v++) {
            const float4 q = r4[v];
            y[4 * v] = q.x; y[4 * v + 1] = q.y; y[4 * v + 2] = q.z; y[4 * v + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int x = 0; x < NX; x++) y[x] = sY[t * NX + x];
        }
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
            if constexpr (sizeof(T) == 4) {            // paired fp32 FMAs over adjacent components
#pragma unroll
              for (int x = 0; x < NX; x += 2) ffma2(acc[a][c][x], acc[a][c][x + 1], w, w, y[x], y[x + 1]);
            } else {
#pragma unroll
              for (int x = 0; x < NX; x++) acc[a][c][x] += w * y[x];
            }
          }
      }
    }
    if (t0 + FWD_TILE >= deg) {                 // row complete
      write_row(i, acc);
#pragma unroll
      for (int a = 0; a < TB; a++)
#pragma unroll
        for (int c = 0; c < TK; c++)
#pragma unroll
          for (int x = 0; x < NX; x++) acc[a][c][x] = T(0);
    }
    __syncthreads();                            // buf[cur] is refilled two tiles from now
    i = ni; e0 = ne0; t0 = nt0; deg = ndeg;
    cur ^= 1;
  }
}

// Backward.  One CTA per row at a time; the row's G (20 x BK, as laid out in global: [x][bk]) sits in shared memory
// and the next row's G is prefetched with cp.async into the other buffer.  Each edge is handled by KS threads, one
// k-chunk of KC channels each, walking (b, k) in lockstep so every G read is a broadcast.  The 20-term dot products
// use four partial sums (independent FMA chains).
template <typename T, int KC, int BMAX>
__global__ void __launch_bounds__(256) dens_bwd_k(const T* __restrict__ phi, const T* __restrict__ msg,
                                                  const T* __restrict__ Y, Planes<const T*> G,
                                                  T* __restrict__ dphi, T* __restrict__ dmsg, T* __restrict__ dY,
                                                  int64_t N, Rows rows, int B, int K, int KS) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int BK = B * K;
  T* sGb[2] = {reinterpret_cast<T*>(smem_raw), reinterpret_cast<T*>(smem_raw) + NX * BK};
  const int kc = tid % KS;                  // this thread's k chunk
  const int slot = tid / KS;                // edge slot within a pass
  const int per_pass = nthr / KS;
  const int k0 = kc * KC;
  auto issue = [&](T* sG, int64_t i) {
#pragma unroll 4
    for (int x = 0; x < NX; x++) stage(sG + x * BK, G.at(i, x), BK, tid, nthr);
    cp_async_commit();
  };
  int cur = 0;
  if ((int64_t)blockIdx.x < N) issue(sGb[0], blockIdx.x);
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    const int64_t inext = i + gridDim.x;
    if (inext < N) {
      issue(sGb[cur ^ 1], inext);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const T* sG = sGb[cur];
    int64_t e0;
    int deg;
    rows.range(i, e0, deg);
    for (int t0 = 0; t0 < deg; t0 += per_pass) {
      const int t = t0 + slot;
      const bool live = t < deg;
      const int64_t e = e0 + (live ? t : 0);
      T y[NX], dy[NX], m[KC], dm[KC];
#pragma unroll
      for (int x = 0; x < NX; x++) { y[x] = live ? Y[e * NX + x] : T(0); dy[x] = T(0); }
#pragma unroll
      for (int c = 0; c < KC; c++) { m[c] = (live && k0 + c < K) ? msg[e * K + k0 + c] : T(0); dm[c] = T(0); }
      T pnext = live ? phi[e * B] : T(0);         // phi_b is loaded one b ahead (hides the load latency)
      for (int b = 0; b < B; b++) {
        const T pb = pnext;
        if (b + 1 < B) pnext = live ? phi[e * B + b + 1] : T(0);
        T dpb = 0;
#pragma unroll
        for (int c = 0; c < KC; c++) {
          const int k = k0 + c < K ? k0 + c : K - 1;
          const T* gg = sG + b * K + k;
          T gx[NX];
#pragma unroll
          for (int x = 0; x < NX; x++) gx[x] = gg[x * BK];
          T s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
          for (int x = 0; x < NX; x += 4) {
            s0 += gx[x] * y[x];
            s1 += gx[x + 1] * y[x + 1];
            s2 += gx[x + 2] * y[x + 2];
            s3 += gx[x + 3] * y[x + 3];
          }
          const T s = (s0 + s1) + (s2 + s3);
          dpb += s * m[c];
          dm[c] += s * pb;
          const T w = pb * m[c];
#pragma unroll
          for (int x = 0; x < NX; x++) dy[x] += gx[x] * w;
        }
        for (int off = 1; off < KS; off <<= 1) dpb += __shfl_xor_sync(0xffffffffu, dpb, off);
        if (live && kc == 0) dphi[e * B + b] = dpb;
      }
      for (int off = 1; off < KS; off <<= 1)
#pragma unroll
        for (int x = 0; x < NX; x++) dy[x] += __shfl_xor_sync(0xffffffffu, dy[x], off);
      if (live) {
#pragma unroll
        for (int c = 0; c < KC; c++)
          if (k0 + c < K) dmsg[e * K + k0 + c] = dm[c];
        if (kc == 0) {
#pragma unroll
          for (int x = 0; x < NX; x++) dY[e * NX + x] = dy[x];
        }
      }
    }
    __syncthreads();                          // sG[cur] is refilled next iteration
    cur ^= 1;
  }
}

template <typename T, int TB, int TK>
int launch_fwd(const void* phi, const void* msg, const void* Y, Planes<T*> D, int64_t N, Rows rows, int B, int K,
               void* stream) {
  const int threads = (B / TB) * (K / TK);
  const int threads_r = ceil_div(threads, 32) * 32;
  const size_t smem = 2 * sizeof(T) * FWD_TILE * (NX + B + K);
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_density_fwd: edge tiles %zu B exceed shared memory", smem);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(dens_fwd_k<T, TB, TK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int grid = grid_for(N, 6);
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

template <typename T, int KC, int BMAX>
int launch_bwd(const void* phi, const void* msg, const void* Y, Planes<const T*> G, void* dphi, void* dmsg,
               void* dY, int64_t N, Rows rows, int B, int K, void* stream) {
  int KS = ceil_div(K, KC);
  int ks2 = 1;
  while (ks2 < KS) ks2 <<= 1;                     // shuffle groups are powers of two
  FACEK_CHECK_ARG(ks2 <= 32, "facek_density_bwd: K=%d too large", K);
  const int threads = ks2 * 48 <= 256 ? ks2 * 48 : 256;   // 48 edge slots per pass (rows of ~45 edges)
  const size_t smem = 2 * sizeof(T) * (size_t)B * K * NX;
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_density_bwd: G tiles %zu B exceed shared memory", smem);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(dens_bwd_k<T, KC, BMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int grid = grid_for(N, 2);
  dens_bwd_k<T, KC, BMAX><<<grid, threads, smem, as_stream(stream)>>>((const T*)phi, (const T*)msg, (const T*)Y, G,
                                                                (T*)dphi, (T*)dmsg, (T*)dY, N, rows, B, K, ks2);
  return launch_status("facek_density_bwd");
}

// Backward, L lanes per edge (fp32, B = 16, K = 32).  A 48 L-thread CTA takes one row (atom) at a time: it stages
// the row's G (20 x 512 fp32, 40 KB) in shared memory with cp.async, then each edge's L lanes walk the 320 rows
// (x, b) of G, each lane reading its 1/L of the row's k range as 16-byte broadcasts:
//   t = sum_k msg[k] g[k] (each lane its part)  ->  dphi[b] += t Y[x],  dY[x] += t phi[b]  (parts joined by shuffles
//   once per x for dY and once per edge for dphi)
//   dmsg[k] += Y[x] phi[b] g[k]
// msg and dmsg parts of the edge in registers.  48 edges per round keeps ~90% of the lanes busy at the alloys'
// ~44 neighbours; five CTAs share an SM, so one CTA's staging overlaps the others' work.  The five G tiles leave
// the SM's L1 cache only ~28 KB, so per-edge global operands come from L2: each component's Y[e, x] is loaded one
// iteration ahead, and the message tables of component c + 1 while component c is contracted.
// With MSG, the lanes also add the message part of dY: msg[e,k] = sum_{c<nc} Y[e,c] (TJ[c,ej,k] + TI[c,ei,k]), so
// dY[e,c] += sum_k dmsg[e,k] (TJ[c,ej,k] + TI[c,ei,k]) while dmsg is still in registers (TI may be null).
template <int BB, int KK, int L, bool MSG>
__global__ void __launch_bounds__(48 * L, L >= 4 ? 4 : 5)
    dens_bwd_lane_k(const float* __restrict__ phi, const float* __restrict__ msg, const float* __restrict__ Y,
                    Planes<const float*> G, float* __restrict__ dphi, float* __restrict__ dmsg, float* __restrict__ dY,
                    int64_t N, Rows rows, const float* __restrict__ TJ, const float* __restrict__ TI,
                    const int32_t* __restrict__ ej, int nc) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sG = reinterpret_cast<float*>(smem_raw);              // [x][b][k]
  constexpr int BK = BB * KK, KH = KK / L;
  const int tid = threadIdx.x, half = tid % L, slot = tid / L;
  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    int64_t e0;
    int deg;
    rows.range(i, e0, deg);
    if (deg == 0) continue;
    __syncthreads();                                           // previous row's readers are done with sG
#pragma unroll 4
    for (int x = 0; x < NX; x++) stage(sG + x * BK, G.at(i, x), BK, tid, 48 * L);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int t0 = 0; t0 < deg; t0 += 48) {
      // the L lanes of an edge take the same branch, so the shuffles below see complete lane groups
      if (t0 + slot >= deg) break;
      const int64_t e = e0 + t0 + slot;
      float m[KH], dm[KH], p[BB], dp[BB];
#pragma unroll
      for (int k = 0; k < KH; k += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(msg + e * KK + half * KH + k));
        m[k] = v.x;
        m[k + 1] = v.y;
        m[k + 2] = v.z;
        m[k + 3] = v.w;
        dm[k] = dm[k + 1] = dm[k + 2] = dm[k + 3] = 0.f;
      }
#pragma unroll
      for (int b = 0; b < BB; b += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(phi + e * BB + b));
        p[b] = v.x;
        p[b + 1] = v.y;
        p[b + 2] = v.z;
        p[b + 3] = v.w;
        dp[b] = dp[b + 1] = dp[b + 2] = dp[b + 3] = 0.f;
      }
      const unsigned pair_mask = __activemask();
      const float* ye = Y + e * NX;
      float ynext = __ldg(ye);
#pragma unroll 1
      for (int x = 0; x < NX; x++) {
        const float yx = ynext;
        if (x + 1 < NX) ynext = __ldg(ye + x + 1);
        const float* gx = sG + x * BK + half * KH;
        float dyx = 0.f;
#pragma unroll
        for (int b = 0; b < BB; b++) {
          float g[KH];
#pragma unroll
          for (int k = 0; k < KH; k += 4) {
            const float4 v = *reinterpret_cast<const float4*>(gx + b * KK + k);
            g[k] = v.x;
            g[k + 1] = v.y;
            g[k + 2] = v.z;
            g[k + 3] = v.w;
          }
          float t0_ = 0.f, t1 = 0.f;
#pragma unroll
          for (int k = 0; k < KH; k += 2) ffma2(t0_, t1, m[k], m[k + 1], g[k], g[k + 1]);
          // this lane's part of t: dp and dY are linear in t, so the lanes' parts are joined once per x (dY)
          // and once per edge (dphi) instead of once per (x, b)
          const float t = t0_ + t1;
          dp[b] += t * yx;
          dyx += t * p[b];
          const float w = yx * p[b];
#pragma unroll
          for (int k = 0; k < KH; k += 2) ffma2(dm[k], dm[k + 1], w, w, g[k], g[k + 1]);
        }
#pragma unroll
        for (int o = 1; o < L; o <<= 1) dyx += __shfl_xor_sync(pair_mask, dyx, o);
        if (half == 0) dY[e * NX + x] = dyx;
      }
#pragma unroll
      for (int b = 0; b < BB; b++)
#pragma unroll
        for (int o = 1; o < L; o <<= 1) dp[b] += __shfl_xor_sync(pair_mask, dp[b], o);
      if (half == 0) {
#pragma unroll
        for (int b = 0; b < BB; b += 4)
          *reinterpret_cast<float4*>(dphi + e * BB + b) = make_float4(dp[b], dp[b + 1], dp[b + 2], dp[b + 3]);
      }
#pragma unroll
      for (int k = 0; k < KH; k += 4)
        *reinterpret_cast<float4*>(dmsg + e * KK + half * KH + k) = make_float4(dm[k], dm[k + 1], dm[k + 2], dm[k + 3]);
      if (MSG) {
        const int64_t NKs = N * KK;
        const float* tjb = TJ + (int64_t)ej[e] * KK + half * KH;
        const float* tib = TI ? TI + i * KK + half * KH : nullptr;
        // tables of component c in (nj, ni), of c + 1 in flight
        float4 nj[KH / 4], ni[KH / 4];
#pragma unroll
        for (int k = 0; k < KH; k += 4) {
          nj[k / 4] = nc > 0 ? __ldg(reinterpret_cast<const float4*>(tjb + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
          ni[k / 4] = tib && nc > 0 ? __ldg(reinterpret_cast<const float4*>(tib + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll 1
        for (int c = 0; c < nc; c++) {
          float4 a[KH / 4];
#pragma unroll
          for (int q = 0; q < KH / 4; q++)
            a[q] = make_float4(nj[q].x + ni[q].x, nj[q].y + ni[q].y, nj[q].z + ni[q].z, nj[q].w + ni[q].w);
          if (c + 1 < nc) {
#pragma unroll
            for (int k = 0; k < KH; k += 4) {
              nj[k / 4] = __ldg(reinterpret_cast<const float4*>(tjb + (c + 1) * NKs + k));
              if (tib) ni[k / 4] = __ldg(reinterpret_cast<const float4*>(tib + (c + 1) * NKs + k));
            }
          }
          float sc = 0.f;
#pragma unroll
          for (int k = 0; k < KH; k += 4) {
            const float4 v = a[k / 4];
            sc += (dm[k] * v.x + dm[k + 1] * v.y) + (dm[k + 2] * v.z + dm[k + 3] * v.w);
          }
#pragma unroll
          for (int o = 1; o < L; o <<= 1) sc += __shfl_xor_sync(pair_mask, sc, o);
          if (half == 0) dY[e * NX + c] += sc;
        }
      }
    }
  }
}

template <typename T>
int density_bwd(const void* phi, const void* msg, const void* Y, Planes<const T*> G, void* dphi, void* dmsg,
                void* dY, int64_t N, int M, int B, int K, const int32_t* row_ptr, void* stream) {
  if (N == 0) return FACEK_OK;
  Rows rows{row_ptr, M};
  FACEK_CHECK_ARG(B <= 32, "facek_density_bwd: B=%d > 32 unsupported", B);
  if constexpr (sizeof(T) == 4) {
    if (B == 16 && K == 32) {                          // flagship shape: lane-per-edge kernel, G in shared memory
      const size_t smem = sizeof(float) * NX * 16 * 32;
      cudaFuncSetAttribute(dens_bwd_lane_k<16, 32, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      dens_bwd_lane_k<16, 32, 2, false><<<grid_for(N, 5), 48 * 2, smem, as_stream(stream)>>>(
          (const float*)phi, (const float*)msg, (const float*)Y, G, (float*)dphi, (float*)dmsg, (float*)dY, N, rows,
          nullptr, nullptr, nullptr, 0);
      return launch_status("facek_density_bwd");
    }
    if (B <= 16) return launch_bwd<T, 8, 16>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
    return launch_bwd<T, 8, 32>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
  } else {
    if (B <= 16) return launch_bwd<T, 4, 16>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
    return launch_bwd<T, 4, 32>(phi, msg, Y, G, dphi, dmsg, dY, N, rows, B, K, stream);
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

// density adjoint plus the message part of dY (xm layout, CSR rows): the lane kernel does both for fp32 B=16 K=32;
// other shapes run the density adjoint and then the message dY kernel accumulating into dY
template <typename T>
int xm_msg_bwd(const void* phi, const void* msg, const void* Y, const void* G0, const void* G1, const void* G2,
               const void* G3, const void* TJ, const void* TI, const int32_t* ei, const int32_t* ej, int nc,
               void* dphi, void* dmsg, void* dY, int64_t N, int64_t E, int B, int K, const int32_t* row_ptr,
               void* stream) {
  if (std::is_same<T, float>::value && B == 16 && K == 32) {
    const int64_t pl = N * (int64_t)B * K;
    Planes<const float*> P{{(const float*)G0, (const float*)G1, (const float*)G2, (const float*)G3}, (int64_t)B * K,
                           pl};
    const size_t smem = sizeof(float) * NX * 16 * 32;
    cudaFuncSetAttribute(dens_bwd_lane_k<16, 32, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dens_bwd_lane_k<16, 32, 2, true><<<grid_for(N, 5), 48 * 2, smem, as_stream(stream)>>>(
        (const float*)phi, (const float*)msg, (const float*)Y, P, (float*)dphi, (float*)dmsg, (float*)dY, N,
        Rows{row_ptr, 0}, (const float*)TJ, (const float*)TI, ej, nc);
    return launch_status("facek_density_msg_xm_bwd");
  }
  int st = xm_bwd<T>(phi, msg, Y, G0, G1, G2, G3, dphi, dmsg, dY, N, B, K, row_ptr, stream);
  if (st) return st;
  return edge_msg_dy(sizeof(T) == 4 ? FACEK_F32 : FACEK_F64, ei, ej, TJ, TI, dmsg, nc, K, N, E, dY, stream);
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_density_msg_xm_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G0,
                                        const void* G1, const void* G2, const void* G3, const void* TJ,
                                        const void* TI, const int32_t* ei, const int32_t* ej, int32_t nc, void* dphi,
                                        void* dmsg, void* dY, int64_t N, int64_t E, int32_t B, int32_t K,
                                        const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && E >= 0 && B > 0 && K > 0 && nc >= 1 && nc <= 10 && row_ptr && G0 && G1 && G2 && G3 &&
                      TJ && ei && ej,
                  "facek_density_msg_xm_bwd: bad arguments");
  if (N == 0) return FACEK_OK;
  return FACEK_DISPATCH(dtype, xm_msg_bwd, phi, msg, Y, G0, G1, G2, G3, TJ, TI, ei, ej, nc, dphi, dmsg, dY, N, E, B,
                        K, row_ptr, stream);
}

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
