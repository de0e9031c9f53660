// Factorised density on the tcgen05 tensor cores (fp32, B = 16, K = 32, CSR rows, component-major planes):
//   D[x, i, b*32 + k] = sum_{e in row i} Y[e, x] phi[e, b] msg[e, k]
// (face-mlip face/kernels.py:22-54 and face/model.py:503-513).  Per atom i it is one small GEMM
//   D_i[(x, b), k] = sum_e V[e, (x, b)] msg[e, k],   V[e, (x, b)] = Y[e, x] phi[e, b],
// M = (x, b) = 320 rows in three 128-row tiles, N = k = 32, K = the row's edges in steps of 8.  Both operands are
// M/N-major, which is how they are produced: each edge's thread writes its own 320 V values, and a msg row is 32
// contiguous k values.  MN-major tf32 operands use the 128-byte-base-32-byte swizzle: 4 K-rows of 128 bytes per
// atom, 32-byte chunks XOR-ed with (row % 4).
// fp32 accuracy through the 3-term tf32 split (tc.cuh); the chain per tile is at most 3 x ceil(deg/8) MMAs.
//
// Status: exact to fp32 level (tests hold it to 1e-5 of float64) but slower than the CUDA-core kernel on the
// cfg5 alloy (38.8 vs 32.7 ms per launch): each atom runs three serialized build -> MMA -> wait -> store rounds
// in two 4-warp CTAs per SM, so the latencies are exposed.  facek_density_xm_fwd keeps the CUDA-core kernel;
// this one is reachable as facek_density_tc_xm_fwd.
//
// CTA = 128 threads (two per SM): thread (e = t % 64, half = t / 64) builds half of a tile's V groups for edge
// e; thread 0 issues the MMAs; for the epilogue thread t owns TMEM lane t, stages its 32 k values in padded
// shared memory and the tile leaves as coalesced 2 KB x-planes.  Atoms with more than 64 edges accumulate over
// 64-edge blocks; atoms without edges get zero rows.  Every wait is bounded (tc.cuh).
#include "common.cuh"
#include "tc.cuh"

namespace facek {
namespace {

using namespace tc;

constexpr int kNX = 20, kB = 16, kK = 32, kBK = kB * kK;
constexpr int kEB = 64;                              // edges per K block
constexpr int kThreads = 128;
constexpr uint32_t kGroup = kEB * 128;               // one 32-wide MN group x 64 edge rows (8 KB)
constexpr uint32_t kVPlane = 4 * kGroup;             // a 128-row M tile's V (hi or lo) plane, 32 KB
constexpr uint32_t kMsgPlane = kEB * 128;            // msg block (hi or lo), 8 KB
constexpr int kStgRow = 36;                          // epilogue staging row stride (floats)
constexpr uint32_t kSmem = 2 * kVPlane + 2 * kMsgPlane + kThreads * kStgRow * 4 + 64 + 1024;

// byte offset of 16-byte quad q (fp32 elements 4q .. 4q+3 along MN) of K-row r in a 128-byte-base-32-byte
// swizzled MN-major plane: 32-byte chunk q/2 goes to position (q/2) ^ (r % 4)
__device__ __forceinline__ uint32_t sw32b(uint32_t r, uint32_t q) {
  return r * 128u + ((((q >> 1) ^ (r & 3u)) << 5) | ((q & 1u) << 4));
}

// MN-major, 128-byte-base-32-byte swizzle (layout type 1): LBO = stride between 32-wide MN groups, SBO = stride
// between 4-row K groups
__device__ __forceinline__ uint64_t desc_mn_sw32b(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)1u << 61;
  return d;
}
// kind::tf32, D fp32, A and B MN-major
__host__ __device__ constexpr uint32_t idesc_tf32_mn(int M, int N) {
  return idesc_tf32(M, N) | (1u << 15) | (1u << 16);
}

__device__ __forceinline__ float4 split_lo4(float4 v) {
  return make_float4(to_tf32(v.x - to_tf32(v.x)), to_tf32(v.y - to_tf32(v.y)), to_tf32(v.z - to_tf32(v.z)),
                     to_tf32(v.w - to_tf32(v.w)));
}
__device__ __forceinline__ float4 split_hi4(float4 v) {
  return make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
}

__global__ void __launch_bounds__(kThreads, 2)
    dens_fwd_tc_k(const float* __restrict__ phi, const float* __restrict__ msg, const float* __restrict__ Y,
                  float* __restrict__ D, int64_t N, int64_t E, const int32_t* __restrict__ row_ptr) {
  extern __shared__ unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* vhi = sm;
  unsigned char* vlo = vhi + kVPlane;
  unsigned char* mhi = vlo + kVPlane;
  unsigned char* mlo = mhi + kMsgPlane;
  float* stg = reinterpret_cast<float*>(mlo + kMsgPlane);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(stg + kThreads * kStgRow);
  uint32_t* slot = reinterpret_cast<uint32_t*>(mbar + 1);
  int* abort_ = reinterpret_cast<int*>(slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int eb = tid & (kEB - 1), half = tid >> 6;
  const int64_t plane = N * (int64_t)kBK;

  if (tid == 0) {
    *abort_ = 0;
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 128);
    tmem_relinquish();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = *slot;
  const uint32_t tl = tbase + ((uint32_t)(warp * 32) << 16);
  volatile int* ab = abort_;
  uint32_t parity = 0;
  const uint32_t idesc = idesc_tf32_mn(128, kK);

  for (int64_t i = blockIdx.x; i < N; i += gridDim.x) {
    const int64_t e0 = row_ptr[i];
    const int deg = row_ptr[i + 1] - (int)e0;
    if (deg == 0) {                                     // zero rows: 20 planes x 512 floats
      for (int q = tid; q < kNX * kBK / 4; q += kThreads) {
        const int x = q / (kBK / 4), c = q % (kBK / 4);
        reinterpret_cast<float4*>(D + x * plane + i * kBK)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      continue;
    }
    const int nkb = (deg + kEB - 1) / kEB;
    for (int T = 0; T < 3; T++) {
      const int g0 = 4 * T;                             // first 32-wide (x, b) group of this tile
      for (int kb = 0; kb < nkb; kb++) {
        const int nb = min(kEB, deg - kb * kEB);        // edges in this block
        const int64_t eblk = e0 + kb * kEB;
        __syncthreads();                                // previous MMA's operands are no longer read
        // msg block: rows eblk .. eblk+63 (rows past the block are other atoms' edges: V is zero there)
        if (T == 0 || nkb > 1) {
          for (int q = tid; q < kEB * 8; q += kThreads) {
            const int r = q >> 3, c = q & 7;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < nb) v = __ldg(reinterpret_cast<const float4*>(msg + (eblk + r) * kK) + c);
            *reinterpret_cast<float4*>(mhi + sw32b(r, c)) = split_hi4(v);
            *reinterpret_cast<float4*>(mlo + sw32b(r, c)) = split_lo4(v);
          }
        }
        // V groups of this tile for edge eb (two groups per thread half; zero rows past the block)
        const bool live = eb < nb;
        const int64_t e = eblk + eb;
        float p[kB];
#pragma unroll
        for (int b = 0; b < kB; b += 4) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live) v = __ldg(reinterpret_cast<const float4*>(phi + e * kB + b));
          p[b] = v.x;
          p[b + 1] = v.y;
          p[b + 2] = v.z;
          p[b + 3] = v.w;
        }
#pragma unroll
        for (int gs = 0; gs < 2; gs++) {
          const int slotg = 2 * half + gs;              // group slot within the tile
          const int g = g0 + slotg;
          if (g >= 10) continue;                        // tile 2 holds groups 8, 9 only
          const float y0 = live ? __ldg(Y + e * kNX + 2 * g) : 0.f;
          const float y1 = live ? __ldg(Y + e * kNX + 2 * g + 1) : 0.f;
          unsigned char* gh = vhi + slotg * kGroup;
          unsigned char* gl = vlo + slotg * kGroup;
#pragma unroll
          for (int q = 0; q < 8; q++) {                 // 16-byte quad q: (x, b) = (2g + q/4, 4(q%4) .. +3)
            const float y = q < 4 ? y0 : y1;
            const int b = 4 * (q & 3);
            const float4 v = make_float4(y * p[b], y * p[b + 1], y * p[b + 2], y * p[b + 3]);
            *reinterpret_cast<float4*>(gh + sw32b(eb, q)) = split_hi4(v);
            *reinterpret_cast<float4*>(gl + sw32b(eb, q)) = split_lo4(v);
          }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (*ab) break;                                 // uniform (read after the barrier)
        if (tid == 0) {
          fence_after_sync();
          const uint32_t ah = smem_u32(vhi), al = smem_u32(vlo), bh = smem_u32(mhi), bl = smem_u32(mlo);
          const uint32_t dcol = tbase + T * kK;
          const int nks = (nb + 7) / 8;
          for (int s = 0; s < nks; s++) {
            const uint64_t dah = desc_mn_sw32b(ah + s * 1024, kGroup, 512);
            const uint64_t dal = desc_mn_sw32b(al + s * 1024, kGroup, 512);
            const uint64_t dbh = desc_mn_sw32b(bh + s * 1024, kMsgPlane, 512);
            const uint64_t dbl = desc_mn_sw32b(bl + s * 1024, kMsgPlane, 512);
            mma_tf32(dcol, dal, dbh, idesc, (kb > 0 || s > 0) ? 1u : 0u);
            mma_tf32(dcol, dah, dbl, idesc, 1u);
            mma_tf32(dcol, dah, dbh, idesc, 1u);
          }
          commit(mbar);
        }
        mbar_wait(mbar, parity, ab);
        parity ^= 1u;
        fence_after_sync();
      }
      if (*ab) break;
      // epilogue of tile T: lane tid = row m = 128 T + tid = x * 16 + b
      float v[kK];
      tmem_ld16(tl + T * kK, v);
      tmem_ld16(tl + T * kK + 16, v + 16);
      tmem_wait_ld();
      fence_before_sync();
#pragma unroll
      for (int q = 0; q < kK; q += 4)
        *reinterpret_cast<float4*>(stg + tid * kStgRow + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      __syncthreads();
      const int nx = T < 2 ? 8 : 4;                     // x planes in this tile
      for (int q = tid; q < nx * kBK / 4; q += kThreads) {
        const int xl = q / (kBK / 4), c = q % (kBK / 4); // c: float4 index within the 512-float plane row
        const int m = xl * 16 + c / 8, kq = (c % 8) * 4;
        const float4 o = *reinterpret_cast<const float4*>(stg + m * kStgRow + kq);
        reinterpret_cast<float4*>(D + (8 * T + xl) * plane + i * kBK)[c] = o;
      }
    }
    if (*ab) break;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, 128);
  }
}

}  // namespace

int density_tc_xm_fwd(const float* phi, const float* msg, const float* Y, float* D, int64_t N,
                      const int32_t* row_ptr, void* stream) {
  if (N == 0) return FACEK_OK;
  FACEK_CHECK_ARG((int)kSmem <= max_smem_optin(), "facek_density_tc_xm_fwd: %u B of shared memory needed", kSmem);
  cudaFuncSetAttribute(dens_fwd_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  dens_fwd_tc_k<<<grid_for(N, 2), kThreads, kSmem, as_stream(stream)>>>(phi, msg, Y, D, N, 0, row_ptr);
  return launch_status("facek_density_tc_xm_fwd");
}

int density_tc_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(tc::g_tc_status, &zero, sizeof(int));
  }
  return v;
}

}  // namespace facek

using namespace facek;

extern "C" int facek_density_tc_xm_fwd(const float* phi, const float* msg, const float* Y, float* D, int64_t N,
                                       int32_t B, int32_t K, const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && B == 16 && K == 32 && row_ptr && D && (N == 0 || (phi && msg && Y)),
                  "facek_density_tc_xm_fwd: needs B = 16, K = 32 and non-null tensors (got B=%d K=%d)", B, K);
  return density_tc_xm_fwd(phi, msg, Y, D, N, row_ptr, stream);
}
