// Dense fp32 GEMM on the tcgen05 tensor cores for the channel-mixing layers of the FACE engine
// (face-mlip face/model.py:502-534 mix / tmix / proj channel maps, :324-339 output MLP and gate):
//
//   C[M, N] (= or +=) A[M, K] . W[K, N] (+ bias[N])
//
// fp32 accuracy on the tf32 datapath through the 3-term split (tc.cuh). W is constant during a step, so it is
// packed once (facek_gemm_pack) into an "image": for every N tile (Nt columns) and every 32-wide K chunk, a tf32
// hi plane and a lo plane in the K-major operand layout. A is streamed from HBM by cp.async straight into the
// K-major operand layout through a ring of S stages; that raw fp32 plane is the hi operand as the tensor core
// reads it (low mantissa bits ignored), and the CTA writes only the lo plane x - trunc(x) (double-buffered).
// One thread issues 4 K-steps x 3 split terms of M=128 x N=Nt x K=8 MMAs into TMEM.
//
// The tensor core accumulates in fp32 with truncation, so a long chain of MMAs into one accumulator drifts toward
// zero. Each K chunk therefore starts a fresh TMEM partial (two alternate), and the CTA adds the partials in fp32
// registers with round-to-nearest; the truncating chain is one chunk (12 MMAs) long whatever K is. Both
// warpgroups read the partial back (half the columns each); the epilogue adds the bias and, for beta = 1, the
// previous C.
//
// CTAs are persistent over (M tile, N tile) units (consecutive units share the A tile, so its re-reads hit L2);
// the chunk sequence runs across units so the ring keeps prefetching through the epilogue. Two mbarriers
// alternate between consecutive chunks' commits, which keeps every parity wait unambiguous (no barrier is ever
// two phases ahead of its waiter).
#include "common.cuh"
#include "tc.cuh"

namespace facek {
namespace {

using namespace tc;

constexpr int kM = 128;                       // rows per tile (MMA M)
constexpr int kKc = 32;                       // K chunk (fp32 elements)
constexpr int kThr = 256;
constexpr uint32_t kPlane = kM * kKc * 4;     // one 128 x 32 fp32 operand plane (16 KB)

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

struct GemmArgs {
  const float* A;
  int64_t M, K, lda;
  const float* img;           // [n_tiles][k_chunks][hi|lo][Nt x kKc]
  int64_t N;
  int Nt, n_tiles, k_chunks;
  const float* bias;          // (N) or null
  float* C;
  int64_t ldc;
  int beta;                   // 1: C += A.W
  uint32_t tmem_cols;
};

// ring depth per N tile (H16 = Nt / 32 sixteen-column groups per warpgroup): S stages of [A | B hi | B lo] plus
// the two lo planes fill the 227 KB opt-in shared memory of sm_100
template <int H16>
struct Ring {
  static constexpr int S = H16 == 1 ? 8 : H16 == 2 ? 6 : H16 <= 4 ? 4 : 3;
};

// position of a chunk in the CTA's work: tile (mt, nt) and K chunk kc; advanced without divisions per chunk
struct Cursor {
  uint32_t u;
  int64_t mt;
  int nt, kc;
  __device__ void start(uint32_t u0, int n_tiles) {
    u = u0;
    kc = 0;
    mt = u / (uint32_t)n_tiles;
    nt = (int)(u % (uint32_t)n_tiles);
  }
  // returns true when the step enters a new tile
  __device__ bool next(int k_chunks, int n_tiles, uint32_t stride) {
    if (++kc < k_chunks) return false;
    start(u + stride, n_tiles);
    return true;
  }
};

template <int H16>
__global__ void __launch_bounds__(kThr, 1) gemm_tc_k(GemmArgs g) {
  constexpr int S = Ring<H16>::S;
  constexpr int Nt = 32 * H16;
  constexpr int HALF = Nt / 2;                                 // columns per warpgroup
  constexpr uint32_t sb = kPlane + 2u * Nt * kKc * 4;          // stage: A (canonical, = hi operand) | B hi | B lo
  constexpr uint32_t img_chunk = 2u * Nt * kKc;                // floats per (n tile, k chunk)
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* ring = sm;
  unsigned char* lo_planes = sm + S * sb;                      // 2 x A lo
  uint64_t* mbar = reinterpret_cast<uint64_t*>(lo_planes + 2 * kPlane);
  uint32_t* slot = reinterpret_cast<uint32_t*>(mbar + 2);
  int* abort_ = reinterpret_cast<int*>(slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, wg = tid >> 7, row = tid & (kM - 1);
  const uint32_t m_tiles = (uint32_t)((g.M + kM - 1) / kM);
  const uint32_t units = m_tiles * (uint32_t)g.n_tiles;
  const uint32_t my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = (int64_t)my_units * g.k_chunks;

  // ---- producer mapping: lane -> row (lane & 7) of an 8-row group, 16-byte column quad (lane >> 3) + 4h;
  // per warp-instruction 8 rows x 64 contiguous bytes (full sectors), and each 8-lane phase writes 8 distinct
  // rows of one core matrix (conflict-free)
  int p_row[4], p_col[4];
  uint32_t p_off[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int grp = warp * 2 + (i & 1), h = i >> 1;
    p_row[i] = grp * 8 + (lane & 7);
    p_col[i] = ((lane >> 3) + 4 * h) * 4;
    p_off[i] = kmajor_off(p_row[i], p_col[i], kM);
  }
  Cursor pc;                                                   // producer cursor
  pc.start(blockIdx.x, g.n_tiles);
  const float* p_src[4];
  bool p_ok[4];
  auto p_rows = [&]() {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t gr = pc.mt * kM + p_row[i];
      p_ok[i] = gr < g.M;
      p_src[i] = g.A + (p_ok[i] ? gr : 0) * g.lda + p_col[i];
    }
  };
  p_rows();
  int64_t p_next = 0;                                          // next chunk index to prefetch
  auto prefetch = [&]() {
    if (p_next < total) {
      unsigned char* st = ring + (uint32_t)(p_next % S) * sb;
      const int64_t k0 = (int64_t)pc.kc * kKc;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const bool ok = p_ok[i] && k0 + p_col[i] < g.K;
        cp_async16_zfill(st + p_off[i], ok ? p_src[i] + k0 : g.A, ok ? 16u : 0u);
      }
      const float* src = g.img + ((int64_t)pc.nt * g.k_chunks + pc.kc) * img_chunk;
      unsigned char* dst = st + kPlane;
#pragma unroll
      for (int q = tid; q < (int)(img_chunk / 4); q += kThr) cp_async16_zfill(dst + q * 16, src + q * 4, 16u);
      if (pc.next(g.k_chunks, g.n_tiles, gridDim.x)) p_rows();
    }
    p_next++;
    asm volatile("cp.async.commit_group;\n" ::: "memory");     // one group per chunk slot, also past the end
  };

  if (tid == 0) {
    *abort_ = 0;
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, g.tmem_cols);
    tmem_relinquish();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = *slot;
  volatile int* ab = abort_;
  const uint32_t idesc = idesc_tf32(kM, Nt);
  const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16) + wg * HALF;

  // wait for the MMAs of chunk t (commits alternate between the two barriers, chunk t writes TMEM buffer t & 1)
  auto wait_mma = [&](int64_t t) { mbar_wait(&mbar[t & 1], (uint32_t)((t >> 1) & 1), ab); };

  float acc[HALF];
#pragma unroll
  for (int c = 0; c < HALF; c++) acc[c] = 0.f;
  Cursor dc;                                                   // drain cursor (one chunk behind the MMAs)
  dc.start(blockIdx.x, g.n_tiles);

  // fold chunk t's partial into acc; store the tile when t is its last chunk
  auto drain = [&](int64_t t) {
    wait_mma(t);
    fence_after_sync();
    const uint32_t src = tl + (uint32_t)(t & 1) * Nt;
#pragma unroll
    for (int c0 = 0; c0 < HALF; c0 += 16) {
      float v[16];
      tmem_ld16(src + c0, v);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 16; q++) acc[c0 + q] += v[q];
    }
    fence_before_sync();
    if (dc.kc == g.k_chunks - 1) {
      const int64_t grow = dc.mt * kM + row;
      const int64_t gc0 = (int64_t)dc.nt * Nt + wg * HALF;
      if (grow < g.M) {
        float* out = g.C + grow * g.ldc + gc0;
#pragma unroll
        for (int q = 0; q < HALF; q += 4) {
          if (gc0 + q < g.N) {
            float4 o = make_float4(acc[q], acc[q + 1], acc[q + 2], acc[q + 3]);
            if (g.bias) {
              o.x += g.bias[gc0 + q];
              o.y += g.bias[gc0 + q + 1];
              o.z += g.bias[gc0 + q + 2];
              o.w += g.bias[gc0 + q + 3];
            }
            if (g.beta) {
              const float4 p = *reinterpret_cast<const float4*>(out + q);
              o.x += p.x;
              o.y += p.y;
              o.z += p.z;
              o.w += p.w;
            }
            *reinterpret_cast<float4*>(out + q) = o;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < HALF; c++) acc[c] = 0.f;
    }
    dc.next(g.k_chunks, g.n_tiles, gridDim.x);
  };

#pragma unroll 1
  for (int s = 0; s < S - 1; s++) prefetch();

  for (int64_t j = 0; j < total; j++) {
    cp_async_wait_n<S - 2>();                                  // chunk j has landed (this thread's copies)
    fence_proxy_async_smem();
    __syncthreads();                                           // ... and every thread's
    if (*ab) break;                                            // uniform: read between two barriers
    unsigned char* st = ring + (uint32_t)(j % S) * sb;
    unsigned char* lo = lo_planes + (uint32_t)(j & 1) * kPlane;
    // lo plane: x - trunc(x) rounded to tf32; thread owns one row, 4 of the 8 column quads
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t off = kmajor_off(row, (wg * 4 + i) * 4, kM);
      const float4 v = *reinterpret_cast<const float4*>(st + off);
      *reinterpret_cast<float4*>(lo + off) =
          make_float4(to_tf32(v.x - tf32_trunc(v.x)), to_tf32(v.y - tf32_trunc(v.y)), to_tf32(v.z - tf32_trunc(v.z)),
                      to_tf32(v.w - tf32_trunc(v.w)));
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      fence_after_sync();
      const uint32_t ah = smem_u32(st), al = smem_u32(lo);
      const uint32_t bh = ah + kPlane, bl = bh + Nt * kKc * 4;
      const uint32_t dst = tbase + (uint32_t)(j & 1) * Nt;
#pragma unroll
      for (int s = 0; s < kKc / 8; s++) {
        const uint64_t dah = desc_kmajor(ah + s * 2 * kM * 16, kM * 16, 128);
        const uint64_t dal = desc_kmajor(al + s * 2 * kM * 16, kM * 16, 128);
        const uint64_t dbh = desc_kmajor(bh + s * 2 * Nt * 16, Nt * 16, 128);
        const uint64_t dbl = desc_kmajor(bl + s * 2 * Nt * 16, Nt * 16, 128);
        mma_tf32(dst, dal, dbh, idesc, s > 0 ? 1u : 0u);       // small terms first
        mma_tf32(dst, dah, dbl, idesc, 1u);
        mma_tf32(dst, dah, dbh, idesc, 1u);
      }
      commit(&mbar[j & 1]);
    }
    // chunk j-1: its MMAs are done -> fold its partial, free ring stage (j-1)%S and lo plane (j+1)&1
    if (j > 0) drain(j - 1);
    prefetch();
  }
  if (!*ab && total > 0) drain(total - 1);
  cp_async_wait_n<0>();
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.tmem_cols);
  }
}

// image[nt][kc][h][kmajor_off(n, k, Nt) / 4] = split_h(W[kc*32 + k][nt*Nt + n]) (0 outside K x N)
__global__ void gemm_pack_k(const float* __restrict__ W, int64_t K, int64_t N, int64_t sk, int64_t sn, int Nt,
                            int k_chunks, int64_t total, float* __restrict__ img) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(q % kKc);
    const int64_t r = q / kKc;
    const int n = (int)(r % Nt);
    const int64_t r2 = r / Nt;
    const int kc = (int)(r2 % k_chunks);
    const int64_t nt = r2 / k_chunks;
    const int64_t gk = (int64_t)kc * kKc + k, gn = nt * Nt + n;
    const float w = (gk < K && gn < N) ? W[gk * sk + gn * sn] : 0.f;
    const float hi = to_tf32(w);
    float* base = img + (nt * k_chunks + kc) * (2LL * Nt * kKc);
    const uint32_t off = kmajor_off(n, k, Nt) / 4;
    base[off] = hi;
    base[Nt * kKc + off] = to_tf32(w - hi);
  }
}

int pick_nt(int64_t N) {
  // N tile: a multiple of 32 (epilogue halves of 16-column loads) up to 192, so that two ring stages fit next to
  // the operand buffers; wider N runs as 128-column tiles
  const int64_t n32 = (N + 31) / 32 * 32;
  return n32 <= 192 ? (int)n32 : 128;
}

template <int H16>
int launch_gemm(const GemmArgs& g, void* stream) {
  constexpr int Nt = 32 * H16;
  const size_t smem = Ring<H16>::S * (kPlane + 2u * Nt * kKc * 4) + 2 * kPlane + 64;
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_gemm_tc: %zu B of shared memory needed", smem);
  cudaFuncSetAttribute(gemm_tc_k<H16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t units = ((g.M + kM - 1) / kM) * g.n_tiles;
  const int grid = (int)std::min<int64_t>(units, sm_count());
  gemm_tc_k<H16><<<grid, kThr, smem, as_stream(stream)>>>(g);
  return launch_status("facek_gemm_tc");
}

}  // namespace

int gemm_tc_status(int clear) {
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

extern "C" int64_t facek_gemm_image_floats(int64_t K, int64_t N) {
  if (K <= 0 || N <= 0) return 0;
  const int Nt = pick_nt(N);
  const int64_t n_tiles = (N + Nt - 1) / Nt, k_chunks = (K + kKc - 1) / kKc;
  return n_tiles * k_chunks * 2 * Nt * kKc;
}

extern "C" int facek_gemm_pack(const float* W, int64_t K, int64_t N, int64_t stride_k, int64_t stride_n, float* image,
                               void* stream) {
  FACEK_CHECK_ARG(K > 0 && N > 0 && W && image, "facek_gemm_pack: bad arguments");
  const int Nt = pick_nt(N);
  const int64_t n_tiles = (N + Nt - 1) / Nt, k_chunks = (K + kKc - 1) / kKc;
  const int64_t total = n_tiles * k_chunks * Nt * kKc;
  gemm_pack_k<<<grid_for(ceil_div<int64_t>(total, 256), 8), 256, 0, as_stream(stream)>>>(
      W, K, N, stride_k, stride_n, Nt, (int)k_chunks, total, image);
  return launch_status("facek_gemm_pack");
}

extern "C" int facek_gemm_tc(const float* A, int64_t M, int64_t K, int64_t lda, const float* image, int64_t N,
                             const float* bias, float* C, int64_t ldc, int32_t beta, void* stream) {
  FACEK_CHECK_ARG(M >= 0 && K > 0 && N > 0, "facek_gemm_tc: bad sizes M=%lld K=%lld N=%lld", (long long)M,
                  (long long)K, (long long)N);
  if (M == 0) return FACEK_OK;
  FACEK_CHECK_ARG(A && image && C, "facek_gemm_tc: null tensor");
  FACEK_CHECK_ARG(K % 4 == 0 && lda % 4 == 0 && lda >= K && (reinterpret_cast<uintptr_t>(A) & 15) == 0,
                  "facek_gemm_tc: A needs K %% 4 == 0, lda %% 4 == 0, lda >= K and 16-byte alignment");
  FACEK_CHECK_ARG(N % 4 == 0 && ldc % 4 == 0 && ldc >= N && (reinterpret_cast<uintptr_t>(C) & 15) == 0,
                  "facek_gemm_tc: C needs N %% 4 == 0, ldc %% 4 == 0, ldc >= N and 16-byte alignment");
  FACEK_CHECK_ARG((reinterpret_cast<uintptr_t>(image) & 15) == 0, "facek_gemm_tc: image not 16-byte aligned");
  GemmArgs g{};
  g.A = A;
  g.M = M;
  g.K = K;
  g.lda = lda;
  g.img = image;
  g.N = N;
  g.Nt = pick_nt(N);
  g.n_tiles = (int)((N + g.Nt - 1) / g.Nt);
  g.k_chunks = (int)((K + kKc - 1) / kKc);
  g.bias = bias;
  g.C = C;
  g.ldc = ldc;
  g.beta = beta ? 1 : 0;
  uint32_t cols = 32;
  while (cols < 2u * (uint32_t)g.Nt) cols <<= 1;                // two chunk partials
  g.tmem_cols = cols;
  switch (g.Nt / 32) {
    case 1: return launch_gemm<1>(g, stream);
    case 2: return launch_gemm<2>(g, stream);
    case 3: return launch_gemm<3>(g, stream);
    case 4: return launch_gemm<4>(g, stream);
    case 5: return launch_gemm<5>(g, stream);
    default: return launch_gemm<6>(g, stream);
  }
}
