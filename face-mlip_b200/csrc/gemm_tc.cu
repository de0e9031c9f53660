// Dense fp32 GEMM on the tcgen05 tensor cores for the channel-mixing layers of the FACE engine
// (face-mlip face/model.py:502-534 mix / tmix / proj channel maps, :324-339 output MLP and gate):
//
//   C[M, N] (= or +=) A[M, K] . W[K, N] (+ bias[N])
//
// A and C may each come as two column blocks (facek_gemm_tc_split): A = [A1 | A2] split at a multiple of 32 columns
// (the A producer takes each 32-wide K chunk from one of two tensor maps) and C = [C1 | C2] split at a multiple of 32
// (each 32-column store block goes to one of two outputs), so a layer on concatenated features reads its inputs
// where they are and its adjoint writes the two input gradients as separate tensors, with no concatenation copy.
//
// fp32 accuracy on the tf32 datapath through the 3-term split (tc.cuh). W is constant during a step, so it is
// packed once (facek_gemm_pack) into an "image": for every N tile (Nt columns) and every 32-wide K chunk, a tf32
// hi plane and a lo plane in the K-major no-swizzle operand layout.
//
// Warp roles (384 threads; each single-thread role has a warp of its own so that no role's waits stall another):
//   warp 8, lane 0     A producer: per K chunk one TMA 2D load of the 128 x 32 fp32 A tile into a 128-byte-
//                      swizzled K-major stage of a deep ring (the hi operand as the tensor core reads raw fp32);
//   warp 9, lane 0     W producer: one bulk copy of the chunk's W image into a shallow ring (L2-resident data);
//                      stages complete on "full" mbarriers and are reused after the MMAs that read them commit
//                      to their "empty" mbarriers, so the HBM stream runs SA - 1 chunks ahead of the MMAs.
//   warps 10, 11,      MMA issuers, even and odd chunks: once all 256 compute threads have arrived on the chunk's
//   lane 0             "split" mbarrier and its A and W chunks have landed, 4 K-steps x 3 split terms of M=128 x
//                      N=Nt x K=8 MMAs into one of four TMEM partials, then commits to the partial's, the A
//                      stage's and the W stage's mbarriers.  The MMA queue holds only a few instructions and each
//                      issuer's three barrier checks take several hundred cycles, so with one issuer the tensor
//                      pipe idled while it checked; with two, one issuer's checks overlap the other's MMAs.  Each
//                      chunk owns its partial, lo plane and ring stages, and a commit tracks only the issuing
//                      thread's MMAs, so the two need no ordering between them.
//   warps 0-7          split: lo = tf32(x - trunc(x)) into one of four lo planes (same swizzle), arrive; the
//                      partial of the chunk three behind is loaded from TMEM while the split runs and folded into
//                      fp32 registers; a finished tile leaves through padded shared memory as coalesced
//                      16-byte stores (bias and accumulate applied there).  No block-wide barrier per chunk.
// Tile store: tiles of 64 or 128 columns leave by TMA (each warpgroup writes its rows' 32-column block into a
// 128-byte-swizzled staging block, one thread issues a bulk tensor store, or a bulk tensor add when accumulating
// into C, and the warpgroup moves on while the copy engine writes HBM); other widths store through padded shared
// memory as coalesced 16-byte stores.  The asynchronous store keeps the compute warps' epilogue short for the
// output-heavy adjoint maps (K = 64, N = 512), where it had been the longest step of each tile.
// The tensor core accumulates in fp32 with truncation, so a long chain of MMAs into one accumulator drifts toward
// zero; each K chunk therefore starts a fresh TMEM partial (four rotate) and the partials are summed in
// registers with round-to-nearest (the truncating chain is 12 MMAs long whatever K is).
//
// CTAs are persistent over (M tile, N tile) units (consecutive units share the A tile, so its re-reads hit L2).
// Every mbarrier wait is bounded and parity-safe: no barrier is ever two phases ahead of a waiter.
#include <cuda.h>

#include <cstring>

#include "common.cuh"
#include "tc.cuh"

namespace facek {
namespace {

using namespace tc;

constexpr int kM = 128;                       // rows per tile (MMA M)
constexpr int kKc = 32;                       // K chunk (fp32 elements) = one 128-byte swizzle row
constexpr int kCompute = 256;                 // warps 0-7
constexpr int kThr = kCompute + 128;          // + A producer, W producer and two MMA issuer warps
constexpr uint32_t kPlane = kM * kKc * 4;     // one 128 x 32 fp32 operand plane (16 KB)

struct GemmArgs {
  int64_t M, K;
  const float* img;           // [n_tiles][k_chunks][hi|lo][Nt x kKc]
  int64_t N;
  int Nt, n_tiles, k_chunks;
  const float* bias;          // (N) or null
  float* C;
  int64_t ldc;
  int beta;                   // 1: C += A.W
  uint32_t tmem_cols;
  int k1_chunks;              // K chunks read from the first A map; the rest from the second (= k_chunks: one map)
  int64_t n1;                 // output columns [0, n1) to C / cmap, [n1, N) to C2 / cmap2 (= N: one output)
  float* C2;
  int64_t ldc2;
};

// Shared memory per N tile (H16 = Nt / 32): a deep ring of SA A tiles (the only HBM stream), a shallow ring of SW
// W chunks (hi + lo, L2-resident), kLo lo planes; with 1 KB alignment slack this fills the 227 KB opt-in shared
// memory of sm_100.
template <int H16>
struct Ring {
  static constexpr int SA = H16 == 1 ? 6 : H16 == 2 ? 4 : H16 == 3 ? 4 : 3;
  static constexpr int SW = H16 == 1 ? 3 : H16 == 2 ? 3 : 2;
};
constexpr int kStgRow = 36;                   // epilogue staging row stride (floats): conflict-free both ways
constexpr uint32_t kStg = kM * kStgRow * 4;   // per warpgroup (18 KB): a 128 x 32 column block
constexpr int kLag = 3;                       // a chunk's TMEM partial is folded kLag iterations after its MMAs
constexpr int kNB = kLag + 1;                 // TMEM partials and lo planes in rotation

// byte offset of the 16-byte quad q of row r in a 128-byte-swizzled K-major plane (1024-byte aligned)
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t q) { return r * 128u + ((q ^ (r & 7u)) << 4); }

// shared-memory descriptor, K-major, 128-byte swizzle: 8-row atoms of 1024 B (SBO), LBO unused (1)
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(mbar))
               : "memory");
}

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
  __device__ void next(int k_chunks, int n_tiles, uint32_t stride) {
    if (++kc < k_chunks) return;
    start(u + stride, n_tiles);
  }
};

// bulk tensor store / add of a 2D box from shared memory (async proxy), grouped per thread
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_add_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// this thread's bulk groups have finished reading their shared-memory sources
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's bulk groups are complete (global writes performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mbar)) : "memory");
}

template <int H16>
__global__ void __launch_bounds__(kThr, 1) gemm_tc_k(const __grid_constant__ CUtensorMap amap,
                                                     const __grid_constant__ CUtensorMap amap2,
                                                     const __grid_constant__ CUtensorMap cmap,
                                                     const __grid_constant__ CUtensorMap cmap2, GemmArgs g) {
  constexpr int SA = Ring<H16>::SA, SW = Ring<H16>::SW;
  constexpr int Nt = 32 * H16;
  constexpr int HALF = Nt / 2;                                 // columns per compute warpgroup
  constexpr bool kTmaOut = HALF % 32 == 0;                     // tile store by TMA (Nt = 64, 128)
  constexpr uint32_t wbytes = 2u * Nt * kKc * 4;               // W hi + lo of one chunk
  extern __shared__ unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);   // 1024-byte aligned
  unsigned char* aring = sm;                                   // SA x A tile (swizzled; = hi operand)
  unsigned char* lo_planes = aring + SA * kPlane;              // kNB x A lo (same swizzle)
  unsigned char* wring = lo_planes + kNB * kPlane;             // SW x [W hi | W lo]
  float* stage_out = reinterpret_cast<float*>(wring + SW * wbytes);   // 2 x epilogue staging
  uint64_t* fullA = reinterpret_cast<uint64_t*>(wring + SW * wbytes + 2 * kStg);
  uint64_t* emptyA = fullA + SA;
  uint64_t* fullW = emptyA + SA;
  uint64_t* emptyW = fullW + SW;
  uint64_t* mma_bar = emptyW + SW;                             // [kNB] MMAs of chunk j done (partial j % kNB)
  uint64_t* split_bar = mma_bar + kNB;                         // [kNB] lo plane j % kNB written (256 arrivals)
  uint32_t* slot = reinterpret_cast<uint32_t*>(split_bar + kNB);
  int* abort_ = reinterpret_cast<int*>(slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, wg = (tid >> 7) & 1, row = tid & (kM - 1);
  const uint32_t m_tiles = (uint32_t)((g.M + kM - 1) / kM);
  const uint32_t units = m_tiles * (uint32_t)g.n_tiles;
  const uint32_t my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = (int64_t)my_units * g.k_chunks;

  if (tid == 0) {
    *abort_ = 0;
    for (int s = 0; s < SA; s++) {
      mbar_init(&fullA[s], 1);
      mbar_init(&emptyA[s], 1);
    }
    for (int s = 0; s < SW; s++) {
      mbar_init(&fullW[s], 1);
      mbar_init(&emptyW[s], 1);
    }
    for (int b = 0; b < kNB; b++) {
      mbar_init(&mma_bar[b], 1);
      mbar_init(&split_bar[b], kCompute);
    }
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

  if (warp >= 8) {
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------------- A producer (TMA, deep ring)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
      if (g.k1_chunks < g.k_chunks)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap2)) : "memory");
      Cursor pc;
      pc.start(blockIdx.x, g.n_tiles);
      for (int64_t j = 0; j < total; j++) {
        const int s = (int)(j % SA);
        if (j >= SA && !mbar_wait(&emptyA[s], (uint32_t)(((j / SA) - 1) & 1), ab)) break;
        mbar_expect_tx(&fullA[s], kPlane);
        if (pc.kc < g.k1_chunks)      // A = [A1 | A2] split at a 32-column chunk (k1_chunks = k_chunks: no A2)
          tma_load_2d(aring + (uint32_t)s * kPlane, &amap, pc.kc * kKc, (int)(pc.mt * kM), &fullA[s]);
        else
          tma_load_2d(aring + (uint32_t)s * kPlane, &amap2, (pc.kc - g.k1_chunks) * kKc, (int)(pc.mt * kM),
                      &fullA[s]);
        pc.next(g.k_chunks, g.n_tiles, gridDim.x);
      }
    } else if (warp == 9 && lane == 0) {
      // ---------------------------------------------------------------- W producer (bulk copies, shallow ring)
      Cursor pc;
      pc.start(blockIdx.x, g.n_tiles);
      for (int64_t j = 0; j < total; j++) {
        const int s = (int)(j % SW);
        if (j >= SW && !mbar_wait(&emptyW[s], (uint32_t)(((j / SW) - 1) & 1), ab)) break;
        mbar_expect_tx(&fullW[s], wbytes);
        bulk_load(wring + (uint32_t)s * wbytes, g.img + ((int64_t)pc.nt * g.k_chunks + pc.kc) * (wbytes / 4), wbytes,
                  &fullW[s]);
        pc.next(g.k_chunks, g.n_tiles, gridDim.x);
      }
    } else if (warp >= 10 && lane == 0) {
      // ---------------------------------------------------------------- MMA issuers (warp 10 even, 11 odd chunks)
      const uint32_t idesc = idesc_tf32(kM, Nt);
      for (int64_t j = warp - 10; j < total; j += 2) {
        const int sa = (int)(j % SA), sw = (int)(j % SW), b = (int)(j % kNB);
        if (!mbar_wait(&fullA[sa], (uint32_t)((j / SA) & 1), ab)) break;       // A tile landed (TMA)
        if (!mbar_wait(&split_bar[b], (uint32_t)((j / kNB) & 1), ab)) break;   // lo plane written
        if (!mbar_wait(&fullW[sw], (uint32_t)((j / SW) & 1), ab)) break;       // W chunk landed
        fence_after_sync();
        const uint32_t ah = smem_u32(aring + (uint32_t)sa * kPlane), al = smem_u32(lo_planes + (uint32_t)b * kPlane);
        const uint32_t bh = smem_u32(wring + (uint32_t)sw * wbytes), bl = bh + Nt * kKc * 4;
        const uint32_t dst = tbase + (uint32_t)b * Nt;
#pragma unroll
        for (int k = 0; k < kKc / 8; k++) {
          const uint64_t dah = desc_sw128(ah + k * 32), dal = desc_sw128(al + k * 32);
          const uint64_t dbh = desc_kmajor(bh + k * 2 * Nt * 16, Nt * 16, 128);
          const uint64_t dbl = desc_kmajor(bl + k * 2 * Nt * 16, Nt * 16, 128);
          mma_tf32(dst, dal, dbh, idesc, k > 0 ? 1u : 0u);     // small terms first
          mma_tf32(dst, dah, dbl, idesc, 1u);
          mma_tf32(dst, dah, dbh, idesc, 1u);
        }
        commit(&mma_bar[b]);
        commit(&emptyA[sa]);
        commit(&emptyW[sw]);
      }
    }
  } else {
    // ------------------------------------------------------------------ compute warps (no block-wide barrier)
    const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16) + wg * HALF;
    float acc[HALF];
#pragma unroll
    for (int c = 0; c < HALF; c++) acc[c] = 0.f;
    Cursor dc;                                                 // drain cursor (kLag chunks behind the split)
    dc.start(blockIdx.x, g.n_tiles);

    // chunk t's partial: wait for its MMAs and start the TMEM loads (completed by drain_finish)
    float part[HALF];
    auto drain_start = [&](int64_t t) -> bool {
      if (!mbar_wait(&mma_bar[t % kNB], (uint32_t)((t / kNB) & 1), ab)) return false;
      fence_after_sync();
      const uint32_t src = tl + (uint32_t)(t % kNB) * Nt;
#pragma unroll
      for (int c0 = 0; c0 < HALF; c0 += 16) tmem_ld16(src + c0, part + c0);
      return true;
    };
    // fold it into acc; store the tile when t is its last chunk
    auto drain_finish = [&]() {
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < HALF; q++) acc[q] += part[q];
      fence_before_sync();
      if (dc.kc == g.k_chunks - 1) {
        // tile store: the warpgroup's HALF columns in blocks of up to 32 go through padded shared memory and
        // leave as coalesced 16-byte stores (8 lanes cover 128 contiguous bytes of one row)
        const int64_t row0 = dc.mt * kM;
        const int64_t gcb = (int64_t)dc.nt * Nt + wg * HALF;
        float* stg = stage_out + wg * (kStg / 4);
        if constexpr (kTmaOut) {
          // dense 128 x 32 block, 16-byte quad q of row r at sw128(r, q) (the TMA box layout, 128-byte swizzle)
          unsigned char* sb = reinterpret_cast<unsigned char*>(stg);
#pragma unroll
          for (int cb = 0; cb < HALF; cb += 32) {
            if (row == 0) bulk_wait_read();                      // the previous store has read the staging
            bar_sync(1 + wg, kM);
            const int64_t gc0 = gcb + cb;
#pragma unroll
            for (int q = 0; q < 8; q++) {
              float4 o = make_float4(acc[cb + 4 * q], acc[cb + 4 * q + 1], acc[cb + 4 * q + 2], acc[cb + 4 * q + 3]);
              if (g.bias) {
                const int64_t gc = gc0 + 4 * q;                  // N % 4 == 0: a quad is all in or all out
                if (gc < g.N) {
                  o.x += g.bias[gc];
                  o.y += g.bias[gc + 1];
                  o.z += g.bias[gc + 2];
                  o.w += g.bias[gc + 3];
                }
              }
              *reinterpret_cast<float4*>(sb + sw128(row, q)) = o;
            }
            fence_proxy_async_smem();                            // staging writes -> async proxy
            bar_sync(1 + wg, kM);
            if (row == 0) {
              // C = [C1 | C2] split at a 32-column block; without C2 every block, including those past N that
              // the copy engine clips, goes to the first map (the second one is empty then)
              const bool second = g.C2 != nullptr && gc0 >= g.n1;
              const CUtensorMap* cm = second ? &cmap2 : &cmap;
              const int x = (int)(second ? gc0 - g.n1 : gc0);
              if (g.beta) tma_add_2d(cm, x, (int)row0, sb);
              else tma_store_2d(cm, x, (int)row0, sb);
              bulk_commit();
            }
          }
        } else {
#pragma unroll
        for (int cb = 0; cb < HALF; cb += 32) {
          const int w = HALF - cb < 32 ? HALF - cb : 32;        // 16 or 32
          bar_sync(1 + wg, kM);                                  // staging free
#pragma unroll
          for (int q = 0; q < 32; q += 4)
            if (q < w)
              *reinterpret_cast<float4*>(stg + row * kStgRow + q) =
                  make_float4(acc[cb + q], acc[cb + q + 1], acc[cb + q + 2], acc[cb + q + 3]);
          bar_sync(1 + wg, kM);
          const int cq = w / 4;                                  // float4 chunks per row
          for (int idx = row; idx < kM * cq; idx += kM) {
            const int r = idx / cq, c = idx - r * cq;
            const int64_t grow = row0 + r, gc = gcb + cb + 4 * c;
            if (grow < g.M && gc < g.N) {
              float4 o = *reinterpret_cast<const float4*>(stg + r * kStgRow + 4 * c);
              if (g.bias) {
                o.x += g.bias[gc];
                o.y += g.bias[gc + 1];
                o.z += g.bias[gc + 2];
                o.w += g.bias[gc + 3];
              }
              float* out = (g.C2 == nullptr || gc < g.n1) ? g.C + grow * g.ldc + gc : g.C2 + grow * g.ldc2 + (gc - g.n1);
              if (g.beta) {
                const float4 p = *reinterpret_cast<const float4*>(out);
                o.x += p.x;
                o.y += p.y;
                o.z += p.z;
                o.w += p.w;
              }
              *reinterpret_cast<float4*>(out) = o;
            }
          }
        }
        }
#pragma unroll
        for (int c = 0; c < HALF; c++) acc[c] = 0.f;
      }
      dc.next(g.k_chunks, g.n_tiles, gridDim.x);
    };

    bool ok = true;
    for (int64_t j = 0; j < total && ok; j++) {
      const int sa = (int)(j % SA), b = (int)(j % kNB);
      const int64_t t = j - kLag;                               // chunk drained in this iteration
      // draining chunk j - kLag also proves lo plane b free: MMA(j - kNB) completed before MMA(j - kLag)
      if (t >= 0 && !(ok = drain_start(t))) break;
      if (!(ok = mbar_wait(&fullA[sa], (uint32_t)((j / SA) & 1), ab))) break;   // A tile landed
      const unsigned char* at = aring + (uint32_t)sa * kPlane;
      unsigned char* lo = lo_planes + (uint32_t)b * kPlane;
      // lo plane: x - trunc(x) rounded to tf32; thread owns one row, 4 of the 8 16-byte quads
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t off = sw128(row, wg * 4 + i);
        const float4 v = *reinterpret_cast<const float4*>(at + off);
        *reinterpret_cast<float4*>(lo + off) =
            make_float4(to_tf32(v.x - tf32_trunc(v.x)), to_tf32(v.y - tf32_trunc(v.y)),
                        to_tf32(v.z - tf32_trunc(v.z)), to_tf32(v.w - tf32_trunc(v.w)));
      }
      if (t >= 0) drain_finish();
      fence_proxy_async_smem();                                // lo writes -> async proxy, TMEM loads done
      mbar_arrive(&split_bar[b]);
    }
    if (ok && !*ab)
      for (int64_t t = total - kLag > 0 ? total - kLag : 0; t < total; t++) {
        if (!drain_start(t)) break;
        drain_finish();
      }
    if (kTmaOut && row == 0) bulk_wait_all();                  // tile stores performed before the CTA exits
  }
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
  // N tile: 32 or 64 for narrow maps, else 128 (the most that four TMEM partials and the W ring hold).  An MMA costs
  // the same for any N up to 128, so a wider tile never costs tensor time, and the 64- and 128-column tiles store
  // by TMA (columns past N are clipped by the copy engine)
  const int64_t n32 = (N + 31) / 32;
  return n32 <= 2 ? (int)n32 * 32 : 128;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <int H16>
int launch_gemm(const CUtensorMap& amap, const CUtensorMap& amap2, const CUtensorMap& cmap, const CUtensorMap& cmap2,
                const GemmArgs& g, void* stream) {
  constexpr int Nt = 32 * H16;
  constexpr int SA = Ring<H16>::SA, SW = Ring<H16>::SW;
  const size_t smem =
      (SA + kNB) * kPlane + SW * (2u * Nt * kKc * 4) + 2 * kStg + (2 * SA + 2 * SW + 2 * kNB) * 8 + 16 + 1024;
  FACEK_CHECK_ARG((int)smem <= max_smem_optin(), "facek_gemm_tc: %zu B of shared memory needed", smem);
  cudaFuncSetAttribute(gemm_tc_k<H16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t units = ((g.M + kM - 1) / kM) * g.n_tiles;
  const int grid = (int)std::min<int64_t>(units, sm_count());
  gemm_tc_k<H16><<<grid, kThr, smem, as_stream(stream)>>>(amap, amap2, cmap, cmap2, g);
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

namespace {

// A 2D fp32 tensor map with 128-byte swizzle: rows x cols (row stride ld floats), box 32 columns x 128 rows
int encode_2d(EncodeTiledFn enc, CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
              CUtensorMapL2promotion promo, const char* what) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kKc, (cuuint32_t)kM};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FACEK_CHECK_ARG(cr == CUDA_SUCCESS, "facek_gemm_tc: %s tensor map encoding failed (%d)", what, (int)cr);
  return FACEK_OK;
}

bool operand_ok(const float* p, int64_t cols, int64_t ld) {
  return p && cols > 0 && cols % 4 == 0 && ld % 4 == 0 && ld >= cols && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// [C1 | C2] (=|+)= [A1 | A2] . W (+ bias): A1 holds K columns 0 .. K1-1 and A2 the rest (A2 null: K1 = K), C1 the
// output columns 0 .. N1-1 and C2 the rest (C2 null: N1 = N)
int gemm_run(const float* A1, int64_t lda1, int64_t K1, const float* A2, int64_t lda2, int64_t M, int64_t K,
             const float* image, int64_t N, const float* bias, float* C1, int64_t ldc1, int64_t N1, float* C2,
             int64_t ldc2, int beta, void* stream) {
  FACEK_CHECK_ARG(M >= 0 && K > 0 && N > 0, "facek_gemm_tc: bad sizes M=%lld K=%lld N=%lld", (long long)M,
                  (long long)K, (long long)N);
  if (M == 0) return FACEK_OK;
  FACEK_CHECK_ARG(image && (reinterpret_cast<uintptr_t>(image) & 15) == 0,
                  "facek_gemm_tc: image null or not 16-byte aligned");
  FACEK_CHECK_ARG(operand_ok(A1, K1, lda1),
                  "facek_gemm_tc: A needs K %% 4 == 0, lda %% 4 == 0, lda >= K and 16-byte alignment");
  FACEK_CHECK_ARG(operand_ok(C1, N1, ldc1),
                  "facek_gemm_tc: C needs N %% 4 == 0, ldc %% 4 == 0, ldc >= N and 16-byte alignment");
  if (A2) {
    FACEK_CHECK_ARG(K1 % kKc == 0 && K1 < K && operand_ok(A2, K - K1, lda2),
                    "facek_gemm_tc_split: A1 needs K1 %% 32 == 0, K1 < K; A2 as A (K - K1 columns)");
  } else {
    FACEK_CHECK_ARG(K1 == K, "facek_gemm_tc_split: without A2, K1 must equal K");
  }
  if (C2) {
    FACEK_CHECK_ARG(N1 % 32 == 0 && N1 < N && operand_ok(C2, N - N1, ldc2),
                    "facek_gemm_tc_split: C1 needs N1 %% 32 == 0, N1 < N; C2 as C (N - N1 columns)");
  } else {
    FACEK_CHECK_ARG(N1 == N, "facek_gemm_tc_split: without C2, N1 must equal N");
  }
  FACEK_CHECK_ARG(M < (int64_t)1 << 31 && K < (int64_t)1 << 31, "facek_gemm_tc: M, K must be < 2^31");
  EncodeTiledFn enc = encode_fn();
  FACEK_CHECK_ARG(enc != nullptr, "facek_gemm_tc: cuTensorMapEncodeTiled unavailable");
  CUtensorMap amap, amap2;
  std::memset(&amap2, 0, sizeof(amap2));
  int st = encode_2d(enc, &amap, A1, M, K1, lda1, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "input");
  if (st != FACEK_OK) return st;
  if (A2 && (st = encode_2d(enc, &amap2, A2, M, K - K1, lda2, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "second input")) !=
                FACEK_OK)
    return st;
  GemmArgs g{};
  g.M = M;
  g.K = K;
  g.img = image;
  g.N = N;
  g.Nt = pick_nt(N);
  g.n_tiles = (int)((N + g.Nt - 1) / g.Nt);
  g.k_chunks = (int)((K + kKc - 1) / kKc);
  g.k1_chunks = A2 ? (int)(K1 / kKc) : g.k_chunks;
  g.bias = bias;
  g.C = C1;
  g.ldc = ldc1;
  g.n1 = N1;
  g.C2 = C2;
  g.ldc2 = ldc2;
  g.beta = beta ? 1 : 0;
  uint32_t cols = 32;
  while (cols < (uint32_t)(kNB * g.Nt)) cols <<= 1;             // kNB chunk partials
  g.tmem_cols = cols;
  // C as a TMA destination for the 64- and 128-column tiles (box 32 columns x 128 rows, 128-byte swizzle; TMA
  // clips the rows >= M and columns >= N of the last tiles); unused by the other widths
  CUtensorMap cmap, cmap2;
  std::memset(&cmap, 0, sizeof(cmap));
  std::memset(&cmap2, 0, sizeof(cmap2));
  if (g.Nt % 64 == 0) {
    if ((st = encode_2d(enc, &cmap, C1, M, N1, ldc1, CU_TENSOR_MAP_L2_PROMOTION_NONE, "output")) != FACEK_OK) return st;
    if (C2 && (st = encode_2d(enc, &cmap2, C2, M, N - N1, ldc2, CU_TENSOR_MAP_L2_PROMOTION_NONE, "second output")) !=
                  FACEK_OK)
      return st;
  }
  switch (g.Nt / 32) {
    case 1: return launch_gemm<1>(amap, amap2, cmap, cmap2, g, stream);
    case 2: return launch_gemm<2>(amap, amap2, cmap, cmap2, g, stream);
    case 3: return launch_gemm<3>(amap, amap2, cmap, cmap2, g, stream);
    default: return launch_gemm<4>(amap, amap2, cmap, cmap2, g, stream);
  }
}

}  // namespace

extern "C" int facek_gemm_tc(const float* A, int64_t M, int64_t K, int64_t lda, const float* image, int64_t N,
                             const float* bias, float* C, int64_t ldc, int32_t beta, void* stream) {
  return gemm_run(A, lda, K, nullptr, 0, M, K, image, N, bias, C, ldc, N, nullptr, 0, beta, stream);
}

extern "C" int facek_gemm_tc_split(const float* A1, int64_t lda1, int64_t K1, const float* A2, int64_t lda2,
                                   int64_t M, int64_t K, const float* image, int64_t N, const float* bias, float* C1,
                                   int64_t ldc1, int64_t N1, float* C2, int64_t ldc2, int32_t beta, void* stream) {
  return gemm_run(A1, lda1, K1, A2, lda2, M, K, image, N, bias, C1, ldc1, N1, C2, ldc2, beta, stream);
}
