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
// Atoms with more than 64 edges accumulate over 64-edge blocks; atoms without edges get zero rows.  The work
// layout and warp roles are described at the kernel.
//
// Status: exact to fp32 level (tests hold it to 1e-5 of float64) but not yet faster than the CUDA-core kernel on
// the cfg5 alloy (43.4 vs 32.9 ms per launch): the eight builder warps both build operands and store finished
// tiles, so the stores stall the build.  facek_density_xm_fwd keeps the CUDA-core kernel; this one is reachable
// as facek_density_tc_xm_fwd.
#include "common.cuh"
#include "tc.cuh"

namespace facek {
namespace {

using namespace tc;

constexpr int kNX = 20, kB = 16, kK = 32, kBK = kB * kK;
constexpr int kEB = 64;                              // edges per K block
constexpr uint32_t kGroup = kEB * 128;               // one 32-wide MN group x 64 edge rows (8 KB)
constexpr uint32_t kVPlane = 4 * kGroup;             // a 128-row M tile's V (hi or lo) plane, 32 KB
constexpr uint32_t kMsgPlane = kEB * 128;            // msg block (hi or lo), 8 KB
constexpr int kStgRow = 36;                          // epilogue staging row stride (floats)

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
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mbar)) : "memory");
}

// Pipelined version.  Work is a sequence of chunks c = (atom, tile T, 64-edge block kb), 3 x nkb per atom.
// Warps 0-7 (builders): wait for ring stage c % 2 to be free, write the chunk's V (hi, lo) and msg (hi, lo) planes,
// arrive on full[c % 2] (256 arrivals).  Warp 8 (MMA issuer): wait full, issue up to 8 K-steps x 3 terms into
// TMEM accumulator (tile index) % 4, commit empty[stage] and, on a tile's last block, done[acc].  The builders
// store tile t two tiles after issuing it (wait done, TMEM -> padded staging -> coalesced 2 KB x-planes), so the
// MMAs of tiles t+1, t+2 overlap its store.  Every wait is bounded; parity waits are never two phases behind.
constexpr int kPThreads = 288;                       // 8 builder warps + MMA warp
constexpr int kAcc = 4;                              // TMEM accumulators in rotation (32 columns each)
constexpr int kLagT = 2;                             // tiles between a tile's last chunk and its store
constexpr uint32_t kStage = 2 * kVPlane + 2 * kMsgPlane;   // 80 KB
constexpr uint32_t kPSmem = 2 * kStage + 2 * 64 * kStgRow * 4 + 128 + 1024;

struct ChunkCursor {                                 // (atom, tile, block) sequence of one CTA
  int64_t i, e0;
  int deg, T, kb, nkb;
  __device__ bool load(int64_t atom, const int32_t* row_ptr, int64_t N) {
    i = atom;
    if (i >= N) return false;
    e0 = row_ptr[i];
    deg = row_ptr[i + 1] - (int)e0;
    T = 0;
    kb = 0;
    nkb = deg > 0 ? (deg + kEB - 1) / kEB : 0;
    return true;
  }
  // next chunk; atoms without edges are skipped (their rows are zeroed separately)
  __device__ bool next(const int32_t* row_ptr, int64_t N, int64_t stride) {
    if (nkb > 0 && ++kb < nkb) return true;
    kb = 0;
    if (nkb > 0 && ++T < 3) return true;
    do {
      if (!load(i + stride, row_ptr, N)) return false;
    } while (nkb == 0);
    return true;
  }
  __device__ bool first(int64_t atom, const int32_t* row_ptr, int64_t N, int64_t stride) {
    if (!load(atom, row_ptr, N)) return false;
    while (nkb == 0)
      if (!load(i + stride, row_ptr, N)) return false;
    return true;
  }
};

__global__ void __launch_bounds__(kPThreads, 1)
    dens_fwd_tc_k(const float* __restrict__ phi, const float* __restrict__ msg, const float* __restrict__ Y,
                  float* __restrict__ D, int64_t N, int64_t E, const int32_t* __restrict__ row_ptr) {
  extern __shared__ unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  float* stg = reinterpret_cast<float*>(sm + 2 * kStage);     // epilogue staging: 128 rows x kStgRow floats
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + 2 * kStage + 2 * 64 * kStgRow * 4);
  uint64_t* empty = full + 2;
  uint64_t* done = empty + 2;                                  // [kAcc]
  uint32_t* slot = reinterpret_cast<uint32_t*>(done + kAcc);
  int* abort_ = reinterpret_cast<int*>(slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t plane = N * (int64_t)kBK;

  if (tid == 0) {
    *abort_ = 0;
    for (int s = 0; s < 2; s++) {
      mbar_init(&full[s], 256);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; a++) mbar_init(&done[a], 1);
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
  volatile int* ab = abort_;

  if (warp == 8) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_mn(128, kK);
      ChunkCursor cc;
      bool more = cc.first(blockIdx.x, row_ptr, N, gridDim.x);
      int64_t tile = 0;                                        // tiles issued so far
      for (int64_t c = 0; more; c++) {
        const int s = (int)(c & 1);
        if (!mbar_wait(&full[s], (uint32_t)((c >> 1) & 1), ab)) break;
        fence_after_sync();
        unsigned char* st = sm + s * kStage;
        const uint32_t ah = smem_u32(st), al = ah + kVPlane, bh = al + kVPlane, bl = bh + kMsgPlane;
        const int acc = (int)(tile % kAcc);
        const uint32_t dcol = tbase + acc * kK;
        const int nb = min(kEB, cc.deg - cc.kb * kEB);
        const int nks = (nb + 7) / 8;
        for (int k = 0; k < nks; k++) {
          const uint64_t dah = desc_mn_sw32b(ah + k * 1024, kGroup, 512);
          const uint64_t dal = desc_mn_sw32b(al + k * 1024, kGroup, 512);
          const uint64_t dbh = desc_mn_sw32b(bh + k * 1024, kMsgPlane, 512);
          const uint64_t dbl = desc_mn_sw32b(bl + k * 1024, kMsgPlane, 512);
          mma_tf32(dcol, dal, dbh, idesc, (cc.kb > 0 || k > 0) ? 1u : 0u);
          mma_tf32(dcol, dah, dbl, idesc, 1u);
          mma_tf32(dcol, dah, dbh, idesc, 1u);
        }
        commit(&empty[s]);
        if (cc.kb == cc.nkb - 1) {
          commit(&done[acc]);
          tile++;
        }
        more = cc.next(row_ptr, N, gridDim.x);
      }
    }
  } else {
    // ------------------------------------------------------------------ builders (warps 0-7)
    const int eb = tid & (kEB - 1), quarter = tid >> 6;        // edge row, V group slot of the tile
    const int ehalf = warp >> 2;                               // epilogue: columns [16 ehalf, +16)
    const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16) + ehalf * 16;

    // store tile t (atom ti, tile index Tt) from accumulator t % kAcc; all 256 builders take part
    auto store_tile = [&](int64_t t, int64_t ti, int Tt) {
      const int acc = (int)(t % kAcc);
      mbar_wait(&done[acc], (uint32_t)((t / kAcc) & 1), ab);
      fence_after_sync();
      float v[16];
      tmem_ld16(tl + acc * kK, v);
      tmem_wait_ld();
      fence_before_sync();
      // staging: row m (= TMEM lane, 0..127) x 32 k, row stride kStgRow floats, in the 2 x 64 x kStgRow buffer
      const int m = tid & 127;
      float* srow = stg + m * kStgRow + ehalf * 16;
#pragma unroll
      for (int q = 0; q < 16; q += 4) *reinterpret_cast<float4*>(srow + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      bar_sync(1, 256);
      const int nx = Tt < 2 ? 8 : 4;
      for (int q = tid; q < nx * kBK / 4; q += 256) {
        const int xl = q / (kBK / 4), c = q % (kBK / 4);
        const int mm = xl * 16 + c / 8, kq = (c % 8) * 4;
        const float4 o = *reinterpret_cast<const float4*>(stg + mm * kStgRow + kq);
        reinterpret_cast<float4*>(D + (8 * Tt + xl) * plane + ti * kBK)[c] = o;
      }
      bar_sync(1, 256);                                        // staging free again
    };

    // pending stores: tiles issued but not stored yet (at most kLagT + 1)
    int64_t pend_atom[kLagT + 1];
    int pend_T[kLagT + 1];
    int64_t tiles_built = 0, tiles_stored = 0;

    // operands of one chunk, loaded one chunk ahead (register prefetch) so global latency overlaps the build
    struct Ops {
      float p[kB];
      float y0, y1;
      float4 mv[2];
    };
    auto load_ops = [&](const ChunkCursor& k, Ops& o) {
      const int nb = min(kEB, k.deg - k.kb * kEB);
      const int64_t eblk = k.e0 + k.kb * kEB;
      const bool live = eb < nb;
      const int64_t e = eblk + eb;
      const int g = 4 * k.T + quarter;
#pragma unroll
      for (int b = 0; b < kB; b += 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live) v = __ldg(reinterpret_cast<const float4*>(phi + e * kB + b));
        o.p[b] = v.x;
        o.p[b + 1] = v.y;
        o.p[b + 2] = v.z;
        o.p[b + 3] = v.w;
      }
      o.y0 = (live && g < 10) ? __ldg(Y + e * kNX + 2 * g) : 0.f;
      o.y1 = (live && g < 10) ? __ldg(Y + e * kNX + 2 * g + 1) : 0.f;
#pragma unroll
      for (int h = 0; h < 2; h++) {                           // msg: 64 rows x 8 quads, 2 per thread
        const int q = tid + 256 * h, r = q >> 3, cq = q & 7;
        o.mv[h] = r < nb ? __ldg(reinterpret_cast<const float4*>(msg + (eblk + r) * kK) + cq)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };

    ChunkCursor cc;
    bool more = cc.first(blockIdx.x, row_ptr, N, gridDim.x);
    int64_t last_atom = (int64_t)blockIdx.x - (int64_t)gridDim.x;
    Ops cur;
    if (more) load_ops(cc, cur);
    for (int64_t c = 0; more; c++) {
      // zero rows for atoms without edges between the previous chunk's atom and this one
      for (int64_t z = last_atom + gridDim.x; z < cc.i; z += gridDim.x)
        for (int q = tid; q < kNX * kBK / 4; q += 256) {
          const int x = q / (kBK / 4), cq = q % (kBK / 4);
          reinterpret_cast<float4*>(D + x * plane + z * kBK)[cq] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      last_atom = cc.i;
      const int s = (int)(c & 1);
      const int g = 4 * cc.T + quarter;                        // this thread's (x, b) group
      // MMAs of chunk c-2 done.  No early exit on an abort: the bounded waits then return at once, and every
      // builder keeps reaching the same named barriers in store_tile
      if (c >= 2) mbar_wait(&empty[s], (uint32_t)(((c >> 1) - 1) & 1), ab);
      unsigned char* st = sm + s * kStage;
      unsigned char* vhi = st;
      unsigned char* vlo = st + kVPlane;
      unsigned char* mhi = vlo + kVPlane;
      unsigned char* mlo = mhi + kMsgPlane;
      if (g < 10) {
        unsigned char* gh = vhi + quarter * kGroup;
        unsigned char* gl = vlo + quarter * kGroup;
#pragma unroll
        for (int q = 0; q < 8; q++) {
          const float y = q < 4 ? cur.y0 : cur.y1;
          const int b = 4 * (q & 3);
          const float4 v = make_float4(y * cur.p[b], y * cur.p[b + 1], y * cur.p[b + 2], y * cur.p[b + 3]);
          *reinterpret_cast<float4*>(gh + sw32b(eb, q)) = split_hi4(v);
          *reinterpret_cast<float4*>(gl + sw32b(eb, q)) = split_lo4(v);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int q = tid + 256 * h, r = q >> 3, cq = q & 7;
        *reinterpret_cast<float4*>(mhi + sw32b(r, cq)) = split_hi4(cur.mv[h]);
        *reinterpret_cast<float4*>(mlo + sw32b(r, cq)) = split_lo4(cur.mv[h]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[s]);
      const bool tile_end = cc.kb == cc.nkb - 1;
      const int64_t ci = cc.i;
      const int cT = cc.T;
      more = cc.next(row_ptr, N, gridDim.x);
      if (more) load_ops(cc, cur);                             // next chunk's loads overlap the store below
      if (tile_end) {                                          // last block of a tile: queue its store
        pend_atom[tiles_built % (kLagT + 1)] = ci;
        pend_T[tiles_built % (kLagT + 1)] = cT;
        tiles_built++;
        if (tiles_built - tiles_stored > kLagT) {
          const int pi = (int)(tiles_stored % (kLagT + 1));
          store_tile(tiles_stored, pend_atom[pi], pend_T[pi]);
          tiles_stored++;
        }
      }
    }
    while (tiles_stored < tiles_built) {
      const int pi = (int)(tiles_stored % (kLagT + 1));
      store_tile(tiles_stored, pend_atom[pi], pend_T[pi]);
      tiles_stored++;
    }
    // zero rows of trailing atoms without edges
    for (int64_t z = last_atom + gridDim.x; z < N; z += gridDim.x)
      for (int q = tid; q < kNX * kBK / 4; q += 256) {
        const int x = q / (kBK / 4), cq = q % (kBK / 4);
        reinterpret_cast<float4*>(D + x * plane + z * kBK)[cq] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
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
  FACEK_CHECK_ARG((int)kPSmem <= max_smem_optin(), "facek_density_tc_xm_fwd: %u B of shared memory needed", kPSmem);
  cudaFuncSetAttribute(dens_fwd_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
  dens_fwd_tc_k<<<grid_for(N, 1), kPThreads, kPSmem, as_stream(stream)>>>(phi, msg, Y, D, N, 0, row_ptr);
  return launch_status("facek_density_tc_xm_fwd");
}

// ===================================================================================================================
// Density adjoint on the tensor cores (fp32, B = 16, K = 32, CSR rows, component-major G planes).  Per atom i and a
// chunk of up to 128 of its edges (the MMA's M), two small GEMMs against the atom's G (20 x 16 x 32):
//   T[e, (x, b)] = sum_k msg[e, k] G[x, b, k]        N = 320, K = 32     (B operand: G rows (x, b), K-major)
//   U[e, (x, k)] = sum_b phi[e, b] G[x, b, k]        N = 640, K = 16     (B operand: G transposed, rows (x, k))
// and a per-edge epilogue on the CUDA cores (one thread per TMEM lane = edge row):
//   dY[e, x] = sum_b phi[e, b] T[e, (x, b)],  dphi[e, b] = sum_x Y[e, x] T[e, (x, b)],
//   dmsg[e, k] = sum_x Y[e, x] U[e, (x, k)]
// -- 1.3 k FMAs per edge instead of the 20 k of the lane-per-edge contraction.  The message part of dY is added
// afterwards by the message kernel (edge_msg_dy).
// fp32 accuracy by the 3-term tf32 split of both operands (tc.cuh); an accumulator sums at most 12 MMAs.
// Status: parity-green, opt-in (facek_density_msg_tc_xm_bwd); slower than the lane-per-edge kernel on the cfg5 alloy
// (105-111 vs 65-70 ms per launch).  Cycles per atom measured with clock64 on the scale-24 alloy: operand staging
// 12.3 k (59%: G's 40 KB written as hi and lo in both orientations by one CTA per SM, nothing overlapping it), MMA
// phase 1 2.7 k, epilogue 1 2.0 k, MMA phase 2 1.8 k, epilogue 2 1.5 k -- the 48 MMAs cost ~90 cycles each; hiding
// the staging needs a second 160 KB G buffer, which does not fit.
// Operands: K-major, no swizzle (kmajor_off).  Tensor memory: 512 columns; phase 1 holds T (columns 0..319) and U for
// x < 5 (320..479), phase 2 U for x >= 5 (0..479).  One CTA per SM (208 KB of shared memory): warps 0-3 stage the
// operands and run the epilogue, thread 128 issues the MMAs.  Every wait is bounded.
namespace {
constexpr int kAX = 20, kAB = 16, kAK = 32;
constexpr int kARows = 128;                                  // edges per chunk (MMA M)
constexpr int kANT = kAX * kAB;                              // 320 T columns
constexpr int kANU = kAX * kAK;                              // 640 U columns
constexpr uint32_t kAPlaneB = kANT * kAK * 4;                // 40 KB, one (hi or lo) plane of either B operand
constexpr uint32_t kAPlaneM = kARows * kAK * 4;              // 16 KB, msg plane
constexpr uint32_t kAPlaneP = kARows * kAB * 4;              // 8 KB, phi plane
constexpr uint32_t oBTh = 0, oBTl = oBTh + kAPlaneB, oBUh = oBTl + kAPlaneB, oBUl = oBUh + kAPlaneB;
constexpr uint32_t oAMh = oBUl + kAPlaneB, oAMl = oAMh + kAPlaneM, oAPh = oAMl + kAPlaneM, oAPl = oAPh + kAPlaneP;
constexpr uint32_t oABar = oAPl + kAPlaneP;
constexpr uint32_t kASmem = oABar + 64;
constexpr int kAThreads = 160;
constexpr int kAN = 160;                                     // N of one MMA (320 = 2 x 160, 640 = 4 x 160)
static_assert(kAX * 128 % (kAThreads * 8) == 0, "G staging assumes an even split into batches of 8 per thread");

struct GPlanes {                                             // component-major G: rank planes, x stride, atom stride
  const float* base[4];
  int64_t sX, sN;
  __device__ __forceinline__ const float* at(int64_t i, int x) const {
    const float* b = x < 1 ? base[0] : (x < 4 ? base[1] : (x < 10 ? base[2] : base[3]));
    const int o = x < 1 ? 0 : (x < 4 ? 1 : (x < 10 ? 4 : 10));
    return b + (int64_t)(x - o) * sX + i * sN;
  }
};

// G of atom i -> both B operands (hi, lo): BT rows (x, b) x K = k, BU rows (x, k) x K = b
__device__ __forceinline__ void stage_g(unsigned char* sm, const GPlanes& G, int64_t i, int tid) {
  // all of this thread's 16 loads in flight first (kAX * 128 = 2560 float4 over 160 threads), then the stores
  constexpr int kPer = kAX * 128 / kAThreads, kBatch = 8;
#pragma unroll 1
  for (int r0 = 0; r0 < kPer; r0 += kBatch) {
  float4 buf[kBatch];
#pragma unroll
  for (int r = 0; r < kBatch; r++) {
    const int q = tid + (r0 + r) * kAThreads;
    buf[r] = __ldg(reinterpret_cast<const float4*>(G.at(i, q >> 7)) + (q & 127));
  }
#pragma unroll
  for (int r = 0; r < kBatch; r++) {
    const int q = tid + (r0 + r) * kAThreads;
    const int x = q >> 7, f = q & 127, b = f >> 3, k0 = (f & 7) * 4;
    const float4 v = buf[r];
    store_split4(sm + oBTh, sm + oBTl, kmajor_off(x * kAB + b, k0, kANT), v.x, v.y, v.z, v.w);
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float h = to_tf32(vv[j]);
      const uint32_t off = kmajor_off(x * kAK + k0 + j, b, kANU);
      *reinterpret_cast<float*>(sm + oBUh + off) = h;
      *reinterpret_cast<float*>(sm + oBUl + off) = to_tf32(vv[j] - h);
    }
  }
  }
}

// D[d_col .. +160) (+)= A . B[rows n0 .. n0+160)^T over K = 8 * nks, 3-term split; A planes of kARows rows
__device__ __forceinline__ void mma_split(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                          uint32_t b_rows, uint32_t n0, int nks) {
  const uint32_t idesc = idesc_tf32(kARows, kAN);
  for (int s = 0; s < nks; s++) {
    const uint64_t ah = desc_kmajor(a_hi + s * 2 * kARows * 16, kARows * 16, 128);
    const uint64_t al = desc_kmajor(a_lo + s * 2 * kARows * 16, kARows * 16, 128);
    const uint32_t boff = s * 2 * b_rows * 16 + (n0 / 8) * 128;
    const uint64_t bh = desc_kmajor(b_hi + boff, b_rows * 16, 128);
    const uint64_t bl = desc_kmajor(b_lo + boff, b_rows * 16, 128);
    mma_tf32(d, al, bh, idesc, s > 0 ? 1u : 0u);
    mma_tf32(d, ah, bl, idesc, 1u);
    mma_tf32(d, ah, bh, idesc, 1u);
  }
}

// the 16 fp32 columns [c, c + 16) of this warp's 32 TMEM lanes, twice (two loads in flight)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
  tmem_wait_ld();
}

__global__ void __launch_bounds__(kAThreads, 1)
    dens_bwd_tc_k(const float* __restrict__ phi, const float* __restrict__ msg, const float* __restrict__ Y,
                  GPlanes G, float* __restrict__ dphi, float* __restrict__ dmsg, float* __restrict__ dY, int64_t N,
                  const int32_t* __restrict__ row_ptr) {
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + oABar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + oABar + 8);
  int* abort_ = reinterpret_cast<int*>(sm + oABar + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    *abort_ = 0;
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = *slot;
  const uint32_t s0 = smem_u32(sm);
  const uint32_t tl = tbase + ((uint32_t)((warp & 3) * 32) << 16);     // epilogue warps 0-3: lanes 32w .. 32w+31
  volatile int* ab = abort_;
  uint32_t parity = 0;
  bool stop = false;

  for (int64_t i = blockIdx.x; i < N && !stop; i += gridDim.x) {
    const int64_t e0 = row_ptr[i];
    const int deg = row_ptr[i + 1] - (int)e0;
    for (int c0 = 0; c0 < deg; c0 += kARows) {
      const int nrow = min(kARows, deg - c0);
      __syncthreads();                       // the previous chunk's MMAs are complete and its TMEM reads done
      fence_after_sync();
      if (*ab) {                             // uniform: the flag is written only before a barrier
        stop = true;
        break;
      }
      if (c0 == 0) stage_g(sm, G, i, tid);
      // A operands (padding rows zero) and this row's epilogue inputs
      float yv[kAX], pv[kAB];
      const bool valid = tid < nrow;
      const int64_t e = e0 + c0 + tid;
      if (tid < kARows) {
        const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kAK; k += 4) {
          const float4 v = valid ? __ldg(reinterpret_cast<const float4*>(msg + e * kAK + k)) : z4;
          store_split4(sm + oAMh, sm + oAMl, kmajor_off(tid, k, kARows), v.x, v.y, v.z, v.w);
        }
#pragma unroll
        for (int b = 0; b < kAB; b += 4) {
          const float4 v = valid ? __ldg(reinterpret_cast<const float4*>(phi + e * kAB + b)) : z4;
          pv[b] = v.x; pv[b + 1] = v.y; pv[b + 2] = v.z; pv[b + 3] = v.w;
          store_split4(sm + oAPh, sm + oAPl, kmajor_off(tid, b, kARows), v.x, v.y, v.z, v.w);
        }
#pragma unroll
        for (int x = 0; x < kAX; x += 4) {
          const float4 v = valid ? __ldg(reinterpret_cast<const float4*>(Y + e * kAX + x)) : z4;
          yv[x] = v.x; yv[x + 1] = v.y; yv[x + 2] = v.z; yv[x + 3] = v.w;
        }
      }
      fence_proxy_async_smem();
      fence_before_sync();
      __syncthreads();
      // ---- phase 1: T -> columns [0, 320), U (x < 5) -> [320, 480)
      if (tid == kARows) {
        fence_after_sync();
        mma_split(tbase, s0 + oAMh, s0 + oAMl, s0 + oBTh, s0 + oBTl, kANT, 0, kAK / 8);
        mma_split(tbase + kAN, s0 + oAMh, s0 + oAMl, s0 + oBTh, s0 + oBTl, kANT, kAN, kAK / 8);
        mma_split(tbase + 2 * kAN, s0 + oAPh, s0 + oAPl, s0 + oBUh, s0 + oBUl, kANU, 0, kAB / 8);
        commit(mbar);
      }
      float dm[kAK];
      if (warp < 4) {
        float dp[kAB], dyv[kAX];
        int ok = 1;
        if (lane == 0) ok = mbar_wait(mbar, parity, ab) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        fence_after_sync();
#pragma unroll
        for (int b = 0; b < kAB; b++) dp[b] = 0.f;
#pragma unroll
        for (int k = 0; k < kAK; k++) dm[k] = 0.f;
        if (ok) {
#pragma unroll
          for (int x = 0; x < kAX; x += 2) {              // T rows (x, b), two x per pair of loads
            float t[32];
            tmem_ld32(tl + x * kAB, t);
#pragma unroll
            for (int h = 0; h < 2; h++) {
              float s = 0.f;
#pragma unroll
              for (int b = 0; b < kAB; b++) {
                s += pv[b] * t[h * kAB + b];
                dp[b] += yv[x + h] * t[h * kAB + b];
              }
              dyv[x + h] = s;
            }
          }
          if (valid) {                                     // dphi, dY are complete after phase 1
#pragma unroll
            for (int b = 0; b < kAB; b += 4)
              *reinterpret_cast<float4*>(dphi + e * kAB + b) = make_float4(dp[b], dp[b + 1], dp[b + 2], dp[b + 3]);
#pragma unroll
            for (int x = 0; x < kAX; x += 4)
              *reinterpret_cast<float4*>(dY + e * kAX + x) = make_float4(dyv[x], dyv[x + 1], dyv[x + 2], dyv[x + 3]);
          }
#pragma unroll
          for (int x = 0; x < 5; x++) {                    // U rows (x, k), x < 5
            float u[32];
            tmem_ld32(tl + 2 * kAN + x * kAK, u);
#pragma unroll
            for (int k = 0; k < kAK; k++) dm[k] += yv[x] * u[k];
          }
        }
      }
      parity ^= 1u;
      fence_before_sync();
      __syncthreads();
      if (*ab) {
        stop = true;
        break;
      }
      // ---- phase 2: U (x >= 5) -> columns [0, 480)
      if (tid == kARows) {
        fence_after_sync();
        for (int q = 1; q < 4; q++)
          mma_split(tbase + (q - 1) * kAN, s0 + oAPh, s0 + oAPl, s0 + oBUh, s0 + oBUl, kANU, q * kAN, kAB / 8);
        commit(mbar);
      }
      if (warp < 4) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(mbar, parity, ab) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        fence_after_sync();
        if (ok) {
#pragma unroll
          for (int x = 5; x < kAX; x++) {
            float u[32];
            tmem_ld32(tl + (x - 5) * kAK, u);
#pragma unroll
            for (int k = 0; k < kAK; k++) dm[k] += yv[x] * u[k];
          }
          if (valid) {
#pragma unroll
            for (int k = 0; k < kAK; k += 4)
              *reinterpret_cast<float4*>(dmsg + e * kAK + k) = make_float4(dm[k], dm[k + 1], dm[k + 2], dm[k + 3]);
          }
        }
      }
      parity ^= 1u;
      fence_before_sync();
    }
  }
  __syncthreads();
  fence_after_sync();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

}  // namespace

int density_tc_xm_bwd(const float* phi, const float* msg, const float* Y, const float* const G[4], float* dphi,
                      float* dmsg, float* dY, int64_t N, const int32_t* row_ptr, void* stream) {
  if (N == 0) return FACEK_OK;
  FACEK_CHECK_ARG((int)kASmem <= max_smem_optin(), "facek_density_tc_xm_bwd: needs %u B of shared memory", kASmem);
  const uintptr_t al = reinterpret_cast<uintptr_t>(phi) | reinterpret_cast<uintptr_t>(msg) |
                       reinterpret_cast<uintptr_t>(Y) | reinterpret_cast<uintptr_t>(dphi) |
                       reinterpret_cast<uintptr_t>(dmsg) | reinterpret_cast<uintptr_t>(dY) |
                       reinterpret_cast<uintptr_t>(G[0]) | reinterpret_cast<uintptr_t>(G[1]) |
                       reinterpret_cast<uintptr_t>(G[2]) | reinterpret_cast<uintptr_t>(G[3]);
  FACEK_CHECK_ARG((al & 15) == 0, "facek_density_tc_xm_bwd: tensors must be 16-byte aligned");
  GPlanes P{{G[0], G[1], G[2], G[3]}, N * (int64_t)(kAB * kAK), (int64_t)(kAB * kAK)};
  cudaFuncSetAttribute(dens_bwd_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kASmem);
  dens_bwd_tc_k<<<grid_for(N, 1), kAThreads, kASmem, as_stream(stream)>>>(phi, msg, Y, P, dphi, dmsg, dY, N,
                                                                          row_ptr);
  return launch_status("facek_density_tc_xm_bwd");
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

extern "C" int facek_density_msg_tc_xm_bwd(const float* phi, const float* msg, const float* Y, const float* G0,
                                           const float* G1, const float* G2, const float* G3, const float* TJ,
                                           const float* TI, const int32_t* ei, const int32_t* ej, int32_t nc,
                                           float* dphi, float* dmsg, float* dY, int64_t N, int64_t E, int32_t B,
                                           int32_t K, const int32_t* row_ptr, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && E >= 0 && B == 16 && K == 32 && nc >= 1 && nc <= 10 && row_ptr && G0 && G1 && G2 && G3 &&
                      TJ && ei && ej && (E == 0 || (phi && msg && Y && dphi && dmsg && dY)),
                  "facek_density_msg_tc_xm_bwd: bad arguments (fp32, B = 16, K = 32 only)");
  if (N == 0) return FACEK_OK;
  const float* G[4] = {G0, G1, G2, G3};
  int st = density_tc_xm_bwd(phi, msg, Y, G, dphi, dmsg, dY, N, row_ptr, stream);
  if (st) return st;
  return edge_msg_dy(FACEK_F32, ei, ej, TJ, TI, dmsg, nc, K, N, E, dY, stream);
}
