// Radial basis x radial MLP per edge on the tcgen05 tensor cores, with forward-mode dphi/dr
// (face-mlip face/model.py:460-470 FactorBlock radial path, :34-37 envelope, :23-31 Bessel basis).
//
//   x_n   = sqrt(2/rc) sin(f_n r)/r * env(r)                       n < nb, f_n = (n+1) pi / rc
//   a1    = silu(W1 x + b1 + pair[z_i, z_j])                        H = 64 hidden units
//   a2    = silu(W2 a1 + b2)
//   phi   = (W3 a2 + b3) * env(r),  dphi/dr by pushing d/dr through the same three layers
//
// One CTA = two groups of 8 warps; each group owns a 128-edge tile, two threads per edge (one TMEM lane, each
// thread half of the 64 hidden units), and runs
//   layer 1 on the CUDA cores -> W2 x [a1 | da1] on the tensor core -> silu epilogue -> W3 x [a2 | da2] on the
//   tensor core -> phi, dphi/dr epilogue,
// so one group's CUDA-core work overlaps the other's MMAs (16 warps per SM hide the CUDA-core latencies).  The
// pair embedding is kept transposed, [hidden][pair] with b1 folded in, so lanes with different element pairs read
// different banks.  The MMAs run kind::tf32 with the 3-term split,
// which keeps fp32 accuracy (tc.cuh). Weights are split once per CTA into shared memory, as one operand of 2R rows
// per layer (lo parts in rows 0 .. R-1, hi parts in rows R .. 2R-1); an MMA costs about the same for any N up to
// 128, so each K step issues two instead of three:
//   [D_s | D_b] (=|+)= A_hi . [W_lo | W_hi]  (N = 2R),   D_s += A_lo . W_hi  (N = R),   result D_s + D_b.
// The CTA is persistent over tiles. Tensor memory: 256 fp32 columns per group (value and tangent accumulators
// of W2, 2 x 64 each; later reused for W3).
#include "common.cuh"
#include "radial.cuh"
#include "tc.cuh"

namespace facek {
namespace {

using namespace tc;

constexpr int kH = 64;                               // hidden width
constexpr int kRows = 128;                           // edges per warpgroup tile = MMA M
constexpr int kThreads = 512;                        // two groups of 8 warps (2 threads per edge row)
constexpr uint32_t kPlane = kRows * kH * 4;          // one fp32 operand plane (32 KB)
constexpr uint32_t kTmemCols = 512;

struct Layout {
  uint32_t a, w2, w3, w1, b1, b2, b3, pair, mbar, slot, abort_, total;
};

__host__ __device__ inline Layout layout_for(int NB, int BO, int n_el) {
  Layout L;
  L.a = 0;                                            // [wg][hi|lo] operand planes
  L.w2 = L.a + 4 * kPlane;                            // W2 [lo | hi] (2 x 64 rows x 64)
  L.w3 = L.w2 + 2 * kH * kH * 4;                      // W3 [lo | hi] (2 x BO rows x 64)
  L.w1 = L.w3 + 2 * BO * kH * 4;                      // W1 (64 x NB), zero-padded basis
  L.b1 = L.w1 + kH * NB * 4;
  L.b2 = L.b1 + kH * 4;
  L.b3 = L.b2 + kH * 4;
  L.pair = L.b3 + BO * 4;                             // b1 + pair embedding, transposed: [64][n_el^2]
  L.mbar = L.pair + n_el * n_el * kH * 4;             // 2 x 8 B
  L.slot = L.mbar + 16;
  L.abort_ = L.slot + 16;                             // 2 x 4 B
  L.total = L.abort_ + 16;
  return L;
}

template <int NB, int BO>
__global__ void __launch_bounds__(kThreads, 1)
    radial_tc_k(const float* __restrict__ vec, const int32_t* __restrict__ ei, const int32_t* __restrict__ ej,
                const int32_t* __restrict__ zidx, int n_el, float rc, int nb, const float* __restrict__ w1,
                const float* __restrict__ b1, const float* __restrict__ pair, const float* __restrict__ w2,
                const float* __restrict__ b2, const float* __restrict__ w3, const float* __restrict__ b3,
                float* __restrict__ phi, float* __restrict__ dphidr, int64_t E) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const Layout L = layout_for(NB, BO, n_el);
  unsigned char* w2s = sm + L.w2;
  unsigned char* w3s = sm + L.w3;
  float* w1s = reinterpret_cast<float*>(sm + L.w1);
  float* b1s = reinterpret_cast<float*>(sm + L.b1);
  float* b2s = reinterpret_cast<float*>(sm + L.b2);
  float* b3s = reinterpret_cast<float*>(sm + L.b3);
  float* pairs = reinterpret_cast<float*>(sm + L.pair);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + L.mbar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.slot);
  int* abort_ = reinterpret_cast<int*>(sm + L.abort_);

  const int tid = threadIdx.x, warp = tid >> 5, wg = tid >> 8, wt = tid & 255, row = wt & (kRows - 1);
  const int half = wt >> 7;                          // hidden units [32 half, 32 half + 32) of this thread's row
  const int np = n_el * n_el;

  // ---- weights -> shared memory (W2, W3 as [lo | hi] tf32 rows in the K-major operand layout)
  for (int q = tid; q < kH * kH; q += kThreads) {
    const float w = w2[q], hi = to_tf32(w);
    *reinterpret_cast<float*>(w2s + kmajor_off(q / kH, q % kH, 2 * kH)) = to_tf32(w - hi);
    *reinterpret_cast<float*>(w2s + kmajor_off(kH + q / kH, q % kH, 2 * kH)) = hi;
  }
  for (int q = tid; q < BO * kH; q += kThreads) {
    const float w = w3[q], hi = to_tf32(w);
    *reinterpret_cast<float*>(w3s + kmajor_off(q / kH, q % kH, 2 * BO)) = to_tf32(w - hi);
    *reinterpret_cast<float*>(w3s + kmajor_off(BO + q / kH, q % kH, 2 * BO)) = hi;
  }
  for (int q = tid; q < kH * NB; q += kThreads) {
    const int h = q / NB, n = q % NB;
    w1s[q] = n < nb ? w1[h * nb + n] : 0.f;
  }
  for (int q = tid; q < kH; q += kThreads) {
    b1s[q] = b1[q];
    b2s[q] = b2[q];
  }
  for (int q = tid; q < BO; q += kThreads) b3s[q] = b3[q];
  for (int q = tid; q < np * kH; q += kThreads) {
    const int pp = q / kH, h = q % kH;
    pairs[h * np + pp] = pair[q] + b1[h];
  }
  if (tid == 0) {
    abort_[0] = 0;
    abort_[1] = 0;
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = *slot;

  unsigned char* a_hi = sm + L.a + wg * 2 * kPlane;
  unsigned char* a_lo = a_hi + kPlane;
  const uint32_t a_hi_s = smem_u32(a_hi), a_lo_s = a_hi_s + kPlane;
  const uint32_t w2_s = smem_u32(w2s), w3_s = smem_u32(w3s);
  const uint32_t col0 = tbase + wg * 256;                                   // this warpgroup's columns
  const uint32_t tl = col0 + ((uint32_t)((warp & 3) * 32) << 16);          // + this warp's lane quarter
  volatile int* ab = &abort_[wg];
  uint32_t parity = 0;

  // one MMA round: operand writes -> async proxy, sync the warpgroup, one thread issues over K = 64 in 8 steps
  //   [D_s | D_b] (=|+)= A_hi . [W_lo | W_hi],  D_s += A_lo . W_hi
  // (D_s at dcol, D_b at dcol + R), commits, and everyone waits for completion
  auto round = [&](uint32_t dcol, uint32_t w_s, uint32_t R) {
    const uint32_t quad = 2 * R * 16;                                       // one 16-byte K quad of both halves
    const uint32_t idesc2 = idesc_tf32(kRows, 2 * R), idesc1 = idesc_tf32(kRows, R);
    fence_proxy_async_smem();
    fence_before_sync();
    bar_sync(1 + wg, 2 * kRows);
    if (wt == 0 && !*ab) {
      fence_after_sync();
#pragma unroll
      for (int s = 0; s < kH / 8; s++) {
        const uint64_t ah = desc_kmajor(a_hi_s + s * 2 * kRows * 16, kRows * 16, 128);
        const uint64_t al = desc_kmajor(a_lo_s + s * 2 * kRows * 16, kRows * 16, 128);
        const uint64_t bb = desc_kmajor(w_s + s * 2 * quad, quad, 128);             // [W_lo | W_hi], 2R rows
        const uint64_t bh = desc_kmajor(w_s + s * 2 * quad + R * 16, quad, 128);    // W_hi, R rows
        mma_tf32(dcol, ah, bb, idesc2, s > 0 ? 1u : 0u);
        mma_tf32(dcol, al, bh, idesc1, 1u);
      }
      commit(&mbar[wg]);
    }
    mbar_wait(&mbar[wg], parity, ab);
    parity ^= 1u;
    fence_after_sync();
  };

  const float cb = sqrtf(2.f / rc);
  const float pi = 3.14159265358979323846f;
  const float th = pi / rc;
  const int64_t ntiles = (E + kRows - 1) / kRows;
  const int64_t tstride = (int64_t)gridDim.x * 2;
  // the next tile's edge geometry and element pair, loaded one tile ahead (ei/ej at the start of the previous
  // tile, zidx after its layer 1), so the dependent ei -> zidx chain is off the critical path
  float nx = 0.f, ny = 0.f, nz = 0.f;
  int ni = 0, nj = 0;
  auto fetch_geom = [&](int64_t tt) {
    const int64_t ee = tt * kRows + row;
    if (tt < ntiles && ee < E) {
      nx = vec[ee * 3];
      ny = vec[ee * 3 + 1];
      nz = vec[ee * 3 + 2];
      ni = ei[ee];
      nj = ej[ee];
    }
  };
  auto fetch_elem = [&](int64_t tt) {
    const int64_t ee = tt * kRows + row;
    if (tt < ntiles && ee < E) {
      ni = zidx[ni];
      nj = zidx[nj];
    }
  };
  {
    const int64_t t0 = (int64_t)blockIdx.x * 2 + wg;
    fetch_geom(t0);
    fetch_elem(t0);
  }
  for (int64_t t = (int64_t)blockIdx.x * 2 + wg; t < ntiles; t += tstride) {
    bar_sync(1 + wg, 2 * kRows);
    if (*ab) break;                                  // uniform: nothing writes the flag between these points
    const int64_t e = t * kRows + row;
    const bool valid = e < E;
    float r = 0.5f * rc;
    int p = 0;
    if (valid) {
      r = sqrtf(nx * nx + ny * ny + nz * nz);
      p = ni * n_el + nj;
    }
    fetch_geom(t + tstride);
    float env, denv;
    envelope(r, rc, env, denv);
    // Bessel basis sqrt(2/rc) sin(f_n r)/r, f_n = (n+1) pi/rc, by the angle-addition recurrence
    //   sin((n+2) x) = sin((n+1) x) cos x + cos((n+1) x) sin x,  cos((n+2) x) = cos((n+1) x) cos x - sin((n+1) x) sin x
    // restarted from a direct sincos every 4 terms (fp32 error <= 3e-7 absolute, below the argument rounding of a
    // direct sin(f_n r) at n ~ 16)
    const float ir = 1.f / r, cbr = cb * ir;
    float rb[NB], drb[NB];
    {
      float s1, c1;
      sincosf(th * r, &s1, &c1);
      float sn = s1, cn = c1;
#pragma unroll
      for (int n = 0; n < NB; n++) {
        if (n > 0 && n % 4 == 0) sincosf(float(n + 1) * th * r, &sn, &cn);
        const float f = float(n + 1) * th;
        const float bes = sn * cbr;
        const float dbes = (f * cn - sn * ir) * cbr;
        rb[n] = n < nb ? bes * env : 0.f;
        drb[n] = n < nb ? dbes * env + bes * denv : 0.f;
        const float s2 = sn * c1 + cn * s1;
        cn = cn * c1 - sn * s1;
        sn = s2;
      }
    }
    // ---- layer 1 on the CUDA cores (this thread's 32 hidden units): a1 -> operand planes, da1 parked in this
    // lane's TMEM columns [128 + h) (free while round 1 writes [0, 128))
    const float* pcol = pairs + p;
    constexpr int kHh = kH / 2;
    const uint32_t park = tl + 128 + half * kHh;
#pragma unroll 1
    for (int hh = 0; hh < kHh; hh += 8) {
      const int h0 = half * kHh + hh;
      float a[8], da[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int h = h0 + j;
        float z = pcol[h * np], dz = 0.f;
#pragma unroll
        for (int n = 0; n < NB; n++) ffma2(z, dz, w1s[h * NB + n], w1s[h * NB + n], rb[n], drb[n]);
        const float sg = sigmoid_f(z);
        a[j] = z * sg;
        da[j] = sg * (1.f + z * (1.f - sg)) * dz;
      }
      store_split4(a_hi, a_lo, kmajor_off(row, h0, kRows), a[0], a[1], a[2], a[3]);
      store_split4(a_hi, a_lo, kmajor_off(row, h0 + 4, kRows), a[4], a[5], a[6], a[7]);
      tmem_st8(park + hh, da);
    }
    fetch_elem(t + tstride);
    tmem_wait_st();
    round(col0, w2_s, kH);                                                   // z2 -> columns [0, 128)
#pragma unroll
    for (int hh = 0; hh < kHh; hh += 8) {
      float v[8];
      tmem_ld8(park + hh, v);
      tmem_wait_ld();
      const int h0 = half * kHh + hh;
      store_split4(a_hi, a_lo, kmajor_off(row, h0, kRows), v[0], v[1], v[2], v[3]);
      store_split4(a_hi, a_lo, kmajor_off(row, h0 + 4, kRows), v[4], v[5], v[6], v[7]);
    }
    round(col0 + 128, w2_s, kH);                                             // dz2 -> columns [128, 256)

    // ---- silu epilogue of layer 2: a2 -> operand planes, da2 parked over the dz2 columns just read
    // (round 3 writes [0, 2 BO), round 4 [64, 64 + 2 BO): [128, 192) stays free until it is read back)
#pragma unroll
    for (int cc = 0; cc < kHh; cc += 8) {
      const int c0 = half * kHh + cc;
      float z[8], dz[8], ts[8], td[8];
      tmem_ld8(tl + c0, z);
      tmem_ld8(tl + 64 + c0, ts);
      tmem_ld8(tl + 128 + c0, dz);
      tmem_ld8(tl + 192 + c0, td);
      tmem_wait_ld();
      float a[8], da[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float zz = (z[j] + ts[j]) + b2s[c0 + j];
        const float sg = sigmoid_f(zz);
        a[j] = zz * sg;
        da[j] = sg * (1.f + zz * (1.f - sg)) * (dz[j] + td[j]);
      }
#pragma unroll
      for (int q = 0; q < 8; q += 4)
        store_split4(a_hi, a_lo, kmajor_off(row, c0 + q, kRows), a[q], a[q + 1], a[q + 2], a[q + 3]);
      tmem_st8(tl + 128 + c0, da);
    }
    tmem_wait_st();
    round(col0, w3_s, BO);                                                   // z3 -> columns [0, 2 BO)
#pragma unroll
    for (int hh = 0; hh < kHh; hh += 8) {
      float v[8];
      tmem_ld8(park + hh, v);
      tmem_wait_ld();
      const int h0 = half * kHh + hh;
      store_split4(a_hi, a_lo, kmajor_off(row, h0, kRows), v[0], v[1], v[2], v[3]);
      store_split4(a_hi, a_lo, kmajor_off(row, h0 + 4, kRows), v[4], v[5], v[6], v[7]);
    }
    round(col0 + 64, w3_s, BO);                                              // dz3 -> columns [64, 64 + 2 BO)

    // ---- output epilogue: 16-column groups split between the two halves (half 1 idle when BO = 16), read
    // 8 columns at a time
#pragma unroll
    for (int c0 = 16 * half; c0 < BO; c0 += 32) {
#pragma unroll
      for (int c8 = c0; c8 < c0 + 16; c8 += 8) {
        float z[8], zb[8], dz[8], dzb[8];
        tmem_ld8(tl + c8, z);
        tmem_ld8(tl + BO + c8, zb);
        tmem_ld8(tl + 64 + c8, dz);
        tmem_ld8(tl + 64 + BO + c8, dzb);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int q = 0; q < 8; q += 4) {
            float v[4], d[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              v[j] = (z[q + j] + zb[q + j]) + b3s[c8 + q + j];
              d[j] = (dz[q + j] + dzb[q + j]) * env + v[j] * denv;
              v[j] *= env;
            }
            *reinterpret_cast<float4*>(phi + e * BO + c8 + q) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4*>(dphidr + e * BO + c8 + q) = make_float4(d[0], d[1], d[2], d[3]);
          }
        }
      }
    }
    fence_before_sync();
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, kTmemCols);
  }
}

template <int NB, int BO>
int radial_tc_launch(const float* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, float rc,
                     int nb, const float* w1, const float* b1, const float* pair, const float* w2, const float* b2,
                     const float* w3, const float* b3, float* phi, float* dphidr, int64_t E, void* stream) {
  const Layout L = layout_for(NB, BO, n_el);
  FACEK_CHECK_ARG((int)L.total <= max_smem_optin(), "facek_radial_tc_fwd: %u B of shared memory needed", L.total);
  cudaFuncSetAttribute(radial_tc_k<NB, BO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
  const int64_t ntiles = (E + kRows - 1) / kRows;
  const int grid = (int)std::min<int64_t>((ntiles + 1) / 2, sm_count());
  radial_tc_k<NB, BO><<<grid, kThreads, L.total, as_stream(stream)>>>(vec, ei, ej, zidx, n_el, rc, nb, w1, b1, pair,
                                                                       w2, b2, w3, b3, phi, dphidr, E);
  return launch_status("facek_radial_tc_fwd");
}

}  // namespace

bool radial_tc_supported(int n_el, int nb, int H, int B) {
  if (H != kH || !(B == 16 || B == 32) || nb < 1 || nb > 16 || n_el < 1) return false;
  return (int)layout_for(nb <= 8 ? 8 : 16, B, n_el).total <= max_smem_optin();
}

int radial_tc_fwd(const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int n_el, double rc,
                  int nb, int H, int B, const void* w1, const void* b1, const void* pair, const void* w2,
                  const void* b2, const void* w3, const void* b3, void* phi, void* dphidr, int64_t E, void* stream) {
  FACEK_CHECK_ARG(radial_tc_supported(n_el, nb, H, B),
                  "facek_radial_tc_fwd: needs H = 64, B in {16, 32}, nb <= 16 (got H=%d B=%d nb=%d n_el=%d)", H, B,
                  nb, n_el);
  if (E == 0) return FACEK_OK;
  auto f = [&](auto launch) {
    return launch((const float*)vec, ei, ej, zidx, n_el, (float)rc, nb, (const float*)w1, (const float*)b1,
                  (const float*)pair, (const float*)w2, (const float*)b2, (const float*)w3, (const float*)b3,
                  (float*)phi, (float*)dphidr, E, stream);
  };
  if (nb <= 8) return B == 16 ? f(radial_tc_launch<8, 16>) : f(radial_tc_launch<8, 32>);
  return B == 16 ? f(radial_tc_launch<16, 16>) : f(radial_tc_launch<16, 32>);
}

}  // namespace facek

using namespace facek;

extern "C" int facek_radial_tc_fwd(const float* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx,
                                   int32_t n_el, double rc, int32_t nb, int32_t H, int32_t B, const float* w1,
                                   const float* b1, const float* pair, const float* w2, const float* b2,
                                   const float* w3, const float* b3, float* phi, float* dphidr, int64_t E,
                                   void* stream) {
  FACEK_CHECK_ARG(E >= 0 && n_el > 0 && rc > 0, "facek_radial_tc_fwd: bad sizes");
  FACEK_CHECK_ARG(E == 0 || (vec && ei && ej && zidx && w1 && b1 && pair && w2 && b2 && w3 && b3 && phi && dphidr),
                  "facek_radial_tc_fwd: null tensor");
  return radial_tc_fwd(vec, ei, ej, zidx, n_el, rc, nb, H, B, w1, b1, pair, w2, b2, w3, b3, phi, dphidr, E, stream);
}

extern "C" int facek_tc_status(int32_t* status, int32_t clear) {
  FACEK_CHECK_ARG(status != nullptr, "facek_tc_status: null output");
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_tc_status, sizeof(int)) != cudaSuccess) return launch_status("facek_tc_status");
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(tc::g_tc_status, &zero, sizeof(int)) != cudaSuccess)
      return launch_status("facek_tc_status");
  }
  const int g = gemm_tc_status(clear), d = density_tc_status(clear);
  if (g < 0 || d < 0) return launch_status("facek_tc_status");
  *status = v | g | d;
  return FACEK_OK;
}
