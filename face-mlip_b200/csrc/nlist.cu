// Neighbour lists for the FACE engine, replacing ase.neighborlist.neighbor_list("ijS", atoms, rc) as used by
// face-mlip (face/neighbors.py:7-37, face/datasets.py:44-97): every (i, j, S) with |pos[j]-pos[i]+S.cell| < rc,
// the zero-shift self pair excluded, periodic self images included; rows centre-sorted, and within a row in
// (j, S0, S1, S2) order.
//
// The inclusion test runs in float64 in a fixed operation order without fused multiply-adds (the same order
// as the CPU enumerator the tests compare against), so edge sets agree bit for bit:
//   sv = (S0*c0 + S1*c1) + S2*c2 ; d = (p_j - p_i) + sv ; |d| = sqrt((dx*dx + dy*dy) + dz*dz) ; |d| < rc
//
// Periodic path: atoms are binned by wrapped fractional coordinate into a grid of cells at least rc/ns wide
// along each lattice plane normal; each atom scans (2ns+1)^3 cells, cell images giving the shift S.  Cell
// contents are sorted by atom index, the per-row output is sorted by key, so the result is deterministic.
// Non-periodic batches: all pairs inside each structure (molecules of tens of atoms).
#include "common.cuh"

namespace facek {
namespace {

struct CellGrid {
  double cell[9];    // rows = lattice vectors
  double inv[9];     // inverse cell, frac = pos @ inv
  int nc[3];         // cells per axis
  int ns[3];         // cell scan half-width per axis
  int64_t ncells;
};

__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }

// exact-order distance test; returns the shift vector in sv
__device__ __forceinline__ bool within(const double* pi, const double* pj, const double* cell, int s0, int s1, int s2,
                                       double rc, double sv[3]) {
  double d2 = 0;
  double dd[3];
#pragma unroll
  for (int x = 0; x < 3; x++) {
    sv[x] = add(add(mul((double)s0, cell[x]), mul((double)s1, cell[3 + x])), mul((double)s2, cell[6 + x]));
    dd[x] = add(sub(pj[x], pi[x]), sv[x]);
  }
  d2 = add(add(mul(dd[0], dd[0]), mul(dd[1], dd[1])), mul(dd[2], dd[2]));
  return __dsqrt_rn(d2) < rc;
}

__device__ __forceinline__ int floor_div(int a, int b) {
  int q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) q--;
  return q;
}

__device__ __forceinline__ uint64_t edge_key(int j, int s0, int s1, int s2) {
  return ((uint64_t)(uint32_t)j << 24) | ((uint64_t)(uint32_t)(s0 + 128) << 16) | ((uint64_t)(uint32_t)(s1 + 128) << 8) |
         (uint64_t)(uint32_t)(s2 + 128);
}

struct Work {        // int32 workspace layout
  int* count;        // ncells
  int* start;        // ncells + 1
  int* fill;         // ncells
  int* acell;        // N
  int* awrap;        // 3N
  int* sorted;       // N
  int* flag;         // 1: error flag (shift out of range / row too long)
};

inline Work carve(void* ws, int64_t N, int64_t ncells) {
  Work w;
  int* p = (int*)ws;
  w.count = p; p += ncells;
  w.start = p; p += ncells + 1;
  w.fill = p; p += ncells;
  w.acell = p; p += N;
  w.awrap = p; p += 3 * N;
  w.sorted = p; p += N;
  w.flag = p; p += 1;
  return w;
}
inline int64_t ws_ints(int64_t N, int64_t ncells) { return 3 * ncells + 1 + 5 * N + 1; }

int make_grid(const double* cell, double rc, CellGrid& g) {
  for (int k = 0; k < 9; k++) g.cell[k] = cell[k];
  const double* a = cell;
  const double* b = cell + 3;
  const double* c = cell + 6;
  const double det = a[0] * (b[1] * c[2] - b[2] * c[1]) - a[1] * (b[0] * c[2] - b[2] * c[0]) + a[2] * (b[0] * c[1] - b[1] * c[0]);
  if (!(fabs(det) > 1e-12)) {
    set_error("neighbour list: singular cell (det=%g)", det);
    return FACEK_EINVAL;
  }
  // inverse (rows of inv = columns of reciprocal basis / 1)
  g.inv[0] = (b[1] * c[2] - b[2] * c[1]) / det;
  g.inv[1] = (a[2] * c[1] - a[1] * c[2]) / det;
  g.inv[2] = (a[1] * b[2] - a[2] * b[1]) / det;
  g.inv[3] = (b[2] * c[0] - b[0] * c[2]) / det;
  g.inv[4] = (a[0] * c[2] - a[2] * c[0]) / det;
  g.inv[5] = (a[2] * b[0] - a[0] * b[2]) / det;
  g.inv[6] = (b[0] * c[1] - b[1] * c[0]) / det;
  g.inv[7] = (a[1] * c[0] - a[0] * c[1]) / det;
  g.inv[8] = (a[0] * b[1] - a[1] * b[0]) / det;
  const double V = fabs(det);
  auto cross_norm = [](const double* u, const double* v) {
    const double x = u[1] * v[2] - u[2] * v[1], y = u[2] * v[0] - u[0] * v[2], z = u[0] * v[1] - u[1] * v[0];
    return sqrt(x * x + y * y + z * z);
  };
  const double h[3] = {V / cross_norm(b, c), V / cross_norm(c, a), V / cross_norm(a, b)};
  g.ncells = 1;
  for (int d = 0; d < 3; d++) {
    // cells strictly wider than rc/ns (shrunk by 1e-9 so that h/rc exactly integral cannot put a neighbour
    // on the far boundary of the scanned block)
    int n = (int)floor(h[d] / rc * (1.0 - 1e-9));
    if (n < 1) n = 1;
    if (n > 1024) n = 1024;
    g.nc[d] = n;
    g.ns[d] = (int)ceil(rc * n / h[d]);
    if (g.ns[d] < 1) g.ns[d] = 1;
    g.ncells *= n;
  }
  return FACEK_OK;
}

__global__ void bin_k(const double* __restrict__ pos, int64_t N, CellGrid g, Work w) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    int c[3];
#pragma unroll
    for (int d = 0; d < 3; d++) {
      const double f = pos[i * 3] * g.inv[d] + pos[i * 3 + 1] * g.inv[3 + d] + pos[i * 3 + 2] * g.inv[6 + d];
      const double wf = floor(f);
      int cc = (int)((f - wf) * g.nc[d]);
      c[d] = cc < 0 ? 0 : (cc >= g.nc[d] ? g.nc[d] - 1 : cc);
      w.awrap[i * 3 + d] = (int)wf;
    }
    const int cell = (c[0] * g.nc[1] + c[1]) * g.nc[2] + c[2];
    w.acell[i] = cell;
    atomicAdd(&w.count[cell], 1);
  }
}

// single-block exclusive scan of counts into start[0..n]
__global__ void scan_k(const int* __restrict__ cnt, int* __restrict__ start, int64_t n) {
  __shared__ int part[1024];
  const int t = threadIdx.x, T = blockDim.x;
  const int64_t per = (n + T - 1) / T;
  const int64_t lo = t * per, hi = lo + per < n ? lo + per : n;
  int s = 0;
  for (int64_t k = lo; k < hi; k++) s += cnt[k];
  part[t] = s;
  __syncthreads();
  if (t == 0) {
    int acc = 0;
    for (int k = 0; k < T; k++) {
      const int v = part[k];
      part[k] = acc;
      acc += v;
    }
    start[n] = acc;
  }
  __syncthreads();
  int acc = part[t];
  for (int64_t k = lo; k < hi; k++) {
    start[k] = acc;
    acc += cnt[k];
  }
}

__global__ void scatter_k(int64_t N, Work w) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const int cell = w.acell[i];
    const int slot = atomicAdd(&w.fill[cell], 1);
    w.sorted[w.start[cell] + slot] = (int)i;
  }
}

__global__ void sort_cells_k(int64_t ncells, Work w) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < ncells; c += (int64_t)gridDim.x * blockDim.x) {
    int* a = w.sorted + w.start[c];
    const int n = w.start[c + 1] - w.start[c];
    for (int k = 1; k < n; k++) {
      const int v = a[k];
      int m = k - 1;
      while (m >= 0 && a[m] > v) {
        a[m + 1] = a[m];
        m--;
      }
      a[m + 1] = v;
    }
  }
}

constexpr int MAXDEG = 512;

// count (FILL=false) or fill + sort (FILL=true) one row per thread
template <bool FILL, typename T>
__global__ void __launch_bounds__(128) cell_rows_k(const double* __restrict__ pos, int64_t N, CellGrid g, Work w,
                                                   double rc, int32_t* __restrict__ deg,
                                                   const int32_t* __restrict__ row_ptr, int32_t* __restrict__ ei,
                                                   int32_t* __restrict__ ej, int32_t* __restrict__ S,
                                                   T* __restrict__ shift) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const double pi[3] = {pos[i * 3], pos[i * 3 + 1], pos[i * 3 + 2]};
    const int cell = w.acell[i];
    const int ci[3] = {cell / (g.nc[1] * g.nc[2]), (cell / g.nc[2]) % g.nc[1], cell % g.nc[2]};
    const int wi[3] = {w.awrap[i * 3], w.awrap[i * 3 + 1], w.awrap[i * 3 + 2]};
    int cnt = 0;
    const int64_t base = FILL ? row_ptr[i] : 0;
    for (int dx = -g.ns[0]; dx <= g.ns[0]; dx++) {
      const int cx = ci[0] + dx, ox = floor_div(cx, g.nc[0]), wx = cx - ox * g.nc[0];
      for (int dy = -g.ns[1]; dy <= g.ns[1]; dy++) {
        const int cy = ci[1] + dy, oy = floor_div(cy, g.nc[1]), wy = cy - oy * g.nc[1];
        for (int dz = -g.ns[2]; dz <= g.ns[2]; dz++) {
          const int cz = ci[2] + dz, oz = floor_div(cz, g.nc[2]), wz = cz - oz * g.nc[2];
          const int cc = (wx * g.nc[1] + wy) * g.nc[2] + wz;
          for (int q = w.start[cc]; q < w.start[cc + 1]; q++) {
            const int j = w.sorted[q];
            const int s0 = ox - w.awrap[j * 3] + wi[0];
            const int s1 = oy - w.awrap[j * 3 + 1] + wi[1];
            const int s2 = oz - w.awrap[j * 3 + 2] + wi[2];
            if (j == i && s0 == 0 && s1 == 0 && s2 == 0) continue;
            double sv[3];
            const double pj[3] = {pos[(int64_t)j * 3], pos[(int64_t)j * 3 + 1], pos[(int64_t)j * 3 + 2]};
            if (!within(pi, pj, g.cell, s0, s1, s2, rc, sv)) continue;
            if (FILL) {
              const int64_t e = base + cnt;
              ej[e] = j;
              S[e * 3] = s0; S[e * 3 + 1] = s1; S[e * 3 + 2] = s2;
            }
            cnt++;
          }
        }
      }
    }
    if (!FILL) {
      deg[i] = cnt;
      // rows longer than MAXDEG are rejected before any row offsets are used: the fill pass cannot sort them, and
      // with every row at most MAXDEG long the int32 prefix sum stays below 2^31 for up to 2^22 rows
      if (cnt > MAXDEG) atomicExch(w.flag, 1);
      continue;
    }
    // sort the row by (j, S) and write shift vectors
    if (cnt > MAXDEG) {
      atomicExch(w.flag, 1);
      continue;
    }
    uint64_t key[MAXDEG];
    for (int k = 0; k < cnt; k++) {
      const int64_t e = base + k;
      if (S[e * 3] < -127 || S[e * 3] > 127 || S[e * 3 + 1] < -127 || S[e * 3 + 1] > 127 || S[e * 3 + 2] < -127 ||
          S[e * 3 + 2] > 127)
        atomicExch(w.flag, 2);
      key[k] = edge_key(ej[e], S[e * 3], S[e * 3 + 1], S[e * 3 + 2]);
    }
    for (int k = 1; k < cnt; k++) {
      const uint64_t v = key[k];
      int m = k - 1;
      while (m >= 0 && key[m] > v) {
        key[m + 1] = key[m];
        m--;
      }
      key[m + 1] = v;
    }
    for (int k = 0; k < cnt; k++) {
      const int64_t e = base + k;
      const int j = (int)(key[k] >> 24);
      const int s0 = (int)((key[k] >> 16) & 0xff) - 128, s1 = (int)((key[k] >> 8) & 0xff) - 128,
                s2 = (int)(key[k] & 0xff) - 128;
      ei[e] = (int)i;
      ej[e] = j;
      S[e * 3] = s0; S[e * 3 + 1] = s1; S[e * 3 + 2] = s2;
#pragma unroll
      for (int x = 0; x < 3; x++)
        shift[e * 3 + x] = (T)add(add(mul((double)s0, g.cell[x]), mul((double)s1, g.cell[3 + x])),
                                  mul((double)s2, g.cell[6 + x]));
    }
  }
}

template <bool FILL, typename T>
__global__ void batch_rows_k(const double* __restrict__ pos, int64_t N, const int32_t* __restrict__ sstart,
                             const int32_t* __restrict__ astruct, double rc, int32_t* __restrict__ deg,
                             const int32_t* __restrict__ row_ptr, int32_t* __restrict__ ei, int32_t* __restrict__ ej,
                             int32_t* __restrict__ S, T* __restrict__ shift) {
  const double zero_cell[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const double pi[3] = {pos[i * 3], pos[i * 3 + 1], pos[i * 3 + 2]};
    const int s = astruct[i];
    int cnt = 0;
    const int64_t base = FILL ? row_ptr[i] : 0;
    for (int j = sstart[s]; j < sstart[s + 1]; j++) {
      if (j == i) continue;
      const double pj[3] = {pos[(int64_t)j * 3], pos[(int64_t)j * 3 + 1], pos[(int64_t)j * 3 + 2]};
      double sv[3];
      if (!within(pi, pj, zero_cell, 0, 0, 0, rc, sv)) continue;
      if (FILL) {
        const int64_t e = base + cnt;
        ei[e] = (int)i;
        ej[e] = j;
        S[e * 3] = 0; S[e * 3 + 1] = 0; S[e * 3 + 2] = 0;
        shift[e * 3] = 0; shift[e * 3 + 1] = 0; shift[e * 3 + 2] = 0;
      }
      cnt++;
    }
    if (!FILL) deg[i] = cnt;
  }
}

__global__ void reverse_k(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ ei,
                          const int32_t* __restrict__ ej, const int32_t* __restrict__ S, int64_t E,
                          int32_t* __restrict__ rev) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = ei[e], j = ej[e];
    const uint64_t want = edge_key(i, -S[e * 3], -S[e * 3 + 1], -S[e * 3 + 2]);
    int lo = row_ptr[j], hi = row_ptr[j + 1] - 1, found = -1;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      const uint64_t k = edge_key(ej[mid], S[(int64_t)mid * 3], S[(int64_t)mid * 3 + 1], S[(int64_t)mid * 3 + 2]);
      if (k == want) { found = mid; break; }
      if (k < want) lo = mid + 1; else hi = mid - 1;
    }
    rev[e] = found;
  }
}

inline int ew_grid(int64_t n) { return grid_for(ceil_div<int64_t>(n, 128), 16); }

template <typename T>
int cell_fill(const double* pos, int64_t N, const double* cell, double rc, void* workspace, const int32_t* row_ptr,
              int32_t* ei, int32_t* ej, int32_t* S, void* shift, void* stream) {
  CellGrid g;
  int st = make_grid(cell, rc, g);
  if (st) return st;
  Work w = carve(workspace, N, g.ncells);
  cudaMemsetAsync(w.flag, 0, sizeof(int), as_stream(stream));
  cell_rows_k<true, T><<<ew_grid(N), 128, 0, as_stream(stream)>>>(pos, N, g, w, rc, nullptr, row_ptr, ei, ej, S,
                                                                  (T*)shift);
  st = launch_status("facek_nlist_cell_fill");
  if (st) return st;
  int flag = 0;
  cudaMemcpyAsync(&flag, w.flag, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream));
  cudaStreamSynchronize(as_stream(stream));
  if (flag == 1) {
    set_error("facek_nlist_cell_fill: a row has more than %d neighbours", MAXDEG);
    return FACEK_EUNSUPPORTED;
  }
  if (flag == 2) {
    set_error("facek_nlist_cell_fill: periodic image shift beyond +-127 cells");
    return FACEK_EUNSUPPORTED;
  }
  return FACEK_OK;
}

template <typename T>
int batch_fill(const double* pos, int64_t N, const int32_t* sstart, const int32_t* astruct, double rc,
               const int32_t* row_ptr, int32_t* ei, int32_t* ej, int32_t* S, void* shift, void* stream) {
  if (N == 0) return FACEK_OK;
  batch_rows_k<true, T><<<ew_grid(N), 128, 0, as_stream(stream)>>>(pos, N, sstart, astruct, rc, nullptr, row_ptr, ei,
                                                                    ej, S, (T*)shift);
  return launch_status("facek_nlist_batch_fill");
}

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free variant of the periodic build.  Its scratch (cell counts and offsets, per-atom bin and wrap, the
// cell-sorted atom order, per-atom degrees) lives in one file-scope device array instead of a caller buffer, for
// callers that cannot allocate device memory.  Limits: NOALLOC_MAX_ATOMS atoms, NOALLOC_MAX_CELLS cells.
constexpr int64_t NOALLOC_MAX_ATOMS = 262144;
constexpr int64_t NOALLOC_MAX_CELLS = 65536;
constexpr int64_t NOALLOC_INTS = 3 * NOALLOC_MAX_CELLS + 1 + 5 * NOALLOC_MAX_ATOMS + 1 + NOALLOC_MAX_ATOMS;

static __device__ __align__(256) int g_nlist_scratch[NOALLOC_INTS];     // about 7.1 MB per device

// Device address of the scratch array on the current device.  g_nlist_scratch named in host code is only a
// host-side stand-in, so the address is looked up with cudaGetSymbolAddress, with the caller's device current, on
// every call: a cached address would go stale if the host application reset the device or its primary context,
// and the lookup costs little next to the call's two stream synchronisations.
int noalloc_scratch(int** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_nlist_scratch);
  if (e != cudaSuccess || !p) {
    set_error("facek_nlist_cell_build_noalloc: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
    return FACEK_ELAUNCH;
  }
  *out = static_cast<int*>(p);
  return FACEK_OK;
}

template <typename T>
int build_noalloc(const double* pos, int64_t N, const double* cell, double rc, int64_t max_edges, int32_t* row_ptr,
                  int32_t* ei, int32_t* ej, int32_t* S, void* shift, int64_t* n_edges, void* stream) {
  CellGrid g;
  int st = make_grid(cell, rc, g);
  if (st) return st;
  FACEK_CHECK_ARG(N <= NOALLOC_MAX_ATOMS, "facek_nlist_cell_build_noalloc: N=%lld atoms exceeds the limit of %lld",
                  (long long)N, (long long)NOALLOC_MAX_ATOMS);
  FACEK_CHECK_ARG(g.ncells <= NOALLOC_MAX_CELLS,
                  "facek_nlist_cell_build_noalloc: %lld cells exceed the limit of %lld (cell too large for rc)",
                  (long long)g.ncells, (long long)NOALLOC_MAX_CELLS);
  int* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  const int64_t used = ws_ints(N, g.ncells);
  Work w = carve(scratch, N, g.ncells);
  int32_t* deg = scratch + used;
  // the array keeps the previous call's contents: clear every counter this call relies on
  if (cudaMemsetAsync(scratch, 0, sizeof(int) * (used + N), s) != cudaSuccess) return launch_status("memset");
  bin_k<<<ew_grid(N), 128, 0, s>>>(pos, N, g, w);
  scan_k<<<1, 1024, 0, s>>>(w.count, w.start, g.ncells);
  scatter_k<<<ew_grid(N), 128, 0, s>>>(N, w);
  sort_cells_k<<<ew_grid(g.ncells), 128, 0, s>>>(g.ncells, w);
  cell_rows_k<false, float><<<ew_grid(N), 128, 0, s>>>(pos, N, g, w, rc, deg, nullptr, nullptr, nullptr, nullptr,
                                                        nullptr);
  scan_k<<<1, 1024, 0, s>>>(deg, row_ptr, N);
  st = launch_status("facek_nlist_cell_build_noalloc(count)");
  if (st) return st;
  int total = 0, too_long = 0;
  cudaMemcpyAsync(&total, row_ptr + N, sizeof(int), cudaMemcpyDeviceToHost, s);
  cudaMemcpyAsync(&too_long, w.flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("facek_nlist_cell_build_noalloc(sync)");
  if (too_long) {
    *n_edges = -1;
    set_error("facek_nlist_cell_build_noalloc: a row has more than %d neighbours", MAXDEG);
    return FACEK_EUNSUPPORTED;
  }
  if (total < 0) {      // unreachable with rows of at most MAXDEG and N <= NOALLOC_MAX_ATOMS; kept as a guard
    *n_edges = -1;
    set_error("facek_nlist_cell_build_noalloc: edge count overflow");
    return FACEK_EUNSUPPORTED;
  }
  *n_edges = total;
  if (total > max_edges) {
    set_error("facek_nlist_cell_build_noalloc: %d edges exceed the output capacity max_edges=%lld", total,
              (long long)max_edges);
    return FACEK_EINVAL;
  }
  if (total == 0) return FACEK_OK;
  cell_rows_k<true, T><<<ew_grid(N), 128, 0, s>>>(pos, N, g, w, rc, nullptr, row_ptr, ei, ej, S, (T*)shift);
  st = launch_status("facek_nlist_cell_build_noalloc(fill)");
  if (st) return st;
  int flag = 0;
  cudaMemcpyAsync(&flag, w.flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("facek_nlist_cell_build_noalloc(sync)");
  if (flag == 1) {
    set_error("facek_nlist_cell_build_noalloc: a row has more than %d neighbours", MAXDEG);
    return FACEK_EUNSUPPORTED;
  }
  if (flag == 2) {
    set_error("facek_nlist_cell_build_noalloc: periodic image shift beyond +-127 cells");
    return FACEK_EUNSUPPORTED;
  }
  return FACEK_OK;
}

}  // namespace
}  // namespace facek

using namespace facek;

extern "C" int facek_nlist_cell_workspace(int64_t N, const double* cell, double rc, int64_t* bytes) {
  FACEK_CHECK_ARG(N >= 0 && rc > 0 && cell && bytes, "facek_nlist_cell_workspace: bad arguments");
  CellGrid g;
  int st = make_grid(cell, rc, g);
  if (st) return st;
  *bytes = 4 * ws_ints(N, g.ncells);
  return FACEK_OK;
}

extern "C" int facek_nlist_cell_count(const double* pos, int64_t N, const double* cell, double rc, void* workspace,
                                      int32_t* deg, void* stream) {
  FACEK_CHECK_ARG(N > 0 && rc > 0 && pos && cell && workspace && deg, "facek_nlist_cell_count: bad arguments");
  CellGrid g;
  int st = make_grid(cell, rc, g);
  if (st) return st;
  Work w = carve(workspace, N, g.ncells);
  cudaStream_t s = as_stream(stream);
  cudaMemsetAsync(workspace, 0, sizeof(int) * ws_ints(N, g.ncells), s);
  bin_k<<<ew_grid(N), 128, 0, s>>>(pos, N, g, w);
  scan_k<<<1, 1024, 0, s>>>(w.count, w.start, g.ncells);
  scatter_k<<<ew_grid(N), 128, 0, s>>>(N, w);
  sort_cells_k<<<ew_grid(g.ncells), 128, 0, s>>>(g.ncells, w);
  cell_rows_k<false, float><<<ew_grid(N), 128, 0, s>>>(pos, N, g, w, rc, deg, nullptr, nullptr, nullptr, nullptr,
                                                        nullptr);
  return launch_status("facek_nlist_cell_count");
}

extern "C" int facek_nlist_cell_fill(int dtype, const double* pos, int64_t N, const double* cell, double rc,
                                     void* workspace, const int32_t* row_ptr, int32_t* ei, int32_t* ej, int32_t* S,
                                     void* shift, void* stream) {
  FACEK_CHECK_ARG(N > 0 && rc > 0 && pos && cell && workspace && row_ptr && ei && ej && S && shift,
                  "facek_nlist_cell_fill: bad arguments");
  return FACEK_DISPATCH(dtype, cell_fill, pos, N, cell, rc, workspace, row_ptr, ei, ej, S, shift, stream);
}

extern "C" int facek_nlist_batch_count(const double* pos, int64_t N, const int32_t* struct_start,
                                       const int32_t* atom_struct, double rc, int32_t* deg, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && rc > 0 && (N == 0 || (pos && struct_start && atom_struct && deg)),
                  "facek_nlist_batch_count: bad arguments");
  if (N == 0) return FACEK_OK;
  batch_rows_k<false, float><<<ew_grid(N), 128, 0, as_stream(stream)>>>(pos, N, struct_start, atom_struct, rc, deg,
                                                                         nullptr, nullptr, nullptr, nullptr, nullptr);
  return launch_status("facek_nlist_batch_count");
}

extern "C" int facek_nlist_batch_fill(int dtype, const double* pos, int64_t N, const int32_t* struct_start,
                                      const int32_t* atom_struct, double rc, const int32_t* row_ptr, int32_t* ei,
                                      int32_t* ej, int32_t* S, void* shift, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && rc > 0, "facek_nlist_batch_fill: bad arguments");
  return FACEK_DISPATCH(dtype, batch_fill, pos, N, struct_start, atom_struct, rc, row_ptr, ei, ej, S, shift, stream);
}

extern "C" int facek_nlist_reverse(const int32_t* row_ptr, const int32_t* ei, const int32_t* ej, const int32_t* S,
                                   int64_t N, int64_t E, int32_t* rev, void* stream) {
  FACEK_CHECK_ARG(N >= 0 && E >= 0 && (E == 0 || (row_ptr && ei && ej && S && rev)), "facek_nlist_reverse: bad args");
  if (E == 0) return FACEK_OK;
  reverse_k<<<ew_grid(E), 128, 0, as_stream(stream)>>>(row_ptr, ei, ej, S, E, rev);
  return launch_status("facek_nlist_reverse");
}

extern "C" int facek_nlist_cell_build_noalloc(int dtype, const double* pos, int64_t N, const double* cell, double rc,
                                              int64_t max_edges, int32_t* row_ptr, int32_t* ei, int32_t* ej,
                                              int32_t* S, void* shift, int64_t* n_edges, void* stream) {
  FACEK_CHECK_ARG(N > 0 && rc > 0 && max_edges >= 0 && pos && cell && row_ptr && n_edges &&
                      (max_edges == 0 || (ei && ej && S && shift)),
                  "facek_nlist_cell_build_noalloc: bad arguments");
  return FACEK_DISPATCH(dtype, build_noalloc, pos, N, cell, rc, max_edges, row_ptr, ei, ej, S, shift, n_edges,
                        stream);
}
