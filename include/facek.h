/* facek.h -- C ABI of libfacek.so, the B200 (sm_100a) kernels behind the face_b200 engine.
 *
 * Conventions (all entry points):
 *   - plain device pointers and sizes, no framework types; the caller owns every buffer (the library never
 *     allocates device memory), exactly like face-mlip's CuPy kernels, which receive DLPack pointers from
 *     torch-allocated tensors (face/kernels.py:131-132, :141; face/node_kernel.py:174-176);
 *   - `dtype` is FACEK_F32 or FACEK_F64 and applies to every floating-point buffer of the call;
 *   - `stream` is a cudaStream_t passed as void* (the reference launches on torch's current stream,
 *     face/kernels.py:145);
 *   - index buffers are int32 (atoms and edges < 2^31); `row_ptr` is the CSR row offset array (N+1 entries)
 *     of a centre-sorted edge list;
 *   - return 0 on success, a negative FACEK_E* code otherwise; facek_last_error() gives the message.
 *     The reference has no error reporting at all (shape limits are implicit, face/kernels.py:146,159-163).
 */
#ifndef FACEK_H
#define FACEK_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { FACEK_F32 = 0, FACEK_F64 = 1 };
enum { FACEK_OK = 0, FACEK_EINVAL = -1, FACEK_ELAUNCH = -2, FACEK_ETIMEOUT = -3, FACEK_EUNSUPPORTED = -4 };

const char* facek_last_error(void);
int facek_version(void);

/* ---------------------------------------------------------------------------------------------------
 * Factorised Cartesian density  D[i, x, b*K + k] = sum_m phi[m, b] * msg[m, k] * Y[m, x],  x = 0..19.
 * Replaces face-mlip face/kernels.py:22-54 (dens_fwd) and :56-118 (dens_bwd) behind
 * face.kernels.factor_density (face/kernels.py:170-172).
 * Rows: padded layout (row_ptr == NULL: row i = edges i*M .. i*M+M-1, the reference's (N,M,*) tensors)
 * or CSR (row_ptr != NULL, M ignored).  phi (E,B), msg (E,K), Y (E,20), D / G (N,20,B*K).
 */
int facek_density_fwd(int dtype, const void* phi, const void* msg, const void* Y, void* D, int64_t N, int32_t M,
                      int32_t B, int32_t K, const int32_t* row_ptr, void* stream);
int facek_density_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G, void* dphi,
                      void* dmsg, void* dY, int64_t N, int32_t M, int32_t B, int32_t K, const int32_t* row_ptr,
                      void* stream);
/* Same contraction for the engine, component-major ("x-major") layout: D is (20, N, B*K), so the rank blocks
 * D[0:1], D[1:4], D[4:10], D[10:20] are contiguous (k_l*N, B*K) GEMM operands for the channel maps
 * (face/model.py:506); the backward takes the four rank gradients as separate (k_l, N, B*K) buffers G0..G3. */
int facek_density_xm_fwd(int dtype, const void* phi, const void* msg, const void* Y, void* D, int64_t N, int32_t B,
                         int32_t K, const int32_t* row_ptr, void* stream);
int facek_density_xm_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G0, const void* G1,
                         const void* G2, const void* G3, void* dphi, void* dmsg, void* dY, int64_t N, int32_t B,
                         int32_t K, const int32_t* row_ptr, void* stream);
/* facek_density_xm_fwd on the tcgen05 tensor cores (fp32, B = 16, K = 32 only): per atom the GEMM
 * D_i[(x,b), k] = sum_e (Y[e,x] phi[e,b]) msg[e,k] with M/N-major operands and the 3-term tf32 split.  Same
 * outputs as facek_density_xm_fwd to fp32 accuracy; at present slower than it on the cfg5 alloy, so the default
 * entry keeps the CUDA-core kernel.  No reference counterpart as a C entry point (face/kernels.py:22-54). */
int facek_density_tc_xm_fwd(const float* phi, const float* msg, const float* Y, float* D, int64_t N, int32_t B,
                            int32_t K, const int32_t* row_ptr, void* stream);
/* Density adjoint fused with the message part of dY (face/model.py:473-513; the reference runs the CuPy density
 * backward, face/kernels.py:56-118, and autograd through the message GEMV): the outputs of facek_density_xm_bwd,
 * with dY[e, c] (c < nc) additionally += sum_k dmsg[e,k] (TJ[c, ej, k] + TI[c, ei, k]), TJ/TI (nc, N, K) as in
 * facek_edge_msg_fwd (TI may be NULL).  dTJ/dTI then come from facek_edge_msg_bwd with dY = NULL. */
int facek_density_msg_xm_bwd(int dtype, const void* phi, const void* msg, const void* Y, const void* G0,
                             const void* G1, const void* G2, const void* G3, const void* TJ, const void* TI,
                             const int32_t* ei, const int32_t* ej, int32_t nc, void* dphi, void* dmsg, void* dY,
                             int64_t N, int64_t E, int32_t B, int32_t K, const int32_t* row_ptr, void* stream);
/* The same outputs on the tcgen05 tensor cores (fp32, B = 16, K = 32 only; no reference counterpart as a C entry
 * point, face/kernels.py:56-118): per atom and chunk of up to 128 edges, T[e,(x,b)] = msg[e,:] . G[x,b,:] and
 * U[e,(x,k)] = phi[e,:] . G[x,:,k] as two MMAs with the edges as M (3-term tf32 split), then dphi, dY and dmsg from
 * T and U on the CUDA cores; the message part of dY follows as in facek_edge_msg_bwd.  Needs 16-byte aligned
 * tensors and ~208 KB of opt-in shared memory.  Same outputs to fp32 accuracy; at present slower than
 * facek_density_msg_xm_bwd on the cfg5 alloy (operand staging bound), so the engine keeps the CUDA-core kernel. */
int facek_density_msg_tc_xm_bwd(const float* phi, const float* msg, const float* Y, const float* G0, const float* G1,
                                const float* G2, const float* G3, const float* TJ, const float* TI, const int32_t* ei,
                                const int32_t* ej, int32_t nc, float* dphi, float* dmsg, float* dY, int64_t N,
                                int64_t E, int32_t B, int32_t K, const int32_t* row_ptr, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Node invariant algebra, reference layout.  Replaces face-mlip face/node_kernel.py:18-64 (node_fwd) and
 * :66-151 (node_bwd) behind face.node_kernel.node_algebra (:207-209).
 * P1,Q1,S1 (N,C,3); P2,Q2,S2 (N,C,6); P3,Q3 (N,C,10) symmetric storage; a, b (4,C) path weights (the
 * reference transposes them to (C,4) before launch, face/node_kernel.py:173).  inv (N,C,8), V (N,C,3),
 * Mf (N,C,3,3).  Backward: gI/gV/gM upstream (gV, gM may be NULL when eq == 0); writes the 8 input
 * gradients and per-(atom,channel) partials da_part, db_part (N,C,4) (may be NULL when eq == 0).
 */
int facek_node_fwd(int dtype, const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2,
                   const void* S2, const void* P3, const void* Q3, const void* a, const void* b, void* inv, void* V,
                   void* Mf, int64_t N, int32_t C, int32_t eq, void* stream);
int facek_node_bwd(int dtype, const void* P1, const void* Q1, const void* S1, const void* P2, const void* Q2,
                   const void* S2, const void* P3, const void* Q3, const void* a, const void* b, const void* gI,
                   const void* gV, const void* gM, void* dP1, void* dQ1, void* dS1, void* dP2, void* dQ2, void* dS2,
                   void* dP3, void* dQ3, void* da_part, void* db_part, int64_t N, int32_t C, int32_t eq,
                   void* stream);

/* Node algebra, engine layout (component-major): the projected moments y_l = proj_l(x_l) as (k_l, N, 3C) with P,
 * Q, S in channel blocks [0,C), [C,2C), [2C,3C) (face/model.py:227 without its transposes); writes the 9 families
 * [P0 | i1..i8] as inv9 (N, 9C) with families above max_body zeroed (face/model.py:244-247), V (3,N,C) and
 * Ms (6,N,C) = symmetric storage of (Mf + Mf^T)/2 (face/model.py:274-276) when eq != 0.
 * Backward writes dy_l in the same layouts (dQ0, dS0, dS3 are zero: unused by the reference). */
int facek_node_engine_fwd(int dtype, const void* y0, const void* y1, const void* y2, const void* y3, const void* a,
                          const void* b, void* inv9, void* V, void* Ms, int64_t N, int32_t C, int32_t eq,
                          int32_t max_body, void* stream);
int facek_node_engine_bwd(int dtype, const void* y0, const void* y1, const void* y2, const void* y3, const void* a,
                          const void* b, const void* g_inv9, const void* gV, const void* gMs, void* dy0, void* dy1,
                          void* dy2, void* dy3, int64_t N, int32_t C, int32_t eq, int32_t max_body, void* stream);

/* Per-atom broadcast scaling over the J components of one Cartesian rank, engine layout (J, N, C):
 * out[j,n,c] = x[j,n,c] * s[n*lds + c] -- the moment scaling by elem_scale / <neighbours> (face/model.py:183-186,
 * :200-201) and the gates of the equivariant products (face/model.py:277-295); s may be a column slice (lds >= C).
 * Backward: dx = g * s and, when ds is non-null, ds[n,c] = sum_j g[j,n,c] x[j,n,c] (dense (N, C)). */
int facek_bcast_mul_fwd(int dtype, const void* x, const void* s, void* out, int32_t J, int64_t N, int32_t C,
                        int64_t lds, void* stream);
int facek_bcast_mul_bwd(int dtype, const void* g, const void* x, const void* s, void* dx, void* ds, int32_t J,
                        int64_t N, int32_t C, int64_t lds, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Neighbour list (cell list, fp64 distance test), replacing ase.neighborlist.neighbor_list("ijS") as called at
 * face-mlip face/neighbors.py:12 and face/datasets.py:51 (+ the stable argsort and slot fill :14, :74-79).
 * Edge set: every (i, j, S) with |pos[j] - pos[i] + S.cell| < rc except the zero-shift self pair; rows are
 * centre-sorted and, within a row, in (j, S0, S1, S2) order.
 * Periodic single structure (pbc on all axes):
 *   facek_nlist_cell_workspace(N, cell, rc, &bytes)  size of the int32 scratch the caller provides;
 *   facek_nlist_cell_count   -> deg (N)
 *   (caller: row_ptr = exclusive prefix sum of deg)
 *   facek_nlist_cell_fill    -> ei (E) centre, ej (E) neighbour, S (E,3 int32) image, shift (E,3) = S.cell in
 *                               the model dtype (face/datasets.py:52)
 * Non-periodic batch of structures (atoms of structure s are struct_start[s] .. struct_start[s+1]-1):
 *   facek_nlist_batch_count / facek_nlist_batch_fill (all pairs within a structure, shift = 0).
 * Reverse index: rev[e] = index of the edge (j, i, -S) (the list is symmetric); used by the atomic-free
 * gathers below.
 */
int facek_nlist_cell_workspace(int64_t N, const double* cell, double rc, int64_t* bytes);
int facek_nlist_cell_count(const double* pos, int64_t N, const double* cell, double rc, void* workspace,
                           int32_t* deg, void* stream);
int facek_nlist_cell_fill(int dtype, const double* pos, int64_t N, const double* cell, double rc, void* workspace,
                          const int32_t* row_ptr, int32_t* ei, int32_t* ej, int32_t* S, void* shift, void* stream);
int facek_nlist_batch_count(const double* pos, int64_t N, const int32_t* struct_start, const int32_t* atom_struct,
                            double rc, int32_t* deg, void* stream);
int facek_nlist_batch_fill(int dtype, const double* pos, int64_t N, const int32_t* struct_start,
                           const int32_t* atom_struct, double rc, const int32_t* row_ptr, int32_t* ei, int32_t* ej,
                           int32_t* S, void* shift, void* stream);
int facek_nlist_reverse(const int32_t* row_ptr, const int32_t* ei, const int32_t* ej, const int32_t* S, int64_t N,
                        int64_t E, int32_t* rev, void* stream);
/* Allocation-free periodic build (no counterpart in the reference): the same edge set, order and outputs as
 * facek_nlist_cell_count + prefix sum + facek_nlist_cell_fill, for callers that cannot allocate device memory
 * themselves (a host framework that hands out only preallocated buffers, or code running inside a memory pool
 * or arena that forbids cudaMalloc).  The scratch lives in a file-scope device array of about 7.1 MB that every
 * GPU loading the library holds until exit; limits: N <= 262,144 atoms and <= 65,536 cells.  The caller passes
 * row_ptr (N+1) and output buffers of capacity max_edges; *n_edges receives the edge count.  When that count exceeds
 * max_edges the call returns FACEK_EINVAL with ei/ej/S/shift untouched but row_ptr already written (the caller can
 * retry with larger buffers); a row longer than 512 neighbours returns FACEK_EUNSUPPORTED before any edge is
 * written (*n_edges = -1).  Calls no cudaMalloc/cudaFree.  The scratch's device address is looked up
 * (cudaGetSymbolAddress) on every call with the caller's device current.  The call synchronises the stream twice
 * (edge count, error flags), so it cannot be captured into a CUDA graph.
 * All calls share the scratch array: calls that overlap on the GPU (other streams, other host threads) race. */
int facek_nlist_cell_build_noalloc(int dtype, const double* pos, int64_t N, const double* cell, double rc,
                                   int64_t max_edges, int32_t* row_ptr, int32_t* ei, int32_t* ej, int32_t* S,
                                   void* shift, int64_t* n_edges, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Edge geometry: vec[e] = pos[ej] - pos[ei] + shift[e] (face/model.py:670) and its adjoint, the force gather
 * dpos[k] = sum_{e in row k} (dvec[rev[e]] - dvec[e]) (autograd through :670 and :693, without atomics).
 * Y[e] = 20 symmetric monomials of u = vec/|vec| (face/cartesian.py:34-46, face/model.py:671-677);
 * sym_bwd accumulates dvec += d(Y)/d(vec)^T dY.
 */
int facek_edge_vec(int dtype, const void* pos, const int32_t* ei, const int32_t* ej, const void* shift, void* vec,
                   int64_t E, void* stream);
int facek_edge_vec_bwd(int dtype, const void* dvec, const int32_t* row_ptr, const int32_t* rev, int64_t N,
                       void* dpos, void* stream);
int facek_edge_sym(int dtype, const void* vec, void* Y, int64_t E, void* stream);
int facek_edge_sym_bwd(int dtype, const void* vec, const void* dY, void* dvec, int32_t accumulate, int64_t E,
                       void* stream);

/* Radial basis x learned radial MLP of one factorised block (face/model.py:28-40, :465-469):
 * phi[e, b] = radial(silu(rad_in(bessel(r)*env(r)) + pair[zi*n_el + zj])) * env(r), and dphi/dr by forward-mode
 * differentiation (replacing autograd through the MLP).  Weights are effective (unit scaling applied):
 * w1 (H,nb) b1 (H) pair (n_el^2,H) w2 (H,H) b2 (H) w3 (B,H) b3 (B).
 * Spline variant: cubic Hermite tables T, dT (n_el^2, G, B) on r = i*dr (face/model.py:383-418).
 * radial_bwd: dvec[e] += u * sum_b dphi[e,b] * dphidr[e,b]. */
int facek_radial_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx,
                     int32_t n_el, double rc, int32_t nb, int32_t H, int32_t B, const void* w1, const void* b1,
                     const void* pair, const void* w2, const void* b2, const void* w3, const void* b3, void* phi,
                     void* dphidr, int64_t E, void* stream);
/* Wide outputs (B > 32: the CP form's B + 4C radials, face/model.py:449; the non-factorised block's 4C or 8C,
 * face/model.py:130) run a CUDA-core kernel that keeps both hidden layers in registers.
 * facek_radial_fwd runs fp32 with H = 64, B in {16, 32}, nb <= 16 on the tcgen05 tensor cores (fp32 accuracy through
 * the 3-term tf32 split); fp64 and other shapes on the CUDA cores. The two explicit variants below pick one path;
 * they have no reference counterpart (the reference has a single PyTorch path, face/model.py:465-469) and exist so
 * that callers and tests can compare the paths. facek_radial_tc_fwd is fp32 only and returns FACEK_EINVAL for
 * shapes it does not cover. */
int facek_radial_simt_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx,
                          int32_t n_el, double rc, int32_t nb, int32_t H, int32_t B, const void* w1, const void* b1,
                          const void* pair, const void* w2, const void* b2, const void* w3, const void* b3, void* phi,
                          void* dphidr, int64_t E, void* stream);
int facek_radial_tc_fwd(const float* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx, int32_t n_el,
                        double rc, int32_t nb, int32_t H, int32_t B, const float* w1, const float* b1,
                        const float* pair, const float* w2, const float* b2, const float* w3, const float* b3,
                        float* phi, float* dphidr, int64_t E, void* stream);
/* Dense fp32 GEMM on the tcgen05 tensor cores for the channel maps (face/model.py:502-534 mix / tmix / proj,
 * :324-339 output MLP and gate; the reference calls torch.nn.Linear there):
 *   C[M, N] (beta ? += : =) A[M, K] . W[K, N] (+ bias[N]),  fp32 accuracy through the 3-term tf32 split, each
 *   32-wide K chunk accumulated separately and the chunk partials summed in fp32 with round-to-nearest.
 * W is packed once into an image of facek_gemm_image_floats(K, N) floats by facek_gemm_pack (W[k, n] at
 * W[k*stride_k + n*stride_n], so a transposed view packs W^T for the adjoint). A, C row-major with leading
 * dimensions lda, ldc; K, N, lda, ldc multiples of 4 and A, C, image 16-byte aligned (FACEK_EINVAL otherwise).
 * No reference counterpart as a C entry point. */
int64_t facek_gemm_image_floats(int64_t K, int64_t N);
int facek_gemm_pack(const float* W, int64_t K, int64_t N, int64_t stride_k, int64_t stride_n, float* image,
                    void* stream);
int facek_gemm_tc(const float* A, int64_t M, int64_t K, int64_t lda, const float* image, int64_t N,
                  const float* bias, float* C, int64_t ldc, int32_t beta, void* stream);
/* The same GEMM on a concatenated input and/or into a split output, without the concatenation in memory (the
 * reference concatenates the passes' moment sets with torch.cat before each projection, face/model.py:209):
 *   [C1 | C2] (beta ? += : =) [A1 | A2] . W (+ bias).
 * A1 is M x K1 (lda1), A2 is M x (K - K1) (lda2), K1 a multiple of 32; A2 = NULL means K1 = K. C1 is M x N1 (ldc1),
 * C2 is M x (N - N1) (ldc2), N1 a multiple of 32; C2 = NULL means N1 = N. Each block follows facek_gemm_tc's rules
 * on widths, strides and alignment. The image is the one packed for the full K x N. */
int facek_gemm_tc_split(const float* A1, int64_t lda1, int64_t K1, const float* A2, int64_t lda2, int64_t M,
                        int64_t K, const float* image, int64_t N, const float* bias, float* C1, int64_t ldc1,
                        int64_t N1, float* C2, int64_t ldc2, int32_t beta, void* stream);
/* Status of the tensor-core kernels (no reference counterpart): bit 0 set when a kernel gave up waiting for its
 * MMAs (bounded wait) and returned early with its outputs incomplete. Synchronises the device; clear != 0 resets. */
int facek_tc_status(int32_t* status, int32_t clear);
int facek_radial_spline_fwd(int dtype, const void* vec, const int32_t* ei, const int32_t* ej, const int32_t* zidx,
                            int32_t n_el, double rc, int32_t G, double dr, int32_t B, const void* T, const void* dT,
                            void* phi, void* dphidr, int64_t E, void* stream);
int facek_radial_bwd(int dtype, const void* vec, const void* dphi, const void* dphidr, int32_t B, void* dvec,
                     int32_t accumulate, int64_t E, void* stream);

/* Edge messages with directional terms (face/model.py:473-494), factorised as
 * msg[e, k] = sum_{c<nc} Y[e, c] * (TJ[c, ej, k] + TI[c, ei, k])   (TI may be NULL),
 * TJ/TI (nc, N, K) per-atom tables built from msg(h), dir_mix and the pvt/pmt projections.
 * Backward: dY[e, c] (+)= ..., dTI (row-local sums) and dTJ (reverse gather), no atomics. */
int facek_edge_msg_fwd(int dtype, const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ,
                       const void* TI, int32_t nc, int32_t K, void* msg, int64_t N, int64_t E, void* stream);
int facek_edge_msg_bwd(int dtype, const void* Y, const int32_t* ei, const int32_t* ej, const void* TJ,
                       const void* TI, const void* dmsg, const int32_t* row_ptr, const int32_t* rev, int32_t nc,
                       int32_t K, void* dY, int32_t accumulate, void* dTJ, void* dTI, int64_t N, int64_t E,
                       void* stream);

/* Transport sums (face/model.py:514-533 with the constant maps :342-362) written per edge:
 * T_o[i, b, kd] = sum_m phi[m,b] * f_o(u_m, Gt[:, ej_m, kd]),  f = [V | M u | M | sym(u (x) V)]  (18 outputs),
 * Gt (9, N, Kd) = [V(3) | M sym(6)] of the transport channels.  DT holds two planes back to back:
 * plane 1 (3, N, 2, B*Kd) = [V_a, (M u)_a] and plane 2 (6, N, 2, B*Kd) = [M_s, sym(u V)_s], so that
 * (3, N, 2*B*Kd) and (6, N, 2*B*Kd) are the contiguous inputs of tmix1 / tmix2 (columns (t, b, kd)).
 * Backward: the two plane gradients dT1, dT2; writes dphi (E,B), dvec (E,3) (+= when accumulate), and dGt via the
 * per-edge scratch dGt_edge (E,9,Kd) reduced by the reverse gather. */
int facek_transport_fwd(int dtype, const void* phi, const void* vec, const int32_t* ej, const void* Gt,
                        const int32_t* row_ptr, void* DT, int64_t N, int32_t B, int32_t Kd, void* stream);
int facek_transport_bwd(int dtype, const void* phi, const void* vec, const int32_t* ej, const void* Gt,
                        const void* dT1, const void* dT2, const int32_t* row_ptr, const int32_t* rev, void* dphi,
                        void* dvec, int32_t accumulate, void* dGt_edge, void* dGt, int64_t N, int64_t E, int32_t B,
                        int32_t Kd, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Smooth PME (face-mlip face/electrostatics.py:34-77) and the Gaussian real-space term (:91-92, :125-127).
 * inv: the 3x3 inverse cell (row-major, as torch.linalg.inv(cell)); mesh (n0*n1*n2) must be zeroed by the
 * caller before spread.  spectrum: the half spectrum of rfftn(mesh), (n0, n1, n2/2+1) complex; green writes
 * energy[0] += 1/(2V) sum_k G(k) B(k) |F(k)|^2 (accumulated in double; zero it first) and
 * conv = G*B*F * (n0 n1 n2 / V) so that irfftn(conv) is the mesh potential dE/dQ.  bmod: |b(m)|^-2 per axis
 * concatenated (n0 + n1 + n2).  gather: dq[i] = scale sum W phi, dpos[i] = scale q_i sum grad W phi.
 * Real space: e_row[i] = 1/2 q_i sum_{e in row i} q_j K(r_e); the adjoint takes the per-row upstream g_row.
 * r_cut > 0 drops edges with r >= r_cut (a neighbour list built with a skin and reused across MD steps gives the
 * same sum as a fresh list at the model cutoff); r_cut <= 0 keeps every edge, as the reference does with its pairs.
 */
int facek_pme_spread(int dtype, const void* pos, const void* q, int64_t N, const double* inv, int32_t n0,
                     int32_t n1, int32_t n2, void* mesh, void* stream);
int facek_pme_green(int dtype, const void* spectrum, int32_t n0, int32_t n1, int32_t n2, const double* inv,
                    double gp, double volume, const void* bmod, double* energy, void* conv, void* stream);
int facek_pme_gather(int dtype, const void* pos, const void* q, int64_t N, const double* inv, int32_t n0,
                     int32_t n1, int32_t n2, const void* potential, double scale, void* dq, void* dpos,
                     void* stream);
int facek_coulomb_real_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* q,
                           double gamma, double gp, double r_cut, int64_t N, void* e_row, void* stream);
int facek_coulomb_real_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* q,
                           double gamma, double gp, double r_cut, const void* g_row, int64_t N, void* dvec,
                           int32_t accumulate, void* dq, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Per-channel Cartesian density of the CP form (face/model.py:496-502, FactorBlock cp=True) and of the
 * non-factorised MomentBlock (face/model.py:160-187): D[x, i, c] = sum_{e in row i} Y[e,x] R[e, l(x), c] m[e, c],
 * D component-major (20, N, C).  R: per-(rank, channel) radial functions, envelope included, at column r_off of rows
 * of stride ldr (the radial output row: CP keeps its B transport radials in columns 0..B-1); m (E, C) the edge
 * message.  The adjoint takes G = dL/dD and writes dR at the same columns (other columns untouched), dm and dY.
 */
int facek_cp_density_fwd(int dtype, const void* Y, const void* R, int64_t ldr, int32_t r_off, const void* m,
                         const int32_t* row_ptr, int64_t N, int32_t C, void* D, void* stream);
int facek_cp_density_bwd(int dtype, const void* Y, const void* R, int64_t ldr, int32_t r_off, const void* m,
                         const void* G, const int32_t* ei, const int32_t* row_ptr, int64_t N, int64_t E, int32_t C,
                         void* dR, void* dm, void* dY, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Readout elementwise kernels (face/model.py:331-339): LayerNorm over rows of W <= 768 features with constant affine
 * weights (nn.LayerNorm: biased variance, y = (x - mean) / sqrt(var + eps) * w + b); the forward stores mean and
 * 1/std per row for the adjoint dx = rstd (g w - mean(g w) - xhat mean(g w xhat)).  SiLU y = x sigmoid(x) and its
 * adjoint.
 */
int facek_layer_norm_fwd(int dtype, const void* x, const void* w, const void* b, double eps, int64_t N, int32_t W,
                         void* y, void* mean, void* rstd, void* stream);
int facek_layer_norm_bwd(int dtype, const void* x, const void* w, const void* g, const void* mean, const void* rstd,
                         int64_t N, int32_t W, void* dx, void* stream);
int facek_silu_fwd(int dtype, const void* x, void* y, int64_t n, void* stream);
int facek_silu_bwd(int dtype, const void* x, const void* g, void* dx, int64_t n, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Pair physics terms, per CSR row over a symmetric neighbour list (vec from facek_edge_vec of that list).
 * ZBL (face/model.py:538-554, the "zbl" term): e_row[i] = 1/2 sum_{e in row i} KE Zi Zj / r phi(r/a) s(r),
 *   a = 0.46850 / (Zi^0.23 + Zj^0.23), phi the universal 4-exponential screening, s the quintic switch from 1 at
 *   r_in to 0 at r_out (reference r_in = 0.6, r_out = 1.2 A); Z = atomic numbers (int32).  The adjoint writes
 *   dvec[e] (+)= g_row[i] / 2 dE/dr u for the row's own edges.
 * Dispersion (face/dispersion.py:36-48, the "disp" term) over the long-range pair list (face/datasets.py:53-55):
 *   e_row[i] = sum_{e in row i} -1/2 sqrt(C6_i C6_j) / (d^6 + R0^6) s(d), R0 = A[0] (r0_i + r0_j)/2 + A[1]
 *   (A = softplus of the learned a1, a2, on the device), s the quintic switch from 1 at r_long - 2 to 0 at r_long.
 *   C6 (N) is the environment-modulated per-atom coefficient and r0 (N) the per-atom vdW radius.  The adjoint
 *   writes dvec[e] (+)= g_row[i] de/dd u and dC6[i] = sum_{e in row i} (g_i + g_j) e_ij / (2 C6_i).
 */
int facek_zbl_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z,
                  double r_in, double r_out, int64_t N, void* e_row, void* stream);
int facek_zbl_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const int32_t* Z,
                  double r_in, double r_out, const void* g_row, int64_t N, void* dvec, int32_t accumulate,
                  void* stream);
int facek_disp_fwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6,
                   const void* r0, const void* A, double r_long, int64_t N, void* e_row, void* stream);
int facek_disp_bwd(int dtype, const void* vec, const int32_t* row_ptr, const int32_t* ej, const void* C6,
                   const void* r0, const void* A, double r_long, const void* g_row, int64_t N, void* dvec,
                   int32_t accumulate, void* dC6, void* stream);

#ifdef __cplusplus
}
#endif
#endif
