"""FACE energy+force engine on libfacek.so.

Each edge- and node-level hot op is a torch.autograd.Function over one C-ABI kernel pair (forward + analytic
backward); torch autograd only sequences them and sums their gradient contributions. In fp32 the channel-mixing
GEMMs run on the library's tcgen05 GEMM with weights packed once per model (Dense); fp64 uses torch matmul.
The forward follows face-mlip's FACE.forward / FactorBlock pass by pass
(face/model.py:665-695, :310-339, :460-534, :204-308); the layouts differ where that removes copies:

Every multi-component per-atom tensor is stored component-major, (components, N, channels), so each rank block
is one contiguous (k_l*N, channels) GEMM operand and no autograd slice ever zero-fills a full-size gradient:
  D            (20, N, B*K) density, rank blocks D[0:1] D[1:4] D[4:10] D[10:20]
  A_l          (k_l, N, C)  (the reference keeps (N, C, k_l) and transposes around every Linear)
  y_l          (k_l, N, 3C) projections, read in place by the node kernel; V (3,N,C), Ms (6,N,C)
  messages     msg[e] = sum_{c<nc} Y[e,c] (TJ[c,j] + TI[c,i]) with per-atom tables TJ/TI (nc, N, K) that fold msg(h),
               the dir_mix weights and the Y2 weights [1,1,1,2,2,2] (face/model.py:473-494 re-associated)
  transport    two planes (3, N, 2*B*Kd) and (6, N, 2*B*Kd), columns (t, b, kd); tmix1/tmix2 columns permuted
               once to that order (face/model.py:525-533)
"""
import math
import os

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib
from .neighbors import graph_from_padded

KE = 14.399645                                      # face/electrostatics.py:20
Y2W = (1.0, 1.0, 1.0, 2.0, 2.0, 2.0)                # face/cartesian.py:81
RANK = [(0, 1), (1, 4), (4, 10), (10, 20)]
# density adjoint of the fp32 B=16 K=32 shape on the tensor cores (facek_density_msg_tc_xm_bwd) instead of the
# lane-per-edge CUDA-core kernel (facek_density_msg_xm_bwd)
DENSITY_ADJOINT_TC = os.environ.get("FACEK_DENSITY_ADJOINT", "simt") == "tc"


def _p(t):
    return _lib.ptr(t)


def _tag(t):
    return _lib.dtype_tag(t)


# ============================================================================================ edge Functions
class EdgeVec(torch.autograd.Function):
    """vec[e] = pos[ej] - pos[ei] + shift[e]; adjoint = the atomic-free force gather."""

    @staticmethod
    def forward(ctx, pos, gr):
        pos = pos.detach().contiguous()
        E = gr["ei"].numel()
        vec = torch.empty(E, 3, dtype=pos.dtype, device=pos.device)
        _lib.call("facek_edge_vec", _tag(pos), _p(pos), _p(gr["ei"]), _p(gr["ej"]), _p(gr["shift"]), _p(vec), E,
                  _lib.stream())
        ctx.gr = gr
        ctx.N = pos.shape[0]
        return vec

    @staticmethod
    def backward(ctx, dvec):
        dvec = dvec.contiguous()
        dpos = torch.empty(ctx.N, 3, dtype=dvec.dtype, device=dvec.device)
        _lib.call("facek_edge_vec_bwd", _tag(dvec), _p(dvec), _p(ctx.gr["row_ptr"]), _p(ctx.gr["rev"]), ctx.N,
                  _p(dpos), _lib.stream())
        return dpos, None


class EdgeSym(torch.autograd.Function):
    """Y[e] = the 20 symmetric monomials of u = vec/|vec| (face/cartesian.py:34-46)."""

    @staticmethod
    def forward(ctx, vec):
        E = vec.shape[0]
        Y = torch.empty(E, 20, dtype=vec.dtype, device=vec.device)
        _lib.call("facek_edge_sym", _tag(vec), _p(vec), _p(Y), E, _lib.stream())
        ctx.save_for_backward(vec)
        return Y

    @staticmethod
    def backward(ctx, dY):
        (vec,) = ctx.saved_tensors
        dY = dY.contiguous()
        dvec = torch.empty_like(vec)
        _lib.call("facek_edge_sym_bwd", _tag(vec), _p(vec), _p(dY), _p(dvec), 0, vec.shape[0], _lib.stream())
        return dvec


class Radial(torch.autograd.Function):
    """phi = radial MLP (or spline) x envelope per edge; dphi/dr from forward-mode differentiation."""

    @staticmethod
    def forward(ctx, vec, gr, blk):
        E = vec.shape[0]
        B = blk.get("R", blk["B"])                 # radial outputs: B, or B + 4C (CP), or 4C / 8C (non-factorised)
        phi = torch.empty(E, B, dtype=vec.dtype, device=vec.device)
        dphidr = torch.empty_like(phi)
        if blk.get("spline") is not None:
            Tt, dTt, dr = blk["spline"]
            _lib.call("facek_radial_spline_fwd", _tag(vec), _p(vec), _p(gr["ei"]), _p(gr["ej"]), _p(gr["zidx"]),
                      blk["n_el"], blk["rc"], Tt.shape[1], dr, B, _p(Tt), _p(dTt), _p(phi), _p(dphidr), E,
                      _lib.stream())
        else:
            _lib.call("facek_radial_fwd", _tag(vec), _p(vec), _p(gr["ei"]), _p(gr["ej"]), _p(gr["zidx"]),
                      blk["n_el"], blk["rc"], blk["nb"], blk["H"], B, _p(blk["w1"]), _p(blk["b1"]), _p(blk["pair"]),
                      _p(blk["w2"]), _p(blk["b2"]), _p(blk["w3"]), _p(blk["b3"]), _p(phi), _p(dphidr), E,
                      _lib.stream())
        ctx.save_for_backward(vec, dphidr)
        return phi

    @staticmethod
    def backward(ctx, dphi):
        vec, dphidr = ctx.saved_tensors
        dphi = dphi.contiguous()
        dvec = torch.empty_like(vec)
        _lib.call("facek_radial_bwd", _tag(vec), _p(vec), _p(dphi), _p(dphidr), dphi.shape[1], _p(dvec), 0,
                  vec.shape[0], _lib.stream())
        return dvec, None, None


class EdgeMsg(torch.autograd.Function):
    """msg[e,k] = sum_{c<nc} Y[e,c] (TJ[ej,c,k] + TI[ei,c,k])."""

    @staticmethod
    def forward(ctx, Y, TJ, TI, gr):
        E = Y.shape[0]
        nc, N, K = TJ.shape
        TJ = TJ.contiguous()
        TI = TI.contiguous() if TI is not None else None
        msg = torch.empty(E, K, dtype=Y.dtype, device=Y.device)
        _lib.call("facek_edge_msg_fwd", _tag(Y), _p(Y), _p(gr["ei"]), _p(gr["ej"]), _p(TJ), _p(TI), nc, K, _p(msg),
                  N, E, _lib.stream())
        ctx.save_for_backward(Y, TJ, TI)
        ctx.gr = gr
        return msg

    @staticmethod
    def backward(ctx, dmsg):
        Y, TJ, TI = ctx.saved_tensors
        gr = ctx.gr
        nc, N, K = TJ.shape
        E = Y.shape[0]
        dmsg = dmsg.contiguous()
        dY = torch.empty_like(Y)
        dTJ = torch.empty_like(TJ)
        dTI = torch.empty_like(TI) if TI is not None else None
        _lib.call("facek_edge_msg_bwd", _tag(Y), _p(Y), _p(gr["ei"]), _p(gr["ej"]), _p(TJ), _p(TI), _p(dmsg),
                  _p(gr["row_ptr"]), _p(gr["rev"]), nc, K, _p(dY), 0, _p(dTJ), _p(dTI), N, E, _lib.stream())
        return dY, dTJ, dTI, None


class Density(torch.autograd.Function):
    """D[x, i, b*K+k] = sum_{e in row i} phi[e,b] msg[e,k] Y[e,x] (CSR rows), returned as the four rank blocks
    (k_l, N, B*K) of one (20, N, B*K) buffer."""

    @staticmethod
    def forward(ctx, phi, msg, Y, gr):
        N = gr["row_ptr"].numel() - 1
        B, K = phi.shape[1], msg.shape[1]
        D = torch.empty(20, N, B * K, dtype=phi.dtype, device=phi.device)
        _lib.call("facek_density_xm_fwd", _tag(phi), _p(phi), _p(msg), _p(Y), _p(D), N, B, K, _p(gr["row_ptr"]),
                  _lib.stream())
        ctx.save_for_backward(phi, msg, Y)
        ctx.gr = gr
        return tuple(D[a:b] for a, b in RANK)

    @staticmethod
    def backward(ctx, *dD):
        phi, msg, Y = ctx.saved_tensors
        N = ctx.gr["row_ptr"].numel() - 1
        B, K = phi.shape[1], msg.shape[1]
        G = [g.contiguous() if g is not None else torch.zeros(b - a, N, B * K, dtype=phi.dtype, device=phi.device)
             for g, (a, b) in zip(dD, RANK)]
        dphi, dmsg, dY = torch.empty_like(phi), torch.empty_like(msg), torch.empty_like(Y)
        _lib.call("facek_density_xm_bwd", _tag(phi), _p(phi), _p(msg), _p(Y), *[_p(g) for g in G], _p(dphi),
                  _p(dmsg), _p(dY), N, B, K, _p(ctx.gr["row_ptr"]), _lib.stream())
        return dphi, dmsg, dY, None


class DensityMsg(torch.autograd.Function):
    """Directional messages and the factorised density in one op: msg[e,k] = sum_{c<nc} Y[e,c] (TJ[c,ej,k] +
    TI[c,ei,k]), D[x, i, b*K+k] = sum_{e in row i} phi[e,b] msg[e,k] Y[e,x] (face/model.py:473-513).  The adjoint
    runs the density backward and the message part of dY in one kernel (facek_density_msg_xm_bwd), then the
    message-table adjoint (facek_edge_msg_bwd without dY).  Returns the four rank blocks of D."""

    @staticmethod
    def forward(ctx, phi, Y, TJ, TI, gr):
        E = Y.shape[0]
        nc, N, K = TJ.shape
        B = phi.shape[1]
        TJ = TJ.contiguous()
        TI = TI.contiguous() if TI is not None else None
        msg = torch.empty(E, K, dtype=Y.dtype, device=Y.device)
        _lib.call("facek_edge_msg_fwd", _tag(Y), _p(Y), _p(gr["ei"]), _p(gr["ej"]), _p(TJ), _p(TI), nc, K, _p(msg),
                  N, E, _lib.stream())
        D = torch.empty(20, N, B * K, dtype=phi.dtype, device=phi.device)
        _lib.call("facek_density_xm_fwd", _tag(phi), _p(phi), _p(msg), _p(Y), _p(D), N, B, K, _p(gr["row_ptr"]),
                  _lib.stream())
        ctx.save_for_backward(phi, msg, Y, TJ, TI)
        ctx.gr = gr
        return tuple(D[a:b] for a, b in RANK)

    @staticmethod
    def backward(ctx, *dD):
        phi, msg, Y, TJ, TI = ctx.saved_tensors
        gr = ctx.gr
        nc, N, K = TJ.shape
        E, B = phi.shape
        G = [g.contiguous() if g is not None else torch.zeros(b - a, N, B * K, dtype=phi.dtype, device=phi.device)
             for g, (a, b) in zip(dD, RANK)]
        dphi, dmsg, dY = torch.empty_like(phi), torch.empty_like(msg), torch.empty_like(Y)
        if DENSITY_ADJOINT_TC and phi.dtype == torch.float32 and B == 16 and K == 32:
            _lib.call("facek_density_msg_tc_xm_bwd", _p(phi), _p(msg), _p(Y), *[_p(g) for g in G], _p(TJ), _p(TI),
                      _p(gr["ei"]), _p(gr["ej"]), nc, _p(dphi), _p(dmsg), _p(dY), N, E, B, K, _p(gr["row_ptr"]),
                      _lib.stream())
        else:
            _lib.call("facek_density_msg_xm_bwd", _tag(phi), _p(phi), _p(msg), _p(Y), *[_p(g) for g in G], _p(TJ),
                      _p(TI), _p(gr["ei"]), _p(gr["ej"]), nc, _p(dphi), _p(dmsg), _p(dY), N, E, B, K,
                      _p(gr["row_ptr"]), _lib.stream())
        dTJ = torch.empty_like(TJ)
        dTI = torch.empty_like(TI) if TI is not None else None
        _lib.call("facek_edge_msg_bwd", _tag(Y), _p(Y), _p(gr["ei"]), _p(gr["ej"]), _p(TJ), _p(TI), _p(dmsg),
                  _p(gr["row_ptr"]), _p(gr["rev"]), nc, K, None, 0, _p(dTJ), _p(dTI), N, E, _lib.stream())
        return dphi, dY, dTJ, dTI, None


class CPDensity(torch.autograd.Function):
    """Per-channel density D[x, i, c] = sum_{e in row i} Y[e,x] R[e, l(x), c] m[e, c] of the CP form and the
    non-factorised block (face/model.py:496-502, :182-187): R = columns r_off .. r_off + 4C of the radial output phi
    (envelope included), m (E, C) the edge message.  Returns the four rank blocks (k_l, N, C) of one (20, N, C)
    buffer; the adjoint returns a full-width dphi whose other columns are zero."""

    @staticmethod
    def forward(ctx, Y, phi, r_off, m, gr):
        N = gr["row_ptr"].numel() - 1
        C = m.shape[1]
        phi, m = phi.contiguous(), m.contiguous()
        D = torch.empty(20, N, C, dtype=phi.dtype, device=phi.device)
        _lib.call("facek_cp_density_fwd", _tag(phi), _p(Y), _p(phi), phi.shape[1], r_off, _p(m), _p(gr["row_ptr"]), N,
                  C, _p(D), _lib.stream())
        ctx.save_for_backward(Y, phi, m)
        ctx.r_off, ctx.gr = r_off, gr
        return tuple(D[a:b] for a, b in RANK)

    @staticmethod
    def backward(ctx, *dD):
        Y, phi, m = ctx.saved_tensors
        gr = ctx.gr
        N = gr["row_ptr"].numel() - 1
        E, C = m.shape
        G = torch.cat([g if g is not None else torch.zeros(b - a, N, C, dtype=phi.dtype, device=phi.device)
                       for g, (a, b) in zip(dD, RANK)], 0).contiguous()
        dphi = torch.zeros_like(phi)
        dm, dY = torch.empty_like(m), torch.empty_like(Y)
        _lib.call("facek_cp_density_bwd", _tag(phi), _p(Y), _p(phi), phi.shape[1], ctx.r_off, _p(m), _p(G),
                  _p(gr["ei"]), _p(gr["row_ptr"]), N, E, C, _p(dphi), _p(dm), _p(dY), _lib.stream())
        return dY, dphi, None, dm, None


def moment_transport(phi, Y, Vt, Mt, gr, C):
    """Rank-1 and rank-2 transport sums of the non-factorised block (face/model.py:188-201), per channel:
    A1[:, i] = sum_e Rt0 V_j + Rt1 M_j u,  A2[:, i] = sum_e Rt2 M_j + Rt3 sym(u V_j), with Rt = phi[:, 4C:8C]
    (envelope included) and V (3, N, C), M (6, N, C) the projected previous-pass tensors (symmetric storage
    xx yy zz xy xz yz).  Written with torch gathers and index_add (this form is not on the benchmark path)."""
    ei, ej = gr["ei"].long(), gr["ej"].long()
    E = ei.numel()
    N = gr["row_ptr"].numel() - 1
    Rt = phi[:, 4 * C:8 * C].reshape(E, 4, C).transpose(0, 1)                        # (4, E, C)
    u = Y[:, 1:4].t()[..., None]                                                      # (3, E, 1)
    Vj, Mj = Vt[:, ej], Mt[:, ej]                                                     # (3|6, E, C)
    xx, yy, zz, xy, xz, yz = Mj.unbind(0)
    Mu = torch.stack([xx * u[0] + xy * u[1] + xz * u[2], xy * u[0] + yy * u[1] + yz * u[2],
                      xz * u[0] + yz * u[1] + zz * u[2]])
    uV = u * Vj
    suv = torch.cat([uV, 0.5 * torch.stack([u[0] * Vj[1] + u[1] * Vj[0], u[0] * Vj[2] + u[2] * Vj[0],
                                            u[1] * Vj[2] + u[2] * Vj[1]])], 0)
    t1 = Rt[0] * Vj + Rt[1] * Mu                                                      # (3, E, C)
    t2 = Rt[2] * Mj + Rt[3] * suv                                                     # (6, E, C)
    A1 = torch.zeros(3, N, C, dtype=phi.dtype, device=phi.device).index_add(1, ei, t1)
    A2 = torch.zeros(6, N, C, dtype=phi.dtype, device=phi.device).index_add(1, ei, t2)
    return A1, A2


class Transport(torch.autograd.Function):
    """Transport sums as two planes (3, N, 2*B*Kd) [V, M u] and (6, N, 2*B*Kd) [M, sym(u V)], Gt (9, N, Kd)."""

    @staticmethod
    def forward(ctx, phi, vec, Gt, gr):
        N = gr["row_ptr"].numel() - 1
        B, Kd = phi.shape[1], Gt.shape[2]
        Gt = Gt.contiguous()
        DT = torch.empty(9 * N * 2 * B * Kd, dtype=phi.dtype, device=phi.device)
        _lib.call("facek_transport_fwd", _tag(phi), _p(phi), _p(vec), _p(gr["ej"]), _p(Gt), _p(gr["row_ptr"]),
                  _p(DT), N, B, Kd, _lib.stream())
        ctx.save_for_backward(phi, vec, Gt)
        ctx.gr = gr
        h = 3 * N * 2 * B * Kd
        return DT[:h].view(3, N, 2 * B * Kd), DT[h:].view(6, N, 2 * B * Kd)

    @staticmethod
    def backward(ctx, dT1, dT2):
        phi, vec, Gt = ctx.saved_tensors
        gr = ctx.gr
        N = gr["row_ptr"].numel() - 1
        E = phi.shape[0]
        B, Kd = phi.shape[1], Gt.shape[2]
        z = lambda k: torch.zeros(k, N, 2 * B * Kd, dtype=phi.dtype, device=phi.device)
        dT1 = dT1.contiguous() if dT1 is not None else z(3)
        dT2 = dT2.contiguous() if dT2 is not None else z(6)
        dphi = torch.empty_like(phi)
        dvec = torch.empty_like(vec)
        dGe = torch.empty(E, 9, Kd, dtype=phi.dtype, device=phi.device)
        dGt = torch.empty_like(Gt)
        _lib.call("facek_transport_bwd", _tag(phi), _p(phi), _p(vec), _p(gr["ej"]), _p(Gt), _p(dT1), _p(dT2),
                  _p(gr["row_ptr"]), _p(gr["rev"]), _p(dphi), _p(dvec), 0, _p(dGe), _p(dGt), N, E, B, Kd,
                  _lib.stream())
        return dphi, dvec, dGt, None


class BcastMul(torch.autograd.Function):
    """x (J, N, C) * s (N, C) broadcast over the J components (face/model.py:183-186 moment scaling, :277-295 gates);
    s may be a column slice of a wider (N, lds) row."""

    @staticmethod
    def forward(ctx, x, s):
        J, N, C = x.shape
        x = x.contiguous()
        if s.stride(1) != 1 or s.stride(0) < C:
            s = s.contiguous()
        out = torch.empty_like(x)
        _lib.call("facek_bcast_mul_fwd", _tag(x), _p(x), _p(s), _p(out), J, N, C, s.stride(0), _lib.stream())
        ctx.save_for_backward(x if ctx.needs_input_grad[1] else None, s)
        return out

    @staticmethod
    def backward(ctx, g):
        x, s = ctx.saved_tensors
        J, N, C = g.shape
        g = g.contiguous()
        dx = torch.empty_like(g)
        ds = torch.empty(N, C, dtype=g.dtype, device=g.device) if x is not None else None
        _lib.call("facek_bcast_mul_bwd", _tag(g), _p(g), _p(x) if x is not None else None, _p(s), _p(dx),
                  _p(ds) if ds is not None else None, J, N, C, s.stride(0), _lib.stream())
        return dx, ds


class NodeAlgebraEngine(torch.autograd.Function):
    """Invariant families + gated products from the (N, k_l, 3C) projections."""

    @staticmethod
    def forward(ctx, y0, y1, y2, y3, a, b, eq, max_body):
        _, N, C3 = y1.shape
        C = C3 // 3
        ys = [y.contiguous() for y in (y0, y1, y2, y3)]
        inv9 = torch.empty(N, 9 * C, dtype=y1.dtype, device=y1.device)
        V = torch.empty(3, N, C, dtype=y1.dtype, device=y1.device) if eq else y1.new_zeros(0)
        Ms = torch.empty(6, N, C, dtype=y1.dtype, device=y1.device) if eq else y1.new_zeros(0)
        _lib.call("facek_node_engine_fwd", _tag(y1), *[_p(y) for y in ys], _p(a), _p(b), _p(inv9),
                  _p(V) if eq else None, _p(Ms) if eq else None, N, C, int(eq), int(max_body), _lib.stream())
        ctx.save_for_backward(*ys)
        ctx.a, ctx.b, ctx.eq, ctx.max_body = a, b, eq, max_body
        if not eq:
            ctx.mark_non_differentiable(V, Ms)
        return inv9, V, Ms

    @staticmethod
    def backward(ctx, g9, gV, gMs):
        ys = ctx.saved_tensors
        _, N, C3 = ys[1].shape
        C = C3 // 3
        g9 = g9.contiguous() if g9 is not None else torch.zeros(N, 9 * C, dtype=ys[1].dtype, device=ys[1].device)
        if ctx.eq:
            gV = gV.contiguous() if gV is not None else torch.zeros(3, N, C, dtype=g9.dtype, device=g9.device)
            gMs = gMs.contiguous() if gMs is not None else torch.zeros(6, N, C, dtype=g9.dtype, device=g9.device)
        dys = [torch.empty_like(y) for y in ys]
        _lib.call("facek_node_engine_bwd", _tag(g9), *[_p(y) for y in ys], _p(ctx.a), _p(ctx.b), _p(g9),
                  _p(gV) if ctx.eq else None, _p(gMs) if ctx.eq else None, *[_p(d) for d in dys], N, C, int(ctx.eq),
                  int(ctx.max_body), _lib.stream())
        return (*dys, None, None, None, None)


class CoulombReal(torch.autograd.Function):
    """e_row[i] = 1/2 q_i sum_{e in row i} q_j (erf(r/gamma) - erf(r/gp))/r (face/electrostatics.py:91-92,125-127).
    A graph built with a skin (reused across MD steps) carries "coul_cut" = the model cutoff, so that the sum runs
    over the same pairs as a fresh list; other graphs sum over every edge, as the reference does."""

    @staticmethod
    def forward(ctx, vec, q, gr, gamma, gp):
        N = q.shape[0]
        q = q.contiguous()
        e_row = torch.empty_like(q)
        cut = float(gr.get("coul_cut") or 0.0)
        _lib.call("facek_coulomb_real_fwd", _tag(q), _p(vec), _p(gr["row_ptr"]), _p(gr["ej"]), _p(q), gamma, gp, cut,
                  N, _p(e_row), _lib.stream())
        ctx.save_for_backward(vec, q)
        ctx.gr, ctx.gamma, ctx.gp, ctx.cut = gr, gamma, gp, cut
        return e_row

    @staticmethod
    def backward(ctx, g_row):
        vec, q = ctx.saved_tensors
        g_row = g_row.contiguous()
        dvec = torch.empty_like(vec)
        dq = torch.empty_like(q)
        _lib.call("facek_coulomb_real_bwd", _tag(q), _p(vec), _p(ctx.gr["row_ptr"]), _p(ctx.gr["ej"]), _p(q),
                  ctx.gamma, ctx.gp, ctx.cut, _p(g_row), q.shape[0], _p(dvec), 0, _p(dq), _lib.stream())
        return dvec, dq, None, None, None


class ZBLTerm(torch.autograd.Function):
    """Per-atom ZBL energy e_row[i] = 1/2 sum_{e in row i} E_zbl(r_e; Z_i, Z_j) (face/model.py:544-554)."""

    @staticmethod
    def forward(ctx, vec, gr, Z32, r_in, r_out):
        N = gr["row_ptr"].numel() - 1
        e_row = torch.empty(N, dtype=vec.dtype, device=vec.device)
        _lib.call("facek_zbl_fwd", _tag(vec), _p(vec), _p(gr["row_ptr"]), _p(gr["ej"]), _p(Z32), r_in, r_out, N,
                  _p(e_row), _lib.stream())
        ctx.save_for_backward(vec, Z32)
        ctx.gr, ctx.r = gr, (r_in, r_out)
        return e_row

    @staticmethod
    def backward(ctx, g_row):
        vec, Z32 = ctx.saved_tensors
        dvec = torch.empty_like(vec)
        _lib.call("facek_zbl_bwd", _tag(vec), _p(vec), _p(ctx.gr["row_ptr"]), _p(ctx.gr["ej"]), _p(Z32), *ctx.r,
                  _p(g_row.contiguous()), g_row.shape[0], _p(dvec), 0, _lib.stream())
        return dvec, None, None, None, None


class DispTerm(torch.autograd.Function):
    """Per-atom dispersion energy over the long-range list (face/dispersion.py:36-48):
    e_row[i] = sum_{e in row i} -1/2 sqrt(C6_i C6_j) / (d^6 + R0_ij^6) s(d)."""

    @staticmethod
    def forward(ctx, vec, C6, lr, r0, A, r_long):
        N = lr["row_ptr"].numel() - 1
        C6 = C6.contiguous()
        e_row = torch.empty(N, dtype=vec.dtype, device=vec.device)
        _lib.call("facek_disp_fwd", _tag(vec), _p(vec), _p(lr["row_ptr"]), _p(lr["ej"]), _p(C6), _p(r0), _p(A), r_long,
                  N, _p(e_row), _lib.stream())
        ctx.save_for_backward(vec, C6, r0, A)
        ctx.lr, ctx.r_long = lr, r_long
        return e_row

    @staticmethod
    def backward(ctx, g_row):
        vec, C6, r0, A = ctx.saved_tensors
        dvec, dC6 = torch.empty_like(vec), torch.empty_like(C6)
        _lib.call("facek_disp_bwd", _tag(vec), _p(vec), _p(ctx.lr["row_ptr"]), _p(ctx.lr["ej"]), _p(C6), _p(r0),
                  _p(A), ctx.r_long, _p(g_row.contiguous()), g_row.shape[0], _p(dvec), 0, _p(dC6), _lib.stream())
        return dvec, dC6, None, None, None, None


def zbl_term(P, gr, geo):
    """ZBL over the model's neighbour list (face/model.py:544-554)."""
    z = P["zbl"]
    return ZBLTerm.apply(geo["vec"], gr, gr["Z"].to(torch.int32).contiguous(), z["r_in"], z["r_out"])


def disp_term(P, gr, pos, h):
    """Dispersion over the long-range list gr["lr"] (face/dispersion.py:36-48); C6_i = c6(Z_i) exp(w . h_i)."""
    c = P["disp"]
    lr = gr.get("lr")
    if lr is None:
        raise KeyError("the dispersion term needs a long-range pair list: build_graph(..., rc_long=...) or the "
                       "reference graph keys lr_i / lr_j / lr_shift")
    Z = gr["Z"]
    C6 = c["c6"][Z] * torch.exp(_layer(c["w"], h).squeeze(-1))
    r0 = c["r0"][Z].contiguous()
    vec = EdgeVec.apply(pos, lr)
    return DispTerm.apply(vec, C6, lr, r0, c["A"], c["r_long"])


_BMOD = {}


def bspline_modulus2(n, dtype, device):
    """|b(m)|^-2 of the order-4 Euler spline (Essmann et al. 1995; face/electrostatics.py:44-51)."""
    key = (n, dtype, str(device))
    if key not in _BMOD:
        m = np.arange(n, dtype=np.float64)
        ang = 2 * np.pi * m[:, None] * np.arange(3)[None] / n
        w = np.array([1 / 6, 4 / 6, 1 / 6])
        den = (w * np.cos(ang)).sum(-1) ** 2 + (w * np.sin(ang)).sum(-1) ** 2
        _BMOD[key] = torch.as_tensor(1.0 / np.maximum(den, 1e-10), dtype=dtype, device=device)
    return _BMOD[key]


class PMERecip(torch.autograd.Function):
    """Smooth-PME reciprocal energy of one periodic structure (face/electrostatics.py:54-77): spread -> cuFFT
    (torch.fft.rfftn) -> Green's function x |b|^2 (energy + convolved spectrum) -> irfftn -> gather."""

    @staticmethod
    def forward(ctx, pos, q, inv, vol, gp, mesh):
        """inv: the cell's inverse (host float64 3x3), vol: its volume (host float), both fixed at graph build."""
        pos, q = pos.detach().contiguous(), q.detach().contiguous()
        n0, n1, n2 = mesh
        invd = _lib.doubles(inv.reshape(-1))
        grid = torch.zeros(n0 * n1 * n2, dtype=pos.dtype, device=pos.device)
        _lib.call("facek_pme_spread", _tag(pos), _p(pos), _p(q), pos.shape[0], invd, n0, n1, n2, _p(grid),
                  _lib.stream())
        spec = torch.view_as_real(torch.fft.rfftn(grid.view(n0, n1, n2))).contiguous()
        bmod = torch.cat([bspline_modulus2(n, pos.dtype, pos.device) for n in (n0, n1, n2)])
        energy = torch.zeros(1, dtype=torch.float64, device=pos.device)
        conv = torch.empty_like(spec)
        _lib.call("facek_pme_green", _tag(pos), _p(spec), n0, n1, n2, invd, float(gp), vol, _p(bmod), _p(energy),
                  _p(conv), _lib.stream())
        pot = torch.fft.irfftn(torch.view_as_complex(conv), s=(n0, n1, n2)).contiguous()
        ctx.save_for_backward(pos, q, pot)
        ctx.inv, ctx.mesh = inv, mesh
        return energy.to(pos.dtype)[0]

    @staticmethod
    def backward(ctx, g):
        pos, q, pot = ctx.saved_tensors
        n0, n1, n2 = ctx.mesh
        potg = (pot * g).contiguous()
        dq = torch.empty_like(q)
        dpos = torch.empty_like(pos)
        _lib.call("facek_pme_gather", _tag(pos), _p(pos), _p(q), pos.shape[0], _lib.doubles(ctx.inv.reshape(-1)), n0,
                  n1, n2, _p(potg), 1.0, _p(dq), _p(dpos), _lib.stream())
        return dpos, dq, None, None, None, None


class SpreadMesh(torch.autograd.Function):
    """Order-4 B-spline charge spreading onto the full PME mesh (the spreading step of face/electrostatics.py:54-77)
    as a differentiable op: forward facek_pme_spread, adjoint facek_pme_gather of the mesh gradient (dq and dpos).
    Used by the slab-distributed PME, where the mesh leaves this op through collectives and FFTs."""

    @staticmethod
    def forward(ctx, pos, q, cell64, mesh):
        pos, q = pos.detach().contiguous(), q.detach().contiguous()
        n0, n1, n2 = mesh
        inv = np.linalg.inv(cell64)         # host-side 3x3 (the slab PME passes a constant cell)
        grid = torch.zeros(n0 * n1 * n2, dtype=pos.dtype, device=pos.device)
        _lib.call("facek_pme_spread", _tag(pos), _p(pos), _p(q), pos.shape[0], _lib.doubles(inv.reshape(-1)), n0,
                  n1, n2, _p(grid), _lib.stream())
        ctx.save_for_backward(pos, q)
        ctx.inv, ctx.mesh = inv, mesh
        return grid

    @staticmethod
    def backward(ctx, g):
        pos, q = ctx.saved_tensors
        n0, n1, n2 = ctx.mesh
        dq = torch.empty_like(q)
        dpos = torch.empty_like(pos)
        _lib.call("facek_pme_gather", _tag(pos), _p(pos), _p(q), pos.shape[0], _lib.doubles(ctx.inv.reshape(-1)), n0,
                  n1, n2, _p(g.contiguous()), 1.0, _p(dq), _p(dpos), _lib.stream())
        return dpos, dq, None, None


class LayerNormK(torch.autograd.Function):
    """nn.LayerNorm over the last dimension with constant affine weights (face/model.py:140-141, :331) on the
    library's warp-per-row kernel; the adjoint uses the per-row mean and 1/std saved by the forward."""

    @staticmethod
    def forward(ctx, x, w, b, eps):
        x = x.contiguous()
        N, W = x.shape
        y = torch.empty_like(x)
        mean = torch.empty(N, dtype=x.dtype, device=x.device)
        rstd = torch.empty_like(mean)
        _lib.call("facek_layer_norm_fwd", _tag(x), _p(x), _p(w), _p(b), float(eps), N, W, _p(y), _p(mean), _p(rstd),
                  _lib.stream())
        ctx.save_for_backward(x, w, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, g):
        x, w, mean, rstd = ctx.saved_tensors
        dx = torch.empty_like(x)
        _lib.call("facek_layer_norm_bwd", _tag(x), _p(x), _p(w), _p(g.contiguous()), _p(mean), _p(rstd), x.shape[0],
                  x.shape[1], _p(dx), _lib.stream())
        return dx, None, None, None


class SiLUK(torch.autograd.Function):
    """x * sigmoid(x) on the library's elementwise kernel (the readout MLP's activations, face/model.py:73-77)."""

    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        y = torch.empty_like(x)
        _lib.call("facek_silu_fwd", _tag(x), _p(x), _p(y), x.numel(), _lib.stream())
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        _lib.call("facek_silu_bwd", _tag(x), _p(x), _p(g.contiguous()), _p(dx), x.numel(), _lib.stream())
        return dx


def silu(x):
    return SiLUK.apply(x) if x.is_cuda else F.silu(x)


# ============================================================================================ channel GEMMs
class Dense:
    """A constant (K, N) fp32 weight packed for the tensor-core GEMM (facek_gemm_tc): the split image of W for
    y = x @ W (+ b) and of W^T for the adjoint dx = dy @ W^T.  K and N must be multiples of 4."""

    def __init__(self, W, b=None):
        assert W.dtype == torch.float32 and W.is_cuda and W.dim() == 2
        self.K, self.N = W.shape
        self.b = None if b is None else b.contiguous()
        self.img = self._pack(W, self.K, self.N, W.stride(0), W.stride(1))
        self.imgT = self._pack(W, self.N, self.K, W.stride(1), W.stride(0))

    @staticmethod
    def _pack(W, K, N, sk, sn):
        n = _lib.lib().facek_gemm_image_floats(K, N)
        img = torch.empty(n, dtype=torch.float32, device=W.device)
        _lib.call("facek_gemm_pack", _p(W), K, N, sk, sn, _p(img), _lib.stream())
        return img

    @staticmethod
    def ok(K, N):
        return K % 4 == 0 and N % 4 == 0


def _gemm(x2, img, K, N, bias, out, beta):
    _lib.call("facek_gemm_tc", _p(x2), x2.shape[0], K, x2.stride(0), _p(img), N, _p(bias), _p(out), out.stride(0),
              beta, _lib.stream())


def _rows(x, K):
    """x as (rows, K) with unit column stride and 16-byte aligned rows (a copy only when the view is not)."""
    x2 = x.reshape(-1, K)
    return x2 if (x2.stride(1) == 1 and x2.stride(0) % 4 == 0 and x2.data_ptr() % 16 == 0) else x2.contiguous()


class TCMatmul(torch.autograd.Function):
    """y = x1 @ W1 (+ x2 @ W2) (+ b1) on the tensor cores; inputs (..., K_i), output (..., N); weights constant."""

    @staticmethod
    def forward(ctx, x1, d1, x2, d2):
        lead = x1.shape[:-1]
        a1 = _rows(x1, d1.K)
        y = torch.empty(a1.shape[0], d1.N, dtype=x1.dtype, device=x1.device)
        _gemm(a1, d1.img, d1.K, d1.N, d1.b, y, 0)
        if x2 is not None:
            _gemm(_rows(x2, d2.K), d2.img, d2.K, d2.N, d2.b, y, 1)
        ctx.d1, ctx.d2, ctx.lead = d1, d2, lead
        ctx.has2 = x2 is not None
        return y.view(*lead, d1.N)

    @staticmethod
    def backward(ctx, dy):
        d1, d2 = ctx.d1, ctx.d2
        g = _rows(dy, d1.N)
        dx1 = torch.empty(g.shape[0], d1.K, dtype=dy.dtype, device=dy.device)
        _gemm(g, d1.imgT, d1.N, d1.K, None, dx1, 0)
        dx2 = None
        if ctx.has2:
            dx2 = torch.empty(g.shape[0], d2.K, dtype=dy.dtype, device=dy.device)
            _gemm(g, d2.imgT, d2.N, d2.K, None, dx2, 0)
            dx2 = dx2.view(*ctx.lead, d2.K)
        return dx1.view(*ctx.lead, d1.K), None, dx2, None


class TCMatmulCat(torch.autograd.Function):
    """y = [x1 | x2] @ W on the tensor cores without the concatenation in memory (facek_gemm_tc_split): the GEMM
    takes each 32-wide K chunk from x1 or x2 where they lie, and the adjoint writes dx1 and dx2 as two tensors, so
    neither the forward's concatenation nor the adjoint's slice copies exist.  x1 (..., K1) with K1 a multiple of
    32, x2 (..., K - K1), D packed for the full (K, N) weight; weights constant."""

    @staticmethod
    def forward(ctx, x1, x2, d):
        lead, K1 = x1.shape[:-1], x1.shape[-1]
        a1, a2 = _rows(x1, K1), _rows(x2, d.K - K1)
        M = a1.shape[0]
        y = torch.empty(M, d.N, dtype=x1.dtype, device=x1.device)
        _lib.call("facek_gemm_tc_split", _p(a1), a1.stride(0), K1, _p(a2), a2.stride(0), M, d.K, _p(d.img), d.N,
                  _p(d.b), _p(y), y.stride(0), d.N, None, 0, 0, _lib.stream())
        ctx.d, ctx.K1, ctx.lead = d, K1, lead
        return y.view(*lead, d.N)

    @staticmethod
    def backward(ctx, dy):
        d, K1 = ctx.d, ctx.K1
        g = _rows(dy, d.N)
        M = g.shape[0]
        dx1 = torch.empty(M, K1, dtype=dy.dtype, device=dy.device)
        dx2 = torch.empty(M, d.K - K1, dtype=dy.dtype, device=dy.device)
        _lib.call("facek_gemm_tc_split", _p(g), g.stride(0), d.N, None, 0, M, d.N, _p(d.imgT), d.K, None, _p(dx1),
                  dx1.stride(0), K1, _p(dx2), dx2.stride(0), 0, _lib.stream())
        return dx1.view(*ctx.lead, K1), dx2.view(*ctx.lead, d.K - K1), None


def mm_cat(xs, W, D=None):
    """torch.cat(xs, -1) @ W; two fp32 inputs whose first width is a multiple of 32 take the split GEMM."""
    if (D is not None and len(xs) == 2 and xs[0].dtype == torch.float32 and xs[0].shape[-1] % 32 == 0
            and xs[1].shape[-1] % 4 == 0):
        return TCMatmulCat.apply(xs[0], xs[1], D)
    return mm(_cat(xs, -1), W, D)


def mm(x, W, D=None, x2=None, W2=None, D2=None):
    """x @ W (+ x2 @ W2): the tensor-core GEMM when packed weights D are given (fp32), else torch."""
    if D is not None and x.dtype == torch.float32 and (x2 is None or D2 is not None):
        return TCMatmul.apply(x, D, x2, D2)
    y = x @ W
    return y if x2 is None else y + x2 @ W2


def linear(x, W, D=None):
    """F.linear with (weight, bias) W, through the packed GEMM when available."""
    if D is not None and x.dtype == torch.float32:
        return TCMatmul.apply(x, D, None, None)
    return F.linear(x, W[0], W[1])


# ============================================================================================ weights
def _lin(model, mod, dtype, dev):
    w = mod.weight.detach()
    if model.unit:
        w = w * w.shape[1] ** -0.5
    b = mod.bias.detach().to(dtype=dtype, device=dev).contiguous() if getattr(mod, "bias", None) is not None else None
    return w.to(dtype=dtype, device=dev).contiguous(), b


def prepare(model, dtype, dev):
    """Effective (unit-scaled), detached, layout-ready weights; cached until the model changes."""
    key = (dtype, str(dev), model.max_body, tuple(id(s) for s in model.spline))
    if model._prepared is not None and model._prepared["key"] == key:
        return model._prepared
    for k, v in model.switches.items():
        if v:
            raise NotImplementedError(k)
    P = {"key": key}
    d = lambda t: t.detach().to(dtype=dtype, device=dev).contiguous()
    P["zmap"] = model.zmap.to(dev)
    P["embed"] = d(model.embed.weight)
    P["E0"], P["scale"], P["avg_nb"] = d(model.E0), d(model.scale), d(model.avg_nb)
    n_el = len(model.elements)
    blocks = []
    for t, blk in enumerate(model.blocks):
        C, B, K, Kd = blk.C, blk.B, blk.Km, blk.Kd
        q = {"B": B, "K": K, "Kd": Kd, "C": C, "n_el": n_el, "rc": float(model.rc), "nb": model.n_basis,
             "directional": blk.directional, "transport": blk.transport, "eq_in": blk.eq_in, "eq_out": blk.eq_out}
        q["w1"], q["b1"] = _lin(model, blk.rad_in, dtype, dev)
        q["H"] = q["w1"].shape[0]
        q["pair"] = d(blk.pair.weight)
        q["w2"], q["b2"] = _lin(model, blk.radial[0], dtype, dev)
        q["w3"], q["b3"] = _lin(model, blk.radial[2], dtype, dev)
        q["R"] = q["w3"].shape[0]
        sp = model.spline[t]
        q["spline"] = None if sp is None else (d(sp[0]), d(sp[1]), float(sp[2]))
        q["form"] = blk.form
        tc = dtype == torch.float32 and torch.device(dev).type == "cuda"
        pk = (lambda W, b=None: Dense(W, b) if tc and Dense.ok(*W.shape) else None)
        if blk.form != "moment":
            q["msg_w"], q["msg_b"] = _lin(model, blk.msg, dtype, dev)
            q["msgD"] = pk(q["msg_w"].t(), q["msg_b"])
            # (B*K, C) factorised, (C, C) CP
            q["mixT"] = [(_lin(model, blk.mix[l], dtype, dev)[0]).t().contiguous() for l in range(4)]
            q["mixD"] = [pk(W) for W in q["mixT"]]
        q["projT"] = [(_lin(model, blk.proj[l], dtype, dev)[0]).t().contiguous() for l in range(4)]    # (cin, 3C)
        q["projD"] = [pk(W) for W in q["projT"]]
        q["elem_scale"] = d(blk.elem_scale.weight)
        q["norm"] = blk.norm_kind
        if blk.norm_kind == "layer":
            q["ln_w"], q["ln_b"], q["ln_eps"] = d(blk.norm.weight), d(blk.norm.bias), blk.norm.eps
        elif blk.norm_kind == "affine":
            q["ln_w"], q["ln_b"] = d(blk.norm.w), d(blk.norm.b)
        q["out"] = [_lin(model, blk.out[i], dtype, dev) for i in (0, 2, 4)]
        q["outD"] = [pk(w.t(), b) for w, b in q["out"]]
        # first readout layer split by input block [inv (9C) | h (C) | lognorms (4, zero here)]: two GEMMs into one
        # output instead of a concatenated input (face/model.py:335)
        w0, b0 = q["out"][0]
        q["out0_inv"], q["out0_h"] = w0[:, :9 * C].t().contiguous(), w0[:, 9 * C:10 * C].t().contiguous()
        q["out0_invD"], q["out0_hD"] = pk(q["out0_inv"], b0), pk(q["out0_h"])
        # last readout layer (2C -> C + 1) zero-padded to a multiple of 4 output columns for the tensor-core GEMM
        w4, b4 = q["out"][2]
        n4 = (w4.shape[0] + 3) // 4 * 4
        q["out4_pad"] = torch.zeros(w4.shape[1], n4, dtype=dtype, device=dev)
        q["out4_pad"][:, :w4.shape[0]] = w4.t()
        q["out4_b"] = torch.zeros(n4, dtype=dtype, device=dev)
        q["out4_b"][:w4.shape[0]] = b4
        q["out4D"] = pk(q["out4_pad"], q["out4_b"])
        if blk.eq_out:
            q["vpath"], q["mpath"] = d(blk.vpath), d(blk.mpath)
            q["gate"] = _lin(model, blk.gate, dtype, dev)
            q["gateD"] = pk(q["gate"][0].t(), q["gate"][1])
        if blk.directional:
            wd, bd = _lin(model, blk.dir_mix, dtype, dev)                                 # (K, 4Kd)
            q["dir"] = [wd[:, i * Kd:(i + 1) * Kd].t().contiguous() for i in range(4)]       # each (Kd, K)
            q["dir_b"] = bd
            if blk.form == "moment":                      # face/model.py:147-150: pv, pm (cprev -> Kd)
                q["pvtT"] = _lin(model, blk.pv, dtype, dev)[0].t().contiguous()             # (cprev, Kd)
                q["pmtT"] = _lin(model, blk.pm, dtype, dev)[0].t().contiguous()
            else:
                q["pvtT"] = _lin(model, blk.pvt, dtype, dev)[0].t().contiguous()            # (cprev, nt*Kd)
                q["pmtT"] = _lin(model, blk.pmt, dtype, dev)[0].t().contiguous()
            q["pvtD"], q["pmtD"] = pk(q["pvtT"]), pk(q["pmtT"])
            q["y2w"] = torch.tensor(Y2W, dtype=dtype, device=dev)[:, None, None]
            # the y2 weights folded into per-component maps: (Md @ w) * y2w == Md @ (w * y2w), one batched matmul
            q["dir_y2"] = [q["y2w"] * q["dir"][i] for i in (1, 3)]                            # each (6, Kd, K)
        if blk.transport and blk.form == "moment":        # face/model.py:151-153: tv, tm (cprev -> C)
            q["tvT"] = _lin(model, blk.tv, dtype, dev)[0].t().contiguous()
            q["tmT"] = _lin(model, blk.tm, dtype, dev)[0].t().contiguous()
        elif blk.transport:
            for name in ("tmix1", "tmix2"):
                w = _lin(model, getattr(blk, name), dtype, dev)[0]                           # (C, B*2*Kd) cols (b,t,kd)
                q[name + "T"] = w.view(C, B, 2, Kd).permute(0, 2, 1, 3).reshape(C, 2 * B * Kd).t().contiguous()
                q[name + "D"] = pk(q[name + "T"])
            # channel map and transport map of ranks 1, 2 as one layer on [D_l | T_l] (facek_gemm_tc_split)
            q["mixtT"] = {l: torch.cat([q["mixT"][l], q["tmix%dT" % l]], 0) for l in (1, 2)}
            q["mixtD"] = {l: pk(q["mixtT"][l]) for l in (1, 2)}
        blocks.append(q)
    P["blocks"] = blocks
    P["terms"] = list(model.terms.keys())
    if "zbl" in model.terms:
        tm = model.terms["zbl"]
        P["zbl"] = {"r_in": float(tm.r_in), "r_out": float(tm.r_out)}
    if "disp" in model.terms:
        tm = model.terms["disp"]
        P["disp"] = {"w": _lin(model, tm.w, dtype, dev), "c6": d(tm.c6), "r0": d(tm.r0), "r_long": float(tm.r_long),
                     # softplus(a1), softplus(a2) of face/dispersion.py:44, kept on the device (no host read)
                     "A": F.softplus(torch.stack([tm.a1.detach(), tm.a2.detach()])).to(dtype=dtype, device=dev)}
    if "coulomb" in model.terms:
        tm = model.terms["coulomb"]
        P["coulomb"] = {"h0": _lin(model, tm.head[0], dtype, dev), "h2": _lin(model, tm.head[2], dtype, dev),
                        "gamma": float(tm.gamma), "gp": float(tm.gp), "mesh": tm.mesh}
    model._prepared = P
    return P


def build_spline(model, t, n_grid=4096):
    """Cubic Hermite tables of block t's radial MLP per element pair (face/model.py:393-405), evaluated once with
    torch on the model's device: T (P, G, B) values, dT (P, G, B) exact r-derivatives, grid step rc/(G-1)."""
    blk = model.blocks[t]
    dev, dt = blk.rad_in.weight.device, blk.rad_in.weight.dtype
    rc = float(model.rc)
    r = torch.linspace(0, rc, n_grid, device=dev, dtype=dt).clamp_min(1e-4)
    pairs = blk.pair.weight.detach()
    lin = lambda mod, x: F.linear(x, mod.weight.detach() * (mod.weight.shape[1] ** -0.5 if model.unit else 1.0),
                                  mod.bias.detach() if mod.bias is not None else None)
    with torch.enable_grad():
        rr = r[None].expand(pairs.shape[0], -1).clone().requires_grad_(True)
        freq = torch.arange(1, model.n_basis + 1, device=dev, dtype=dt) * math.pi / rc
        x = rr / rc
        env = (1 - 28 * x ** 6 + 48 * x ** 7 - 21 * x ** 8) * (x < 1)
        bes = torch.sin(freq * rr[..., None]) / rr[..., None] * math.sqrt(2 / rc)
        h = F.silu(lin(blk.rad_in, bes * env[..., None]) + pairs[:, None, :])
        T = lin(blk.radial[2], F.silu(lin(blk.radial[0], h)))
        dT = torch.stack([torch.autograd.grad(T[..., b].sum(), rr, retain_graph=True)[0] for b in range(T.shape[-1])],
                         -1)
    return (T.detach().contiguous(), dT.detach().contiguous(), rc / (n_grid - 1))


# ============================================================================================ forward
def _layer(W, x):
    w, b = W
    return F.linear(x, w, b)


def channel_moments(q, gr, geo, h, A_sets, eq, phi):
    """Moments of the CP form and of the non-factorised block (face/model.py:496-502 with :533-534; :160-201): the
    per-channel edge message (h_j or msg(h)_j, plus the directional term as per-atom tables), the per-channel
    density, the C -> C channel map (CP only) and the transport increments, before the element scaling."""
    N, C, B, Kd = h.shape[0], q["C"], q["B"], q["Kd"]
    vec, Y = geo["vec"], geo["Y"]
    cp = q["form"] == "cp"
    base = F.linear(h, q["msg_w"], q["msg_b"]) if cp else h                        # (N, C)
    Gt = tsrc = None
    if q["directional"]:
        src1 = eq[0] if q["eq_in"] else _cat([A[1] for A in A_sets], 2)        # (3, N, cprev)
        src2 = eq[1] if q["eq_in"] else _cat([A[2] for A in A_sets], 2)        # (6, N, cprev)
        Vb = src1 @ q["pvtT"]
        Mb = src2 @ q["pmtT"]
        Vd, Md = Vb[..., :Kd], Mb[..., :Kd]
        w1, w2, w3, w4 = q["dir"]
        w2y, w4y = q["dir_y2"]
        TJ = torch.cat([(base + q["dir_b"])[None], Vd @ w1, Md @ w2y], 0)            # (10, N, C)
        TI = torch.cat([torch.zeros_like(base)[None], Vd @ w3, Md @ w4y], 0)
        m = EdgeMsg.apply(Y, TJ, TI, gr)                                               # (E, C)
        if q["transport"]:
            if cp:
                Gt = torch.cat([Vb[..., Kd:], Mb[..., Kd:]], 0)                        # (9, N, Kd)
            else:
                tsrc = (src1 @ q["tvT"], src2 @ q["tmT"])                              # (3|6, N, C)
    else:
        m = EdgeMsg.apply(Y, base[None], None, gr)
    D = CPDensity.apply(Y, phi, B if cp else 0, m, gr)                                # 4 x (k_l, N, C)
    if cp:
        tpl = {}
        if Gt is not None:
            T1, T2 = Transport.apply(phi[:, :B].contiguous(), vec, Gt, gr)
            tpl = {1: (T1, q["tmix1T"], q["tmix1D"]), 2: (T2, q["tmix2T"], q["tmix2D"])}
        return [_mix(q, l, D[l], tpl) for l in range(4)]
    A = list(D)
    if tsrc is not None:
        A1, A2 = moment_transport(phi, Y, tsrc[0], tsrc[1], gr, C)
        A[1] = A[1] + A1
        A[2] = A[2] + A2
    return A


def _mix(q, l, Dl, tpl):
    """Channel map of rank l, plus the transport map where the pass has one: one GEMM on [D_l | T_l] when the
    stacked weight is packed, else D_l @ mix (+ T_l @ tmix)."""
    t = tpl.get(l)
    if t is not None and q.get("mixtD", {}).get(l) is not None:
        return mm_cat([Dl, t[0]], q["mixtT"][l], q["mixtD"][l])
    return mm(Dl, q["mixT"][l], q["mixD"][l], *(t or (None, None, None)))


def _cat(ts, dim):
    """torch.cat, without the copy when there is one tensor."""
    return ts[0] if len(ts) == 1 else torch.cat(ts, dim)


def block_forward(P, t, gr, geo, h, A_sets, eq):
    """One interaction pass (face/model.py:310-339 with FactorBlock.moments :460-534, or the CP form and the
    non-factorised MomentBlock.moments :160-201)."""
    q = P["blocks"][t]
    N = h.shape[0]
    C, B, K, Kd = q["C"], q["B"], q["K"], q["Kd"]
    vec, Y = geo["vec"], geo["Y"]
    phi = Radial.apply(vec, gr, q)                                                   # (E, B), env included
    s = geo["consts"].get(("scale", t))
    if s is None:                                # elem_scale[Z] / avg_nb as (4, N, C): fixed by graph and weights
        s = (q["elem_scale"][geo["zidx"]] / geo["avg_nb"]).view(N, 4, C).transpose(0, 1).contiguous()
        geo["consts"][("scale", t)] = s
    if q["form"] != "factor":
        A = channel_moments(q, gr, geo, h, A_sets, eq, phi)
        A = [BcastMul.apply(A[l], s[l]) for l in range(4)]
        return _invariants_readout(P, q, h, A_sets, A, N)
    msgtab = linear(h, (q["msg_w"], q["msg_b"]), q["msgD"])                          # (N, K)
    Gt = None
    if q["directional"]:
        src1 = eq[0] if q["eq_in"] else _cat([A[1] for A in A_sets], 2)        # (3, N, cprev)
        src2 = eq[1] if q["eq_in"] else _cat([A[2] for A in A_sets], 2)        # (6, N, cprev)
        Vb = mm(src1, q["pvtT"], q["pvtD"])                                           # (3, N, nt*Kd)
        Mb = mm(src2, q["pmtT"], q["pmtD"])                                           # (6, N, nt*Kd)
        Vd, Md = Vb[..., :Kd], Mb[..., :Kd]
        w1, w2, w3, w4 = q["dir"]
        w2y, w4y = q["dir_y2"]
        TJ = torch.cat([(msgtab + q["dir_b"])[None], Vd @ w1, Md @ w2y], 0)                  # (10, N, K)
        TI = torch.cat([torch.zeros_like(msgtab)[None], Vd @ w3, Md @ w4y], 0)
        if q["transport"]:
            Gt = torch.cat([Vb[..., Kd:], Mb[..., Kd:]], 0)                           # (9, N, Kd)
        D = DensityMsg.apply(phi, Y, TJ, TI, gr)                                     # 4 x (k_l, N, B*K)
    else:
        D = DensityMsg.apply(phi, Y, msgtab[None], None, gr)
    tpl = {}
    if Gt is not None:
        T1, T2 = Transport.apply(phi, vec, Gt, gr)                                   # (3|6, N, 2*B*Kd)
        tpl = {1: (T1, q["tmix1T"], q["tmix1D"]), 2: (T2, q["tmix2T"], q["tmix2D"])}
    A = [_mix(q, l, D[l], tpl) for l in range(4)]                                    # (k_l, N, C)
    A = [BcastMul.apply(A[l], s[l]) for l in range(4)]
    return _invariants_readout(P, q, h, A_sets, A, N)


def _invariants_readout(P, q, h, A_sets, A, N):
    """Invariants, norm, readout and gated equivariant outputs of a pass (face/model.py:204-339)."""
    # invariants (face/model.py:204-270): projections straight into the node kernel's layout
    sets = A_sets + [A]
    ys = [mm_cat([a[l] for a in sets], q["projT"][l], q["projD"][l]) for l in range(4)]         # (k_l, N, 3C)
    a_w = q["vpath"] if q["eq_out"] else None
    b_w = q["mpath"] if q["eq_out"] else None
    inv, V, Ms = NodeAlgebraEngine.apply(*ys, a_w, b_w, q["eq_out"], P["max_body"])
    if q["norm"] == "layer" and inv.shape[1] <= 768:
        inv = LayerNormK.apply(inv, q["ln_w"], q["ln_b"], q["ln_eps"])
    elif q["norm"] == "layer":                            # rows wider than the kernel's register tile (C > 85)
        inv = F.layer_norm(inv, (inv.shape[1],), q["ln_w"], q["ln_b"], q["ln_eps"])
    elif q["norm"] == "affine":
        inv = inv * q["ln_w"] + q["ln_b"]
    # readout MLP on z = [inv | h | 0] (the reference's lognorm features are zero without momnorm, face/model.py:334)
    if q["out0_invD"] is not None and q["out0_hD"] is not None:
        o0 = TCMatmul.apply(inv, q["out0_invD"], h, q["out0_hD"])
    else:
        o0 = inv @ q["out0_inv"] + h @ q["out0_h"] + q["out"][0][1]
    o1 = linear(silu(o0), q["out"][1], q["outD"][1])
    if q["out4D"] is not None:
        o = TCMatmul.apply(silu(o1), q["out4D"], None, None)             # (N, C + 1 padded to a multiple of 4)
    else:
        o = linear(silu(o1), q["out"][2], None)
    eq_new = None
    if q["eq_out"]:
        gv, gm = linear(inv, q["gate"], q["gateD"]).chunk(2, dim=-1)
        eq_new = (BcastMul.apply(V, gv), BcastMul.apply(Ms, gm))
    return o[:, 0], h + o[:, 1:h.shape[1] + 1], A, eq_new


def seg_sum(x, batch, nstr):
    """Per-structure sums; a plain reduction when the batch holds one structure (an index_add of N atoms into one
    element serialises on atomics)."""
    if nstr == 1:
        return x.sum(0, keepdim=True)
    return torch.zeros(nstr, *x.shape[1:], dtype=x.dtype, device=x.device).index_add(0, batch, x)


def per_atom(v, batch, nstr):
    """Broadcast per-structure values to atoms (expand, whose adjoint is a reduction, for a single structure)."""
    if nstr == 1:
        return v.expand(batch.shape[0], *v.shape[1:])
    return v[batch]


def cell_meta(gr):
    """Host-side per-structure data of a graph: atom offsets, inverse cells, volumes (host and device), lattice
    lengths.  Graphs from build_graph carry it from construction; other graphs get it here once (one host read)."""
    meta = gr.get("meta")
    if meta is None:
        from .neighbors import structure_meta
        meta = structure_meta([int(n) for n in gr["natoms"].tolist()], gr["cell64"], gr["pos"].device)
        gr["meta"] = meta
    return meta


def coulomb_term(P, gr, geo, h, pos):
    """LatentCharges.forward, mode 'local' (face/electrostatics.py:132-176)."""
    c = P["coulomb"]
    chi, hard = _layer(c["h2"], F.silu(_layer(c["h0"], h))).unbind(-1)
    J = F.softplus(hard) + 0.1
    batch, nstr = gr["batch"], gr["nstr"]
    invJ = 1.0 / J
    num = seg_sum(chi * invJ, batch, nstr)
    den = seg_sum(invJ, batch, nstr)
    Q = gr["charge"].to(chi.dtype)
    mu = (Q + num) / den
    q = -(chi - per_atom(mu, batch, nstr)) * invJ
    gamma, gp = c["gamma"], c["gp"]
    natoms = gr["natoms"]
    if not all(gr["pbc"]):
        if any(gr["pbc"]):
            raise NotImplementedError("Coulomb term on a batch mixing periodic and non-periodic structures")
        # molecules: dense Gaussian-charge Coulomb inside each structure (face/electrostatics.py:178-198)
        d = torch.sqrt(((pos[:, None] - pos[None]) ** 2).sum(-1) + torch.eye(len(q), dtype=pos.dtype, device=pos.device))
        same = (batch[:, None] == batch[None, :]) & ~torch.eye(len(q), dtype=torch.bool, device=pos.device)
        A = torch.where(same, torch.erf(d / gamma) / d, torch.zeros_like(d))
        return chi * q + 0.5 * J * q * q + 0.5 * KE * q * (A @ q), q
    e_row = CoulombReal.apply(geo["vec"], q, gr, gamma, gp)
    e_real = seg_sum(e_row, batch, nstr)
    q2 = seg_sum(q * q, batch, nstr)
    qs = seg_sum(q, batch, nstr)
    # per-structure host data (atom offsets, inverse cells, volumes, PME meshes) was fixed when the graph was built,
    # so this loop launches kernels without reading anything back from the device (the reference's per-structure
    # loop, face/electrostatics.py:144-146, syncs on nonzero()/item())
    meta = cell_meta(gr)
    offs = meta["offs"]
    e_recip = []
    for s in range(nstr):
        mesh = c["mesh"]
        if mesh is None:                                       # face/electrostatics.py:56-58
            spacing = gp / 4.0
            mesh = tuple(max(8, int(math.ceil(float(L) / spacing))) for L in meta["lengths"][s])
        sl = slice(offs[s], offs[s + 1])
        e_recip.append(PMERecip.apply(pos[sl], q[sl], meta["inv"][s], meta["vol"][s], gp, tuple(mesh)))
    e_recip = torch.stack(e_recip)
    vol = meta["vol_t"].to(q.dtype)
    e_es = KE * (e_recip + e_real - q2 / (math.sqrt(math.pi) * gp) - 0.5 * math.pi * gp ** 2 / vol * qs ** 2)
    return chi * q + 0.5 * J * q * q + per_atom(e_es / natoms.to(q.dtype), batch, nstr), q


def _graph_consts(P, Z):
    """Per-graph constants of an evaluation: element indices (int64 and int32) and, filled in by the passes, the
    per-atom element scalings.  They depend only on the atomic numbers and the prepared weights, so they are kept
    for the most recent Z tensor (same object, unmodified) and rebuilt when the graph changes."""
    c = P.get("_graph_consts")
    if c is None or c[0] is not Z or c[1] != Z._version:
        zidx = P["zmap"][Z]
        c = (Z, Z._version, zidx, zidx.to(torch.int32).contiguous(), {})
        P["_graph_consts"] = c
    return c[2], c[3], c[4]


def local_energies(model, gr, pos, between=None):
    """Per-atom model energies (without physics terms) and final features h for positions `pos` (any
    differentiable tensor) on graph `gr` (face/model.py:665-686).

    between(t, h, A_sets, eq) -> (h, A_sets, eq), when given, runs after every pass but the last: the spatial
    decomposition replaces its ghost atoms' features there with their owners' (a halo exchange).  Layouts: h (N, C),
    each A_sets[k][l] (k_l, N, C), eq = (V (3, N, C), Ms (6, N, C)) or None."""
    dtype = model.embed.weight.dtype
    P = prepare(model, dtype, pos.device)
    P["max_body"] = model.max_body
    zidx, zidx32, consts = _graph_consts(P, gr["Z"])
    gr = dict(gr, zidx=zidx32)
    vec = EdgeVec.apply(pos, gr)
    Y = EdgeSym.apply(vec)
    geo = {"vec": vec, "Y": Y, "zidx": zidx, "avg_nb": P["avg_nb"], "consts": consts}
    h = P["embed"][zidx]
    e_at = P["E0"][zidx]
    A_sets, eq = [], None
    n = len(P["blocks"])
    for t in range(n):
        e, h, A, eq = block_forward(P, t, gr, geo, h, A_sets, eq)
        A_sets.append(A)
        e_at = e_at + P["scale"] * e
        if between is not None and t + 1 < n:
            h, A_sets, eq = between(t, h, A_sets, eq)
    return e_at, h, P, gr, geo


def face_forward(model, g, forces=True):
    """Energy (per structure), per-atom energy and forces for a graph dict (face/model.py:665-695).  `g` is either
    the engine's CSR graph (face_b200.neighbors.build_graph) or the reference's padded dict."""
    gr = g if "row_ptr" in g else graph_from_padded(g)
    pos = g["pos"]
    if not pos.is_cuda:
        raise RuntimeError("face_b200 runs on CUDA only (no CPU path)")
    dtype = model.embed.weight.dtype
    if pos.dtype != dtype:
        raise TypeError(f"positions are {pos.dtype}, model is {dtype}")
    if forces and not pos.requires_grad:
        pos.requires_grad_(True)
    with torch.set_grad_enabled(forces):
        e_at, h, P, gr, geo = local_energies(model, gr, pos)
        qv = None
        for name in P["terms"]:                          # face/model.py:686-687, in the model's term order
            if name == "coulomb":
                ea, qv = coulomb_term(P, gr, geo, h, pos)
            elif name == "zbl":
                ea = zbl_term(P, gr, geo)
            elif name == "disp":
                ea = disp_term(P, gr, pos, h)
            else:
                raise NotImplementedError(name)
            e_at = e_at + ea
        E = seg_sum(e_at, gr["batch"], gr["nstr"])
        out = {"energy": E.detach(), "atom_energy": e_at.detach()}
        if qv is not None:
            out["q"] = qv.detach()
        if forces:
            (grad,) = torch.autograd.grad(E.sum(), pos)
            out["forces"] = -grad
    return out
