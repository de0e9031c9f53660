"""Drop-in for face-mlip `face.node_kernel.node_algebra` (face/node_kernel.py:207-209).

    node_algebra(P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, eq=True) -> inv (N,C,8), V (N,C,3), Mf (N,C,3,3)

Symmetric storage in (P*,Q*,S*: (N,C,3|6|10)), path weights a, b (4,C).  Gradients for all tensors, with
da/db summed over atoms (face/node_kernel.py:204).  Runs libfacek.so's facek_node_fwd / facek_node_bwd.
"""
import torch

from . import _lib


class NodeAlgebra(torch.autograd.Function):
    @staticmethod
    def forward(ctx, P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, eq):
        ins = [P1, Q1, S1, P2, Q2, S2, P3, Q3]
        _lib.require_cuda(*ins, a, b)
        dt = P1.dtype if P1.dtype in (torch.float32, torch.float64) else torch.float32
        ins = [x.detach().to(dt).contiguous() for x in ins]
        a, b = a.detach().to(dt).contiguous(), b.detach().to(dt).contiguous()
        N, C = ins[0].shape[:2]
        inv = torch.empty(N, C, 8, device=P1.device, dtype=dt)
        V = torch.zeros(N, C, 3, device=P1.device, dtype=dt)
        Mf = torch.zeros(N, C, 3, 3, device=P1.device, dtype=dt)
        _lib.call("facek_node_fwd", _lib.dtype_tag(inv), *[_lib.ptr(x) for x in ins], _lib.ptr(a), _lib.ptr(b),
                  _lib.ptr(inv), _lib.ptr(V), _lib.ptr(Mf), N, C, int(bool(eq)), _lib.stream())
        ctx.save_for_backward(*ins, a, b)
        ctx.eq = bool(eq)
        return inv, V, Mf

    @staticmethod
    def backward(ctx, gI, gV, gM):
        *ins, a, b = ctx.saved_tensors
        N, C = ins[0].shape[:2]
        dev, dt = ins[0].device, ins[0].dtype
        gI = (gI if gI is not None else torch.zeros(N, C, 8, device=dev, dtype=dt)).to(dt).contiguous()
        gV = (gV if gV is not None else torch.zeros(N, C, 3, device=dev, dtype=dt)).to(dt).contiguous()
        gM = (gM if gM is not None else torch.zeros(N, C, 3, 3, device=dev, dtype=dt)).to(dt).contiguous()
        outs = [torch.empty_like(x) for x in ins]
        da = torch.zeros(N, C, 4, device=dev, dtype=dt)
        db = torch.zeros(N, C, 4, device=dev, dtype=dt)
        _lib.call("facek_node_bwd", _lib.dtype_tag(gI), *[_lib.ptr(x) for x in ins], _lib.ptr(a), _lib.ptr(b),
                  _lib.ptr(gI), _lib.ptr(gV), _lib.ptr(gM), *[_lib.ptr(x) for x in outs], _lib.ptr(da), _lib.ptr(db),
                  N, C, int(ctx.eq), _lib.stream())
        return (*outs, da.sum(0).t(), db.sum(0).t(), None)


def node_algebra(P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, eq=True):
    """P2,Q2,S2: (N,C,6) and P3,Q3: (N,C,10) symmetric components; a, b: (4,C)."""
    return NodeAlgebra.apply(P1, Q1, S1, P2, Q2, S2, P3, Q3, a, b, eq)
