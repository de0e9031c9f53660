"""Drop-in for face-mlip `face.kernels.factor_density` (face/kernels.py:170-172).

    factor_density(phi, msg, Y) -> D      (N,M,B), (N,M,K), (N,M,20) -> (N,20,B*K)
    D[i, x, b*K + k] = sum_m phi[i,m,b] * msg[i,m,k] * Y[i,m,x]

First-order differentiable.  Same argument meaning as the reference; unlike the reference (which always
casts to float32, face/kernels.py:140), float64 inputs are computed in float64.  Runs libfacek.so's
facek_density_fwd / facek_density_bwd on torch's current stream; CUDA tensors only.
"""
import torch

from . import _lib


def _dens_fwd(phi, msg, Y, row_ptr=None):
    N, M, B = phi.shape if row_ptr is None else (row_ptr.numel() - 1, 0, phi.shape[-1])
    K = msg.shape[-1]
    D = torch.empty(N, 20, B * K, device=phi.device, dtype=phi.dtype)
    _lib.call("facek_density_fwd", _lib.dtype_tag(phi), _lib.ptr(phi), _lib.ptr(msg), _lib.ptr(Y), _lib.ptr(D), N, M, B,
              K, _lib.ptr(row_ptr), _lib.stream())
    return D


def _dens_bwd(phi, msg, Y, G, row_ptr=None):
    N, M, B = phi.shape if row_ptr is None else (row_ptr.numel() - 1, 0, phi.shape[-1])
    K = msg.shape[-1]
    dphi, dmsg, dY = torch.empty_like(phi), torch.empty_like(msg), torch.empty_like(Y)
    _lib.call("facek_density_bwd", _lib.dtype_tag(phi), _lib.ptr(phi), _lib.ptr(msg), _lib.ptr(Y), _lib.ptr(G),
              _lib.ptr(dphi), _lib.ptr(dmsg), _lib.ptr(dY), N, M, B, K, _lib.ptr(row_ptr), _lib.stream())
    return dphi, dmsg, dY


class FactorDensity(torch.autograd.Function):
    @staticmethod
    def forward(ctx, phi, msg, Y):
        _lib.require_cuda(phi, msg, Y)
        dt = torch.promote_types(torch.promote_types(phi.dtype, msg.dtype), Y.dtype)
        if dt not in (torch.float32, torch.float64):
            dt = torch.float32
        phi, msg, Y = (x.detach().to(dt).contiguous() for x in (phi, msg, Y))
        if phi.shape[:2] != msg.shape[:2] or phi.shape[:2] != Y.shape[:2] or Y.shape[-1] != 20:
            raise ValueError(f"factor_density: shapes {tuple(phi.shape)} {tuple(msg.shape)} {tuple(Y.shape)}")
        ctx.save_for_backward(phi, msg, Y)
        return _dens_fwd(phi, msg, Y)

    @staticmethod
    def backward(ctx, G):
        phi, msg, Y = ctx.saved_tensors
        return _dens_bwd(phi, msg, Y, G.to(phi.dtype).contiguous())


def factor_density(phi, msg, Y):
    """(N,M,B), (N,M,K), (N,M,20) -> (N,20,B*K); first-order differentiable."""
    return FactorDensity.apply(phi, msg, Y)
