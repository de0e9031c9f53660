"""FACE energy+force engine for B200 (sm_100a).

Drop-in for face-mlip's `face.model.FACE` on the inference hot path `FACE.forward(g, forces=True)`
(face-mlip `face/model.py:558-695`): same constructor, same `state_dict` keys (checkpoints of the factorised,
CP and non-factorised forms load unchanged), same `set_*` / `fuse()` / `compile_radial()` switches (the ones the
engine does not implement raise), same graph-dict input and output dict ({"energy", "atom_energy", "forces"}),
physics terms coulomb, zbl and disp.

The edge-level work (geometry, radial basis x radial MLP, the factorised Cartesian density, directional
messages, transport sums, their analytic backward and the force gather) runs in the hand-written CUDA
kernels of libfacek.so behind a C ABI (face_b200._lib); in fp32 the node-level channel-mixing GEMMs run on the
library's tcgen05 tensor-core GEMM (fp64 uses torch matmul); the node invariant algebra runs in its own kernel.  There is no CPU path: the model refuses to run on a
device other than CUDA, and raises if the native library is missing.
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .params import BlockParams, Bessel, ChargeParams, DispParams, ZBLParams, seeded_state

BODY_ORDER = [2, 3, 3, 3, 4, 4, 4, 4, 5]          # face/model.py:246,268
RANK_SLICE = {0: slice(0, 1), 1: slice(1, 4), 2: slice(4, 10), 3: slice(10, 20)}
_UNSUPPORTED_SWITCHES = ("calib", "momnorm", "saturate", "standardise", "elem_proj", "eq_linear", "poly",
                         "transport3")


class FACE(nn.Module):
    def __init__(self, elements, C=64, n_basis=8, rc=5.0, n_passes=2, terms=(), radial_hidden=64, K_dir=16,
                 norm="layer", transport=False, eqmsg=False, factor=False, B=16, K=32, cp=False, unit=False):
        super().__init__()
        self.form = ("cp" if cp else "factor") if factor else "moment"      # face/model.py:568-569
        self.rc, self.C, self.n_passes, self.elements = rc, C, n_passes, list(elements)
        self.B, self.K, self.K_dir, self.n_basis = B, K, K_dir, n_basis
        self.transport, self.eqmsg, self.norm_kind = transport, eqmsg, norm
        self.unit = unit
        self.max_body = 5
        self.switches = {k: False for k in _UNSUPPORTED_SWITCHES}
        zmap = torch.full((119,), -1, dtype=torch.long)
        for k, z in enumerate(elements):
            zmap[z] = k
        self.register_buffer("zmap", zmap)
        n_el = len(elements)
        self.basis = Bessel(n_basis, rc)
        self.embed = nn.Embedding(n_el, C)
        self.blocks = nn.ModuleList([
            BlockParams(C, n_basis, t + 1, radial_hidden, n_el, K_dir, norm, transport,
                        eq_in=eqmsg and t > 0, eq_out=eqmsg and t < n_passes - 1, B=B, K=K, form=self.form)
            for t in range(n_passes)])
        self.register_buffer("E0", torch.zeros(n_el))
        self.register_buffer("scale", torch.tensor(1.0))
        self.register_buffer("avg_nb", torch.tensor(10.0))
        self.terms = nn.ModuleDict()
        for t in terms:                                  # face/model.py:580-590, evaluated in this order
            if t == "coulomb":
                self.terms[t] = ChargeParams(C)
            elif t == "zbl":
                self.terms[t] = ZBLParams()
            elif t == "disp":
                self.terms[t] = DispParams(C)
            elif t == "qeq":
                raise NotImplementedError("the 'qeq' term (LatentCharges mode 'full', an O(N^3) charge solve) is not "
                                          "implemented in the B200 engine")
            else:
                raise ValueError(t)
        self.spline = [None] * n_passes
        self._prepared = None

    # ---------------------------------------------------------------- reference switches (face/model.py:592-663)
    def _switch(self, name, on):
        if on:
            raise NotImplementedError(f"set_{name}(True) is not implemented in the B200 engine")
        return self

    def set_transport3(self, on=True):
        return self._switch("transport3", on)

    def set_poly_readout(self, on=True):
        return self._switch("poly", on)

    def set_elem_proj(self, on=True):
        return self._switch("elem_proj", on)

    def set_eq_linear(self, on=True):
        return self._switch("eq_linear", on)

    def set_calib(self, on=True, clip_c=10.0, keep_ln=False):
        return self._switch("calib", on)

    def set_momnorm(self, on=True, eps=1e-6):
        return self._switch("momnorm", on)

    def set_standardise(self, on=True):
        return self._switch("standardise", on)

    def set_saturation(self, on=True, scale=4.0):
        return self._switch("saturate", on)

    def set_max_body(self, n=5):
        self.max_body = n
        self._prepared = None
        return self

    def fuse(self, on=True):
        """Accepted for API compatibility: the engine always runs its CUDA kernels (there is no unfused path)."""
        return self

    def compile_radial(self, n_grid=4096, on=True):
        """Tabulate each block's radial MLP per element pair (cubic Hermite, face/model.py:644-655)."""
        self.spline = [None] * self.n_passes
        if on and self.form != "moment":               # the non-factorised block has no compiled radial
            for t in range(self.n_passes):
                self.spline[t] = ops.build_spline(self, t, n_grid)
        self._prepared = None
        return self

    def set_pme(self, gp=None, mesh=None):
        """Override the Coulomb term's Ewald width gp (= 1/alpha) and PME mesh (the reference hard-codes them,
        face/electrostatics.py:86 and :56-58)."""
        t = self.terms["coulomb"]
        if gp is not None:
            t.gp = gp
        t.mesh = tuple(mesh) if mesh is not None else None
        return self

    def seed_(self, seed, perturb=0.25):
        """Deterministic random-init weights (see face_b200.params.seeded_state)."""
        self.load_state_dict(seeded_state(self, seed, perturb), strict=False)
        self._prepared = None
        return self

    def load_state_dict(self, state, strict=True, assign=False):
        self._prepared = None
        return super().load_state_dict(state, strict=strict, assign=assign)

    def forward(self, g, forces=True, create_graph=False):
        if create_graph:
            raise NotImplementedError("second derivatives (training) are not provided by the B200 engine")
        return ops.face_forward(self, g, forces)
