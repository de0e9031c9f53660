"""Parameter layout of face-mlip's FACE model (same state_dict keys and shapes as the reference, so its
checkpoints of the three block forms load unchanged) and deterministic seeded weights.

Key layout follows face-mlip `face/model.py`:
  embed (Embedding n_el x C) :570 ; buffers zmap/E0/scale/avg_nb/basis.freq :564-578
  blocks.t (FactorBlock :421-458 over MomentBlock :99-158)
     rad_in, pair, radial.{0,2}, msg, mix.{0..3}, proj.{0..3}, elem_scale, pqs_gate, norm, out.{0,2,4},
     dir_mix/pvt/pmt (pass >= 2), tmix1/2/3 (transport), vpath/mpath/gate (equivariant out)
  terms.coulomb.head.{0,2} (LatentCharges :80-88)
"""
import zlib

import numpy as np
import torch
import torch.nn as nn

LINEAR_NAMES = ("rad_in", "radial.0", "radial.2", "msg", "dir_mix", "pvt", "pmt", "pv", "pm", "tv", "tm", "tmix1",
                "tmix2", "tmix3",
                "gate", "head.0", "head.2") + tuple(f"mix.{l}" for l in range(4)) + tuple(
    f"proj.{l}" for l in range(4)) + ("out.0", "out.2", "out.4")


def _mlp(sizes):
    layers = []
    for a, b in zip(sizes[:-1], sizes[1:]):
        layers += [nn.Linear(a, b), nn.SiLU()]
    return nn.Sequential(*layers[:-1])


class Bessel(nn.Module):
    def __init__(self, n, rc):
        super().__init__()
        self.rc, self.n = rc, n
        self.register_buffer("freq", torch.arange(1, n + 1) * torch.pi / rc)


class Affine(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.w = nn.Parameter(torch.ones(n))
        self.b = nn.Parameter(torch.zeros(n))


class BlockParams(nn.Module):
    """Parameters of one interaction pass (no compute here; see face_b200.model), in one of three forms:
      "factor"  FactorBlock, B radials x K-channel messages (face/model.py:421-458)
      "cp"      FactorBlock with cp=True: per-channel messages (K = C), B + 4C radials, C -> C channel maps
                (face/model.py:436-449)
      "moment"  the non-factorised MomentBlock: 4C (8C with transport) radials, neighbour features h_j as the
                message, no channel map, per-channel transport maps tv / tm (face/model.py:99-158)"""
    N_INV = 9

    def __init__(self, C, n_basis, n_sets, radial_hidden, n_el, K_dir, norm, transport, eq_in, eq_out, B, K,
                 form="factor"):
        super().__init__()
        self.form = form
        if form == "cp":
            K = C
        self.C, self.B, self.Km, self.Kd, self.n_el = C, B, K, K_dir, n_el
        self.eq_in, self.eq_out = eq_in, eq_out
        self.directional = n_sets > 1
        self.transport = transport and self.directional
        self.pqs_gate = nn.Embedding(n_el, 12 * C)
        self.register_buffer("mom_scale", torch.ones(4))
        self.register_buffer("eq_scale", torch.ones(2))
        self.register_buffer("inv_scale", torch.ones(self.N_INV))
        self.register_buffer("calibrated", torch.tensor(False))
        self.rad_in = nn.Linear(n_basis, radial_hidden)
        self.pair = nn.Embedding(n_el * n_el, radial_hidden)
        cin = C * n_sets
        self.proj = nn.ModuleList([nn.Linear(cin, 3 * C, bias=False) for _ in range(4)])
        self.elem_scale = nn.Embedding(n_el, 4 * C)
        self.out = _mlp([self.N_INV * C + C + 4, 2 * C, 2 * C, C + 1])
        self.norm_kind = norm
        if norm == "layer":
            self.norm = nn.LayerNorm(self.N_INV * C)
        elif norm == "affine":
            self.norm = Affine(self.N_INV * C)
        else:
            self.norm = nn.Identity()
        if eq_out:
            self.vpath = nn.Parameter(torch.ones(4, C))
            self.mpath = nn.Parameter(torch.ones(4, C))
            self.gate = nn.Linear(self.N_INV * C, 2 * C)
        cprev = C if eq_in else C * (n_sets - 1)
        if form == "moment":
            self.radial = _mlp([radial_hidden, radial_hidden, (8 if self.transport else 4) * C])
            if self.directional:
                self.pv = nn.Linear(cprev, K_dir, bias=False)
                self.pm = nn.Linear(cprev, K_dir, bias=False)
                self.dir_mix = nn.Linear(4 * K_dir, C)
            if self.transport:
                self.tv = nn.Linear(cprev, C, bias=False)
                self.tm = nn.Linear(cprev, C, bias=False)
            return
        self.radial = _mlp([radial_hidden, radial_hidden, B + (4 * C if form == "cp" else 0)])
        self.msg = nn.Linear(C, K)
        self.mix = nn.ModuleList([nn.Linear(C if form == "cp" else B * K, C, bias=False) for _ in range(4)])
        if self.directional:
            self.dir_mix = nn.Linear(4 * K_dir, K)
            nt = 2 if self.transport else 1
            self.pvt = nn.Linear(cprev, nt * K_dir, bias=False)
            self.pmt = nn.Linear(cprev, nt * K_dir, bias=False)
        if self.transport:
            self.tmix1 = nn.Linear(B * 2 * K_dir, C, bias=False)
            self.tmix2 = nn.Linear(B * 2 * K_dir, C, bias=False)
            self.tmix3 = nn.Linear(B * 2 * K_dir, C, bias=False)


class ChargeParams(nn.Module):
    """LatentCharges parameters (face/electrostatics.py:81-88)."""

    def __init__(self, C, sigma=0.5, rc_real=5.0, acc=3.5):
        super().__init__()
        self.head = nn.Sequential(nn.Linear(C, C), nn.SiLU(), nn.Linear(C, 2))
        self.sigma, self.gamma = sigma, 2 * sigma
        self.gp = max(rc_real / acc, 1.05 * self.gamma)
        self.kcut = 2 * acc / self.gp
        self.mesh = None            # None -> face-mlip's rule n = max(8, ceil(L / (gp/4)))


class ZBLParams(nn.Module):
    """The ZBL term (face/model.py:538-541): no parameters, inner and outer switching radii."""

    def __init__(self, r_in=0.6, r_out=1.2):
        super().__init__()
        self.r_in, self.r_out = r_in, r_out


# Tkatchenko-Scheffler free-atom C6 (Hartree Bohr^6) and vdW radii (Bohr), the published values the reference's
# dispersion term tabulates (face/dispersion.py:16-19); elements without an entry take carbon's.
_TS_C6 = {1: 6.50, 6: 46.6, 7: 24.2, 8: 15.6, 11: 1556.0, 12: 627.0, 13: 528.0, 17: 94.6, 47: 339.0, 79: 298.0}
_TS_R0 = {1: 3.10, 6: 3.59, 7: 3.34, 8: 3.19, 11: 3.74, 12: 3.66, 13: 3.84, 17: 3.71, 47: 3.82, 79: 3.86}
_HARTREE_EV, _BOHR_A = 27.211386, 0.529177


class DispParams(nn.Module):
    """Dispersion term parameters (face/dispersion.py:22-34): w (C -> 1) modulating the free-atom C6 by the
    environment, Becke-Johnson damping a1/a2, per-element C6 (eV A^6) and radii (A) buffers over Z = 0..118."""

    def __init__(self, C, r_long=10.0):
        super().__init__()
        self.r_long = r_long
        self.w = nn.Linear(C, 1)
        self.a1 = nn.Parameter(torch.tensor(0.4))
        self.a2 = nn.Parameter(torch.tensor(2.5))
        unit = _HARTREE_EV * _BOHR_A ** 6
        c6 = torch.full((119,), _TS_C6[6] * unit)
        r0 = torch.full((119,), _TS_R0[6] * _BOHR_A)
        for z, v in _TS_C6.items():
            c6[z] = v * unit
        for z, v in _TS_R0.items():
            r0[z] = v * _BOHR_A
        self.register_buffer("c6", c6)
        self.register_buffer("r0", r0)


def _fan_in(model, name):
    return model.get_parameter(name.rsplit(".", 1)[0] + ".weight").shape[1]


def seeded_state(model, seed, perturb=0.25):
    """Deterministic random weights: each parameter from its own stream keyed by (seed, crc32(name)), with the
    reference's initial distribution (nn.Linear uniform(+-1/sqrt(fan_in)) -- stored as uniform(+-1) under unit
    parameterisation --, embeddings N(0,1), ones/zeros where the reference initialises them so), then every
    stored parameter gets + perturb * N(0,1) as in face-mlip tests/test_symmetry.py:32-33.  Without the
    perturbation a random-init model gives forces of ~1e-3 eV/A; with 0.25 the 5-element alloy model gives
    force rms ~0.5 eV/A and charge rms ~0.3 e (physical magnitudes)."""
    out = {}
    unit = getattr(model, "unit", False)
    for name, p in model.named_parameters():
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        amp = perturb
        sh = tuple(p.shape)
        mod, leaf = name.rsplit(".", 1)
        last = mod.split(".")[-1]
        two = ".".join(mod.split(".")[-2:])
        is_lin = last in LINEAR_NAMES or two in LINEAR_NAMES
        if last == "gate":                                  # face/model.py:158
            base = np.zeros(sh) if leaf == "weight" else np.ones(sh)
        elif last == "disp" and leaf in ("a1", "a2"):     # face/dispersion.py:27
            base = np.full(sh, 0.4 if leaf == "a1" else 2.5)
        elif mod.endswith("disp.w"):                       # face/dispersion.py:26: zero-initialised modulation
            base = np.zeros(sh)
        elif is_lin and leaf == "weight":
            bound = 1.0 if unit else _fan_in(model, name) ** -0.5
            base = rng.uniform(-bound, bound, sh)
        elif is_lin and leaf == "bias":
            bound = _fan_in(model, name) ** -0.5
            base = rng.uniform(-bound, bound, sh)
        elif last == "pair":                                # face/model.py:128
            base = np.zeros(sh)
        elif last in ("elem_scale", "pqs_gate") or leaf in ("vpath", "mpath") or (last == "norm" and leaf in ("weight", "w")):
            base = np.ones(sh)
        elif last == "norm":
            base = np.zeros(sh)
        else:                                               # embed.weight
            base = rng.standard_normal(sh)
        # rounded to float32 so that float32 and float64 models hold identical values
        val = (base + amp * rng.standard_normal(sh)).astype(np.float32).astype(np.float64)
        out[name] = torch.as_tensor(val, dtype=p.dtype)
    return out
