"""Drop-in for face-mlip `face.calculator` (face/calculator.py:10-78): `load_face` rebuilds a FACE model from a
reference checkpoint ({"state", "args", "elements", "Eref"}, face/train.py:206-207) and `FACECalculator` evaluates
energy and forces of an atoms object on the B200 engine.

ASE is optional: with ASE installed the calculator is an `ase.calculators.calculator.Calculator`; without it the
same `calculate` / `get_potential_energy` / `get_forces` methods work on any atoms-like object
(`positions`, `numbers`, `cell`, `pbc`).
"""
import numpy as np
import torch

from .model import FACE
from .neighbors import _as_struct, build_graph

try:                                                   # pragma: no cover - depends on the environment
    from ase.calculators.calculator import Calculator, all_changes
except Exception:                                      # ASE absent: minimal stand-in with the same surface
    all_changes = ("positions", "numbers", "cell", "pbc")

    class Calculator:
        implemented_properties = []

        def __init__(self, **kw):
            self.results = {}
            self.atoms = None

        def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
            if atoms is not None:
                self.atoms = atoms

        def get_potential_energy(self, atoms=None):
            self.calculate(atoms)
            return self.results["energy"]

        def get_forces(self, atoms=None):
            self.calculate(atoms)
            return self.results["forces"]

_ALLOWED_MISSING = ("inv_scale", "calibrated", "mom_scale", "eq_scale", "pqs_gate.weight", "tmix3.weight")


def load_face(path, device="cuda"):
    """Rebuild FACE from a reference checkpoint (face/calculator.py:10-32)."""
    c = torch.load(path, weights_only=False, map_location="cpu")
    a = c["args"]
    terms = [t for t in a.get("terms", "").split(",") if t]
    m = FACE(c.get("elements", sorted(c.get("E0", {}))), C=a["C"], n_basis=a.get("nbasis", 8), rc=a["rc"],
             n_passes=a["passes"], terms=terms, radial_hidden=a.get("radial_hidden", 64), K_dir=a.get("kdir", 16),
             norm=a.get("norm", "layer"), transport=bool(a.get("transport", 0)), eqmsg=bool(a.get("eqmsg", 0)),
             factor=bool(a.get("factor", 0)), B=a.get("B", 16), K=a.get("K", 32), cp=bool(a.get("cp", 0)),
             unit=bool(a.get("unit", 0)))
    m.set_standardise(bool(a.get("standardise", 0)))
    m.set_momnorm(bool(a.get("momnorm", 0)))
    m.set_calib(bool(a.get("calib", 0)), keep_ln=bool(a.get("calib_ln", 0)))
    m.set_eq_linear(bool(a.get("eq_linear", 0)))
    m.set_max_body(a.get("max_body", 5))
    m.set_elem_proj(bool(a.get("elem_proj", 0)))
    m.set_poly_readout(bool(a.get("poly", 0)))
    m.set_transport3(bool(a.get("t3", 0)))
    missing, unexpected = m.load_state_dict(c["state"], strict=False)
    if unexpected or not all(k.endswith(_ALLOWED_MISSING) for k in missing):
        raise RuntimeError(f"checkpoint does not match the model: missing={missing} unexpected={unexpected}")
    m = m.to(device).eval()
    return m, c


class FACECalculator(Calculator):
    """Energy and forces of one atoms object (face/calculator.py:35-55).

    `fused` (default True) compiles the radial MLP of a checkpoint-loaded model into its cubic Hermite tables, as the
    reference's calculator does (face/calculator.py:42-44); the engine has only its CUDA path otherwise.
    `skin` (Angstrom, default 0 = the reference's behaviour, a fresh neighbour list every call) keeps the neighbour
    list of pairs closer than rc + skin across calls while no atom has moved more than skin/2 since it was built
    (and species, cell and periodicity are unchanged), as MD drivers do (face/neighbors.py:7 builds such lists).
    The model's envelope is zero beyond rc and the Coulomb real-space sum is cut at rc, so a reused list gives the
    same energies and forces as a fresh one.  The reuse test costs one device-side max and one scalar read.
    `cuda_graph` replays one captured CUDA graph per evaluation while the list is reused (face_b200.graphs)."""
    implemented_properties = ["energy", "forces"]

    def __init__(self, path=None, device="cuda", fused=True, e_shift=0.0, model=None, dtype=torch.float32, skin=0.0,
                 cuda_graph=False, **kw):
        super().__init__(**kw)
        if model is None:
            model, ck = load_face(path, device)
            e_shift = e_shift + float(ck.get("Eref", 0.0))
            if fused and torch.device(device).type == "cuda" and model.form != "moment" and model.spline[0] is None:
                model.compile_radial()                    # as the reference's calculator does (face/calculator.py:42-44)
        self.model = model.to(device=device, dtype=dtype)
        self.device, self.dtype = device, dtype
        self.e_shift = e_shift
        self.skin = float(skin)
        self._graph, self._key, self._stage = None, None, None
        self.rebuilds = 0
        # cuda_graph: each evaluation on a reused neighbour list is one CUDA-graph replay (face_b200.graphs), captured
        # again after every rebuild; worthwhile with a skin, for systems small enough to be launch-bound
        self.cuda_graph = bool(cuda_graph)
        self._replay, self._replay_of = None, None

    def _positions(self, pos):
        """Host positions -> device float64 through a pinned staging buffer."""
        if self._stage is None or self._stage.shape != pos.shape:
            self._stage = torch.empty(pos.shape, dtype=torch.float64, pin_memory=True)
        self._stage.numpy()[:] = pos
        return self._stage.to(self.device, non_blocking=True)

    def graph(self, at):
        """The neighbour graph for `at`: rebuilt, or (skin > 0) the previous one with the new positions."""
        pos, Z, cell, pbc, q = _as_struct(at)
        key = (Z.tobytes(), cell.tobytes(), pbc, q)
        if self.skin > 0 and self._graph is not None and key == self._key:
            p64 = self._positions(pos)
            g = self._graph
            if 2.0 * float((p64 - g["pos64"]).norm(dim=1).max()) < self.skin:
                return dict(g, pos=p64.to(self.dtype))
        rc_long = self.model.terms["disp"].r_long if "disp" in self.model.terms else None
        self._graph = build_graph([at], self.model.rc, device=self.device, dtype=self.dtype, skin=self.skin,
                                  rc_long=rc_long, pos64=self._positions(pos))
        self._key = key
        self.rebuilds += 1
        return self._graph

    def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        at = self.atoms if atoms is None else atoms
        g = self.graph(at)
        if self.cuda_graph:
            from .graphs import GraphedEvaluation
            if self._replay_of is not self._graph:
                self._replay = None                        # release the previous capture before the next one
                self._replay = GraphedEvaluation(self.model, self._graph)
                self._replay_of = self._graph
            o = self._replay(g["pos"])
        else:
            o = self.model(g)
        self.results["energy"] = float(o["energy"].item()) + self.e_shift
        self.results["forces"] = o["forces"].detach().double().cpu().numpy()


class FACEEnsembleCalculator(Calculator):
    """Mean energy/forces of several checkpoints and their spread (face/calculator.py:58-78)."""
    implemented_properties = ["energy", "forces"]

    def __init__(self, paths, device="cuda", fused=True, **kw):
        super().__init__(**kw)
        self.members = [FACECalculator(p, device=device) for p in paths]

    def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        at = self.atoms if atoms is None else atoms
        Es, Fs = [], []
        for c in self.members:
            c.calculate(at, properties, system_changes)
            Es.append(c.results["energy"])
            Fs.append(c.results["forces"])
        Es, Fs = np.array(Es), np.array(Fs)
        self.results["energy"] = float(Es.mean())
        self.results["forces"] = Fs.mean(0)
        self.results["energy_std"] = float(Es.std())
        self.results["forces_std"] = np.linalg.norm(Fs.std(0), axis=-1)
