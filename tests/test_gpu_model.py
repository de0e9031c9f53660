"""Full energy+force evaluation on the B200 engine against the reference's own outputs (golden fixtures generated
from face-mlip itself) and the oracle, plus the reference's symmetry / finite-difference checks
(face-mlip tests/test_symmetry.py, tests/test_periodic.py).

Bars: fp64 energies within 1e-10 relative; fp32 energies within 1e-6 relative and forces within
1e-4 eV/A (also 1e-4 relative to the largest force)."""
import numpy as np
import pytest
import torch

from _golden import MODEL_CASES, RC_LONG, case_inputs

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _engine(spec, seed, pme, dtype, spline=False):
    from face_b200.model import FACE
    kw = dict(spec)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    m.seed_(seed)
    if "coulomb" in kw.get("terms", ()):
        m.set_pme(gp=pme["gp"], mesh=pme.get("mesh"))
    m = m.to("cuda", dtype)
    if spline:
        m.compile_radial()
    return m


def _run(name, dtype):
    from face_b200.neighbors import build_graph
    structs, spec, pme, d = case_inputs(name)
    m = _engine(spec, d["meta"]["seed"], pme, dtype, d["meta"]["spline"])
    g = build_graph(structs, spec["rc"], dtype=dtype, rc_long=RC_LONG if "disp" in spec.get("terms", ()) else None)
    o = m(g)
    return o, d


@pytest.mark.parametrize("name", MODEL_CASES)
def test_neighbour_list_matches_golden_edges(name):
    """The GPU cell list gives, bit for bit, the (i, j, S) edge list (canonical row order) that the reference's model
    consumed when the golden was made: the fixture holds the SHA-256 of that int64 (E, 5) array."""
    import hashlib
    from face_b200.neighbors import build_graph
    structs, spec, pme, d = case_inputs(name)
    g = build_graph(structs, spec["rc"], dtype=torch.float64)
    edges = torch.cat([g["ei"][:, None], g["ej"][:, None], g["S"]], 1).to(torch.int64).cpu().numpy()
    assert len(edges) == d["meta"]["n_edges"]
    assert hashlib.sha256(np.ascontiguousarray(edges).tobytes()).hexdigest() == str(d["edge_hash"])


@pytest.mark.parametrize("name", MODEL_CASES)
def test_fp64_matches_reference(name):
    o, d = _run(name, torch.float64)
    E, F = o["energy"].cpu().numpy(), o["forces"].cpu().numpy()
    assert np.abs(E - d["energy64"]).max() <= 1e-10 * np.abs(d["energy64"]).max(), (E, d["energy64"])
    assert np.abs(F - d["forces64"]).max() <= 1e-9
    assert np.abs(o["atom_energy"].cpu().numpy() - d["atom_energy64"]).max() <= 1e-9


@pytest.mark.parametrize("name", MODEL_CASES)
def test_fp32_matches_reference(name):
    """fp32 bars: energy within 1e-6 relative, forces within 1e-4 eV/A.  Model cases are held to both the reference's
    fp64 and fp32 outputs.  The compiled-radial case is held to the reference's fp32 outputs: its Hermite tables are
    built in the model's precision (face/model.py:393-405), so the fp32 spline is a different function from the fp64
    one at the 1e-7 level of the table entries.  Where the reference's own fp32 result misses its fp64 result by more
    than these bars (the ZBL case: close contacts with forces near 90 eV/A), the bar is twice the reference's own fp32
    deviation."""
    o, d = _run(name, torch.float32)
    E, F = o["energy"].double().cpu().numpy(), o["forces"].double().cpu().numpy()
    scale = np.abs(d["energy64"]).max()
    gap_e = np.abs(d["energy32"] - d["energy64"]).max()
    gap_f = np.abs(d["forces32"] - d["forces64"]).max()
    tol_e = max(1e-6 * scale, 2 * gap_e)
    tol_f = max(1e-4, 2 * gap_f)
    refs = [("32", d["energy32"], d["forces32"])]
    if not d["meta"]["spline"]:
        refs.append(("64", d["energy64"], d["forces64"]))
    for tag, Er, Fr in refs:
        assert np.abs(E - Er).max() <= tol_e, (tag, E, Er, tol_e)
        dF = np.abs(F - Fr).max()
        assert dF <= tol_f, (tag, dF, tol_f)


def test_reference_padded_graph_input():
    """The reference's padded graph dict (face/model.py:7-14) gives the same result as the engine's CSR graph."""
    from face_b200.neighbors import build_graph, to_padded
    structs, spec, pme, d = case_inputs("cfg5_small")
    m = _engine(spec, 0, pme, torch.float64)
    g = build_graph(structs, spec["rc"], dtype=torch.float64)
    o1 = m(g)
    p = to_padded(g)
    p["pos"] = p["pos"].detach().clone()
    o2 = m(p)
    assert float((o1["energy"] - o2["energy"]).abs().max()) < 1e-10 * float(o1["energy"].abs().max())
    assert float((o1["forces"] - o2["forces"]).abs().max()) < 1e-10


def test_symmetry_and_finite_differences_fp64():
    """Rotation/reflection + translation and permutation invariance, central-difference forces
    (face-mlip tests/test_symmetry.py:37-52) on a non-periodic batch."""
    from face_b200 import systems
    from face_b200.neighbors import build_graph
    spec = systems.model_kwargs(3)
    m = _engine(spec, 1, {}, torch.float64)
    mol = systems.molecule(14, seed=5)
    E0 = lambda st: m(build_graph([st], spec["rc"], dtype=torch.float64))
    o = E0(mol)
    E, F = float(o["energy"][0]), o["forces"].cpu().numpy()
    rng = np.random.default_rng(0)
    for sign in (1, -1):
        Q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
        Q = sign * Q * np.sign(np.linalg.det(Q))
        st = systems.Structure(mol.positions @ Q.T + rng.normal(size=3), mol.numbers)
        o2 = E0(st)
        assert abs(float(o2["energy"][0]) - E) < 1e-9
        assert np.abs(o2["forces"].cpu().numpy() - F @ Q.T).max() < 1e-8
    perm = rng.permutation(len(mol.numbers))
    o3 = E0(systems.Structure(mol.positions[perm], mol.numbers[perm]))
    assert abs(float(o3["energy"][0]) - E) < 1e-9 and np.abs(o3["forces"].cpu().numpy() - F[perm]).max() < 1e-8
    h = 1e-5
    for i, c in [(0, 0), (3, 2), (7, 1)]:
        pp, pm = mol.positions.copy(), mol.positions.copy()
        pp[i, c] += h
        pm[i, c] -= h
        fd = -(float(E0(systems.Structure(pp, mol.numbers))["energy"][0]) -
               float(E0(systems.Structure(pm, mol.numbers))["energy"][0])) / (2 * h)
        assert abs(fd - F[i, c]) < 1e-6 * (1 + abs(fd)), (fd, F[i, c])


def test_periodic_invariances_fp64():
    """Lattice translation + wrap, 2x1x1 extensivity and rotation of positions+cell with the PME Coulomb term
    (face-mlip tests/test_periodic.py:34-53; PME bars 1e-3 there, exact-Ewald-free terms are tighter here)."""
    from face_b200 import systems
    from face_b200.neighbors import build_graph
    spec = systems.model_kwargs(2)
    m = _engine(spec, 2, {"gp": 1 / 0.32, "mesh": (32, 32, 32)}, torch.float64)
    st = systems.rocksalt(2, 5.64, 0.15, seed=0)
    run = lambda s: m(build_graph([s], spec["rc"], dtype=torch.float64))
    o = run(st)
    E, F = float(o["energy"][0]), o["forces"].cpu().numpy()
    b = systems.Structure(st.positions + 3.1 * st.cell[0] / 5.64 + 0.37, st.numbers, st.cell, True)
    ob = run(b)
    assert abs(float(ob["energy"][0]) - E) < 1e-3 * (1 + abs(E))
    assert np.abs(ob["forces"].cpu().numpy() - F).max() < 1e-3
    Q, _ = np.linalg.qr(np.random.default_rng(2).normal(size=(3, 3)))
    r = systems.Structure(st.positions @ Q.T, st.numbers, st.cell @ Q.T, True)
    orr = run(r)
    assert abs(float(orr["energy"][0]) - E) < 1e-3 * (1 + abs(E))
    assert np.abs(orr["forces"].cpu().numpy() - F @ Q.T).max() < 1e-3


def test_distributed_model_single_rank_matches_engine():
    """The decomposition driver on one rank (one brick, no ghosts) reproduces the plain engine, Coulomb included."""
    from face_b200 import systems
    from face_b200.domain import DistributedModel
    from face_b200.neighbors import build_graph
    structs, spec, pme, d = case_inputs("cfg5_small")
    m = _engine(spec, 0, pme, torch.float64)
    dm = DistributedModel(m, structs[0], 0, 1, torch.device("cuda"), torch.float64)
    pos = torch.as_tensor(structs[0].positions, dtype=torch.float64, device="cuda")
    E, F = dm.energy_forces(pos[dm.gid_owned])
    F = torch.zeros_like(F).index_copy(0, dm.gid_owned, F)
    assert abs(float(E) - d["energy64"][0]) <= 1e-10 * abs(d["energy64"][0])
    assert np.abs(F.cpu().numpy() - d["forces64"]).max() <= 1e-9
