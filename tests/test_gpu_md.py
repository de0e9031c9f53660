"""Evaluation without host synchronisation and neighbour-list reuse across MD-style steps.

The reference routes around int(batch.max()) with g["nstr"] to stay sync-free (face/model.py:689) but its PME
Coulomb term still reads the device per structure (face/electrostatics.py:58,144-146).  Here a fixed graph carries its
per-structure host data (offsets, inverse cells, volumes) from construction, so an energy+force evaluation issues no
synchronising torch call; the library itself synchronises only inside the neighbour-list build."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _model(cfg, dtype, seed=0, pme=None):
    from face_b200 import systems
    from face_b200.model import FACE
    kw = systems.model_kwargs(cfg)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    m.seed_(seed)
    if pme is not None:
        m.set_pme(**pme)
    return m.to("cuda", dtype), kw["rc"]


@pytest.mark.parametrize("case", ["periodic_batch", "molecules"])
def test_evaluation_issues_no_host_sync(case):
    from face_b200 import systems
    from face_b200.neighbors import build_graph
    if case == "periodic_batch":            # two rock-salt boxes: Coulomb + PME looped over structures
        m, rc = _model(2, torch.float32, pme={"gp": 1 / 0.32, "mesh": (24, 24, 24)})
        structs = [systems.rocksalt(3, 5.64, 0.05, seed=s) for s in (0, 1)]
    else:
        m, rc = _model(3, torch.float32)
        structs = systems.config_structures(3, seed=0, scale=5)
    g = build_graph(structs, rc, dtype=torch.float32)
    ref = m(dict(g, pos=g["pos"].clone()))                   # warm-up: weight packing, FFT plans, tables
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        o = m(dict(g, pos=g["pos"].clone()))
    finally:
        torch.cuda.set_sync_debug_mode("default")
    # same result (not bit for bit: the PME charge spreading adds with atomics, in no fixed order)
    assert float((o["energy"] - ref["energy"]).abs().max()) <= 1e-6 * float(ref["energy"].abs().max())
    assert float((o["forces"] - ref["forces"]).abs().max()) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_calculator_skin_reuse_matches_fresh_lists(dtype):
    """MD-like trajectory: the calculator with a 1 A skin rebuilds only when an atom moved more than 0.5 A and
    otherwise reuses the list; every step matches a calculator that builds a fresh list (the reference's calculator,
    face/calculator.py:49-53) to the fp64 / fp32 bars."""
    from face_b200 import systems
    from face_b200.calculator import FACECalculator
    m, rc = _model(2, dtype, seed=3, pme={"gp": 1 / 0.32, "mesh": (32, 32, 32)})
    st = systems.rocksalt(3, 5.64, 0.05, seed=4)
    fresh = FACECalculator(model=m, device="cuda", dtype=dtype)
    reuse = FACECalculator(model=m, device="cuda", dtype=dtype, skin=1.0)
    rng = np.random.default_rng(0)
    pos = st.positions.copy()
    for step in range(8):
        pos = pos + rng.normal(0, 0.12, pos.shape)            # random walk: the 0.5 A trigger is crossed midway
        at = systems.Structure(pos.copy(), st.numbers, st.cell, True)
        fresh.calculate(at)
        reuse.calculate(at)
        e0, e1 = fresh.results["energy"], reuse.results["energy"]
        f0, f1 = fresh.results["forces"], reuse.results["forces"]
        tol_e, tol_f = (1e-10, 1e-9) if dtype == torch.float64 else (1e-6, 1e-4)
        assert abs(e1 - e0) <= tol_e * abs(e0), (step, e0, e1)
        assert np.abs(f1 - f0).max() <= tol_f, step
    assert fresh.rebuilds == 8 and 1 < reuse.rebuilds < 8, reuse.rebuilds


@pytest.mark.parametrize("case", ["molecules", "periodic_coulomb"])
def test_graphed_evaluation_matches_eager(case):
    """One captured CUDA graph of the whole forward + force backward (face_b200.graphs), replayed at new positions,
    against the eager evaluation at the same positions (fp32; PME spreads with atomics, so not bit for bit)."""
    from face_b200 import systems
    from face_b200.graphs import GraphedEvaluation
    from face_b200.neighbors import build_graph
    if case == "molecules":
        m, rc = _model(3, torch.float32)
        structs = systems.config_structures(3, seed=1, scale=6)
    else:
        m, rc = _model(2, torch.float32, pme={"gp": 1 / 0.32, "mesh": (24, 24, 24)})
        structs = [systems.rocksalt(3, 5.64, 0.05, seed=2)]
    g = build_graph(structs, rc, dtype=torch.float32, skin=0.5)
    ev = GraphedEvaluation(m, g)
    gen = torch.Generator(device="cuda").manual_seed(0)
    for _ in range(3):
        pos = g["pos"] + 0.05 * torch.randn(g["pos"].shape, device="cuda", generator=gen)
        o1 = ev(pos)
        o2 = m(dict(g, pos=pos.clone()))
        assert float((o1["energy"] - o2["energy"]).abs().max()) <= 1e-6 * float(o2["energy"].abs().max())
        assert float((o1["forces"] - o2["forces"]).abs().max()) <= 1e-5


def test_calculator_cuda_graph_with_skin():
    """The calculator with a skin and CUDA-graph replays (recaptured at every rebuild) against fresh eager lists."""
    from face_b200 import systems
    from face_b200.calculator import FACECalculator
    m, rc = _model(3, torch.float32, seed=2)
    mol = systems.molecule(30, seed=9)
    fresh = FACECalculator(model=m, device="cuda", dtype=torch.float32)
    graphed = FACECalculator(model=m, device="cuda", dtype=torch.float32, skin=1.0, cuda_graph=True)
    rng = np.random.default_rng(1)
    pos = mol.positions.copy()
    for step in range(6):
        pos = pos + rng.normal(0, 0.1, pos.shape)
        at = systems.Structure(pos.copy(), mol.numbers)
        fresh.calculate(at)
        graphed.calculate(at)
        assert abs(graphed.results["energy"] - fresh.results["energy"]) <= 1e-6 * abs(fresh.results["energy"]) + 1e-6
        assert np.abs(graphed.results["forces"] - fresh.results["forces"]).max() <= 1e-4
    assert 1 <= graphed.rebuilds < 6
