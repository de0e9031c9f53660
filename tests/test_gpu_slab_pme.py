"""Slab-distributed PME (face_b200/domain.py SlabPME over ops.SpreadMesh) on one GPU: the decomposed evaluation with
world = 1 and the mesh handled by the slab pipeline (spread -> 2-D FFT -> 1-D FFT, energy share from the k block,
forces through the spreading adjoint facek_pme_gather) against the single-GPU engine, whose PME runs
spread -> rfftn -> Green's function -> irfftn -> gather (face/electrostatics.py:54-77).  fp64, 1e-10 relative energy,
1e-9 eV/A forces."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "face-mlip_b200"))

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_slab_pme_one_rank_matches_engine():
    from face_b200 import systems
    from face_b200.domain import DistributedModel
    from face_b200.model import FACE
    from face_b200.neighbors import build_graph
    dev = torch.device("cuda", 0)
    spec = dict(systems.model_kwargs(5))
    mb = spec.pop("max_body")
    m = FACE(**spec)
    m.set_max_body(mb)
    m.seed_(2)
    m.set_pme(gp=1 / 0.32, mesh=(32, 30, 28))
    m = m.to(dev, torch.float64)
    st = systems.fcc(6, 3.6, 0.08, systems.MODELS[5]["elements"], seed=1)
    dm = DistributedModel(m, st, 0, 1, dev, torch.float64)
    pos = torch.as_tensor(st.positions, dtype=torch.float64, device=dev)
    for _ in range(2):                                   # twice: the cached slab factors are reused
        E, F = dm.energy_forces(pos[dm.gid_owned])
        o = m(build_graph([st], m.rc, device=dev, dtype=torch.float64))
        assert abs(float(E) - float(o["energy"][0])) <= 1e-10 * abs(float(o["energy"][0]))
        assert float((F - o["forces"][dm.gid_owned]).abs().max()) <= 1e-9
