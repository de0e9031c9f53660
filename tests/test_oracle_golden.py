"""The CPU oracle (oracle/) against golden vectors produced by the face-mlip reference itself."""
import hashlib

import numpy as np
import pytest
import torch

from _golden import RC_LONG, SMALL_CASES, TERM_CASES, case_inputs, load
from oracle import face_ref, nlist


def _engine_state(spec, seed):
    from face_b200.model import FACE
    kw = dict(spec)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    return m.seed_(seed).state_dict()


def _long_range(structs, r_long):
    I, J, SH, off = [], [], [], 0
    for st in structs:
        pbc = bool(np.any(st.pbc))
        i, j, S = nlist.neighbor_list_ijS(st.positions, st.cell, pbc, r_long)
        I.append(i + off)
        J.append(j + off)
        SH.append(nlist.shift_vectors(S, np.asarray(st.cell, np.float64)) if pbc else np.zeros((len(i), 3)))
        off += len(st.numbers)
    return {"lr_i": np.concatenate(I), "lr_j": np.concatenate(J), "lr_shift": np.concatenate(SH)}


@pytest.mark.parametrize("name", SMALL_CASES + TERM_CASES)
def test_oracle_matches_reference(name):
    structs, spec, pme, d = case_inputs(name)
    g = nlist.padded_graph(structs, spec["rc"])
    if "disp" in spec.get("terms", ()):
        g.update(_long_range(structs, RC_LONG))
    ei = np.repeat(np.arange(len(g["nbr"])), g["mask"].sum(1))
    edges = np.concatenate([ei[:, None], g["nbr"][g["mask"]][:, None], g["S"][g["mask"]]], 1).astype(np.int64)
    assert hashlib.sha256(np.ascontiguousarray(edges).tobytes()).hexdigest() == str(d["edge_hash"])
    state = _engine_state(spec, d["meta"]["seed"])
    spline = d["meta"]["spline"]
    o = face_ref.forward(state, spec, g, torch.float64, spline=spline, pme=pme)
    E, F = o["energy"].numpy(), o["forces"].numpy()
    # fp64: energies within 1e-10 relative, forces to 1e-9 eV/A
    assert np.abs(E - d["energy64"]).max() <= 1e-10 * np.abs(d["energy64"]).max()
    assert np.abs(F - d["forces64"]).max() <= 1e-9
    assert np.abs(o["atom_energy"].numpy() - d["atom_energy64"]).max() <= 1e-9
    o32 = face_ref.forward(state, spec, g, torch.float32, spline=spline, pme=pme)
    assert np.abs(o32["energy"].double().numpy() - d["energy32"]).max() <= 1e-6 * np.abs(d["energy64"]).max()
    assert np.abs(o32["forces"].double().numpy() - d["forces32"]).max() <= 1e-4


def test_oracle_kernel_twins():
    k = load("kernels")
    t = lambda x: torch.tensor(x, requires_grad=True)
    for tag in ("a", "b"):
        phi, msg, Y = t(k[f"fd{tag}_phi"]), t(k[f"fd{tag}_msg"]), t(k[f"fd{tag}_Y"])
        D = face_ref.factor_density(phi, msg, Y)
        gr = torch.autograd.grad((D * torch.tensor(k[f"fd{tag}_G"])).sum(), (phi, msg, Y))
        assert np.allclose(D.detach().numpy(), k[f"fd{tag}_D"], rtol=1e-12, atol=1e-12)
        for gx, nm in zip(gr, ("dphi", "dmsg", "dY")):
            assert np.allclose(gx.numpy(), k[f"fd{tag}_{nm}"], rtol=1e-12, atol=1e-12)
    names = ["P1", "Q1", "S1", "P2", "Q2", "S2", "P3", "Q3"]
    ranks = [1, 1, 1, 2, 2, 2, 3, 3]
    xs = [t(k["na_" + n]) for n in names]
    a, b = t(k["na_a"]), t(k["na_b"])
    inv, V, Mf = face_ref.node_products(*[face_ref.to_full(x, l) for x, l in zip(xs, ranks)], a, b)
    L = (inv * torch.tensor(k["na_gI"])).sum() + (V * torch.tensor(k["na_gV"])).sum() + (Mf * torch.tensor(k["na_gM"])).sum()
    grads = torch.autograd.grad(L, xs + [a, b])
    assert np.allclose(inv.detach().numpy(), k["na_inv"], rtol=1e-12, atol=1e-12)
    assert np.allclose(V.detach().numpy(), k["na_V"], rtol=1e-12, atol=1e-12)
    assert np.allclose(Mf.detach().numpy(), k["na_Mf"], rtol=1e-12, atol=1e-12)
    for gx, nm in zip(grads, ["d" + n for n in names] + ["da", "db"]):
        assert np.allclose(gx.numpy(), k["na_" + nm], rtol=1e-11, atol=1e-11), nm


def test_oracle_ewald_pme():
    k = load("electrostatics")
    pos, cell, q = k["rand_pos"], k["rand_cell"], k["rand_q"]
    i, j, S = nlist.neighbor_list_ijS(pos, cell, True, 5.0)
    pr = (torch.tensor(i), torch.tensor(j), torch.tensor(nlist.shift_vectors(S, cell)))
    for use_pme, tag in ((False, "exact"), (True, "pme")):
        p = torch.tensor(pos, requires_grad=True)
        e = face_ref.ewald_energy(torch.tensor(q), p, torch.tensor(cell), pr, 1.0, float(k["rand_gp"]),
                                  use_pme=use_pme, kcut=float(k["rand_kcut"]))
        f = -torch.autograd.grad(e, p)[0]
        assert abs(float(e) - float(k[f"rand_{tag}_e"])) <= 1e-10 * abs(float(k[f"rand_{tag}_e"]))
        assert np.abs(f.numpy() - k[f"rand_{tag}_f"]).max() <= 1e-10
    # PME vs exact Ewald (face-mlip tests/test_electrostatics.py:152-153 bar, 1e-3 relative)
    assert abs(k["rand_pme_e"] - k["rand_exact_e"]) / abs(k["rand_exact_e"]) < 1e-3
    p = torch.tensor(pos, requires_grad=True)
    qq = torch.tensor(q, requires_grad=True)
    spacing = 12.0 * 0.9 / 20 * (1 + 1e-9)                 # the spacing the fixture passed to the reference
    mesh = [max(8, int(np.ceil(L / spacing))) for L in np.linalg.norm(cell, axis=1)]
    assert mesh == [23, 20, 25]
    e = face_ref.pme_recip_energy(qq, p, torch.tensor(cell), 1 / 0.32, mesh=mesh)
    gp_, gq_ = torch.autograd.grad(e, (p, qq))
    assert abs(float(e) - float(k["recip_e"])) <= 1e-12 * abs(float(k["recip_e"]))
    assert np.abs(gp_.numpy() - k["recip_dpos"]).max() <= 1e-11
    assert np.abs(gq_.numpy() - k["recip_dq"]).max() <= 1e-11


def test_madelung_known_answer():
    """NaCl Madelung constant -1.747565 (face-mlip tests/test_electrostatics.py:112-124), exact Ewald."""
    from face_b200 import systems
    st = systems.rocksalt(1, 5.64, 0.0, 0)
    q = torch.tensor([1.0 if z == 11 else -1.0 for z in st.numbers], dtype=torch.float64)
    ref = -1.747565 * face_ref.KE / (5.64 / 2) * 4
    for rc in (5.0, 7.0):
        gp = max(rc / 3.5, 1.05 * 0.04)
        i, j, S = nlist.neighbor_list_ijS(st.positions, st.cell, True, rc)
        pr = (torch.tensor(i), torch.tensor(j), torch.tensor(nlist.shift_vectors(S, st.cell)))
        e = face_ref.KE * face_ref.ewald_energy(q, torch.tensor(st.positions), torch.tensor(st.cell), pr, 0.04, gp,
                                                use_pme=False, kcut=2 * 3.5 / gp)
        assert abs(float(e) - ref) / abs(ref) < 1e-5
