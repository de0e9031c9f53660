"""Generate golden fixtures from the face-mlip reference itself (run in a container that has the reference
checked out; the fixtures are committed, the reference is not needed to run the tests).

    python tests/golden/make_golden.py --ref /path/to/face-mlip [--only NAME]

For every case: seeded structure (face_b200.systems) -> canonical neighbour list (oracle.nlist, the
reference's ASE call is not installed) -> the reference's own FACE (face/model.py) with seeded weights
loaded through a strict state_dict load (so the key layout is checked too) -> energies, per-atom energies,
charges and forces in float64 and float32.  Also the reference's kernel twins (face/kernels.py:175-178,
face/node_kernel.py:212-228 with face/cartesian.py:59-66 expansion) and its Ewald/PME functions
(face/electrostatics.py:54-129) on seeded inputs.
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "face-mlip_b200"))

from oracle import nlist                                    # noqa: E402
from face_b200 import systems                               # noqa: E402
from face_b200.model import FACE as EngineFACE              # noqa: E402

# model cases: (name, cfg, scale, model overrides, pme mesh override, spline)
CASES = [
    ("cfg1", 1, None, {}, None, False),
    ("cfg1_spline", 1, None, {}, None, True),
    ("cfg2", 2, None, {}, None, False),
    ("cfg3_small", 3, 6, {}, None, False),
    ("cfg4_small", 4, 600, {}, (24, 24, 24), False),
    ("cfg5_small", 5, 4, {}, (24, 24, 24), False),
    # the benchmark configurations at full size (cfg3), the largest cfg4 box whose reference evaluation fits a 62 GB
    # host (16,384 atoms at the same 0.1 A^-3 density, PME mesh at the 96^3 spacing of the full box: 54.7 A / 76;
    # the full 32,768-atom box needs more memory in the reference's unfused float64 path), and a 37,044-atom cfg5
    # sub-box (21^3 conventional cells, PME mesh at the 256^3 spacing of the full alloy: 75.6 A / 84 = 230.4 A / 256)
    ("cfg3", 3, None, {}, None, False),
    ("cfg4_16k", 4, 16384, {}, (76, 76, 76), False),
    ("cfg5_37k", 5, 21, {}, (84, 84, 84), False),
]
# physics terms (face/model.py:538-590): ZBL on molecules (close contacts below the 1.2 A switch), dispersion over the
# 10 A long-range list on molecules and on a periodic rock-salt box together with the PME Coulomb term
TERM_CASES = [
    ("zbl_mol", 3, 6, {"terms": ("zbl",)}, None, False),
    ("disp_mol", 3, 6, {"terms": ("disp",)}, None, False),
    ("disp_nacl", 2, 2, {"terms": ("coulomb", "disp")}, (20, 20, 20), False),
]
# the other density forms of the shipped checkpoints (face/model.py:99-202, :421-534): the CP form (cp=True, per-channel
# messages) and the non-factorised MomentBlock (factor=False), both with transport and equivariant messages
FORM_CASES = [
    ("cp_small", 5, 4, {"cp": True}, (24, 24, 24), False),
    ("cp_mol", 3, 6, {"cp": True, "C": 32}, None, False),
    ("cp_spline", 1, None, {"cp": True}, None, True),
    ("moment_small", 5, 4, {"factor": False}, (24, 24, 24), False),
    ("moment_mol", 3, 6, {"factor": False, "C": 32}, None, False),
]
CASES += TERM_CASES + FORM_CASES
R_LONG = 10.0       # the dispersion term's default r_long, also the long-range list cutoff here
BIG = 4000          # cases above this many atoms store a position hash instead of the positions


def build_reference_model(face_model, cfg, over, state):
    kw = systems.model_kwargs(cfg, **over)
    unit, max_body = kw.pop("unit"), kw.pop("max_body")
    m = face_model.FACE(**kw)
    if unit:
        face_model.unit_parameterise(m)
    m.set_max_body(max_body)
    missing, unexpected = m.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert all(k.endswith(("inv_scale", "calibrated", "mom_scale", "eq_scale", "zmap", "E0", "scale", "avg_nb",
                           "freq")) for k in missing), missing
    return m, dict(kw, unit=unit, max_body=max_body)


def engine_state(cfg, over, seed):
    kw = systems.model_kwargs(cfg, **over)
    max_body = kw.pop("max_body")
    e = EngineFACE(**kw)
    e.set_max_body(max_body)
    st = e.seed_(seed).state_dict()
    return {k: v for k, v in st.items() if not k.endswith(("zmap", "freq"))}


def run_model_case(ref, name, cfg, scale, over, mesh, spline, seed=0):
    import face.model as fm
    import face.electrostatics as fe
    structs = systems.config_structures(cfg, seed=seed, scale=scale)
    state = engine_state(cfg, over, seed)
    pme = dict(systems.MODELS[cfg].get("pme", {}))
    if mesh is not None:
        pme["mesh"] = mesh
    rc = systems.MODELS[cfg]["rc"]
    g = nlist.padded_graph(structs, rc)
    lr = long_range_pairs(structs, R_LONG) if "disp" in systems.model_kwargs(cfg, **over)["terms"] else None
    out = {}
    orig = fe.pme_recip_energy
    for dt, tag in ((torch.float64, "64"), (torch.float32, "32")):
        torch.set_default_dtype(dt)
        m, spec = build_reference_model(fm, cfg, over, {k: v.to(dt) for k, v in state.items()})
        m = m.to(dt).eval()
        if "coulomb" in m.terms:
            m.terms["coulomb"].gp = pme["gp"]
            n = pme["mesh"]

            def patched(q, pos, cell, gp, spacing=None, _n=n):
                L = float(cell.norm(dim=-1)[0])
                return orig(q, pos, cell, gp, spacing=L / _n[0] * (1 + 1e-9))
            fe.pme_recip_energy = patched
        if spline:
            m.compile_radial()
        gg = {"pos": torch.tensor(g["pos"], dtype=dt), "Z": torch.tensor(g["Z"]), "nbr": torch.tensor(g["nbr"]),
              "shift": torch.tensor(g["shift"], dtype=dt), "mask": torch.tensor(g["mask"]),
              "batch": torch.tensor(g["batch"]), "cell": torch.tensor(g["cell"], dtype=dt),
              "charge": torch.tensor(g["charge"], dtype=dt), "nstr": int(g["nstr"])}
        if lr is not None:
            gg.update(lr_i=torch.tensor(lr[0]), lr_j=torch.tensor(lr[1]), lr_shift=torch.tensor(lr[2], dtype=dt))
        o = m(gg)
        fe.pme_recip_energy = orig
        out["energy" + tag] = o["energy"].detach().double().numpy()
        out["atom_energy" + tag] = o["atom_energy"].detach().double().numpy()
        out["forces" + tag] = o["forces"].detach().double().numpy()
        if "q" in gg:
            out["q" + tag] = gg["q"].detach().double().numpy()
    torch.set_default_dtype(torch.float64)
    ei = np.repeat(np.arange(len(g["nbr"])), g["mask"].sum(1))
    edges = np.concatenate([ei[:, None], g["nbr"][g["mask"]][:, None], g["S"][g["mask"]]], 1).astype(np.int64)
    meta = {"cfg": cfg, "scale": scale, "seed": seed, "over": over, "mesh": mesh, "spline": spline,
            "spec": spec, "pme": {k: (list(v) if isinstance(v, tuple) else v) for k, v in pme.items()},
            "n_edges": int(len(edges)), "M": int(g["nbr"].shape[1])}
    pos = np.concatenate([s.positions for s in structs])
    if len(pos) > BIG:
        # large cases: the positions are regenerated from the seed and checked against this hash; fp32 outputs are
        # kept in float32 (their own precision)
        geo = {"pos_sha256": np.array(_hash(np.ascontiguousarray(pos, np.float64)))}
        out = {k: (v.astype(np.float32) if k.endswith("32") else v) for k, v in out.items()}
    else:
        geo = {"pos": pos}
    np.savez_compressed(os.path.join(HERE, name + ".npz"), meta=json.dumps(meta),
                        Z=np.concatenate([s.numbers for s in structs]), edge_hash=np.array(_hash(edges)), **geo,
                        **out)
    print(f"{name}: N={len(g['pos'])} E={len(edges)} M={g['nbr'].shape[1]}  E64={out['energy64'][:3]}  "
          f"|F|max={np.abs(out['forces64']).max():.3e}  dE32/E={np.abs(out['energy32'] - out['energy64']).max() / np.abs(out['energy64']).max():.1e}")


def long_range_pairs(structs, r_long):
    """GraphSet's long-range list (face/datasets.py:53-55, 90-95): (i, j, S @ cell) of every structure, offset."""
    I, J, SH, off = [], [], [], 0
    for st in structs:
        pbc = bool(np.any(st.pbc))
        i, j, S = nlist.neighbor_list_ijS(st.positions, st.cell, pbc, r_long)
        I.append(i + off)
        J.append(j + off)
        SH.append(nlist.shift_vectors(S, np.asarray(st.cell, np.float64)) if pbc else np.zeros((len(i), 3)))
        off += len(st.numbers)
    return np.concatenate(I), np.concatenate(J), np.concatenate(SH)


def _hash(edges):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(edges).tobytes()).hexdigest()


def kernel_cases(ref):
    from face.kernels import factor_density_ref
    from face.node_kernel import node_algebra_ref
    from face.cartesian import expand
    torch.set_default_dtype(torch.float64)
    rng = np.random.default_rng(7)
    out = {}
    for tag, (N, M, B, K) in {"a": (9, 7, 4, 8), "b": (5, 13, 16, 32)}.items():
        phi, msg, Y = (torch.tensor(rng.standard_normal(s), requires_grad=True) for s in
                       ((N, M, B), (N, M, K), (N, M, 20)))
        G = torch.tensor(rng.standard_normal((N, 20, B * K)))
        D = factor_density_ref(phi, msg, Y)
        gr = torch.autograd.grad((D * G).sum(), (phi, msg, Y))
        out.update({f"fd{tag}_phi": phi.detach().numpy(), f"fd{tag}_msg": msg.detach().numpy(),
                    f"fd{tag}_Y": Y.detach().numpy(), f"fd{tag}_G": G.numpy(), f"fd{tag}_D": D.detach().numpy(),
                    f"fd{tag}_dphi": gr[0].numpy(), f"fd{tag}_dmsg": gr[1].numpy(), f"fd{tag}_dY": gr[2].numpy()})
    N, C = 6, 5
    shapes = [(3,), (3,), (3,), (6,), (6,), (6,), (10,), (10,)]
    xs = [torch.tensor(rng.standard_normal((N, C) + s), requires_grad=True) for s in shapes]
    a = torch.tensor(rng.standard_normal((4, C)), requires_grad=True)
    b = torch.tensor(rng.standard_normal((4, C)), requires_grad=True)
    gI, gV, gM = (torch.tensor(rng.standard_normal(s)) for s in ((N, C, 8), (N, C, 3), (N, C, 3, 3)))
    ranks = [1, 1, 1, 2, 2, 2, 3, 3]
    inv, V, Mf = node_algebra_ref(*[expand(x, l) for x, l in zip(xs, ranks)], a, b)
    grads = torch.autograd.grad((inv * gI).sum() + (V * gV).sum() + (Mf * gM).sum(), xs + [a, b])
    names = ["P1", "Q1", "S1", "P2", "Q2", "S2", "P3", "Q3"]
    for n_, x, gx in zip(names, xs, grads[:8]):
        out["na_" + n_] = x.detach().numpy()
        out["na_d" + n_] = gx.numpy()
    out.update({"na_a": a.detach().numpy(), "na_b": b.detach().numpy(), "na_gI": gI.numpy(), "na_gV": gV.numpy(),
                "na_gM": gM.numpy(), "na_inv": inv.detach().numpy(), "na_V": V.detach().numpy(),
                "na_Mf": Mf.detach().numpy(), "na_da": grads[8].numpy(), "na_db": grads[9].numpy()})
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)
    print("kernels: factor_density x2, node_algebra")


def electrostatics_cases(ref):
    from face.electrostatics import LatentCharges, pme_recip_energy, KE
    torch.set_default_dtype(torch.float64)
    out = {}
    # random charges in a skewed orthorhombic box (face-mlip tests/test_electrostatics.py:140-154 setting)
    rng = np.random.default_rng(3)
    L, n = 12.0, 60
    pos = rng.uniform(0, L, (n, 3))
    cell = np.diag([L, 0.9 * L, 1.1 * L])
    q = rng.normal(0, 0.5, n); q -= q.mean()
    st = systems.Structure(pos, np.ones(n, np.int64), cell, True)
    i, j, S = nlist.neighbor_list_ijS(pos, cell, True, 5.0)
    pr = (torch.tensor(i), torch.tensor(j), torch.tensor(nlist.shift_vectors(S, cell)))
    for use_pme in (False, True):
        es = LatentCharges(8, sigma=0.5)
        es.use_pme = use_pme
        p = torch.tensor(pos, requires_grad=True)
        e = es.ewald_energy(torch.tensor(q), p, torch.tensor(cell), pr)
        f = -torch.autograd.grad(e, p)[0]
        tag = "pme" if use_pme else "exact"
        out[f"rand_{tag}_e"] = np.array(float(e)); out[f"rand_{tag}_f"] = f.numpy()
    out.update(rand_pos=pos, rand_cell=cell, rand_q=q, rand_gp=np.array(LatentCharges(8, sigma=0.5).gp),
               rand_kcut=np.array(LatentCharges(8, sigma=0.5).kcut))
    # PME reciprocal energy alone at an explicit mesh, alpha = 0.32 (benchmark configuration 2 setting)
    p = torch.tensor(pos, requires_grad=True)
    qq = torch.tensor(q, requires_grad=True)
    e = pme_recip_energy(qq, p, torch.tensor(cell), 1 / 0.32, spacing=L * 0.9 / 20 * (1 + 1e-9))
    gp_, gq_ = torch.autograd.grad(e, (p, qq))
    out.update(recip_e=np.array(float(e)), recip_dpos=gp_.numpy(), recip_dq=gq_.numpy())
    np.savez_compressed(os.path.join(HERE, "electrostatics.npz"), **out)
    print(f"electrostatics: exact {out['rand_exact_e']:.8f} pme {out['rand_pme_e']:.8f} recip {out['recip_e']:.8f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the face-mlip reference (read-only)")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    if not os.path.isdir(os.path.join(a.ref, "face")):
        sys.exit(f"reference package not found at {a.ref}")
    sys.path.insert(0, a.ref)
    torch.set_num_threads(max(1, os.cpu_count()))
    for c in CASES:
        if not a.only or a.only == c[0] or (a.only.endswith("*") and c[0].startswith(a.only[:-1])):
            run_model_case(a.ref, *c)
    if not a.only or a.only == "kernels":
        kernel_cases(a.ref)
    if not a.only or a.only == "electrostatics":
        electrostatics_cases(a.ref)


if __name__ == "__main__":
    main()
