"""GPU cell-list neighbour build against the fp64 enumerator of ASE's ijS semantics (oracle/nlist.py): the edge
sets must agree bit for bit, shift vectors exactly, reverse indices must be consistent, and the padded export must
equal the oracle's padded graph."""
import numpy as np
import pytest
import torch

from oracle import nlist

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _cases():
    from face_b200 import systems
    S = systems.Structure
    rng = np.random.default_rng(11)
    skew = np.array([[9.0, 0.0, 0.0], [2.5, 8.0, 0.0], [1.5, -2.0, 10.0]])
    tri = S(rng.uniform(-2, 12, (90, 3)), rng.choice([24, 25], 90), skew, True)         # triclinic, unwrapped atoms
    tiny = S(rng.uniform(0, 4.2, (7, 3)), np.full(7, 29), np.diag([4.2, 4.6, 5.1]), True)  # L < rc: many images
    return [("cfg1", systems.config_structures(1, 0), 5.0), ("cfg2", systems.config_structures(2, 0), 6.0),
            ("cfg3", systems.config_structures(3, 0, scale=12), 5.0),
            ("cfg4", systems.config_structures(4, 0, scale=2000), 5.5),
            ("cfg5", systems.config_structures(5, 0, scale=6), 5.0), ("triclinic", [tri], 5.0), ("tiny", [tiny], 5.0)]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_edge_set_bit_exact(case):
    from face_b200.neighbors import build_graph
    name, structs, rc = case
    g = build_graph(structs, rc, dtype=torch.float64)
    ei, ej, S = g["ei"].cpu().numpy(), g["ej"].cpu().numpy(), g["S"].cpu().numpy()
    offs = np.concatenate([[0], np.cumsum([len(s.numbers) for s in structs])])
    I, J, SS, SH = [], [], [], []
    for k, st in enumerate(structs):
        i, j, s = nlist.neighbor_list_ijS(st.positions, st.cell, bool(np.any(st.pbc)), rc)
        I.append(i + offs[k]); J.append(j + offs[k]); SS.append(s)
        SH.append(nlist.shift_vectors(s, np.asarray(st.cell, np.float64)) if np.any(st.pbc) else np.zeros((len(i), 3)))
    I, J, SS, SH = np.concatenate(I), np.concatenate(J), np.concatenate(SS), np.concatenate(SH)
    # identical arrays: same set and same canonical (i, j, S) order
    assert len(ei) == len(I), (name, len(ei), len(I))
    assert np.array_equal(ei, I) and np.array_equal(ej, J) and np.array_equal(S, SS), name
    assert np.array_equal(g["shift"].cpu().numpy(), SH), name
    rp = g["row_ptr"].cpu().numpy()
    assert np.array_equal(rp, np.concatenate([[0], np.cumsum(np.bincount(I, minlength=offs[-1]))]))
    rev = g["rev"].cpu().numpy()
    assert (rev >= 0).all() and np.array_equal(ei[rev], ej) and np.array_equal(ej[rev], ei)
    assert np.array_equal(S[rev], -S) and np.array_equal(rev[rev], np.arange(len(rev)))


def test_padded_export_matches_reference_layout():
    from face_b200 import systems
    from face_b200.neighbors import padded_graph
    structs = systems.config_structures(3, 0, scale=5)
    gp = padded_graph(structs, 5.0, dtype=torch.float64)
    go = nlist.padded_graph(structs, 5.0)
    for k in ("nbr", "mask", "shift", "batch"):
        assert np.array_equal(gp[k].cpu().numpy(), go[k]), k


def test_full_size_alloy_properties():
    """1,048,576-atom alloy: symmetric, bit-exact on a random sample of rows (minimum-image brute force)."""
    from face_b200 import systems
    from face_b200.neighbors import build_graph
    st = systems.config_structures(5, 0)[0]
    g = build_graph([st], 5.0, dtype=torch.float32)
    N = len(st.numbers)
    rp = g["row_ptr"].cpu().numpy()
    deg = np.diff(rp)
    assert deg.min() > 20 and deg.max() < 80
    rev = g["rev"].cpu().numpy()
    ei, ej, S = g["ei"].cpu().numpy(), g["ej"].cpu().numpy(), g["S"].cpu().numpy()
    assert np.array_equal(rev[rev], np.arange(len(rev))) and np.array_equal(ei[rev], ej)
    rng = np.random.default_rng(0)
    pos, cell = st.positions, st.cell
    L = np.diag(cell)
    for i in rng.choice(N, 64, replace=False):
        d = pos - pos[i]
        s = -np.round(d / L)                                 # L >> 2 rc: one image per pair
        sv = nlist.shift_vectors(s.astype(np.int64), cell)
        r = np.sqrt(((pos - pos[i]) + sv) ** 2 @ np.ones(3))
        dd = (pos - pos[i]) + sv
        r = np.sqrt((dd[:, 0] * dd[:, 0] + dd[:, 1] * dd[:, 1]) + dd[:, 2] * dd[:, 2])
        want = {(int(j), *map(int, s[j])) for j in np.nonzero((r < 5.0) & (np.arange(N) != i))[0]}
        got = {(int(j), *map(int, sj)) for j, sj in zip(ej[rp[i]:rp[i + 1]], S[rp[i]:rp[i + 1]])}
        assert got == want, i
