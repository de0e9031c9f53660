"""ORACLE (test infrastructure only -- never imported by the product path).

CPU restatement, in numpy float64, of the neighbour list the reference builds with ASE and pads into its
graph dict:

* face-mlip `face/neighbors.py:7-37` (`padded_graph`) and `face/datasets.py:47-57,62-97` (`GraphSet`)
  call `ase.neighborlist.neighbor_list("ijS", atoms, rc)` (ase==3.29.0, `requirements.txt:5`; not
  vendored, not installed here).  Its published contract: every (i, j, S) with
  |pos[j] - pos[i] + S @ cell| < rc, the zero-shift self pair excluded, periodic self images included;
  non-periodic structures give all pairs i != j closer than rc.  Distances are fp64.
* The reference then sorts the triples stably by centre i (`face/neighbors.py:14`,
  `face/datasets.py:75`), computes shift = S @ cell (zeros when not periodic, `face/datasets.py:52`), fills
  row slots in that order, pads each row to M = max degree with mask=False, nbr=first atom of the
  structure, shift=0 (`face/datasets.py:74-79`), and offsets indices by the structure's first atom.

ASE's within-row order is an implementation detail of its binning; here rows are in canonical
(j, S0, S1, S2) order.  The energy is a sum over edges, so only the edge SET is part of the contract,
and the GPU builder is checked against this enumerator as a set (bit-exact (i, j, S) triples and shift
vectors).  No ASE golden vectors exist for this path, so the enumerator itself is anchored only on its
definition (parity unpinned against ASE itself).

Distance arithmetic follows a fixed order that the GPU kernel repeats exactly (no fused multiply-add):
  sv = S0*cell[0] + S1*cell[1] + S2*cell[2];  d = (pos[j] - pos[i]) + sv;  |d| = sqrt((dx*dx + dy*dy) + dz*dz)
"""
import numpy as np


def _heights(cell):
    V = abs(np.linalg.det(cell))
    a, b, c = cell
    return np.array([V / np.linalg.norm(np.cross(b, c)), V / np.linalg.norm(np.cross(c, a)),
                     V / np.linalg.norm(np.cross(a, b))])


def shift_vectors(S, cell):
    S = S.astype(np.float64)
    return (S[:, 0:1] * cell[0][None] + S[:, 1:2] * cell[1][None]) + S[:, 2:3] * cell[2][None]


def _dist(pos, i, j, sv):
    d = (pos[j] - pos[i]) + sv
    return np.sqrt((d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2])


def neighbor_list_ijS(positions, cell, pbc, rc, chunk=256):
    """(i, j, S) int arrays, canonical order (i, j, S0, S1, S2)."""
    pos = np.asarray(positions, np.float64)
    n = len(pos)
    cell = np.asarray(cell, np.float64)
    if n == 0:
        z = np.zeros(0, np.int64)
        return z, z, np.zeros((0, 3), np.int64)
    if not pbc:
        I, J = [], []
        for a in range(0, n, chunk):
            d = pos[None, :, :] - pos[a:a + chunk, None, :]
            r = np.sqrt((d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2])
            ii, jj = np.nonzero(r < rc)
            ii = ii + a
            keep = ii != jj
            I.append(ii[keep]); J.append(jj[keep])
        I, J = np.concatenate(I), np.concatenate(J)
        S = np.zeros((len(I), 3), np.int64)
    else:
        inv = np.linalg.inv(cell)
        frac = pos @ inv
        w = np.floor(frac)
        pw = pos - w @ cell                                      # wrapped into the cell
        m = np.ceil(rc / _heights(cell)).astype(np.int64)
        rng = [np.arange(-m[d], m[d] + 1) for d in range(3)]
        imgs = np.stack(np.meshgrid(*rng, indexing="ij"), -1).reshape(-1, 3)
        isv = imgs.astype(np.float64) @ cell                     # candidate filter only
        # candidates: every (i, j, image) whose wrapped-frame distance is below rc + 1e-6, from a k-d tree over all
        # images of the wrapped atoms (a superset of the pairs the exact test below keeps)
        from scipy.spatial import cKDTree
        pts = (pw[None, :, :] + isv[:, None, :]).reshape(-1, 3)  # index = image * n + j
        tree = cKDTree(pts)
        I, J, S = [], [], []
        for a in range(0, n, 4096):
            hits = tree.query_ball_point(pw[a:a + 4096], rc + 1e-6)
            cnt = np.fromiter((len(h) for h in hits), np.int64, len(hits))
            flat = np.fromiter((x for h in hits for x in h), np.int64, int(cnt.sum()))
            ii = np.repeat(np.arange(a, a + len(hits)), cnt)
            kk, jj = flat // n, flat % n
            I.append(ii); J.append(jj)
            # shift in the original (unwrapped) frame: pw_j - pw_i + s.cell = pos_j - pos_i + (s - w_j + w_i).cell
            S.append(imgs[kk] - w[jj].astype(np.int64) + w[ii].astype(np.int64))
        I, J, S = np.concatenate(I), np.concatenate(J), np.concatenate(S)
        sv = shift_vectors(S, cell)
        keep = (_dist(pos, I, J, sv) < rc) & ~((I == J) & (S == 0).all(1))
        I, J, S = I[keep], J[keep], S[keep]
    order = np.lexsort((S[:, 2], S[:, 1], S[:, 0], J, I))
    return I[order].astype(np.int64), J[order].astype(np.int64), S[order].astype(np.int64)


def padded_graph(structures, rc, dtype=np.float64):
    """Reference graph dict (numpy) for a batch of structures (face/datasets.py:62-97 layout)."""
    rows, off = [], 0
    for st in structures:
        n = len(st.numbers)
        pbc = bool(np.any(st.pbc))
        i, j, S = neighbor_list_ijS(st.positions, st.cell, pbc, rc)
        sv = shift_vectors(S, np.asarray(st.cell, np.float64)) if pbc else np.zeros((len(i), 3))
        rows.append((st, i, j, S, sv, np.bincount(i, minlength=n), off))
        off += n
    N = off
    M = max(1, max((int(r[5].max()) if len(r[5]) else 1) for r in rows))
    NB = np.zeros((N, M), np.int64)
    SH = np.zeros((N, M, 3))
    SI = np.zeros((N, M, 3), np.int64)
    MK = np.zeros((N, M), bool)
    pos, Z, bt, cell, Q = [], [], [], [], []
    for k, (st, i, j, S, sv, cnt, o) in enumerate(rows):
        n = len(st.numbers)
        if len(i):
            start = np.concatenate([[0], np.cumsum(cnt)[:-1]])
            slot = np.arange(len(i)) - start[i]
            NB[o + i, slot] = o + j
            SH[o + i, slot] = sv
            SI[o + i, slot] = S
            MK[o + i, slot] = True
        NB[o:o + n][~MK[o:o + n]] = o
        pos.append(np.asarray(st.positions, np.float64)); Z.append(np.asarray(st.numbers, np.int64))
        bt.append(np.full(n, k))
        cell.append(np.asarray(st.cell, np.float64) if np.any(st.pbc) else np.zeros((3, 3)))
        Q.append(float(getattr(st, "charge", 0.0)))
    return {"pos": np.concatenate(pos).astype(dtype), "Z": np.concatenate(Z), "nbr": NB,
            "shift": SH.astype(dtype), "S": SI, "mask": MK, "batch": np.concatenate(bt),
            "cell": np.stack(cell).astype(dtype), "charge": np.asarray(Q, dtype),
            "natoms": np.asarray([len(r[0].numbers) for r in rows]), "nstr": len(rows)}


def edge_set(i, j, S):
    """Canonical set view of a neighbour list for exact comparison."""
    return {(int(a), int(b), int(s0), int(s1), int(s2)) for a, b, (s0, s1, s2) in zip(i, j, S)}
