"""Seeded synthetic structures for the five benchmark configurations.

The reference benchmarks on periodic boxes of aspirin molecules built from the rMD17 data set
(face-mlip `tools/bench.py:18-30`), which is not redistributed.  These generators stand in for it with
seeded inputs of the shapes, sizes and value distributions named by the benchmark configurations:

  cfg1  108-atom fcc 3x3x3 conventional, a=3.61, N(0, 0.05^2) displacements, Z=29 (periodic)
  cfg2  1,000-atom rock salt 5x5x5, a=5.64, Z=11/17, sigma=0.05 (periodic, neutral)
  cfg3  batch of non-periodic molecules, 20..40 atoms, H/C/N/O with p=.5/.3/.1/.1, random-walk chains
  cfg4  32,768-atom random 3-element mixture at 0.1 atoms/A^3 with 1.2 A minimum distance (periodic)
  cfg5  1,048,576-atom fcc 64^3, a=3.6, sigma=0.08, 5-element equiatomic random alloy (periodic)

A `Structure` is the minimal ASE-like record the engine needs (positions, numbers, cell, pbc, charge);
the calculator also accepts real `ase.Atoms` through duck typing.
"""
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Structure:
    positions: np.ndarray            # (n,3) float64, Angstrom
    numbers: np.ndarray              # (n,) int64 atomic numbers
    cell: np.ndarray = field(default_factory=lambda: np.zeros((3, 3)))   # rows = lattice vectors
    pbc: bool = False
    charge: float = 0.0

    def __len__(self):
        return len(self.numbers)


def _fcc_positions(n_side, a):
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    g = np.arange(n_side)
    cells = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 1, 3)
    return ((cells + basis[None]) * a).reshape(-1, 3)


def fcc(n_side, a, sigma, elements, seed, equiatomic=True):
    rng = np.random.default_rng(seed)
    pos = _fcc_positions(n_side, a)
    pos = pos + rng.normal(0.0, sigma, pos.shape)
    n = len(pos)
    if len(elements) == 1:
        Z = np.full(n, elements[0], np.int64)
    elif equiatomic:
        Z = np.asarray(elements, np.int64)[rng.permutation(np.arange(n) % len(elements))]
    else:
        Z = rng.choice(np.asarray(elements, np.int64), n)
    return Structure(pos, Z, np.eye(3) * a * n_side, True, 0.0)


def rocksalt(n_side, a, sigma, seed, elements=(11, 17)):
    rng = np.random.default_rng(seed)
    fc = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    basis = np.concatenate([fc, fc + np.array([.5, 0, 0])])          # cation fcc + anion fcc shifted a/2
    kinds = np.array([0] * 4 + [1] * 4)
    g = np.arange(n_side)
    cells = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 1, 3)
    pos = ((cells + basis[None]) * a).reshape(-1, 3)
    Z = np.asarray(elements, np.int64)[np.tile(kinds, len(cells))]
    pos = pos + rng.normal(0.0, sigma, pos.shape)
    return Structure(pos, Z, np.eye(3) * a * n_side, True, 0.0)


def random_mixture(n, density, dmin, elements, seed):
    """Random sequential addition in a periodic cube, rejecting points closer than dmin (cell grid)."""
    rng = np.random.default_rng(seed)
    L = (n / density) ** (1.0 / 3.0)
    nc = max(1, int(L // dmin))
    w = L / nc
    grid = {}
    pos = np.empty((n, 3))
    k = 0
    offs = np.array([(i, j, l) for i in (-1, 0, 1) for j in (-1, 0, 1) for l in (-1, 0, 1)])
    while k < n:
        batch = rng.uniform(0.0, L, (4096, 3))
        for p in batch:
            c = np.floor(p / w).astype(np.int64) % nc
            ok = True
            for o in offs:
                cc = tuple((c + o) % nc)
                for q in grid.get(cc, ()):
                    d = p - pos[q]
                    d -= L * np.round(d / L)
                    if d @ d < dmin * dmin:
                        ok = False
                        break
                if not ok:
                    break
            if ok:
                pos[k] = p
                grid.setdefault(tuple(c), []).append(k)
                k += 1
                if k == n:
                    break
    Z = np.asarray(elements, np.int64)[rng.permutation(np.arange(n) % len(elements))]
    return Structure(pos, Z, np.eye(3) * L, True, 0.0)


def molecule(n, seed, step=(1.0, 1.5), h_jitter=0.15, min_sep=0.9):
    """Self-avoiding random-walk chain: heavy/H atoms with p = .5/.3/.1/.1 for H/C/N/O."""
    rng = np.random.default_rng(seed)
    Z = rng.choice(np.array([1, 6, 7, 8]), n, p=[0.5, 0.3, 0.1, 0.1]).astype(np.int64)
    pos = np.zeros((n, 3))
    for k in range(1, n):
        for _ in range(100):
            d = rng.normal(size=3)
            d /= np.linalg.norm(d)
            p = pos[k - 1] + d * rng.uniform(*step)
            if np.min(np.linalg.norm(pos[:k] - p, axis=1)) >= min_sep:
                break
        pos[k] = p
    h = Z == 1
    pos[h] += rng.normal(0.0, h_jitter, (int(h.sum()), 3))
    return Structure(pos, Z, np.zeros((3, 3)), False, 0.0)


def molecule_batch(n_mol, seed, n_range=(20, 40)):
    rng = np.random.default_rng(seed)
    sizes = rng.integers(n_range[0], n_range[1] + 1, n_mol)
    seeds = rng.integers(0, 2 ** 31, n_mol)
    return [molecule(int(s), int(sd)) for s, sd in zip(sizes, seeds)]


# --------------------------------------------------------------------------------------------- configs
# Model form per configuration (face-mlip flagship form: factorised blocks with transport + equivariant
# messages, B=16, K=32, K_dir=16, unit-parameterised linear layers; `max_body` = correlation order + 1).
MODELS = {
    1: dict(elements=[29], C=32, n_basis=8, rc=5.0, n_passes=1, terms=(), max_body=4),
    2: dict(elements=[11, 17], C=32, n_basis=8, rc=6.0, n_passes=2, terms=("coulomb",), max_body=5,
            pme=dict(gp=1 / 0.32, mesh=(48, 48, 48))),
    3: dict(elements=[1, 6, 7, 8], C=64, n_basis=8, rc=5.0, n_passes=2, terms=(), max_body=5),
    4: dict(elements=[8, 12, 14], C=64, n_basis=16, rc=5.5, n_passes=2, terms=("coulomb",), max_body=5,
            pme=dict(gp=1 / 0.32, mesh=(96, 96, 96))),
    5: dict(elements=[24, 25, 26, 27, 28], C=64, n_basis=8, rc=5.0, n_passes=2, terms=("coulomb",),
            max_body=5, pme=dict(gp=1 / 0.32, mesh=(256, 256, 256))),
}
FLAGSHIP = dict(radial_hidden=64, K_dir=16, norm="layer", transport=True, eqmsg=True, factor=True,
                B=16, K=32, cp=False, unit=True)


def model_kwargs(cfg, **over):
    kw = dict(FLAGSHIP)
    kw.update({k: v for k, v in MODELS[cfg].items() if k not in ("pme",)})
    kw.update(over)
    return kw


def config_structures(cfg, seed=0, scale=None):
    """Structures for configuration `cfg`.  `scale` shrinks the system for parity cases:
    cfg1/2/5 -> conventional cells per side, cfg3 -> number of molecules, cfg4 -> number of atoms."""
    if cfg == 1:
        return [fcc(scale or 3, 3.61, 0.05, [29], seed)]
    if cfg == 2:
        return [rocksalt(scale or 5, 5.64, 0.05, seed)]
    if cfg == 3:
        return molecule_batch(scale or 512, seed)
    if cfg == 4:
        return [random_mixture(scale or 32768, 0.1, 1.2, MODELS[4]["elements"], seed)]
    if cfg == 5:
        return [fcc(scale or 64, 3.6, 0.08, MODELS[5]["elements"], seed)]
    raise ValueError(cfg)
