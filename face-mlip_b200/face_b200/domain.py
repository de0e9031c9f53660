"""Multi-GPU evaluation: spatial decomposition of a periodic system with a per-pass halo exchange, one process per
GPU; batches of independent molecules sharded by structure.

Periodic systems.  The box (orthorhombic) is split into a grid of bricks (2x1x1, 2x2x1, 2x2x2, ...), one per rank.
A rank owns the atoms of its brick and holds, as ghosts, every atom within rc of the brick along the split axes (at
the periodic image nearest the brick).  Along unsplit axes the local system keeps the full periodicity, and the
local extent along split axes stays below L - rc, so the local neighbour list is the ordinary periodic build with
the original cell.  Coupling, all through one differentiable halo exchange (HaloExchange: an all-to-all of the
ghost rows from their owners forward, and of the ghost gradients back to the owners, summed into the owned rows):

  * positions: each rank holds only its owned atoms' coordinates; ghost coordinates come from their owners (plus the
    periodic image shift), and the gradient with respect to a ghost's coordinates goes back to its owner, which is
    the reverse sum of ghost forces: no global position array and no N x 3 all-reduce;
  * pass features: after every pass but the last, the ghosts' features that the next pass reads at a neighbour
    (h, and the equivariant tensors V, M or the previous moment sets) are replaced by their owners' values, so the
    next pass of every owned atom is exact although the ghost shell is only rc deep (face-mlip face/model.py:479-483
    makes exactly these per-atom quantities available to the neighbour messages);
  * latent charges: the two neutrality sums are all-reduced scalars (face/electrostatics.py:165-167), the charges of
    ghosts come through the halo exchange for the real-space rows, and the PME reciprocal sum is mesh-distributed
    (SlabPME: each rank spreads its owned charges, reduce-scatter into x-slabs, 2-D FFT, all-to-all transpose, 1-D
    FFT);
  * energy: one all-reduced scalar.
Ghost rows keep only their edges to owned atoms (the reverse edges the adjoint gathers need): their outputs are
overwritten by the halo or dropped, so ghost-ghost edges would be wasted work.
Every rank runs the same collectives in the same order, forward and backward.
"""
import json
import math
import os
import statistics
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

KE = 14.399645


def brick_grid(world):
    """Most cubic factorisation nx >= ny >= nz of the world size."""
    best = None
    for nx in range(1, world + 1):
        if world % nx:
            continue
        for ny in range(1, world // nx + 1):
            if (world // nx) % ny:
                continue
            nz = world // (nx * ny)
            g = tuple(sorted((nx, ny, nz), reverse=True))
            score = max(g) / min(g)
            if best is None or score < best[0]:
                best = (score, g)
    return best[1]


def select_local(pos, L, grid, rank, halo):
    """Owned atoms and ghost images of brick `rank` (row-major over grid).  pos (N,3) float64 on any device, L (3,)
    box lengths.  Returns gid (local -> global index, sorted), img (local image shift, so that local position =
    pos[gid] + img), owned (bool)."""
    dev = pos.device
    Lt = torch.as_tensor(L, dtype=torch.float64, device=dev)
    f = pos / Lt
    fl = torch.floor(f)
    fw = f - fl                                                   # wrapped fractional coordinates in [0, 1)
    n = torch.as_tensor(grid, device=dev)
    b = torch.clamp((fw * n).long(), max=n - 1)
    rb = [(rank // (grid[1] * grid[2])) % grid[0], (rank // grid[2]) % grid[1], rank % grid[2]]
    owned = (b[:, 0] == rb[0]) & (b[:, 1] == rb[1]) & (b[:, 2] == rb[2])
    keep = torch.ones(pos.shape[0], dtype=torch.bool, device=dev)
    img = torch.zeros_like(pos)
    for d in range(3):
        if grid[d] == 1:
            continue
        lo, hi = rb[d] / grid[d], (rb[d] + 1) / grid[d]
        ks = torch.tensor([-1.0, 0.0, 1.0], dtype=torch.float64, device=dev)
        x = fw[:, d, None] + ks[None]                             # candidate images
        dd = torch.clamp(torch.maximum(lo - x, x - hi), min=0.0) * float(L[d])
        best = dd.argmin(1)
        keep &= dd.gather(1, best[:, None])[:, 0] <= halo
        img[:, d] = (ks[best] - fl[:, d]) * float(L[d])           # wrapped position + k L - original position
    local = keep | owned
    gid = torch.nonzero(local)[:, 0]
    return gid, img[gid], owned[gid]


class LocalSystem:
    """Positions-only view of a rank's local atoms (ASE-like for the neighbour builder)."""

    def __init__(self, positions, numbers, cell):
        self.positions = positions
        self.numbers = numbers
        self.cell = cell
        self.pbc = True
        self.charge = 0.0


def brick_of(pos, L, grid):
    """Owning rank (row-major over the grid) of every atom, from its wrapped position."""
    Lt = torch.as_tensor(L, dtype=torch.float64, device=pos.device)
    fw = torch.remainder(pos.double() / Lt, 1.0)
    n = torch.as_tensor(grid, device=pos.device)
    b = torch.clamp((fw * n).long(), max=n - 1)
    return (b[:, 0] * grid[1] + b[:, 1]) * grid[2] + b[:, 2]


class HaloPlan:
    """One rank's owned atoms, rc-deep ghosts and the exchange lists of the halo.

    Local order: owned atoms (ascending global id), then ghosts grouped by owner rank (ascending), ascending global id
    within an owner, so the all-to-all's receive buffer is the ghost block as is.  send_idx lists, peer by peer, the
    owned rows that are ghosts on that peer, in the peer's order.  Built once from the global positions (every rank
    derives every rank's ghost set with the same deterministic selection, so no index lists are exchanged)."""

    def __init__(self, pos, L, grid, rank, world, halo, group=None):
        self.rank, self.world, self.group = rank, world, group
        dev = pos.device
        owner = brick_of(pos, L, grid)
        N = pos.shape[0]

        def ghosts_of(r):
            gid, img, own = select_local(pos, L, grid, r, halo)
            gg, gi = gid[~own], img[~own]
            order = torch.argsort(owner[gg] * N + gg)
            return gid[own], img[own], gg[order], gi[order]

        og, oi, gg, gi = ghosts_of(rank)
        self.gid = torch.cat([og, gg])                       # local -> global id
        self.img = torch.cat([oi, gi])                       # local position = global position + img
        self.n_owned, self.n_ghost = int(og.numel()), int(gg.numel())
        self.n_local = self.n_owned + self.n_ghost
        own_g = gg.new_zeros(0)
        self.recv_counts = [int((owner[gg] == q).sum()) for q in range(world)]
        send, counts = [], []
        for p in range(world):
            if p == rank:
                counts.append(0)
                continue
            _, _, gp, _ = ghosts_of(p)
            mine = gp[owner[gp] == rank]                        # ascending global id (the peer's order)
            send.append(torch.searchsorted(og, mine))
            counts.append(int(mine.numel()))
        self.send_idx = torch.cat(send) if send else og.new_zeros(0)
        self.send_counts = counts
        self.n_send = int(sum(counts))
        del own_g


class HaloExchange(torch.autograd.Function):
    """y = x with its ghost rows (along `dim`) replaced by the owners' rows; x holds the local rows or only the owned
    rows (then the ghost rows are appended).  Adjoint: the ghost rows' gradients go back to the owners (the reverse
    all-to-all) and are added to the owned rows they came from."""

    @staticmethod
    def forward(ctx, x, plan, dim):
        ctx.plan, ctx.dim, ctx.rows = plan, dim, x.shape[dim]
        xs = x.movedim(dim, 0)
        owned = xs[:plan.n_owned]
        if plan.world == 1:
            return owned.movedim(0, dim).contiguous()
        send = owned[plan.send_idx].contiguous()
        recv = xs.new_empty((plan.n_ghost,) + tuple(xs.shape[1:]))
        dist.all_to_all_single(recv, send, plan.recv_counts, plan.send_counts, group=plan.group)
        return torch.cat([owned, recv], 0).movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, g):
        plan, dim = ctx.plan, ctx.dim
        gs = g.movedim(dim, 0)
        go = gs[:plan.n_owned]
        if plan.world > 1:
            back = gs[plan.n_owned:].contiguous()
            recv = gs.new_empty((plan.n_send,) + tuple(gs.shape[1:]))
            dist.all_to_all_single(recv, back, plan.send_counts, plan.recv_counts, group=plan.group)
            go = go.index_add(0, plan.send_idx, recv)
        if ctx.rows > plan.n_owned:
            go = torch.cat([go, gs.new_zeros((ctx.rows - plan.n_owned,) + tuple(gs.shape[1:]))], 0)
        return go.movedim(0, dim).contiguous(), None, None


def halo(x, plan, dim=0):
    return HaloExchange.apply(x, plan, dim)


def pass_exchange(plan, blocks_next, atom_dim):
    """between(t, h, A_sets, eq) for the model's pass loop: the ghosts' features read by pass t + 1 at a neighbour
    come from their owners.  atom_dim: (of h, of each A_sets tensor, of eq tensors)."""
    dh, dA, de = atom_dim

    def between(t, h, A_sets, eq):
        nxt = blocks_next(t + 1)
        h = halo(h, plan, dh)
        if eq is not None:
            eq = (halo(eq[0], plan, de), halo(eq[1], plan, de))
        if nxt.get("directional") and not nxt.get("eq_in"):
            A_sets = [[A[0], halo(A[1], plan, dA), halo(A[2], plan, dA), A[3]] for A in A_sets]
        return h, A_sets, eq
    return between


def rank_energy(pos_owned, plan, local_model, coulomb=None):
    """This rank's share of the total energy as a differentiable function of its owned atoms' positions.

    local_model(pos_local) -> (e_at, h) over the local atoms (owned first; it applies the pass exchange itself).
    coulomb (optional): dict with head(h) -> (chi, J); real_rows(pos_local, q_local) -> e_row; pme_slab(pos_owned,
    q_owned) -> this rank's share of the reciprocal energy; gp, volume, charge (total charge Q).
    Sum over ranks = the system's energy."""
    from torch.distributed.nn import functional as dnn
    no = plan.n_owned
    pos_local = halo(pos_owned, plan, 0) + plan.img.to(pos_owned.dtype)
    e_at, h = local_model(pos_local)
    e = e_at[:no].sum()
    if coulomb is None:
        return e
    chi, J = coulomb["head"](h)
    chi_o, J_o = chi[:no], J[:no]
    allr = (lambda x: dnn.all_reduce(x, group=plan.group)) if plan.world > 1 else (lambda x: x)
    s1 = allr((chi_o / J_o).sum())
    s2 = allr((1.0 / J_o).sum())
    mu = (coulomb["charge"] + s1) / s2
    q_o = -(chi_o - mu) / J_o
    q_loc = halo(q_o, plan, 0)
    e_real = coulomb["real_rows"](pos_local, q_loc)[:no].sum()
    e_recip_share = coulomb["pme_slab"](pos_local[:no], q_o)
    gp = coulomb["gp"]
    self_o = -(q_o * q_o).sum() / (math.sqrt(math.pi) * gp)
    qsum = allr(q_o.sum())
    bg = -0.5 * math.pi * gp ** 2 / coulomb["volume"] * qsum * qsum
    e_es = KE * (e_real + e_recip_share + self_o + bg / plan.world)
    return e + (chi_o * q_o + 0.5 * J_o * q_o * q_o).sum() + e_es


class SlabPME:
    """Smooth-PME reciprocal energy (face/electrostatics.py:54-77) with the mesh distributed over the ranks in slabs.

    Each rank spreads its own atoms' charges onto a full-size mesh (`spread(pos, q) -> (n0*n1*n2,)`, differentiable);
    a reduce-scatter along x leaves rank r the summed x-planes [r*n0/W, (r+1)*n0/W) (the spreading stencil's overlap
    into neighbouring slabs is summed by the same collective).  A 2-D FFT over (y, z) of the slab, an all-to-all that
    trades x-slabs for y-slabs, and a 1-D FFT along x give the rank the full structure factor S(k) for its k_y
    block; its energy share is 1/(2V) sum G(k) |b(k)|^2 |S(k)|^2 over that block, and the shares sum to the energy.
    All collectives are the differentiable ones of torch.distributed.nn, so forces and charge gradients flow back
    through the transposes to the spreading adjoint (the gather).  n0 and n1 must be multiples of the world size."""

    def __init__(self, cell64, gp, mesh, rank, world, spread, dtype, device, group=None):
        n0, n1, n2 = (int(n) for n in mesh)
        if n0 % world or n1 % world:
            raise ValueError(f"PME mesh {mesh} not divisible into {world} slabs along x and y")
        self.mesh, self.rank, self.world, self.group, self.spread = (n0, n1, n2), rank, world, group, spread
        cell = np.asarray(cell64, np.float64)
        inv = np.linalg.inv(cell)
        self.volume = abs(float(np.linalg.det(cell)))
        nb = n1 // world
        m = [np.fft.fftfreq(n, 1.0 / n) for n in (n0, n1, n2)]
        m[1] = m[1][rank * nb:(rank + 1) * nb]
        mg = np.stack(np.meshgrid(*m, indexing="ij"), -1)
        k = 2 * math.pi * mg @ inv.T
        k2 = (k * k).sum(-1)
        G = np.where(k2 > 1e-12, 4 * math.pi / np.maximum(k2, 1e-12) * np.exp(-gp ** 2 * k2 / 4), 0.0)
        bm = [_bspline_modulus2(n) for n in (n0, n1, n2)]
        Bm = bm[0][:, None, None] * bm[1][None, rank * nb:(rank + 1) * nb, None] * bm[2][None, None, :]
        self.gfac = torch.as_tensor(0.5 / self.volume * G * Bm, dtype=dtype, device=device)

    def __call__(self, pos, q):
        from torch.distributed.nn import functional as dnn
        n0, n1, n2 = self.mesh
        W = self.world
        grid = self.spread(pos, q).view(n0, n1, n2)
        if W > 1:
            slab = dnn.reduce_scatter(grid.new_empty(n0 // W, n1, n2), list(grid.chunk(W, 0)), group=self.group)
        else:
            slab = grid
        A = torch.fft.fft2(slab, dim=(1, 2))                                  # (n0/W, n1, n2), this x-slab
        if W > 1:
            send = [c.contiguous() for c in torch.view_as_real(A).chunk(W, 1)]  # y-blocks of the x-slab
            recv = dnn.all_to_all([torch.empty_like(send[0]) for _ in range(W)], send, group=self.group)
            A = torch.view_as_complex(torch.cat(list(recv), 0).contiguous())  # (n0, n1/W, n2), this y-block
        S = torch.fft.fft(A, dim=0)
        return (self.gfac * (S.real * S.real + S.imag * S.imag)).sum()


def _bspline_modulus2(n):
    """|b(m)|^-2 of the order-4 B-spline interpolation (Essmann et al. 1995; face/electrostatics.py:44-51)."""
    m = np.arange(n, dtype=np.float64)
    w = np.array([1 / 6, 4 / 6, 1 / 6])
    ang = 2 * math.pi * m[:, None] * np.arange(3)[None] / n
    den = (w * np.cos(ang)).sum(-1) ** 2 + (w * np.sin(ang)).sum(-1) ** 2
    return 1.0 / np.maximum(den, 1e-10)


# --------------------------------------------------------------------------------------------- GPU engine
class DistributedModel:
    """Energy and forces of one periodic structure on `world` GPUs (this process = one rank), with the per-pass halo
    exchange.  `energy_forces(pos_owned)` takes this rank's owned positions (global ids `gid_owned`, in that order)
    and returns (total energy, forces on the owned atoms)."""

    def __init__(self, model, structure, rank, world, device, dtype=torch.float32, group=None, pme="slab"):
        from . import ops
        if pme != "slab":
            raise ValueError("the halo decomposition distributes the PME mesh in slabs (pme='slab')")
        self.ops, self.pme_mode = ops, pme
        self.model, self.rank, self.world, self.dev, self.dtype, self.group = model, rank, world, device, dtype, group
        cell = np.asarray(structure.cell, np.float64)
        if np.abs(cell - np.diag(np.diag(cell))).max() > 0:
            raise NotImplementedError("spatial decomposition needs an orthorhombic cell")
        self.L = np.diag(cell).copy()
        self.cell64 = cell
        self.grid = brick_grid(world)
        self.halo = model.rc
        for d in range(3):
            if self.grid[d] > 1 and self.L[d] / self.grid[d] + 2 * self.halo + model.rc >= self.L[d]:
                raise ValueError(f"box too small for a {self.grid} decomposition with halo {self.halo} A")
        self.Q = float(getattr(structure, "charge", 0.0))
        pos = torch.as_tensor(np.asarray(structure.positions), dtype=torch.float64, device=device)
        self.plan = HaloPlan(pos, self.L, self.grid, rank, world, self.halo, group)
        self.gid_owned = self.plan.gid[:self.plan.n_owned]
        self.Z_local = torch.as_tensor(np.asarray(structure.numbers), dtype=torch.long, device=device)[self.plan.gid]
        self.pos_owned = pos[self.gid_owned].to(dtype)          # this rank's coordinates (the only ones it keeps)
        self.rebuild(pos[self.gid_owned])
        self._slab = None
        self.coulomb = None
        if "coulomb" in model.terms:
            tm = model.terms["coulomb"]
            mesh = tm.mesh or tuple(max(8, int(math.ceil(L / (tm.gp / 4.0)))) for L in self.L)
            cell64, mesh_t = self.cell64, tuple(mesh)
            self._slab = SlabPME(cell64, float(tm.gp), mesh_t, rank, world,
                                 lambda p, q: ops.SpreadMesh.apply(p, q.contiguous(), cell64, mesh_t), dtype, device,
                                 group)
            self.coulomb = {"head": self.head, "real_rows": self.real_rows, "pme_slab": self._slab,
                            "gp": float(tm.gp), "volume": float(abs(np.linalg.det(cell))), "charge": self.Q}

    def rebuild(self, pos_owned64):
        """Local neighbour list from this rank's owned float64 positions: ghost coordinates from their owners through
        the halo, the list built on the device."""
        from .neighbors import keep_edges, periodic_graph_device
        with torch.no_grad():
            loc = halo(pos_owned64.contiguous(), self.plan, 0) + self.plan.img
        g = periodic_graph_device(loc, self.Z_local, self.cell64, self.model.rc, self.dtype)
        # ghost-ghost edges only feed ghost rows, whose outputs the halo overwrites (pass 1) or the energy drops
        # (last pass): keep the edges that touch an owned atom (a symmetric condition, so reverse edges stay)
        no = self.plan.n_owned
        self.graph = keep_edges(g, (g["ei"] < no) | (g["ej"] < no)) if self.world > 1 else g

    # engine callables of rank_energy
    def local_model(self, pos_local):
        P = self.ops.prepare(self.model, self.dtype, pos_local.device)
        between = pass_exchange(self.plan, lambda t: P["blocks"][t], (0, 1, 1))
        e_at, h, P, gr, geo = self.ops.local_energies(self.model, self.graph, pos_local, between=between)
        self.P, self.gr, self.geo = P, gr, geo
        return e_at, h

    def head(self, h):
        import torch.nn.functional as F
        c = self.P["coulomb"]
        chi, hard = self.ops._layer(c["h2"], F.silu(self.ops._layer(c["h0"], h))).unbind(-1)
        return chi, F.softplus(hard) + 0.1

    def real_rows(self, pos_local, q_local):
        c = self.P["coulomb"]
        return self.ops.CoulombReal.apply(self.geo["vec"], q_local.contiguous(), self.gr, c["gamma"], c["gp"])

    def energy_forces(self, pos_owned=None):
        """pos_owned: (n_owned, 3) model-dtype device tensor (default: the positions given at construction).
        Returns (E_total on every rank, forces on the owned atoms)."""
        pos = (self.pos_owned if pos_owned is None else pos_owned).detach().requires_grad_(True)
        e = rank_energy(pos, self.plan, self.local_model, self.coulomb)
        (g,) = torch.autograd.grad(e, pos)
        et = e.detach().reshape(1).clone()
        if self.world > 1:
            dist.all_reduce(et, group=self.group)
        return et[0], -g


# --------------------------------------------------------------------------------------------- structure sharding
def shard_structures(natoms, world):
    """Independent structures (a molecule batch) to ranks, balanced by atom count.

    Largest structure first, each to the rank with the fewest atoms so far (ties to the lower rank), so every rank's
    share is within one structure of the mean.  Returns one ascending index array per rank (possibly empty when there
    are fewer structures than ranks)."""
    natoms = np.asarray(natoms, np.int64)
    load = np.zeros(world, np.int64)
    own = [[] for _ in range(world)]
    for s in np.argsort(-natoms, kind="stable"):
        r = int(np.argmin(load))
        own[r].append(int(s))
        load[r] += natoms[s]
    return [np.array(sorted(o), np.int64) for o in own]


class ShardedBatch:
    """Energies and forces of a batch of independent non-periodic structures on `world` GPUs (this process = one rank).

    face-mlip evaluates a batch in one `FACE.forward` and sums atom energies per structure with `index_add` over
    `batch` (face/model.py:680-695); structures never interact, so each rank evaluates only its own share
    (`shard_structures`) and the data path has no collective.  One all-reduce of the zero-filled per-structure energy
    vector (each entry written by exactly one rank) gives every rank the batch's energies; forces stay on the rank
    that owns the structure, in the order of `self.ids`.

    `evaluate(structures) -> (energy (n,), forces (atoms, 3))` evaluates a list of structures on this rank; the
    default builds the engine's CSR graph and runs `model`."""

    def __init__(self, model, structures, rank, world, device, dtype=torch.float32, group=None, evaluate=None):
        self.rank, self.world, self.dev, self.dtype, self.group = rank, world, device, dtype, group
        self.nstr = len(structures)
        self.ids = shard_structures([len(s.numbers) for s in structures], world)[rank]
        self.local = [structures[i] for i in self.ids]
        self.n_local_atoms = int(sum(len(s.numbers) for s in self.local))
        self.model = model
        self.evaluate = evaluate or self._engine
        self.graph = None
        if evaluate is None and self.local:
            from .neighbors import build_graph
            self.graph = build_graph(self.local, model.rc, device=device, dtype=dtype)

    def _engine(self, structures):
        out = self.model(dict(self.graph, pos=self.graph["pos"].detach().clone()))
        return out["energy"].detach(), out["forces"]

    def energy_forces(self):
        """Returns (energies of all structures (nstr,), forces of this rank's atoms (n_local_atoms, 3))."""
        E = torch.zeros(self.nstr, dtype=self.dtype, device=self.dev)
        if self.local:
            e, F = self.evaluate(self.local)
            E[torch.as_tensor(self.ids, device=self.dev)] = e.to(self.dtype)
        else:
            F = torch.zeros(0, 3, dtype=self.dtype, device=self.dev)
        if self.world > 1:
            dist.all_reduce(E, group=self.group)
        return E, F


# --------------------------------------------------------------------------------------------- benchmark
def bench_multi(a):
    """bench.py --gpus N under torchrun: the 1,048,576-atom alloy decomposed over N GPUs (strong scaling)."""
    import datetime
    if a.config == 3:
        return bench_sharded(a)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench as B
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        dtype = torch.float64 if a.config == 1 else torch.float32
        structs, spec, pme = B.workload(a.config, scale=a.scale)
        if a.scale and a.config == 5:
            pme["mesh"] = tuple(max(8, int(round(n * a.scale / 64))) for n in pme["mesh"])
        model = B.make_model(spec, pme, dev, dtype)
        st = structs[0]
        natoms = len(st.numbers)
        dm = DistributedModel(model, st, rank, world, dev, dtype, pme="slab")
        pos = dm.pos_owned                                   # this rank's owned coordinates only
        n_local = dm.plan.n_local
        for _ in range(a.warmup):
            dm.energy_forces(pos)
        torch.cuda.synchronize()
        dist.barrier()
        from . import _lib, perf
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        perf.start()
        _lib.CALLS.clear()
        _lib.COUNTING = True
        with B.Clocks(local) as clk:
            torch.cuda.synchronize()
            dist.barrier()
            e0.record()
            for _ in range(a.steps):
                E, F = dm.energy_forces(pos)
            e1.record()
            torch.cuda.synchronize()
            dist.barrier()
        _lib.COUNTING = False
        launches = torch.tensor([_lib.launches()], device=dev)
        dist.all_reduce(launches)                           # library kernels launched by all ranks
        ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms)
        # roofline of the dominant kernels on this rank's local system (face_b200.perf)
        g = dm.graph
        El, Nl = int(g["ei"].numel()), int(g["row_ptr"].numel()) - 1
        root = os.path.dirname(os.path.abspath(B.__file__))
        rows, pk = perf.collect(El, Nl, spec["B"], spec["K"], 4 if dtype == torch.float32 else 8, a.steps, root,
                                traffic=perf.traffic_full_size(root, El, Nl))
        roof = perf.headline(rows, pk)
        if roof is not None:
            roof["kernel"] += ", rank 0 local system"
        # e2e: each rank's owned coordinates from pinned host memory, ghost coordinates through the halo, the local
        # neighbour list rebuilt on the device, forces on the owned atoms back to the host
        e2e = None
        if not a.no_e2e:
            host = torch.as_tensor(st.positions[dm.gid_owned.cpu().numpy()], dtype=torch.float64).pin_memory()
            fh = torch.empty(host.shape, dtype=torch.float64).pin_memory()
            ke = max(2, a.steps // 2)

            def e2e_step():
                p64 = host.to(dev, non_blocking=True)
                dm.rebuild(p64)
                E, F = dm.energy_forces(p64.to(dtype))
                fh.copy_(F.double(), non_blocking=True)
                torch.cuda.current_stream().synchronize()
                return E

            for _ in range(2):                           # untimed: the rebuild path's first allocations
                e2e_step()
            torch.cuda.synchronize()
            dist.barrier()
            t0 = time.perf_counter()
            for _ in range(ke):
                E = e2e_step()
            torch.cuda.synchronize()
            dist.barrier()
            dt = torch.tensor([(time.perf_counter() - t0) / ke], device=dev)
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
            nb = int(host.numel()) * 8
            e2e = {"value": natoms / float(dt), "unit": B.UNIT, "h2d_bytes_per_step": nb, "d2h_bytes_per_step": nb,
                   "ms_per_step": float(dt) * 1e3, "note": "bytes per rank (its owned atoms); time max over ranks"}
        counts = torch.tensor([n_local], device=dev)
        allc = [torch.zeros_like(counts) for _ in range(world)]
        dist.all_gather(allc, counts)
        if rank == 0:
            out = {"metric": B.METRIC, "value": natoms * 1e3 / ms, "unit": B.UNIT, "n_gpus": world, "steps": a.steps,
                   "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                   "vs_baseline": None, "dtype": "f32" if dtype == torch.float32 else "f64",
                   "data": "synthetic (seeded geometry, seeded random-init weights)",
                   "config": {"workload": f"cfg{a.config}: {natoms}-atom periodic system, spatial decomposition",
                              "atoms": natoms, "bricks": list(dm.grid), "halo_A": dm.halo,
                              "local_atoms_per_rank": [int(c) for c in allc],
                              "l2": "inputs larger than L2",
                              "parallelism": f"spatial {dm.grid} over NCCL, rc-deep ghosts, per-pass halo exchange",
                              "pme": "slab (mesh in x-slabs, all-to-all FFT transpose)"},
                   "e2e": e2e, "energy": float(E), "clocks": clk.summary(),
                   "roofline": roof,
                   "gpu_launches": int(launches)}
            print(json.dumps(out), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def bench_sharded(a):
    """bench.py --config 3 --gpus N under torchrun: the 512-molecule batch sharded by structure (weak per-structure
    work, fixed batch: every rank evaluates its share, one all-reduce of the per-structure energies per step)."""
    import datetime
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench as B
    from . import _lib
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        dtype = torch.float32
        structs, spec, pme = B.workload(3, scale=a.scale)
        model = B.make_model(spec, pme, dev, dtype)
        natoms = sum(len(s.numbers) for s in structs)
        sb = ShardedBatch(model, structs, rank, world, dev, dtype)
        for _ in range(a.warmup):
            sb.energy_forces()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _lib.CALLS.clear()
        _lib.COUNTING = True
        with B.Clocks(local) as clk:
            torch.cuda.synchronize()
            dist.barrier()
            e0.record()
            for _ in range(a.steps):
                E, F = sb.energy_forces()
            e1.record()
            torch.cuda.synchronize()
            dist.barrier()
        _lib.COUNTING = False
        launches = torch.tensor([_lib.launches()], device=dev)
        dist.all_reduce(launches)
        ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms)
        # e2e: this rank's positions from pinned host memory each step, forces back to the host
        e2e = None
        if not a.no_e2e and sb.graph is not None:
            host = sb.graph["pos"].detach().cpu().pin_memory()
            ke = max(1, a.steps // 2)
            torch.cuda.synchronize()
            dist.barrier()
            t0 = time.perf_counter()
            for _ in range(ke):
                sb.graph["pos"] = host.to(dev, non_blocking=True)
                E, F = sb.energy_forces()
                Fh = F.cpu()
            torch.cuda.synchronize()
            dist.barrier()
            dt = torch.tensor([(time.perf_counter() - t0) / ke], device=dev)
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
            e2e = {"value": natoms / float(dt), "unit": B.UNIT, "h2d_bytes_per_step": sb.n_local_atoms * 3 * 4,
                   "d2h_bytes_per_step": sb.n_local_atoms * 3 * 4, "ms_per_step": float(dt) * 1e3,
                   "note": "per rank, max over ranks"}
        counts = torch.tensor([sb.n_local_atoms], device=dev)
        allc = [torch.zeros_like(counts) for _ in range(world)]
        dist.all_gather(allc, counts)
        if rank == 0:
            out = {"metric": B.METRIC, "value": natoms * 1e3 / ms, "unit": B.UNIT, "n_gpus": world, "steps": a.steps,
                   "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                   "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded geometry, seeded random-init weights)",
                   "config": {"workload": f"cfg3: {len(structs)} molecules, {natoms} atoms, sharded by structure",
                              "atoms": natoms, "atoms_per_rank": [int(c) for c in allc],
                              "l2": "batch smaller than L2 (cfg3 is a small workload)",
                              "parallelism": f"structure sharding over {world} ranks, NCCL all-reduce of energies"},
                   "e2e": e2e, "energy_sum": float(E.sum()), "clocks": clk.summary(), "gpu_launches": int(launches)}
            print(json.dumps(out), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()
