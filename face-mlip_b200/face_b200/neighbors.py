"""Neighbour lists on the GPU.

`build_graph(structures, rc)` returns the engine's CSR graph dict; `padded_graph(structures, rc)` is the drop-in
for face-mlip `face.neighbors.padded_graph` (face/neighbors.py:7-37) and `GraphSet.batch` (face/datasets.py:62-97),
returning the reference's padded-dense dict (pos, Z, nbr, shift, mask, batch, cell, charge, natoms, nstr).

Structures are `face_b200.systems.Structure` records or anything ASE-like (`positions`, `numbers`, `cell`,
`pbc`, optional `info["charge"]`).  Periodic structures must be periodic along all three axes (the reference's
configurations are either fully periodic or molecules); mixed periodicity raises.

CSR graph dict (all on the device):
  pos (N,3) dtype, Z (N,) int64, batch (N,) int64, nstr, natoms (nstr,), cell (nstr,3,3) dtype, charge (nstr,)
  row_ptr (N+1) int32, ei / ej (E,) int32 centre / neighbour, S (E,3) int32 images, shift (E,3) dtype,
  rev (E,) int32 reverse edge, pos64 (N,3) float64 (the positions the edge set was built from)
"""
import numpy as np
import torch

from . import _lib


def _as_struct(at):
    pos = np.asarray(at.positions, np.float64)
    Z = np.asarray(at.numbers, np.int64)
    cell = np.asarray(getattr(at.cell, "array", at.cell), np.float64).reshape(3, 3)
    pbc = np.asarray(at.pbc).reshape(-1)
    if pbc.size == 1:
        pbc = np.repeat(pbc, 3)
    if pbc.any() and not pbc.all():
        raise NotImplementedError("mixed periodicity is not supported (periodic structures need pbc on all axes)")
    info = getattr(at, "info", None)
    q = float(info.get("charge", 0.0)) if isinstance(info, dict) else float(getattr(at, "charge", 0.0))
    return pos, Z, cell, bool(pbc.all()), q


def _cumsum0(deg):
    rp = torch.zeros(deg.numel() + 1, dtype=torch.int64, device=deg.device)
    rp[1:] = torch.cumsum(deg.to(torch.int64), 0)
    return rp


def _periodic_rows(pos64, cell, rc, dtype):
    N = pos64.shape[0]
    c = _lib.doubles(cell.reshape(-1))
    nbytes = _lib.ctypes.c_int64(0)
    _lib.call("facek_nlist_cell_workspace", N, c, float(rc), _lib.ctypes.byref(nbytes))
    ws = torch.empty((nbytes.value + 3) // 4, dtype=torch.int32, device=pos64.device)
    deg = torch.empty(N, dtype=torch.int32, device=pos64.device)
    _lib.call("facek_nlist_cell_count", _lib.ptr(pos64), N, c, float(rc), _lib.ptr(ws), _lib.ptr(deg), _lib.stream())
    rp = _cumsum0(deg)
    E = int(rp[-1])
    ei = torch.empty(E, dtype=torch.int32, device=pos64.device)
    ej = torch.empty(E, dtype=torch.int32, device=pos64.device)
    S = torch.empty(E, 3, dtype=torch.int32, device=pos64.device)
    sh = torch.empty(E, 3, dtype=dtype, device=pos64.device)
    if E:
        _lib.call("facek_nlist_cell_fill", _lib.dtype_tag(sh), _lib.ptr(pos64), N, c, float(rc), _lib.ptr(ws),
                  _lib.ptr(rp.to(torch.int32)), _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), _lib.ptr(sh), _lib.stream())
    return rp, ei, ej, S, sh


def _molecule_rows(pos64, sstart, astruct, rc, dtype):
    N = pos64.shape[0]
    deg = torch.empty(N, dtype=torch.int32, device=pos64.device)
    _lib.call("facek_nlist_batch_count", _lib.ptr(pos64), N, _lib.ptr(sstart), _lib.ptr(astruct), float(rc),
              _lib.ptr(deg), _lib.stream())
    rp = _cumsum0(deg)
    E = int(rp[-1])
    ei = torch.empty(E, dtype=torch.int32, device=pos64.device)
    ej = torch.empty(E, dtype=torch.int32, device=pos64.device)
    S = torch.empty(E, 3, dtype=torch.int32, device=pos64.device)
    sh = torch.empty(E, 3, dtype=dtype, device=pos64.device)
    if E:
        _lib.call("facek_nlist_batch_fill", _lib.dtype_tag(sh), _lib.ptr(pos64), N, _lib.ptr(sstart),
                  _lib.ptr(astruct), float(rc), _lib.ptr(rp.to(torch.int32)), _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S),
                  _lib.ptr(sh), _lib.stream())
    return rp, ei, ej, S, sh


def structure_meta(sizes, cells, device):
    """Host-side per-structure data the evaluation needs without reading the device: atom offsets, inverse cells and
    volumes (host float64, and volumes also on the device) and lattice-vector lengths (for the PME mesh rule)."""
    offs = [0]
    for n in sizes:
        offs.append(offs[-1] + int(n))
    cells = np.asarray(cells, np.float64).reshape(-1, 3, 3)
    inv, vol = [], []
    for c in cells:
        periodic = np.abs(c).sum() > 0
        inv.append(np.linalg.inv(c) if periodic else np.zeros((3, 3)))
        vol.append(abs(float(np.linalg.det(c))) if periodic else 0.0)
    return {"offs": offs, "inv": inv, "vol": vol, "lengths": [np.linalg.norm(c, axis=1) for c in cells],
            "vol_t": torch.as_tensor(vol, dtype=torch.float64, device=device)}


LR_KEYS = ("row_ptr", "ei", "ej", "S", "shift", "rev")


def build_graph(structures, rc, device="cuda", dtype=torch.float32, skin=0.0, rc_long=None, pos64=None):
    """CSR neighbour graph of a batch of structures, built on the GPU (see module docstring).  With skin > 0 the
    list holds every pair closer than rc + skin (for reuse across MD steps; "coul_cut" = rc keeps the Coulomb
    real-space sum on the pairs closer than rc, and the model's envelope is zero beyond rc).  rc_long adds the
    long-range pair list of the dispersion term under "lr" (face/datasets.py:53-55, GraphSet(rc_long=...)).
    pos64, when given, is the batch's positions already on the device (float64, (N, 3), e.g. uploaded from pinned
    memory by the caller) and replaces the upload from the structures."""
    g = _build_graph(structures, rc + skin, device, dtype, pos64)
    if skin > 0:
        g["coul_cut"] = float(rc)
        g["rc"] = float(rc)
        g["skin"] = float(skin)
    if rc_long:
        lr = _build_graph(structures, rc_long + skin, device, dtype, g["pos64"])
        g["lr"] = {k: lr[k] for k in LR_KEYS}
    return g


def _build_graph(structures, rc, device="cuda", dtype=torch.float32, pos64=None):
    """CSR neighbour graph of a batch of structures, built on the GPU (see module docstring)."""
    items = [_as_struct(s) for s in structures]
    if not items:
        raise ValueError("empty batch")
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("build_graph runs on CUDA only")
    sizes = [len(it[1]) for it in items]
    offs = np.concatenate([[0], np.cumsum(sizes)])
    pos_np = np.concatenate([it[0] for it in items])
    if pos64 is None:
        pos64 = torch.as_tensor(pos_np, dtype=torch.float64, device=dev)
    pos64 = pos64.contiguous()
    N = pos64.shape[0]
    if tuple(pos64.shape) != (len(pos_np), 3) or pos64.dtype != torch.float64 or pos64.device.type != "cuda":
        raise ValueError("pos64 must be the batch's (N, 3) float64 positions on the build device")
    pieces = []
    if not any(it[3] for it in items):
        sstart = torch.as_tensor(offs, dtype=torch.int32, device=dev)
        astruct = torch.as_tensor(np.repeat(np.arange(len(items)), sizes), dtype=torch.int32, device=dev)
        pieces.append((0, 0, *_molecule_rows(pos64, sstart, astruct, rc, dtype)))
    else:
        for k, (p, Z, cell, pbc, q) in enumerate(items):
            o = int(offs[k])
            sub = pos64[o:o + sizes[k]].contiguous()
            if pbc:
                rows = _periodic_rows(sub, cell, rc, dtype)
            else:
                ss = torch.tensor([0, sizes[k]], dtype=torch.int32, device=dev)
                aa = torch.zeros(sizes[k], dtype=torch.int32, device=dev)
                rows = _molecule_rows(sub, ss, aa, rc, dtype)
            pieces.append((o, 0, *rows))
    if len(pieces) == 1:                          # one piece (one structure, or the batched molecule rows)
        _, _, rp, ei, ej, S, shift = pieces[0]
        row_ptr = rp.to(torch.int32)
    else:                                         # concatenate rows in atom order with global indices
        rps, eis, ejs, Ss, shs = [], [], [], [], []
        e_off = 0
        for o, _, rp, ei, ej, S, sh in pieces:
            rps.append(rp[:-1] + e_off)
            eis.append(ei + o)
            ejs.append(ej + o)
            Ss.append(S)
            shs.append(sh)
            e_off += int(rp[-1])
        row_ptr = torch.cat(rps + [torch.tensor([e_off], dtype=torch.int64, device=dev)]).to(torch.int32)
        ei, ej = torch.cat(eis).contiguous(), torch.cat(ejs).contiguous()
        S, shift = torch.cat(Ss).contiguous(), torch.cat(shs).contiguous()
    E = ei.numel()
    rev = torch.empty(E, dtype=torch.int32, device=dev)
    _lib.call("facek_nlist_reverse", _lib.ptr(row_ptr), _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), N, E, _lib.ptr(rev),
              _lib.stream())
    if E and bool((rev < 0).any()):
        raise RuntimeError("neighbour list is not symmetric (reverse edge missing)")
    cells = np.stack([it[2] if it[3] else np.zeros((3, 3)) for it in items])
    return {"pos": pos64.to(dtype, copy=True), "pos64": pos64,
            "meta": structure_meta(sizes, cells, dev),
            "Z": torch.as_tensor(np.concatenate([it[1] for it in items]), dtype=torch.long, device=dev),
            "batch": (torch.zeros(N, dtype=torch.long, device=dev) if len(items) == 1 else
                      torch.as_tensor(np.repeat(np.arange(len(items)), sizes), dtype=torch.long, device=dev)),
            "nstr": len(items), "natoms": torch.as_tensor(sizes, dtype=torch.long, device=dev),
            "cell": torch.as_tensor(cells, dtype=dtype, device=dev),
            "cell64": cells, "pbc": [it[3] for it in items],
            "charge": torch.as_tensor([it[4] for it in items], dtype=dtype, device=dev),
            "row_ptr": row_ptr, "ei": ei, "ej": ej, "S": S, "shift": shift, "rev": rev, "rc": float(rc)}


def periodic_graph_device(pos64, Z, cell, rc, dtype=torch.float32):
    """CSR graph of one periodic structure whose positions are already on the device (float64, (N, 3)); Z (N,) int64
    on the device, cell (3, 3) host array.  Used by the spatial decomposition to rebuild a rank's local list from
    halo-exchanged positions without a host round trip of the coordinates."""
    dev = pos64.device
    cell = np.asarray(cell, np.float64)
    pos64 = pos64.contiguous()
    N = pos64.shape[0]
    rp, ei, ej, S, sh = _periodic_rows(pos64, cell, rc, dtype)
    row_ptr = rp.to(torch.int32)
    E = ei.numel()
    rev = torch.empty(E, dtype=torch.int32, device=dev)
    _lib.call("facek_nlist_reverse", _lib.ptr(row_ptr), _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), N, E, _lib.ptr(rev),
              _lib.stream())
    return {"pos": pos64.to(dtype, copy=True), "pos64": pos64, "meta": structure_meta([N], cell[None], dev), "Z": Z,
            "batch": torch.zeros(N, dtype=torch.long, device=dev), "nstr": 1,
            "natoms": torch.tensor([N], dtype=torch.long, device=dev),
            "cell": torch.as_tensor(cell[None], dtype=dtype, device=dev), "cell64": cell[None], "pbc": [True],
            "charge": torch.zeros(1, dtype=dtype, device=dev), "row_ptr": row_ptr, "ei": ei, "ej": ej, "S": S,
            "shift": sh, "rev": rev, "rc": float(rc)}


def keep_edges(g, keep):
    """The graph restricted to the edges where `keep` (E,) is true; `keep` must be symmetric (an edge and its reverse
    kept together), so that rows stay in canonical order and every kept edge keeps its reverse."""
    idx = torch.nonzero(keep)[:, 0]
    N = g["row_ptr"].numel() - 1
    ei, ej, S, sh = g["ei"][idx].contiguous(), g["ej"][idx].contiguous(), g["S"][idx].contiguous(), g["shift"][idx]
    row_ptr = _cumsum0(torch.bincount(ei.long(), minlength=N)).to(torch.int32)
    E = ei.numel()
    rev = torch.empty(E, dtype=torch.int32, device=ei.device)
    _lib.call("facek_nlist_reverse", _lib.ptr(row_ptr), _lib.ptr(ei), _lib.ptr(ej), _lib.ptr(S), N, E, _lib.ptr(rev),
              _lib.stream())
    return dict(g, row_ptr=row_ptr, ei=ei, ej=ej, S=S, shift=sh.contiguous(), rev=rev)


def to_padded(graph):
    """CSR graph -> the reference's padded-dense dict (face/datasets.py:74-97 layout)."""
    rp, ei, ej = graph["row_ptr"].long(), graph["ei"].long(), graph["ej"].long()
    N = rp.numel() - 1
    deg = rp[1:] - rp[:-1]
    M = max(1, int(deg.max())) if N else 1
    slot = torch.arange(ei.numel(), device=ei.device) - rp[ei]
    first = torch.zeros(graph["nstr"], dtype=torch.long, device=ei.device)
    first[1:] = torch.cumsum(graph["natoms"], 0)[:-1]
    nbr = first[graph["batch"]][:, None].expand(N, M).clone()
    nbr[ei, slot] = ej
    shift = torch.zeros(N, M, 3, dtype=graph["shift"].dtype, device=ei.device)
    shift[ei, slot] = graph["shift"]
    mask = torch.zeros(N, M, dtype=torch.bool, device=ei.device)
    mask[ei, slot] = True
    return {"pos": graph["pos"], "Z": graph["Z"], "nbr": nbr, "shift": shift, "mask": mask, "batch": graph["batch"],
            "cell": graph["cell"], "charge": graph["charge"], "natoms": graph["natoms"], "nstr": graph["nstr"]}


def padded_graph(atoms_list, rc, device="cuda", dtype=torch.float32, skin=0.0):
    """Drop-in for face.neighbors.padded_graph (face/neighbors.py:7-37), built on the GPU."""
    return to_padded(build_graph(atoms_list, rc + skin, device, dtype))


def _csr_from_pairs(ei, ej, sh, batch, cell, N):
    """(i, j, shift) pairs -> canonical CSR rows (i, j, S0, S1, S2 order) with the reverse-edge index."""
    dev = ei.device
    S = torch.zeros(ei.numel(), 3, dtype=torch.int64, device=dev)
    if cell is not None and bool((cell.abs().sum((1, 2)) > 0).any()):
        c64 = cell.detach().double().cpu().numpy()
        inv = np.stack([np.linalg.inv(c) if np.abs(c).sum() > 0 else np.zeros((3, 3)) for c in c64])
        inv = torch.as_tensor(inv, device=dev)
        S = torch.round(torch.einsum("ex,exy->ey", sh.double(), inv[batch[ei]])).long()
    order = torch.arange(ei.numel(), device=dev)
    for keycol in (S[:, 2], S[:, 1], S[:, 0], ej, ei):          # stable lexicographic (ei, ej, S0, S1, S2)
        order = order[torch.sort(keycol[order], stable=True).indices]
    ei, ej, S, sh = ei[order], ej[order], S[order], sh[order]
    deg = torch.bincount(ei, minlength=N)
    row_ptr = _cumsum0(deg).to(torch.int32)
    ei32, ej32, S32 = ei.int().contiguous(), ej.int().contiguous(), S.int().contiguous()
    E = ei32.numel()
    rev = torch.empty(E, dtype=torch.int32, device=dev)
    _lib.call("facek_nlist_reverse", _lib.ptr(row_ptr), _lib.ptr(ei32), _lib.ptr(ej32), _lib.ptr(S32), N, E,
              _lib.ptr(rev), _lib.stream())
    if E and bool((rev < 0).any()):
        raise RuntimeError("graph_from_padded: neighbour list is not symmetric")
    return {"row_ptr": row_ptr, "ei": ei32, "ej": ej32, "S": S32, "shift": sh.contiguous(), "rev": rev}


def graph_from_padded(g):
    """Reference padded graph dict -> engine CSR graph (edges re-ordered canonically within rows); the long-range
    pair list lr_i / lr_j / lr_shift (face/datasets.py:92-95), when present, becomes g["lr"]."""
    nbr, mask, shift = g["nbr"], g["mask"], g["shift"]
    dev = nbr.device
    N, M = nbr.shape
    ei = torch.arange(N, device=dev)[:, None].expand(N, M)[mask]
    ej = nbr[mask]
    sh = shift[mask]
    batch = g["batch"]
    nstr = int(g["nstr"]) if "nstr" in g else int(batch.max()) + 1
    cell = g.get("cell")
    csr = _csr_from_pairs(ei, ej, sh, batch, cell, N)
    natoms = torch.bincount(batch, minlength=nstr)
    cells = cell if cell is not None else torch.zeros(nstr, 3, 3, dtype=g["pos"].dtype, device=dev)
    cell64 = cells.detach().double().cpu().numpy()
    return {"pos": g["pos"], "Z": g["Z"], "batch": batch, "nstr": nstr, "natoms": natoms, "cell": cells,
            "cell64": cell64, "meta": structure_meta(natoms.tolist(), cell64, dev),
            "pbc": [bool(c.abs().sum() > 0) for c in cells.detach().cpu()],
            "charge": g.get("charge", torch.zeros(nstr, dtype=g["pos"].dtype, device=dev)), **csr,
            **({"lr": _csr_from_pairs(g["lr_i"].long(), g["lr_j"].long(), g["lr_shift"].to(g["pos"].dtype), batch,
                                      cell, N)} if "lr_i" in g else {})}
