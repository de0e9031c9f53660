"""Structure sharding of a molecule batch (face_b200/domain.py: shard_structures, ShardedBatch) on CPU ranks (gloo).

The local evaluator is the CPU oracle, so this checks the batch partition and the energy all-reduce without a GPU:
two ranks, each evaluating its own molecules, must reproduce the oracle evaluated on the whole batch in one process
(face-mlip evaluates a batch in one FACE.forward, face/model.py:680-695).
"""
import datetime
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import face_ref, nlist

SPEC = dict(elements=[1, 6, 7, 8], C=8, n_basis=4, rc=4.0, n_passes=2, terms=(), max_body=5, radial_hidden=8,
            K_dir=4, norm="layer", transport=True, eqmsg=True, factor=True, B=4, K=4, cp=False, unit=True)


def _batch():
    from face_b200 import systems
    return systems.molecule_batch(7, seed=11, n_range=(5, 12))


def _state():
    from face_b200.model import FACE
    kw = dict(SPEC)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    return {k: v.double() if v.is_floating_point() else v for k, v in m.seed_(5).state_dict().items()}


def _oracle(structures):
    out = face_ref.forward(_state(), dict(SPEC), nlist.padded_graph(structures, SPEC["rc"]), torch.float64)
    return out["energy"], out["forces"]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from face_b200 import domain
        sb = domain.ShardedBatch(None, _batch(), rank, world, torch.device("cpu"), torch.float64, evaluate=_oracle)
        E, F = sb.energy_forces()
        out.put((rank, E.numpy(), F.detach().numpy(), sb.ids))
        out.close()
        out.join_thread()                              # the result is in the pipe before this process ends
        dist.barrier()
    finally:
        dist.destroy_process_group()
    os._exit(0)                                        # see test_domain_gloo: no interpreter finalisation


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_structures_balance():
    from face_b200.domain import shard_structures
    sizes = [20, 40, 33, 27, 38, 21, 25, 31, 39, 22]
    for world in (1, 2, 3, 4, 8):
        parts = shard_structures(sizes, world)
        assert sorted(np.concatenate(parts).tolist()) == list(range(len(sizes)))     # each structure once
        loads = [sum(sizes[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(sizes)
    parts = shard_structures([5, 6], 4)                                              # more ranks than structures
    assert [len(p) for p in parts] == [1, 1, 0, 0]


def test_two_rank_sharded_batch_matches_whole_batch():
    batch = _batch()
    E_ref, F_ref = _oracle(batch)
    off = np.concatenate([[0], np.cumsum([len(s.numbers) for s in batch])])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    seen = []
    for rank, E, F, ids in res:
        assert np.abs(E - E_ref.numpy()).max() <= 1e-12 * np.abs(E_ref.numpy()).max()   # every rank has all
        Fr = np.concatenate([F_ref.numpy()[off[i]:off[i + 1]] for i in ids])
        assert np.abs(F - Fr).max() <= 1e-12
        seen += list(ids)
    assert sorted(seen) == list(range(len(batch)))
