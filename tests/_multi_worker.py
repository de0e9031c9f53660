"""Worker for tests/test_gpu_multi.py: fp64 alloy (cfg5 model, 15x15x15 cells, 54 A box) decomposed over the torchrun world;
ranks exchange rc-deep ghosts and the pass-1 features through the halo, the PME mesh is distributed in x-slabs; rank 0
compares energy and the gathered owned forces with the single-GPU engine and writes the differences to argv[1].  Then
a 16-molecule batch (cfg3 model, fp64) sharded by structure, against the whole batch on one GPU."""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "face-mlip_b200"))


def main():
    from face_b200 import systems
    from face_b200.domain import DistributedModel, ShardedBatch
    from face_b200.model import FACE
    from face_b200.neighbors import build_graph
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        spec = systems.model_kwargs(5)
        kw = dict(spec)
        mb = kw.pop("max_body")
        m = FACE(**kw)
        m.set_max_body(mb)
        m.seed_(0)
        m.set_pme(gp=1 / 0.32, mesh=(60, 60, 60))
        m = m.to(dev, torch.float64)
        st = systems.fcc(15, 3.6, 0.08, systems.MODELS[5]["elements"], seed=0)
        dm = DistributedModel(m, st, rank, world, dev, torch.float64)
        E, F_owned = dm.energy_forces()                          # this rank's owned atoms
        # gather the owned forces by global id (test harness only: the decomposition itself keeps them local)
        n = torch.tensor([dm.plan.n_owned], device=dev)
        sizes = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(sizes, n)
        mx = int(max(int(x) for x in sizes))
        pf = torch.zeros(mx, 3, dtype=torch.float64, device=dev)
        pf[:dm.plan.n_owned] = F_owned
        pi = torch.full((mx,), -1, dtype=torch.long, device=dev)
        pi[:dm.plan.n_owned] = dm.gid_owned
        fs, ids = [torch.zeros_like(pf) for _ in range(world)], [torch.zeros_like(pi) for _ in range(world)]
        dist.all_gather(fs, pf)
        dist.all_gather(ids, pi)
        F = torch.zeros(len(st.numbers), 3, dtype=torch.float64, device=dev)
        for f, i in zip(fs, ids):
            F[i[i >= 0]] = f[i >= 0]
        # molecule batch sharded by structure (cfg3 model) against the whole batch on one GPU
        spec3 = dict(systems.model_kwargs(3))
        mb3 = spec3.pop("max_body")
        m3 = FACE(**spec3)
        m3.set_max_body(mb3)
        m3 = m3.seed_(1).to(dev, torch.float64)
        mols = systems.molecule_batch(16, seed=3)
        sb = ShardedBatch(m3, mols, rank, world, dev, torch.float64)
        Es, Fs = sb.energy_forces()
        off = np.concatenate([[0], np.cumsum([len(s.numbers) for s in mols])])
        o3 = m3(build_graph(mols, m3.rc, device=dev, dtype=torch.float64))
        Fr = torch.cat([o3["forces"][off[i]:off[i + 1]] for i in sb.ids]) if len(sb.ids) else Fs
        dEs = torch.tensor([float((Es - o3["energy"]).abs().max() / o3["energy"].abs().max()),
                            float((Fs - Fr).abs().max()) if len(sb.ids) else 0.0, float(len(sb.ids))], device=dev)
        allm = [torch.zeros_like(dEs) for _ in range(world)]
        dist.all_gather(allm, dEs)
        if rank == 0:
            o = m(build_graph([st], 5.0, device=dev, dtype=torch.float64))
            res = {"dE_rel": abs(float(E) - float(o["energy"][0])) / abs(float(o["energy"][0])),
                   "dF": float((F - o["forces"]).abs().max()), "E": float(E),
                   "n_owned": int(dm.plan.n_owned), "n_local": int(dm.plan.n_local),
                   "shard_dE_rel": max(float(t[0]) for t in allm), "shard_dF": max(float(t[1]) for t in allm),
                   "shard_counts": [int(t[2]) for t in allm]}
            open(sys.argv[1], "w").write(json.dumps(res))
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
