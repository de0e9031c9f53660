"""Spatial decomposition with the per-pass halo exchange on 2 GPUs (NCCL, slab-distributed PME) against the single-GPU
engine on the same periodic alloy, and a molecule batch sharded by structure against the whole batch on one GPU.  Runs only when
two or more GPUs are visible (launched as two torchrun processes)."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_gpu_decomposition_matches_single_gpu(tmp_path):
    out = tmp_path / "multi.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", "29517", os.path.join(ROOT, "tests", "_multi_worker.py"), str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["dE_rel"] <= 1e-10 and res["dF"] <= 1e-9, res
    assert res["n_local"] > res["n_owned"], res                                 # ghosts exchanged
    # structure sharding: every molecule on exactly one rank, energies and forces as evaluated in one batch
    assert sum(res["shard_counts"]) == 16 and min(res["shard_counts"]) > 0, res
    assert res["shard_dE_rel"] <= 1e-10 and res["shard_dF"] <= 1e-9, res
