"""Energy+force throughput of the FACE engine on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 5]

Workload (default): 1,048,576-atom fcc 5-element random alloy (64^3 cells, a=3.6 A,
sigma=0.08 A), cutoff 5 A, factorised FACE model C=64, 2 passes, transport + equivariant messages, latent-charge
Coulomb with smooth PME on a 256^3 mesh (alpha = 0.32 1/A), float32, seeded synthetic geometry and seeded
random-init weights.  A step is one energy + forces evaluation of the whole system (the reference's timed unit,
face-mlip tools/bench.py:57-60; neighbour list built once outside the device-timed region, as there).

One JSON line on rank 0 with: value (atoms/s over all GPUs), e2e (the public calculator call with host positions in
pinned memory, neighbour list, forces back to the host), roofline of the dominant kernel by time per step
(algorithmic bytes and FLOPs per launch / CUDA-event launch time, against the measured HBM copy bandwidth and the
FP32 SIMT peak; the density forward, density adjoint and channel GEMM each have a row, see face_b200.perf),
cpu_baseline (the CPU oracle on a bounded sub-box on the host cores), clocks sampled during the timed region,
gpu_launches.

--impl reference: face-mlip's own algorithm (the CPU restatement in oracle/, the reference being a PyTorch package
that cannot run here) on the host cores, same metric and configuration, each step a bounded sub-box sample.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "face-mlip_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)
# the full-size step peaks at ~150 GiB of the GPU's 178 in buffers of up to tens of GiB; growable segments keep
# the caching allocator from failing on fragmentation (set before torch initialises CUDA)
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import torch  # noqa: E402

METRIC = "energy+force atoms/sec"
UNIT = "atoms/s"


# --------------------------------------------------------------------------------------------- workload
def workload(cfg, scale=None):
    from face_b200 import systems
    structs = systems.config_structures(cfg, seed=0, scale=scale)
    spec = systems.model_kwargs(cfg)
    pme = dict(systems.MODELS[cfg].get("pme", {}))
    return structs, spec, pme


def make_model(spec, pme, device, dtype):
    from face_b200.model import FACE
    kw = dict(spec)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    m.seed_(0)
    if "coulomb" in kw.get("terms", ()):
        m.set_pme(gp=pme["gp"], mesh=pme.get("mesh"))
    return m.to(device=device, dtype=dtype).eval()


def sub_box_sample(cfg, pme):
    """A bounded sample of the workload for the CPU: a periodic sub-box of the same material, PME mesh scaled to
    keep the grid spacing."""
    from face_b200 import systems
    if cfg == 5:
        side = 5
        st = systems.fcc(side, 3.6, 0.08, systems.MODELS[5]["elements"], seed=0)
        mesh = tuple(max(8, int(round(n * side / 64))) for n in pme["mesh"])
    elif cfg == 4:
        st = systems.random_mixture(600, 0.1, 1.2, systems.MODELS[4]["elements"], seed=0)
        mesh = (24, 24, 24)
    elif cfg == 3:
        return systems.config_structures(3, 0, scale=8), None, "8 molecules of the 512-molecule batch"
    elif cfg == 2:
        return systems.config_structures(2, 0), pme.get("mesh"), "the full 1,000-atom box"
    else:
        return systems.config_structures(1, 0), None, "the full 108-atom cell"
    n = len(st.numbers)
    return [st], mesh, f"{n}-atom periodic sub-box of the same material, PME mesh {mesh[0]}^3 (same spacing)"


def time_cpu_oracle(cfg, steps=None, warmup=1, budget_s=12.0):
    """The CPU oracle (face-mlip's PyTorch path restated) on the host cores: atoms/s on a bounded sample."""
    from oracle import face_ref, nlist
    from face_b200.model import FACE
    structs, spec, pme = workload(cfg, scale=1 if cfg in (1, 2, 5) else 8)
    sample, mesh, desc = sub_box_sample(cfg, pme)
    ncores = len(os.sched_getaffinity(0))
    torch.set_num_threads(ncores)
    g = nlist.padded_graph(sample, spec["rc"], dtype=np.float32 if cfg != 1 else np.float64)
    kw = dict(spec)
    mb = kw.pop("max_body")
    m = FACE(**kw)
    m.set_max_body(mb)
    state = m.seed_(0).state_dict()
    dt = torch.float64 if cfg == 1 else torch.float32
    pm = dict(pme, mesh=mesh) if mesh is not None else pme
    run = lambda: face_ref.forward(state, spec, g, dt, pme=pm)
    for _ in range(warmup):
        run()
    ts = []
    t_end = time.perf_counter() + budget_s
    while (steps is None and (time.perf_counter() < t_end or len(ts) < 3)) or (steps is not None and len(ts) < steps):
        t0 = time.perf_counter()
        run()
        ts.append(time.perf_counter() - t0)
    n = len(g["pos"])
    return {"value": n / statistics.median(ts), "unit": UNIT, "cores": ncores, "kind": "port",
            "sample": f"{desc}; median of {len(ts)} evaluations (float{'64' if cfg == 1 else '32'})"}, ts, n


# --------------------------------------------------------------------------------------------- clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p is not None:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        rows = []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]) if rows else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------------------------- GPU arm
def run_ours(a):
    from face_b200 import _lib, perf
    from face_b200.calculator import FACECalculator
    from face_b200.neighbors import build_graph
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1 or a.gpus > 1:
        from face_b200 import domain
        return domain.bench_multi(a)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dtype = torch.float64 if a.config == 1 else torch.float32
    structs, spec, pme = workload(a.config, scale=a.scale)
    if a.scale and a.config == 5:                           # keep the PME grid spacing of the full box
        pme["mesh"] = tuple(max(8, int(round(n * a.scale / 64))) for n in pme["mesh"])
    model = make_model(spec, pme, dev, dtype)
    if a.compiled_radial:                         # the reference's inference mode (fused + compiled radial)
        model.compile_radial()
    natoms = sum(len(s.numbers) for s in structs)
    g = build_graph(structs, spec["rc"], device=dev, dtype=dtype)
    E = int(g["ei"].numel())

    if a.graph:                                   # the whole evaluation as one CUDA-graph replay (face_b200.graphs)
        from face_b200.graphs import GraphedEvaluation
        ev = GraphedEvaluation(model, g)

        def step():
            return ev(g["pos"])["forces"]
    else:
        def step():
            gg = dict(g, pos=g["pos"].detach().clone())
            return model(gg)["forces"]

    t0 = time.perf_counter()
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    print(f"# warmup {a.warmup} steps {time.perf_counter() - t0:.2f} s, E={E} edges, peak mem "
          f"{torch.cuda.max_memory_allocated() / 2**30:.1f} GiB", file=sys.stderr, flush=True)
    # device-timed region: K steps, inputs resident in HBM (well above the 126 MB L2: edge tensors are GBs)
    for name in _lib.SIGNATURES:
        _lib.TIMED[name] = []
    perf.start()
    _lib.CALLS.clear()
    _lib.COUNTING = True
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(a.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    _lib.COUNTING = False
    launches = ev.launches * a.steps if a.graph else _lib.launches()
    ms = e0.elapsed_time(e1) / a.steps
    kernel_ms = {k[6:]: round(sum(s.elapsed_time(t) for s, t in v) / a.steps, 3) for k, v in _lib.TIMED.items() if v}
    value = natoms * a.steps / (e0.elapsed_time(e1) / 1e3)
    # roofline of the dominant kernels: algorithmic bytes and FLOPs per launch (face_b200.perf) over CUDA-event times
    esz = 4 if dtype == torch.float32 else 8
    rows, pk = perf.collect(E, natoms, spec["B"], spec["K"], esz, a.steps, ROOT,
                            traffic=perf.traffic_full_size(ROOT, E, natoms))
    _lib.TIMED.clear()
    # e2e: the public calculator call (host positions -> pinned -> device, neighbour list, forces back to host)
    e2e = None
    if not a.no_e2e:
        calc = FACECalculator(model=model, device=dev, dtype=dtype)
        at = structs[0] if len(structs) == 1 else None
        if at is not None:
            for _ in range(max(1, a.warmup // 2)):
                calc.calculate(at)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ke = max(1, a.steps // 2)
            for _ in range(ke):
                calc.calculate(at)
            torch.cuda.synchronize()
            dt_e2e = (time.perf_counter() - t0) / ke
            e2e = {"value": natoms / dt_e2e, "unit": UNIT, "h2d_bytes_per_step": natoms * (3 * 8 + 8) + 72,
                   "d2h_bytes_per_step": natoms * 3 * 8 + esz, "ms_per_step": dt_e2e * 1e3}
    cpu = None
    if not a.no_cpu:
        cpu, _, _ = time_cpu_oracle(a.config, budget_s=a.cpu_budget)
    out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f32" if dtype == torch.float32 else "f64", "data": "synthetic (seeded geometry, seeded random-init weights)",
           "config": {"workload": f"cfg{a.config}: " + ("1,048,576-atom fcc 5-element alloy, C64, 2 passes, PME 256^3"
                                                         if a.config == 5 and not a.scale else
                                                         f"BASELINE configuration {a.config}, scale {a.scale}"),
                      "atoms": natoms, "edges": E, "l2": ("inputs larger than L2 (edge tensors of several GB)" if E * 4 * 20 > 126e6 else
                             "small workload: edge tensors fit in L2, not flushed between steps"),
                      "parallelism": "single GPU", "cuda_graph": bool(a.graph),
                      "radial": "compiled (cubic Hermite tables)" if a.compiled_radial else "MLP"},
           "e2e": e2e,
           "roofline": perf.headline(rows, pk),
           "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": launches,
           "kernel_ms_per_step": kernel_ms}
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_reference(a):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    cpu, ts, n = time_cpu_oracle(a.config, steps=a.steps, warmup=a.warmup)
    med = statistics.median(ts)
    out = {"metric": METRIC, "value": n / med, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": med * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f64" if a.config == 1 else "f32", "data": "synthetic (seeded geometry, seeded random-init weights)",
           "impl": "reference", "config": {"workload": f"cfg{a.config} (bounded CPU sample: {cpu['sample']})"},
           "cpu_baseline": cpu, "e2e": {"value": n / med, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--compiled-radial", action="store_true",
                    help="radial MLP replaced by its per-pair spline tables, the reference's inference mode")
    ap.add_argument("--graph", action="store_true", help="single GPU: each step one CUDA-graph replay of the evaluation")
    ap.add_argument("--scale", type=int, default=None,
                    help="smaller system of the same configuration (cfg5: conventional cells per side), for profiling")
    a = ap.parse_args()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
