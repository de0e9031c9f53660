"""Roofline accounting of the engine's dominant kernels, from CUDA-event times recorded around each C-ABI call
(face_b200._lib.TIMED) and the call arguments (face_b200._lib.ARGS).

Per launch, the ALGORITHMIC bytes (each input read once, each output written once) and FLOPs:

  density forward   facek_density_xm_fwd      bytes  e*E*(B+K+20) + e*N*20*B*K + 4(N+1)
                                              flops  2*E*20*B*K
  density adjoint   facek_density_msg_xm_bwd  bytes  e*N*20*B*K (G) + 2*e*E*(B+K+20) (phi, msg, Y in; dphi, dmsg,
                                                     dY out) + 2*e*nc*N*K (message tables) + 4(N+1) + 8E (rows, ei, ej)
                                              flops  2*E*(40*B*K + 40*B + 2*nc*K)
  channel GEMM      facek_gemm_tc             bytes  4*rows*(K + N*(1+beta)) + 8*K*N (split weight image)
                    facek_gemm_tc_split       flops  2*rows*K*N  (both entries, one row)

(e = element size, E edges, N atoms; the tensor-core density adjoint facek_density_msg_tc_xm_bwd has the same
algorithmic bytes and FLOPs as the CUDA-core one.)  Each kernel is reported against the measured HBM copy bandwidth and against
the FP32 SIMT peak (148 SMs x 128 FP32 lanes x 2 FLOP x the maximum SM clock); the attainable fraction is
max(bytes / HBM, flops / FP32 peak) / measured time, the roofline of a kernel that both streams and computes.
The GEMM runs on the tensor cores with a 3-term TF32 split; its attainable bound is HBM.
"""
import json
import os
import statistics

from . import _lib

SMS, FP32_LANES = 148, 128

ENTRIES = {"dens_bwd": "facek_density_msg_xm_bwd", "dens_bwd_tc": "facek_density_msg_tc_xm_bwd",
           "gemm": ("facek_gemm_tc", "facek_gemm_tc_split"), "dens_fwd": "facek_density_xm_fwd"}
KERNEL_NAMES = {"dens_bwd": "dens_bwd_lane_k (facek_density_msg_xm_bwd)",
                "dens_bwd_tc": "dens_bwd_tc_k + message dY (facek_density_msg_tc_xm_bwd)",
                "gemm": "gemm_tc_k (facek_gemm_tc, facek_gemm_tc_split)",
                "dens_fwd": "dens_fwd_k (facek_density_xm_fwd)"}


def _names(v):
    return v if isinstance(v, tuple) else (v,)


def peaks(root):
    try:
        pk = json.load(open(os.path.join(root, "MEASURED_PEAKS.json")))
    except Exception:
        pk = {}
    hbm = pk.get("hbm_gbs")
    mhz = pk.get("sm_max_mhz", 1965.0)
    return {"hbm_gbs": hbm if hbm else 6650.0, "hbm_source": "measured" if hbm else "fallback",
            "fp32_tflops": SMS * FP32_LANES * 2 * mhz * 1e6 / 1e12, "sm_mhz": mhz}


def start():
    """Record events and arguments of the dominant entry points from now on."""
    for names in ENTRIES.values():
        for name in _names(names):
            _lib.TIMED[name] = []
            _lib.ARGS[name] = []


def _sizes(name, args, E, N, B, K, esz):
    if name == "facek_density_xm_fwd":
        return (esz * E * (B + K + 20) + esz * N * 20 * B * K + 4 * (N + 1), 2.0 * E * 20 * B * K)
    if name in ("facek_density_msg_xm_bwd", "facek_density_msg_tc_xm_bwd"):
        nc = int(args[12] if name == "facek_density_msg_xm_bwd" else args[11])
        return (esz * N * 20 * B * K + 2 * esz * E * (B + K + 20) + 2 * esz * nc * N * K + 4 * (N + 1) + 8 * E,
                2.0 * E * (40 * B * K + 40 * B + 2 * nc * K))
    if name == "facek_gemm_tc":
        rows, k, n, beta = int(args[1]), int(args[2]), int(args[5]), int(args[9])
        return 4 * rows * (k + n * (1 + beta)) + 8 * k * n, 2.0 * rows * k * n
    if name == "facek_gemm_tc_split":
        rows, k, n, beta = int(args[5]), int(args[6]), int(args[8]), int(args[15])
        return 4 * rows * (k + n * (1 + beta)) + 8 * k * n, 2.0 * rows * k * n
    raise KeyError(name)


def collect(E, N, B, K, esz, steps, root, traffic=None):
    """Per-kernel roofline rows from the events and arguments recorded since start(); clears them.
    `traffic` maps a kernel key to measured DRAM bytes per launch (ncu), when known."""
    pk = peaks(root)
    rows = []
    for key, names in ENTRIES.items():
        ev, sz = [], []
        for name in _names(names):
            e_n = _lib.TIMED.pop(name, None) or []
            a_n = _lib.ARGS.pop(name, None) or []
            ev += e_n
            sz += [_sizes(name, a, E, N, B, K, esz) for a in a_n]
        if not ev:
            continue
        ts = [s.elapsed_time(t) / 1e3 for s, t in ev]
        by, fl = zip(*sz)
        t_tot, b_tot, f_tot = sum(ts), sum(by), sum(fl)
        launches = len(ts)
        gbs = b_tot / t_tot / 1e9
        tfs = f_tot / t_tot / 1e12
        t_bound = max(b_tot / (pk["hbm_gbs"] * 1e9), 0.0 if key == "gemm" else f_tot / (pk["fp32_tflops"] * 1e12))
        row = {"kernel": KERNEL_NAMES[key], "launches_per_step": launches / steps,
               "ms_per_step": t_tot * 1e3 / steps, "launch_ms": statistics.mean(ts) * 1e3,
               "launch_ms_first_step": [round(t * 1e3, 3) for t in ts[:launches // steps]],
               "bytes_per_launch": b_tot / launches, "flops_per_launch": f_tot / launches,
               "hbm": {"achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"]},
               "fp32": None if key == "gemm" else
               {"achieved": tfs, "peak": pk["fp32_tflops"], "unit": "TFLOP/s", "frac": tfs / pk["fp32_tflops"]},
               "attainable_frac": t_bound / t_tot,
               "bound": "hbm" if key == "gemm" or b_tot / pk["hbm_gbs"] / 1e9 >= f_tot / pk["fp32_tflops"] / 1e12
               else "fp32 (SIMT)",
               "traffic": (traffic or {}).get(key)}
        rows.append(row)
    rows.sort(key=lambda r: -r["ms_per_step"])
    return rows, pk


def headline(rows, pk):
    """The contract's roofline object for the dominant kernel (largest time per step), with the other rows."""
    if not rows:
        return None
    top = rows[0]
    return {"kernel": top["kernel"], "bound": "hbm", "achieved": top["hbm"]["achieved"], "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": top["hbm"]["frac"], "traffic": top["traffic"],
            "bytes_per_launch": top["bytes_per_launch"], "launch_ms": top["launch_ms"],
            "peak_source": pk["hbm_source"] + " (MEASURED_PEAKS.json hbm_gbs)",
            "fp32": top["fp32"], "attainable_frac": top["attainable_frac"], "attainable_bound": top["bound"],
            "fp32_peak_source": f"nominal SIMT: {SMS} SMs x {FP32_LANES} lanes x 2 FLOP x {pk['sm_mhz']:.0f} MHz",
            "kernels": rows}


def traffic_full_size(root, E, N):
    """Measured DRAM bytes per launch from the committed ncu summaries (small case scaled by edges and atoms)."""
    out = {}
    for key, fn in (("dens_fwd", "density_fwd_traffic.json"), ("dens_bwd", "density_bwd_traffic.json")):
        p = os.path.join(root, "profiles", fn)
        if not os.path.exists(p):
            continue
        d = json.load(open(p))
        sc = d["small_case"]
        if sc["atoms"] == N and sc["edges"] == E:
            out[key] = sc["dram_read_bytes"] + sc["dram_write_bytes"]
        else:
            out[key] = (sc["dram_read_bytes"] + sc["dram_write_bytes"]) * (E / sc["edges"])
    return out
