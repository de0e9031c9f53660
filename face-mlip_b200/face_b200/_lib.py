"""ctypes binding of libfacek.so (C ABI declared in include/facek.h).

The library is loaded on first use from this package directory.  There is no fallback: if it is missing or
a call fails, a RuntimeError carries the library's own error message.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FACEK_LIB") or os.path.join(_HERE, "libfacek.so")    # FACEK_LIB: another build

F32, F64 = 0, 1
P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
D = ctypes.c_double
PD = ctypes.POINTER(ctypes.c_double)
PI64 = ctypes.POINTER(ctypes.c_int64)

# name -> argument types (all return int status)
SIGNATURES = {
    "facek_density_fwd": [I32, P, P, P, P, I64, I32, I32, I32, P, P],
    "facek_density_bwd": [I32, P, P, P, P, P, P, P, I64, I32, I32, I32, P, P],
    "facek_density_xm_fwd": [I32, P, P, P, P, I64, I32, I32, P, P],
    "facek_density_xm_bwd": [I32, P, P, P, P, P, P, P, P, P, P, I64, I32, I32, P, P],
    "facek_node_fwd": [I32] + [P] * 13 + [I64, I32, I32, P],
    "facek_node_bwd": [I32] + [P] * 23 + [I64, I32, I32, P],
    "facek_node_engine_fwd": [I32] + [P] * 9 + [I64, I32, I32, I32, P],
    "facek_node_engine_bwd": [I32] + [P] * 13 + [I64, I32, I32, I32, P],
    "facek_bcast_mul_fwd": [I32, P, P, P, I32, I64, I32, I64, P],
    "facek_bcast_mul_bwd": [I32, P, P, P, P, P, I32, I64, I32, I64, P],
    "facek_nlist_cell_workspace": [I64, PD, D, PI64],
    "facek_nlist_cell_count": [P, I64, PD, D, P, P, P],
    "facek_nlist_cell_fill": [I32, P, I64, PD, D, P, P, P, P, P, P, P],
    "facek_nlist_batch_count": [P, I64, P, P, D, P, P],
    "facek_nlist_batch_fill": [I32, P, I64, P, P, D, P, P, P, P, P, P],
    "facek_nlist_reverse": [P, P, P, P, I64, I64, P, P],
    "facek_nlist_cell_build_noalloc": [I32, P, I64, PD, D, I64, P, P, P, P, P, PI64, P],
    "facek_edge_vec": [I32, P, P, P, P, P, I64, P],
    "facek_edge_vec_bwd": [I32, P, P, P, I64, P, P],
    "facek_edge_sym": [I32, P, P, I64, P],
    "facek_edge_sym_bwd": [I32, P, P, P, I32, I64, P],
    "facek_radial_fwd": [I32, P, P, P, P, I32, D, I32, I32, I32, P, P, P, P, P, P, P, P, P, I64, P],
    "facek_density_tc_xm_fwd": [P, P, P, P, I64, I32, I32, P, P],
    "facek_density_msg_xm_bwd": [I32, P, P, P, P, P, P, P, P, P, P, P, I32, P, P, P, I64, I64, I32, I32, P, P],
    "facek_density_msg_tc_xm_bwd": [P, P, P, P, P, P, P, P, P, P, P, I32, P, P, P, I64, I64, I32, I32, P, P],
    "facek_radial_simt_fwd": [I32, P, P, P, P, I32, D, I32, I32, I32, P, P, P, P, P, P, P, P, P, I64, P],
    "facek_radial_tc_fwd": [P, P, P, P, I32, D, I32, I32, I32, P, P, P, P, P, P, P, P, P, I64, P],
    "facek_tc_status": [P, I32],
    "facek_gemm_image_floats": [I64, I64],
    "facek_gemm_pack": [P, I64, I64, I64, I64, P, P],
    "facek_gemm_tc": [P, I64, I64, I64, P, I64, P, P, I64, I32, P],
    "facek_gemm_tc_split": [P, I64, I64, P, I64, I64, I64, P, I64, P, P, I64, I64, P, I64, I32, P],
    "facek_radial_spline_fwd": [I32, P, P, P, P, I32, D, I32, D, I32, P, P, P, P, I64, P],
    "facek_radial_bwd": [I32, P, P, P, I32, P, I32, I64, P],
    "facek_edge_msg_fwd": [I32, P, P, P, P, P, I32, I32, P, I64, I64, P],
    "facek_edge_msg_bwd": [I32, P, P, P, P, P, P, P, P, I32, I32, P, I32, P, P, I64, I64, P],
    "facek_transport_fwd": [I32, P, P, P, P, P, P, I64, I32, I32, P],
    "facek_transport_bwd": [I32, P, P, P, P, P, P, P, P, P, P, I32, P, P, I64, I64, I32, I32, P],
    "facek_pme_spread": [I32, P, P, I64, PD, I32, I32, I32, P, P],
    "facek_pme_green": [I32, P, I32, I32, I32, PD, D, D, P, P, P, P],
    "facek_pme_gather": [I32, P, P, I64, PD, I32, I32, I32, P, D, P, P, P],
    "facek_cp_density_fwd": [I32, P, P, I64, I32, P, P, I64, I32, P, P],
    "facek_cp_density_bwd": [I32, P, P, I64, I32, P, P, P, P, I64, I64, I32, P, P, P, P],
    "facek_layer_norm_fwd": [I32, P, P, P, D, I64, I32, P, P, P, P],
    "facek_layer_norm_bwd": [I32, P, P, P, P, P, I64, I32, P, P],
    "facek_silu_fwd": [I32, P, P, I64, P],
    "facek_silu_bwd": [I32, P, P, P, I64, P],
    "facek_zbl_fwd": [I32, P, P, P, P, D, D, I64, P, P],
    "facek_zbl_bwd": [I32, P, P, P, P, D, D, P, I64, P, I32, P],
    "facek_disp_fwd": [I32, P, P, P, P, P, P, D, I64, P, P],
    "facek_disp_bwd": [I32, P, P, P, P, P, P, D, P, I64, P, I32, P, P],
    "facek_coulomb_real_fwd": [I32, P, P, P, P, D, D, D, I64, P, P],
    "facek_coulomb_real_bwd": [I32, P, P, P, P, D, D, D, P, I64, P, I32, P, P],
}

_lib = None

# kernels launched per entry point (for launch accounting in the benchmark)
RESTYPES = {"facek_gemm_image_floats": ctypes.c_int64}     # everything else returns an int status
LAUNCHES_PER_CALL = {"facek_nlist_cell_count": 5, "facek_edge_msg_bwd": 2, "facek_transport_bwd": 2}
CALLS = {}            # name -> number of calls since reset (only while COUNTING)
COUNTING = False
TIMED = {}            # name -> list of (start, end) CUDA events, recorded around each call while enabled
ARGS = {}             # name -> list of argument tuples of the timed calls (for per-call byte/FLOP accounting)


def launches():
    return sum(n * LAUNCHES_PER_CALL.get(k, 1) for k, n in CALLS.items())


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (run `python -m face_b200.build` or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        L.facek_last_error.restype = ctypes.c_char_p
        L.facek_last_error.argtypes = []
        L.facek_version.restype = ctypes.c_int
        _lib = L
    return _lib


def call(name, *args):
    if COUNTING:
        CALLS[name] = CALLS.get(name, 0) + 1
    ev = TIMED.get(name)
    if ev is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        rc = getattr(lib(), name)(*args)
        e1.record()
        ev.append((e0, e1))
        if name in ARGS:
            ARGS[name].append(args)
    else:
        rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().facek_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def dtype_tag(t):
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float64:
        return F64
    raise TypeError(f"libfacek supports float32/float64, got {t.dtype}")


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def doubles(values):
    vals = [float(v) for v in values]
    return (ctypes.c_double * len(vals))(*vals)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("face_b200 kernels run on CUDA tensors only (no CPU path)")
