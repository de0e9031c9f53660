"""Build libfacek.so (all CUDA sources in ../csrc) in-tree for sm_100a with nvcc.

    python -m face_b200.build [-v] [--ptxas]

The library is linked against the static CUDA runtime (nvcc's default) so it does not depend on which
libcudart the Python process has already loaded.
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(PKG), "csrc")
LIB = os.path.join(PKG, "libfacek.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(os.path.dirname(os.path.dirname(PKG)), "include", "*.h"))
    return any(os.path.getmtime(f) > t for f in deps)


OBJ = os.path.join(os.path.dirname(PKG), "_build")
COMPILE = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2"]


def _compile(src, ptxas):
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *COMPILE, *(["-Xptxas", "-v"] if ptxas else []), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, obj, r


def build(verbose=False, ptxas=False, force=False):
    """Compile every csrc/*.cu in parallel, link libfacek.so; skipped when up to date."""
    if not force and not stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(OBJ, exist_ok=True)
    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas), sources()))
    for src, obj, r in results:
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
        if verbose or ptxas:
            sys.stderr.write(r.stderr)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", *[o for _, o, _ in results], "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking libfacek.so")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.v, a.ptxas, a.force or a.ptxas))
