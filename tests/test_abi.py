"""CPU checks of the C ABI: the library loads without a GPU, exports every symbol include/facek.h declares, and the
ctypes argument lists match the header's parameter counts (no kernel is called)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "facek.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"(?:int64_t|int|const char\*)\s+(facek_\w+)\s*\(([^)]*)\)\s*;", src):
        params = [p for p in m.group(2).split(",") if p.strip() and p.strip() != "void"]
        out[m.group(1)] = len(params)
    return out


def test_header_parses():
    d = _declared()
    assert len(d) >= 30 and "facek_density_fwd" in d and "facek_last_error" in d


def test_library_exports_every_declared_symbol():
    from face_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libfacek.so not built")
    L = _lib.lib()
    for name in _declared():
        assert hasattr(L, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in nm.splitlines() if " T " in l}
    assert set(_declared()) <= exported


def test_ctypes_signatures_match_header():
    from face_b200 import _lib
    d = _declared()
    for name, args in _lib.SIGNATURES.items():
        assert name in d, name
        assert len(args) == d[name], (name, len(args), d[name])
    missing = set(d) - set(_lib.SIGNATURES) - {"facek_last_error", "facek_version"}
    assert not missing, missing


def test_error_path_without_gpu():
    """An invalid argument is rejected on the host with a readable message (no device work)."""
    from face_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libfacek.so not built")
    with pytest.raises(RuntimeError, match="bad sizes"):
        _lib.call("facek_density_fwd", 0, None, None, None, None, -1, 4, 16, 32, None, None)
