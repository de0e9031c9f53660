"""Tensor-core radial MLP (facek_radial_tc_fwd, tcgen05 kind::tf32 with the 3-term split) against the CUDA-core
kernel in fp64 and fp32 on the same edges: phi and the forward-mode dphi/dr, ragged tails (E not a multiple of the
128-edge tile, E < one tile, E = 0), both basis sizes and both output widths, edges beyond the cutoff, and the
bounded-wait status word.  Reference path: face-mlip face/model.py:465-469 (radial MLP) and :34-37 (envelope)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = "cuda"
RC = 5.0


def _edges(E, N, n_el, seed):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(E, 3, generator=g, dtype=torch.float64)
    u = u / u.norm(dim=1, keepdim=True).clamp_min(1e-12)
    r = 0.6 + (RC * 1.04 - 0.6) * torch.rand(E, generator=g, dtype=torch.float64)   # ~4% beyond the cutoff
    vec = (u * r[:, None]).to(DEV)
    ei = torch.randint(0, N, (E,), generator=g, dtype=torch.int32).to(DEV)
    ej = torch.randint(0, N, (E,), generator=g, dtype=torch.int32).to(DEV)
    zidx = torch.randint(0, n_el, (N,), generator=g, dtype=torch.int32).to(DEV)
    return vec, ei, ej, zidx


def _weights(n_el, nb, H, B, seed):
    g = torch.Generator().manual_seed(seed)
    w = lambda *s, sc=1.0: (torch.randn(*s, generator=g, dtype=torch.float64) * sc).to(DEV)
    return {"w1": w(H, nb, sc=nb ** -0.5), "b1": w(H, sc=0.3), "pair": w(n_el * n_el, H, sc=0.5),
            "w2": w(H, H, sc=H ** -0.5), "b2": w(H, sc=0.3), "w3": w(B, H, sc=H ** -0.5), "b3": w(B, sc=0.3)}


def _run(name, vec, ei, ej, zidx, W, n_el, nb, H, B):
    from face_b200 import _lib
    E = vec.shape[0]
    phi = torch.full((E, B), float("nan"), dtype=vec.dtype, device=DEV)
    dphidr = torch.full_like(phi, float("nan"))
    p = _lib.ptr
    keep = [W[k].to(vec.dtype).contiguous() for k in ("w1", "b1", "pair", "w2", "b2", "w3", "b3")]
    w = [p(t) for t in keep]
    head = [] if name == "facek_radial_tc_fwd" else [_lib.dtype_tag(vec)]
    _lib.call(name, *head, p(vec), p(ei), p(ej), p(zidx), n_el, RC, nb, H, B, *w, p(phi), p(dphidr), E,
              _lib.stream())
    torch.cuda.synchronize()
    return phi, dphidr


def _status():
    import ctypes
    from face_b200 import _lib
    v = ctypes.c_int32(-1)
    _lib.call("facek_tc_status", ctypes.byref(v), 1)
    return v.value


def _rel(a, b):
    return float((a.double() - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("E", [1, 127, 128, 129, 1000, 33_333])
@pytest.mark.parametrize("nb,B", [(8, 16), (16, 16), (8, 32), (16, 32)])
def test_radial_tc_matches_fp64(E, nb, B):
    n_el, H = 5, 64
    vec, ei, ej, zidx = _edges(E, 257, n_el, seed=E + nb + B)
    W = _weights(n_el, nb, H, B, seed=7)
    p64, d64 = _run("facek_radial_simt_fwd", vec, ei, ej, zidx, W, n_el, nb, H, B)
    p32, d32 = _run("facek_radial_simt_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    ptc, dtc = _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    assert _status() == 0
    assert torch.isfinite(ptc).all() and torch.isfinite(dtc).all()
    # fp32 accuracy: within a few times the CUDA-core fp32 kernel's own error, and 2e-6 of the largest value
    for tc, s32, ref in ((ptc, p32, p64), (dtc, d32, d64)):
        e_tc, e_32 = _rel(tc, ref), _rel(s32, ref)
        assert e_tc < max(4 * e_32, 2e-6), (e_tc, e_32)
    # beyond the cutoff both outputs are exactly zero
    out = (vec.norm(dim=1) >= RC)
    assert (ptc[out] == 0).all() and (dtc[out] == 0).all()


def test_radial_dispatch_uses_tensor_cores_for_fp32():
    n_el, nb, H, B = 3, 8, 64, 16
    vec, ei, ej, zidx = _edges(4099, 100, n_el, seed=3)
    W = _weights(n_el, nb, H, B, seed=8)
    a = _run("facek_radial_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    b = _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_radial_tc_single_element_and_empty():
    n_el, nb, H, B = 1, 8, 64, 16
    W = _weights(n_el, nb, H, B, seed=9)
    vec, ei, ej, zidx = _edges(0, 4, n_el, seed=1)
    phi, _ = _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    assert phi.numel() == 0
    vec, ei, ej, zidx = _edges(515, 4, n_el, seed=2)
    p64, _ = _run("facek_radial_simt_fwd", vec, ei, ej, zidx, W, n_el, nb, H, B)
    p32, _ = _run("facek_radial_simt_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    ptc, _ = _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    assert _rel(ptc, p64) < max(4 * _rel(p32, p64), 2e-6)
    assert _status() == 0


def test_radial_tc_rejects_unsupported_shapes():
    n_el, nb, H, B = 2, 8, 32, 16                      # hidden width 32 is a CUDA-core shape
    vec, ei, ej, zidx = _edges(10, 4, n_el, seed=2)
    W = _weights(n_el, nb, H, B, seed=1)
    with pytest.raises(RuntimeError, match="facek_radial_tc_fwd"):
        _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    phi, _ = _run("facek_radial_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)   # falls back to CUDA cores
    assert torch.isfinite(phi).all()


def test_radial_tc_many_tiles_persistent():
    """3.1M edges: every 128-edge tile of the persistent grid is written (NaN-filled outputs beforehand), to the
    same fp64-anchored bar as the small cases."""
    n_el, nb, H, B = 5, 8, 64, 16
    vec, ei, ej, zidx = _edges(3_100_003, 5000, n_el, seed=11)
    W = _weights(n_el, nb, H, B, seed=12)
    p64, d64 = _run("facek_radial_simt_fwd", vec, ei, ej, zidx, W, n_el, nb, H, B)
    p32, d32 = _run("facek_radial_simt_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    ptc, dtc = _run("facek_radial_tc_fwd", vec.float(), ei, ej, zidx, W, n_el, nb, H, B)
    assert _status() == 0
    assert torch.isfinite(ptc).all() and torch.isfinite(dtc).all()
    for tc, s32, ref in ((ptc, p32, p64), (dtc, d32, d64)):
        e_tc, e_32 = _rel(tc, ref), _rel(s32, ref)
        assert e_tc < max(4 * e_32, 2e-6), (e_tc, e_32)
