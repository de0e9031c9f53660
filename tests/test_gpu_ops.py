"""Kernel-level parity on the GPU: each libfacek.so op against the reference's golden vectors and against a plain
PyTorch (float64/float32) statement of the same op, forward and first-order gradients."""
import numpy as np
import pytest
import torch

from _golden import load
from oracle import face_ref

pytestmark = pytest.mark.gpu
cuda = pytest.importorskip("torch").cuda
if not cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = "cuda"


def rel(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


# ------------------------------------------------------------------------------------------ factor_density
def test_factor_density_golden_fp64():
    from face_b200.kernels import factor_density
    k = load("kernels")
    for tag in ("a", "b"):
        t = lambda n: torch.tensor(k[f"fd{tag}_{n}"], device=DEV, requires_grad=True)
        phi, msg, Y = t("phi"), t("msg"), t("Y")
        D = factor_density(phi, msg, Y)
        gr = torch.autograd.grad((D * torch.tensor(k[f"fd{tag}_G"], device=DEV)).sum(), (phi, msg, Y))
        assert rel(D, torch.tensor(k[f"fd{tag}_D"], device=DEV)) < 1e-13
        for g, n in zip(gr, ("dphi", "dmsg", "dY")):
            assert rel(g, torch.tensor(k[f"fd{tag}_{n}"], device=DEV)) < 1e-13, n


@pytest.mark.parametrize("B,K", [(16, 32), (32, 32), (8, 16), (3, 5)])
def test_factor_density_fp32(B, K):
    """face-mlip tests/test_kernels.py:7-20 shapes (N=300, M=37); 1e-4 relative-to-max bar (:19)."""
    from face_b200.kernels import factor_density
    torch.manual_seed(0)
    N, M = 300, 37
    phi = torch.randn(N, M, B, device=DEV, requires_grad=True)
    msg = torch.randn(N, M, K, device=DEV, requires_grad=True)
    Y = torch.randn(N, M, 20, device=DEV, requires_grad=True)
    G = torch.randn(N, 20, B * K, device=DEV)
    D1 = factor_density(phi, msg, Y)
    g1 = torch.autograd.grad((D1 * G).sum(), (phi, msg, Y))
    p64 = [x.detach().double().requires_grad_() for x in (phi, msg, Y)]
    D2 = face_ref.factor_density(*p64)
    g2 = torch.autograd.grad((D2 * G.double()).sum(), p64)
    errs = [rel(D1.double(), D2)] + [rel(a.double(), b) for a, b in zip(g1, g2)]
    assert max(errs) < 1e-4, errs


def test_factor_density_empty_rows():
    from face_b200.kernels import factor_density
    phi = torch.zeros(5, 0, 16, device=DEV)
    msg = torch.zeros(5, 0, 32, device=DEV)
    Y = torch.zeros(5, 0, 20, device=DEV)
    assert factor_density(phi, msg, Y).abs().max() == 0
    assert factor_density(phi[:0], msg[:0], Y[:0]).shape == (0, 20, 512)


# ------------------------------------------------------------------------------------------ node algebra
NAMES = ["P1", "Q1", "S1", "P2", "Q2", "S2", "P3", "Q3"]
RANKS = [1, 1, 1, 2, 2, 2, 3, 3]


def test_node_algebra_golden_fp64():
    from face_b200.node_kernel import node_algebra
    k = load("kernels")
    xs = [torch.tensor(k["na_" + n], device=DEV, requires_grad=True) for n in NAMES]
    a = torch.tensor(k["na_a"], device=DEV, requires_grad=True)
    b = torch.tensor(k["na_b"], device=DEV, requires_grad=True)
    inv, V, Mf = node_algebra(*xs, a, b, True)
    T = lambda n: torch.tensor(k[n], device=DEV)
    L = (inv * T("na_gI")).sum() + (V * T("na_gV")).sum() + (Mf * T("na_gM")).sum()
    grads = torch.autograd.grad(L, xs + [a, b])
    assert rel(inv, T("na_inv")) < 1e-13 and rel(V, T("na_V")) < 1e-13 and rel(Mf, T("na_Mf")) < 1e-13
    for g, n in zip(grads, ["d" + n for n in NAMES] + ["da", "db"]):
        assert rel(g, T("na_" + n)) < 1e-12, n


@pytest.mark.parametrize("eq", [True, False])
def test_node_algebra_fp32(eq):
    """face-mlip tests/test_node_kernel.py:8-28 setting (N=50, C=24), 1e-4 relative bar (:26)."""
    from face_b200.node_kernel import node_algebra
    torch.manual_seed(1)
    N, C = 50, 24
    shapes = [(3,), (3,), (3,), (6,), (6,), (6,), (10,), (10,)]
    xs = [torch.randn(N, C, *s, device=DEV, requires_grad=True) for s in shapes]
    a = torch.randn(4, C, device=DEV, requires_grad=True)
    b = torch.randn(4, C, device=DEV, requires_grad=True)
    gI, gV, gM = torch.randn(N, C, 8, device=DEV), torch.randn(N, C, 3, device=DEV), torch.randn(N, C, 3, 3, device=DEV)
    o1 = node_algebra(*xs, a, b, eq)
    x64 = [x.detach().double().requires_grad_() for x in xs + [a, b]]
    o2 = face_ref.node_products(*[face_ref.to_full(x, l) for x, l in zip(x64[:8], RANKS)], x64[8], x64[9])
    Lf = lambda o: (o[0] * gI.to(o[0].dtype)).sum() + (((o[1] * gV.to(o[1].dtype)).sum() + (o[2] * gM.to(o[2].dtype)).sum()) if eq else 0)
    wrt1 = xs + ([a, b] if eq else [])
    wrt2 = x64[:8] + ([x64[8], x64[9]] if eq else [])
    g1 = torch.autograd.grad(Lf(o1), wrt1)
    g2 = torch.autograd.grad(Lf(o2), wrt2)
    errs = [rel(o1[0].double(), o2[0])] + ([rel(o1[1].double(), o2[1]), rel(o1[2].double(), o2[2])] if eq else [])
    errs += [rel(u.double(), v) for u, v in zip(g1, g2)]
    assert max(errs) < 1e-4, errs


@pytest.mark.parametrize("max_body", [5, 4, 3])
def test_node_engine_layout_fp64(max_body):
    """Engine layout (k,N,3C) -> inv9 (N,9C) (P0 + 8 families, masked by body order), V (3,N,C), Ms (6,N,C)."""
    from face_b200.ops import NodeAlgebraEngine
    torch.manual_seed(2)
    N, C = 17, 6
    ys = [torch.randn(k, N, 3 * C, device=DEV, dtype=torch.float64, requires_grad=True) for k in (1, 3, 6, 10)]
    a = torch.randn(4, C, device=DEV, dtype=torch.float64)
    b = torch.randn(4, C, device=DEV, dtype=torch.float64)
    inv9, V, Ms = NodeAlgebraEngine.apply(*ys, a, b, True, max_body)
    # torch statement
    P = [[y[:, :, i * C:(i + 1) * C].permute(1, 2, 0) for i in range(3)] for y in ys]  # (N,C,k)
    full = lambda t, l: face_ref.to_full(t, l)
    inv8, V2, Mf2 = face_ref.node_products(full(P[1][0], 1), full(P[1][1], 1), full(P[1][2], 1), full(P[2][0], 2),
                                           full(P[2][1], 2), full(P[2][2], 2), full(P[3][0], 3), full(P[3][1], 3), a, b)
    fams = [P[0][0][..., 0]] + list(inv8.unbind(-1))
    fams = [f if bo <= max_body else torch.zeros_like(f) for f, bo in zip(fams, face_ref.BODY_ORDER)]
    inv_ref = torch.cat(fams, 1)
    Ms_ref = face_ref._sym6(0.5 * (Mf2 + Mf2.transpose(-1, -2))).permute(2, 0, 1)
    V_ref = V2.permute(2, 0, 1)
    assert rel(inv9, inv_ref) < 1e-13 and rel(V, V_ref) < 1e-13 and rel(Ms, Ms_ref) < 1e-13
    g9, gV, gM = torch.randn_like(inv9), torch.randn_like(V), torch.randn_like(Ms)
    L1 = (inv9 * g9).sum() + (V * gV).sum() + (Ms * gM).sum()
    L2 = (inv_ref * g9).sum() + (V_ref * gV).sum() + (Ms_ref * gM).sum()
    for u, v in zip(torch.autograd.grad(L1, ys), torch.autograd.grad(L2, ys)):
        assert rel(u, v) < 1e-12


# ------------------------------------------------------------------------------------------ edge ops
@pytest.fixture(scope="module")
def small_graph():
    from face_b200 import systems
    from face_b200.neighbors import build_graph
    st = systems.config_structures(5, seed=3, scale=3)
    g = build_graph(st, 5.0, dtype=torch.float64)
    g["zidx"] = (g["Z"] - 24).to(torch.int32)
    return g


def _torch_vec(g, pos):
    return pos[g["ej"].long()] - pos[g["ei"].long()] + g["shift"]


def test_edge_vec_sym_fp64(small_graph):
    from face_b200.ops import EdgeSym, EdgeVec
    g = small_graph
    pos = g["pos"].clone().requires_grad_(True)
    vec = EdgeVec.apply(pos, g)
    Y = EdgeSym.apply(vec)
    pos2 = g["pos"].clone().requires_grad_(True)
    v2 = _torch_vec(g, pos2)
    Y2 = face_ref.monomials(v2 / v2.norm(dim=-1, keepdim=True))
    assert rel(vec, v2) < 1e-15 and rel(Y, Y2) < 1e-14
    G = torch.randn_like(Y)
    d1 = torch.autograd.grad((Y * G).sum(), pos)[0]
    d2 = torch.autograd.grad((Y2 * G).sum(), pos2)[0]
    assert rel(d1, d2) < 1e-12


def _radial_ref(q, r, zp, spline=None):
    """torch statement on the CPU (the oracle helpers allocate there)"""
    c = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in q.items()}
    r, zp = r.cpu(), zp.cpu().long()
    if spline is not None:
        T, dT, dr = spline
        raw = face_ref.spline_eval(T.cpu(), dT.cpu(), dr, r, zp)
    else:
        rb = face_ref.bessel(r, c["nb"], c["rc"], r.dtype) * face_ref.envelope(r, c["rc"])[..., None]
        x = torch.nn.functional.silu(rb @ c["w1"].t() + c["b1"] + c["pair"][zp])
        raw = torch.nn.functional.silu(x @ c["w2"].t() + c["b2"]) @ c["w3"].t() + c["b3"]
    return (raw * face_ref.envelope(r, c["rc"])[..., None]).to(DEV)


@pytest.mark.parametrize("spline", [False, True])
def test_radial_fp64(small_graph, spline):
    from face_b200.ops import EdgeVec, Radial
    g = small_graph
    torch.manual_seed(4)
    n_el, H, nb, B = 5, 64, 8, 16
    dd = dict(dtype=torch.float64, device=DEV)
    q = {"B": B, "n_el": n_el, "rc": 5.0, "nb": nb, "H": H, "w1": torch.randn(H, nb, **dd) / 3,
         "b1": torch.randn(H, **dd), "pair": torch.randn(n_el * n_el, H, **dd) / 3, "w2": torch.randn(H, H, **dd) / 8,
         "b2": torch.randn(H, **dd), "w3": torch.randn(B, H, **dd) / 8, "b3": torch.randn(B, **dd), "spline": None}
    if spline:
        G = 1024
        q["spline"] = (torch.randn(n_el * n_el, G, B, **dd), torch.randn(n_el * n_el, G, B, **dd), 5.0 / (G - 1))
    pos = g["pos"].clone().requires_grad_(True)
    phi = Radial.apply(EdgeVec.apply(pos, g), g, q)
    again = Radial.apply(EdgeVec.apply(g["pos"].clone(), g), g, q)
    # the kernel is deterministic (no atomics, weights staged once per block behind a barrier): two launches agree
    # bit for bit, so a mismatch below would point at the inputs, not at the kernel
    assert torch.equal(phi.detach(), again), "radial kernel not bitwise reproducible"
    pos2 = g["pos"].clone().requires_grad_(True)
    v2 = _torch_vec(g, pos2)
    zp = g["zidx"][g["ei"].long()] * n_el + g["zidx"][g["ej"].long()]
    phi2 = _radial_ref(q, v2.norm(dim=-1), zp, q["spline"])
    err = (phi.detach() - phi2).abs()
    e_bad = int(err.max(1).values.argmax())
    assert rel(phi, phi2) < 1e-12, (rel(phi, phi2), e_bad, float(v2[e_bad].norm()), phi[e_bad].tolist(),
                                    phi2[e_bad].tolist())
    G_ = torch.randn_like(phi)
    assert rel(torch.autograd.grad((phi * G_).sum(), pos)[0], torch.autograd.grad((phi2 * G_).sum(), pos2)[0]) < 1e-10


@pytest.mark.parametrize("B", [16, 6])
def test_radial_spline_fp32(small_graph, B):
    """fp32 compiled radial (B % 4 == 0 runs the 16-byte vector kernel, B = 6 the scalar one) against the fp64 torch
    statement of the same fp32 tables: the bar is fp32 rounding of a cubic Hermite evaluation (rel 1e-5).  The tables
    are smooth (sinusoids and their derivatives, like a compiled MLP): with random knot values the interpolant's slope
    in grid units is O(1), so fp32 rounding of x = r/dr alone (ulp 6e-5 at x ~ 600) moves phi by ~1e-4."""
    from face_b200.ops import EdgeVec, Radial
    g = small_graph
    torch.manual_seed(14)
    n_el, G = 5, 1024
    d32 = dict(dtype=torch.float32, device=DEV)
    rg = torch.arange(G, dtype=torch.float64, device=DEV) * (5.0 / (G - 1))
    amp, w, ph = (torch.randn(n_el * n_el, 1, B, dtype=torch.float64, device=DEV), 1 + 2 * torch.rand(1, 1, B, dtype=torch.float64, device=DEV),
                  torch.rand(n_el * n_el, 1, B, dtype=torch.float64, device=DEV) * 6)
    arg = w * rg[None, :, None] + ph
    T, dT = (amp * torch.sin(arg)).to(**d32), (amp * w * torch.cos(arg)).to(**d32)
    q = {"B": B, "n_el": n_el, "rc": 5.0, "spline": (T, dT, 5.0 / (G - 1))}
    g32 = dict(g, shift=g["shift"].float())
    pos = g["pos"].float().clone().requires_grad_(True)
    phi = Radial.apply(EdgeVec.apply(pos, g32), g32, q)
    assert phi.dtype == torch.float32 and phi.shape[1] == B
    pos2 = g["pos"].float().double().clone().requires_grad_(True)
    v2 = _torch_vec(g, pos2)
    zp = g["zidx"][g["ei"].long()] * n_el + g["zidx"][g["ej"].long()]
    phi2 = _radial_ref(q, v2.norm(dim=-1), zp, (T.double(), dT.double(), 5.0 / (G - 1)))
    assert rel(phi.double(), phi2) < 1e-5
    G_ = torch.randn_like(phi2)
    d1 = torch.autograd.grad((phi.double() * G_).sum(), pos)[0].double()
    d2 = torch.autograd.grad((phi2 * G_).sum(), pos2)[0]
    assert rel(d1, d2) < 1e-4


@pytest.mark.parametrize("dt", [torch.float64, torch.float32])
@pytest.mark.parametrize("nc", [1, 10])
def test_edge_msg_fp64(small_graph, nc, dt):
    """EdgeMsg (fp32 K = 32 runs the eight-lanes-per-edge kernel) against the torch statement of the message."""
    from face_b200.ops import EdgeMsg, EdgeSym, EdgeVec
    g = small_graph
    N = g["pos"].shape[0]
    K = 32
    torch.manual_seed(5)
    pos = g["pos"].clone().to(dt).requires_grad_(True)
    gg = dict(g, shift=g["shift"].to(dt))
    Y = EdgeSym.apply(EdgeVec.apply(pos, gg))
    TJ = torch.randn(nc, N, K, device=DEV, dtype=dt, requires_grad=True)
    TI = torch.randn(nc, N, K, device=DEV, dtype=dt, requires_grad=True) if nc > 1 else None
    tol_f, tol_b = (1e-14, 1e-12) if dt == torch.float64 else (2e-6, 2e-5)
    g = gg
    m = EdgeMsg.apply(Y, TJ, TI, g)
    ei, ej = g["ei"].long(), g["ej"].long()
    tab = (TJ[:, ej] + (TI[:, ei] if TI is not None else 0)).transpose(0, 1)            # (E, nc, K)
    m2 = (Y[:, :nc, None] * tab).sum(1)
    assert rel(m, m2) < tol_f
    G = torch.randn_like(m)
    wrt = [pos, TJ] + ([TI] if TI is not None else [])
    g1 = torch.autograd.grad((m * G).sum(), wrt, retain_graph=True)
    g2 = torch.autograd.grad((m2 * G).sum(), wrt)
    for u, v in zip(g1, g2):
        assert rel(u, v) < tol_b


def test_density_csr_fp64(small_graph):
    from face_b200.ops import Density
    g = small_graph
    E = g["ei"].numel()
    N = g["pos"].shape[0]
    torch.manual_seed(6)
    phi = torch.randn(E, 16, device=DEV, dtype=torch.float64, requires_grad=True)
    msg = torch.randn(E, 32, device=DEV, dtype=torch.float64, requires_grad=True)
    Y = torch.randn(E, 20, device=DEV, dtype=torch.float64, requires_grad=True)
    D = torch.cat(Density.apply(phi, msg, Y, g), 0)                                     # (20, N, BK)
    w = (phi[:, :, None] * msg[:, None, :]).reshape(E, -1)
    D2 = torch.zeros(N, 20, 512, device=DEV, dtype=torch.float64).index_add(0, g["ei"].long(), Y[:, :, None] * w[:, None, :])
    D2 = D2.transpose(0, 1)
    assert rel(D, D2) < 1e-13
    G = torch.randn_like(D)
    for u, v in zip(torch.autograd.grad((D * G).sum(), (phi, msg, Y)), torch.autograd.grad((D2 * G).sum(), (phi, msg, Y))):
        assert rel(u, v) < 1e-12


@pytest.mark.parametrize("dt,nc", [(torch.float64, 10), (torch.float32, 10), (torch.float32, 1)])
def test_density_msg_fused_matches_composed(small_graph, dt, nc):
    """DensityMsg (message + density with the fused adjoint) against EdgeMsg followed by Density on the same
    inputs: D and the gradients with respect to phi, Y, TJ, TI."""
    from face_b200.ops import Density, DensityMsg, EdgeMsg
    g = small_graph
    E = g["ei"].numel()
    N = g["pos"].shape[0]
    torch.manual_seed(11)
    mk = lambda *s: torch.randn(*s, device=DEV, dtype=torch.float64).to(dt).requires_grad_(True)
    phi, Y, TJ = mk(E, 16), mk(E, 20), mk(nc, N, 32)
    TI = mk(nc, N, 32) if nc > 1 else None
    wrt = [phi, Y, TJ] + ([TI] if TI is not None else [])
    D1 = torch.cat(DensityMsg.apply(phi, Y, TJ, TI, g), 0)
    D2 = torch.cat(Density.apply(phi, EdgeMsg.apply(Y, TJ, TI, g), Y, g), 0)
    tol = 1e-12 if dt == torch.float64 else 1e-5
    assert rel(D1.detach().double(), D2.detach().double()) < tol
    G = torch.randn_like(D1)
    g1 = torch.autograd.grad((D1 * G).sum(), wrt)
    g2 = torch.autograd.grad((D2 * G).sum(), wrt)
    for a, b in zip(g1, g2):
        assert rel(a.double(), b.double()) < tol


@pytest.mark.parametrize("rows", ["alloy", "long_rows"])
@pytest.mark.parametrize("nc", [1, 10])
def test_density_adjoint_tensor_core(small_graph, rows, nc):
    """facek_density_msg_tc_xm_bwd (tcgen05, edges as M) against the float64 CUDA-core adjoint on the same inputs:
    dphi, dmsg, dY with the message part.  "long_rows": rows of 130-300 edges (chunks of 128 edges of one atom)
    and empty rows.  Bar: 4x the error of the fp32 CUDA-core kernel against float64 (and at most 2e-5 relative)."""
    from face_b200 import _lib
    if rows == "alloy":
        rp = small_graph["row_ptr"].long()
        ei, ej = small_graph["ei"], small_graph["ej"]
    else:
        deg = torch.tensor([130, 0, 300, 7, 0, 256, 129, 45], device=DEV)
        rp = torch.zeros(deg.numel() + 1, dtype=torch.long, device=DEV)
        rp[1:] = torch.cumsum(deg, 0)
        ei = torch.repeat_interleave(torch.arange(deg.numel(), device=DEV), deg).int()
        ej = torch.randint(0, deg.numel(), (int(rp[-1]),), device=DEV).int()
    N, E = rp.numel() - 1, int(rp[-1])
    torch.manual_seed(13)
    r64 = lambda *sh: torch.randn(*sh, device=DEV, dtype=torch.float64)
    phi, msg, Y = r64(E, 16), r64(E, 32), r64(E, 20)
    G = [r64(k, N, 512) for k in (1, 3, 6, 10)]
    TJ, TI = r64(nc, N, 32), r64(nc, N, 32)
    row_ptr = rp.int().contiguous()

    def run(dt, tc):
        a = [t.to(dt).contiguous() for t in (phi, msg, Y)]
        gg = [t.to(dt).contiguous() for t in G]
        tj, ti = TJ.to(dt).contiguous(), TI.to(dt).contiguous()
        out = [torch.empty_like(a[0]), torch.empty_like(a[1]), torch.empty_like(a[2])]
        if tc:
            _lib.call("facek_density_msg_tc_xm_bwd", *[_lib.ptr(t) for t in a], *[_lib.ptr(t) for t in gg],
                      _lib.ptr(tj), _lib.ptr(ti), _lib.ptr(ei), _lib.ptr(ej), nc, *[_lib.ptr(t) for t in out], N, E,
                      16, 32, _lib.ptr(row_ptr), _lib.stream())
        else:
            _lib.call("facek_density_msg_xm_bwd", _lib.dtype_tag(a[0]), *[_lib.ptr(t) for t in a],
                      *[_lib.ptr(t) for t in gg], _lib.ptr(tj), _lib.ptr(ti), _lib.ptr(ei), _lib.ptr(ej), nc,
                      *[_lib.ptr(t) for t in out], N, E, 16, 32, _lib.ptr(row_ptr), _lib.stream())
        return [t.double() for t in out]

    ref, simt, tc = run(torch.float64, False), run(torch.float32, False), run(torch.float32, True)
    st = _lib.ctypes.c_int32(0)
    _lib.call("facek_tc_status", _lib.ctypes.byref(st), 1)
    assert st.value == 0, "tensor-core wait ran out"
    for name, r, a, b in zip(("dphi", "dmsg", "dY"), ref, simt, tc):
        e_simt, e_tc = rel(a, r), rel(b, r)
        assert e_tc <= max(4 * e_simt, 1e-7) and e_tc < 2e-5, (name, e_tc, e_simt)


def test_transport_fp64(small_graph):
    from face_b200.ops import EdgeVec, Transport
    g = small_graph
    E = g["ei"].numel()
    N = g["pos"].shape[0]
    B, Kd = 16, 16
    torch.manual_seed(7)
    pos = g["pos"].clone().requires_grad_(True)
    vec = EdgeVec.apply(pos, g)
    phi = torch.randn(E, B, device=DEV, dtype=torch.float64, requires_grad=True)
    Gt = torch.randn(9, N, Kd, device=DEV, dtype=torch.float64, requires_grad=True)
    T1, T2 = Transport.apply(phi, vec, Gt, g)
    DT = torch.cat([T1.reshape(-1), T2.reshape(-1)])
    # torch statement: face_ref.transport_sums on a single padded row per edge, laid out as the two planes
    u = vec / vec.norm(dim=-1, keepdim=True)
    f_src = Gt[:, g["ej"].long()].permute(1, 2, 0)                                       # (E, Kd, 9)
    per = face_ref.transport_sums(phi[:, None, :], u[:, None, :], f_src[:, None])        # (E, B, Kd, 18)
    S = torch.zeros(N, B, Kd, 18, device=DEV, dtype=torch.float64).index_add(0, g["ei"].long(), per)
    S = S.permute(3, 0, 1, 2).reshape(18, N, B * Kd)                                     # (o, N, BKd)
    P1 = torch.stack([S[0:3], S[3:6]], 2).reshape(3, N, 2 * B * Kd)                      # (a, N, [t, BKd])
    P2 = torch.stack([S[6:12], S[12:18]], 2).reshape(6, N, 2 * B * Kd)
    DT2 = torch.cat([P1.reshape(-1), P2.reshape(-1)])
    assert rel(DT, DT2) < 1e-13
    G = torch.randn_like(DT)
    wrt = (pos, phi, Gt)
    for u_, v_ in zip(torch.autograd.grad((DT * G).sum(), wrt), torch.autograd.grad((DT2 * G).sum(), wrt)):
        assert rel(u_, v_) < 1e-12


def test_transport_fp32_matches_fp64(small_graph):
    """fp32 transport (the lane-per-edge backward for B = 16) against the same op in float64 on the same inputs."""
    from face_b200.ops import EdgeVec, Transport
    g = small_graph
    E = g["ei"].numel()
    N = g["pos"].shape[0]
    B, Kd = 16, 16
    torch.manual_seed(9)
    phi0 = torch.randn(E, B, device=DEV, dtype=torch.float64)
    Gt0 = torch.randn(9, N, Kd, device=DEV, dtype=torch.float64)
    G1, G2 = None, None
    out = {}
    for dt in (torch.float64, torch.float32):
        gg = dict(g, pos=g["pos"].to(dt), shift=g["shift"].to(dt))
        pos = gg["pos"].clone().requires_grad_(True)
        phi = phi0.to(dt).requires_grad_(True)
        Gt = Gt0.to(dt).requires_grad_(True)
        T1, T2 = Transport.apply(phi, EdgeVec.apply(pos, gg), Gt, gg)
        if G1 is None:
            G1, G2 = torch.randn_like(T1), torch.randn_like(T2)
        grads = torch.autograd.grad((T1 * G1.to(dt)).sum() + (T2 * G2.to(dt)).sum(), (pos, phi, Gt))
        out[dt] = [T1, T2] + list(grads)
    for a, b in zip(out[torch.float32], out[torch.float64]):
        assert rel(a.detach().double(), b.detach()) < 2e-5


def test_coulomb_real_fp64(small_graph):
    from face_b200.ops import CoulombReal, EdgeVec
    g = small_graph
    N = g["pos"].shape[0]
    torch.manual_seed(8)
    pos = g["pos"].clone().requires_grad_(True)
    q = torch.randn(N, device=DEV, dtype=torch.float64, requires_grad=True)
    e = CoulombReal.apply(EdgeVec.apply(pos, g), q, g, 1.0, 3.125)
    pos2 = g["pos"].clone().requires_grad_(True)
    r = _torch_vec(g, pos2).norm(dim=-1)
    ei, ej = g["ei"].long(), g["ej"].long()
    K = (torch.erf(r / 1.0) - torch.erf(r / 3.125)) / r
    e2 = torch.zeros(N, device=DEV, dtype=torch.float64).index_add(0, ei, 0.5 * q[ei] * q[ej] * K)
    assert rel(e, e2) < 1e-13
    w = torch.rand(N, device=DEV, dtype=torch.float64)
    for u, v in zip(torch.autograd.grad((e * w).sum(), (pos, q)), torch.autograd.grad((e2 * w).sum(), (pos2, q))):
        assert rel(u, v) < 1e-11


def test_pme_golden_fp64():
    """Reciprocal PME energy and its position/charge gradients against the reference (golden) at an explicit mesh."""
    from face_b200.ops import PMERecip
    k = load("electrostatics")
    pos = torch.tensor(k["rand_pos"], device=DEV, requires_grad=True)
    q = torch.tensor(k["rand_q"], device=DEV, requires_grad=True)
    cell = np.asarray(k["rand_cell"], np.float64)
    e = PMERecip.apply(pos, q, np.linalg.inv(cell), abs(float(np.linalg.det(cell))), 1 / 0.32, (23, 20, 25))
    gp, gq = torch.autograd.grad(e, (pos, q))
    assert abs(float(e) - float(k["recip_e"])) < 1e-12 * abs(float(k["recip_e"]))
    assert float((gp.cpu() - torch.tensor(k["recip_dpos"])).abs().max()) < 1e-11
    assert float((gq.cpu() - torch.tensor(k["recip_dq"])).abs().max()) < 1e-11


@pytest.mark.parametrize("entry", ["facek_density_xm_fwd", "facek_density_tc_xm_fwd"])
def test_density_xm_fwd_fp32_ragged_rows(entry):
    """Flagship shape (B=16, K=32) in fp32 (CUDA-core default and tensor-core entry) on CSR rows of degree 0..150
    (empty rows, ragged 8-edge steps, rows spanning three 64-edge blocks) through the C ABI, against the default
    entry point in float64."""
    from face_b200 import _lib
    g = torch.Generator().manual_seed(12)
    N = 2003
    deg = torch.randint(0, 80, (N,), generator=g)
    deg[::9] = 0
    deg[5::97] = 150
    row_ptr = torch.zeros(N + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(deg, 0).to(torch.int32)
    E = int(row_ptr[-1])
    row_ptr = row_ptr.to(DEV)
    phi = torch.randn(E, 16, generator=g, dtype=torch.float64).to(DEV)
    msg = torch.randn(E, 32, generator=g, dtype=torch.float64).to(DEV)
    Y = torch.randn(E, 20, generator=g, dtype=torch.float64).to(DEV)
    out = {}
    for dt in (torch.float64, torch.float32):
        a = [t.to(dt).contiguous() for t in (phi, msg, Y)]
        D = torch.full((20, N, 512), float("nan"), dtype=dt, device=DEV)
        p = _lib.ptr
        if dt == torch.float32 and entry == "facek_density_tc_xm_fwd":
            _lib.call(entry, *[p(t) for t in a], p(D), N, 16, 32, p(row_ptr), _lib.stream())
        else:
            _lib.call("facek_density_xm_fwd", _lib.dtype_tag(a[0]), *[p(t) for t in a], p(D), N, 16, 32,
                      p(row_ptr), _lib.stream())
        torch.cuda.synchronize()
        out[dt] = D
    assert torch.isfinite(out[torch.float32]).all()
    assert rel(out[torch.float32].double(), out[torch.float64]) < 1e-5
    empty = (deg == 0).nonzero().flatten().to(DEV)
    assert (out[torch.float32][:, empty] == 0).all()
    import ctypes
    st = ctypes.c_int32(-1)
    _lib.call("facek_tc_status", ctypes.byref(st), 1)
    assert st.value == 0


def test_density_xm_bwd_fp32_ragged_rows():
    """Flagship shape (B=16, K=32) in fp32 on CSR rows of degree 0..70 (empty rows included) through the C ABI,
    against the same entry point in float64."""
    from face_b200 import _lib
    g = torch.Generator().manual_seed(8)
    N = 3001
    deg = torch.randint(0, 71, (N,), generator=g)
    deg[::7] = 0
    row_ptr = torch.zeros(N + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(deg, 0).to(torch.int32)
    E = int(row_ptr[-1])
    row_ptr = row_ptr.to(DEV)
    phi = torch.randn(E, 16, generator=g, dtype=torch.float64).to(DEV)
    msg = torch.randn(E, 32, generator=g, dtype=torch.float64).to(DEV)
    Y = torch.randn(E, 20, generator=g, dtype=torch.float64).to(DEV)
    Gs = [torch.randn(k, N, 512, generator=g, dtype=torch.float64).to(DEV) for k in (1, 3, 6, 10)]
    out = {}
    for dt in (torch.float64, torch.float32):
        a = [t.to(dt).contiguous() for t in (phi, msg, Y)]
        G = [t.to(dt).contiguous() for t in Gs]
        d = [torch.full((E, c), float("nan"), dtype=dt, device=DEV) for c in (16, 32, 20)]
        p = _lib.ptr
        _lib.call("facek_density_xm_bwd", _lib.dtype_tag(a[0]), *[p(t) for t in a], *[p(t) for t in G],
                  *[p(t) for t in d], N, 16, 32, p(row_ptr), _lib.stream())
        torch.cuda.synchronize()
        out[dt] = d
    for u, v in zip(out[torch.float32], out[torch.float64]):
        assert torch.isfinite(u).all()
        assert rel(u.double(), v) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("J,N,C,lds", [(1, 1000, 64, 64), (10, 3001, 64, 128), (6, 257, 6, 6), (3, 50, 8, 11), (0, 5, 4, 4)])
def test_bcast_mul_matches_torch(dtype, J, N, C, lds):
    """facek_bcast_mul_fwd/bwd (moment scaling and gates, face/model.py:183-186, :277-295) against torch: exact in
    the forward and dx (one product each), ds within rounding of a J-term sum; s as a column slice of wider rows."""
    from face_b200 import _lib
    from face_b200.ops import BcastMul
    g = torch.Generator(device="cuda").manual_seed(J * 7 + C)
    x = torch.randn(J, N, C, dtype=dtype, device="cuda", generator=g, requires_grad=True)
    wide = torch.randn(N, lds, dtype=dtype, device="cuda", generator=g)
    s = wide[:, :C].requires_grad_(False)
    s_req = s.clone().requires_grad_(True)
    y = BcastMul.apply(x, s_req)
    assert torch.equal(y, x * s_req[None])
    G = torch.randn_like(y)
    dx, ds = torch.autograd.grad((y * G).sum(), (x, s_req))
    assert torch.equal(dx, G * s_req[None])
    tol = 1e-5 if dtype == torch.float32 else 1e-13
    ref = (G * x).sum(0)
    assert (ds - ref).abs().max() <= tol * max(1.0, float(ref.abs().max()))
    # column slice without a copy (lds > C) and without ds
    out = torch.empty(J, N, C, dtype=dtype, device="cuda")
    _lib.call("facek_bcast_mul_fwd", _lib.dtype_tag(x), _lib.ptr(x.detach()), _lib.ptr(s), _lib.ptr(out), J, N, C,
              lds, _lib.stream())
    assert torch.equal(out, x.detach() * s[None])
    dx2 = torch.empty_like(out)
    _lib.call("facek_bcast_mul_bwd", _lib.dtype_tag(x), _lib.ptr(G), None, _lib.ptr(s), _lib.ptr(dx2), None, J, N, C,
              lds, _lib.stream())
    assert torch.equal(dx2, G * s[None])
