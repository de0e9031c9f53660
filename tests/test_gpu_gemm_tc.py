"""Tensor-core GEMM (facek_gemm_tc, tcgen05 kind::tf32 with the 3-term split and per-chunk fp32 partial sums)
against float64 torch on the same inputs: ragged M, K and N tails, strided A, bias and accumulate epilogues, the
wide-N tiling, and the autograd Function the engine routes its channel maps through (face-mlip
face/model.py:502-534, :324-339 use torch.nn.Linear there).  Bar: within 4x the error of torch's own fp32
(CUDA-core) GEMM on the same inputs, or 2e-6 of the largest output."""
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = "cuda"


def _rel(a, b):
    return float((a.double() - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _status():
    import ctypes
    from face_b200 import _lib
    v = ctypes.c_int32(-1)
    _lib.call("facek_tc_status", ctypes.byref(v), 1)
    return v.value


@pytest.mark.parametrize("M,K,N", [(1, 4, 4), (127, 32, 64), (128, 64, 192), (1000, 644, 128), (5000, 512, 64),
                                   (3000, 64, 512), (300, 128, 192), (257, 36, 20), (70_001, 512, 64),
                                   (2048, 576, 128), (129, 8, 256)])
def test_gemm_matches_fp64(M, K, N):
    from face_b200.ops import Dense, _gemm
    g = torch.Generator(device=DEV).manual_seed(M + K + N)
    A = torch.randn(M, K, device=DEV, generator=g)
    W = torch.randn(K, N, device=DEV, generator=g) * K ** -0.5
    b = torch.randn(N, device=DEV, generator=g)
    d = Dense(W, b)
    C = torch.full((M, N), float("nan"), device=DEV)
    _gemm(A, d.img, K, N, d.b, C, 0)
    ref = A.double() @ W.double() + b.double()
    e_tc, e_32 = _rel(C, ref), _rel(A @ W + b, ref)
    assert torch.isfinite(C).all()
    assert e_tc < max(4 * e_32, 2e-6), (e_tc, e_32)
    # adjoint image: dA = dC . W^T
    G = torch.randn(M, N, device=DEV, generator=g)
    dA = torch.empty(M, K, device=DEV)
    _gemm(G, d.imgT, N, K, None, dA, 0)
    r2 = G.double() @ W.double().t()
    assert _rel(dA, r2) < max(4 * _rel(G @ W.t(), r2), 2e-6)
    assert _status() == 0


def test_gemm_strided_a_and_accumulate():
    from face_b200.ops import Dense, _gemm
    g = torch.Generator(device=DEV).manual_seed(1)
    big = torch.randn(6000, 48, device=DEV, generator=g)
    A = big[:, :32]                                                # lda = 48 > K = 32
    W = torch.randn(32, 96, device=DEV, generator=g) / 6
    C0 = torch.randn(6000, 96, device=DEV, generator=g)
    C = C0.clone()
    d = Dense(W)
    _gemm(A, d.img, 32, 96, None, C, 1)
    ref = C0.double() + A.double() @ W.double()
    assert _rel(C, ref) < 2e-6
    assert _status() == 0


def test_gemm_rejects_unaligned_k():
    from face_b200.ops import Dense, _gemm
    d = Dense(torch.randn(8, 8, device=DEV))
    A = torch.randn(10, 6, device=DEV)                             # K = 6 is not a multiple of 4
    with pytest.raises(RuntimeError, match="facek_gemm_tc"):
        _gemm(A, d.img, 6, 8, None, torch.empty(10, 8, device=DEV), 0)


def test_tcmatmul_autograd_two_terms():
    from face_b200.ops import Dense, TCMatmul
    g = torch.Generator(device=DEV).manual_seed(2)
    x1 = torch.randn(3, 777, 512, device=DEV, generator=g, requires_grad=True)
    x2 = torch.randn(3, 777, 256, device=DEV, generator=g, requires_grad=True)
    W1 = torch.randn(512, 64, device=DEV, generator=g) / 22
    W2 = torch.randn(256, 64, device=DEV, generator=g) / 16
    y = TCMatmul.apply(x1, Dense(W1), x2, Dense(W2))
    G = torch.randn_like(y)
    g1, g2 = torch.autograd.grad((y * G).sum(), (x1, x2))
    X1, X2 = x1.double().detach(), x2.double().detach()
    assert _rel(y, X1 @ W1.double() + X2 @ W2.double()) < 2e-6
    assert _rel(g1, G.double() @ W1.double().t()) < 2e-6
    assert _rel(g2, G.double() @ W2.double().t()) < 2e-6
    assert _status() == 0


@pytest.mark.parametrize("M,K,N", [(1001, 64, 100), (300, 64, 512), (129, 512, 64), (5000, 96, 128)])
def test_gemm_tma_store_bias_and_accumulate(M, K, N):
    """64- and 128-column tiles leave by TMA (bulk store; bulk add when accumulating): ragged M and N tails are
    clipped by the copy engine, bias is added before the store, and C += A.W + b goes through the bulk add."""
    from face_b200.ops import Dense, _gemm
    g = torch.Generator(device=DEV).manual_seed(M * 3 + N)
    big = torch.full((M + 3, N + 8), float("nan"), device=DEV)
    A = torch.randn(M, K, device=DEV, generator=g)
    W = torch.randn(K, N, device=DEV, generator=g) * K ** -0.5
    b = torch.randn(N, device=DEV, generator=g)
    d = Dense(W, b)
    C = big[:M, :N]                                                 # ldc = N + 8; neighbours stay NaN
    C0 = torch.randn(M, N, device=DEV, generator=g)
    C.copy_(C0)
    _gemm(A, d.img, K, N, d.b, C, 1)
    ref = C0.double() + A.double() @ W.double() + b.double()
    assert _rel(C, ref) < max(4 * _rel(C0 + A @ W + b, ref), 2e-6)
    assert torch.isnan(big[:M, N:]).all() and torch.isnan(big[M:]).all()    # nothing written outside C
    _gemm(A, d.img, K, N, d.b, C, 0)
    ref = A.double() @ W.double() + b.double()
    assert _rel(C, ref) < max(4 * _rel(A @ W + b, ref), 2e-6)
    assert _status() == 0


def _split(A1, A2, d, C1, N1, C2, beta, bias=None):
    from face_b200 import _lib
    p = _lib.ptr
    K1 = A1.shape[1]
    _lib.call("facek_gemm_tc_split", p(A1), A1.stride(0), K1, p(A2), A2.stride(0) if A2 is not None else 0,
              A1.shape[0], d.K, p(d.img), d.N, p(bias), p(C1), C1.stride(0), N1, p(C2),
              C2.stride(0) if C2 is not None else 0, beta, _lib.stream())


@pytest.mark.parametrize("M,K1,K2,N", [(1000, 64, 64, 192), (70_001, 64, 64, 128), (257, 32, 36, 64),
                                       (3000, 576, 64, 128), (129, 128, 4, 512)])
def test_gemm_split_input_is_the_concatenated_gemm(M, K1, K2, N):
    """[A1 | A2] . W from two tensors (facek_gemm_tc_split) reads the same bytes into the same MMAs as the GEMM on
    the concatenated input, so the outputs agree bit for bit (bias included, ragged rows, ragged K2)."""
    from face_b200.ops import Dense, _gemm
    g = torch.Generator(device=DEV).manual_seed(M + K2 + N)
    A1 = torch.randn(M, K1, device=DEV, generator=g)
    A2 = torch.randn(M, K2, device=DEV, generator=g)
    W = torch.randn(K1 + K2, N, device=DEV, generator=g) * (K1 + K2) ** -0.5
    b = torch.randn(N, device=DEV, generator=g)
    d = Dense(W, b)
    C = torch.full((M, N), float("nan"), device=DEV)
    _gemm(torch.cat([A1, A2], 1), d.img, K1 + K2, N, d.b, C, 0)
    Cs = torch.full((M, N), float("nan"), device=DEV)
    _split(A1, A2, d, Cs, N, None, 0, d.b)
    assert torch.equal(C, Cs)
    assert _status() == 0


@pytest.mark.parametrize("M,K,N,N1", [(1000, 192, 128, 64), (70_001, 192, 128, 64), (300, 64, 512, 256),
                                      (129, 64, 96, 32), (5000, 128, 640, 576)])
@pytest.mark.parametrize("beta", [0, 1])
def test_gemm_split_output_is_the_single_output(M, K, N, N1, beta):
    """C = [C1 | C2] written as two tensors (each 32-column store block to one of them; bulk add when accumulating)
    equals the single-output GEMM's columns bit for bit, and nothing outside C1, C2 is written."""
    from face_b200.ops import Dense, _gemm
    g = torch.Generator(device=DEV).manual_seed(M + N1 + beta)
    A = torch.randn(M, K, device=DEV, generator=g)
    d = Dense(torch.randn(K, N, device=DEV, generator=g) * K ** -0.5)
    C0 = torch.randn(M, N, device=DEV, generator=g)
    C = C0.clone()
    _gemm(A, d.img, K, N, None, C, beta)
    big1 = torch.full((M + 2, N1 + 8), float("nan"), device=DEV)
    big2 = torch.full((M + 2, N - N1 + 4), float("nan"), device=DEV)
    C1, C2 = big1[:M, :N1], big2[:M, :N - N1]
    C1.copy_(C0[:, :N1])
    C2.copy_(C0[:, N1:])
    _split(A, None, d, C1, N1, C2, beta)
    assert torch.equal(C1, C[:, :N1]) and torch.equal(C2, C[:, N1:])
    assert torch.isnan(big1[:M, N1:]).all() and torch.isnan(big1[M:]).all()
    assert torch.isnan(big2[:M, N - N1:]).all() and torch.isnan(big2[M:]).all()
    assert _status() == 0


def test_tcmatmul_cat_autograd():
    """The engine's split-input layer: forward and both input gradients against float64 torch on the concatenation."""
    from face_b200.ops import Dense, TCMatmulCat
    g = torch.Generator(device=DEV).manual_seed(5)
    x1 = torch.randn(10, 3001, 64, device=DEV, generator=g, requires_grad=True)
    x2 = torch.randn(10, 3001, 64, device=DEV, generator=g, requires_grad=True)
    W = torch.randn(128, 192, device=DEV, generator=g) / 11
    y = TCMatmulCat.apply(x1, x2, Dense(W))
    G = torch.randn_like(y)
    g1, g2 = torch.autograd.grad((y * G).sum(), (x1, x2))
    X = torch.cat([x1, x2], -1).double().detach()
    ref = X @ W.double()
    assert _rel(y, ref) < max(4 * _rel(torch.cat([x1, x2], -1).detach() @ W, ref), 2e-6)
    dX = G.double() @ W.double().t()
    assert g1.is_contiguous() and g2.is_contiguous()
    assert _rel(g1, dX[..., :64]) < 2e-6 and _rel(g2, dX[..., 64:]) < 2e-6
    assert _status() == 0


def test_gemm_split_rejects_bad_blocks():
    from face_b200.ops import Dense
    A1 = torch.randn(64, 36, device=DEV)                           # K1 not a multiple of 32
    A2 = torch.randn(64, 28, device=DEV)
    d = Dense(torch.randn(64, 64, device=DEV))
    C = torch.empty(64, 64, device=DEV)
    with pytest.raises(RuntimeError, match="facek_gemm_tc_split"):
        _split(A1, A2, d, C, 64, None, 0)
    A = torch.randn(64, 64, device=DEV)
    C1, C2 = torch.empty(64, 48, device=DEV), torch.empty(64, 16, device=DEV)   # N1 not a multiple of 32
    with pytest.raises(RuntimeError, match="facek_gemm_tc_split"):
        _split(A, None, d, C1, 48, C2, 0)
