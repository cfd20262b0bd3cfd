"""g2q_gram_update_noalloc (library-owned static scratch) against g2q_gram_update
with caller-provided scratch, both called through the C ABI.

Two calls in a row on each (an alpha-scaled first fold, then an accumulating
one) must agree within the tensor-core Gram tolerance (1e-5 relative
Frobenius error, the same bar as the other tensor-core Gram tests); requests
above the static scratch must be rejected with G2Q_ERR_SCRATCH_LIMIT.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from g2ptq_b200 import _lib  # noqa: E402

DEV = "cuda"
BF16, F32 = 0, 1
TOL = 1e-5


def rel_fro(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def code(t):
    return BF16 if t.dtype == torch.bfloat16 else F32


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def existing(lib, D, A, B, s, sym, alpha, beta, status=None):
    T, M = A.shape
    N = B.shape[1]
    nbytes = lib.g2q_gram_workspace_bytes(M, N, T, 1)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=DEV)
    return lib.g2q_gram_update(ptr(D), D.stride(0), M, N, ptr(A), code(A), A.stride(0), ptr(B),
                               code(B), B.stride(0), ptr(s), 0 if s is None else s.stride(0), T,
                               int(sym), alpha, beta, 1, ptr(ws), nbytes, ptr(status), stream())


def noalloc(lib, D, A, B, s, sym, alpha, beta, status=None):
    T, M = A.shape
    N = B.shape[1]
    return lib.g2q_gram_update_noalloc(ptr(D), D.stride(0), M, N, ptr(A), code(A), A.stride(0),
                                       ptr(B), code(B), B.stride(0), ptr(s),
                                       0 if s is None else s.stride(0), T, int(sym), alpha, beta,
                                       ptr(status), stream())


@pytest.mark.parametrize("case", ["f32_sym", "bf16_scaled", "f32_cross", "bf16_plain"])
def test_noalloc_matches_existing_two_calls(case):
    lib = _lib.load()
    g = torch.Generator(device=DEV).manual_seed(17)
    T, C = (1024, 4096) if case == "f32_sym" else (1000, 640)
    D0 = torch.randn(C, C, device=DEV, generator=g)
    D0 = D0 + D0.T
    D_ref, D_new = D0.clone(), D0.clone()
    expect = D0.double()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for step, alpha in enumerate((0.5, 1.0)):
        X = torch.randn(T, C, device=DEV, generator=g)
        X[:, 3] *= 20
        s = None
        Y, sym = X, True
        if case == "bf16_scaled":
            X = X.to(torch.bfloat16)
            Y = X
            s = torch.rand(T, 2, device=DEV, generator=g)[:, 1]
            sym = True
        elif case == "f32_cross":
            Y = torch.randn(T, C, device=DEV, generator=g)
            sym = False
        elif case == "bf16_plain":
            X = X.to(torch.bfloat16)
            Y = X
        beta = 2.0 / (step + 3)
        assert existing(lib, D_ref, Y, X, s, sym, alpha, beta) == 0
        assert noalloc(lib, D_new, Y, X, s, sym, alpha, beta, status) == 0
        w = torch.ones(T, device=DEV, dtype=torch.float64) if s is None else s.double()
        expect = alpha * expect + beta * (Y.double().T @ (X.double() * w[:, None]))
    torch.cuda.synchronize()
    assert int(status.item()) == 0  # no tensor-core wait gave up
    assert rel_fro(D_new, D_ref) < TOL
    assert rel_fro(D_new, expect) < TOL
    assert torch.isfinite(D_new).all()


def test_noalloc_rejects_requests_above_the_static_scratch():
    lib = _lib.load()
    cap = lib.g2q_gram_static_scratch_bytes()
    assert cap == 40 << 20
    C = 4096
    T = cap // (8 * C) + 64  # the four bf16 split buffers no longer fit
    assert lib.g2q_gram_workspace_bytes(C, C, T, 1) > cap
    D = torch.zeros(C, C, device=DEV)
    X = torch.zeros(T, C, device=DEV)
    st = noalloc(lib, D, X, X, None, True, 1.0, 1.0)
    assert st == _lib.G2Q_ERR_SCRATCH_LIMIT
    assert "static scratch" in _lib.status_string(st)
    # BF16 without a row scale needs no scratch: the same size is accepted
    Xb = torch.ones(T, C, device=DEV, dtype=torch.bfloat16)
    assert noalloc(lib, D, Xb, Xb, None, True, 0.0, 1.0 / T) == 0
    torch.cuda.synchronize()
    assert torch.allclose(D, torch.ones_like(D), rtol=1e-6, atol=0)
