"""Damped Cholesky chain: ``H -> U`` with ``H^-1 = U^T U`` (numpy float32).

``damped_upper_inverse_factor`` follows the reference chain
(gptq_utils.py:286-311, duplicated in g2ptq_utils.py:424-450,
gptaq_utils.py:317-343, gptq_guided_utils.py:140-165):

    damp = p * mean(diag H);  L = chol(H + damp I);  Hinv = cholesky_inverse(L)
    U = chol(Hinv, upper=True)
    on a non-PD pivot or a NaN: p += 0.0015 and retry while 0 < p < 1.

``ul_upper_inverse_factor`` is the route the GPU kernel takes to the same
``U``: the "upper-lower" factorization ``H + damp I = V V^T`` with ``V`` upper
triangular gives ``H^-1 = V^-T V^-1``, so ``U = V^-1``.  ``V`` is the reversal
of the ordinary lower factor of the reversed matrix.  It costs
potrf + trtri (2C^3/3) instead of potrf + potri + potrf (4C^3/3).
"""

import numpy as np

f32 = np.float32
DAMP_INCREMENT = 0.0015


class NotPositiveDefinite(Exception):
    """Raised where torch raises ``torch._C._LinAlgError``."""


def _chol_lower(A):
    try:
        return np.linalg.cholesky(A.astype(f32)).astype(f32)
    except np.linalg.LinAlgError as e:
        raise NotPositiveDefinite(str(e))


def reference_chain(H, damp_percent):
    """One attempt of gptq_utils.py:295-304 at a fixed damp percentage."""
    C = H.shape[0]
    damp = f32(damp_percent) * np.mean(np.diag(H), dtype=f32)
    Ht = H.astype(f32).copy()
    Ht[np.arange(C), np.arange(C)] += damp
    L = _chol_lower(Ht)
    Linv = np.linalg.inv(L).astype(f32)
    Hinv = (Linv.T @ Linv).astype(f32)
    Hinv = ((Hinv + Hinv.T) * f32(0.5)).astype(f32)
    U = _chol_lower(Hinv).T.copy()
    if np.isnan(U).any():
        raise NotPositiveDefinite("NaN")
    return U, Hinv


def ul_chain(H, damp_percent):
    """One attempt of the UL route at a fixed damp percentage -> ``(U, Hinv)``."""
    C = H.shape[0]
    damp = f32(damp_percent) * np.mean(np.diag(H), dtype=f32)
    Ht = H.astype(f32).copy()
    Ht[np.arange(C), np.arange(C)] += damp
    R = Ht[::-1, ::-1]
    Lr = _chol_lower(R)
    V = Lr[::-1, ::-1]
    U = np.linalg.inv(V).astype(f32)
    U = np.triu(U)
    if np.isnan(U).any():
        raise NotPositiveDefinite("NaN")
    return U, (U.T @ U).astype(f32)


def damped_upper_inverse_factor(H, percdamp=0.01, route="reference"):
    """The retry loop of gptq_utils.py:291-311 -> ``(U, Hinv, damp_percent)``."""
    chain = reference_chain if route == "reference" else ul_chain
    damp_percent = percdamp
    while 1 > damp_percent > 0:
        try:
            U, Hinv = chain(H, damp_percent)
            return U, Hinv, damp_percent
        except NotPositiveDefinite:
            damp_percent += DAMP_INCREMENT
    raise ValueError(
        f"Quantization: `damp_percent` must between 0 and 1. current is {damp_percent}")
