"""The reference's GPTQ path restated with torch CPU operations -- the CPU
baseline of bench.py (test and measurement infrastructure: the product never
imports anything under ``oracle/``).

The reference runs its quantizer objects with torch; on a host without a GPU
the same torch operations run on the CPU cores (MKL / OpenMP matmuls and
LAPACK factorizations).  This module performs those operations in the order
the reference performs them, so that its timings stand for the reference's
own CPU cost on the same host:

  add_batch      gptq_utils.py:115-126   H <- H n/(n+b); X <- sqrt(2/(n+b)) X; H += X^T X
  factor         gptq_utils.py:291-311   Cholesky -> cholesky_inverse -> upper Cholesky,
                                          damp auto-increment on failure
  compensate     gptq_utils.py:165-232   128-column blocks; per column quantize,
                 (+ _run_torch_compensation, error, rank-1 update of the block's
                  gptq_utils.py:28-51)    remaining columns; trailing baddbmm
  fasterquant    gptq_utils.py:234-353   static groups, dead columns, act-order

Quantizer arithmetic follows utils/quant_utils.py:8-16 and 380-404
(``asym_quant`` / ``asym_dequant``, min/max parameters with the range forced
to contain 0).  Only the plain min/max search is restated (no --w_clip).
The reference itself can be imported in the development container; a CPU
test checks this module against it there and against the numpy oracle
everywhere.
"""

import math
import time

import torch

DAMP_INCREMENT = 0.0015


def qrange(bits):
    """``maxq = 2^(b-1) - 1``, ``minq = -(maxq + 1)`` (quant_utils.py:350-375)."""
    maxq = 2 ** (bits - 1) - 1
    return maxq, -(maxq + 1)


def find_params(x, bits, sym):
    """Per-row scale / zero of ``x [rows, cols]`` (quant_utils.py:380-404)."""
    maxq, minq = qrange(bits)
    bit_range = maxq - minq
    lo = torch.clamp(x.min(dim=1).values, max=0)
    hi = torch.clamp(x.max(dim=1).values, min=0)
    if sym:
        scale = torch.maximum(lo.abs(), hi) / (bit_range / 2)
        zero = torch.zeros_like(scale)
    else:
        scale = (hi - lo) / bit_range
        zero = torch.clamp(torch.round(minq - lo / scale), minq, maxq)
    return scale, torch.round(zero)


def quantize(w, scale, zero, maxq):
    """``asym_quant`` then ``asym_dequant`` (quant_utils.py:8-16) -> (q, code)."""
    code = torch.clamp(torch.round(w / scale) + zero, -(maxq + 1), maxq)
    return scale * (code - zero), code


def add_batch(H, n, X):
    """One hook call on ``X [b, S, C]`` (or ``[t, C]``: b = 1) -> ``(H, n)``."""
    if X.dim() == 2:
        X = X.unsqueeze(0)
    b = X.shape[0]
    X = X.reshape(-1, X.shape[-1]).t()
    H *= n / (n + b)
    n += b
    X = math.sqrt(2 / n) * X.float()
    H += X.matmul(X.t())
    return H, n


def factor(H, percdamp=0.01):
    """The damped chain on one ``[C, C]`` Hessian -> ``(U, damp_percent)``."""
    C = H.shape[0]
    d = percdamp
    while 1 > d > 0:
        try:
            Ht = H.clone()
            idx = torch.arange(C)
            Ht[idx, idx] += d * torch.mean(torch.diag(H))
            L = torch.linalg.cholesky(Ht)
            U = torch.linalg.cholesky(torch.cholesky_inverse(L), upper=True)
            if torch.isnan(U).any():
                raise torch._C._LinAlgError
            return U, d
        except torch._C._LinAlgError:
            d += DAMP_INCREMENT
    raise ValueError(f"Quantization: `damp_percent` must between 0 and 1. current is {d}")


def _block(Wb, Ub, S, Z, maxq):
    """One compensation block in the kernel layout ``[B, blk, R]``; in place."""
    B, blk, R = Wb.shape
    codes = torch.empty_like(Wb)
    err = torch.empty_like(Wb)
    for c in range(blk):
        w = Wb[:, c]
        q, code = quantize(w, S[:, c], Z[:, c], maxq)
        e = (w - q) / Ub[:, c, c].unsqueeze(1)
        Wb[:, c] = q
        codes[:, c] = code
        err[:, c] = e
        if c + 1 < blk:
            Wb[:, c + 1:].baddbmm_(Ub[:, c, c + 1:].unsqueeze(2), e.unsqueeze(1), alpha=-1)
    return codes, err


def compensate(W, U, scale, zero, colgroup, bits, blocksize=128, dynamic=None):
    """Block traversal of ``W [B, R, C]`` (in place -> Q) with per-column
    parameter columns ``colgroup[c]`` of ``scale`` / ``zero`` ``[B*R, ngroups]``.
    ``dynamic = (groupsize, sym)`` finds each group's parameters at its first
    column on the current W.  Returns the integer codes ``[B, R, C]``."""
    B, R, C = W.shape
    maxq, _ = qrange(bits)
    codes = torch.empty_like(W)
    for i1 in range(0, C, blocksize):
        i2 = min(i1 + blocksize, C)
        if dynamic is not None:
            gs, sym = dynamic
            for g0 in range((i1 + gs - 1) // gs * gs, i2, gs):
                s, z = find_params(W[:, :, g0:g0 + gs].reshape(B * R, -1), bits, sym)
                scale[:, g0 // gs], zero[:, g0 // gs] = s, z
        cols = colgroup[i1:i2]
        S = scale[:, cols].reshape(B, R, i2 - i1).transpose(1, 2).contiguous()
        Z = zero[:, cols].reshape(B, R, i2 - i1).transpose(1, 2).contiguous()
        Wb = W[:, :, i1:i2].transpose(1, 2).contiguous()
        cb, err = _block(Wb, U[:, i1:i2, i1:i2].contiguous(), S, Z, maxq)
        W[:, :, i1:i2] = Wb.transpose(1, 2)
        codes[:, :, i1:i2] = cb.transpose(1, 2)
        if i2 < C:
            W[:, :, i2:].baddbmm_(err.transpose(1, 2), U[:, i1:i2, i2:], alpha=-1)
    return codes


def fasterquant(W, H, bits, sym, groupsize=128, actorder=False, static_groups=False,
                percdamp=0.01, blocksize=128, timings=None):
    """gptq_utils.py:234-353 on ``W [B, R, C]``, ``H [B, C, C]`` (fp32, CPU)
    -> ``(Q, codes)`` in the original column order.  ``timings`` (a dict)
    receives the seconds spent in the factorization and in the compensation."""
    W = W.float().clone()
    H = H.float().clone()
    B, R, C = W.shape
    ng = 1 if groupsize == -1 else (C + groupsize - 1) // groupsize
    scale = torch.zeros(B * R, ng)
    zero = torch.zeros(B * R, ng)
    dynamic = None
    if groupsize == -1:
        scale[:, 0], zero[:, 0] = find_params(W.reshape(B * R, C), bits, sym)
    elif static_groups:
        Wf = W.reshape(B * R, C)
        for g in range(ng):
            scale[:, g], zero[:, g] = find_params(Wf[:, g * groupsize:(g + 1) * groupsize], bits,
                                                  sym)
    else:
        dynamic = (groupsize, sym)
    for b in range(B):
        if (H[b] == 0).all():
            H[b] = torch.eye(C)
        dead = torch.diag(H[b]) == 0
        H[b, dead, dead] = 1
        W[b, :, dead] = 0
    perm = None
    if actorder:
        perm = torch.argsort(torch.mean(torch.diagonal(H, dim1=1, dim2=2), dim=0),
                             descending=True, stable=True)
        W = W[:, :, perm]
        H = H[:, perm][:, :, perm]
    t0 = time.perf_counter()
    U = torch.stack([factor(H[b], percdamp)[0] for b in range(B)])
    t1 = time.perf_counter()
    if groupsize == -1:
        colgroup = torch.zeros(C, dtype=torch.long)
    elif static_groups and perm is not None:
        colgroup = perm // groupsize
    else:
        colgroup = torch.arange(C) // groupsize
    codes = compensate(W, U, scale, zero, colgroup, bits, blocksize, dynamic)
    t2 = time.perf_counter()
    if timings is not None:
        timings["factor"] = timings.get("factor", 0.0) + (t1 - t0)
        timings["compensate"] = timings.get("compensate", 0.0) + (t2 - t1)
    if perm is not None:
        inv = torch.argsort(perm)
        W, codes = W[:, :, inv], codes[:, :, inv]
    return W, codes
