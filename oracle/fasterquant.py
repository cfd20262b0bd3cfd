"""Whole ``fasterquant`` pipelines (numpy float32).

  gptq_fasterquant    gptq_utils.py:234-353
  g2ptq_fasterquant   g2ptq_utils.py:349-519
  gptaq_fasterquant   gptaq_utils.py:263-391
  guided_fasterquant  gptq_guided_utils.py:83-211
Inputs are the stacked layer weights ``[B, R, C]`` and the accumulated
statistics; outputs are ``(Q, W_int, Scale)`` in the original column order
(the values the reference writes back / hands to ``compress``).
"""

import numpy as np

from . import linalg
from .compensation import (run_compensation_gptq, run_compensation_g2ptq,
                           run_compensation_gptaq)

f32 = np.float32


def _init_static(quantizers, W_flat, groupsize, static_groups, H_diag):
    """gptq_utils.py:259-270."""
    if groupsize == -1 or static_groups:
        for i, qz in enumerate(quantizers):
            if not qz.ready():
                if groupsize == -1:
                    qz.find_params(W_flat, H_diag)
                else:
                    qz.find_params(W_flat[:, i * groupsize:(i + 1) * groupsize],
                                   None if H_diag is None
                                   else H_diag[:, i * groupsize:(i + 1) * groupsize])


def _dead_columns(H, W):
    """gptq_utils.py:272-277 on one layer; mutates both."""
    C = H.shape[0]
    if (H == 0).all():
        H[:] = np.eye(C, dtype=f32)
    dead = np.diag(H) == 0
    H[dead, dead] = 1
    W[:, dead] = 0
    return dead


def argsort_desc(v):
    """``torch.argsort(v, descending=True)``; ties keep index order."""
    return np.argsort(-np.asarray(v, np.float64), kind="stable")


def _factor_all(H, percdamp, route):
    B, C, _ = H.shape
    U = np.empty_like(H)
    Hinv = np.empty_like(H)
    damps = []
    for b in range(B):
        U[b], Hinv[b], d = linalg.damped_upper_inverse_factor(H[b], percdamp, route)
        damps.append(d)
    return U, Hinv, damps


def _given_factor(U):
    """A factor supplied by the caller (a test comparing the compensation on
    one shared U): ``(U, U^T U, damps unknown)``."""
    U = np.asarray(U, f32)
    return U, (U.transpose(0, 2, 1) @ U).astype(f32), None


def gptq_fasterquant(W, H, quantizers, blocksize=128, percdamp=0.01, groupsize=-1,
                     actorder=False, static_groups=False, route="reference", U=None):
    """gptq_utils.py:234-353 -> ``(Q, W_int, Scale, info)``.

    ``U`` (optional, ``[B, C, C]``, in the act-order column order) replaces the
    damped Cholesky chain, so that the rest of the pipeline can be compared
    on a factor computed elsewhere."""
    W = np.asarray(W, f32).copy()
    H = np.asarray(H, f32).copy()
    B, R, C = W.shape
    hclip = quantizers[0].hclip
    H_diag = np.diagonal(H, axis1=1, axis2=2).copy() if hclip else None
    _init_static(quantizers, W.reshape(B * R, C), groupsize, static_groups, H_diag)
    for b in range(B):
        _dead_columns(H[b], W[b])
    perm = invperm = None
    if actorder:
        perm = argsort_desc(np.mean(np.diagonal(H, axis1=1, axis2=2), axis=0))
        invperm = np.argsort(perm)
        W = W[:, :, perm].copy()
        H = H[:, perm][:, :, perm].copy()
    U, _, damps = _factor_all(H, percdamp, route) if U is None else _given_factor(U)
    if H_diag is not None and actorder:
        H_diag = H_diag[:, perm].copy()
    Q, W_int, Scale = run_compensation_gptq(
        W, U, quantizers, blocksize, groupsize, static_groups,
        perm if (static_groups and actorder) else None, H_diag)
    if actorder:
        Q, W_int, Scale = Q[:, :, invperm], W_int[:, :, invperm], Scale[:, :, invperm]
    return Q, W_int, Scale, {"perm": perm, "U": U, "damp": damps}


def gptaq_fasterquant(W, H, dXXT, quantizers, blocksize=128, percdamp=0.01, groupsize=-1,
                      actorder=False, static_groups=False, alpha=0.25, route="reference"):
    """gptaq_utils.py:263-391 -> ``(Q, W_int, Scale, info)``."""
    W = np.asarray(W, f32).copy()
    H = np.asarray(H, f32).copy()
    dXXT = np.asarray(dXXT, f32).copy()
    B, R, C = W.shape
    hclip = quantizers[0].hclip
    H_diag = np.diagonal(H, axis1=1, axis2=2).copy() if hclip else None
    _init_static(quantizers, W.reshape(B * R, C), groupsize, static_groups, H_diag)
    for b in range(B):
        dead = _dead_columns(H[b], W[b])
        dXXT[b][:, dead] = 0
    perm = invperm = None
    if actorder:
        perm = argsort_desc(np.mean(np.diagonal(H, axis1=1, axis2=2), axis=0))
        invperm = np.argsort(perm)
        W = W[:, :, perm].copy()
        H = H[:, perm][:, :, perm].copy()
        dXXT = dXXT[:, perm][:, :, perm].copy()
    U, _, damps = _factor_all(H, percdamp, route)
    if H_diag is not None and actorder:
        H_diag = H_diag[:, perm].copy()
    P = (f32(alpha) * (np.triu(dXXT @ U.transpose(0, 2, 1), 1) @ U)).astype(f32)
    Q, W_int, Scale = run_compensation_gptaq(
        W, U, P, quantizers, blocksize, groupsize, static_groups,
        perm if (static_groups and actorder) else None, H_diag)
    if actorder:
        Q, W_int, Scale = Q[:, :, invperm], W_int[:, :, invperm], Scale[:, :, invperm]
    return Q, W_int, Scale, {"perm": perm, "U": U, "P": P, "damp": damps}


def fake_quantize_grouped(quantizers, weight, groupsize):
    """common_utils.py:33-45."""
    flat = weight.shape[0] * weight.shape[1]
    width = weight.shape[-1] if groupsize == -1 else groupsize
    out = []
    for g, qz in enumerate(quantizers):
        s = g * width
        e = min(s + width, weight.shape[-1])
        vals = weight[:, :, s:e].reshape(flat, e - s)
        out.append(qz.fake_quantize(vals)[0].reshape(*weight.shape[:2], e - s))
    return np.concatenate(out, axis=-1)


def trust_region(grad, Hinv_init, Q_sub, W_sub, alpha):
    """g2ptq_utils.py:459-472 -> ``beta`` ``[B*G, R/G]``."""
    eps = np.finfo(np.float32).tiny
    GH = (grad @ Hinv_init).astype(f32)
    qe = (Q_sub - W_sub).astype(f32)
    dH = np.diagonal(Hinv_init, axis1=1, axis2=2)[:, None, :]
    loss = np.abs((qe * GH + qe ** 2 / f32(2)) / dH).astype(f32)
    c = (grad * GH).sum(axis=2, keepdims=True, dtype=f32) - (GH ** 2) / dH
    c = np.maximum(c, f32(2 * alpha) * loss)
    c = np.maximum(c, f32(eps))
    beta = (f32(1) - np.sqrt(np.maximum(f32(1) - (f32(2 * alpha) * loss) / c, f32(0)))).mean(
        -1, dtype=f32)
    return beta.astype(f32)


def g2ptq_fasterquant(W, H, act_square, gradients, quantizers, num_groups, blocksize=128,
                      percdamp=0.01, groupsize=-1, actorder=False, static_groups=False,
                      enable_gradient_update=True, alpha=0.0, route="reference", U=None,
                      approx_beta=0.0):
    """g2ptq_utils.py:349-519 -> ``(Q, W_int, Scale, info)``; ``approx_beta`` is
    the object's ``approx_grad_beta`` (the ``--approx_grad`` ablation).

    ``H`` is ``[B, G, C, C]``, ``gradients`` ``[B, R, C]``, ``act_square`` ``[B, C]``;
    ``U`` (optional, ``[B*G, C, C]`` in the act-order column order) replaces the
    damped Cholesky chain (see ``gptq_fasterquant``).
    """
    W = np.asarray(W, f32).copy()
    B, R, C = W.shape
    G = num_groups
    rps = R // G
    W_flat = W.reshape(B * R, C).copy()
    W_sub = W.reshape(B * G, rps, C)
    grad = np.asarray(gradients, f32).reshape(B * G, rps, C).copy()
    H_sub = np.asarray(H, f32).reshape(B * G, C, C).copy()
    hclip = quantizers[0].hclip
    H_diag = np.diagonal(H_sub, axis1=1, axis2=2).copy() if hclip else None
    _init_static(quantizers, W_flat, groupsize, static_groups, H_diag)
    for b in range(B * G):
        if (H_sub[b] == 0).all():
            H_sub[b] = np.eye(C, dtype=f32)
            grad[b] = 0
        dead = np.diag(H_sub[b]) == 0
        H_sub[b][dead, dead] = 1
        W_sub[b][:, dead] = 0
    Q_sub = None
    use_grad = enable_gradient_update and alpha > 0
    if use_grad:
        if groupsize != -1 and not static_groups:
            for i, qz in enumerate(quantizers):
                qz.find_params(W_sub[:, :, i * groupsize:(i + 1) * groupsize].reshape(B * R, -1))
        Q_sub = fake_quantize_grouped(quantizers, W_sub, groupsize)
    perm = invperm = None
    if actorder:
        perm = argsort_desc(np.mean(np.asarray(act_square, f32), axis=0))
        invperm = np.argsort(perm)
        W_sub = W_sub[:, :, perm].copy()
        H_sub = H_sub[:, perm][:, :, perm].copy()
        grad = grad[:, :, perm].copy()
    U, Hinv_init, damps = (_factor_all(H_sub, percdamp, route) if U is None
                           else _given_factor(U))
    if Q_sub is not None and actorder:
        Q_sub = Q_sub[:, :, perm]
    if H_diag is not None and actorder:
        H_diag = H_diag[:, perm].copy()
    if use_grad:
        beta = trust_region(grad, Hinv_init, Q_sub, W_sub, alpha)
    else:
        beta = np.zeros((B * G, 1), f32)
    Z = ((grad @ U.transpose(0, 2, 1)) * beta[:, :, None]).astype(f32)
    GHinv = (Z @ U).astype(f32)
    Wc = W_sub.copy()
    Q, W_int, Scale = run_compensation_g2ptq(
        Wc, U, Z, GHinv, quantizers, blocksize, groupsize, static_groups,
        perm if (static_groups and actorder) else None, H_diag, approx_beta)
    if actorder:
        Q, W_int, Scale = Q[:, :, invperm], W_int[:, :, invperm], Scale[:, :, invperm]
    return (Q.reshape(B, R, C), W_int.reshape(B, R, C), Scale.reshape(B, R, C),
            {"perm": perm, "U": U, "beta": beta, "Z": Z, "damp": damps})


def guided_fasterquant(W, H, act_square, quantizers, num_groups, blocksize=128,
                       percdamp=0.01, groupsize=-1, actorder=False, static_groups=False,
                       route="reference"):
    """gptq_guided_utils.py:83-211 -> ``(Q, W_int, Scale, info)``."""
    W = np.asarray(W, f32).copy()
    B, R, C = W.shape
    G = num_groups
    rps = R // G
    W_flat = W.reshape(B * R, C).copy()
    W_sub = W.reshape(B * G, rps, C)
    H_sub = np.asarray(H, f32).reshape(B * G, C, C).copy()
    hclip = quantizers[0].hclip
    H_diag = np.diagonal(H_sub, axis1=1, axis2=2).copy() if hclip else None
    _init_static(quantizers, W_flat, groupsize, static_groups, H_diag)
    for b in range(B * G):
        _dead_columns(H_sub[b], W_sub[b])
    perm = invperm = None
    if actorder:
        perm = argsort_desc(np.mean(np.asarray(act_square, f32), axis=0))
        invperm = np.argsort(perm)
        W_sub = W_sub[:, :, perm].copy()
        H_sub = H_sub[:, perm][:, :, perm].copy()
    U, _, damps = _factor_all(H_sub, percdamp, route)
    if H_diag is not None and actorder:
        H_diag = H_diag[:, perm].copy()
    Wc = W_sub.copy()
    Q, W_int, Scale = run_compensation_gptq(
        Wc, U, quantizers, blocksize, groupsize, static_groups,
        perm if (static_groups and actorder) else None, H_diag)
    if actorder:
        Q, W_int, Scale = Q[:, :, invperm], W_int[:, :, invperm], Scale[:, :, invperm]
    return (Q.reshape(B, R, C), W_int.reshape(B, R, C), Scale.reshape(B, R, C),
            {"perm": perm, "U": U, "damp": damps})
