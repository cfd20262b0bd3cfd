"""Lazy-batch column compensation (numpy float32).

Block kernels (the reference's kernel-level boundary ``run_eager``, layout
``[B, blk, R]``, in place on ``weight`` and, for G2PTQ, ``ghinv``):
  gptq_block     gptq_utils.py:28-51   (_run_torch_compensation)
  g2ptq_block    g2ptq_utils.py:34-74  (_run_torch_compensation)
  gptaq_block    gptaq_utils.py:28-56  (_run_torch_compensation)
Block traversal with group parameters and the trailing update:
  run_compensation_gptq   gptq_utils.py:165-232
  run_compensation_g2ptq  g2ptq_utils.py:252-347
  run_compensation_gptaq  gptaq_utils.py:193-261
"""

import numpy as np

from . import quant

f32 = np.float32


class Quantizer:
    """State of one ``WeightQuantizer`` (quant_utils.py:341-465) as used here."""

    def __init__(self, bits, sym, mse=False, hclip=False):
        self.bits, self.sym, self.mse, self.hclip = bits, sym, mse, hclip
        self.maxq, self.minq, self.bit_range = quant.qrange(bits)
        self.scale = None
        self.zero = None
        self._ready = False

    def ready(self):
        return self._ready

    def find_params(self, x, h_diag=None):
        s, z = quant.find_params(x, self.bits, self.sym, mse=self.mse,
                                 h_diag=h_diag if self.hclip else None)
        self.scale, self.zero, self._ready = s, z, True

    def fake_quantize(self, x):
        return quant.fake_quantize(x, self.scale, self.zero, self.maxq)

    def copy(self):
        q = Quantizer(self.bits, self.sym, self.mse, self.hclip)
        q.scale = None if self.scale is None else self.scale.copy()
        q.zero = None if self.zero is None else self.zero.copy()
        q._ready = self._ready
        return q


def make_group_quantizers(template, columns, groupsize):
    """common_utils.py:13-16."""
    n = 1 if groupsize == -1 else (columns + groupsize - 1) // groupsize
    return [template.copy() for _ in range(n)]


def _quant_column(w, s, z, maxq):
    q = quant.asym_quant(w, s, z, maxq)
    return quant.asym_dequant(q, s, z), q


def gptq_block(weight, hinv, scale, zero, maxq):
    """gptq_utils.py:28-51 on ``[B, blk, R]`` -> ``(weight, int_weight, error)``."""
    weight = weight.astype(f32).copy()
    B, cols, R = weight.shape
    int_weight = np.empty_like(weight)
    error = np.empty_like(weight)
    for c in range(cols):
        w = weight[:, c].copy()
        q, qi = _quant_column(w, scale[:, c], zero[:, c], maxq)
        err = ((w - q) / hinv[:, c, c][:, None]).astype(f32)
        weight[:, c] = q
        int_weight[:, c] = qi
        error[:, c] = err
        if c + 1 < cols:
            weight[:, c + 1:] -= hinv[:, c, c + 1:][:, :, None] * err[:, None, :]
    return weight, int_weight, error


def g2ptq_block(weight, hinv, scale, zero, z, ghinv, maxq, weight_raw=None, approx_beta=0.0):
    """g2ptq_utils.py:34-74 -> ``(weight, int_weight, error, ghinv)``.

    ``approx_beta`` != 0 (the ``--approx_grad`` ablation, lines 48-51 and
    71-73): the column error also subtracts ``(w - weight_raw) * beta``, and
    after each column's update the next column is pulled toward its raw
    value by ``(w_next - raw_next) * beta``."""
    weight = weight.astype(f32).copy()
    ghinv = ghinv.astype(f32).copy()
    beta = f32(approx_beta)
    B, cols, R = weight.shape
    int_weight = np.empty_like(weight)
    error = np.empty_like(weight)
    for c in range(cols):
        w = weight[:, c].copy()
        q, qi = _quant_column(w, scale[:, c], zero[:, c], maxq)
        num = (w - q - ghinv[:, c]).astype(f32)
        if approx_beta:
            num = (num - ((w - weight_raw[:, c]).astype(f32) * beta).astype(f32)).astype(f32)
        err = (num / hinv[:, c, c][:, None]).astype(f32)
        weight[:, c] = q
        int_weight[:, c] = qi
        error[:, c] = err
        if c + 1 < cols:
            row = hinv[:, c, c + 1:][:, :, None]
            weight[:, c + 1:] -= ghinv[:, c + 1:]
            weight[:, c + 1:] -= row * err[:, None, :]
            ghinv[:, c + 1:] -= row * z[:, c][:, None, :]
            if approx_beta:
                drift = ((weight[:, c + 1] - weight_raw[:, c + 1]).astype(f32) * beta)
                weight[:, c + 1] -= drift.astype(f32)
    return weight, int_weight, error, ghinv


def gptaq_block(weight, hinv, p, scale, zero, maxq):
    """gptaq_utils.py:28-56 -> ``(weight, int_weight, error)``."""
    weight = weight.astype(f32).copy()
    B, cols, R = weight.shape
    int_weight = np.empty_like(weight)
    error = np.empty_like(weight)
    for c in range(cols):
        w = weight[:, c].copy()
        q, qi = _quant_column(w, scale[:, c], zero[:, c], maxq)
        err = ((w - q) / hinv[:, c, c][:, None]).astype(f32)
        weight[:, c] = q
        int_weight[:, c] = qi
        error[:, c] = err
        if c + 1 < cols:
            weight[:, c + 1:] -= hinv[:, c, c + 1:][:, :, None] * err[:, None, :]
            weight[:, c + 1:] += p[:, c, c + 1:][:, :, None] * w[:, None, :]
    return weight, int_weight, error


def column_quantizers(quantizers, W, i1, i2, groupsize, static_groups,
                      qparam_perm, num_layers, rows, H_diag=None):
    """The per-block quantizer selection of gptq_utils.py:185-205.

    Dynamic groups call ``find_params`` at each group start on the current
    (already trailing-updated) ``W`` before the block runs.
    """
    if groupsize == -1:
        return [quantizers[0]] * (i2 - i1)
    if static_groups:
        idx = range(i1, i2) if qparam_perm is None else list(qparam_perm[i1:i2])
        return [quantizers[int(i) // groupsize] for i in idx]
    out = []
    for i in range(i1, i2):
        qz = quantizers[i // groupsize]
        if i % groupsize == 0:
            qz.find_params(W[:, :, i:i + groupsize].reshape(num_layers * rows, -1),
                           None if H_diag is None else H_diag[:, i:i + groupsize])
        out.append(qz)
    return out


def _stack_params(cq, shape):
    S = np.stack([q.scale for q in cq], axis=1).reshape(shape).astype(f32)
    Z = np.stack([q.zero for q in cq], axis=1).reshape(shape).astype(f32)
    return S, Z


def run_compensation_gptq(W, Hinv, quantizers, blocksize, groupsize, static_groups,
                          qparam_perm=None, H_diag=None):
    """gptq_utils.py:165-232; mutates ``W`` like the reference -> ``(Q, W_int, Scale)``."""
    B, R, C = W.shape
    Q = np.zeros_like(W)
    W_int = np.zeros_like(W)
    Scale = np.zeros_like(W)
    maxq = quantizers[0].maxq
    for i1 in range(0, C, blocksize):
        i2 = min(i1 + blocksize, C)
        W1 = W[:, :, i1:i2].copy()
        cq = column_quantizers(quantizers, W, i1, i2, groupsize, static_groups,
                               qparam_perm, B, R, H_diag)
        S1, Z1 = _stack_params(cq, W1.shape)
        q, qi, err = gptq_block(W1.transpose(0, 2, 1), Hinv[:, i1:i2, i1:i2],
                                S1.transpose(0, 2, 1), Z1.transpose(0, 2, 1), maxq)
        Q[:, :, i1:i2] = q.transpose(0, 2, 1)
        W_int[:, :, i1:i2] = qi.transpose(0, 2, 1)
        Scale[:, :, i1:i2] = S1
        Err1 = err.transpose(0, 2, 1)
        W[:, :, i2:] -= (Err1 @ Hinv[:, i1:i2, i2:]).astype(f32)
    return Q, W_int, Scale


def run_compensation_g2ptq(W, Hinv, Z, GHinv, quantizers, blocksize, groupsize,
                           static_groups, qparam_perm=None, H_diag=None, approx_beta=0.0):
    """g2ptq_utils.py:252-347; mutates ``W`` and ``GHinv`` -> ``(Q, W_int, Scale)``.
    With ``approx_beta`` the raw weights are the traversal's input ``W``
    (snapshot taken before the first block, line 273)."""
    B, R, C = W.shape
    W_raw = W.copy() if approx_beta else None
    Q = np.zeros_like(W)
    W_int = np.zeros_like(W)
    Scale = np.zeros_like(W)
    D = np.arange(blocksize - 1, -1, -1).astype(f32)
    maxq = quantizers[0].maxq
    for i1 in range(0, C, blocksize):
        i2 = min(i1 + blocksize, C)
        W1 = W[:, :, i1:i2].copy()
        Z1 = Z[:, :, i1:i2]
        GH1 = GHinv[:, :, i1:i2].copy()
        cq = column_quantizers(quantizers, W, i1, i2, groupsize, static_groups,
                               qparam_perm, B, R, H_diag)
        S1, Zr1 = _stack_params(cq, W1.shape)
        q, qi, err, _ = g2ptq_block(W1.transpose(0, 2, 1), Hinv[:, i1:i2, i1:i2],
                                    S1.transpose(0, 2, 1), Zr1.transpose(0, 2, 1),
                                    Z1.transpose(0, 2, 1), GH1.transpose(0, 2, 1), maxq,
                                    None if W_raw is None
                                    else W_raw[:, :, i1:i2].transpose(0, 2, 1), approx_beta)
        Q[:, :, i1:i2] = q.transpose(0, 2, 1)
        W_int[:, :, i1:i2] = qi.transpose(0, 2, 1)
        Scale[:, :, i1:i2] = S1
        if i2 == C:
            continue
        Err1 = err.transpose(0, 2, 1)
        U12 = Hinv[:, i1:i2, i2:]
        # gradient_update is ``blocksize * GHinv`` even for a ragged block
        # (g2ptq_utils.py:327), D has blocksize entries (line 269).
        gu = f32(blocksize) * GHinv[:, :, i2:] - ((Z1 * D[: i2 - i1]) @ U12).astype(f32)
        W[:, :, i2:] -= gu
        W[:, :, i2:] -= (Err1 @ U12).astype(f32)
        GHinv[:, :, i2:] -= (Z1 @ U12).astype(f32)
    return Q, W_int, Scale


def run_compensation_gptaq(W, Hinv, P, quantizers, blocksize, groupsize, static_groups,
                           qparam_perm=None, H_diag=None):
    """gptaq_utils.py:193-261; mutates ``W`` -> ``(Q, W_int, Scale)``."""
    B, R, C = W.shape
    Q = np.zeros_like(W)
    W_int = np.zeros_like(W)
    Scale = np.zeros_like(W)
    maxq = quantizers[0].maxq
    for i1 in range(0, C, blocksize):
        i2 = min(i1 + blocksize, C)
        W1 = W[:, :, i1:i2].copy()
        cq = column_quantizers(quantizers, W, i1, i2, groupsize, static_groups,
                               qparam_perm, B, R, H_diag)
        S1, Z1 = _stack_params(cq, W1.shape)
        q, qi, err = gptaq_block(W1.transpose(0, 2, 1), Hinv[:, i1:i2, i1:i2],
                                 P[:, i1:i2, i1:i2], S1.transpose(0, 2, 1),
                                 Z1.transpose(0, 2, 1), maxq)
        Q1 = q.transpose(0, 2, 1)
        Q[:, :, i1:i2] = Q1
        W_int[:, :, i1:i2] = qi.transpose(0, 2, 1)
        Scale[:, :, i1:i2] = S1
        Err1 = err.transpose(0, 2, 1)
        W[:, :, i2:] -= (Err1 @ Hinv[:, i1:i2, i2:]).astype(f32)
        W[:, :, i2:] += (Q1 @ P[:, i1:i2, i2:]).astype(f32)
    return Q, W_int, Scale
