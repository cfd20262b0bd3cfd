"""Quantization primitives and group-parameter search (numpy float32).

Follows ``utils/quant_utils.py`` of the reference:
  asym_quant / asym_dequant          quant_utils.py:8-16
  _minmax                            quant_utils.py:47-57
  _params_from_range_sym / _asym     quant_utils.py:60-68
  WeightQuantizer.configure          quant_utils.py:350-375
  WeightQuantizer.find_params        quant_utils.py:377-433 (incl. the
                                     --w_clip / --w_hclip grid, 106-133)
  WeightQuantizer.fake_quantize      quant_utils.py:435-459
``torch.round`` rounds half to even, which is ``np.rint``.
"""

import numpy as np

f32 = np.float32


def qrange(bits):
    """``maxq, minq, bit_range`` as in quant_utils.py:372-374."""
    maxq = 2 ** (bits - 1) - 1
    minq = -(maxq + 1)
    return maxq, minq, maxq - minq


def asym_quant(x, scale, zero, maxq):
    """quant_utils.py:8-12: ``clamp(round(x / scale) + zero, -(maxq+1), maxq)``."""
    x = np.asarray(x, f32)
    q = np.rint(x / scale) + zero
    return np.clip(q, f32(-(maxq + 1)), f32(maxq)).astype(f32)


def asym_dequant(q, scale, zero):
    """quant_utils.py:15-16: ``scale * (q - zero)``."""
    return (scale * (q - zero)).astype(f32)


def minmax(x):
    """quant_utils.py:47-57 with clip_ratio 1: per-row range clamped to include 0."""
    xmin = np.minimum(x.min(axis=-1, keepdims=True), f32(0))
    xmax = np.maximum(x.max(axis=-1, keepdims=True), f32(0))
    return xmin, xmax


def params_sym(xmin, xmax, bit_range):
    """quant_utils.py:60-62."""
    scale = np.maximum(np.abs(xmin), xmax) / f32(bit_range / 2)
    return scale.astype(f32), np.zeros_like(scale, dtype=f32)


def params_asym(xmin, xmax, bit_range, minq, maxq):
    """quant_utils.py:65-68."""
    scale = ((xmax - xmin) / f32(bit_range)).astype(f32)
    zero = np.clip(np.rint(f32(minq) - xmin / scale), f32(minq), f32(maxq))
    return scale, zero.astype(f32)


def _quant_err(fq, x, norm, h_diag=None):
    """quant_utils.py:84-103."""
    if h_diag is None:
        return (np.abs(fq - x) ** f32(norm)).astype(f32).sum(-1, dtype=f32)
    err = (fq - x) ** 2
    shape = err.shape[:-1]
    err = err.reshape(h_diag.shape[0], -1, *h_diag.shape[1:]) * h_diag[:, None]
    return err.sum(-1, dtype=f32).reshape(shape)


def find_params(x, bits, sym, mse=False, h_diag=None, norm=2.4, grid=50,
                maxshrink=0.5, weight_groupsize=-1):
    """WeightQuantizer.find_params, quant_utils.py:377-433.

    ``x`` is ``[rows, cols]``.  Returns ``(scale, zero)`` shaped ``[rows, 1]``
    for per-channel quantizers (weight_groupsize == -1) or
    ``[rows, cols // g]`` for grouped ones, as the reference stores them.
    """
    x = np.asarray(x, f32)
    maxq, minq, bit_range = qrange(bits)
    rows, cols = x.shape
    if weight_groupsize > 0:
        xv = x.reshape(rows, cols // weight_groupsize, weight_groupsize)
    else:
        xv = x.reshape(rows, 1, cols)
    if h_diag is not None:
        h_diag = np.asarray(h_diag, f32).reshape(h_diag.shape[0], *xv.shape[1:])
        if h_diag.min() == h_diag.max():
            h_diag = None
    xmin, xmax = minmax(xv)
    if sym:
        scale, zero = params_sym(xmin, xmax, bit_range)
    else:
        scale, zero = params_asym(xmin, xmax, bit_range, minq, maxq)
    if mse:
        best = np.full(xv.shape[:-1], np.inf, dtype=f32)
        for i in range(int(maxshrink * grid)):
            for j in range(int(maxshrink * grid)):
                xmin1 = f32(1 - i / grid) * xmin
                xmax1 = f32(1 - j / grid) * xmax
                if sym:
                    s1, z1 = params_sym(xmin1, xmax1, bit_range)
                else:
                    s1, z1 = params_asym(xmin1, xmax1, bit_range, minq, maxq)
                fq = asym_dequant(asym_quant(xv, s1, z1, maxq), s1, z1)
                err = _quant_err(fq, xv, norm, h_diag)
                better = err < best
                scale = np.where(better[..., None], s1, scale)
                zero = np.where(better[..., None], z1, zero)
                best = np.where(better, err, best)
    zero = np.rint(zero)
    scale = scale[..., 0].astype(f32)
    zero = zero[..., 0].astype(f32)
    if not (scale.min() > 0):
        raise RuntimeError("WeightQuantizer.find_params: non-positive scale")
    return scale, zero


def fake_quantize(x, scale, zero, maxq, weight_groupsize=-1):
    """WeightQuantizer.fake_quantize, quant_utils.py:435-459 -> ``(fq, q)``."""
    x = np.asarray(x, f32)
    if weight_groupsize > 0:
        rows, cols = x.shape
        xv = x.reshape(rows, cols // weight_groupsize, weight_groupsize)
        s, z = scale[..., None], zero[..., None]
        q = asym_quant(xv, s, z, maxq)
        return asym_dequant(q, s, z).reshape(x.shape), q.reshape(x.shape)
    q = asym_quant(x, scale, zero, maxq)
    return asym_dequant(q, scale, zero), q
