"""Hessian accumulation restatements (numpy float32).

  GPTQ.add_batch        gptq_utils.py:115-126
  G2PTQ.add_batch       g2ptq_utils.py:182-201
  GPTAQ.add_batch       gptaq_utils.py:130-148
  GPTQGuided.add_batch  gptq_guided_utils.py:60-81
Each function takes the running state and returns the new one; it does not
mutate its inputs.
"""

import math

import numpy as np

f32 = np.float32


def gptq_add_batch(H, nsamples, inp):
    """gptq_utils.py:115-126.

    ``inp`` is ``[b, S, C]`` or ``[t, C]``; a 2-D input counts as one sample
    (``unsqueeze(0)``, line 116-118).  Returns ``(H, nsamples)``.
    """
    inp = np.asarray(inp)
    if inp.ndim == 2:
        inp = inp[None]
    tmp = inp.shape[0]
    x = inp.reshape(-1, inp.shape[-1]).astype(f32).T
    H = (H * f32(nsamples / (nsamples + tmp))).astype(f32)
    nsamples = nsamples + tmp
    x = f32(math.sqrt(2 / nsamples)) * x
    H = (H + x @ x.T).astype(f32)
    return H, nsamples


def gptaq_add_batch(H, dXXT, nsamples, inp, fp_inp):
    """gptaq_utils.py:130-148: ``H`` as GPTQ plus ``dXXT += (sqrt(2/n) X_fp - x) x^T``."""
    inp = np.asarray(inp)
    fp = np.asarray(fp_inp).reshape(-1, np.asarray(fp_inp).shape[-1]).astype(f32).T
    if inp.ndim == 2:
        inp = inp[None]
    tmp = inp.shape[0]
    x = inp.reshape(-1, inp.shape[-1]).astype(f32).T
    ratio = f32(nsamples / (nsamples + tmp))
    H = (H * ratio).astype(f32)
    dXXT = (dXXT * ratio).astype(f32)
    nsamples = nsamples + tmp
    s = f32(math.sqrt(2 / nsamples))
    x = s * x
    H = (H + x @ x.T).astype(f32)
    dX = fp * s - x
    dXXT = (dXXT + dX @ x.T).astype(f32)
    return H, dXXT, nsamples


def g2ptq_add_batch(H, act_square, index, total_tokens, inp, sal):
    """g2ptq_utils.py:182-201.

    ``H`` is ``[G, C, C]``, ``sal`` is ``[t, G]`` per-token saliency.
    ``H[g] <- H[g] * k/(k+1) + (1/(t (k+1))) * sum_n s[n,g] x_n x_n^T`` and a
    running mean of ``x^2`` in ``act_square``.
    """
    x = np.asarray(inp).reshape(-1, np.asarray(inp).shape[-1]).astype(f32)
    s = np.asarray(sal, f32)
    n_tok = x.shape[0]
    H = (H * f32(index / (index + 1))).astype(f32)
    index = index + 1
    act_square = (act_square * f32(total_tokens / (total_tokens + n_tok))).astype(f32)
    total_tokens = total_tokens + n_tok
    block = np.einsum("ni,nj,ng->gij", x, x, s, optimize=True).astype(f32)
    H = (H + block * f32(1 / (n_tok * index))).astype(f32)
    act_square = (act_square + (x * x).sum(0, dtype=f32) * f32(1 / total_tokens)).astype(f32)
    return H, act_square, index, total_tokens


def guided_add_batch(H, act_square, index, inp, sal):
    """gptq_guided_utils.py:60-81: un-normalized saliency-weighted sum.

    ``inp`` is ``[b, S, C]`` or ``[t, C]``; ``sal`` is the caller's full
    saliency array ``[N, S, G]`` sliced at ``index``.
    """
    inp = np.asarray(inp)
    if inp.ndim == 2:
        inp = inp[None]
    bsz = inp.shape[0]
    sb = np.asarray(sal, f32)[index:index + bsz]
    index = index + bsz
    x = inp.reshape(-1, inp.shape[-1]).astype(f32)
    sb = sb.reshape(-1, sb.shape[-1])
    n_tok = x.shape[0]
    block = np.einsum("ni,nj,ng->gij", x, x, sb, optimize=True).astype(f32)
    H = (H + block).astype(f32)
    act_square = (act_square + (x * x).sum(0, dtype=f32) * f32(1 / n_tok)).astype(f32)
    return H, act_square, index
