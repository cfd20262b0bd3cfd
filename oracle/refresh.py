"""Oracle for the G2PTQ refresh step (TEST INFRASTRUCTURE, see oracle/__init__.py).

numpy restatement of the saliency / gradient caches and the block-loss heads
of the reference's ``gptq_utils/g2ptq_utils.py``:

* ``saliency``            SaliencyCache.grad_hook           g2ptq_utils.py:605-618
* ``weighted_sum``        summarize_saliency / _gradients   g2ptq_utils.py:620-640, 704-711
* ``running_mean``        GradientCache.cache_gradient      g2ptq_utils.py:693-702
* ``normalize_loss_weights``                                g2ptq_utils.py:578-583
* ``nll_head`` / ``kl_head``  the two losses of compute_kl_grad_hessian  :969-1001
* ``mse_head``            the loss of compute_mse_grad_hessian          :1004-1035

The loss heads return the loss and its gradient with respect to the input
rows, computed in float64 (the reference runs them in the model dtype).
Pinned by tests/golden/refresh.npz (the reference's own caches and loss
functions run on CPU over a seeded two-linear block).
"""

import numpy as np


def saliency(grad, num_groups):
    """``grad.float().pow(2).view(n, G, R/G).mean(-1)`` (g2ptq_utils.py:611-616)."""
    g = np.asarray(grad, dtype=np.float32).reshape(-1, grad.shape[-1])
    n, R = g.shape
    if R % num_groups:
        raise ValueError("hidden size not divisible by the number of groups")
    sq = (g * g).astype(np.float32)
    return sq.reshape(n, num_groups, R // num_groups).mean(-1, dtype=np.float32)


def weighted_sum(items):
    """``sum(w * t for t, w in items)``, fp32, each term rounded
    (g2ptq_utils.py:637-638 and 709-711)."""
    acc = None
    for t, w in items:
        term = (np.float32(w) * np.asarray(t, dtype=np.float32)).astype(np.float32)
        acc = term + np.float32(0.0) if acc is None else (acc + term).astype(np.float32)
    return acc


def running_mean(cache, index, grad, n_tokens):
    """One ``GradientCache.cache_gradient`` step (g2ptq_utils.py:693-702);
    ``cache`` None on the first call.  Returns ``(cache, index + 1)``.  The
    division is a true fp32 division, as torch does it on CPU."""
    keep = np.float32(index / (index + 1))
    index += 1
    term = (np.asarray(grad, dtype=np.float32) / np.float32(n_tokens * index)).astype(np.float32)
    if cache is None:
        return term + np.float32(0.0), index
    return ((cache * keep).astype(np.float32) + term).astype(np.float32), index


def normalize_loss_weights(loss_weights):
    """g2ptq_utils.py:578-583."""
    total = sum(loss_weights.values())
    if total == 0:
        return {k: 0.0 for k in loss_weights}
    return {k: w / total for k, w in loss_weights.items()}


def _log_softmax(x):
    x = np.asarray(x, dtype=np.float64)
    m = x.max(-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(-1, keepdims=True))


def nll_head(logits, labels):
    """``F.cross_entropy(logits, labels, reduction="sum")`` and its gradient
    ``softmax(logits) - onehot(labels)``; label -100 is ignored
    (g2ptq_utils.py:981-985)."""
    x = np.asarray(logits, dtype=np.float64).reshape(-1, logits.shape[-1])
    lab = np.asarray(labels).reshape(-1)
    ls = _log_softmax(x)
    keep = lab != -100
    rows = np.nonzero(keep)[0]
    loss = -ls[rows, lab[rows]].sum()
    grad = np.exp(ls)
    grad[rows, lab[rows]] -= 1.0
    grad[~keep] = 0.0
    return loss, grad


def kl_head(logits, logits_fp):
    """``F.kl_div(F.log_softmax(logits), F.softmax(logits_fp), "none").sum()``
    and its gradient ``softmax(logits) * sum(p) - p`` (g2ptq_utils.py:992-997)."""
    x = np.asarray(logits, dtype=np.float64).reshape(-1, logits.shape[-1])
    t = np.asarray(logits_fp, dtype=np.float64).reshape(-1, logits_fp.shape[-1])
    lq, lp = _log_softmax(x), _log_softmax(t)
    p = np.exp(lp)
    loss = (p * (lp - lq)).sum()
    grad = np.exp(lq) * p.sum(-1, keepdims=True) - p
    return loss, grad


def mse_head(h, target):
    """``F.mse_loss(h, target, "none").mean(-1).sum() / 2`` and its gradient
    ``(h - target) / D`` (g2ptq_utils.py:1020-1033)."""
    x = np.asarray(h, dtype=np.float64).reshape(-1, h.shape[-1])
    t = np.asarray(target, dtype=np.float64).reshape(-1, h.shape[-1])
    d = x - t
    D = x.shape[-1]
    return (d * d).mean(-1).sum() / 2.0, d / D
