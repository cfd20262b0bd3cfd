"""G2PTQ refresh step: the saliency and gradient caches and the block-loss
heads whose backward fills them (gptq_utils/g2ptq_utils.py:578-766 and
:969-1035 of the reference).

Same classes, methods and call order as the reference's ``SaliencyCache``,
``GradientCache``, ``normalize_loss_weights``, ``compute_kl_grad_hessian`` and
``compute_mse_grad_hessian``; re-exported from ``g2ptq_utils``.  The
arithmetic runs in libg2ptq_b200:

* ``SaliencyCache.grad_hook`` -> ``g2q_saliency`` (one read of the output
  gradient, ``[T, G]`` group means of its square);
* ``GradientCache.cache_gradient`` -> ``g2q_running_mean`` (the running mean
  of the weight gradient, in place in one pass);
* the weighted sums over loss types -> ``g2q_scaled_accumulate``;
* the loss heads (sampled-label cross entropy and KL over the vocabulary, the
  row-mean squared error over the hidden size) -> ``g2q_block_loss_forward`` /
  ``g2q_block_loss_backward``: one pass over the rows forward and one
  backward, in fp32 whatever the logits' dtype, where the reference's
  ``log_softmax`` / ``softmax`` / ``kl_div`` chain materialises several
  full-size temporaries.

The backward through the decoder block between the loss and the linears is
the model's own autograd, as in the reference.  The label and noise draws use
the reference's torch calls in the reference's order, so a seeded generator
gives the same labels and noise.
"""

import gc
import contextlib
import functools
import math

import numpy as np
import torch

from .. import ops, _lib


def normalize_loss_weights(loss_weights):
    """g2ptq_utils.py:578-583: scale a {loss_type: weight} dict to sum 1."""
    total = sum(loss_weights.values())
    if total == 0:
        return {k: 0.0 for k in loss_weights}
    return {k: w / total for k, w in loss_weights.items()}


def _cleanup_memory():
    gc.collect()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.empty_cache()


def zero_onloaded_grads(full=None):
    """Stand-in for ``offload_utils.zero_onloaded_grads`` (utils/offload_utils.py:458-464):
    clears ``.grad`` of the parameters of the modules in ``full``.  The caches
    read the per-backward gradients their hooks receive, so this only frees
    memory, as in the reference."""
    if not full:
        return
    for module in full.values():
        if module is None:
            continue
        for p in module.parameters():
            p.grad = None


def _weighted_sum(tensors_and_weights):
    """``sum(w * t for t, w in ...)`` with the reference's per-term rounding."""
    acc = None
    for i, (t, w) in enumerate(tensors_and_weights):
        t = t.float().contiguous()
        if acc is None:
            acc = torch.empty_like(t)
        ops.scaled_accumulate(acc, t, w, first=(i == 0))
    return acc


class SaliencyCache:
    """Output-gradient saliencies per linear (g2ptq_utils.py:586-679)."""

    def __init__(self, names, num_groups):
        self.num_groups = num_groups
        self.saliency_cache = {}
        self.outs = {}
        self.names = names
        for name in self.names:
            self.saliency_cache[name] = {}   # loss -> list of per-batch [tokens, G] tensors
            self.outs[name] = 0
        self.handles = []
        self.hooks_enabled = False

    def cache_saliency(self, module, inp, out, name):
        self.outs[name] = out

    def grad_hook(self, grad, name, loss_type):
        """g2ptq_utils.py:605-618: ``[tokens, G]`` means of ``grad**2`` over
        each of the G channel groups."""
        if not self.hooks_enabled:
            return
        grad = grad.reshape(-1, grad.shape[-1])
        sal = ops.saliency(grad, self.num_groups)
        self.saliency_cache[name].setdefault(loss_type, []).append(sal)

    def summarize_saliency(self, loss_weights):
        """g2ptq_utils.py:620-640: per batch, the weighted sum over loss types."""
        for name in self.names:
            per_loss = self.saliency_cache[name]
            present = [(l, w) for l, w in loss_weights.items() if l in per_loss]
            if not present:
                self.saliency_cache[name] = []
                continue
            lengths = [len(per_loss[l]) for l, _ in present]
            assert len(set(lengths)) == 1, (
                f"Saliency for '{name}' has mismatched per-loss batch counts: "
                f"{ {l: len(per_loss[l]) for l, _ in present} }"
            )
            self.saliency_cache[name] = [
                _weighted_sum([(per_loss[l][i], w) for l, w in present])
                for i in range(lengths[0])
            ]

    def set_forward_hook(self, full):
        for name in self.names:
            module = full.get(name, full.get(name + ".module", None))
            self.handles.append(
                module.register_forward_hook(functools.partial(self.cache_saliency, name=name)))

    def backward(self, loss_tensor, loss_type="block", retain_graph=True):
        """g2ptq_utils.py:652-669: gradients of the loss at every cached output."""
        names = [name for name in self.names if isinstance(self.outs[name], torch.Tensor)]
        if not names:
            return
        self.hooks_enabled = True
        try:
            grads = torch.autograd.grad(loss_tensor, [self.outs[name] for name in names],
                                        retain_graph=retain_graph, allow_unused=True)
            for name, grad in zip(names, grads):
                if grad is not None:
                    self.grad_hook(grad, name=name, loss_type=loss_type)
        finally:
            self.hooks_enabled = False

    def clear_hook(self):
        for h in self.handles:
            h.remove()
        self.handles = []
        self.hooks_enabled = False

    def clear_cache(self):
        for name in self.names:
            self.saliency_cache[name] = {}
            self.outs[name] = 0
        _cleanup_memory()


class GradientCache:
    """Running-mean weight gradients per linear (g2ptq_utils.py:682-763)."""

    def __init__(self, names, num_groups):
        self.num_groups = num_groups
        self.gradients_cache = {}
        self.index = {}
        self.current_batch_tokens = {}
        self.names = names
        for name in self.names:
            self.gradients_cache[name] = {}   # loss -> running-mean gradient tensor
            self.index[name] = {}             # loss -> accumulation count
        self.handles = []
        self.hooks_enabled = False

    def forward_hook(self, module, inp, out, name):
        x = inp[0]
        self.current_batch_tokens[name] = x.numel() // x.shape[-1]

    def cache_gradient(self, grad, name, loss_type):
        """g2ptq_utils.py:693-702: ``cache <- cache i/(i+1) + grad / (n_tok (i+1))``
        in one pass, in place."""
        if not self.hooks_enabled:
            return
        n_tokens = self.current_batch_tokens[name]
        index = self.index[name].get(loss_type, 0)
        cache = self.gradients_cache[name].get(loss_type, 0)
        keep = index / (index + 1)
        index += 1
        # torch divides a CUDA tensor by a host scalar as a multiply by the
        # scalar's fp32 reciprocal
        inv = float(np.float32(1.0) / np.float32(n_tokens * index))
        grad = grad.contiguous()
        first = not torch.is_tensor(cache)
        if first:
            cache = torch.empty(grad.shape, dtype=torch.float32, device=grad.device)
        ops.running_mean(cache, grad, keep, inv, first)
        self.gradients_cache[name][loss_type] = cache
        self.index[name][loss_type] = index

    def summarize_gradients(self, loss_weights):
        """g2ptq_utils.py:704-711: the weighted sum over loss types (0 if none)."""
        for name in self.names:
            per_loss = self.gradients_cache[name]
            present = [(l, w) for l, w in loss_weights.items() if l in per_loss]
            self.gradients_cache[name] = (_weighted_sum([(per_loss[l], w) for l, w in present])
                                          if present else 0)

    def set_forward_hook(self, full):
        for name in self.names:
            module = full.get(name, full.get(name + ".module", None))
            self.handles.append(
                module.register_forward_hook(functools.partial(self.forward_hook, name=name)))

    @contextlib.contextmanager
    def set_backward_hook(self, full, loss_type="block"):
        self.hooks_enabled = True
        handles = []
        for name in self.names:
            module = full.get(name, full.get(name + ".module", None))
            handles.append(module.weight.register_hook(
                functools.partial(self.cache_gradient, name=name, loss_type=loss_type)))
        try:
            yield
        finally:
            for h in handles:
                h.remove()
            self.hooks_enabled = False

    def clear_hook(self):
        for h in self.handles:
            h.remove()
        self.handles = []
        self.hooks_enabled = False

    def clear_cache(self):
        for name in self.names:
            self.gradients_cache[name] = {}
            self.index[name] = {}
        _cleanup_memory()


class _BlockLoss(torch.autograd.Function):
    """A block-loss head (``_lib.LOSS_*``) as one autograd node: the forward
    keeps the per-row log-sum-exp, the backward writes the gradient with
    respect to ``x`` in one pass.  The target (and the labels) take no
    gradient."""

    @staticmethod
    def forward(ctx, x, target, labels, kind):
        if target is not None and target.requires_grad:
            raise NotImplementedError("g2ptq_b200 block losses take no gradient for the target")
        loss, stats, x2, t2, lab = ops.block_loss_forward(kind, x, target, labels)
        ctx.kind = kind
        ctx.x_shape = x.shape
        ctx.save_for_backward(stats, x2, t2, lab)
        return loss

    @staticmethod
    def backward(ctx, grad_out):
        stats, x2, t2, lab = ctx.saved_tensors
        g = ops.block_loss_backward(ctx.kind, stats, x2, t2, lab, grad_scale=grad_out)
        return g.view(ctx.x_shape), None, None, None


def block_loss(kind, x, target=None, labels=None):
    """Differentiable block loss: ``_lib.LOSS_KL`` (sum over rows of
    KL(softmax(target) || softmax(x))), ``_lib.LOSS_NLL`` (summed cross
    entropy against ``labels``, -100 ignored) or ``_lib.LOSS_MSE`` (sum over
    rows of mean((x - target)^2) / 2).  fp32 scalar."""
    return _BlockLoss.apply(x, target, labels, kind)


def compute_kl_grad_hessian(logits, logits_fp, saliency_cache, gradients_cache, full, args,
                            loss_type="block", retain_graph=False, compute_gradient=True):
    """g2ptq_utils.py:969-1001: saliencies from the cross entropy against labels
    sampled from ``softmax(logits_fp)``, weight gradients from the KL to it.
    Returns the detached KL (fp32 scalar)."""
    if args.kl_topk > 0:
        logits_fp, indices = logits_fp.topk(args.kl_topk, dim=-1, sorted=False)
        logits = logits.gather(-1, indices)

    labels = torch.distributions.Categorical(logits=logits_fp).sample()
    nll_loss = block_loss(_lib.LOSS_NLL, logits, labels=labels)
    zero_onloaded_grads(full)
    saliency_cache.backward(nll_loss, loss_type=loss_type, retain_graph=True)

    kl_loss = block_loss(_lib.LOSS_KL, logits, target=logits_fp.detach())
    if compute_gradient:
        zero_onloaded_grads(full)
        with gradients_cache.set_backward_hook(full, loss_type=loss_type):
            kl_loss.backward(retain_graph=retain_graph)
    return kl_loss.detach().float()


def compute_mse_grad_hessian(hidden_states, hidden_states_fp, saliency_cache, gradients_cache,
                             full, args, loss_type="block", retain_graph=False,
                             compute_gradient=True):
    """g2ptq_utils.py:1004-1035: saliencies from the squared error to a noisy
    copy of ``hidden_states``, weight gradients from the squared error to
    ``hidden_states_fp``.  Returns the detached loss (fp32 scalar)."""
    hidden_states_noise = torch.distributions.Normal(
        loc=torch.zeros_like(hidden_states),
        scale=math.sqrt(hidden_states.size(-1))
    ).sample()
    mse_loss = block_loss(_lib.LOSS_MSE, hidden_states,
                          target=(hidden_states + hidden_states_noise).detach())
    zero_onloaded_grads(full)
    saliency_cache.backward(mse_loss, loss_type=loss_type, retain_graph=True)

    mse_loss = block_loss(_lib.LOSS_MSE, hidden_states,
                          target=hidden_states_fp.detach().to(hidden_states.dtype))
    if compute_gradient:
        zero_onloaded_grads(full)
        with gradients_cache.set_backward_hook(full, loss_type=loss_type):
            mse_loss.backward(retain_graph=retain_graph)
    return mse_loss.detach().float()
