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


def _present(per_loss, loss_weights):
    """``(loss_type, weight)`` pairs of ``loss_weights`` that have cached data."""
    return [(lt, w) for lt, w in loss_weights.items() if lt in per_loss]


class _LinearHooks:
    """Hook bookkeeping shared by the two caches: the block's linears are
    looked up by name (or ``name + ".module"`` for wrapped ones), forward
    hooks are kept in ``handles`` until ``clear_hook``, and ``hooks_enabled``
    gates the gradient-side hooks to the backward passes the caller asks for."""

    def __init__(self, names, num_groups):
        self.names = names
        self.num_groups = num_groups
        self.handles = []
        self.hooks_enabled = False

    @staticmethod
    def _linear(full, name):
        module = full.get(name)
        return module if module is not None else full.get(name + ".module")

    def _on_forward(self, name):
        raise NotImplementedError

    def set_forward_hook(self, full):
        for name in self.names:
            self.handles.append(self._linear(full, name).register_forward_hook(
                self._on_forward(name)))

    @contextlib.contextmanager
    def _gradients_on(self):
        self.hooks_enabled = True
        try:
            yield
        finally:
            self.hooks_enabled = False

    def clear_hook(self):
        while self.handles:
            self.handles.pop().remove()
        self.hooks_enabled = False


class SaliencyCache(_LinearHooks):
    """Per linear and loss type, the per-batch ``[tokens, G]`` saliencies of
    its output gradient (g2ptq_utils.py:586-679): ``saliency_cache[name]`` maps
    a loss type to the list of batches until ``summarize_saliency`` collapses
    it to one list weighted over loss types."""

    def __init__(self, names, num_groups):
        super().__init__(names, num_groups)
        self.outs = {name: 0 for name in names}
        self.saliency_cache = {name: {} for name in names}

    def cache_saliency(self, module, inp, out, name):
        self.outs[name] = out

    def _on_forward(self, name):
        return functools.partial(self.cache_saliency, name=name)

    def grad_hook(self, grad, name, loss_type):
        """Group means of ``grad**2`` over the G channel groups of the output
        (g2ptq_utils.py:605-618), one kernel pass over the gradient."""
        if self.hooks_enabled:
            sal = ops.saliency(grad.reshape(-1, grad.shape[-1]), self.num_groups)
            self.saliency_cache[name].setdefault(loss_type, []).append(sal)

    def backward(self, loss_tensor, loss_type="block", retain_graph=True):
        """The loss's gradient at every output captured since the last clear
        (g2ptq_utils.py:652-669), turned into saliencies."""
        live = [(n, out) for n, out in self.outs.items() if isinstance(out, torch.Tensor)]
        if not live:
            return
        with self._gradients_on():
            grads = torch.autograd.grad(loss_tensor, [out for _, out in live],
                                        retain_graph=retain_graph, allow_unused=True)
            for (name, _), grad in zip(live, grads):
                if grad is not None:
                    self.grad_hook(grad, name=name, loss_type=loss_type)

    def summarize_saliency(self, loss_weights):
        """Batch by batch, the ``loss_weights``-weighted sum over loss types
        (g2ptq_utils.py:620-640); every loss type must hold the same number of
        batches."""
        for name in self.names:
            per_loss = self.saliency_cache[name]
            terms = _present(per_loss, loss_weights)
            counts = {lt: len(per_loss[lt]) for lt, _ in terms}
            if len(set(counts.values())) > 1:
                raise AssertionError(f"saliency batches of {name!r} differ between loss types: "
                                     f"{counts}")
            batches = next(iter(counts.values()), 0)
            self.saliency_cache[name] = [
                _weighted_sum([(per_loss[lt][i], w) for lt, w in terms]) for i in range(batches)]

    def clear_cache(self):
        self.outs = {name: 0 for name in self.names}
        self.saliency_cache = {name: {} for name in self.names}
        _cleanup_memory()


class GradientCache(_LinearHooks):
    """Per linear and loss type, the running mean over backward passes of the
    weight gradient divided by the batch's token count (g2ptq_utils.py:682-763):
    ``gradients_cache[name][loss_type]`` and its count ``index[name][loss_type]``
    until ``summarize_gradients`` collapses the loss types."""

    def __init__(self, names, num_groups):
        super().__init__(names, num_groups)
        self.current_batch_tokens = {}
        self.gradients_cache = {name: {} for name in names}
        self.index = {name: {} for name in names}

    def forward_hook(self, module, inp, out, name):
        x = inp[0]  # [batch, seq, hidden] or, for routed experts, [tokens, hidden]
        self.current_batch_tokens[name] = x.numel() // x.shape[-1]

    def _on_forward(self, name):
        return functools.partial(self.forward_hook, name=name)

    def cache_gradient(self, grad, name, loss_type):
        """``cache <- cache i/(i+1) + grad / (n_tok (i+1))`` (g2ptq_utils.py:693-702),
        in place in one kernel pass."""
        if not self.hooks_enabled:
            return
        i = self.index[name].get(loss_type, 0)
        cache = self.gradients_cache[name].get(loss_type)
        first = cache is None
        if first:
            cache = torch.empty(grad.shape, dtype=torch.float32, device=grad.device)
        # the reference divides a CUDA tensor by a host scalar, which torch
        # evaluates as a multiply by the scalar's fp32 reciprocal
        inv = float(np.float32(1.0) / np.float32(self.current_batch_tokens[name] * (i + 1)))
        ops.running_mean(cache, grad.contiguous(), i / (i + 1), inv, first)
        self.gradients_cache[name][loss_type] = cache
        self.index[name][loss_type] = i + 1

    @contextlib.contextmanager
    def set_backward_hook(self, full, loss_type="block"):
        """Gradient hooks on the linears' weights for the backward passes run
        inside the context."""
        hooks = [self._linear(full, name).weight.register_hook(
                     functools.partial(self.cache_gradient, name=name, loss_type=loss_type))
                 for name in self.names]
        with self._gradients_on():
            try:
                yield
            finally:
                for h in hooks:
                    h.remove()

    def summarize_gradients(self, loss_weights):
        """The ``loss_weights``-weighted sum over loss types, or 0 where
        nothing was cached (g2ptq_utils.py:704-711)."""
        for name in self.names:
            per_loss = self.gradients_cache[name]
            terms = _present(per_loss, loss_weights)
            self.gradients_cache[name] = (_weighted_sum([(per_loss[lt], w) for lt, w in terms])
                                          if terms else 0)

    def clear_cache(self):
        self.gradients_cache = {name: {} for name in self.names}
        self.index = {name: {} for name in self.names}
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

    # F.mse_loss promotes mixed operand dtypes: a bf16 block output against an
    # fp32 target is compared in fp32, the target never rounded to bf16
    dt = torch.promote_types(hidden_states.dtype, hidden_states_fp.dtype)
    mse_loss = block_loss(_lib.LOSS_MSE, hidden_states.to(dt),
                          target=hidden_states_fp.detach().to(dt))
    if compute_gradient:
        zero_onloaded_grads(full)
        with gradients_cache.set_backward_hook(full, loss_type=loss_type):
            mse_loss.backward(retain_graph=retain_graph)
    return mse_loss.detach().float()
