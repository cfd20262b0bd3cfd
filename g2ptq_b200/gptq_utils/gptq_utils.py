"""GPTQ quantizer object, a drop-in for gptq_utils/gptq_utils.py of the reference.

Same constructor, ``add_batch`` / ``fasterquant`` / ``free`` signatures,
attributes (``H``, ``nsamples``, ``quantizer``, ``layers`` ...) and error
behaviour (ValueError on an exhausted damp retry or NaN weights) as
``GPTQ`` (gptq_utils.py:93-359), plus the kernel-level boundary ``run_eager``
(gptq_utils.py:67-90) and ``reduce_to_target_rank`` (gptq_utils.py:362-391).
All arithmetic runs in libg2ptq_b200's sm_100a kernels.
"""

import contextlib

import torch

from .. import ops, _lib
from . import _engine, collectives
from .common_utils import make_group_quantizers, merge_group_quantizers  # noqa: F401
from .graph_utils import validate_tensors


def run_eager(weight, hinv, scale, zero, maxq, backend="torch", int_weight=None, error=None):
    """One prepared compensation block, reference layout ``[B, blk, R]``
    (gptq_utils.py:67-90).  ``backend`` is accepted and ignored: there is a
    single CUDA implementation.  Returns ``(weight, int_weight, error)``."""
    validate_tensors("GPTQ", weight, hinv, scale, zero, int_weight, error)
    B, blk, R = weight.shape
    W = weight.transpose(1, 2).contiguous()
    S = scale.transpose(1, 2).contiguous().reshape(B * R, blk)
    Z = zero.transpose(1, 2).contiguous().reshape(B * R, blk)
    colmap = torch.arange(blk, dtype=torch.int32, device=weight.device)
    codes = torch.empty(B, R, blk, dtype=torch.int8, device=weight.device)
    err = torch.empty(B, blk, R, dtype=torch.float32, device=weight.device)
    ops.compensate_block(_lib.METHOD_GPTQ, W, hinv.contiguous(), S, Z, colmap, maxq,
                         codes=codes, err=err)
    weight.copy_(W.transpose(1, 2))
    int_weight.copy_(codes.transpose(1, 2))
    error.copy_(err)
    return weight, int_weight, error


class GPTQ(_engine.StagingMixin):
    nsamples = _engine.lazy_counter("nsamples")
    _share_folds = True  # linears fed the same tensor share their Gram folds
    _share_factor = True  # ... and, in fasterquant_all, their Cholesky factor
    _h_exposed = False  # H was handed out through the public property

    def __init__(self, layers, offload_hessians: bool = False):
        self.layers = layers
        self.num_layers = len(layers)
        self.offload_hessians = offload_hessians
        weight = layers[0].weight
        self.dev = weight.device
        if self.dev.type != "cuda":
            raise RuntimeError("g2ptq_b200 GPTQ requires layers on a CUDA device")
        self.rows, self.columns = weight.shape
        H_device = "cpu" if offload_hessians else self.dev
        self._H = torch.zeros((self.num_layers, self.columns, self.columns),
                              dtype=torch.float32, device=H_device)
        self.nsamples = torch.zeros(self.num_layers, dtype=torch.long, device=self.dev)
        self._n = [0] * self.num_layers          # host copy of nsamples
        self._n_folded = [0] * self.num_layers   # samples already folded into H
        self._init_stages()

    # -- Hessian ----------------------------------------------------------
    @property
    def H(self):
        self._flush_all()
        self._h_exposed = True  # the caller may change it: no shared factor
        return self._H

    def _hessian(self):
        self._flush_all()
        return self._H

    @H.setter
    def H(self, value):
        if value is not self._H:
            self._leave_groups()
        self._H = value

    def _stats_on_device(self):
        return self._H is not None and self._H.device.type == "cuda"

    def _copy_folded(self, idx, src, src_idx):
        """Take the folded Hessian and its sample count from ``src``'s layer
        ``src_idx`` (a fold-group member with the same calls)."""
        self._H[idx].copy_(src._H[src_idx])
        self._n_folded[idx] = src._n_folded[src_idx]

    def _settle(self, idx):
        n, nf = self._n[idx], self._n_folded[idx]
        if n != nf and n > 0:
            self._require_device_stats(self._H)
            self._H[idx] *= nf / n
            self._n_folded[idx] = n

    def _maybe_onload_hessian(self, idx=None):
        """Onload the Hessian for the duration of the context (gptq_utils.py:109-113)."""
        if not self.offload_hessians:
            return contextlib.nullcontext()
        return _onload(self, ("_H",))

    def add_batch(self, idx, inp, out):
        """gptq_utils.py:115-126 (the product is folded in lazily, see _engine)."""
        if len(inp.shape) == 2:
            inp = inp.unsqueeze(0)
        tmp = inp.shape[0]
        self._n[idx] += tmp
        _engine.bump(self, "nsamples", idx, tmp)
        x = _engine.as_rows(inp, self.columns)
        if not self._shared_call(idx, x, tmp):
            self._append(idx, x)

    def _fold(self, idx, X, sub, scales, n_new=None):
        n_old = self._n_folded[idx]
        n_new = self._n[idx] if n_new is None else n_new
        self._require_device_stats(self._H)
        ops.gram_update(self._H[idx], X, alpha=n_old / n_new, beta=2.0 / n_new,
                        precision=_engine.PRECISION)
        self._n_folded[idx] = n_new

    # -- quantization -------------------------------------------------------
    def fasterquant(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                    static_groups=False, export_compressed_tensors=False, backend="torch",
                    graph=False):
        """gptq_utils.py:234-353.  ``backend`` and ``graph`` are accepted and ignored."""
        pending = self._fq_launch(blocksize=blocksize, percdamp=percdamp, groupsize=groupsize,
                                  actorder=actorder, static_groups=static_groups,
                                  export_compressed_tensors=export_compressed_tensors)
        self._last_damps = pending.finish()

    def _fq_launch(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                   static_groups=False, export_compressed_tensors=False, backend="torch",
                   graph=False, factor_out=None, factor_in=None):
        """Enqueue the whole of fasterquant on the current stream (no host sync).

        ``factor_out`` / ``factor_in``: a slot through which objects with
        bit-identical Hessians (``_engine.factor_roles``) share one damped
        inverse-Cholesky factor; the owner fills it, the others wait for its
        event and take U, the status word and the damps from it."""
        B, R, C = self.num_layers, self.rows, self.columns
        q0 = self.quantizer[0]
        with self._maybe_onload_hessian():
            H = self._hessian()
            self.H = None
        H_diag = _engine.hessian_diag(H, q0)
        W = torch.stack([l.weight.data for l in self.layers]).float().contiguous()
        params = _engine.ParamSet(self.quantizer, B * R, C, groupsize, self.dev)
        dynamic = not (groupsize == -1 or static_groups)
        if not dynamic:
            params.init_static(W.view(B * R, C), H_diag)
        ops.prepare_hessian(H, W)
        perm = None
        if actorder:
            if factor_in is not None:
                # the owner's Hessian is bit-identical: so is its permutation,
                # and only the owner factors the permuted Hessian
                stream = torch.cuda.current_stream(self.dev)
                stream.wait_event(factor_in["perm_event"])
                perm = factor_in["perm"]
                perm.record_stream(stream)
                W = ops.permute_cols(W, perm)
            else:
                perm, _ = _engine.act_order_perm(ops.mean_diag(H))
                if factor_out is not None:
                    ev = torch.cuda.Event()
                    ev.record(torch.cuda.current_stream(self.dev))
                    factor_out.update(perm=perm, perm_event=ev)
                W = ops.permute_cols(W, perm)
                H = ops.permute_sym(H, perm)
        clip, clip_hd = _engine.dynamic_clip(q0, H_diag, perm, B * R, C) if dynamic else (None,
                                                                                          None)
        if factor_in is not None:
            stream = torch.cuda.current_stream(self.dev)
            stream.wait_event(factor_in["event"])
            U, info, damps = factor_in["U"], factor_in["info"], factor_in["damps"]
            U.record_stream(stream)
            info.record_stream(stream)
        else:
            U, info, damps = _engine.factor_with_retry(H, percdamp)
            if factor_out is not None:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.dev))
                factor_out.update(U=U, info=info, damps=damps, event=ev)
        colgroup = params.colgroup(perm, static_groups, self.dev)
        codes = torch.empty(B, R, C, dtype=torch.int8, device=self.dev)

        def run(Wp):
            ops.compensate(_lib.METHOD_GPTQ, Wp, U, params.scale, params.zero, colgroup, dynamic,
                           groupsize, q0.bits, q0.sym, blocksize, codes, status=params.status,
                           precision=_engine.PRECISION, clip=clip)
            _ = clip_hd  # the diagonal the clip configuration points to stays alive
            Q, cq = Wp, codes
            if actorder:
                Q = ops.permute_cols(Wp, perm, inverse=True)
                cq = ops.permute_cols(codes, perm, inverse=True)
            nan, outs = _engine.write_back(self.layers, Q, cq, params, q0.bits, groupsize, C,
                                           export_compressed_tensors)
            return nan, outs, cq

        return _engine.Pending(self.layers, B, H, U, info, damps, params, run, W, q0.bits,
                               groupsize, C, R, export_compressed_tensors, dynamic, actorder,
                               borrowed_factor=factor_in is not None,
                               lent_factor=factor_out is not None)

    def free(self):
        self._leave_groups()
        self._H = None
        self.Losses = None
        self.nsamples = None
        self._stages = None


@contextlib.contextmanager
def _onload(owner, names):
    staged = {}
    for n in names:
        host = getattr(owner, n, None)
        if host is not None:
            staged[n] = host
            setattr(owner, n, host.to(owner.dev, non_blocking=host.is_pinned()))
    try:
        yield
    finally:
        for n in names:
            v = getattr(owner, n, None)
            if v is None or v.device.type == "cpu":
                continue
            if hasattr(owner, "_flush_all") and n == "_H":
                owner._flush_all()
                v = getattr(owner, n)
            setattr(owner, n, v.to("cpu"))


def fasterquant_all(gptqs, **kwargs):
    """Run ``fasterquant(**kwargs)`` of several objects with their device work
    overlapped on a small stream pool (same results as calling them in turn)."""
    _engine.fasterquant_all(gptqs, **kwargs)


def reduce_to_target_rank(gptqs, gptq2rank):
    """gptq_utils.py:362-391: sum the rank-local Hessians, each rescaled by its
    rank's share of the samples, onto the object's owner rank; the owner's
    ``nsamples`` becomes the global count.  One count all_reduce for all
    objects and one packed-upper-triangle reduce per owner rank
    (``collectives.reduce_objects``)."""

    def counts(g):
        g._hessian()        # pending folds first
        g._leave_groups()   # the reduced Hessian no longer follows a fold group
        return list(g._n)

    def entries(g, local, glob, owner):
        out = []
        for b in range(g.num_layers):
            if glob[b] == 0:
                g._H[b].zero_()
            else:
                out.append(collectives.Entry(owner, g._H[b], symmetric=True,
                                             weight=local[b] / glob[b]))
        return out

    def commit(g, glob):
        g.nsamples = torch.tensor(glob, dtype=torch.long, device=g.dev)
        g._n = list(glob)
        g._n_folded = list(glob)

    collectives.reduce_objects(gptqs, gptq2rank, counts, entries, commit,
                               lambda g: g._maybe_onload_hessian())
