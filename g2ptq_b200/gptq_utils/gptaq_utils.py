"""GPTAQ quantizer object, a drop-in for gptq_utils/gptaq_utils.py of the reference
(``GPTAQ`` gptaq_utils.py:103-399, ``run_eager`` :74-100, ``reduce_to_target_rank``
:402-439).

Statistics: ``H`` as GPTQ and ``dXX^T <- dXX^T n/(n+b) + (2/(n+b)) (X_fp - X)^T X``
(gptaq_utils.py:139-146), staged as ``X`` plus the fp32 difference ``X_fp - X``.
Compensation adds ``+ w_c * P[c, c+1:]`` with
``P = alpha * triu(dXX^T U^T, 1) U`` (gptaq_utils.py:349-352).
"""

import contextlib

import torch

from .. import ops, _lib
from . import _engine, collectives
from .graph_utils import validate_tensors
from .gptq_utils import _onload


def run_eager(weight, hinv, p, scale, zero, maxq, backend="torch", column_weight=None,
              int_weight=None, error=None):
    """One GPTAQ compensation block, reference layout ``[B, blk, R]``
    (gptaq_utils.py:74-100)."""
    validate_tensors("GPTAQ", weight, hinv, p, scale, zero, int_weight, error)
    B, blk, R = weight.shape
    W = weight.transpose(1, 2).contiguous()
    S = scale.transpose(1, 2).contiguous().reshape(B * R, blk)
    Z = zero.transpose(1, 2).contiguous().reshape(B * R, blk)
    colmap = torch.arange(blk, dtype=torch.int32, device=weight.device)
    codes = torch.empty(B, R, blk, dtype=torch.int8, device=weight.device)
    err = torch.empty(B, blk, R, dtype=torch.float32, device=weight.device)
    ops.compensate_block(_lib.METHOD_GPTAQ, W, hinv.contiguous(), S, Z, colmap, maxq,
                         codes=codes, err=err, p=p.contiguous())
    weight.copy_(W.transpose(1, 2))
    int_weight.copy_(codes.transpose(1, 2))
    error.copy_(err)
    return weight, int_weight, error


class GPTAQ(_engine.StagingMixin):
    nsamples = _engine.lazy_counter("nsamples")

    def __init__(self, layers, offload_hessians: bool = False):
        self.layers = layers
        self.num_layers = len(layers)
        self.offload_hessians = offload_hessians
        weight = layers[0].weight
        self.dev = weight.device
        if self.dev.type != "cuda":
            raise RuntimeError("g2ptq_b200 GPTAQ requires layers on a CUDA device")
        self.rows, self.columns = weight.shape
        H_device = "cpu" if offload_hessians else self.dev
        self._H = torch.zeros((self.num_layers, self.columns, self.columns),
                              dtype=torch.float32, device=H_device)
        self._dXXT = torch.zeros_like(self._H)
        self.nsamples = torch.zeros(self.num_layers, dtype=torch.long, device=self.dev)
        self.fp_inp = [[] for _ in range(self.num_layers)]
        self._n = [0] * self.num_layers
        self._n_folded = [0] * self.num_layers
        self._init_stages()

    @property
    def H(self):
        self._flush_all()
        return self._H

    @H.setter
    def H(self, value):
        self._H = value

    @property
    def dXXT(self):
        self._flush_all()
        return self._dXXT

    @dXXT.setter
    def dXXT(self, value):
        self._dXXT = value

    def _maybe_onload_hessian(self):
        """gptaq_utils.py:123-128."""
        if not self.offload_hessians:
            return contextlib.nullcontext()
        return _onload(self, ("_H", "_dXXT"))

    def add_batch(self, idx, inp, out):
        """gptaq_utils.py:130-148."""
        fp = self.fp_inp[idx][0].to(inp, non_blocking=True)
        if len(inp.shape) == 2:
            inp = inp.unsqueeze(0)
        tmp = inp.shape[0]
        x = _engine.as_rows(inp, self.columns)
        fp = _engine.as_rows(fp, self.columns)
        self._n[idx] += tmp
        _engine.bump(self, "nsamples", idx, tmp)
        self._append(idx, x, sub=fp)
        del self.fp_inp[idx][0]

    def _settle(self, idx):
        """An add_batch call without tokens still rescales by n / (n + b)."""
        n, nf = self._n[idx], self._n_folded[idx]
        if n != nf and n > 0:
            self._require_device_stats(self._H)
            self._H[idx] *= nf / n
            self._dXXT[idx] *= nf / n
            self._n_folded[idx] = n

    def _fold(self, idx, X, diff, scales):
        n_old, n_new = self._n_folded[idx], self._n[idx]
        self._require_device_stats(self._H)
        a, b = n_old / n_new, 2.0 / n_new
        ops.gram_update(self._H[idx], X, alpha=a, beta=b, precision=_engine.PRECISION)
        ops.gram_update(self._dXXT[idx], diff, X, alpha=a, beta=b, symmetric=False,
                        precision=_engine.PRECISION)
        self._n_folded[idx] = n_new

    def fasterquant(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                    static_groups=False, alpha=0.25, export_compressed_tensors=False,
                    backend="torch", graph=False):
        """gptaq_utils.py:263-391 (``backend`` / ``graph`` accepted and ignored)."""
        pending = self._fq_launch(blocksize=blocksize, percdamp=percdamp, groupsize=groupsize,
                                  actorder=actorder, static_groups=static_groups, alpha=alpha,
                                  export_compressed_tensors=export_compressed_tensors)
        self._last_damps = pending.finish()

    def _fq_launch(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                   static_groups=False, alpha=0.25, export_compressed_tensors=False,
                   backend="torch", graph=False):
        B, R, C = self.num_layers, self.rows, self.columns
        q0 = self.quantizer[0]
        with self._maybe_onload_hessian():
            H = self.H
            dX = self.dXXT
            self.H = None
        H_diag = _engine.hessian_diag(H, q0)
        W = torch.stack([l.weight.data for l in self.layers]).float().contiguous()
        params = _engine.ParamSet(self.quantizer, B * R, C, groupsize, self.dev)
        dynamic = not (groupsize == -1 or static_groups)
        if not dynamic:
            params.init_static(W.view(B * R, C), H_diag)
        ops.prepare_hessian(H, W, extra=dX)
        perm = None
        if actorder:
            perm, _ = _engine.act_order_perm(ops.mean_diag(H))
            W = ops.permute_cols(W, perm)
            H = ops.permute_sym(H, perm)
            dX = ops.permute_sym(dX, perm)
        clip, clip_hd = _engine.dynamic_clip(q0, H_diag, perm, B * R, C) if dynamic else (None,
                                                                                          None)
        U, info, damps = _engine.factor_with_retry(H, percdamp)
        colgroup = params.colgroup(perm, static_groups, self.dev)
        codes = torch.empty(B, R, C, dtype=torch.int8, device=self.dev)

        def run(Wp):
            T = ops.gemm(torch.empty_like(dX), dX, U, transB=True, mask=_lib.MASK_STRICT_UPPER,
                         precision=_engine.PRECISION)
            P = ops.gemm(torch.empty_like(dX), T, U, beta=float(alpha), precision=_engine.PRECISION)
            ops.compensate(_lib.METHOD_GPTAQ, Wp, U, params.scale, params.zero, colgroup,
                           dynamic, groupsize, q0.bits, q0.sym, blocksize, codes, p=P,
                           status=params.status, precision=_engine.PRECISION, clip=clip)
            _ = clip_hd  # the diagonal the clip configuration points to stays alive
            Q, cq = Wp, codes
            if actorder:
                Q = ops.permute_cols(Wp, perm, inverse=True)
                cq = ops.permute_cols(codes, perm, inverse=True)
            nan, outs = _engine.write_back(self.layers, Q, cq, params, q0.bits, groupsize, C,
                                           export_compressed_tensors)
            return nan, outs, cq

        return _engine.Pending(self.layers, B, H, U, info, damps, params, run, W, q0.bits,
                               groupsize, C, R, export_compressed_tensors, dynamic, actorder)

    def free(self):
        self._H = None
        self.Losses = None
        self._dXXT = None
        self.nsamples = None
        self.fp_inp = None
        self._stages = None


def reduce_to_target_rank(gptqs, gptq2rank):
    """gptaq_utils.py:402-439: H and dXX^T rescaled by each rank's share of the
    samples and summed onto the owner (one count all_reduce, one packed
    reduce per owner rank; dXX^T is not symmetric and travels whole)."""

    def counts(g):
        g._flush_all()
        return list(g._n)

    def entries(g, local, glob, owner):
        out = []
        for b in range(g.num_layers):
            if glob[b] == 0:
                g._H[b].zero_()
                g._dXXT[b].zero_()
                continue
            w = local[b] / glob[b]
            out += [collectives.Entry(owner, g._H[b], symmetric=True, weight=w),
                    collectives.Entry(owner, g._dXXT[b], weight=w)]
        return out

    def commit(g, glob):
        g.nsamples = torch.tensor(glob, dtype=torch.long, device=g.dev)
        g._n, g._n_folded = list(glob), list(glob)

    collectives.reduce_objects(gptqs, gptq2rank, counts, entries, commit,
                               lambda g: g._maybe_onload_hessian())
