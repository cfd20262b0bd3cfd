"""GuidedQuant quantizer object, a drop-in for gptq_utils/gptq_guided_utils.py of
the reference (``GPTQGuided`` gptq_guided_utils.py:25-219, ``reduce_to_target_rank``
:222-249).  Saliency-weighted block Hessians, un-normalized
(``H[g] += sum_n s[n,g] x_n x_n^T``, gptq_guided_utils.py:78-80), quantized with
GPTQ's compensation over ``num_layers * num_groups`` row blocks.
"""

import contextlib

import torch

from .. import ops, _lib
from . import _engine, collectives
from .gptq_utils import GPTQ, _onload


class GPTQGuided(GPTQ):
    index = _engine.lazy_counter("index")
    # per-linear saliency weights: no two objects share a fold, and H is a
    # plain sum (nothing to renormalize)
    _share_folds = False
    _share_factor = False
    _settle = _engine.StagingMixin._settle

    def __init__(self, layers, saliencies, num_groups: int, offload_hessians: bool = False):
        self.layers = layers
        self.num_layers = len(layers)
        self.offload_hessians = offload_hessians
        weight = layers[0].weight
        self.dev = weight.device
        if self.dev.type != "cuda":
            raise RuntimeError("g2ptq_b200 GPTQGuided requires layers on a CUDA device")
        self.rows, self.columns = weight.shape
        self.num_groups = num_groups
        self.saliencies = [s.float() for s in saliencies]
        H_device = "cpu" if offload_hessians else self.dev
        self._H = torch.zeros((self.num_layers, num_groups, self.columns, self.columns),
                              dtype=torch.float32, device=H_device)
        self.act_square = torch.zeros((self.num_layers, self.columns), device=self.dev)
        self.index = torch.zeros(self.num_layers, dtype=torch.long, device=self.dev)
        self._idx = [0] * self.num_layers
        assert self.rows % self.num_groups == 0, (
            f"Number of rows ({self.rows}) must be divisible by num_groups ({self.num_groups})")
        self._init_stages(groups=num_groups)

    def _maybe_onload_hessian(self):
        if not self.offload_hessians:
            return contextlib.nullcontext()
        return _onload(self, ("_H",))

    @torch.no_grad()
    def add_batch(self, idx, inp, out):
        """gptq_guided_utils.py:60-81."""
        if inp.dim() == 2:
            inp = inp.unsqueeze(0)
        else:
            assert inp.dim() == 3, "Input must be 2D or 3D. Got %dD." % inp.dim()
        bsz = inp.shape[0]
        i0 = self._idx[idx]
        sal = self.saliencies[idx][i0:i0 + bsz].to(self.dev)
        self._idx[idx] += bsz
        _engine.bump(self, "index", idx, bsz)
        x = _engine.as_rows(inp, self.columns)
        sal = sal.reshape(-1, sal.shape[-1]).float().contiguous()
        n_tokens = x.shape[0]
        ops.sq_colsum(self.act_square[idx], x, keep=1.0, scale=1.0 / n_tokens)
        self._append(idx, x, scales=sal)

    def _fold(self, idx, X, sub, scales):
        self._require_device_stats(self._H)
        ops.gram_update_grouped(self._H[idx], X, scales, alpha=1.0, beta=1.0,
                                precision=_engine.PRECISION)

    def fasterquant(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                    static_groups=False, export_compressed_tensors=False, backend="torch",
                    graph=False):
        """gptq_guided_utils.py:83-211."""
        pending = self._fq_launch(blocksize=blocksize, percdamp=percdamp, groupsize=groupsize,
                                  actorder=actorder, static_groups=static_groups,
                                  export_compressed_tensors=export_compressed_tensors)
        self._last_damps = pending.finish()

    def _fq_launch(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                   static_groups=False, export_compressed_tensors=False, backend="torch",
                   graph=False):
        B, R, C, G = self.num_layers, self.rows, self.columns, self.num_groups
        rps = R // G
        nl = B * G
        q0 = self.quantizer[0]
        W = torch.stack([l.weight.data for l in self.layers]).float().contiguous()
        with self._maybe_onload_hessian():
            H = self.H.view(nl, C, C)
            self.H = None
        H_diag = _engine.hessian_diag(H, q0)
        W_sub = W.view(nl, rps, C)
        params = _engine.ParamSet(self.quantizer, B * R, C, groupsize, self.dev)
        dynamic = not (groupsize == -1 or static_groups)
        if not dynamic:
            params.init_static(W.view(B * R, C), H_diag)
        ops.prepare_hessian(H, W_sub)
        perm = None
        if actorder:
            perm, _ = _engine.act_order_perm(torch.mean(self.act_square, dim=0))
            W_sub = ops.permute_cols(W_sub, perm)
            H = ops.permute_sym(H, perm)
        clip, clip_hd = _engine.dynamic_clip(q0, H_diag, perm, B * R, C) if dynamic else (None,
                                                                                          None)
        U, info, damps = _engine.factor_with_retry(H, percdamp)
        colgroup = params.colgroup(perm, static_groups, self.dev)
        codes = torch.empty(nl, rps, C, dtype=torch.int8, device=self.dev)

        def run(Wp):
            ops.compensate(_lib.METHOD_GPTQ, Wp, U, params.scale, params.zero, colgroup,
                           dynamic, groupsize, q0.bits, q0.sym, blocksize, codes,
                           status=params.status, precision=_engine.PRECISION, clip=clip)
            _ = clip_hd  # the diagonal the clip configuration points to stays alive
            Q, cq = Wp, codes
            if actorder:
                Q = ops.permute_cols(Wp, perm, inverse=True)
                cq = ops.permute_cols(codes, perm, inverse=True)
            Q, cq = Q.view(B, R, C), cq.view(B, R, C)
            nan, outs = _engine.write_back(self.layers, Q, cq, params, q0.bits, groupsize, C,
                                           export_compressed_tensors)
            return nan, outs, cq

        return _engine.Pending(self.layers, nl, H, U, info, damps, params, run, W_sub, q0.bits,
                               groupsize, C, R, export_compressed_tensors, dynamic, actorder)

    def free(self):
        self._H = None
        self.Losses = None
        self.act_square = None
        self.saliencies = None
        self.index = None
        self._stages = None


def reduce_to_target_rank(gptqs, gptq2rank):
    """gptq_guided_utils.py:222-249: the un-normalized block-wise Hessians,
    squared-activation sums and call counts summed onto the owner (one count
    all_reduce, one packed reduce per owner rank)."""

    def counts(g):
        g._flush_all()
        return list(g._idx)

    def entries(g, local, glob, owner):
        return [collectives.Entry(owner, g._H[b], symmetric=True)
                for b in range(g.num_layers)] + [collectives.Entry(owner, g.act_square)]

    def commit(g, glob):
        g.index = torch.tensor(glob, dtype=torch.long, device=g.dev)
        g._idx = list(glob)

    collectives.reduce_objects(gptqs, gptq2rank, counts, entries, commit,
                               lambda g: g._maybe_onload_hessian())
