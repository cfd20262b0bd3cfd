"""G2PTQ quantizer object, a drop-in for gptq_utils/g2ptq_utils.py of the reference
(``G2PTQ`` g2ptq_utils.py:129-527, ``run_eager`` :97-126, ``reduce_to_target_rank``
:530-575).

Block-wise Hessians: ``H[g] <- H[g] k/(k+1) + (1/(t (k+1))) sum_n s[n,g] x_n x_n^T``
(g2ptq_utils.py:193-200).  Unrolled over calls this is
``H[g] = (1/K) sum_calls (1/t_call) sum_n s[n,g] x_n x_n^T``, so each staged
token carries the weight ``s[n,g] / t_call`` and a fold rescales by
``K_folded / K_now`` -- one saliency-weighted Gram product per row group.
"""

import contextlib

import torch

from .. import ops, _lib
from . import _engine, collectives
from .common_utils import fake_quantize_grouped
from .graph_utils import validate_tensors
from .gptq_utils import _onload
from .refresh import (SaliencyCache, GradientCache, normalize_loss_weights,  # noqa: F401
                      compute_kl_grad_hessian, compute_mse_grad_hessian, block_loss)


def run_eager(weight, hinv, scale, zero, z, ghinv, maxq, backend="torch", int_weight=None,
              error=None, weight_raw=None, approx_beta=0.0):
    """One G2PTQ compensation block, reference layout ``[B, blk, R]``
    (g2ptq_utils.py:97-126); updates ``weight`` and ``ghinv`` in place.
    ``weight_raw`` with ``approx_beta`` != 0 runs the --approx_grad ablation
    (lines 48-51, 71-73)."""
    tensors = [weight, hinv, scale, zero, z, ghinv, int_weight, error]
    if weight_raw is not None:
        tensors.append(weight_raw)
    validate_tensors("G2PTQ", *tensors)
    B, blk, R = weight.shape
    W = weight.transpose(1, 2).contiguous()
    S = scale.transpose(1, 2).contiguous().reshape(B * R, blk)
    Zp = zero.transpose(1, 2).contiguous().reshape(B * R, blk)
    zz = z.transpose(1, 2).contiguous()
    gh = ghinv.transpose(1, 2).contiguous()
    colmap = torch.arange(blk, dtype=torch.int32, device=weight.device)
    codes = torch.empty(B, R, blk, dtype=torch.int8, device=weight.device)
    err = torch.empty(B, blk, R, dtype=torch.float32, device=weight.device)
    raw = (weight_raw.transpose(1, 2).contiguous()
           if (approx_beta and weight_raw is not None) else None)
    ops.compensate_block(_lib.METHOD_G2PTQ, W, hinv.contiguous(), S, Zp, colmap, maxq,
                         codes=codes, err=err, z=zz, ghinv=gh, wraw=raw,
                         approx_beta=approx_beta if raw is not None else 0.0)
    weight.copy_(W.transpose(1, 2))
    ghinv.copy_(gh.transpose(1, 2))
    int_weight.copy_(codes.transpose(1, 2))
    error.copy_(err)
    return weight, int_weight, error


class G2PTQ(_engine.StagingMixin):
    index = _engine.lazy_counter("index")
    total_tokens = _engine.lazy_counter("total_tokens")

    def __init__(self, layers, saliencies, gradients, num_groups: int,
                 offload_hessians: bool = False, approx_grad_beta: float = 0.0):
        self.layers = layers
        self.num_layers = len(layers)
        self.offload_hessians = offload_hessians
        self.approx_grad_beta = approx_grad_beta
        weight = layers[0].weight
        self.dev = weight.device
        if self.dev.type != "cuda":
            raise RuntimeError("g2ptq_b200 G2PTQ requires layers on a CUDA device")
        self.rows, self.columns = weight.shape
        self.num_groups = num_groups
        self.saliencies = []
        for saliency in saliencies:
            self.saliencies.append([s.float() for s in saliency] if saliency is not None
                                   else None)
        H_device = "cpu" if offload_hessians else self.dev
        self.gradients = torch.zeros((self.num_layers, self.rows, self.columns),
                                     dtype=torch.float32, device=H_device)
        for b, gradient in enumerate(gradients):
            if gradient is not None and isinstance(gradient, torch.Tensor):
                self.gradients[b].copy_(gradient, non_blocking=True)
        self._H = torch.zeros((self.num_layers, num_groups, self.columns, self.columns),
                              dtype=torch.float32, device=H_device)
        self.act_square = torch.zeros((self.num_layers, self.columns), device=self.dev)
        self.index = torch.zeros(self.num_layers, dtype=torch.long, device=self.dev)
        self.total_tokens = torch.zeros(self.num_layers, dtype=torch.long, device=self.dev)
        self._k = [0] * self.num_layers
        self._k_folded = [0] * self.num_layers
        self._tok = [0] * self.num_layers
        assert self.rows % self.num_groups == 0, (
            f"Number of rows ({self.rows}) must be divisible by num_groups ({self.num_groups})")
        self._init_stages(groups=num_groups)

    @property
    def H(self):
        self._flush_all()
        return self._H

    @H.setter
    def H(self, value):
        self._H = value

    def _maybe_onload_hessian_grad(self, hessian=True, gradients=False):
        """g2ptq_utils.py:172-180."""
        if not self.offload_hessians:
            return contextlib.nullcontext()
        names = ("_H",) if hessian else ()
        if gradients:
            names += ("gradients",)
        return _onload(self, names)

    @torch.no_grad()
    def add_batch(self, idx, inp, out):
        """g2ptq_utils.py:182-201."""
        if inp.dim() == 3:
            inp = inp.reshape(-1, inp.shape[-1])
        x = _engine.as_rows(inp, self.columns)
        n_tokens = x.shape[0]
        sal = self.saliencies[idx][0].to(self.dev).float()
        del self.saliencies[idx][0]
        self._k[idx] += 1
        _engine.bump(self, "index", idx, 1)
        t_old = self._tok[idx]
        self._tok[idx] += n_tokens
        _engine.bump(self, "total_tokens", idx, n_tokens)
        ops.sq_colsum(self.act_square[idx], x, keep=t_old / self._tok[idx],
                      scale=1.0 / self._tok[idx])
        w = (sal.reshape(n_tokens, self.num_groups) * (1.0 / n_tokens)).contiguous()
        self._append(idx, x, scales=w)

    def _fold(self, idx, X, sub, scales):
        k_old, k_new = self._k_folded[idx], self._k[idx]
        self._require_device_stats(self._H)
        ops.gram_update_grouped(self._H[idx], X, scales, alpha=k_old / k_new, beta=1.0 / k_new,
                                precision=_engine.PRECISION)
        self._k_folded[idx] = k_new

    def fasterquant(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                    static_groups=False, enable_gradient_update=True, alpha=0.0,
                    export_compressed_tensors=False, backend="torch", graph=False):
        """g2ptq_utils.py:349-519 (``backend`` / ``graph`` accepted and ignored)."""
        pending = self._fq_launch(blocksize=blocksize, percdamp=percdamp, groupsize=groupsize,
                                  actorder=actorder, static_groups=static_groups,
                                  enable_gradient_update=enable_gradient_update, alpha=alpha,
                                  export_compressed_tensors=export_compressed_tensors)
        self._last_damps = pending.finish()

    def _fq_launch(self, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                   static_groups=False, enable_gradient_update=True, alpha=0.0,
                   export_compressed_tensors=False, backend="torch", graph=False):
        B, R, C, G = self.num_layers, self.rows, self.columns, self.num_groups
        rps = R // G
        nl = B * G
        q0 = self.quantizer[0]
        W = torch.stack([l.weight.data for l in self.layers]).float().contiguous()
        W_flat = W.view(B * R, C)
        W_sub = W.view(nl, rps, C)
        with self._maybe_onload_hessian_grad(gradients=True):
            grad = self.gradients.to(self.dev, copy=True).view(nl, rps, C).contiguous()
            H = self.H.view(nl, C, C)
            self.H = None
        H_diag = _engine.hessian_diag(H, q0)
        params = _engine.ParamSet(self.quantizer, B * R, C, groupsize, self.dev)
        dynamic = not (groupsize == -1 or static_groups)
        if not dynamic:
            params.init_static(W_flat, H_diag)
        ops.prepare_hessian(H, W_sub, gzero=grad)
        use_grad = enable_gradient_update and alpha > 0
        Q_sub = None
        if use_grad:
            if dynamic:
                for i, q in enumerate(self.quantizer):
                    # g2ptq_utils.py:405-412 passes no Hessian diagonal here
                    q.find_params(W_sub[:, :, i * groupsize:(i + 1) * groupsize]
                                  .reshape(B * R, -1))
            Q_sub = fake_quantize_grouped(self.quantizer, W_sub, groupsize).contiguous()
        perm = None
        if actorder:
            perm, _ = _engine.act_order_perm(torch.mean(self.act_square, dim=0))
            W_sub = ops.permute_cols(W_sub, perm)
            H = ops.permute_sym(H, perm)
            grad = ops.permute_cols(grad, perm)
            if Q_sub is not None:
                Q_sub = ops.permute_cols(Q_sub, perm)
        clip, clip_hd = _engine.dynamic_clip(q0, H_diag, perm, B * R, C) if dynamic else (None,
                                                                                          None)
        U, info, damps = _engine.factor_with_retry(H, percdamp)
        colgroup = params.colgroup(perm, static_groups, self.dev)
        W0 = W_sub.contiguous()
        codes = torch.empty(nl, rps, C, dtype=torch.int8, device=self.dev)

        def run(Wp):
            # Z = (G U^T) * beta, GHinv = Z U  (g2ptq_utils.py:459-476)
            T1 = ops.gemm(torch.empty_like(grad), grad, U, transB=True,
                          precision=_engine.PRECISION)
            if use_grad:
                GH0 = ops.gemm(torch.empty_like(grad), T1, U, precision=_engine.PRECISION)
                dinv = ops.diag_of_utu(U)
                beta = ops.trust_region_beta(grad, GH0, Q_sub, W0, dinv, alpha)
            else:
                beta = torch.zeros(nl, rps, dtype=torch.float32, device=self.dev)
            Z = ops.scale_rows(T1, beta)
            GH = ops.gemm(torch.empty_like(grad), Z, U, precision=_engine.PRECISION)
            # --approx_grad: W0 is the reference's W_raw snapshot (the traversal's
            # input after act-order and dead columns, g2ptq_utils.py:270-273)
            approx = float(self.approx_grad_beta or 0.0)
            ops.compensate(_lib.METHOD_G2PTQ, Wp, U, params.scale, params.zero, colgroup,
                           dynamic, groupsize, q0.bits, q0.sym, blocksize, codes, z=Z, gh=GH,
                           status=params.status, precision=_engine.PRECISION, clip=clip,
                           wraw=W0 if approx else None, approx_beta=approx)
            _ = clip_hd  # the diagonal the clip configuration points to stays alive
            Q, cq = Wp, codes
            if actorder:
                Q = ops.permute_cols(Wp, perm, inverse=True)
                cq = ops.permute_cols(codes, perm, inverse=True)
            Q, cq = Q.view(B, R, C), cq.view(B, R, C)
            nan, outs = _engine.write_back(self.layers, Q, cq, params, q0.bits, groupsize, C,
                                           export_compressed_tensors)
            return nan, outs, cq

        return _engine.Pending(self.layers, nl, H, U, info, damps, params, run, W0, q0.bits,
                               groupsize, C, R, export_compressed_tensors, dynamic, actorder)

    def free(self):
        self._H = None
        self.Losses = None
        self.gradients = None
        self.saliencies = None
        self.act_square = None
        self._stages = None


def reduce_to_target_rank(g2ptqs, g2ptq2rank):
    """g2ptq_utils.py:530-575: the block-wise Hessians and the gradients
    rescaled by each rank's share of the calls, the squared-activation means by
    its share of the tokens, summed onto the owner, whose ``index`` /
    ``total_tokens`` become the global counts (one count all_reduce, one
    packed reduce per owner rank)."""

    def counts(g):
        g._flush_all()
        return list(g._k) + list(g._tok)

    def entries(g, local, glob, owner):
        B = g.num_layers
        out = []
        for b in range(B):
            k_loc, k_glob = local[b], glob[b]
            t_loc, t_glob = local[B + b], glob[B + b]
            if k_glob == 0:
                g._H[b].zero_()
                g.gradients[b].zero_()
                g.act_square[b].zero_()
                continue
            w = k_loc / k_glob
            out += [collectives.Entry(owner, g._H[b], symmetric=True, weight=w),
                    collectives.Entry(owner, g.act_square[b], weight=t_loc / t_glob),
                    collectives.Entry(owner, g.gradients[b], weight=w)]
        return out

    def commit(g, glob):
        B = g.num_layers
        g.index = torch.tensor(glob[:B], dtype=torch.long, device=g.dev)
        g.total_tokens = torch.tensor(glob[B:], dtype=torch.long, device=g.dev)
        g._k, g._k_folded, g._tok = list(glob[:B]), list(glob[:B]), list(glob[B:])

    collectives.reduce_objects(g2ptqs, g2ptq2rank, counts, entries, commit,
                               lambda g: g._maybe_onload_hessian_grad(gradients=True))
