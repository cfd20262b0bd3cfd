"""Shared machinery of the quantizer objects: token staging for ``add_batch``
and the device pipeline behind ``fasterquant``.

Staging.  The reference updates the running Hessian on every hook call
(``H <- H n/(n+b) + (2/(n+b)) X^T X``, gptq_utils.py:123-126), i.e. a full
read-modify-write of the C x C matrix per 2048-token sequence at the default
``--bsz 1``, which costs as much HBM time as the product itself.  Here each
call only copies its tokens into a per-layer staging buffer; the buffer is
folded into ``H`` by one Gram launch when it fills up or when ``H`` is read.
Folding b pending samples at once applies the same rescale the reference
applies call by call: ``H <- H n_old/n_new + (2/n_new) sum X^T X``.

fasterquant.  Everything between the stacked weights and the written-back
quantized weights runs on the device (find_params, dead columns, act-order
permutation, damped inverse-Cholesky, compensation, un-permutation, cast and
NaN count).  The host reads back one small status vector per call; the
damp auto-increment of the reference (gptq_utils.py:291-311) re-runs only
when a layer's factorization failed.

Shared folds.  Linears fed the same tensor (q/k/v of an attention block,
gate/up of an MLP) get identical Hessians; the reference computes each one.
GPTQ objects whose add_batch calls carry the same source tensors, in the same
order, share one stage and one Gram fold per window (``FoldGroup``); every
member keeps its own ``H``, refreshed by a copy after each fold, so a member
that later receives a different input leaves the group with exactly the
state it would have had alone.
"""

import logging
import os
import weakref

import torch

from .. import ops, _lib
from ..utils import compressed_tensors_utils

DAMP_INCREMENT = 0.0015
STAGE_TOKENS = int(os.environ.get("G2PTQ_B200_STAGE_TOKENS", "16384"))
STAGE_BYTES = int(os.environ.get("G2PTQ_B200_STAGE_BYTES", str(512 << 20)))
# 0 = fp32 CUDA cores, 1 = tcgen05 tensor cores (Gram products and trailing updates)
PRECISION = int(os.environ.get("G2PTQ_B200_PRECISION", "1"))
# objects fed the same tensors share their Gram folds (0 disables)
SHARE_FOLDS = os.environ.get("G2PTQ_B200_SHARE_FOLDS", "1") != "0"


class TokenStage:
    """Pending calibration tokens of one layer, folded into a Gram matrix lazily.

    ``buf`` holds the tokens (bf16 for bf16 inputs, else fp32), ``sub_buf``
    an optional fp32 second operand (GPTAQ's ``X_fp - X``), ``scale_buf`` optional
    per-token weights ``[cap, groups]`` (G2PTQ / GuidedQuant saliencies).
    """

    def __init__(self, columns, device, groups=0):
        self.columns = columns
        self.device = device
        self.groups = groups
        self.buf = None
        self.sub_buf = None
        self.scale_buf = None
        self.rows = 0
        self.dtype = None

    def capacity(self, elem):
        return max(1, min(STAGE_TOKENS, STAGE_BYTES // (self.columns * elem)))

    def _ensure(self, dtype, with_sub):
        if self.buf is None or self.buf.dtype != dtype or (with_sub and self.sub_buf is None):
            cap = self.capacity(torch.tensor([], dtype=dtype).element_size() +
                                (4 if with_sub else 0))
            self.buf = torch.empty(cap, self.columns, dtype=dtype, device=self.device)
            self.sub_buf = (torch.empty(cap, self.columns, dtype=torch.float32,
                                        device=self.device) if with_sub else None)
            self.scale_buf = (torch.empty(cap, self.groups, dtype=torch.float32,
                                          device=self.device) if self.groups else None)
            self.dtype = dtype

    def cap(self):
        return self.buf.shape[0]

    def free(self):
        self.buf = None
        self.sub_buf = None
        self.scale_buf = None
        self.rows = 0


def lazy_counter(name):
    """Class attribute for a per-layer int64 device counter (``nsamples``,
    ``index``, ``total_tokens``) whose ``add_batch`` increments stay on the
    host until the attribute is read: one add kernel per layer at a read
    instead of one per hook call.  Reads see every increment so far, and edits
    made in place through a read are kept (increments are added, never
    overwritten)."""
    store, pend = "_" + name + "_dev", "_" + name + "_pending"

    def get(self):
        t = self.__dict__.get(store)
        p = self.__dict__.get(pend)
        if t is not None and p:
            for i, d in p.items():
                t[i] += d
            p.clear()
        return t

    def set(self, value):
        self.__dict__[store] = value
        self.__dict__[pend] = {}

    return property(get, set)


def bump(obj, name, idx, delta):
    """Record ``obj.<name>[idx] += delta`` for the next read of the counter."""
    p = obj.__dict__["_" + name + "_pending"]
    p[idx] = p.get(idx, 0) + delta


def stage_dtype(x):
    return torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32


def as_rows(x, columns):
    x = x.reshape(-1, columns)
    if x.stride(1) != 1:
        x = x.contiguous()
    return x


def sync_check(*tensors):
    """One device->host read of several small int tensors."""
    flat = torch.cat([t.reshape(-1).to(torch.int64) for t in tensors])
    return flat.cpu().tolist()


def factor_with_retry(H, percdamp, info=None):
    """Damped inverse-Cholesky of every ``H[b]``; the reference's damp
    auto-increment runs for each failing ``b`` (one host read per attempt).

    Returns ``(U, damps)``.
    """
    nl = H.shape[0]
    damps = [float(percdamp)] * nl
    if not (1 > percdamp > 0):
        raise ValueError(f"Quantization: `damp_percent` must between 0 and 1. current is "
                         f"{percdamp}")
    U, info = ops.chol_upper_inverse(H, damps, info, precision=PRECISION)
    return U, info, damps


def raise_device_errors(info, statuses, timeouts_only=False):
    """Raise for device conditions other than a failed pivot: a tensor-core
    wait that gave up (in a Cholesky ``info`` or a status word) and, unless
    ``timeouts_only``, a non-positive quantization scale (``find_params``)."""
    if any(s == _lib.G2Q_ERR_TIMEOUT for s in list(info) + list(statuses)):
        raise RuntimeError("g2ptq_b200: a tensor-core pipeline wait timed out "
                           f"({_lib.status_string(_lib.G2Q_ERR_TIMEOUT)})")
    if not timeouts_only and any(s != 0 for s in statuses):
        raise RuntimeError("WeightQuantizer.find_params: non-positive scale")


def retry_failed(H, U, info_list, damps):
    """Re-factor failing layers with the damp auto-increment."""
    for b, inf in enumerate(info_list):
        if inf == 0:
            continue
        d = damps[b]
        while True:
            logging.warning(f"Quantization: Current `damp_percent = {d:.5f}` is too low, "
                            f"auto-incrementing by `{DAMP_INCREMENT:.5f}`")
            d += DAMP_INCREMENT
            if not (1 > d > 0):
                raise ValueError(
                    f"Quantization: `damp_percent` must between 0 and 1. current is {d}")
            Ub, ib = ops.chol_upper_inverse(H[b:b + 1].contiguous(), [d], precision=PRECISION)
            code = int(ib.item())
            raise_device_errors([code], [])
            if code == 0:
                U[b].copy_(Ub[0])
                break
        damps[b] = d
    return U


class ParamSet:
    """Quantization parameters of a layer batch: ``[nl*rows, ngroups]`` scale
    and zero arrays plus the column -> parameter-column map.  Each group
    quantizer's ``scale`` / ``zero`` becomes a ``[nl*rows, 1]`` view of one
    column, so callers reading the quantizers see the final values."""

    def __init__(self, quantizers, total_rows, columns, groupsize, device):
        self.quantizers = quantizers
        self.ng = len(quantizers)
        self.groupsize = groupsize
        self.scale = torch.zeros(total_rows, self.ng, dtype=torch.float32, device=device)
        self.zero = torch.zeros_like(self.scale)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.columns = columns

    def init_static(self, W_flat, H_diag=None):
        """gptq_utils.py:259-270 for ungrouped / static-group quantizers.

        Fresh per-channel quantizers of one configuration without the clip
        search (the usual case) get their parameters from a single launch over
        all groups instead of one ``find_params`` call each."""
        gs = self.groupsize
        qs = self.quantizers
        q0 = qs[0]
        if (gs > 0 and len(qs) == (self.columns + gs - 1) // gs and q0.bits < 16
                and all(not q.ready() and not q.mse and q.perchannel and q.bits == q0.bits
                        and q.sym == q0.sym and getattr(q, "weight_groupsize", -1) <= 0
                        for q in qs)):
            ops.find_params_groups(self.scale, self.zero, W_flat, q0.bits, q0.sym, gs,
                                   self.status)
            for i, q in enumerate(qs):
                q.scale, q.zero = self.scale[:, i:i + 1], self.zero[:, i:i + 1]
                q._ready = True
            return
        for i, q in enumerate(self.quantizers):
            sv = self.scale[:, i:i + 1]
            zv = self.zero[:, i:i + 1]
            if not q.ready():
                cols = slice(None) if gs == -1 else slice(i * gs, (i + 1) * gs)
                q.find_params(W_flat[:, cols],
                              None if H_diag is None else H_diag[:, cols], out=(sv, zv))
            else:
                sv.copy_(q.scale.reshape(-1, 1).to(sv))
                zv.copy_(q.zero.reshape(-1, 1).to(zv))
            q.scale, q.zero = sv, zv

    def bind_dynamic(self):
        for i, q in enumerate(self.quantizers):
            q.scale = self.scale[:, i:i + 1]
            q.zero = self.zero[:, i:i + 1]
            q._ready = True

    def statuses(self):
        out = [self.status]
        for q in self.quantizers:
            if getattr(q, "_status", None) is not None:
                out.append(q._status)
        return out

    def colgroup(self, perm, static_groups, device):
        C = self.columns
        if self.groupsize == -1:
            return torch.zeros(C, dtype=torch.int32, device=device)
        idx = perm if (perm is not None and static_groups) else torch.arange(C, device=device)
        return (idx // self.groupsize).to(torch.int32).contiguous()


def hessian_diag(H, quantizer):
    """``torch.diagonal(H).clone()`` when the quantizers use ``hclip`` (the
    reference takes it before the dead-column / damping edits), else None."""
    if not quantizer.hclip:
        return None
    return torch.diagonal(H, dim1=-2, dim2=-1).reshape(-1, H.shape[-1]).clone()


def dynamic_clip(quantizer, H_diag, perm, total_rows, columns):
    """Clip-search configuration for parameters found during the traversal
    (dynamic groups), with the diagonal in the traversal's column order.
    Returns ``(config or None, tensor to keep alive)``."""
    if not quantizer.mse:
        return None, None
    hd = H_diag
    if hd is not None and perm is not None:
        hd = hd[:, perm].contiguous()
    return quantizer.clip_config(hd, total_rows, columns), hd


def act_order_perm(key):
    """``torch.argsort(key, descending=True)`` (stable) and its inverse."""
    perm = ops.argsort_desc(key.contiguous())
    invperm = torch.empty_like(perm)
    invperm[perm] = torch.arange(perm.numel(), device=perm.device)
    return perm, invperm


def write_back(layers, Q, codes, params, bits, groupsize, columns, export, perm_dynamic=None):
    """Cast, NaN check and hand-over of the quantized weights (gptq_utils.py:329-353).

    Returns the list of device tensors to check on the host; ``finish`` applies them."""
    nan = torch.zeros(1, dtype=torch.int32, device=Q.device)
    outs = []
    for b, layer in enumerate(layers):
        outs.append(ops.cast_check(Q[b].contiguous(), layer.weight.dtype, nan))
    return nan, outs


def finish(layers, outs, codes, params, bits, groupsize, columns, export, rows):
    for b, layer in enumerate(layers):
        if export:
            if groupsize == -1:
                gscale = params.scale[b * rows:(b + 1) * rows, :1]
            else:
                gscale = params.scale[b * rows:(b + 1) * rows]
            compressed_tensors_utils.compress_grouped(layer, gscale, codes[b], bits)
        layer.weight.data.copy_(outs[b].reshape(layer.weight.shape))


def source_key(x, samples):
    """Identity of an add_batch input: storage address, shape, strides, dtype,
    version counter (a write through any view bumps it) and the samples the
    call counts.  A group holds the tensor while its key is in use, so the
    address cannot be reused by another tensor meanwhile."""
    return (x.data_ptr(), tuple(x.shape), tuple(x.stride()), x.dtype, x._version, samples)


# groups that have not folded yet, by the key of their first call: a fresh
# object whose first input has that key joins instead of starting its own
_OPEN_GROUPS = weakref.WeakValueDictionary()


class FoldGroup:
    """Members ``(object, layer)`` whose add_batch calls so far carried the
    same source tensors in the same order.

    The group stages each call's tokens once (the first member to make the
    call copies them; the others only compare keys) and folds the window into
    the first member's statistics with that member's ``_fold``; the other
    members copy the result and its sample count (``_copy_folded``).  A
    member's state is its own statistics plus the window's first ``pos``
    calls.  A window is folded only when every member has made all of its
    calls; members that lag at that point, or whose next input differs, leave
    with a private stage holding their part of the window.  The fold's sample
    count is the one a lone object would use: the folded count, the window's
    samples and, for a fold that a new call triggers, that call's samples.

    Members are held by weak reference (each member holds its group), so the
    window's tensors go with the last member even if it is dropped without
    ``free()``.
    """

    def __init__(self, obj, idx, dtype, columns, device):
        self._members = [(weakref.ref(obj), idx)]
        self.pos = [0]
        self.stage = TokenStage(columns, device)
        self.stage._ensure(dtype, False)
        self.keys, self.srcs, self.row_ends = [], [], []
        self.samples = 0  # samples counted by the window's calls
        self.folded = False
        self.first_key = None

    # -- membership -------------------------------------------------------
    @property
    def members(self):
        """Live members ``(object, layer)``; members whose objects are gone are
        dropped (with their positions)."""
        live = [(r(), i) for r, i in self._members]
        if any(o is None for o, _ in live):
            keep = [k for k, (o, _) in enumerate(live) if o is not None]
            self._members = [self._members[k] for k in keep]
            self.pos = [self.pos[k] for k in keep]
            live = [live[k] for k in keep]
            if not live:
                self.close()
        return live

    def _index(self, obj, idx):
        for k, (r, i) in enumerate(self._members):
            if r() is obj and i == idx:
                return k
        raise KeyError("not a member")

    def can_join(self, key, dtype):
        return (not self.folded and self.keys and self.keys[0] == key
                and self.stage.dtype == dtype)

    def join(self, obj, idx):
        self._members.append((weakref.ref(obj), idx))
        self.pos.append(0)

    def detach(self, obj, idx):
        """Remove a member; its private stage receives the tokens of the
        calls it made in this window."""
        k = self._index(obj, idx)
        p = self.pos.pop(k)
        self._members.pop(k)
        obj._groups[idx] = None
        rows = self.row_ends[p - 1] if p else 0
        if rows:
            st = obj._stages[idx]
            st._ensure(self.stage.dtype, False)
            st.buf[:rows].copy_(self.stage.buf[:rows])
            st.rows = rows
        if not self._members:
            self.close()

    def dissolve(self):
        for o, i in self.members:
            self.detach(o, i)

    def close(self):
        self.stage.free()
        self.keys, self.srcs, self.row_ends = [], [], []
        self.samples = 0
        self.folded = True

    # -- calls ------------------------------------------------------------
    def call(self, obj, idx, x, key, samples):
        """Handle one add_batch call of a member (``samples`` already added to
        its count); False when the caller must stage ``x`` itself (the member
        has left the group)."""
        k = self._index(obj, idx)
        p = self.pos[k]
        if p < len(self.keys):
            if self.keys[p] == key:
                self.pos[k] = p + 1
                return True
            self.detach(obj, idx)
            return False
        t = x.shape[0]
        if stage_dtype(x) != self.stage.dtype or t > self.stage.cap():
            self.dissolve()
            return False
        if self.stage.rows + t > self.stage.cap():
            self.fold(trigger_samples=samples)
            if obj._groups[idx] is not self:  # left while the window closed
                return False
        ops.stage_tokens(self.stage.buf, self.stage.rows, x)
        self.stage.rows += t
        self.samples += samples
        self.keys.append(key)
        self.srcs.append(x)
        self.row_ends.append(self.stage.rows)
        self.pos[self._index(obj, idx)] = len(self.keys)
        return True

    def fold(self, trigger_samples=0):
        """Fold the window for every member that made all of its calls; the
        others leave first with their part of it."""
        n = len(self.keys)
        members = self.members
        for o, i in [m for m, p in zip(members, self.pos) if p < n]:
            self.detach(o, i)
        members = self.members
        if not members or self.stage.rows == 0:
            return
        o0, i0 = members[0]
        if len({o._n_folded[i] for o, i in members}) != 1:
            self.dissolve()
            return
        n_new = o0._n_folded[i0] + self.samples + trigger_samples
        o0._fold(i0, self.stage.buf[:self.stage.rows], None, None, n_new=n_new)
        for o, i in members[1:]:
            o._copy_folded(i, o0, i0)
        self.stage.rows = 0
        # the triggering call is staged next, but its samples are in n_new
        self.samples = -trigger_samples
        self.keys, self.srcs, self.row_ends = [], [], []
        self.pos = [0] * len(self._members)
        if not self.folded:
            self.folded = True
            if self.first_key is not None and _OPEN_GROUPS.get(self.first_key) is self:
                del _OPEN_GROUPS[self.first_key]


class StagingMixin:
    """``add_batch`` plumbing shared by the quantizer objects.

    Subclasses provide ``_fold(idx, X, sub, scales)``, which folds staged
    tokens into their statistics using the counts recorded so far.  Because
    every fold rescales by (counts already folded) / (counts now), any split
    of the pending tokens into folds gives the same statistics.  Subclasses
    that set ``_share_folds`` and provide ``_copy_folded(idx, src, src_idx)``
    (copy the folded statistics and counts of another object's layer) share
    folds with objects fed the same tensors (``FoldGroup``).
    """

    _share_folds = False

    def _init_stages(self, groups=0):
        self._stages = [TokenStage(self.columns, self.dev, groups)
                        for _ in range(self.num_layers)]
        self._groups = [None] * self.num_layers
        self._calls = [0] * self.num_layers

    def _shared_call(self, idx, x, samples):
        """Route an add_batch call (``samples`` already counted) through a fold
        group; False when the tokens must go to the object's own stage."""
        calls = self._calls[idx]
        self._calls[idx] = calls + 1
        if not (SHARE_FOLDS and self._share_folds):
            return False
        g = self._groups[idx]
        key = source_key(x, samples)
        if g is None:
            if calls != 0 or self._stages[idx].rows or not self._stats_on_device():
                return False
            reg = (key, self.columns, self.dev)
            g = _OPEN_GROUPS.get(reg)
            if g is not None and g.can_join(key, stage_dtype(x)):
                g.join(self, idx)
            else:
                g = FoldGroup(self, idx, stage_dtype(x), self.columns, self.dev)
                g.first_key = reg
                _OPEN_GROUPS[reg] = g
            self._groups[idx] = g
        return g.call(self, idx, x, key, samples)

    def _stats_on_device(self):
        return True

    def _settle(self, idx):
        """Called by a flush with nothing pending; subclasses whose folded
        count can differ from the count at that point (a fold-group member
        that left right after a fold another member's call triggered, or an
        add_batch call without tokens) rescale their statistics to it."""

    def _leave_groups(self):
        for i, g in enumerate(getattr(self, "_groups", None) or []):
            if g is not None:
                g.detach(self, i)

    def _append(self, idx, x, sub=None, scales=None):
        st = self._stages[idx]
        dt = stage_dtype(x)
        if st.rows and st.dtype != dt:
            self._flush(idx)
        st._ensure(dt, sub is not None)
        cap = st.cap()
        t = x.shape[0]
        for s in range(0, t, cap):
            e = min(t, s + cap)
            if st.rows + (e - s) > cap:
                self._flush(idx)
            ops.stage_tokens(st.buf, st.rows, x[s:e])
            if sub is not None:
                ops.stage_tokens(st.sub_buf, st.rows, sub[s:e], x[s:e])
            if scales is not None:
                st.scale_buf[st.rows:st.rows + (e - s)].copy_(scales[s:e])
            st.rows += e - s

    def _flush(self, idx):
        g = self._groups[idx] if getattr(self, "_groups", None) else None
        if g is not None:
            g.fold()  # this member, if it lags, leaves with its calls staged privately
        st = self._stages[idx]
        if st.rows == 0:
            self._settle(idx)
            return
        self._fold(idx, st.buf[:st.rows],
                   None if st.sub_buf is None else st.sub_buf[:st.rows],
                   None if st.scale_buf is None else st.scale_buf[:st.rows])
        st.rows = 0

    def _flush_all(self):
        if getattr(self, "_stages", None) is None:
            return
        for i in range(self.num_layers):
            self._flush(i)

    def _require_device_stats(self, t):
        if t.device.type != "cuda":
            raise RuntimeError("add_batch needs the statistics on the device; wrap the "
                               "calibration forward in the object's onload context when "
                               "offload_hessians=True")


class Pending:
    """A launched ``fasterquant`` whose results are still on the device.

    ``run(W_init)`` enqueues compensation, un-permutation and the cast / NaN
    count and returns ``(nan, outs, codes)``; ``finish()`` reads every status
    word in one device-to-host copy, re-factors failing layers with the damp
    auto-increment (re-running the compensation from ``W0``), raises where the
    reference raises and hands the weights (and export qparams) to the layers.
    """

    def __init__(self, layers, nl, H, U, info, damps, params, run, W0, bits, groupsize,
                 columns, rows, export, dynamic, actorder, borrowed_factor=False,
                 lent_factor=False):
        self.layers, self.nl, self.H, self.U, self.info = layers, nl, H, U, info
        self.damps, self.params, self.run, self.W0 = damps, params, run, W0
        self.bits, self.groupsize, self.columns, self.rows = bits, groupsize, columns, rows
        self.export, self.dynamic, self.actorder = export, dynamic, actorder
        # U, info and damps belong to another object's launch (shared factor),
        # which finishes first and re-factors U in place if it must
        self.borrowed_factor = borrowed_factor
        # other objects' compensations, on other streams, read this launch's U
        self.lent_factor = lent_factor
        self.nan, self.outs, self.codes = run(W0.clone())

    def _flags(self):
        """One device-to-host read: per-layer Cholesky info, the NaN count and
        the status words (the device's tensor-core word, then the parameters')."""
        return sync_check(self.info, self.nan, ops.device_status(self.U.device),
                          *self.params.statuses())

    def finish(self):
        nl = self.nl
        flags = self._flags()
        # a timeout is fatal; a non-positive scale is judged after any re-run
        # (a failed factorization can leave NaN weights behind it)
        raise_device_errors(flags[:nl], flags[nl + 1:], timeouts_only=True)
        if any(i != 0 for i in flags[:nl]):
            if self.borrowed_factor:
                torch.cuda.synchronize(self.U.device)  # the owner's re-factored U
            else:
                if self.lent_factor:
                    # the borrowers' first compensations still read U on their
                    # own streams: let them end before U is re-factored in place
                    # (their results are discarded and re-run with the new U)
                    torch.cuda.synchronize(self.U.device)
                retry_failed(self.H, self.U, flags[:nl], self.damps)
            self.params.status.zero_()
            self.nan, self.outs, self.codes = self.run(self.W0.clone())
            flags = self._flags()
            flags[:nl] = [0] * nl
        raise_device_errors(flags[:nl], flags[nl + 1:])
        if flags[nl] != 0:
            raise ValueError("NaN in weights")
        if self.dynamic:
            self.params.bind_dynamic()
        if self.export and self.dynamic and self.actorder:
            raise AssertionError("Scales in the same quantization group should be the same.")
        finish(self.layers, self.outs, self.codes, self.params, self.bits, self.groupsize,
               self.columns, self.export, self.rows)
        return self.damps


_STREAMS = {}


def factor_roles(objs):
    """Which of ``objs`` (in launch order) can share a damped inverse-Cholesky
    factor: one-layer objects that offer it (``_share_factor``), are still
    members of the same fold group and whose Hessian was never handed out
    through the public ``H`` property hold bit-identical Hessians (copies of
    one fold), hence identical factors.  Returns ``{position: ("factor_out" |
    "factor_in", slot)}``: the first of each group computes the factor and
    fills the slot, the others take it from there."""
    slots, roles = {}, {}
    for n, o in enumerate(objs):
        if not (SHARE_FOLDS and getattr(o, "_share_factor", False) and o.num_layers == 1):
            continue
        groups = getattr(o, "_groups", None)
        g = groups[0] if groups else None
        if g is None or getattr(o, "_h_exposed", False):
            continue
        if id(g) in slots:
            roles[n] = ("factor_in", slots[id(g)])
        else:
            slots[id(g)] = {"group": g}
            roles[n] = ("factor_out", slots[id(g)])
    # a group with a single eligible member has nothing to share
    owners = [n for n, (r, sl) in roles.items() if r == "factor_out"
              and not any(r2 == "factor_in" and sl2 is sl for r2, sl2 in roles.values())]
    for n in owners:
        del roles[n]
    return roles


def stream_pool(device, n=4):
    """``n`` side streams of ``device``: the first at the highest priority the
    device offers (it carries the longest chain), the others at the default."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), n)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(device=device, priority=-16 if i == 0 else 0)
                         for i in range(n)]
    return _STREAMS[key]


def fasterquant_all(objs, streams=4, **kwargs):
    """Quantize several quantizer objects concurrently: each object's pipeline
    is enqueued on one stream of a small pool (longest first), then every
    object is finished (status read, retry, write-back).  Equivalent to
    calling ``obj.fasterquant(**kwargs)`` for each object in turn."""
    if not objs:
        return
    cur = torch.cuda.current_stream(objs[0].dev)
    pool = stream_pool(objs[0].dev, streams)
    # launch the longest chains first (factorization ~ C^3, compensation ~ R C^2)
    order = sorted(range(len(objs)), key=lambda i: -objs[i].num_layers * (
        objs[i].columns ** 3 + objs[i].rows * objs[i].columns ** 2))
    # Pending add_batch folds are large Gram products that fill the GPU on
    # their own: run them in order on the caller's stream first, and overlap
    # only the latency-bound factorization / compensation chains.
    for o in objs:
        if not getattr(o, "offload_hessians", False):
            o._flush_all()
    roles = factor_roles([objs[i] for i in order])
    # The longest chain takes the high-priority stream, so that its kernels go
    # first whenever SMs free up; the shorter chains fill the gaps.
    launched = []
    for n, i in enumerate(order):
        o = objs[i]
        s = pool[0] if n == 0 else pool[1 + (n - 1) % (len(pool) - 1)]
        s.wait_stream(cur)
        extra = {}
        if n in roles:
            extra = {roles[n][0]: roles[n][1]}
        with torch.cuda.stream(s):
            launched.append((s, o, o._fq_launch(**kwargs, **extra)))
    for s, o, pending in launched:
        with torch.cuda.stream(s):
            o._last_damps = pending.finish()
        cur.wait_stream(s)
        if pending.export:
            # export buffers were allocated on the side stream and live on
            # with the layer: tie their reuse to the caller's stream too
            for layer in o.layers:
                for name in compressed_tensors_utils.Q_PARAMS:
                    buf = getattr(layer, name, None)
                    if isinstance(buf, torch.Tensor) and buf.is_cuda:
                        buf.record_stream(cur)
