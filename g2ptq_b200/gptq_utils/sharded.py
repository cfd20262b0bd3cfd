"""Row-sharded quantization of GPTQ objects over the ranks of a process group.

The reference hands each quantizer object to one owner rank, which runs its
whole ``fasterquant`` while the other ranks wait, then broadcasts the result
tensor by tensor (gptq_utils.py:362-391 and the driver loop :455-560,
common_utils.py:96-165).  The largest linear then bounds the step however
many ranks there are.

Rows of a layer are independent once the factor ``U`` is fixed: every row
walks the same columns with the same ``U`` and only its own weights, errors
and quantization parameters.  So here, after the token-parallel calibration:

1. each distinct Hessian is reduced once (packed upper triangle, weighted
   by the ranks' sample shares) to its factor owner; objects whose Hessians
   are bit-identical copies of one shared fold (q/k/v, gate/up) reduce and
   factor once;
2. the distinct Hessian with the largest factorization (the critical path:
   down_proj's C = 14336 in a Llama layer) is factored on rank 0, which
   broadcasts U (packed), the permutation, the raw Hessian diagonal, the
   damps and the status words in one buffer; meanwhile the other ranks
   quantize the other layers whole (LPT over their work);
3. when the large factor arrives, every rank quantizes its slice of rows of
   the layers that use it (static group parameters, dead columns,
   compensation, un-permutation, cast, code packing) with exactly the
   kernels of the single-GPU path, so that every row comes out
   bit-identical to it; a failed factorization is re-done with the damp
   auto-increment afterwards;
4. one ``all_gather`` hands all slices of all layers (weights, packed codes,
   export scales, quantizer parameters) to every rank.

Error conditions found on any rank (NaN weights, a non-positive scale, a
tensor-core timeout) are combined with one all_reduce before the gather, so
every rank raises the same error at the same point.
"""

import contextlib
import copy

import torch
import torch.distributed as dist

from .. import ops, _lib
from . import _engine, collectives
from .common_utils import export_shapes, greedy_bin_packing

# row slices start at multiples of this (the tensor-core trailing update
# needs rows % 8 == 0 to describe its operands; 16 matches the block kernel's
# rows per CTA)
ROW_ALIGN = 16


def row_ranges(rows, world):
    """Contiguous ``[r0, r1)`` per rank covering ``rows``, boundaries at
    multiples of ``ROW_ALIGN`` (the last ranks may get none)."""
    per = -(-rows // world)
    per = -(-per // ROW_ALIGN) * ROW_ALIGN
    return [(min(rows, r * per), min(rows, (r + 1) * per)) for r in range(world)]


def _distinct(objs):
    """``{obj: representative}``: one-layer objects that are members of the
    same fold group with Hessians never handed out hold bit-identical
    statistics; the first of them stands for all."""
    seen, rep = {}, {}
    for o in objs:
        key = None
        groups = getattr(o, "_groups", None)
        if (_engine.SHARE_FOLDS and getattr(o, "_share_factor", False) and o.num_layers == 1
                and groups and groups[0] is not None and not getattr(o, "_h_exposed", False)):
            key = id(groups[0])
        if key is not None and key in seen:
            rep[o] = seen[key]
        else:
            rep[o] = o
            if key is not None:
                seen[key] = o
    return rep


def _slice_quantizer(q, layers, rows, r0, r1):
    """A copy of group quantizer ``q`` for rows ``[r0, r1)`` of each layer."""
    c = copy.deepcopy(q)
    if q.ready() and torch.is_tensor(q.scale) and q.scale.numel() == layers * rows:
        n = r1 - r0
        c.scale = q.scale.reshape(layers, rows)[:, r0:r1].reshape(layers * n, 1).contiguous()
        c.zero = q.zero.reshape(layers, rows)[:, r0:r1].reshape(layers * n, 1).contiguous()
        c._ready = True
    return c


class _Rows:
    """One object's row slice ``[r0, r1)`` on this rank, enqueued on the
    current stream: the single-GPU pipeline after the factorization."""

    def __init__(self, obj, U, shared, r0, r1, blocksize, groupsize, actorder, static_groups,
                 export):
        B, R, C = obj.num_layers, obj.rows, obj.columns
        n = r1 - r0
        self.n = n
        q0 = obj.quantizer[0]
        dev = obj.dev
        self.dynamic = not (groupsize == -1 or static_groups)
        qs = [_slice_quantizer(q, B, R, r0, r1) for q in obj.quantizer]
        self.params = _engine.ParamSet(qs, B * n, C, groupsize, dev)
        self.nan = torch.zeros(1, dtype=torch.int32, device=dev)
        self.outs, self.packed, self.gscale = [], [], []
        if n == 0:
            return
        W = torch.stack([l.weight.data[r0:r1] for l in obj.layers]).float().contiguous()
        diag = shared["diag"]
        H_diag = diag.clone() if q0.hclip else None
        if not self.dynamic:
            self.params.init_static(W.view(B * n, C), H_diag)
        # the owner's RTN fallback / dead columns on this rank's rows: columns
        # whose Hessian diagonal is zero are zeroed, unless the whole diagonal is
        zero = diag == 0
        dead = zero & ~zero.all(dim=1, keepdim=True)
        W.masked_fill_(dead[:, None, :], 0.0)
        perm = shared.get("perm")
        if actorder:
            W = ops.permute_cols(W, perm)
        clip, self._clip_hd = (_engine.dynamic_clip(q0, H_diag, perm, B * n, C) if self.dynamic
                               else (None, None))
        colgroup = self.params.colgroup(perm, static_groups, dev)
        codes = torch.empty(B, n, C, dtype=torch.int8, device=dev)
        ops.compensate(_lib.METHOD_GPTQ, W, U, self.params.scale, self.params.zero, colgroup,
                       self.dynamic, groupsize, q0.bits, q0.sym, blocksize, codes,
                       status=self.params.status, precision=_engine.PRECISION, clip=clip)
        Q, cq = W, codes
        if actorder:
            Q = ops.permute_cols(W, perm, inverse=True)
            cq = ops.permute_cols(codes, perm, inverse=True)
        for b, layer in enumerate(obj.layers):
            self.outs.append(ops.cast_check(Q[b].contiguous(), layer.weight.dtype, self.nan))
            if export:
                self.packed.append(ops.pack_int32(cq[b].contiguous(), q0.bits))
                s = self.params.scale[b * n:(b + 1) * n]
                s = s[:, :1] if groupsize == -1 else s
                self.gscale.append(s.to(layer.weight.dtype).contiguous())

    def flags(self):
        """The NaN count, then the parameters' status words."""
        return [self.nan] + self.params.statuses()


def _mark(marks, name, dev):
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        marks.append((name, ev))


class _FactorBundle:
    """What a factor owner sends for one distinct Hessian, laid out in one
    byte buffer (every part 16-byte aligned) so that it crosses NCCL in one
    broadcast and every rank reads it in place: the packed factor U, the raw
    Hessian diagonal, the act-order permutation, the damps and the
    factorization status words."""

    def __init__(self, B, C, actorder, dev):
        parts = [("U", B * C * (C + 1) // 2, torch.float32), ("diag", B * C, torch.float32),
                 ("damps", B, torch.float32), ("info", B, torch.int32)]
        if actorder:
            parts.append(("perm", C, torch.int64))
        offs, off = {}, 0
        for name, n, dt in parts:
            nbytes = n * torch.tensor([], dtype=dt).element_size()
            offs[name] = (off, n, dt)
            off += -(-nbytes // 16) * 16
        self.buf = torch.zeros(off, dtype=torch.uint8, device=dev)
        self.t = {name: self.buf[o:o + n * torch.tensor([], dtype=dt).element_size()].view(dt)
                  for name, (o, n, dt) in offs.items()}
        self.t["diag"] = self.t["diag"].view(B, C)
        self.B, self.C = B, C
        self.U = None  # the unpacked factor, once known on this rank


def _factor_on_owner(o, bundle, percdamp, actorder):
    """The owner's part for one distinct Hessian, enqueued on the current
    stream: RTN fallback / dead columns, act-order permutation, the damped
    inverse-Cholesky chain; results written into the bundle.  Returns what a
    damp retry needs."""
    t, H = bundle.t, o._H
    t["diag"].copy_(torch.diagonal(H, dim1=-2, dim2=-1))
    ops.prepare_hessian(H)
    if actorder:
        perm, _ = _engine.act_order_perm(ops.mean_diag(H))
        t["perm"].copy_(perm)
        H = ops.permute_sym(H, perm)
    U, info, damps = _engine.factor_with_retry(H, percdamp)
    ops.pack_upper(U, 1.0, out=t["U"])
    t["info"].copy_(info)
    t["damps"].fill_(float(percdamp))
    bundle.U = U
    return H, U, damps


def fasterquant_rows(objs, blocksize=128, percdamp=0.01, groupsize=-1, actorder=False,
                     static_groups=False, export_compressed_tensors=False, backend="torch",
                     graph=False, streams=4, marks=None):
    """``fasterquant`` of every GPTQ object in ``objs`` (the same list on every
    rank, calibrated on each rank's token shard) with the work split over
    all ranks.  On return every rank holds every layer's quantized weights,
    export buffers and quantizer parameters, as after ``fasterquant`` on a
    single GPU with the summed statistics.  ``backend`` and ``graph`` are
    accepted and ignored.

    The distinct Hessian with the largest factorization is factored on rank 0
    and broadcast; the rows of the layers that use it are split over all
    ranks.  Every other distinct Hessian goes whole to one of the other ranks
    (LPT over its factorization and compensation work), so that their work
    overlaps the large factorization.  A failed factorization is re-done
    with the damp auto-increment after the row work (collectively for the
    shared one).

    ``marks`` (optional list) receives ``(phase, CUDA event)`` pairs at the end
    of the reduce, the factorizations + row work, and the gather."""
    if not objs:
        return
    if export_compressed_tensors and actorder and not (groupsize == -1 or static_groups):
        raise AssertionError("Scales in the same quantization group should be the same.")
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = objs[0].dev
    cur = torch.cuda.current_stream(dev)
    rows_of = {o: row_ranges(o.rows, world)[rank] for o in objs}
    args = (blocksize, groupsize, actorder, static_groups, export_compressed_tensors)
    with contextlib.ExitStack() as onloaded:
        for o in objs:
            onloaded.enter_context(o._maybe_onload_hessian())
        for o in objs:
            o._flush_all()
        rep = _distinct(objs)
        distinct = [o for o in objs if rep[o] is o]
        for o in objs:
            o._leave_groups()

        # 0. the plan: the distinct Hessian with the largest factorization is
        # factored on rank 0 and its rows are sharded over all ranks; every
        # other one goes whole (factor and rows) to one of the other ranks by
        # LPT over its factorization and compensation work
        users = {o: [u for u in objs if rep[u] is o] for o in distinct}
        fcost = {o: o.num_layers * o.columns ** 3 for o in distinct}
        ccost = {o: sum(u.num_layers * u.rows * u.columns ** 2 for u in users[o])
                 for o in distinct}
        big = max(distinct, key=lambda o: fcost[o]) if world > 1 else None
        rest = [o for o in distinct if o is not big]
        owner = {}
        if big is not None:
            owner[big] = 0
        if rest:
            others = world - 1 if world > 1 else 1
            _, _, placed = greedy_bin_packing(rest, others, lambda o: fcost[o] + ccost[o])
            for o in rest:
                owner[o] = placed[o] + (1 if world > 1 else 0)
        rows_of = {}
        for o in distinct:
            for u in users[o]:
                if o is big:
                    rows_of[u] = row_ranges(u.rows, world)[rank]
                else:  # whole on its owner; slices in rank order for the gather
                    rows_of[u] = ((0, u.rows) if rank == owner[o] else
                                  (0, 0) if rank < owner[o] else (u.rows, u.rows))

        # 1. statistics of the distinct Hessians to their factor owners
        local = [list(o._n) for o in distinct]
        glob = collectives.sum_counts(local, dev)
        entries = []
        for o, loc, gl in zip(distinct, local, glob):
            for b in range(o.num_layers):
                if gl[b] == 0:
                    o._H[b].zero_()
                else:
                    entries.append(collectives.Entry(owner[o], o._H[b], symmetric=True,
                                                     weight=loc[b] / gl[b]))
        collectives.reduce_to_owners(entries, dev)
        _mark(marks, "reduce", dev)

        # 2. The large factorization (the critical path) and its broadcast run
        # on the pool's high-priority stream; whole objects run factor-then-rows
        # on the other streams of their owner; the shared rows of the large one
        # wait for its broadcast on their own stream, never on the host.
        pool = _engine.stream_pool(dev, max(2, streams))
        fs, row_streams = pool[0], pool[1:]
        for s in pool:
            s.wait_stream(cur)
        bundles, retry_state, work = {}, {}, {}
        n_launched = 0
        for o in distinct:
            bundles[o] = _FactorBundle(o.num_layers, o.columns, actorder, dev)
        if big is not None:
            bundle = bundles[big]
            with torch.cuda.stream(fs):
                if rank == owner[big]:
                    retry_state[big] = _factor_on_owner(big, bundle, percdamp, actorder)
                _mark(marks, "big_factor", dev)
                done = dist.broadcast(bundle.buf, src=owner[big], async_op=True)
        for o in sorted(rest, key=lambda o: -(fcost[o] + ccost[o])):
            if owner[o] != rank:
                for u in users[o]:
                    work[u] = _Rows(u, None, bundles[o].t, *rows_of[u], *args)
                continue
            s = row_streams[n_launched % len(row_streams)]
            n_launched += 1
            with torch.cuda.stream(s):
                retry_state[o] = _factor_on_owner(o, bundles[o], percdamp, actorder)
                for u in users[o]:
                    work[u] = _Rows(u, bundles[o].U, bundles[o].t, *rows_of[u], *args)
        n_first_big = n_launched
        if big is not None:
            bundle = bundles[big]
            for u in sorted(users[big], key=lambda u: -u.rows):
                s = row_streams[n_launched % len(row_streams)]
                n_launched += 1
                with torch.cuda.stream(s):
                    done.wait()  # this stream waits for the broadcast, not the host
                    if n_launched == n_first_big + 1:
                        _mark(marks, "big_received", dev)
                    if bundle.U is None:
                        B, C = bundle.B, bundle.C
                        bundle.U = ops.unpack_upper(
                            torch.empty(B, C, C, dtype=torch.float32, device=dev),
                            bundle.t["U"], mirror=False)
                    work[u] = _Rows(u, bundle.U, bundle.t, *rows_of[u], *args)
        for s in pool:
            cur.wait_stream(s)

        # a failed factorization: its owner retries with the damp increment and
        # re-runs the rows that used it; for the shared factor the retry is
        # collective (its status words reached every rank with the broadcast)
        mine = [o for o in distinct if o is big or owner[o] == rank]
        infos = _engine.sync_check(*[bundles[o].t["info"] for o in mine])
        k, failed = 0, []
        for o in mine:
            codes = infos[k:k + o.num_layers]
            k += o.num_layers
            _engine.raise_device_errors(codes, [], timeouts_only=True)
            if any(codes):
                failed.append((o, codes))
        for o, codes in failed:
            bundle = bundles[o]
            if owner[o] == rank:
                H, U, damps = retry_state[o]
                _engine.retry_failed(H, U, codes, damps)
                ops.pack_upper(U, 1.0, out=bundle.t["U"])
                bundle.t["damps"].copy_(torch.tensor(damps, dtype=torch.float32))
                bundle.t["info"].zero_()
            if o is big:
                dist.broadcast(bundle.buf, src=owner[o])
                if owner[o] != rank:
                    ops.unpack_upper(bundle.U, bundle.t["U"], mirror=False)
            for u in users[o]:
                work[u] = _Rows(u, bundle.U, bundle.t, *rows_of[u], *args)
        for o in objs:
            o._H = None
        retry_state.clear()
    _mark(marks, "factor_and_compensate", dev)

    # errors on any rank stop every rank before the gather
    flat = _engine.sync_check(ops.device_status(dev),
                              *[f for o in objs for f in work[o].flags()])
    nan, bad = 0, 0
    timeout = int(flat[0] == _lib.G2Q_ERR_TIMEOUT)
    k = 1
    for o in objs:
        vals = flat[k:k + len(work[o].flags())]
        k += len(vals)
        nan |= int(vals[0] != 0)
        for s in vals[1:]:
            if s == _lib.G2Q_ERR_TIMEOUT:
                timeout = 1
            elif s != 0:
                bad = 1
    err = torch.tensor([nan, timeout, bad], dtype=torch.int32).to(dev)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    nan, timeout, bad = err.cpu().tolist()
    if timeout:
        raise RuntimeError("g2ptq_b200: a tensor-core pipeline wait timed out "
                           f"({_lib.status_string(_lib.G2Q_ERR_TIMEOUT)})")
    if bad:
        raise RuntimeError("WeightQuantizer.find_params: non-positive scale")
    if nan:
        raise ValueError("NaN in weights")

    # 4. every slice to every rank
    pieces, full_params, staged = [], {}, {}
    for o in objs:
        w = work[o]
        B, R, C = o.num_layers, o.rows, o.columns
        ng = len(o.quantizer)
        fs = torch.empty(B * R, ng, dtype=torch.float32, device=dev)
        fz = torch.empty_like(fs)
        full_params[o] = (fs, fz)
        bits = o.quantizer[0].bits
        for b, layer in enumerate(o.layers):
            pieces.append((w.outs[b] if w.n else layer.weight.data[:0], layer.weight.data))
            pieces.append((w.params.scale.view(B, w.n, ng)[b], fs.view(B, R, ng)[b]))
            pieces.append((w.params.zero.view(B, w.n, ng)[b], fz.view(B, R, ng)[b]))
            if export_compressed_tensors:
                shapes = export_shapes(bits, ng if groupsize != -1 else 1, layer)
                qp = {k: torch.empty(shape, dtype=dt, device=dev)
                      for k, (shape, dt) in shapes.items()}
                qp["weight_shape"][0], qp["weight_shape"][1] = R, C
                pieces.append((w.packed[b] if w.n else qp["weight_packed"][:0],
                               qp["weight_packed"]))
                pieces.append((w.gscale[b] if w.n else qp["weight_scale"][:0],
                               qp["weight_scale"]))
                staged[(o, b)] = qp
    # the damps of every factorization, from its owner (one small exchange)
    collectives.broadcast_from_owners(
        [collectives.Entry(owner[o], bundles[o].t["damps"]) for o in distinct if o is not big],
        dev)
    damps_of = {o: bundles[o].t["damps"].tolist() for o in distinct}
    collectives.all_gather_rows(pieces, dev)
    _mark(marks, "gather", dev)
    for o in objs:
        fs, fz = full_params[o]
        for i, q in enumerate(o.quantizer):
            q.scale, q.zero = fs[:, i:i + 1], fz[:, i:i + 1]
            q._ready = True
        for b, layer in enumerate(o.layers):
            if export_compressed_tensors:
                layer._export_qparams = staged[(o, b)]
        o._last_damps = damps_of[rep[o]]
        o._stages = None
