"""Coalesced NCCL exchanges of the quantizer objects' statistics and results.

The reference moves every tensor of every object in its own collective: per
object a count ``all_reduce`` and a blocking host read, then one ``reduce``
per Hessian, gradient and activation statistic (gptq_utils.py:362-391,
g2ptq_utils.py:530-575, gptaq_utils.py:402-439, gptq_guided_utils.py:222-249),
and after quantization one ``broadcast`` per tensor plus a pickled metadata
broadcast per object (common_utils.py:96-165).

Here one step exchanges each kind of data once per destination rank:

* ``sum_counts``: every object's per-layer counters in one int64
  ``all_reduce`` and one host read;
* ``reduce_to_owners``: all tensors bound for one rank packed into one fp32
  buffer -- symmetric matrices by their upper triangle (half the bytes), each
  tensor multiplied by its sample-share weight on the way in -- and summed
  there by one ``reduce``; the owner unpacks in place;
* ``broadcast_from_owners``: all tensors one rank produced, packed into one
  byte buffer per source rank and broadcast once; every rank knows the
  shapes in advance, so nothing is pickled;
* ``all_gather_rows``: row slices computed on every rank assembled into full
  tensors everywhere with one ``all_gather``.

Every rank must call these with the same entries in the same order.  The
packing of symmetric matrices runs in this library's kernels
(``ops.pack_upper`` / ``ops.unpack_upper``, bound below as ``pack_upper`` /
``unpack_upper``); tests of the host logic on gloo ranks rebind them to CPU
stand-ins inside their rank processes.
"""

from collections import defaultdict
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops

pack_upper = ops.pack_upper
unpack_upper = ops.unpack_upper


def sum_counts(counts, device):
    """``counts``: a list of per-object lists of ints.  Returns the same
    structure summed over ranks (one all_reduce, one device-to-host read)."""
    flat = [int(c) for cs in counts for c in cs]
    if not flat:
        return [[] for _ in counts]
    t = torch.tensor(flat, dtype=torch.int64).to(device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    summed = t.cpu().tolist()
    out, k = [], 0
    for cs in counts:
        out.append(summed[k:k + len(cs)])
        k += len(cs)
    return out


@dataclass
class Entry:
    """One tensor of a coalesced exchange.  ``symmetric``: ``t`` is ``[C, C]``
    (or ``[B, C, C]``) symmetric and travels as its upper triangle."""
    rank: int
    t: torch.Tensor
    symmetric: bool = False
    weight: float = 1.0

    def numel(self):
        if self.symmetric:
            C = self.t.shape[-1]
            return self.t.numel() // (C * C) * (C * (C + 1) // 2)
        return self.t.numel()


def _by_rank(entries):
    groups = defaultdict(list)
    for e in entries:
        groups[e.rank].append(e)
    return [(r, groups[r]) for r in sorted(groups)]


def reduce_to_owners(entries, device):
    """Sum ``weight * t`` over ranks into ``t`` on ``rank`` for every entry,
    one fp32 ``reduce`` per destination rank.  Tensors of the other ranks are
    left as they were (their objects are freed next)."""
    me = dist.get_rank()
    launched = []
    for dst, es in _by_rank(entries):
        buf = torch.empty(sum(e.numel() for e in es), dtype=torch.float32, device=device)
        off = 0
        for e in es:
            n = e.numel()
            if e.symmetric:
                pack_upper(e.t, e.weight, out=buf[off:off + n])
            else:
                torch.mul(e.t.reshape(-1).float(), e.weight, out=buf[off:off + n])
            off += n
        launched.append((dst, es, buf, dist.reduce(buf, dst=dst, async_op=True)))
    for dst, es, buf, work in launched:
        work.wait()
        if dst != me:
            continue
        off = 0
        for e in es:
            n = e.numel()
            if e.symmetric:
                unpack_upper(e.t, buf[off:off + n])
            else:
                e.t.copy_(buf[off:off + n].view(e.t.shape))
            off += n


def _bytes(t):
    return t.contiguous().view(-1).view(torch.uint8)


def _dest_bytes(t):
    """A contiguous destination tensor as a flat byte view of its storage."""
    if not t.is_contiguous():
        raise ValueError("collectives: destination tensors must be contiguous")
    return t.view(-1).view(torch.uint8)


def broadcast_from_owners(entries, device):
    """Copy every entry's tensor from its ``rank`` into the same tensor on all
    other ranks: one byte buffer and one ``broadcast`` per source rank.
    Entries must have the same shapes and dtypes on every rank."""
    me = dist.get_rank()
    launched = []
    for src, es in _by_rank(entries):
        sizes = [e.t.numel() * e.t.element_size() for e in es]
        if me == src:
            buf = torch.cat([_bytes(e.t) for e in es])
        else:
            buf = torch.empty(sum(sizes), dtype=torch.uint8, device=device)
        launched.append((src, es, sizes, buf, dist.broadcast(buf, src=src, async_op=True)))
    for src, es, sizes, buf, work in launched:
        work.wait()
        if src == me:
            continue
        off = 0
        for e, n in zip(es, sizes):
            # bytes into the destination seen as bytes: a slice of the buffer
            # need not be aligned for the destination's element type
            _dest_bytes(e.t).copy_(buf[off:off + n])
            off += n


def all_gather_rows(pieces, device):
    """``pieces``: this rank's list of ``(tensor, full)`` pairs, where
    ``tensor`` is this rank's contiguous slice of the contiguous ``full`` along
    dim 0 (same list structure on every rank, slices of any sizes, rank r's
    slice before rank r + 1's).  Every rank ends with every ``full`` assembled,
    through one ``all_gather`` of one byte buffer per rank (padded to the
    largest rank's) and one small ``all_gather`` of the slice sizes."""
    world = dist.get_world_size()
    me = dist.get_rank()
    for _, full in pieces:
        if not full.is_contiguous():
            raise ValueError("all_gather_rows: full tensors must be contiguous")
    mine = [_bytes(t) for t, _ in pieces]
    sizes = torch.tensor([sum(b.numel() for b in mine)] +
                         [b.numel() for b in mine], dtype=torch.int64).to(device)
    table = [torch.empty_like(sizes) for _ in range(world)]
    dist.all_gather(table, sizes)
    table = [t.cpu().tolist() for t in table]
    width = max(1, max(t[0] for t in table))
    send = torch.zeros(width, dtype=torch.uint8, device=device)
    if table[me][0]:
        send[:table[me][0]] = torch.cat(mine)
    recv = torch.empty(world * width, dtype=torch.uint8, device=device)
    dist.all_gather_into_tensor(recv, send)
    for k, (_, full) in enumerate(pieces):
        dst = _dest_bytes(full)
        pos = 0
        for r in range(world):
            off = sum(table[r][1:1 + k])
            n = table[r][1 + k]
            dst[pos:pos + n].copy_(recv[r * width + off:r * width + off + n])
            pos += n
        if pos != dst.numel():
            raise ValueError("all_gather_rows: slices do not cover the full tensor")


def reduce_objects(objs, owner_of, counts_fn, entries_fn, commit_fn, onload_fn):
    """The statistics exchange of ``reduce_to_target_rank`` for quantizer
    objects of one method.

    ``counts_fn(obj)``: the object's host counters (one list of ints);
    ``entries_fn(obj, local, global_, owner)``: the ``Entry`` list of its
    statistics, weighted by their sample shares (it also clears layers that
    no rank saw); ``commit_fn(obj, global_)``: the owner's counters after the
    sum; ``onload_fn(obj)``: the object's onload context.  Objects whose
    statistics live on the device go through one coalesced exchange; objects
    with offloaded statistics go one at a time inside their onload context."""
    if not objs:
        return
    dev = objs[0].dev
    local = [counts_fn(o) for o in objs]
    glob = sum_counts(local, dev)
    resident = [k for k, o in enumerate(objs) if not getattr(o, "offload_hessians", False)]
    entries = []
    for k in resident:
        entries += entries_fn(objs[k], local[k], glob[k], owner_of[objs[k]])
    reduce_to_owners(entries, dev)
    for k, o in enumerate(objs):
        if k in resident:
            continue
        with onload_fn(o):
            reduce_to_owners(entries_fn(o, local[k], glob[k], owner_of[o]), dev)
    me = dist.get_rank()
    for k, o in enumerate(objs):
        if owner_of[o] == me:
            commit_fn(o, glob[k])
