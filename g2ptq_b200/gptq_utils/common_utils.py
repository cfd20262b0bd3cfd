"""Layer batching, owner assignment and result broadcast, mirroring
gptq_utils/common_utils.py of the reference (same names and semantics).

``greedy_bin_packing`` restates ``compressed_tensors.distributed.greedy_bin_packing``
(compressed-tensors 0.18.0, which the reference calls from ``partition_layers``,
common_utils.py:88-93): longest-processing-time-first, heaviest item to the
least-loaded bin, lowest bin index on ties.
"""

import copy
from collections import defaultdict
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..utils import compressed_tensors_utils


def make_group_quantizers(quantizer, columns, groupsize):
    """common_utils.py:13-16: one independent quantizer per weight group."""
    num_groups = 1 if groupsize == -1 else (columns + groupsize - 1) // groupsize
    return [copy.deepcopy(quantizer) for _ in range(num_groups)]


def merge_group_quantizers(quantizers, start, end, groupsize):
    """common_utils.py:19-30: one per-layer quantizer from a batched group list."""
    result = copy.deepcopy(quantizers[0])
    result.scale = torch.cat([q.scale[start:end].reshape(end - start, -1) for q in quantizers],
                             dim=1).clone()
    result.zero = torch.cat([q.zero[start:end].reshape(end - start, -1) for q in quantizers],
                            dim=1).clone()
    result.weight_groupsize = groupsize
    result._ready = all(q.ready() for q in quantizers)
    return result


def fake_quantize_grouped(quantizers, weight, groupsize):
    """common_utils.py:33-45."""
    flat_rows = weight.shape[0] * weight.shape[1]
    width = weight.shape[-1] if groupsize == -1 else groupsize
    out = []
    for group, quantizer in enumerate(quantizers):
        start = group * width
        end = min(start + width, weight.shape[-1])
        values = weight[:, :, start:end]
        q = quantizer.fake_quantize(values.reshape(flat_rows, end - start))[0]
        out.append(q.reshape(*weight.shape[:2], end - start))
    return torch.cat(out, dim=-1)


@dataclass(eq=False)
class ChunkSpec:
    """A batch of same-shaped modules quantized by one quantizer instance."""
    chunk_names: tuple
    rows: int
    columns: int

    @property
    def num_layers(self):
        return len(self.chunk_names)


def build_chunk_specs(subset, layer_bsz, group_key_fn=None):
    """common_utils.py:60-85."""
    groups = defaultdict(list)
    for name, module in subset.items():
        key = module.weight.shape
        if group_key_fn is not None:
            key = (key, group_key_fn(name))
        groups[key].append(name)
    specs = []
    for group_names in groups.values():
        rows, columns = subset[group_names[0]].weight.shape
        for s in range(0, len(group_names), layer_bsz):
            specs.append(ChunkSpec(tuple(group_names[s:s + layer_bsz]), rows, columns))
    return specs


def greedy_bin_packing(items, num_bins, item_weight_fn):
    """LPT packing -> ``(items ordered by weight, {bin: [items]}, {item: bin})``."""
    order = sorted(range(len(items)), key=lambda i: -item_weight_fn(items[i]))
    load = [0] * num_bins
    bin2items = {b: [] for b in range(num_bins)}
    item2bin = {}
    ordered = []
    for i in order:
        b = min(range(num_bins), key=lambda k: (load[k], k))
        load[b] += item_weight_fn(items[i])
        bin2items[b].append(items[i])
        item2bin[items[i]] = b
        ordered.append(items[i])
    return ordered, bin2items, item2bin


def partition_layers(gptqs, world_size):
    """common_utils.py:88-93."""
    return greedy_bin_packing(
        gptqs, world_size,
        item_weight_fn=lambda g: g.num_layers * g.rows * g.columns)


def broadcast_quantized_param(gptqs, gptq2rank, export_compressed_tensors=False):
    """common_utils.py:96-165: refresh every rank's weights (and export qparams)
    from the rank that quantized them."""
    shared_qparams = ["weight"]
    export_qparams = (list(compressed_tensors_utils.Q_PARAMS)
                      if export_compressed_tensors else [])
    rank = dist.get_rank()
    dist.barrier()
    pending = []
    for gptq in gptqs:
        src = gptq2rank[gptq]
        for b in range(gptq.num_layers):
            layer = gptq.layers[b]
            for attr in shared_qparams:
                pending.append(dist.broadcast(getattr(layer, attr).data, src=src,
                                              async_op=True))
    if not export_qparams:
        for w in pending:
            w.wait()
        dist.barrier()
        return {}
    broadcasted = {}
    for gptq in gptqs:
        src = gptq2rank[gptq]
        meta_list = [None]
        if rank == src:
            metas = []
            for b in range(gptq.num_layers):
                qp = gptq.layers[b].__dict__.get("_export_qparams", None)
                metas.append(None if qp is None else
                             {a: {"shape": tuple(t.shape), "dtype": t.dtype}
                              for a, t in qp.items()})
            meta_list = [metas]
        dist.broadcast_object_list(meta_list, src=src)
        metas = meta_list[0]
        dev = gptq.layers[0].weight.device
        for b in range(gptq.num_layers):
            layer = gptq.layers[b]
            meta = metas[b]
            if meta is None:
                continue
            if rank == src:
                qp = {a: t.detach().to(dev) for a, t in layer._export_qparams.items()}
            else:
                qp = {a: torch.empty(m["shape"], dtype=m["dtype"], device=dev)
                      for a, m in meta.items()}
            for attr in export_qparams:
                pending.append(dist.broadcast(qp[attr], src=src, async_op=True))
            layer._export_qparams = qp
            broadcasted[(id(gptq), b)] = qp
    for w in pending:
        w.wait()
    dist.barrier()
    return broadcasted
