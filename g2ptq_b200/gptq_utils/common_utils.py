"""Layer batching, owner assignment and the hand-over of quantized results --
the names and semantics of the reference's gptq_utils/common_utils.py
(make_group_quantizers :13-16, merge_group_quantizers :19-30,
fake_quantize_grouped :33-45, ChunkSpec / build_chunk_specs :48-85,
partition_layers :88-93, broadcast_quantized_param :96-165), built here
around device-side parameter matrices and coalesced collectives.

``greedy_bin_packing`` restates ``compressed_tensors.distributed.greedy_bin_packing``
(compressed-tensors 0.18.0, called by ``partition_layers``): items by
decreasing weight, each to the currently least-loaded bin, the lowest bin
index winning ties.
"""

import copy
import heapq

import torch
import torch.distributed as dist

from .. import ops
from ..utils import compressed_tensors_utils
from . import collectives


def make_group_quantizers(quantizer, columns, groupsize):
    """One independent copy of ``quantizer`` per weight group (a single one
    for ``groupsize == -1``)."""
    count = 1 if groupsize == -1 else -(-columns // groupsize)
    return [copy.deepcopy(quantizer) for _ in range(count)]


def merge_group_quantizers(quantizers, start, end, groupsize):
    """A single quantizer for rows ``[start, end)`` of a batched group list:
    its ``scale`` / ``zero`` hold one column block per group, group g's rows
    in block g."""
    n = end - start
    blocks_s = [q.scale[start:end].reshape(n, -1) for q in quantizers]
    blocks_z = [q.zero[start:end].reshape(n, -1) for q in quantizers]
    width = sum(b.shape[1] for b in blocks_s)
    ref = blocks_s[0]
    scale = torch.empty(n, width, dtype=ref.dtype, device=ref.device)
    zero = torch.empty(n, width, dtype=blocks_z[0].dtype, device=ref.device)
    col = 0
    for bs, bz in zip(blocks_s, blocks_z):
        w = bs.shape[1]
        scale[:, col:col + w] = bs
        zero[:, col:col + w] = bz
        col += w
    merged = copy.deepcopy(quantizers[0])
    merged.scale, merged.zero = scale, zero
    merged.weight_groupsize = groupsize
    merged._ready = all(q.ready() for q in quantizers)
    return merged


def fake_quantize_grouped(quantizers, weight, groupsize):
    """Quantize-dequantize ``weight [B, R, C]`` with quantizer ``c // groupsize``
    on column c (one quantizer for all columns when ``groupsize == -1``).

    The groups' per-row parameters are gathered into one ``[B*R, groups]``
    matrix and the whole weight goes through a single kernel launch, which
    performs each element's quantization exactly as the group's own
    ``fake_quantize`` would (same quotient, rounding and clamp)."""
    B, R, C = weight.shape
    flat = weight.reshape(B * R, C).float().contiguous()
    q0 = quantizers[0]
    if groupsize == -1:
        return q0.fake_quantize(flat)[0].reshape(B, R, C)
    if any(q.maxq != q0.maxq or not q.ready() for q in quantizers):
        raise ValueError("fake_quantize_grouped: quantizers must be ready and share a bit width")
    scale = torch.stack([q.scale.reshape(-1) for q in quantizers], dim=1).float().contiguous()
    zero = torch.stack([q.zero.reshape(-1) for q in quantizers], dim=1).float().contiguous()
    colmap = (torch.arange(C, device=weight.device, dtype=torch.int32) // groupsize)
    out, _ = ops.fake_quantize(flat, scale, zero, q0.maxq, colmap=colmap)
    return out.reshape(B, R, C).to(weight.dtype)


class ChunkSpec:
    """A batch of same-shaped modules that one quantizer object handles."""

    __slots__ = ("chunk_names", "rows", "columns")

    def __init__(self, chunk_names, rows, columns):
        self.chunk_names = tuple(chunk_names)
        self.rows = rows
        self.columns = columns

    @property
    def num_layers(self):
        return len(self.chunk_names)

    def __repr__(self):
        return f"ChunkSpec({self.chunk_names}, rows={self.rows}, columns={self.columns})"


def build_chunk_specs(subset, layer_bsz, group_key_fn=None):
    """Modules of ``subset`` (name -> module) grouped by weight shape (and
    ``group_key_fn(name)`` when given), in order of first appearance, each
    group cut into chunks of at most ``layer_bsz`` names."""
    order = {}
    for name, module in subset.items():
        key = tuple(module.weight.shape)
        if group_key_fn is not None:
            key = (key, group_key_fn(name))
        order.setdefault(key, []).append(name)
    specs = []
    for names in order.values():
        rows, columns = subset[names[0]].weight.shape
        specs.extend(ChunkSpec(names[i:i + layer_bsz], rows, columns)
                     for i in range(0, len(names), layer_bsz))
    return specs


def greedy_bin_packing(items, num_bins, item_weight_fn):
    """Longest-processing-time packing -> ``(items by decreasing weight,
    {bin: [items]}, {item: bin})``."""
    weights = [item_weight_fn(it) for it in items]
    ranked = sorted(range(len(items)), key=lambda i: -weights[i])  # stable on ties
    heap = [(0, b) for b in range(num_bins)]  # (load, bin): least load, then lowest index
    bins = {b: [] for b in range(num_bins)}
    owner = {}
    for i in ranked:
        load, b = heapq.heappop(heap)
        bins[b].append(items[i])
        owner[items[i]] = b
        heapq.heappush(heap, (load + weights[i], b))
    return [items[i] for i in ranked], bins, owner


def partition_layers(gptqs, world_size):
    """Owner ranks of quantizer objects by LPT over ``num_layers * rows * columns``."""
    return greedy_bin_packing(gptqs, world_size,
                              lambda g: g.num_layers * g.rows * g.columns)


def export_shapes(bits, groups, layer):
    """Shapes and dtypes of the staged compressed-tensors buffers of one
    layer (``compressed_tensors_utils.compress_grouped``), known from the
    quantizer configuration on every rank."""
    rows, cols = layer.weight.shape
    return {"weight_packed": ((rows, -(-cols // (32 // bits))), torch.int32),
            "weight_scale": ((rows, groups), layer.weight.dtype),
            "weight_shape": ((layer.weight.dim(),), torch.long)}


def broadcast_quantized_param(gptqs, gptq2rank, export_compressed_tensors=False):
    """Give every rank the weights (and, with export, the staged
    compressed-tensors buffers) of the layers each owner rank quantized.

    One byte buffer per owner rank is broadcast once; non-owners allocate the
    export buffers from the shapes their own copy of the object implies.
    Returns ``{(id(gptq), b): export buffers}`` for the layers that have them."""
    rank = dist.get_rank()
    entries = []
    staged = {}
    for gptq in gptqs:
        src = gptq2rank[gptq]
        for b, layer in enumerate(gptq.layers):
            entries.append(collectives.Entry(src, layer.weight.data))
            if not export_compressed_tensors:
                continue
            if rank == src:
                qp = layer.__dict__.get("_export_qparams")
                if qp is None:
                    raise RuntimeError("broadcast_quantized_param: the owner staged no export "
                                       "buffers (fasterquant without export_compressed_tensors)")
                qp = {k: v.to(layer.weight.device) for k, v in qp.items()}
            else:
                shapes = export_shapes(gptq.quantizer[0].bits, len(gptq.quantizer), layer)
                qp = {k: torch.empty(shape, dtype=dt, device=layer.weight.device)
                      for k, (shape, dt) in shapes.items()}
            layer._export_qparams = qp
            staged[(id(gptq), b)] = qp
            for name in compressed_tensors_utils.Q_PARAMS:
                entries.append(collectives.Entry(src, qp[name]))
    dev = gptqs[0].layers[0].weight.device if gptqs else torch.device("cpu")
    collectives.broadcast_from_owners(entries, dev)
    return staged
