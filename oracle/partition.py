"""Layer batching and owner assignment (pure Python).

``build_chunk_specs`` follows gptq_utils/common_utils.py:60-85.
``partition_layers`` (common_utils.py:88-93) calls
``compressed_tensors.distributed.greedy_bin_packing`` (compressed-tensors
0.18.0, pinned by the reference's requirements.txt:14; absent from the 0.15
copy installed here).  ``greedy_bin_packing`` restates its published
algorithm, longest-processing-time-first: order items by weight, heaviest
first, and give each to the bin with the least load so far (lowest bin index
on ties).  It only decides ownership; no numeric result depends on it.
"""

from collections import defaultdict


def build_chunk_specs(shapes, layer_bsz, group_key=None):
    """``shapes``: ordered ``{name: (rows, columns)}`` -> list of
    ``(chunk_names, rows, columns)``."""
    groups = defaultdict(list)
    for name, shape in shapes.items():
        key = tuple(shape)
        if group_key is not None:
            key = (key, group_key(name))
        groups[key].append(name)
    specs = []
    for names in groups.values():
        rows, cols = shapes[names[0]]
        for s in range(0, len(names), layer_bsz):
            specs.append((tuple(names[s:s + layer_bsz]), rows, cols))
    return specs


def greedy_bin_packing(items, num_bins, weight):
    order = sorted(range(len(items)), key=lambda i: -weight(items[i]))
    load = [0] * num_bins
    bin_items = {b: [] for b in range(num_bins)}
    item_bin = {}
    ordered = []
    for i in order:
        b = min(range(num_bins), key=lambda k: (load[k], k))
        load[b] += weight(items[i])
        bin_items[b].append(items[i])
        item_bin[i] = b
        ordered.append(items[i])
    return ordered, bin_items, [item_bin[i] for i in range(len(items))]
