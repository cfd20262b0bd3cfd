"""The layer-by-layer calibration pass of the reference's ``gptq_fwrd``
(gptq_utils/gptq_utils.py:395-595; G2PTQ: g2ptq_utils.py:1098-1653, with
its gradients synthesised) for Llama-style decoder layers.

The reference quantizes a layer's linears in its sequential groups --
[q, k, v], [o], [up, gate], [down] (utils/models/base.py ATTN_GROUPS /
MLP_GROUPS) -- running a whole forward of the layer over the calibration set
for each group with forward hooks calling ``add_batch`` (the earlier groups
already quantized), and one more forward to propagate the layer's output to
the next layer: five forwards per layer.

Here each group's inputs are computed incrementally and kept in HBM:
``input_layernorm(x)`` for [q, k, v]; the attention output with the quantized
q/k/v for [o]; ``post_attention_layernorm(x + o(attn))`` with the quantized o
for [up, gate]; ``act(gate(h)) * up(h)`` with the quantized gate/up for
[down]; and ``h1 + down(mlp_in)`` as the next layer's input.  These are the
layer's own modules applied in the order its forward applies them, so every
group sees exactly what the reference's hooks see, at the cost of about one
forward per layer.

With a process group the calibration set is split by sequences over the
ranks (the reference's ``main.py:32-37``); after each group's statistics are
reduced the quantized weights are handed to every rank before the next
stage, through the owner flow (``reduce_to_target_rank`` + owner
``fasterquant`` + ``broadcast_quantized_param``) or the row-sharded
``sharded.fasterquant_rows``.
"""

import time

import torch
import torch.distributed as dist

from .common_utils import (broadcast_quantized_param, build_chunk_specs, make_group_quantizers,
                           partition_layers)
from . import gptq_utils, g2ptq_utils
from .. import ops
from ..utils.quant_utils import WeightQuantizer

SEQUENTIAL_GROUPS = (("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"),
                     ("self_attn.o_proj",),
                     ("mlp.up_proj", "mlp.gate_proj"),
                     ("mlp.down_proj",))


def _module(layer, name):
    m = layer
    for part in name.split("."):
        m = getattr(m, part)
    return m


class Calibration:
    """Settings of one pass (the reference's ``process_args.py`` names)."""

    def __init__(self, method="gptq", w_bits=4, w_asym=False, w_groupsize=128, act_order=True,
                 percdamp=0.01, blocksize=128, layer_bsz=1, export_compressed_tensors=False,
                 num_groups=4, alpha=1.0, enable_gradient_update=True, grad_std=1e-3,
                 grad_seed=44, multi="owner", bsz=8):
        self.method = method
        self.w_bits, self.w_asym, self.w_groupsize = w_bits, w_asym, w_groupsize
        self.act_order, self.percdamp, self.blocksize = act_order, percdamp, blocksize
        self.layer_bsz = layer_bsz
        self.export = export_compressed_tensors
        self.num_groups, self.alpha = num_groups, alpha
        self.enable_gradient_update = enable_gradient_update
        self.grad_std, self.grad_seed = grad_std, grad_seed
        self.multi = multi
        self.bsz = bsz  # sequences per forward batch (the add_batch calls stay per batch)


def _world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def _synthetic_g2ptq_inputs(cal, names, subset, stage_inputs, layer_idx):
    """G2PTQ's saliencies and weight gradients from synthetic per-token output
    gradients N(0, grad_std) BF16 [tokens, rows] of every linear (the stand-in
    for the refresh step's backward): saliency s[n, g] = mean over the rows of
    group g of grad_out[n, r]^2, gradient = mean over batches of
    grad_out^T X / tokens (g2ptq_utils.py:605-618, 693-711)."""
    sal, grad = {}, {}
    for k, name in enumerate(names):
        lin = subset[name]
        rows = lin.weight.shape[0]
        G = cal.num_groups
        g = torch.Generator(device=lin.weight.device).manual_seed(
            cal.grad_seed + 1000 * layer_idx + k)
        acc = torch.zeros(rows, lin.weight.shape[1], device=lin.weight.device)
        sal[name] = []
        for x in stage_inputs:
            t = x.shape[0] * x.shape[1]
            go = (torch.randn(t, rows, device=x.device, generator=g) * cal.grad_std).to(
                torch.bfloat16)
            # what SaliencyCache.grad_hook computes from the output gradient
            sal[name].append(ops.saliency(go, G))
            acc += (go.T @ x.reshape(t, -1)).float() / t
        grad[name] = acc / max(1, len(stage_inputs))
    return sal, grad


def _quantize_group(cal, layer, names, stage_inputs, layer_idx):
    """Build the group's quantizer objects (chunks of ``layer_bsz`` same-shape
    linears), feed every stage batch to ``add_batch``, reduce over ranks and
    quantize; on return every rank's linears hold the quantized weights."""
    world, rank = _world()
    subset = {n: _module(layer, n) for n in names}
    specs = build_chunk_specs(subset, cal.layer_bsz)
    g2 = cal.method == "g2ptq"
    if g2:
        sal, grad = _synthetic_g2ptq_inputs(cal, names, subset, stage_inputs, layer_idx)
    objs = []
    for spec in specs:
        mods = [subset[n] for n in spec.chunk_names]
        if g2:
            obj = g2ptq_utils.G2PTQ(mods, [list(sal[n]) for n in spec.chunk_names],
                                    [grad[n] for n in spec.chunk_names],
                                    num_groups=cal.num_groups)
        else:
            obj = gptq_utils.GPTQ(mods)
        q = WeightQuantizer()
        q.configure(cal.w_bits, perchannel=True, sym=not cal.w_asym, mse=False)
        obj.quantizer = make_group_quantizers(q, spec.columns, cal.w_groupsize)
        objs.append(obj)
    for x in stage_inputs:
        for obj in objs:
            for idx in range(obj.num_layers):
                obj.add_batch(idx, x, None)
    kw = dict(blocksize=cal.blocksize, percdamp=cal.percdamp, groupsize=cal.w_groupsize,
              actorder=cal.act_order, static_groups=cal.act_order,
              export_compressed_tensors=cal.export)
    if g2:
        kw.update(enable_gradient_update=cal.enable_gradient_update, alpha=cal.alpha)
    if world == 1:
        gptq_utils.fasterquant_all(objs, **kw)
    elif cal.multi == "rows" and not g2:
        from . import sharded
        sharded.fasterquant_rows(objs, **kw)
    else:
        mod = g2ptq_utils if g2 else gptq_utils
        _, _, owner = partition_layers(objs, world)
        mod.reduce_to_target_rank(objs, owner)
        gptq_utils.fasterquant_all([o for o in objs if owner[o] == rank], **kw)
        broadcast_quantized_param(objs, owner, export_compressed_tensors=cal.export)
    for o in objs:
        o.free()


@torch.no_grad()
def calibrate_layer(cal, layer, inps, position_embeddings, layer_idx=0, times=None):
    """Quantize one decoder layer on this rank's calibration batches ``inps``
    (a list of ``[bsz, S, hidden]`` tensors) and replace each of them, in place,
    by the layer's output with the quantized weights."""
    t = times if times is not None else {}

    def tick(key, t0):
        torch.cuda.synchronize()
        t[key] = t.get(key, 0.0) + time.perf_counter() - t0
        return time.perf_counter()

    t0 = time.perf_counter()
    # [q, k, v]: the normalised layer input
    normed = [layer.input_layernorm(x) for x in inps]
    t0 = tick("forward", t0)
    _quantize_group(cal, layer, SEQUENTIAL_GROUPS[0], normed, layer_idx)
    t0 = tick("quantize", t0)
    # [o]: the attention output with the quantized q / k / v
    attn_in = []
    hook = layer.self_attn.o_proj.register_forward_pre_hook(
        lambda m, args: attn_in.append(args[0]))
    try:
        for h in normed:
            layer.self_attn(hidden_states=h, position_embeddings=position_embeddings,
                            attention_mask=None)
    finally:
        hook.remove()
    del normed
    t0 = tick("forward", t0)
    _quantize_group(cal, layer, SEQUENTIAL_GROUPS[1], attn_in, layer_idx)
    t0 = tick("quantize", t0)
    # [up, gate]: the post-attention normalised residual with the quantized o
    resid, mlp_norm = [], []
    for x, a in zip(inps, attn_in):
        h1 = x + layer.self_attn.o_proj(a)
        resid.append(h1)
        mlp_norm.append(layer.post_attention_layernorm(h1))
    del attn_in
    t0 = tick("forward", t0)
    _quantize_group(cal, layer, SEQUENTIAL_GROUPS[2], mlp_norm, layer_idx)
    t0 = tick("quantize", t0)
    # [down]: the gated activation with the quantized gate / up
    mlp = layer.mlp
    mlp_in = [mlp.act_fn(mlp.gate_proj(h)) * mlp.up_proj(h) for h in mlp_norm]
    del mlp_norm
    t0 = tick("forward", t0)
    _quantize_group(cal, layer, SEQUENTIAL_GROUPS[3], mlp_in, layer_idx)
    t0 = tick("quantize", t0)
    # the layer's output with every linear quantized, in place
    for k, (h1, m) in enumerate(zip(resid, mlp_in)):
        inps[k].copy_(h1 + mlp.down_proj(m))
    tick("forward", t0)
    return t


def calibrate(cal, layers, inps, position_embeddings, on_layer=None):
    """All layers in order (``gptq_fwrd``'s loop); ``inps`` (this rank's
    batches) ends as the last layer's output.  Returns the seconds spent in
    the forwards and in the quantization."""
    times = {}
    for i, layer in enumerate(layers):
        calibrate_layer(cal, layer, inps, position_embeddings, i, times)
        if on_layer is not None:
            on_layer(i, times)
    return times
