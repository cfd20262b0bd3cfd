"""compressed-tensors export, mirroring utils/compressed_tensors_utils.py.

``compress`` has the reference's signature and checks; the int32 packing runs
in the ``g2q_pack_int32`` kernel (same bit layout as
``compressed_tensors.compressors.pack_to_int32``).  ``compress_grouped`` is the
direct path used by ``fasterquant``: it takes the per-group scales and int8
codes the kernels already produce and skips the per-element Scale tensor.
``register_qparam_buffers``, ``expand_ignore_list`` and
``save_to_compressed_tensors`` write the quantized model as a "pack-quantized"
compressed-tensors checkpoint (host code: the compressed-tensors quantization
config and the transformers checkpoint writer).
"""

import logging
import os
import re

import torch

from .. import ops

Q_PARAMS = ("weight_packed", "weight_scale", "weight_shape")
# fused projections of inference engines: an ignored member ignores the fused module too
MERGE_PATTERNS = {
    "qkv_proj": r"(q_proj|k_proj|v_proj)",
    "in_proj_qkvz": r"(in_proj_qkv|in_proj_z)",
    "in_proj_ba": r"(in_proj_b|in_proj_a)",
}


def compress_grouped(layer, group_scale, codes, bits):
    """Stage ``weight_packed`` / ``weight_scale`` / ``weight_shape`` on ``layer``.

    ``group_scale`` is ``[rows, columns // groupsize]`` fp32, ``codes`` is the
    ``[rows, columns]`` int8 code matrix.
    """
    weight = layer.weight
    # torch.tensor(weight.shape) on the device, filled there: a copy from pageable
    # host memory would synchronise the stream
    shape = torch.empty(weight.dim(), dtype=torch.long, device=weight.device)
    for i, n in enumerate(weight.shape):
        shape[i] = n
    layer._export_qparams = {
        "weight_packed": ops.pack_int32(codes.contiguous(), bits),
        "weight_scale": group_scale.to(weight.dtype).contiguous(),
        "weight_shape": shape,
    }


def compress(layer, Scale, W_int, bits, groupsize):
    """compressed_tensors_utils.py:22-42 on per-element ``Scale`` / ``W_int``."""
    weight = layer.weight
    rows, columns = weight.shape
    quantized_weight = W_int.reshape(weight.shape).to(torch.int8)
    group_scale = Scale.reshape(rows, columns // groupsize, groupsize)
    assert (group_scale == group_scale[..., 0:1]).all(), \
        "Scales in the same quantization group should be the same."
    compress_grouped(layer, group_scale[:, :, 0].float(), quantized_weight, bits)


def register_qparam_buffers(modules):
    """compressed_tensors_utils.py:45-53."""
    for module in modules:
        qparams = module.__dict__.pop("_export_qparams", None)
        if qparams is None:
            continue
        for name, tensor in qparams.items():
            module.register_buffer(name, tensor)


def _expert_stack(experts, n, part, attr, dim0_pair=None):
    """``[n, ...]`` stack of ``experts[i].<part>.<attr>``; with ``dim0_pair`` the
    per-expert entry is that part's tensor followed (along dim 0) by the same
    attribute of the ``dim0_pair`` part."""
    rows = []
    for i in range(n):
        t = getattr(getattr(experts[i], part), attr)
        if dim0_pair is not None:
            t = torch.cat([t, getattr(getattr(experts[i], dim0_pair), attr)], dim=0)
        rows.append(t)
    return torch.nn.Parameter(torch.stack(rows, dim=0), requires_grad=False)


def stack_experts(experts, weight_packed=False):
    """MoE expert stacking before export (utils/models/mixins.py:93-144,
    ``MoEMixin.stack_experts``): the per-expert ``gate_proj`` / ``up_proj`` /
    ``down_proj`` linears of an experts container (``num_experts``, indexable,
    submodules named ``"0"``, ``"1"``, ...) become 3-D parameters, the layout
    the exported checkpoint stores for fused experts:

    * ``weight_packed=True``: ``gate_up_proj_packed`` / ``gate_up_proj_scale``
      ``[E, 2I, .]`` (gate rows, then up rows), ``down_proj_packed`` /
      ``down_proj_scale`` ``[E, H, .]`` and the int64 shape tensors
      ``gate_up_proj_shape = (E, 2I, H)``, ``down_proj_shape = (E, H, I)``;
    * else ``gate_up_proj`` ``[E, 2I, H]`` and ``down_proj`` ``[E, H, I]``.

    The per-expert submodules are removed.  The container is then meant for
    saving: its forward is left as it was (it indexed the removed submodules).
    """
    n = experts.num_experts
    if weight_packed:
        experts.gate_up_proj_packed = _expert_stack(experts, n, "gate_proj", "weight_packed",
                                                    "up_proj")
        experts.down_proj_packed = _expert_stack(experts, n, "down_proj", "weight_packed")
        experts.gate_up_proj_scale = _expert_stack(experts, n, "gate_proj", "weight_scale",
                                                   "up_proj")
        experts.down_proj_scale = _expert_stack(experts, n, "down_proj", "weight_scale")
        inter, hidden = (int(v) for v in experts[0].gate_proj.weight_shape[:2])
        experts.gate_up_proj_shape = torch.tensor((n, 2 * inter, hidden))
        experts.down_proj_shape = torch.tensor((n, hidden, inter))
    else:
        experts.gate_up_proj = _expert_stack(experts, n, "gate_proj", "weight", "up_proj")
        experts.down_proj = _expert_stack(experts, n, "down_proj", "weight")
    for i in range(n):
        del experts._modules[str(i)]


def expand_ignore_list(ignore_list, merge_patterns=None):
    """compressed_tensors_utils.py:56-80: the ignore list plus, for every entry
    naming a member of a fused projection, the fused module's name; sorted and
    without duplicates."""
    patterns = MERGE_PATTERNS if merge_patterns is None else merge_patterns
    out = set(ignore_list)
    for name in ignore_list:
        for fused, pat in patterns.items():
            if re.search(pat, name):
                out.add(re.sub(pat, fused, name))
    return sorted(out)


def save_to_compressed_tensors(source_model, config, model, tokenizer, processor, save_path,
                               bits=4, group_size=128, sym=True, export_mtp=False):
    """compressed_tensors_utils.py:83-156: write ``model`` (its quantized linears
    carrying ``weight_packed`` / ``weight_scale`` / ``weight_shape`` buffers, see
    ``register_qparam_buffers``) as a pack-quantized compressed-tensors
    checkpoint with its config, generation config, tokenizer and processor.
    Linears (and convolutions) without packed weights are listed as ignored;
    packed ones lose their float ``weight``."""
    from compressed_tensors.quantization import (QuantizationArgs, QuantizationConfig,
                                                 QuantizationScheme, QuantizationStrategy,
                                                 QuantizationType)
    assert bits in (4, 8) and sym, "pack-quantized export supports symmetric 4 / 8 bits"
    os.makedirs(save_path, exist_ok=True)
    ignore = ["re:^mtp.*"]
    for name, module in model.named_modules():
        if isinstance(module, (torch.nn.Linear, torch.nn.modules.conv._ConvNd)):
            if hasattr(module, "weight_packed"):
                del module.weight
            else:
                ignore.append(name)
    ignore = expand_ignore_list(ignore)
    weights = QuantizationArgs(
        num_bits=bits, type=QuantizationType.INT,
        strategy=QuantizationStrategy.CHANNEL if group_size == -1 else QuantizationStrategy.GROUP,
        group_size=group_size, symmetric=sym, dynamic=False)
    scheme = QuantizationScheme(targets=["Linear"], format="pack-quantized", weights=weights)
    qconfig = QuantizationConfig(config_groups={"group_0": scheme}, ignore=ignore,
                                 format="pack-quantized", quant_method="compressed-tensors",
                                 quantization_status="compressed")
    if hasattr(config, "quantization_config"):
        delattr(config, "quantization_config")
    config.quantization_config = qconfig.model_dump()
    logging.info(f"Saving compressed model to {save_path}...")
    config.save_pretrained(save_path)
    model.generation_config.save_pretrained(save_path)
    tokenizer.save_pretrained(save_path)
    processor.save_pretrained(save_path)
    model.save_pretrained(save_path, safe_serialization=True, save_original_format=False)
    if export_mtp:
        from compressed_tensors.utils import save_mtp_tensors_to_checkpoint
        save_mtp_tensors_to_checkpoint(source_model=source_model, dest_dir=save_path)
