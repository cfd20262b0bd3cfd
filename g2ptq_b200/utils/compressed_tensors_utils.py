"""compressed-tensors export staging, mirroring utils/compressed_tensors_utils.py:22-53.

``compress`` has the reference's signature and checks; the int32 packing runs
in the ``g2q_pack_int32`` kernel (same bit layout as
``compressed_tensors.compressors.pack_to_int32``).  ``compress_grouped`` is the
direct path used by ``fasterquant``: it takes the per-group scales and int8
codes the kernels already produce and skips the per-element Scale tensor.
"""

import torch

from .. import ops

Q_PARAMS = ("weight_packed", "weight_scale", "weight_shape")


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
