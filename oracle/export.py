"""compressed-tensors export staging (numpy).

``compress`` follows utils/compressed_tensors_utils.py:22-42.  Its packing step
calls ``compressed_tensors.compressors.pack_to_int32`` (compressed-tensors,
pinned 0.18.0 by the reference's requirements.txt:14; 0.15.0.1 is the copy
installed here).  ``pack_to_int32`` below restates that published routine:
add ``2^(bits-1)`` to the int8 codes, view them as unsigned, zero-pad each row
to a multiple of ``32 // bits`` values and pack ``32 // bits`` consecutive
values per int32, the first value in the lowest bits.
"""

import numpy as np


def pack_to_int32(codes, bits):
    codes = np.asarray(codes)
    if codes.dtype != np.int8:
        raise ValueError("Tensor must be quantized to torch.int8 before packing")
    if bits > 8:
        raise ValueError("Packing is only supported for less than 8 bits")
    offset = 1 << (bits - 1)
    u = (codes.astype(np.int32) + offset).astype(np.uint8).astype(np.uint32)
    factor = 32 // bits
    rows, cols = u.shape
    padded = -(-cols // factor) * factor
    if padded != cols:
        u = np.pad(u, ((0, 0), (0, padded - cols)))
    u = u.reshape(rows, padded // factor, factor)
    shifts = (np.arange(factor, dtype=np.uint32) * bits).astype(np.uint32)
    packed = (u << shifts).sum(axis=2, dtype=np.uint64) & 0xFFFFFFFF
    return packed.astype(np.uint32).view(np.int32)


def compress(Scale, W_int, bits, groupsize, weight_shape):
    """compressed_tensors_utils.py:22-42 -> dict of export arrays (scale in float32)."""
    rows, columns = weight_shape
    q = np.asarray(W_int).reshape(rows, columns).astype(np.int8)
    gs = np.asarray(Scale, np.float32).reshape(rows, columns // groupsize, groupsize)
    if not (gs == gs[..., :1]).all():
        raise AssertionError("Scales in the same quantization group should be the same.")
    return {
        "weight_packed": pack_to_int32(q, bits),
        "weight_scale": gs[:, :, 0].copy(),
        "weight_shape": np.array([rows, columns], dtype=np.int64),
    }
