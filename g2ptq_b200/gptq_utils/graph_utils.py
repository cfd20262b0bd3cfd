"""Tensor checks at the kernel boundary, the one part of the reference's
gptq_utils/graph_utils.py this package keeps.

``validate_tensors`` is the interface check every ``run_eager`` performs in the
reference (graph_utils.py:12-20): all tensors on CUDA, on one device, and
contiguous, with the same exception types and messages, so that callers
relying on them see the same behaviour.  The reference's CUDA-graph replay of
compensation blocks (``run_graph``) has no counterpart: ``fasterquant``'s
``graph=True`` is accepted and ignored, because the whole traversal of a layer
is already one short sequence of library launches.
"""


def validate_tensors(description, *tensors):
    """Raise unless every non-None tensor is a contiguous CUDA tensor on one
    device; returns that device."""
    present = [t for t in tensors if t is not None]
    for t in present:
        if not t.is_cuda:
            raise RuntimeError(f"{description} requires every tensor to be on CUDA.")
    device = present[0].device
    for t in present:
        if t.device != device:
            raise ValueError(f"{description} requires every tensor on the same device.")
    for t in present:
        if not t.is_contiguous():
            raise ValueError(f"{description} requires contiguous tensors.")
    return device
