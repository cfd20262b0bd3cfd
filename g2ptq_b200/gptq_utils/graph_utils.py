"""CUDA-graph capture of compensation blocks, mirroring gptq_utils/graph_utils.py.

``validate_tensors`` keeps the reference's checks and messages
(graph_utils.py:12-20); ``run_graph`` captures ``run_eager(**params)`` once per
(shape, dtype, constants) key and replays it (graph_utils.py:53-101).
"""

import torch

_GRAPH_CACHE = {}


def validate_tensors(description, *tensors):
    tensors = [t for t in tensors if t is not None]
    if any(not t.is_cuda for t in tensors):
        raise RuntimeError(f"{description} requires every tensor to be on CUDA.")
    device = tensors[0].device
    if any(t.device != device for t in tensors):
        raise ValueError(f"{description} requires every tensor on the same device.")
    if any(not t.is_contiguous() for t in tensors):
        raise ValueError(f"{description} requires contiguous tensors.")
    return device


def _key(name, run_eager, params, input_names, output_names, device):
    tensors = tuple((k, tuple(v.shape), v.dtype) for k, v in params.items()
                    if isinstance(v, torch.Tensor))
    consts = tuple((k, v) for k, v in params.items() if not isinstance(v, torch.Tensor))
    return (name, run_eager, device.index, tensors, consts, tuple(input_names),
            tuple(output_names))


def run_graph(run_eager, params, *, input_names, output_names, name):
    device = validate_tensors(f"CUDA Graph {name}",
                              *[v for v in params.values() if isinstance(v, torch.Tensor)])
    key = _key(name, run_eager, params, input_names, output_names, device)
    with torch.cuda.device(device):
        state = _GRAPH_CACHE.get(key)
        if state is None:
            static = {k: torch.empty_like(v) if isinstance(v, torch.Tensor) else v
                      for k, v in params.items()}
            for n in input_names:
                static[n].copy_(params[n])
            cur = torch.cuda.current_stream(device)
            side = torch.cuda.Stream(device=device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                run_eager(**static)
            cur.wait_stream(side)
            for n in input_names:
                static[n].copy_(params[n])
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                run_eager(**static)
            state = {"graph": graph, "params": static}
            _GRAPH_CACHE[key] = state
        for n in input_names:
            state["params"][n].copy_(params[n])
        state["graph"].replay()
        for n in output_names:
            params[n].copy_(state["params"][n])
    return tuple(params[n] for n in output_names)


def clear_graph_cache():
    _GRAPH_CACHE.clear()
