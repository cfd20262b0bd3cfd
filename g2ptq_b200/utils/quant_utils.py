"""Weight quantizer, mirroring ``utils/quant_utils.py`` of the reference.

Same names, fields and call semantics as the reference's ``WeightQuantizer``
(quant_utils.py:341-465) and quantize / dequantize helpers (quant_utils.py:8-34),
with every computation done by the sm_100a kernels of ``libg2ptq_b200``.
Tensors must live on a CUDA device.
"""

import collections
import copy

import torch

from .. import ops


def asym_quant(x, scale, zero, maxq):
    """quant_utils.py:8-12 -> ``(q, scale, zero)``; elementwise parameters."""
    x2 = x.reshape(-1, 1).contiguous().float()
    s = torch.broadcast_to(scale.to(x.device).float(), x.shape).reshape(-1, 1).contiguous()
    z = torch.broadcast_to(zero.to(x.device).float(), x.shape).reshape(-1, 1).contiguous()
    codes = torch.empty(x2.shape, dtype=torch.int8, device=x.device)
    ops.fake_quantize(x2, s, z, maxq, codes=codes)
    return codes.float().reshape(x.shape), scale, zero


def asym_dequant(q, scale, zero):
    """quant_utils.py:15-16."""
    return scale * (q - zero)


def sym_quant(x, scale, maxq):
    q, scale, _ = asym_quant(x, scale, torch.zeros_like(scale), maxq)
    return q, scale


def sym_dequant(q, scale):
    return scale * q


# value types __deepcopy__ shares as they are / rebuilds as containers
_PLAIN = (bool, int, float, str, type(None))
_CONTAINERS = (dict, collections.OrderedDict, set)


class WeightQuantizer(torch.nn.Module):
    """Per-channel / per-group weight quantizer (quant_utils.py:341-465)."""

    def __init__(self, shape: int = 1) -> None:
        super().__init__()
        self.register_buffer("scale", torch.zeros(shape))
        self.register_buffer("zero", torch.zeros(shape))
        self._ready = False
        self._status = None

    def configure(self, bits, perchannel: bool = False, sym: bool = True, mse: bool = False,
                  norm: float = 2.4, grid: int = 50, maxshrink: float = 0.5,
                  weight_groupsize: int = -1, hclip: bool = False) -> None:
        self.bits = bits
        self.perchannel = perchannel
        self.sym = sym
        self.mse = mse
        self.hclip = hclip
        self.norm = norm
        self.grid = grid
        self.maxshrink = maxshrink
        self.weight_groupsize = weight_groupsize
        self.maxq = 2 ** (bits - 1) - 1
        self.minq = -(self.maxq + 1)
        self.bit_range = self.maxq - self.minq
        self._ready = False

    def __deepcopy__(self, memo):
        """What ``copy.deepcopy`` makes of the quantizer, without the generic
        ``nn.Module`` traversal: ``make_group_quantizers`` copies one quantizer
        per weight group (hundreds per decoder layer), and the generic path
        costs about a tenth of a millisecond each.  Tensors are cloned, the
        module's bookkeeping containers copied (empty ones shallowly), other
        values deep-copied; the device status word is left for the copy to
        allocate."""
        new = object.__new__(self.__class__)
        memo[id(self)] = new
        d = {}
        for k, v in self.__dict__.items():
            t = type(v)
            if t in _PLAIN:
                pass
            elif k == "_status":
                v = None
            elif t in _CONTAINERS:
                if not v:
                    v = t()
                elif t is set:
                    v = copy.deepcopy(v, memo)
                else:
                    v = t((kk, vv.clone() if isinstance(vv, torch.Tensor)
                           else copy.deepcopy(vv, memo)) for kk, vv in v.items())
            elif isinstance(v, torch.Tensor):
                v = v.clone()
            else:
                v = copy.deepcopy(v, memo)
            d[k] = v
        new.__dict__ = d
        return new

    def status_tensor(self, device):
        if self._status is None or self._status.device != device:
            self._status = torch.zeros(1, dtype=torch.int32, device=device)
        return self._status

    def clip_config(self, H_diag, rows, cols):
        """The clip search of ``find_params`` (quant_utils.py:385-425) as a
        ``g2q_clip_t``, or None without ``mse``.  ``H_diag`` (``[blocks, cols]``,
        used with ``hclip``) weights the error by the Hessian diagonal of each
        block of ``rows / blocks`` rows; a constant diagonal falls back to the
        ``|fq - x|^norm`` error, as in the reference."""
        if not self.mse:
            return None
        hd = None
        if self.hclip and H_diag is not None:
            hd = H_diag.to(device="cuda" if not H_diag.is_cuda else H_diag.device,
                           dtype=torch.float32).reshape(H_diag.shape[0], cols).contiguous()
            if bool((hd.min() == hd.max()).item()):
                hd = None
        return ops.clip_config(self.grid, self.maxshrink, self.norm, hd,
                               None if hd is None else rows // hd.shape[0])

    def find_params(self, x, H_diag=None, out=None) -> None:
        """quant_utils.py:377-433, with the ``mse`` / ``hclip`` clip search.

        ``out`` -- optional ``(scale, zero)`` pair of ``[rows, 1]`` views to
        write into (used by the layer-batched quantizer objects so that all
        group parameters sit in one ``[rows, ngroups]`` array).
        """
        if self.bits == 16:
            return
        if not x.is_cuda:
            raise RuntimeError("g2ptq_b200 WeightQuantizer requires CUDA tensors")
        x = x.float() if x.dtype != torch.float32 else x
        rows, cols = x.shape
        status = self.status_tensor(x.device)
        if self.weight_groupsize > 0:
            ng = cols // self.weight_groupsize
            gs = self.weight_groupsize
            scale = torch.empty(rows, ng, dtype=torch.float32, device=x.device)
            zero = torch.empty_like(scale)
            for g in range(ng):
                xg = x[:, g * gs:(g + 1) * gs]
                clip = self.clip_config(
                    None if H_diag is None
                    else H_diag.reshape(H_diag.shape[0], cols)[:, g * gs:(g + 1) * gs],
                    rows, gs)
                if clip is None:
                    ops.find_params(scale, zero, xg, self.bits, self.sym, status, param_col=g)
                else:
                    ops.find_params_clip(scale, zero, xg, self.bits, self.sym, clip, status,
                                         param_col=g)
        else:
            if not self.perchannel:
                x = x.reshape(1, -1)
                rows = 1
            if x.stride(1) != 1:
                x = x.contiguous()
            if out is not None:
                scale, zero = out
            else:
                scale = torch.empty(rows, 1, dtype=torch.float32, device=x.device)
                zero = torch.empty_like(scale)
            clip = self.clip_config(H_diag, rows, x.shape[1])
            if clip is None:
                ops.find_params(scale, zero, x, self.bits, self.sym, status)
            else:
                ops.find_params_clip(scale, zero, x, self.bits, self.sym, clip, status)
        self.scale = scale
        self.zero = zero
        self._ready = True

    def check(self):
        """Raise where the reference's ``torch._assert_async(scale.min() > 0)`` fires."""
        if self._status is not None and int(self._status.item()) != 0:
            raise RuntimeError("WeightQuantizer.find_params: non-positive scale")

    def fake_quantize(self, x):
        """quant_utils.py:435-459 -> ``(fq, q, scale)``."""
        x_dtype = x.dtype
        if not (self.ready() and self.bits < 16):
            return None, None, None
        rows, cols = x.shape
        xf = x.float().contiguous()
        if self.weight_groupsize > 0:
            colmap = (torch.arange(cols, device=x.device, dtype=torch.int32)
                      // self.weight_groupsize)
            scale = self.scale.contiguous()
            zero = self.zero.contiguous()
        else:
            colmap = None
            scale = self.scale.reshape(-1, 1).contiguous()
            zero = self.zero.reshape(-1, 1).contiguous()
            if scale.shape[0] == 1 and rows > 1:
                scale = scale.expand(rows, 1).contiguous()
                zero = zero.expand(rows, 1).contiguous()
        codes = torch.empty(rows, cols, dtype=torch.int8, device=x.device)
        fq, _ = ops.fake_quantize(xf, scale, zero, self.maxq, colmap=colmap, codes=codes)
        return fq.to(x_dtype), codes.float(), self.scale

    def enabled(self):
        return self.maxq > 0

    def ready(self):
        return self._ready
