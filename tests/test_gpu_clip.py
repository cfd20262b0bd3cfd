"""Clip search of WeightQuantizer.find_params (--w_clip / --w_hclip,
quant_utils.py:373-425) on the GPU against the reference's own outputs (golden
fixtures) and the numpy oracle, and fasterquant with it end to end.

Bars: the (row, group) choices equal the reference's (fixtures) and the
oracle's except at near-ties -- the error sums over the group are reduced in a
different order than torch's, so when two grid points score within a few fp32
ulps of each other either may win -- where the error of the GPU's choice,
re-evaluated in float64, is within 1e-4 relative of the reference's choice;
at least 95% of the choices are identical.  Quantized weights of a whole
fasterquant agree on >= 99%.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from g2ptq_b200.gptq_utils import gptq_utils  # noqa: E402
from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers  # noqa: E402
from g2ptq_b200.utils.quant_utils import WeightQuantizer  # noqa: E402
from oracle import compensation as ocomp, fasterquant as ofq, quant as oquant  # noqa: E402

DEV = "cuda"
f32 = np.float32


def t(a):
    return torch.as_tensor(np.asarray(a)).to(DEV, torch.float32)


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("hclip", [False, True])
def test_clip_find_params_vs_reference(golden, bits, sym, hclip):
    m = golden("misc.npz")
    tag = f"fp_b{bits}_{'sym' if sym else 'asym'}_1{int(hclip)}"
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=True, hclip=hclip)
    x, hd = m["fp_x"], m["fp_hdiag"]
    q.find_params(t(x), t(hd) if hclip else None)
    s_g = q.scale.cpu().numpy().reshape(-1, 1)
    z_g = q.zero.cpu().numpy().reshape(-1, 1)
    s_r, z_r = m[tag + "_scale"].reshape(-1, 1), m[tag + "_zero"].reshape(-1, 1)
    _check_choices(x, s_g, z_g, s_r, z_r, bits, hd if hclip else None, x.shape[1])


def _err(x, s, z, maxq, norm, h):
    """Error of one grid choice, float64 (quant_utils.py:84-103)."""
    q = np.clip(np.rint(x / s) + z, -(maxq + 1), maxq)
    d = (s * (q - z) - x).astype(np.float64)
    if h is None:
        return float((np.abs(d) ** norm).sum())
    return float((d * d * h).sum())


def _check_choices(x, s_g, z_g, s_r, z_r, bits, hd, g, min_same=0.95):
    """(row, group) parameters [R, ngroups] of the GPU vs the reference."""
    R = x.shape[0]
    same = np.isclose(s_g, s_r, rtol=1e-6, atol=0) & (z_g == z_r)
    assert same.mean() >= min_same, same.mean()
    maxq = 2 ** (bits - 1) - 1
    for r, c in zip(*np.nonzero(~same)):
        xs = x[r, c * g:(c + 1) * g]
        h = None if hd is None else hd[r // (R // hd.shape[0]), c * g:(c + 1) * g]
        e_g = _err(xs, s_g[r, c], z_g[r, c], maxq, 2.4, h)
        e_r = _err(xs, s_r[r, c], z_r[r, c], maxq, 2.4, h)
        assert e_g <= e_r * (1 + 1e-4), (r, c, e_g, e_r)


@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("hclip", [False, True])
@pytest.mark.parametrize("gs", [128, -1])
def test_clip_find_params_vs_oracle(sym, hclip, gs):
    rng = np.random.default_rng(11 + int(sym) + 2 * int(hclip))
    R, C, bits = 256, 512, 4
    x = (rng.standard_normal((R, C)) * 0.02).astype(f32)
    x[:, :3] *= 10
    hd = (rng.random((4, C)) + 0.1).astype(f32)
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=True, hclip=hclip, weight_groupsize=gs)
    q.find_params(t(x), t(hd) if hclip else None)
    s_g = q.scale.cpu().numpy().reshape(R, -1)
    z_g = q.zero.cpu().numpy().reshape(R, -1)
    s_o, z_o = oquant.find_params(x, bits, sym, mse=True, h_diag=hd if hclip else None,
                                  weight_groupsize=gs)
    s_o, z_o = s_o.reshape(R, -1), z_o.reshape(R, -1)
    _check_choices(x, s_g, z_g, s_o, z_o, bits, hd if hclip else None, C if gs == -1 else gs)


def _linear(W):
    lin = torch.nn.Linear(W.shape[1], W.shape[0], bias=False, device=DEV)
    lin.weight.data = t(W).clone()
    return lin


@pytest.mark.parametrize("act,hclip", [(True, False), (True, True), (False, True)])
def test_gptq_fasterquant_with_clip_vs_oracle(act, hclip):
    rng = np.random.default_rng(5)
    R, C, gs, bits = 128, 384, 128, 4
    W = (rng.standard_normal((1, R, C)) * 0.02).astype(f32)
    X = rng.standard_normal((2048, C)).astype(f32)
    X[:, :4] *= 20
    H = (X.T.astype(np.float64) @ X / 1024).astype(f32)[None]
    layers = [_linear(W[0])]
    obj = gptq_utils.GPTQ(layers)
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=False, mse=True, hclip=hclip)
    obj.quantizer = make_group_quantizers(q, C, gs)
    obj.H = t(H).clone()
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act)
    Q = layers[0].weight.data[None].cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(bits, False, mse=True, hclip=hclip), C, gs)
    Qo, _, _, _ = ofq.gptq_fasterquant(W, H, oq, 128, 0.01, gs, act, act, route="ul")
    assert float(np.mean(np.isclose(Q, Qo, rtol=2e-5, atol=2e-5))) >= 0.99
