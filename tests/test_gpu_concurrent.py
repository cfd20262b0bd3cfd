"""``fasterquant_all``: several quantizer objects with their device work overlapped
on a stream pool must give exactly what calling ``fasterquant`` on each in turn
gives (same kernels, same inputs, so bit-identical), including the export
buffers and a layer that needs the damp auto-increment retry."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from g2ptq_b200.gptq_utils import gptq_utils, gptaq_utils, g2ptq_utils  # noqa: E402
from g2ptq_b200.gptq_utils import _engine  # noqa: E402
from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers  # noqa: E402
from g2ptq_b200.utils.quant_utils import WeightQuantizer  # noqa: E402
from g2ptq_b200.utils.compressed_tensors_utils import Q_PARAMS  # noqa: E402

DEV = "cuda"


def quantizers(bits, sym, C, gs):
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=False)
    return make_group_quantizers(q, C, gs)


def make_linear(R, C, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lin = torch.nn.Linear(C, R, bias=False, device=DEV, dtype=torch.bfloat16)
    lin.weight.data = (torch.randn(R, C, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    return lin


def acts(T, C, seed):
    g = torch.Generator(device=DEV).manual_seed(1000 + seed)
    x = torch.randn(T, C, device=DEV, generator=g)
    x[:, :2] *= 20
    return x.to(torch.bfloat16)


SHAPES = [(256, 512), (128, 384), (384, 256), (64, 1024), (96, 80)]


def gptq_objects(lowrank_H=None):
    objs = []
    for i, (R, C) in enumerate(SHAPES):
        obj = gptq_utils.GPTQ([make_linear(R, C, i)])
        gs = 128 if C % 128 == 0 else -1
        obj.quantizer = quantizers(4, True, C, gs)
        if lowrank_H is not None and C == lowrank_H.shape[0]:
            obj.H = lowrank_H.clone()[None]
            obj.nsamples[0] = 1
        else:
            for s in range(3):
                obj.add_batch(0, acts(200 + 37 * s, C, 10 * i + s), None)
        objs.append((obj, gs))
    return objs


def snapshot(objs):
    out = []
    for obj, _ in objs:
        for lin in obj.layers:
            out.append(lin.weight.data.clone())
            for n in Q_PARAMS:
                b = getattr(lin, n, None)
                if isinstance(b, torch.Tensor):
                    out.append(b.clone())
    return out


@pytest.mark.parametrize("with_retry", [False, True])
def test_gptq_fasterquant_all_matches_sequential(with_retry):
    H80 = None
    if with_retry:
        # eigenvalues 1 except one at -0.011: damp 0.01 leaves it negative,
        # one auto-increment (to 0.0115) makes the matrix positive definite
        g = torch.Generator().manual_seed(11)
        Qm, _ = torch.linalg.qr(torch.randn(80, 80, dtype=torch.float64, generator=g))
        lam = torch.ones(80, dtype=torch.float64)
        lam[7] = -0.011
        H80 = ((Qm * lam) @ Qm.T).float().to(DEV)
    kw = dict(blocksize=128, percdamp=0.01, actorder=True, static_groups=True,
              export_compressed_tensors=True)
    seq = gptq_objects(H80)
    for obj, gs in seq:
        obj.fasterquant(groupsize=gs, **kw)
    ref = snapshot(seq)
    damps_ref = [o._last_damps for o, _ in seq]

    par = gptq_objects(H80)
    # one groupsize per call: run the two groupsize classes as two batches
    for gs in (128, -1):
        batch = [o for o, g in par if g == gs]
        gptq_utils.fasterquant_all(batch, groupsize=gs, **kw)
    torch.cuda.synchronize()
    got = snapshot(par)
    assert len(ref) == len(got)
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    assert [o._last_damps for o, _ in par] == damps_ref
    if with_retry:
        assert damps_ref[-1][0] > 0.01


def test_gptaq_and_g2ptq_fasterquant_all_match_sequential():
    def build():
        objs = []
        for i, (R, C) in enumerate(SHAPES[:3]):
            lin = make_linear(R, C, 50 + i)
            ob = gptaq_utils.GPTAQ([lin])
            for s in range(2):
                x = acts(150 + s, C, 60 + i + s)
                ob.fp_inp[0].append((x.float() + 0.01 * acts(150 + s, C, 70 + s).float())[None])
                ob.add_batch(0, x, None)
            ob.quantizer = quantizers(3, False, C, 64)
            objs.append(ob)
        g2 = []
        for i, (R, C) in enumerate(SHAPES[:3]):
            lin = make_linear(R, C, 80 + i)
            gen = torch.Generator(device=DEV).manual_seed(90 + i)
            grad = torch.randn(R, C, device=DEV, generator=gen) * 1e-3
            sal = [torch.rand(1, 128, 4, device=DEV, generator=gen) for _ in range(2)]
            ob = g2ptq_utils.G2PTQ([lin], [sal], [grad], num_groups=4)
            for s in range(2):
                ob.add_batch(0, acts(128, C, 100 + i + s)[None], None)
            ob.quantizer = quantizers(4, True, C, 64)
            g2.append(ob)
        return objs, g2

    kw_a = dict(blocksize=64, percdamp=0.01, groupsize=64, actorder=False)
    kw_g = dict(blocksize=64, percdamp=0.01, groupsize=64, actorder=True, static_groups=True,
                enable_gradient_update=True, alpha=1.0)
    a_seq, g_seq = build()
    for o in a_seq:
        o.fasterquant(**kw_a)
    for o in g_seq:
        o.fasterquant(**kw_g)
    ref = [o.layers[0].weight.data.clone() for o in a_seq + g_seq]
    a_par, g_par = build()
    _engine.fasterquant_all(a_par, **kw_a)
    _engine.fasterquant_all(g_par, **kw_g)
    torch.cuda.synchronize()
    got = [o.layers[0].weight.data for o in a_par + g_par]
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    assert not np.isnan(np.array([float(x.float().abs().sum()) for x in got])).any()
