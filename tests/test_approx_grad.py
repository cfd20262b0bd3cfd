"""G2PTQ's ``--approx_grad`` ablation (``approx_grad_beta`` != 0).

The fixtures (tests/golden/approx.npz, ``make_golden.py --only approx``) are
the reference's own ``_run_torch_compensation`` with a raw-weight snapshot on
the reference test file's block cases, and whole ``G2PTQ.fasterquant`` runs
built with ``approx_grad_beta``.  CPU: the oracle against them.  GPU: the
block kernel (through ``run_eager``) and the object pipeline against them.
Tolerances as for the other block kernels: codes exact, floats 2e-5; whole
pipelines: >= 99.9 % of the weights equal within 2e-5 and the proxy loss
within 1e-3.
"""

import numpy as np
import pytest
import torch

from oracle import compensation as ocomp, fasterquant as ofq

BLOCK_NAMES = ["symmetric_2bit_tail", "asymmetric_2bit_tail", "symmetric_4bit_batched",
               "asymmetric_4bit_batched", "symmetric_8bit_small", "asymmetric_8bit_small",
               "asymmetric_3bit_fullblock", "symmetric_4bit_fullblock"]
FQ_CASES = [("w4_sym_g40_actorder", 4, True, 40, True, 128),
            ("w3_asym_g40_dynamic", 3, False, 40, False, 64)]


def _close(a, b):
    np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(b, np.float32),
                               rtol=2e-5, atol=2e-5)


def proxy_loss(W, Q, H):
    d = (np.asarray(W, np.float64) - np.asarray(Q, np.float64))
    return np.einsum("brc,bcd,brd->b", d, np.asarray(H, np.float64), d)


def _group_loss(W, Q, H, G):
    B, R, C = W.shape
    return proxy_loss(W.reshape(B * G, R // G, C), Q.reshape(B * G, R // G, C),
                      H.reshape(B * G, C, C))


@pytest.mark.parametrize("name", BLOCK_NAMES)
def test_oracle_block_matches_reference(golden, name):
    blocks, g = golden("blocks.npz"), golden("approx.npz")
    k = lambda s: blocks[f"{name}__{s}"]
    q, qi, err, gh = ocomp.g2ptq_block(k("weight"), k("hinv"), k("scale"), k("zero"), k("z"),
                                       k("ghinv"), int(k("maxq")), g[f"{name}__raw"],
                                       float(g["beta"]))
    np.testing.assert_array_equal(qi, g[f"{name}__int"])
    _close(q, g[f"{name}__q"])
    _close(err, g[f"{name}__err"])
    _close(gh, g[f"{name}__ghinv"])
    # the ablation changes the result (the fixture is not the default path)
    q0, _, _, _ = ocomp.g2ptq_block(k("weight"), k("hinv"), k("scale"), k("zero"), k("z"),
                                    k("ghinv"), int(k("maxq")))
    assert not np.allclose(q0, g[f"{name}__q"]) or not np.allclose(
        ocomp.g2ptq_block(k("weight"), k("hinv"), k("scale"), k("zero"), k("z"), k("ghinv"),
                          int(k("maxq")))[2], g[f"{name}__err"])


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_oracle_fasterquant_matches_reference(golden, case):
    g = golden("approx.npz")
    name, bits, sym, gs, act, blk = case
    W, H = g[f"{name}__W"], g[f"{name}__H"]
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(bits, sym), W.shape[2], gs)
    Q, _, _, _ = ofq.g2ptq_fasterquant(W, H, g[f"{name}__act_square"], g[f"{name}__grad"], oq,
                                       4, blk, 0.01, gs, act, act, True, 1.0,
                                       approx_beta=float(g["beta"]))
    same = float(np.mean(np.isclose(Q, g[f"{name}__Q"], rtol=2e-5, atol=2e-5)))
    assert same >= 0.999, same
    np.testing.assert_allclose(_group_loss(W, Q, H, 4), _group_loss(W, g[f"{name}__Q"], H, 4),
                               rtol=1e-3)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("name", BLOCK_NAMES)
def test_block_kernel_matches_reference(golden, name):
    from g2ptq_b200.gptq_utils import g2ptq_utils
    blocks, g = golden("blocks.npz"), golden("approx.npz")
    t = lambda a: torch.as_tensor(np.asarray(a)).cuda().float()
    k = lambda s: t(blocks[f"{name}__{s}"])
    W, gh = k("weight").clone(), k("ghinv").clone()
    qi, er = torch.empty_like(W), torch.empty_like(W)
    g2ptq_utils.run_eager(W, k("hinv"), k("scale"), k("zero"), k("z"), gh,
                          int(blocks[f"{name}__maxq"]), int_weight=qi, error=er,
                          weight_raw=t(g[f"{name}__raw"]), approx_beta=float(g["beta"]))
    np.testing.assert_array_equal(qi.cpu().numpy(), g[f"{name}__int"])
    _close(W.cpu().numpy(), g[f"{name}__q"])
    _close(er.cpu().numpy(), g[f"{name}__err"])
    _close(gh.cpu().numpy(), g[f"{name}__ghinv"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_g2ptq_object_matches_reference(golden, case):
    from g2ptq_b200.gptq_utils import g2ptq_utils
    from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    g = golden("approx.npz")
    name, bits, sym, gs, act, blk = case
    W, H = g[f"{name}__W"], g[f"{name}__H"]
    B, R, C = W.shape
    layers = []
    for b in range(B):
        lin = torch.nn.Linear(C, R, bias=False, device="cuda")
        lin.weight.data = torch.as_tensor(W[b]).cuda().clone()
        layers.append(lin)
    grads = [torch.as_tensor(x).cuda() for x in g[f"{name}__grad"]]
    obj = g2ptq_utils.G2PTQ(layers, [[] for _ in range(B)], grads, num_groups=4,
                            approx_grad_beta=float(g["beta"]))
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=False)
    obj.quantizer = make_group_quantizers(q, C, gs)
    obj.H = torch.as_tensor(H).cuda().clone()
    obj.act_square = torch.as_tensor(g[f"{name}__act_square"]).cuda().clone()
    obj.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act,
                    enable_gradient_update=True, alpha=1.0)
    Q = torch.stack([l.weight.data for l in layers]).cpu().numpy()
    same = float(np.mean(np.isclose(Q, g[f"{name}__Q"], rtol=2e-5, atol=2e-5)))
    assert same >= 0.999, same
    np.testing.assert_allclose(_group_loss(W, Q, H, 4), _group_loss(W, g[f"{name}__Q"], H, 4),
                               rtol=1e-3)
