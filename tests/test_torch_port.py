"""The torch CPU restatement of the reference path (``oracle/torch_port.py``,
the CPU baseline of bench.py) against the reference's golden fixtures and the
numpy oracle (CPU only)."""

import numpy as np
import pytest
import torch

from oracle import hessian as ohess, torch_port as tp

FQ_CASES = [
    ("w4_sym_ungrouped", 4, True, -1, False, 128),
    ("w4_sym_g40_actorder", 4, True, 40, True, 128),
    ("w3_asym_g40_dynamic", 3, False, 40, False, 64),
    ("w2_asym_g64_dynamic", 2, False, 64, False, 128),
    ("w4_asym_g128_actorder", 4, False, 128, True, 128),
]


def proxy_loss(W, Q, H):
    d = (np.asarray(W, np.float64) - np.asarray(Q, np.float64))
    return np.einsum("brc,bcd,brd->b", d, np.asarray(H, np.float64), d)


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_torch_port_fasterquant_matches_reference_fixtures(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W, H = g[f"{name}__W"], g[f"{name}__H"]
    Q, codes = tp.fasterquant(torch.from_numpy(W), torch.from_numpy(H), bits, sym, gs, act, act,
                              0.01, blk)
    same = float(np.mean(codes.numpy() == g[f"{name}__gptq_W_int"]))
    assert same >= 0.999, same
    np.testing.assert_allclose(proxy_loss(W, Q.numpy(), H),
                               proxy_loss(W, g[f"{name}__gptq_Q"], H), rtol=1e-3)


def test_torch_port_add_batch_matches_oracle():
    rng = np.random.default_rng(3)
    C = 96
    H_t, n_t = torch.zeros(C, C), 0
    H_o, n_o = np.zeros((C, C), np.float32), 0
    for b, t in [(2, 64), (1, 128), (3, 32)]:
        x = rng.standard_normal((b, t, C)).astype(np.float32)
        H_t, n_t = tp.add_batch(H_t, n_t, torch.from_numpy(x))
        H_o, n_o = ohess.gptq_add_batch(H_o, n_o, x)
    assert n_t == n_o
    err = np.linalg.norm(H_t.numpy() - H_o) / np.linalg.norm(H_o)
    assert err < 1e-6, err


def test_torch_port_timings_are_reported():
    rng = np.random.default_rng(4)
    W = torch.from_numpy((rng.standard_normal((1, 64, 256)) * 0.02).astype(np.float32))
    X = torch.from_numpy(rng.standard_normal((1, 512, 256)).astype(np.float32))
    H, _ = tp.add_batch(torch.zeros(256, 256), 0, X)
    timings = {}
    tp.fasterquant(W, H[None], 4, True, 128, True, True, timings=timings)
    assert timings["factor"] > 0 and timings["compensate"] > 0
