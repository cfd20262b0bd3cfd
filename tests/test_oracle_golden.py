"""Pin the numpy oracle against fixtures produced by the reference itself.

Tolerances follow the reference's own test file (floats rtol = atol = 2e-5,
integer codes exact; tests/test_triton_compensation.py:46-47) for the block
kernels, and the parity gates of the port for whole pipelines: Hessians within
1e-5 relative Frobenius error, codes identical on at least 99.9% of weights,
and per-layer ``||(W-Q)X||^2`` within 1e-3 relative.
"""

import numpy as np
import pytest

from oracle import compensation as comp
from oracle import export, fasterquant as fq, hessian, linalg, partition, quant

f32 = np.float32


def rel_fro(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


# ---------------------------------------------------------------------------
# add_batch
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_gptq_add_batch(golden, tag):
    g = golden("hessians.npz")
    C = g[f"gptq_{tag}_H"].shape[0]
    H, n = np.zeros((C, C), f32), 0
    for i in range(4):
        H, n = hessian.gptq_add_batch(H, n, g[f"gptq_{tag}_x{i}"])
    assert n == int(g[f"gptq_{tag}_n"])
    assert rel_fro(H, g[f"gptq_{tag}_H"]) < 1e-6


def test_g2ptq_add_batch(golden):
    g = golden("hessians.npz")
    C = g["g2ptq_H"].shape[-1]
    H, a, k, t = np.zeros((4, C, C), f32), np.zeros(C, f32), 0, 0
    for i in range(3):
        H, a, k, t = hessian.g2ptq_add_batch(H, a, k, t, g[f"g2ptq_x{i}"], g[f"g2ptq_s{i}"])
    assert k == int(g["g2ptq_index"]) and t == int(g["g2ptq_total_tokens"])
    assert rel_fro(H, g["g2ptq_H"]) < 1e-6
    assert rel_fro(a, g["g2ptq_act_square"]) < 1e-6


def test_gptaq_add_batch(golden):
    g = golden("hessians.npz")
    C = g["gptaq_H"].shape[0]
    H, D, n = np.zeros((C, C), f32), np.zeros((C, C), f32), 0
    for i in range(3):
        H, D, n = hessian.gptaq_add_batch(H, D, n, g[f"gptaq_x{i}"], g[f"gptaq_fp{i}"])
    assert n == int(g["gptaq_n"])
    assert rel_fro(H, g["gptaq_H"]) < 1e-6
    assert rel_fro(D, g["gptaq_dXXT"]) < 1e-5


def test_guided_add_batch(golden):
    g = golden("hessians.npz")
    C = g["guided_H"].shape[-1]
    H, a, idx = np.zeros((4, C, C), f32), np.zeros(C, f32), 0
    for i in range(2):
        H, a, idx = hessian.guided_add_batch(H, a, idx, g[f"guided_x{i}"], g["guided_sal"])
    assert idx == 3
    assert rel_fro(H, g["guided_H"]) < 1e-6
    assert rel_fro(a, g["guided_act_square"]) < 1e-6


# ---------------------------------------------------------------------------
# Block kernels
# ---------------------------------------------------------------------------

BLOCK_NAMES = ["symmetric_2bit_tail", "asymmetric_2bit_tail", "symmetric_4bit_batched",
               "asymmetric_4bit_batched", "symmetric_8bit_small", "asymmetric_8bit_small",
               "asymmetric_3bit_fullblock", "symmetric_4bit_fullblock"]


def _close(a, b):
    np.testing.assert_allclose(a, b, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("name", BLOCK_NAMES)
def test_block_kernels(golden, name):
    g = golden("blocks.npz")
    k = lambda s: g[f"{name}__{s}"]
    maxq = int(k("maxq"))
    q, qi, err = comp.gptq_block(k("weight"), k("hinv"), k("scale"), k("zero"), maxq)
    np.testing.assert_array_equal(qi, k("gptq_int"))
    _close(q, k("gptq_q"))
    _close(err, k("gptq_err"))
    q, qi, err, gh = comp.g2ptq_block(k("weight"), k("hinv"), k("scale"), k("zero"),
                                      k("z"), k("ghinv"), maxq)
    np.testing.assert_array_equal(qi, k("g2ptq_int"))
    _close(q, k("g2ptq_q"))
    _close(err, k("g2ptq_err"))
    _close(gh, k("g2ptq_ghinv"))
    q, qi, err = comp.gptaq_block(k("weight"), k("hinv"), k("p"), k("scale"), k("zero"), maxq)
    np.testing.assert_array_equal(qi, k("gptaq_int"))
    _close(q, k("gptaq_q"))
    _close(err, k("gptaq_err"))


# ---------------------------------------------------------------------------
# Whole pipelines
# ---------------------------------------------------------------------------

FQ_CASES = [
    ("w4_sym_ungrouped", 4, True, -1, False, 128),
    ("w4_sym_g40_actorder", 4, True, 40, True, 128),
    ("w3_asym_g40_dynamic", 3, False, 40, False, 64),
    ("w2_asym_g64_dynamic", 2, False, 64, False, 128),
    ("w4_asym_g128_actorder", 4, False, 128, True, 128),
]


def codes_match(a, b):
    return float(np.mean(a == b))


def proxy_loss(W, Q, H):
    """Per-layer ``||(W-Q)X||^2`` up to the constant n/2: ``tr(dW H dW^T)``."""
    d = (W - Q).astype(np.float64)
    return np.einsum("brc,bcd,brd->b", d, H.astype(np.float64), d)


def quantizers_for(bits, sym, C, gs):
    return comp.make_group_quantizers(comp.Quantizer(bits, sym), C, gs)


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
@pytest.mark.parametrize("route", ["reference", "ul"])
def test_gptq_fasterquant(golden, case, route):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W, H = g[f"{name}__W"], g[f"{name}__H"]
    Q, W_int, Scale, _ = fq.gptq_fasterquant(W, H, quantizers_for(bits, sym, W.shape[2], gs),
                                             blk, 0.01, gs, act, act, route=route)
    assert codes_match(W_int, g[f"{name}__gptq_W_int"]) >= 0.999
    np.testing.assert_allclose(Scale, g[f"{name}__gptq_Scale"], rtol=1e-6, atol=0)
    ref_loss = proxy_loss(W, g[f"{name}__gptq_Q"], H)
    loss = proxy_loss(W, Q, H)
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-3)
    if route == "reference":
        _close(Q, g[f"{name}__gptq_Q"])


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_gptaq_fasterquant(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W, H, D = g[f"{name}__W"], g[f"{name}__H"], g[f"{name}__gptaq_dXXT"]
    Q, _, _, _ = fq.gptaq_fasterquant(W, H, D, quantizers_for(bits, sym, W.shape[2], gs),
                                      blk, 0.01, gs, act, act)
    _close(Q, g[f"{name}__gptaq_Q"])


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_g2ptq_fasterquant(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W = g[f"{name}__W"]
    Q, _, _, _ = fq.g2ptq_fasterquant(W, g[f"{name}__g2_H"], g[f"{name}__g2_act_square"],
                                      g[f"{name}__g2_grad"],
                                      quantizers_for(bits, sym, W.shape[2], gs), 4, blk, 0.01,
                                      gs, act, act, True, 1.0)
    ref = g[f"{name}__g2ptq_Q"]
    assert float(np.mean(np.isclose(Q, ref, rtol=2e-5, atol=2e-5))) >= 0.999


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_guided_fasterquant(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W = g[f"{name}__W"]
    Q, _, _, _ = fq.guided_fasterquant(W, g[f"{name}__guided_H"],
                                       g[f"{name}__guided_act_square"],
                                       quantizers_for(bits, sym, W.shape[2], gs), 4, blk,
                                       0.01, gs, act, act)
    ref = g[f"{name}__guided_Q"]
    assert float(np.mean(np.isclose(Q, ref, rtol=2e-5, atol=2e-5))) >= 0.999


# ---------------------------------------------------------------------------
# find_params, Cholesky chain, export packing, partition
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("mode", ["00", "10", "11"])
def test_find_params(golden, bits, sym, mode):
    g = golden("misc.npz")
    tag = f"fp_b{bits}_{'sym' if sym else 'asym'}_{mode}"
    if tag + "_scale" not in g:
        pytest.skip("clip search not generated for 8 bits")
    x = g["fp_x"]
    hd = np.repeat(g["fp_hdiag"], 6, axis=0) if mode == "11" else None
    s, z = quant.find_params(x, bits, sym, mse=mode[0] == "1", h_diag=hd)
    np.testing.assert_allclose(s, g[tag + "_scale"], rtol=1e-6, atol=0)
    np.testing.assert_array_equal(z, g[tag + "_zero"])
    maxq = quant.qrange(bits)[0]
    fqv, q = quant.fake_quantize(x, s, z, maxq)
    np.testing.assert_array_equal(q, g[tag + "_q"])
    np.testing.assert_allclose(fqv, g[tag + "_fq"], rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("tag", ["pd", "lowrank"])
@pytest.mark.parametrize("route", ["reference", "ul"])
def test_cholesky_chain(golden, tag, route):
    g = golden("misc.npz")
    H = g[f"chol_{tag}_H"]
    U, _, damp = linalg.damped_upper_inverse_factor(H, 0.01, route)
    assert abs(damp - float(g[f"chol_{tag}_damp"])) < 1e-9
    assert rel_fro(U, g[f"chol_{tag}_U"]) < 1e-4
    assert np.allclose(np.tril(U, -1), 0)


def test_cholesky_retry_exhausts():
    H = -np.eye(8, dtype=f32)
    with pytest.raises(ValueError):
        linalg.damped_upper_inverse_factor(H, 0.01)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_pack_to_int32(golden, bits):
    g = golden("misc.npz")
    np.testing.assert_array_equal(export.pack_to_int32(g[f"pack_b{bits}_codes"], bits),
                                  g[f"pack_b{bits}_packed"])


def test_partition_lpt():
    items = [("a", 8), ("b", 7), ("c", 6), ("d", 5), ("e", 4)]
    ordered, bins, owner = partition.greedy_bin_packing(items, 2, lambda it: it[1])
    assert [it[0] for it in ordered] == ["a", "b", "c", "d", "e"]
    loads = [sum(it[1] for it in bins[b]) for b in range(2)]
    assert sorted(loads) == [13, 17]
    specs = partition.build_chunk_specs({"q": (64, 32), "k": (16, 32), "v": (16, 32),
                                         "o": (32, 64)}, 1)
    assert [s[0] for s in specs] == [("q",), ("k",), ("v",), ("o",)]
    specs = partition.build_chunk_specs({"k": (16, 32), "v": (16, 32), "q": (64, 32)}, 4)
    assert [s[0] for s in specs] == [("k", "v"), ("q",)]
