"""GPU parity of libg2ptq_b200 against the reference's golden fixtures and the oracle.

Tolerances: block kernels as the reference's own tests (codes exact, floats
rtol = atol = 2e-5, tests/test_triton_compensation.py:46-47); Hessians 1e-5
relative Frobenius error; whole pipelines: codes identical on >= 99.9% of
weights and per-layer ||(W-Q)X||^2 within 1e-3 relative.
"""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from g2ptq_b200 import ops, _lib  # noqa: E402
from g2ptq_b200.gptq_utils import _engine  # noqa: E402
from g2ptq_b200.gptq_utils import gptq_utils, g2ptq_utils, gptaq_utils, gptq_guided_utils  # noqa
from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers  # noqa: E402
from g2ptq_b200.utils.quant_utils import WeightQuantizer  # noqa: E402
from oracle import compensation as ocomp, fasterquant as ofq, hessian as ohess  # noqa: E402

DEV = "cuda"


def t(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(DEV, dtype)


def rel_fro(a, b):
    a = a.detach().double().cpu() if torch.is_tensor(a) else torch.as_tensor(a).double()
    b = b.detach().double().cpu() if torch.is_tensor(b) else torch.as_tensor(b).double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def close(a, b, rtol=2e-5, atol=2e-5):
    torch.testing.assert_close(a.detach().float().cpu(), torch.as_tensor(np.asarray(b)).float(),
                               rtol=rtol, atol=atol)


@pytest.fixture(autouse=True)
def _tf32_off():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def linear(W):
    lin = torch.nn.Linear(W.shape[1], W.shape[0], bias=False, device=DEV)
    lin.weight.data = t(W).clone()
    return lin


def quantizers(bits, sym, C, gs):
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=False)
    return make_group_quantizers(q, C, gs)


# ---------------------------------------------------------------------------
# building blocks
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("mask", [_lib.MASK_FULL, _lib.MASK_LOWER, _lib.MASK_STRICT_UPPER])
def test_gemm_fp32_vs_torch(ta, tb, mask):
    g = torch.Generator(device=DEV).manual_seed(7)
    M, N, K, B = 200, 136, 77, 2
    A = torch.randn(B, K, M, device=DEV, generator=g) if ta else torch.randn(B, M, K, device=DEV,
                                                                            generator=g)
    Bm = torch.randn(B, N, K, device=DEV, generator=g) if tb else torch.randn(B, K, N, device=DEV,
                                                                             generator=g)
    C0 = torch.randn(B, M, N, device=DEV, generator=g)
    Cm = C0.clone()
    ops.gemm(Cm, A, Bm, transA=ta, transB=tb, alpha=0.5, beta=-2.0, mask=mask)
    Aop = A.transpose(1, 2) if ta else A
    Bop = Bm.transpose(1, 2) if tb else Bm
    ref = 0.5 * C0 - 2.0 * (Aop.double() @ Bop.double()).float()
    i = torch.arange(M, device=DEV)[:, None]
    j = torch.arange(N, device=DEV)[None, :]
    if mask == _lib.MASK_LOWER:
        ref = torch.where(i >= j, ref, C0)
    if mask == _lib.MASK_STRICT_UPPER:
        ref = torch.where(i < j, ref, torch.zeros_like(ref))
    torch.testing.assert_close(Cm, ref, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("sym,scaled", [(True, False), (False, False), (True, True)])
def test_gram_update_vs_torch(dtype, sym, scaled):
    g = torch.Generator(device=DEV).manual_seed(11)
    T, C = 1000, 200
    X = torch.randn(T, C, device=DEV, generator=g).to(dtype)
    Y = X if sym else torch.randn(T, C, device=DEV, generator=g)
    s = torch.rand(T, 3, device=DEV, generator=g) if scaled else None
    D0 = torch.randn(C, C, device=DEV, generator=g)
    D0 = D0 + D0.T
    D = D0.clone()
    ops.gram_update(D, Y if not sym else X, X, row_scale=None if s is None else s[:, 1],
                    alpha=0.75, beta=0.125, symmetric=sym)
    Xd = X.double()
    Yd = (Y if not sym else X).double()
    w = torch.ones(T, device=DEV, dtype=torch.float64) if s is None else s[:, 1].double()
    ref = 0.75 * D0.double() + 0.125 * (Yd.T @ (Xd * w[:, None]))
    assert rel_fro(D, ref) < 5e-6


def test_chol_upper_inverse_matches_oracle(golden):
    from oracle import linalg
    m = golden("misc.npz")
    for tag in ("pd", "lowrank"):
        H = t(m[f"chol_{tag}_H"])[None].contiguous()
        U, info, damps = _engine.factor_with_retry(H, 0.01)
        info_list = info.cpu().tolist()
        _engine.retry_failed(H, U, info_list, damps)
        assert abs(damps[0] - float(m[f"chol_{tag}_damp"])) < 1e-9
        assert rel_fro(U[0], m[f"chol_{tag}_U"]) < 1e-4
        Uo, _, _ = linalg.damped_upper_inverse_factor(m[f"chol_{tag}_H"], 0.01, "ul")
        assert rel_fro(U[0], Uo) < 1e-4


def test_chol_large_identity_check():
    g = torch.Generator(device=DEV).manual_seed(5)
    C = 1100
    X = torch.randn(3000, C, device=DEV, generator=g)
    H = ((X.T @ X) / 3000)[None].contiguous()
    U, info = ops.chol_upper_inverse(H, 0.01)
    assert int(info.item()) == 0
    Hd = H[0].double() + 0.01 * torch.diagonal(H[0]).double().mean() * torch.eye(C, device=DEV,
                                                                                dtype=torch.float64)
    resid = (U[0].double().T @ U[0].double()) @ Hd - torch.eye(C, device=DEV, dtype=torch.float64)
    assert float(resid.abs().max()) < 1e-3
    assert float(torch.tril(U[0], -1).abs().max()) == 0.0


@pytest.mark.parametrize("precision,C,B,budget", [(0, 640, 6, None), (1, 640, 6, None),
                                                 (1, 600, 5, 1), (1, 256, 70, None)])
def test_chol_batch_lanes_match_one_by_one(precision, C, B, budget, monkeypatch):
    """A batch of factorizations in one call gives each matrix's result of a
    call on its own, bit for bit, including a failing one in the middle of the
    batch: precision 0 runs up to four side by side on forked streams,
    precision 1 advances chains of the batch panel by panel together (one
    chain of four and a single one when the workspace holds four; a partial
    last panel at C = 600; more than the 64 damps one launch carries)."""
    if budget is not None:
        monkeypatch.setattr(ops, "CHOL_BATCH_BYTES", budget)
    g = torch.Generator(device=DEV).manual_seed(17)
    X = torch.randn(B, 2 * C, C, device=DEV, generator=g)
    H = (X.transpose(1, 2) @ X / (2 * C)).contiguous()
    H[3] = -torch.eye(C, device=DEV)
    damps = [(0.01, 0.02, 0.05)[b % 3] for b in range(B)]
    U, info = ops.chol_upper_inverse(H, damps, precision=precision)
    for b in range(B):
        Ub, ib = ops.chol_upper_inverse(H[b:b + 1].contiguous(), [damps[b]], precision=precision)
        assert int(ib.item()) == int(info[b].item())
        if b != 3:
            assert torch.equal(Ub[0], U[b])
    assert int(info[3].item()) != 0


def test_chol_reports_failure():
    H = -torch.eye(64, device=DEV)[None].contiguous()
    U, info = ops.chol_upper_inverse(H, 0.01)
    assert int(info.item()) != 0
    with pytest.raises(ValueError):
        _engine.retry_failed(H, U, info.cpu().tolist(), [0.01])


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("sym", [True, False])
def test_find_params_and_fake_quantize(golden, bits, sym):
    m = golden("misc.npz")
    tag = f"fp_b{bits}_{'sym' if sym else 'asym'}_00"
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym)
    x = t(m["fp_x"])
    q.find_params(x)
    q.check()
    close(q.scale.reshape(-1), m[tag + "_scale"].reshape(-1), rtol=1e-6, atol=0)
    close(q.zero.reshape(-1), m[tag + "_zero"].reshape(-1), rtol=0, atol=0)
    fq, qi, _ = q.fake_quantize(x)
    close(qi, m[tag + "_q"], rtol=0, atol=0)
    close(fq, m[tag + "_fq"], rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("bits,sym", [(4, True), (3, False), (2, False)])
def test_find_params_groups_matches_per_group(bits, sym):
    """One launch over all groups (static-group set-up) = one call per group,
    bit for bit, ragged last group included."""
    g = torch.Generator(device=DEV).manual_seed(bits)
    rows, C, gs = 300, 1376, 128
    W = torch.randn(rows, C, device=DEV, generator=g) * 0.02
    W[:, 7] *= 40
    ng = (C + gs - 1) // gs
    s1, z1 = torch.empty(rows, ng, device=DEV), torch.empty(rows, ng, device=DEV)
    ops.find_params_groups(s1, z1, W, bits, sym, gs)
    s2, z2 = torch.empty_like(s1), torch.empty_like(z1)
    for gi in range(ng):
        ops.find_params(s2, z2, W[:, gi * gs:(gi + 1) * gs], bits, sym, param_col=gi)
    assert torch.equal(s1, s2) and torch.equal(z1, z2)


@pytest.mark.parametrize("dtype,T,C", [(torch.bfloat16, 2048, 4096), (torch.bfloat16, 300, 1376),
                                       (torch.bfloat16, 77, 200), (torch.float32, 513, 640)])
def test_sq_colsum(dtype, T, C):
    """acc <- acc * keep + scale * sum_t X[t]^2 (the act_square running mean of
    G2PTQ / GuidedQuant add_batch), vectorized BF16 path and general path."""
    g = torch.Generator(device=DEV).manual_seed(T)
    X = (torch.randn(T, C, device=DEV, generator=g) * 3).to(dtype)
    acc0 = torch.rand(C, device=DEV, generator=g)
    acc = acc0.clone()
    ops.sq_colsum(acc, X, keep=0.25, scale=1.0 / 4096)
    ref = acc0.double() * 0.25 + (X.double() ** 2).sum(0) / 4096
    torch.testing.assert_close(acc.double(), ref, rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_pack_int32(golden, bits):
    m = golden("misc.npz")
    out = ops.pack_int32(t(m[f"pack_b{bits}_codes"], torch.int8), bits)
    np.testing.assert_array_equal(out.cpu().numpy(), m[f"pack_b{bits}_packed"])


# ---------------------------------------------------------------------------
# block kernels (the reference's run_eager boundary)
# ---------------------------------------------------------------------------

BLOCK_NAMES = ["symmetric_2bit_tail", "asymmetric_2bit_tail", "symmetric_4bit_batched",
               "asymmetric_4bit_batched", "symmetric_8bit_small", "asymmetric_8bit_small",
               "asymmetric_3bit_fullblock", "symmetric_4bit_fullblock"]


@pytest.mark.parametrize("name", BLOCK_NAMES)
def test_block_kernels_vs_reference(golden, name):
    g = golden("blocks.npz")
    k = lambda s: t(g[f"{name}__{s}"])
    maxq = int(g[f"{name}__maxq"])
    w = k("weight")
    qi, er = torch.empty_like(w), torch.empty_like(w)
    W = w.clone()
    gptq_utils.run_eager(W, k("hinv"), k("scale"), k("zero"), maxq, int_weight=qi, error=er)
    close(qi, g[f"{name}__gptq_int"], rtol=0, atol=0)
    close(W, g[f"{name}__gptq_q"])
    close(er, g[f"{name}__gptq_err"])
    W, gh = w.clone(), k("ghinv")
    g2ptq_utils.run_eager(W, k("hinv"), k("scale"), k("zero"), k("z"), gh, maxq, int_weight=qi,
                          error=er)
    close(qi, g[f"{name}__g2ptq_int"], rtol=0, atol=0)
    close(W, g[f"{name}__g2ptq_q"])
    close(er, g[f"{name}__g2ptq_err"])
    close(gh, g[f"{name}__g2ptq_ghinv"])
    W = w.clone()
    gptaq_utils.run_eager(W, k("hinv"), k("p"), k("scale"), k("zero"), maxq, int_weight=qi,
                          error=er)
    close(qi, g[f"{name}__gptaq_int"], rtol=0, atol=0)
    close(W, g[f"{name}__gptaq_q"])
    close(er, g[f"{name}__gptaq_err"])


@pytest.mark.parametrize("coupled", [False, True])
def test_block_kernels_at_rounding_ties(coupled):
    """Weights whose quotient w / s sits on or within two units in the last
    place of a half-integer: the block kernels take the quotient from a
    multiply by 1 / s and must fall back to the division exactly where the
    rounding could differ.  ``coupled`` adds small off-diagonal U entries, so
    that the later columns move off the ties through the updates."""
    rng = np.random.default_rng(11)
    B, cols, R, maxq = 2, 128, 320, 7
    scale = rng.uniform(1e-3, 1e-2, (B, cols, R)).astype(np.float32)
    zero = np.zeros_like(scale)
    n = rng.integers(-9, 9, (B, cols, R)).astype(np.float32)
    w = ((n + np.float32(0.5)) * scale).astype(np.float32)
    steps = rng.integers(-2, 3, w.shape)
    for _ in range(2):
        w = np.where(steps > 0, np.nextafter(w, np.float32(np.inf)), w)
        w = np.where(steps < 0, np.nextafter(w, np.float32(-np.inf)), w)
        steps = steps - np.sign(steps)
    hinv = np.zeros((B, cols, cols), np.float32)
    idx = np.arange(cols)
    hinv[:, idx, idx] = rng.uniform(0.5, 1.5, (B, cols)).astype(np.float32)
    if coupled:
        hinv += np.triu(rng.standard_normal((B, cols, cols)).astype(np.float32) * 1e-3, 1)
    ratio = w / scale
    assert np.mean(np.abs(np.abs(ratio - np.floor(ratio)) - 0.5) < 1e-5) > 0.5
    wt, qi = t(w), torch.empty(B, cols, R, device=DEV)
    er = torch.empty_like(qi)
    W = wt.clone()
    gptq_utils.run_eager(W, t(hinv), t(scale), t(zero), maxq, int_weight=qi, error=er)
    ow, oq, oe = ocomp.gptq_block(w, hinv, scale, zero, maxq)
    close(qi, oq, rtol=0, atol=0)
    close(W, ow)
    close(er, oe)
    p = np.triu(rng.standard_normal((B, cols, cols)).astype(np.float32) * 1e-3, 1)
    W = wt.clone()
    gptaq_utils.run_eager(W, t(hinv), t(p), t(scale), t(zero), maxq, int_weight=qi, error=er)
    ow, oq, oe = ocomp.gptaq_block(w, hinv, p, scale, zero, maxq)
    close(qi, oq, rtol=0, atol=0)
    close(W, ow)
    close(er, oe)
    z = (rng.standard_normal((B, cols, R)) * 1e-4).astype(np.float32)
    gh0 = (rng.standard_normal((B, cols, R)) * 1e-6).astype(np.float32)
    W, gh = wt.clone(), t(gh0)
    g2ptq_utils.run_eager(W, t(hinv), t(scale), t(zero), t(z), gh, maxq, int_weight=qi,
                          error=er)
    ow, oq, oe, og = ocomp.g2ptq_block(w, hinv, scale, zero, z, gh0, maxq)
    close(qi, oq, rtol=0, atol=0)
    close(W, ow)
    close(er, oe)
    close(gh, og)


# ---------------------------------------------------------------------------
# add_batch through the objects
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["f32", "bf16"])
@pytest.mark.parametrize("stage_tokens", [16384, 50])
def test_gptq_add_batch(golden, tag, stage_tokens, monkeypatch):
    monkeypatch.setattr(_engine, "STAGE_TOKENS", stage_tokens)
    g = golden("hessians.npz")
    C = g[f"gptq_{tag}_H"].shape[0]
    lin = linear(np.zeros((32, C), np.float32))
    obj = gptq_utils.GPTQ([lin])
    dt = torch.float32 if tag == "f32" else torch.bfloat16
    for i in range(4):
        obj.add_batch(0, t(g[f"gptq_{tag}_x{i}"], dt), None)
    assert int(obj.nsamples[0]) == int(g[f"gptq_{tag}_n"])
    assert rel_fro(obj.H[0], g[f"gptq_{tag}_H"]) < 1e-5


def test_g2ptq_add_batch(golden):
    g = golden("hessians.npz")
    C = g["g2ptq_H"].shape[-1]
    lin = linear(np.zeros((32, C), np.float32))
    sals = [t(g[f"g2ptq_s{i}"]) for i in range(3)]
    obj = g2ptq_utils.G2PTQ([lin], [list(sals)], [torch.zeros(32, C, device=DEV)], num_groups=4)
    for i in range(3):
        obj.add_batch(0, t(g[f"g2ptq_x{i}"]), None)
    assert int(obj.index[0]) == int(g["g2ptq_index"])
    assert rel_fro(obj.H[0], g["g2ptq_H"]) < 1e-5
    assert rel_fro(obj.act_square[0], g["g2ptq_act_square"]) < 1e-5


def test_gptaq_add_batch(golden):
    g = golden("hessians.npz")
    C = g["gptaq_H"].shape[0]
    lin = linear(np.zeros((32, C), np.float32))
    obj = gptaq_utils.GPTAQ([lin])
    for i in range(3):
        obj.fp_inp[0].append(t(g[f"gptaq_fp{i}"])[0])
        obj.add_batch(0, t(g[f"gptaq_x{i}"]), None)
    assert rel_fro(obj.H[0], g["gptaq_H"]) < 1e-5
    assert rel_fro(obj.dXXT[0], g["gptaq_dXXT"]) < 1e-5


def test_guided_add_batch(golden):
    g = golden("hessians.npz")
    C = g["guided_H"].shape[-1]
    lin = linear(np.zeros((32, C), np.float32))
    obj = gptq_guided_utils.GPTQGuided([lin], [t(g["guided_sal"])], num_groups=4)
    for i in range(2):
        obj.add_batch(0, t(g[f"guided_x{i}"]), None)
    assert rel_fro(obj.H[0], g["guided_H"]) < 1e-5
    assert rel_fro(obj.act_square[0], g["guided_act_square"]) < 1e-5


# ---------------------------------------------------------------------------
# whole fasterquant pipelines vs the reference
# ---------------------------------------------------------------------------

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


def frac_close(a, b):
    a = a.detach().float().cpu().numpy() if torch.is_tensor(a) else a
    return float(np.mean(np.isclose(a, b, rtol=2e-5, atol=2e-5)))


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_gptq_fasterquant_vs_reference(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W, H = g[f"{name}__W"], g[f"{name}__H"]
    B, R, C = W.shape
    layers = [linear(W[b]) for b in range(B)]
    obj = gptq_utils.GPTQ(layers)
    obj.quantizer = quantizers(bits, sym, C, gs)
    obj.H = t(H).clone()
    obj.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act,
                    export_compressed_tensors=(gs != 40 or act))
    Q = torch.stack([l.weight.data for l in layers])
    ref_Q = g[f"{name}__gptq_Q"]
    assert frac_close(Q, ref_Q) >= 0.999
    loss, ref_loss = proxy_loss(W, Q.cpu().numpy(), H), proxy_loss(W, ref_Q, H)
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-3)
    if gs != 40 or act:
        ref_int = g[f"{name}__gptq_W_int"]
        for b, l in enumerate(layers):
            packed = l._export_qparams["weight_packed"].cpu().numpy()
            from oracle.export import pack_to_int32
            ref_packed = pack_to_int32(ref_int[b].astype(np.int8), bits)
            assert float(np.mean(packed == ref_packed)) >= 0.99
            shape = l._export_qparams["weight_shape"]
            assert shape.dtype == torch.int64 and shape.cpu().tolist() == [R, C]


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_gptaq_fasterquant_vs_reference(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W, H, D = g[f"{name}__W"], g[f"{name}__H"], g[f"{name}__gptaq_dXXT"]
    B, R, C = W.shape
    layers = [linear(W[b]) for b in range(B)]
    obj = gptaq_utils.GPTAQ(layers)
    obj.quantizer = quantizers(bits, sym, C, gs)
    obj.H = t(H).clone()
    obj.dXXT = t(D).clone()
    obj.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act)
    Q = torch.stack([l.weight.data for l in layers])
    assert frac_close(Q, g[f"{name}__gptaq_Q"]) >= 0.999


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_g2ptq_fasterquant_vs_reference(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W = g[f"{name}__W"]
    B, R, C = W.shape
    layers = [linear(W[b]) for b in range(B)]
    obj = g2ptq_utils.G2PTQ(layers, [None] * B, [t(x) for x in g[f"{name}__g2_grad"]],
                            num_groups=4)
    obj.quantizer = quantizers(bits, sym, C, gs)
    obj.H = t(g[f"{name}__g2_H"]).clone()
    obj.act_square = t(g[f"{name}__g2_act_square"]).clone()
    obj.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act,
                    enable_gradient_update=True, alpha=1.0)
    Q = torch.stack([l.weight.data for l in layers])
    assert frac_close(Q, g[f"{name}__g2ptq_Q"]) >= 0.999


@pytest.mark.parametrize("case", FQ_CASES, ids=[c[0] for c in FQ_CASES])
def test_guided_fasterquant_vs_reference(golden, case):
    g = golden("fasterquant.npz")
    name, bits, sym, gs, act, blk = case
    W = g[f"{name}__W"]
    B, R, C = W.shape
    layers = [linear(W[b]) for b in range(B)]
    obj = gptq_guided_utils.GPTQGuided(layers, [t(x) for x in g[f"{name}__guided_sal"]],
                                       num_groups=4)
    obj.quantizer = quantizers(bits, sym, C, gs)
    obj.H = t(g[f"{name}__guided_H"]).clone()
    obj.act_square = t(g[f"{name}__guided_act_square"]).clone()
    obj.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act)
    Q = torch.stack([l.weight.data for l in layers])
    assert frac_close(Q, g[f"{name}__guided_Q"]) >= 0.999


# ---------------------------------------------------------------------------
# larger shapes against the numpy oracle
# ---------------------------------------------------------------------------

def synthetic_hessian(C, T, seed, outliers=4, calls=4):
    """Activations of ``calls`` sequences and the oracle's running Hessian over them."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((calls, T // calls, C)).astype(np.float32)
    X[..., rng.choice(C, outliers, replace=False)] *= 20.0
    H = np.zeros((C, C), np.float32)
    n = 0
    for s in range(calls):
        H, n = ohess.gptq_add_batch(H, n, X[s:s + 1])
    return X, H


@pytest.mark.parametrize("rows,cols,bits,sym,gs,act", [
    (512, 1376, 4, False, 128, False),   # tiny-config down_proj: ragged last block
    (384, 512, 4, True, 128, True),
    (256, 768, 3, False, 128, True),
])
def test_gptq_pipeline_vs_oracle(rows, cols, bits, sym, gs, act):
    rng = np.random.default_rng(rows + cols)
    W = (rng.standard_normal((1, rows, cols)) * 0.02).astype(np.float32)
    X, H = synthetic_hessian(cols, 2048, cols)
    layers = [linear(W[0])]
    obj = gptq_utils.GPTQ(layers)
    obj.quantizer = quantizers(bits, sym, cols, gs)
    for s in range(X.shape[0]):
        obj.add_batch(0, t(X[s:s + 1]), None)
    assert rel_fro(obj.H[0], H) < 1e-5
    Hd = obj.H.clone()
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=gs, actorder=act, static_groups=act)
    Q = layers[0].weight.data[None].cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(bits, sym), cols, gs)
    Qo, Wio, _, _ = ofq.gptq_fasterquant(W, Hd.cpu().numpy(), oq, 128, 0.01, gs, act, act,
                                         route="ul")
    assert float(np.mean(np.isclose(Q, Qo, rtol=2e-5, atol=2e-5))) >= 0.999
    l_gpu, l_or = proxy_loss(W, Q, Hd.cpu().numpy()), proxy_loss(W, Qo, Hd.cpu().numpy())
    np.testing.assert_allclose(l_gpu, l_or, rtol=1e-3)


def test_moe_experts_layer_batched_vs_oracle():
    """Layer-batched expert quantization (BASELINE configs[3] in miniature):
    eight same-shape experts in one GPTQ object, each with its own Hessian
    from a ragged number of routed tokens (add_batch per expert index, 2-D
    routed-token inputs), W4 group 128, act-order with static groups; every
    expert against the oracle on its own Hessian."""
    rng = np.random.default_rng(30)
    E, R, C, gs = 8, 192, 384, 128
    W = (rng.standard_normal((E, R, C)) * 0.02).astype(np.float32)
    layers = [linear(W[e]) for e in range(E)]
    obj = gptq_utils.GPTQ(layers)
    obj.quantizer = quantizers(4, True, C, gs)
    Hs = []
    for e in range(E):
        H, n = np.zeros((C, C), np.float32), 0
        for call in range(3):  # three forward batches, routed-token counts differ
            T = int(rng.integers(40, 700))
            x = rng.standard_normal((T, C)).astype(np.float32)
            x[:, e] *= 15.0
            obj.add_batch(e, t(x), None)
            H, n = ohess.gptq_add_batch(H, n, x)
        Hs.append(H)
    Hd = obj.H.clone()
    for e in range(E):
        assert rel_fro(Hd[e], Hs[e]) < 1e-5
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=gs, actorder=True, static_groups=True,
                    export_compressed_tensors=True)
    Q = torch.stack([l.weight.data for l in layers]).cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(4, True), C, gs)
    Qo, _, _, _ = ofq.gptq_fasterquant(W, Hd.cpu().numpy(), oq, 128, 0.01, gs, True, True,
                                       route="ul")
    for e in range(E):
        assert float(np.mean(np.isclose(Q[e], Qo[e], rtol=2e-5, atol=2e-5))) >= 0.999, e
        np.testing.assert_allclose(proxy_loss(W[e:e + 1], Q[e:e + 1], Hd[e:e + 1].cpu().numpy()),
                                   proxy_loss(W[e:e + 1], Qo[e:e + 1], Hd[e:e + 1].cpu().numpy()),
                                   rtol=1e-3)
        assert layers[e]._export_qparams["weight_packed"].shape[0] == R


@pytest.mark.parametrize("dtype", [torch.float32, torch.int8])
@pytest.mark.parametrize("nl,rows,C", [(1, 37, 4096), (3, 16, 768), (2, 5, 600), (1, 3, 14336)])
def test_permute_cols_matches_indexing(dtype, nl, rows, C):
    """Act-order column permutation and its inverse, exact against indexing:
    the shared-memory staged kernel (C a multiple of 16) and the direct one."""
    g = torch.Generator(device=DEV).manual_seed(C + rows)
    if dtype == torch.float32:
        src = torch.randn(nl, rows, C, device=DEV, generator=g)
    else:
        src = torch.randint(-8, 8, (nl, rows, C), device=DEV, generator=g).to(torch.int8)
    perm = torch.randperm(C, device=DEV, generator=g)
    fwd = ops.permute_cols(src, perm)
    assert torch.equal(fwd, src[:, :, perm])
    back = ops.permute_cols(fwd, perm, inverse=True)
    assert torch.equal(back, src)
