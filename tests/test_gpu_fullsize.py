"""Parity at the sizes the benchmark runs (GPU; the oracle runs on the host).

BASELINE configs[1] (Llama-3-8B GPTQ W4 sym g128, act-order with static
groups) has its largest factorization at C = 14336 (mlp.down_proj) and its
largest compensation at 14336 x 4096 (gate/up_proj); configs[2] (G2PTQ W3
asym g128, four row groups, trust radius 1.0) runs 4096 x 4096 linears;
configs[3] quantizes 64-expert chunks of 768 x 2048 experts with ragged
routed-token counts.  Each case here runs that shape through the public
object API and checks:

* the damped inverse-Cholesky factor against an fp64 factor of the same
  matrix, next to the reference's own fp32 chain (``torch.linalg`` Cholesky ->
  ``cholesky_inverse`` -> Cholesky, gptq_utils.py:295-304) measured the same way;
* the compensation: the numpy oracle given this library's factor (so both
  walk the same U) must produce the same integer codes on >= 99.9 % of the
  weights (the GPTQ recursion amplifies rounding-level differences of U into
  code flips, so codes are compared on a shared factor);
* end to end: ``||(W - Q) X||^2`` within 1e-3 relative of the oracle run on an
  fp64 factor of the same Hessian.

Activations follow the benchmark: BF16 N(0, 1) with 4 outlier channels x20,
weights N(0, 0.02) BF16; fewer calibration tokens than the benchmark (the
Hessian's size, not its token count, sets the cost of the path under test).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from g2ptq_b200 import ops  # noqa: E402
from g2ptq_b200.gptq_utils import _engine, gptq_utils, g2ptq_utils  # noqa: E402
from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers  # noqa: E402
from g2ptq_b200.utils.quant_utils import WeightQuantizer  # noqa: E402
from oracle import compensation as ocomp, fasterquant as ofq  # noqa: E402

DEV = torch.device("cuda", 0)


def rel_fro(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def ul_factor_fp64(H, percdamp=0.01):
    """fp64 ``U`` (upper) with ``U^T U = (H + d I)^-1``, d = percdamp * mean diag:
    the upper-lower factorization H + dI = V V^T, U = V^-1."""
    Hd = H.double()
    C = Hd.shape[-1]
    eye = torch.eye(C, dtype=torch.float64, device=H.device)
    Hd = Hd + percdamp * torch.diagonal(Hd, dim1=-2, dim2=-1).mean(-1)[..., None, None] * eye
    L = torch.linalg.cholesky(torch.flip(Hd, (-2, -1)))
    V = torch.flip(L, (-2, -1))
    return torch.linalg.solve_triangular(V, eye.expand_as(V), upper=True)


def reference_chain_fp32(H, percdamp=0.01):
    """The reference's own chain in fp32 (gptq_utils.py:295-304)."""
    C = H.shape[-1]
    Hd = H.clone()
    damp = percdamp * torch.mean(torch.diag(Hd))
    Hd[torch.arange(C), torch.arange(C)] += damp
    L = torch.linalg.cholesky(Hd)
    Hinv = torch.cholesky_inverse(L)
    return torch.linalg.cholesky(Hinv, upper=True)


def activations(C, seqs, seed, seq_len=2048):
    g = torch.Generator(device=DEV).manual_seed(seed)
    idx = torch.randperm(C, device=DEV, generator=g)[:4]
    out = []
    for _ in range(seqs):
        x = torch.randn(1, seq_len, C, device=DEV, generator=g)
        x[..., idx] *= 20.0
        out.append(x.to(torch.bfloat16))
    return out


def bf16_linear(rows, cols, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lin = torch.nn.Linear(cols, rows, bias=False, device=DEV, dtype=torch.bfloat16)
    lin.weight.data = (torch.randn(rows, cols, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    return lin


def quantizers(bits, sym, C, gs=128):
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=False)
    return make_group_quantizers(q, C, gs)


class Capture:
    """Records, for every finished fasterquant, the factor U (act-order
    column order), the Hessian it factored and the integer codes (original
    column order)."""

    def __init__(self, monkeypatch):
        self.items = []
        orig = _engine.Pending.finish
        cap = self

        def finish(self_):
            out = orig(self_)
            cap.items.append({"U": self_.U.detach().clone(), "H": self_.H.detach().clone(),
                              "codes": self_.codes.detach().clone()})
            return out

        monkeypatch.setattr(_engine.Pending, "finish", finish)


def proxy_loss(W, Q, H):
    """sum_b ||(W_b - Q_b) X||^2 up to the Hessian's normalisation, in fp64."""
    d = (W.double() - Q.double())
    return float(torch.einsum("brc,bcd,brd->", d, H.double(), d))


# ---------------------------------------------------------------------------
# damped inverse-Cholesky at the benchmark's column counts
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("C", [8192, 14336])
def test_cholesky_fullsize_vs_fp64(C):
    X = torch.cat([x[0] for x in activations(C, 8, C)])  # 16384 BF16 tokens
    H = torch.zeros(C, C, device=DEV)
    ops.gram_update(H, X, alpha=0.0, beta=2.0 / X.shape[0], precision=1)
    U, info = ops.chol_upper_inverse(H[None].contiguous(), 0.01, precision=1)
    assert int(info.item()) == 0
    U = U[0]
    U64 = ul_factor_fp64(H)
    err = rel_fro(U, U64)
    Uref = reference_chain_fp32(H)
    err_ref = rel_fro(Uref, U64)
    print(f"C={C}: U rel. Frobenius error vs fp64 {err:.2e} (reference fp32 chain {err_ref:.2e})")
    assert err < max(1e-5, 2.0 * err_ref), (err, err_ref)
    assert float(torch.tril(U, -1).abs().max()) == 0.0
    # residual U^T U (H + dI) - I, against the reference chain's
    Hd = H.double() + 0.01 * torch.diagonal(H).double().mean() * torch.eye(
        C, dtype=torch.float64, device=DEV)
    eye = torch.eye(C, dtype=torch.float64, device=DEV)
    res = float(((U.double().T @ U.double()) @ Hd - eye).norm() / C ** 0.5)
    res_ref = float(((Uref.double().T @ Uref.double()) @ Hd - eye).norm() / C ** 0.5)
    print(f"C={C}: residual {res:.2e} (reference fp32 chain {res_ref:.2e})")
    assert res < max(1e-4, 2.0 * res_ref), (res, res_ref)


# ---------------------------------------------------------------------------
# GPTQ W4 sym g128 act-order at the bench's largest shapes
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("rows,cols", [(14336, 4096), (4096, 14336)],
                         ids=["gate_proj_14336x4096", "down_proj_4096x14336"])
def test_gptq_fullsize_vs_oracle(rows, cols, monkeypatch):
    cap = Capture(monkeypatch)
    lin = bf16_linear(rows, cols, rows + cols)
    W = lin.weight.data.float()[None].clone()
    obj = gptq_utils.GPTQ([lin])
    obj.quantizer = quantizers(4, True, cols)
    for x in activations(cols, 8, 43):
        obj.add_batch(0, x, None)
    H = obj.H.clone()
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=128, actorder=True,
                    static_groups=True, export_compressed_tensors=True)
    Q = lin.weight.data.float()[None]
    item = cap.items[-1]
    codes = item["codes"].cpu().numpy()
    # export buffers carry exactly these codes
    packed = ops.pack_int32(item["codes"][0].contiguous(), 4)
    assert torch.equal(lin._export_qparams["weight_packed"], packed)

    Wn, Hn = W.cpu().numpy(), H.cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(4, True), cols, 128)
    _, Wi_o, _, info = ofq.gptq_fasterquant(Wn, Hn, oq, 128, 0.01, 128, True, True,
                                            U=item["U"].cpu().numpy())
    same = float(np.mean(codes == Wi_o.astype(np.int8)))
    print(f"{rows}x{cols}: codes identical to the oracle on the same U: {same:.6f}")
    assert same >= 0.999, same

    # end to end against the oracle on an fp64 factor of the same (permuted) Hessian
    U64 = ul_factor_fp64(item["H"]).float().cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(4, True), cols, 128)
    Qo, _, _, _ = ofq.gptq_fasterquant(Wn, Hn, oq, 128, 0.01, 128, True, True, U=U64)
    Qo_bf16 = torch.from_numpy(Qo).to(torch.bfloat16).float().to(DEV)
    l_gpu, l_or = proxy_loss(W, Q, H), proxy_loss(W, Qo_bf16, H)
    print(f"{rows}x{cols}: loss {l_gpu:.6e} vs oracle(fp64 U) {l_or:.6e}")
    assert abs(l_gpu - l_or) / l_or < 1e-3


# ---------------------------------------------------------------------------
# G2PTQ W3 asym g128, four row groups, trust radius 1.0
# ---------------------------------------------------------------------------

def test_g2ptq_fullsize_vs_oracle(monkeypatch):
    cap = Capture(monkeypatch)
    R = C = 4096
    G = 4
    lin = bf16_linear(R, C, 7)
    W = lin.weight.data.float()[None].clone()
    xs = activations(C, 4, 45)
    g = torch.Generator(device=DEV).manual_seed(44)
    sal, grad = [], torch.zeros(R, C, device=DEV)
    for x in xs:
        go = (torch.randn(x.shape[1], R, device=DEV, generator=g) * 1e-3).to(torch.bfloat16)
        gf = go.float()
        sal.append((gf * gf).reshape(-1, G, R // G).mean(-1))
        grad += (go.T @ x[0]).float() / x.shape[1]
    grad /= len(xs)
    obj = g2ptq_utils.G2PTQ([lin], [list(sal)], [grad], num_groups=G)
    obj.quantizer = quantizers(3, False, C)
    for x in xs:
        obj.add_batch(0, x, None)
    H = obj.H.clone()
    act_sq = obj.act_square.clone()
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=128, actorder=False,
                    static_groups=False, enable_gradient_update=True, alpha=1.0)
    Q = lin.weight.data.float()[None]
    item = cap.items[-1]
    codes = item["codes"].cpu().numpy()

    Wn, Hn = W.cpu().numpy(), H.cpu().numpy()
    args = (Wn, Hn, act_sq.cpu().numpy(), grad[None].cpu().numpy())
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(3, False), C, 128)
    _, Wi_o, _, _ = ofq.g2ptq_fasterquant(*args, oq, G, 128, 0.01, 128, False, False, True, 1.0,
                                          U=item["U"].cpu().numpy())
    same = float(np.mean(codes == Wi_o.astype(np.int8)))
    print(f"G2PTQ {R}x{C}: codes identical to the oracle on the same U: {same:.6f}")
    assert same >= 0.999, same

    U64 = ul_factor_fp64(item["H"]).float().cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(3, False), C, 128)
    Qo, _, _, _ = ofq.g2ptq_fasterquant(*args, oq, G, 128, 0.01, 128, False, False, True, 1.0,
                                        U=U64)
    Qo_bf16 = torch.from_numpy(Qo).to(torch.bfloat16).float().to(DEV)
    Hg = H.view(G, C, C)
    l_gpu = proxy_loss(W.view(G, R // G, C), Q.view(G, R // G, C), Hg)
    l_or = proxy_loss(W.view(G, R // G, C), Qo_bf16.view(G, R // G, C), Hg)
    print(f"G2PTQ {R}x{C}: loss {l_gpu:.6e} vs oracle(fp64 U) {l_or:.6e}")
    assert abs(l_gpu - l_or) / l_or < 1e-3


# ---------------------------------------------------------------------------
# one 64-expert chunk of 768 x 2048 experts, ragged routed tokens
# ---------------------------------------------------------------------------

def test_moe_expert_chunk_vs_oracle(monkeypatch):
    cap = Capture(monkeypatch)
    E, R, C = 64, 768, 2048
    g = torch.Generator(device=DEV).manual_seed(30)
    layers = [bf16_linear(R, C, 1000 + e) for e in range(E)]
    W = torch.stack([l.weight.data.float() for l in layers])
    obj = gptq_utils.GPTQ(layers)
    obj.quantizer = quantizers(4, True, C)
    hidden = activations(C, 2, 46)
    for x in hidden:  # two forward batches, each expert sees its routed tokens
        toks = x[0]
        for e in range(E):
            n = int(torch.randint(256, 4096, (1,), device=DEV, generator=g).item())
            idx = torch.randint(0, toks.shape[0], (n,), device=DEV, generator=g)
            obj.add_batch(e, toks[idx], None)
    H = obj.H.clone()
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=128, actorder=True,
                    static_groups=True, export_compressed_tensors=True)
    Q = torch.stack([l.weight.data.float() for l in layers])
    item = cap.items[-1]
    codes = item["codes"].cpu().numpy()

    Wn, Hn = W.cpu().numpy(), H.cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(4, True), C, 128)
    _, Wi_o, _, _ = ofq.gptq_fasterquant(Wn, Hn, oq, 128, 0.01, 128, True, True,
                                         U=item["U"].cpu().numpy())
    same = np.mean(codes == Wi_o.astype(np.int8), axis=(1, 2))
    print(f"MoE chunk: worst expert's code identity on the same U: {same.min():.6f}")
    assert same.min() >= 0.999, same.min()

    U64 = ul_factor_fp64(item["H"]).float().cpu().numpy()
    oq = ocomp.make_group_quantizers(ocomp.Quantizer(4, True), C, 128)
    Qo, _, _, _ = ofq.gptq_fasterquant(Wn, Hn, oq, 128, 0.01, 128, True, True, U=U64)
    Qo_bf16 = torch.from_numpy(Qo).to(torch.bfloat16).float().to(DEV)
    for e in range(E):
        l_gpu = proxy_loss(W[e:e + 1], Q[e:e + 1], H[e:e + 1])
        l_or = proxy_loss(W[e:e + 1], Qo_bf16[e:e + 1], H[e:e + 1])
        assert abs(l_gpu - l_or) / l_or < 1e-3, (e, l_gpu, l_or)


# ---------------------------------------------------------------------------
# what the benchmark step itself produces
# ---------------------------------------------------------------------------

def test_bench_step_output(monkeypatch):
    """One step of bench.py's workload (7 Llama-3-8B linears, shared folds and
    factors, fasterquant_all on the stream pool) with 4 sequences: every
    linear's weight is the dequantized export (bf16 of scale x code with its
    static group's scale), its packed export holds the codes, and GPTQ beats
    round-to-nearest on the Hessian it was calibrated with."""
    import bench
    cap = Capture(monkeypatch)
    layers = bench.make_layers(torch, DEV)
    W0 = {n: l.weight.data.float().clone() for n, l in layers.items()}
    acts, n_local = bench.make_inputs(torch, DEV, 0, 1, 4, 2048)
    objs = bench.one_step(torch, layers, acts, n_local, 1, 0, None)
    assert len(cap.items) == len(bench.LINEARS)
    by_rows_cols = {}
    for it in cap.items:
        by_rows_cols.setdefault(tuple(it["codes"].shape[1:]), []).append(it)
    for name, rows, cols, grp in bench.LINEARS:
        lin = layers[name]
        qp = lin._export_qparams
        w = lin.weight.data.float()
        assert torch.isfinite(w).all()
        scale = qp["weight_scale"].float()  # [rows, cols / 128]
        cands = [it for it in by_rows_cols[(rows, cols)]
                 if torch.equal(qp["weight_packed"], ops.pack_int32(it["codes"][0].contiguous(),
                                                                     4))]
        assert cands, name
        codes = cands[0]["codes"][0].float()
        assert int(codes.min()) >= -8 and int(codes.max()) <= 7
        deq = (scale.repeat_interleave(128, dim=1)[:, :cols] * codes).to(torch.bfloat16).float()
        # the bf16 scale of the export and the fp32 scale of the write-back
        # differ by the scale's bf16 rounding
        assert float((deq - w).abs().max() / w.abs().max()) < 1e-2, name
    # GPTQ vs round-to-nearest on down_proj's own Hessian
    name = "mlp.down_proj"
    x = acts["down"].reshape(-1, bench.INTER)
    H = torch.zeros(bench.INTER, bench.INTER, device=DEV)
    ops.gram_update(H, x, alpha=0.0, beta=2.0 / n_local, precision=1)
    W = W0[name]
    scale = layers[name]._export_qparams["weight_scale"].float()
    s = scale.repeat_interleave(128, dim=1)
    rtn = (torch.clamp(torch.round(W / s), -8, 7) * s)
    l_gptq = proxy_loss(W[None], layers[name].weight.data.float()[None], H[None])
    l_rtn = proxy_loss(W[None], rtn[None], H[None])
    print(f"down_proj: GPTQ loss {l_gptq:.4e}, RTN loss {l_rtn:.4e}")
    assert l_gptq < 0.9 * l_rtn
    del objs
