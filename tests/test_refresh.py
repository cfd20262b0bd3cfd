"""G2PTQ refresh step: SaliencyCache / GradientCache and the block-loss heads.

CPU tests pin the numpy oracle (oracle/refresh.py) to the reference's own
caches and loss functions (tests/golden/refresh.npz, made by
tests/golden/make_golden.py --only refresh) and check the host logic; GPU
tests compare the CUDA path with the oracle on the same inputs.
"""

import numpy as np
import pytest
import torch

import oracle.refresh as OR
from g2ptq_b200 import ops, _lib
from g2ptq_b200.gptq_utils import g2ptq_utils as G

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                            "refresh.npz"))

# the fixture's scenario (tests/golden/make_golden.py, gen_refresh)
D, HID, V, NG = 16, 32, 40, 4
CALLS = [("block", "kl", 0, 100, True), ("topk", "kl", 8, 300, True),
         ("patch", "mse", 0, 200, False)]
WEIGHTS = {"block": 1.0, "topk": 0.25, "patch": 0.5}
BATCHES = 2


def _relu(v):
    return np.maximum(v, 0.0)


def replay_oracle(params, inputs, draws):
    """The fixture's sequence of calls through the oracle: the block
    ``b(relu(a(x)))`` and its head ``Wh``, backpropagated by hand (float64)."""
    Wa, ba, Wb, bb, Wh = (np.asarray(params[k], np.float64) for k in ("Wa", "ba", "Wb", "bb",
                                                                       "Wh"))
    sal = {"a": {}, "b": {}}
    cache = {"a": {}, "b": {}}
    losses = {}
    for j in range(BATCHES):
        x = np.asarray(inputs[f"x{j}"], np.float64).reshape(-1, D)
        hfp = np.asarray(inputs[f"hfp{j}"], np.float64).reshape(-1, D)
        za = x @ Wa.T + ba
        r = _relu(za)
        h = r @ Wb.T + bb
        n_tok = x.shape[0]
        for lt, kind, topk, _seed, _retain in CALLS:
            if kind == "kl":
                logits, lfp = h @ Wh.T, hfp @ Wh.T
                idx = None
                if topk:
                    idx = np.asarray(draws[f"idx{j}_{lt}"]).reshape(-1, topk)
                    logits = np.take_along_axis(logits, idx, -1)
                    lfp = np.take_along_axis(lfp, idx, -1)
                labels = np.asarray(draws[f"labels{j}_{lt}"]).reshape(-1)
                _, g_s = OR.nll_head(logits, labels)
                loss, g_g = OR.kl_head(logits, lfp)

                def to_h(g, idx=idx):
                    if idx is not None:
                        full = np.zeros((g.shape[0], V))
                        np.put_along_axis(full, idx, g, -1)
                        g = full
                    return g @ Wh
                dh_s, dh_g = to_h(g_s), to_h(g_g)
            else:
                noise = np.asarray(draws[f"noise{j}_{lt}"], np.float64).reshape(-1, D)
                _, dh_s = OR.mse_head(h, h + noise)
                loss, dh_g = OR.mse_head(h, hfp)
            losses[f"loss{j}_{lt}"] = loss
            da_s = (dh_s @ Wb) * (za > 0)
            sal["b"].setdefault(lt, []).append(OR.saliency(dh_s.astype(np.float32), NG))
            sal["a"].setdefault(lt, []).append(OR.saliency(da_s.astype(np.float32), NG))
            da_g = (dh_g @ Wb) * (za > 0)
            for name, gw in (("b", dh_g.T @ r), ("a", da_g.T @ x)):
                c, i = cache[name].get(lt, (None, 0))
                cache[name][lt] = OR.running_mean(c, i, gw.astype(np.float32), n_tok)
    w = OR.normalize_loss_weights(dict(WEIGHTS))
    out = dict(losses)
    for name in ("a", "b"):
        for j in range(BATCHES):
            out[f"sal_{name}{j}"] = OR.weighted_sum([(sal[name][lt][j], w[lt]) for lt in w])
        out[f"grad_{name}"] = OR.weighted_sum([(cache[name][lt][0], w[lt]) for lt in w])
    return out


# ---------------------------------------------------------------------------
# CPU: oracle against the reference's fixtures, host logic
# ---------------------------------------------------------------------------

def test_oracle_cache_hooks_match_reference():
    assert np.array_equal(OR.saliency(GOLDEN["sal_in"], 3), GOLDEN["sal_out"])
    c, i = None, 0
    for k, n in enumerate((10, 4, 7)):
        c, i = OR.running_mean(c, i, GOLDEN[f"rm_in{k}"], n)
    assert np.array_equal(c, GOLDEN["rm_out"])


def test_oracle_refresh_sequence_matches_reference():
    out = replay_oracle(GOLDEN, GOLDEN, GOLDEN)
    for k, v in out.items():
        ref = GOLDEN[k]
        tol = 2e-6 * float(np.abs(ref).max())
        assert np.abs(np.asarray(v, np.float64) - ref).max() <= tol, k


def test_normalize_loss_weights_matches_oracle():
    for lw in ({"block": 1.0}, {"block": 1.0, "patch": 0.3, "gate": 0.2}, {"a": 0.0}):
        assert G.normalize_loss_weights(dict(lw)) == OR.normalize_loss_weights(dict(lw))


def test_summarize_saliency_rejects_mismatched_counts():
    sc = G.SaliencyCache(["a"], 4)
    t = torch.zeros(3, 4)
    sc.saliency_cache["a"] = {"block": [t, t], "patch": [t]}
    with pytest.raises(AssertionError, match="differ between loss types"):
        sc.summarize_saliency({"block": 0.5, "patch": 0.5})


def test_summaries_without_entries():
    sc = G.SaliencyCache(["a"], 4)
    gc = G.GradientCache(["a"], 4)
    sc.summarize_saliency({"block": 1.0})
    gc.summarize_gradients({"block": 1.0})
    assert sc.saliency_cache["a"] == [] and gc.gradients_cache["a"] == 0


def test_hooks_do_nothing_while_disabled():
    sc = G.SaliencyCache(["a"], 4)
    gc = G.GradientCache(["a"], 4)
    sc.grad_hook(torch.ones(2, 8), name="a", loss_type="block")
    gc.current_batch_tokens["a"] = 2
    gc.cache_gradient(torch.ones(2, 8), name="a", loss_type="block")
    assert sc.saliency_cache["a"] == {} and gc.gradients_cache["a"] == {}


def test_refresh_ops_refuse_cpu_tensors():
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.saliency(torch.ones(2, 8), 4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.running_mean(torch.zeros(4), torch.ones(4), 0.5, 0.25, False)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        G.block_loss(_lib.LOSS_MSE, torch.ones(2, 8), target=torch.zeros(2, 8))


def test_forward_hooks_record_outputs_and_token_counts():
    lin = torch.nn.Linear(8, 12)
    sc = G.SaliencyCache(["l"], 4)
    gc = G.GradientCache(["l"], 4)
    sc.set_forward_hook({"l": lin})
    gc.set_forward_hook({"l": lin})
    y = lin(torch.ones(3, 5, 8))
    assert sc.outs["l"] is y and gc.current_batch_tokens["l"] == 15
    sc.clear_hook()
    gc.clear_hook()
    lin(torch.ones(2, 8))
    assert gc.current_batch_tokens["l"] == 15 and sc.handles == [] and gc.handles == []


# ---------------------------------------------------------------------------
# GPU: CUDA path against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("T,R,G_", [(10, 32, 4), (7, 12, 3), (33, 1024, 4), (5, 14336, 4)])
def test_saliency_kernel(dtype, T, R, G_):
    gen = torch.Generator().manual_seed(T * R + G_)
    g = (torch.randn(T, R, generator=gen) * 1e-2).to(dtype)
    got = ops.saliency(g.cuda(), G_).cpu().numpy()
    want = OR.saliency(g.float().numpy(), G_)
    np.testing.assert_allclose(got, want, rtol=2e-6 * np.sqrt(R // G_), atol=0)


@pytest.mark.gpu
def test_saliency_kernel_strided_rows_and_3d_input():
    gen = torch.Generator().manual_seed(5)
    big = torch.randn(2, 6, 72, generator=gen).to(torch.bfloat16).cuda()
    view = big[..., 8:72]                       # row stride 72, 16-byte aligned start
    got = ops.saliency(view, 4).cpu().numpy()
    want = OR.saliency(view.float().cpu().numpy(), 4)
    np.testing.assert_allclose(got, want, rtol=1e-5)
    odd = big[..., 3:67]                        # misaligned start: scalar path
    np.testing.assert_allclose(ops.saliency(odd, 4).cpu().numpy(),
                               OR.saliency(odd.float().cpu().numpy(), 4), rtol=1e-5)


@pytest.mark.gpu
def test_saliency_rejects_indivisible_groups():
    with pytest.raises(RuntimeError, match="is invalid for input"):
        ops.saliency(torch.ones(2, 10, device="cuda"), 4)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(6, 7), (64, 128), (4096, 1000)])
def test_running_mean_kernel(dtype, shape):
    """Bit-exact against torch's own CUDA arithmetic of the reference line
    (g2ptq_utils.py:697-700); the oracle divides on the CPU, where torch
    divides rather than multiplies by the reciprocal, so it agrees to an
    ulp of the operands (absolute, the steps may cancel)."""
    gen = torch.Generator().manual_seed(shape[0])
    gc = G.GradientCache(["w"], 4)
    gc.hooks_enabled = True
    ref = 0
    oc, oi = None, 0
    for i, n_tok in enumerate((10, 4, 7, 2048)):
        gw = torch.randn(*shape, generator=gen).to(dtype).cuda()
        gc.current_batch_tokens["w"] = n_tok
        gc.cache_gradient(gw, name="w", loss_type="block")
        ref = ref * (i / (i + 1))
        ref = ref + gw.float() / (n_tok * (i + 1))
        oc, oi = OR.running_mean(oc, oi, gw.float().cpu().numpy(), n_tok)
    got = gc.gradients_cache["w"]["block"]
    assert torch.equal(got, ref)
    np.testing.assert_allclose(got.cpu().numpy(), oc, rtol=0,
                               atol=4 * 2.0 ** -23 * float(np.abs(oc).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, 4096, 1 << 20])
def test_scaled_accumulate_kernel(n):
    gen = torch.Generator().manual_seed(n)
    xs = [torch.randn(n, generator=gen) for _ in range(3)]
    ws = [0.6, 0.15, 0.25]
    out = torch.empty(n, device="cuda")
    for i, (x, w) in enumerate(zip(xs, ws)):
        ops.scaled_accumulate(out, x.cuda(), w, first=(i == 0))
    want = OR.weighted_sum([(x.numpy(), w) for x, w in zip(xs, ws)])
    assert np.array_equal(out.cpu().numpy(), want)


def _head_oracle(kind, x, t=None, labels=None):
    if kind == _lib.LOSS_KL:
        return OR.kl_head(x, t)
    if kind == _lib.LOSS_NLL:
        return OR.nll_head(x, labels)
    return OR.mse_head(x, t)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [_lib.LOSS_KL, _lib.LOSS_NLL, _lib.LOSS_MSE])
@pytest.mark.parametrize("dtype,rows,V", [(torch.float32, 16, 40), (torch.float32, 9, 37),
                                          (torch.bfloat16, 6, 37), (torch.bfloat16, 32, 128256),
                                          (torch.float16, 8, 4096)])
def test_block_loss_heads(kind, dtype, rows, V):
    """Loss and gradient of each head against the float64 oracle.  Tolerances:
    the loss within 1e-5 of its scale (KL: of the log-sum-exp terms it is
    the difference of); the gradient within 1e-5 of the softmax terms it is
    made of (KL, NLL) or 1e-6 of itself (MSE), plus one rounding to the output
    dtype (half an ulp, and half the fp16 subnormal spacing)."""
    gen = torch.Generator().manual_seed(rows * V + kind)
    scale = 3.0 if kind != _lib.LOSS_MSE else 1.0
    x = (torch.randn(rows, V, generator=gen) * scale).to(dtype)
    t = (x.float() + 0.3 * torch.randn(rows, V, generator=gen)).to(dtype)
    labels = torch.randint(0, V, (rows,), generator=gen)
    labels[rows // 2] = -100
    xc = x.cuda().requires_grad_(True)
    tc = None if kind == _lib.LOSS_NLL else t.cuda()
    lc = labels.cuda() if kind == _lib.LOSS_NLL else None
    loss = G.block_loss(kind, xc, target=tc, labels=lc)
    (loss * 2.5).backward()
    xn, tn = x.float().numpy().astype(np.float64), t.float().numpy().astype(np.float64)
    want_loss, want_grad = _head_oracle(kind, xn, tn, labels.numpy())
    lse_scale = np.abs(xn).max() * rows if kind == _lib.LOSS_KL else abs(want_loss)
    assert abs(float(loss) - want_loss) <= 1e-5 * max(lse_scale, 1.0) + 1e-6
    got = xc.grad.float().cpu().numpy()
    want = 2.5 * want_grad

    def softmax(v):
        e = np.exp(v - v.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)
    if kind == _lib.LOSS_MSE:
        comp = 1e-6 * np.abs(want)
    else:
        other = softmax(tn) if kind == _lib.LOSS_KL else np.abs(want_grad - softmax(xn))
        comp = 1e-5 * 2.5 * (softmax(xn) + other)
    half_ulp = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}[dtype]
    floor = 2.0 ** -25 if dtype == torch.float16 else 0.0
    assert np.all(np.abs(got - want) <= comp + half_ulp * np.abs(want) + floor + 1e-30)
    if kind == _lib.LOSS_NLL:
        assert not got[rows // 2].any()


@pytest.mark.gpu
def test_block_loss_out_of_range_label_gives_nan_loss():
    x = torch.randn(3, 16, device="cuda", requires_grad=True)
    labels = torch.tensor([1, 99, 2], device="cuda")
    loss = G.block_loss(_lib.LOSS_NLL, x, labels=labels)
    assert torch.isnan(loss)
    loss.backward()
    assert not x.grad[1].any()


@pytest.mark.gpu
def test_block_loss_refuses_target_with_grad():
    x = torch.randn(3, 16, device="cuda", requires_grad=True)
    with pytest.raises(NotImplementedError):
        G.block_loss(_lib.LOSS_KL, x, target=x)


def _gpu_block(params):
    nn = torch.nn
    a, b = nn.Linear(D, HID), nn.Linear(HID, D)
    head = nn.Linear(D, V, bias=False)
    with torch.no_grad():
        a.weight.copy_(torch.as_tensor(params["Wa"]))
        a.bias.copy_(torch.as_tensor(params["ba"]))
        b.weight.copy_(torch.as_tensor(params["Wb"]))
        b.bias.copy_(torch.as_tensor(params["bb"]))
        head.weight.copy_(torch.as_tensor(params["Wh"]))
    head.weight.requires_grad_(False)
    return a.cuda(), b.cuda(), head.cuda()


@pytest.mark.gpu
def test_refresh_sequence_on_gpu_matches_oracle():
    """The fixture's sequence through this package's caches and loss
    functions on the GPU; the labels / top-k indices / noise each call drew are
    re-drawn from the same seeds and handed to the oracle."""
    a, b, head = _gpu_block(GOLDEN)
    full = {"a": a, "b": b}
    sc = G.SaliencyCache(["a", "b"], NG)
    sc.set_forward_hook(full)
    gc = G.GradientCache(["a", "b"], NG)
    gc.set_forward_hook(full)
    draws, losses = {}, {}
    for j in range(BATCHES):
        x = torch.as_tensor(GOLDEN[f"x{j}"]).cuda()
        hfp = torch.as_tensor(GOLDEN[f"hfp{j}"]).cuda()
        with torch.enable_grad():
            h = b(torch.relu(a(x)))
            for lt, kind, topk, seed, retain in CALLS:
                args = __import__("types").SimpleNamespace(kl_topk=topk)
                torch.manual_seed(seed + j)
                if kind == "kl":
                    loss = G.compute_kl_grad_hessian(head(h), head(hfp), sc, gc, full, args,
                                                     loss_type=lt, retain_graph=retain)
                    lf = head(hfp).detach()
                    if topk:
                        lf, idx = lf.topk(topk, dim=-1, sorted=False)
                        draws[f"idx{j}_{lt}"] = idx.cpu().numpy()
                    torch.manual_seed(seed + j)
                    draws[f"labels{j}_{lt}"] = torch.distributions.Categorical(
                        logits=lf).sample().cpu().numpy()
                else:
                    loss = G.compute_mse_grad_hessian(h, hfp, sc, gc, full, args, loss_type=lt,
                                                      retain_graph=retain)
                    torch.manual_seed(seed + j)
                    draws[f"noise{j}_{lt}"] = torch.distributions.Normal(
                        loc=torch.zeros_like(h), scale=4.0).sample().cpu().numpy()
                losses[f"loss{j}_{lt}"] = float(loss)
    sc.clear_hook()
    gc.clear_hook()
    w = G.normalize_loss_weights(dict(WEIGHTS))
    sc.summarize_saliency(w)
    gc.summarize_gradients(w)
    want = replay_oracle(GOLDEN, GOLDEN, draws)
    for k, v in losses.items():
        assert abs(v - want[k]) <= 1e-4 * max(abs(want[k]), 1.0), k
    for name in ("a", "b"):
        for j in range(BATCHES):
            got = sc.saliency_cache[name][j].cpu().numpy()
            ref = want[f"sal_{name}{j}"]
            assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), (name, j)
        got = gc.gradients_cache[name].cpu().numpy()
        ref = want[f"grad_{name}"]
        assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), name


@pytest.mark.gpu
def test_refresh_kernels_on_empty_inputs():
    """No tokens: an empty saliency, a zero loss and an empty gradient (the
    reference's torch ops give the same for empty batches)."""
    sal = ops.saliency(torch.empty(0, 64, device="cuda", dtype=torch.bfloat16), 4)
    assert sal.shape == (0, 4)
    for kind in (_lib.LOSS_KL, _lib.LOSS_NLL, _lib.LOSS_MSE):
        x = torch.empty(0, 40, device="cuda", requires_grad=True)
        t = None if kind == _lib.LOSS_NLL else torch.empty(0, 40, device="cuda")
        lab = torch.empty(0, dtype=torch.int64, device="cuda") if kind == _lib.LOSS_NLL else None
        loss = G.block_loss(kind, x, target=t, labels=lab)
        loss.backward()
        assert float(loss.detach()) == 0.0 and x.grad.shape == (0, 40)


@pytest.mark.gpu
def test_mse_gradient_loss_promotes_mixed_dtypes():
    """A bf16 block output against an fp32 target: the gradient loss compares
    them in fp32 (F.mse_loss's type promotion, g2ptq_utils.py:1025), the
    target not rounded to bf16, and the gradient reaches the bf16 output."""
    import types
    g = torch.Generator(device="cuda").manual_seed(9)
    h0 = torch.randn(6, 48, device="cuda", generator=g).to(torch.bfloat16)
    hfp = h0.float() + 1e-3 * torch.randn(6, 48, device="cuda", generator=g)
    lin = torch.nn.Linear(48, 48, bias=False, device="cuda")
    sc = G.SaliencyCache(["l"], 4)
    gc = G.GradientCache(["l"], 4)
    full = {"l": lin}
    sc.set_forward_hook(full)
    gc.set_forward_hook(full)
    with torch.enable_grad():
        h = h0.clone().requires_grad_(True)
        torch.manual_seed(1)
        loss = G.compute_mse_grad_hessian(h, hfp, sc, gc, full, types.SimpleNamespace(),
                                          loss_type="block")
    sc.clear_hook()
    gc.clear_hook()
    want, dh = OR.mse_head(h0.float().cpu().numpy(), hfp.cpu().numpy())
    rounded, _ = OR.mse_head(h0.float().cpu().numpy(),
                             hfp.to(torch.bfloat16).float().cpu().numpy())
    assert abs(float(loss) - want) <= 1e-5 * want
    assert abs(rounded - want) > 1e-3 * want  # the bf16-rounded target would be detected
    assert h.grad is not None and h.grad.dtype == torch.bfloat16
    ref = torch.from_numpy(dh).float().reshape(h.shape).to(torch.bfloat16)
    torch.testing.assert_close(h.grad.cpu(), ref, rtol=1e-2, atol=1e-6)
