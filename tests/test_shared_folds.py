"""Shared Gram folds of quantizer objects fed the same tensors (FoldGroup).

CPU tests drive the staging mixin with a float64 stand-in object (stage copy
and fold done by torch on the CPU) and compare every call pattern with the
same calls made with sharing off: identical Hessians, fewer folds.  The GPU
test compares real GPTQ objects with and without sharing (bit-identical).
"""

import pytest
import torch

from g2ptq_b200 import ops
from g2ptq_b200.gptq_utils import _engine


class FakeObj(_engine.StagingMixin):
    """One-layer object with the GPTQ fold rule ``H <- H n_old/n_new +
    (2/n_new) X^T X`` in float64 on the CPU."""

    _share_folds = True

    def __init__(self, C, layers=1):
        self.columns, self.dev, self.num_layers = C, torch.device("cpu"), layers
        self._H = torch.zeros(layers, C, C, dtype=torch.float64)
        self._n, self._n_folded = [0] * layers, [0] * layers
        self._init_stages()
        self.folds = 0
        self.fold_counts = []   # (n_old, n_new) of every fold this object made
        self.rescales = 0

    def add_batch(self, idx, inp):
        if inp.dim() == 2:
            inp = inp.unsqueeze(0)
        self._n[idx] += inp.shape[0]
        x = _engine.as_rows(inp, self.columns)
        if not self._shared_call(idx, x, inp.shape[0]):
            self._append(idx, x)

    def _fold(self, idx, X, sub, scales, n_new=None):
        n_old = self._n_folded[idx]
        n_new = self._n[idx] if n_new is None else n_new
        X = X.double()
        self._H[idx] = self._H[idx] * (n_old / n_new) + (2.0 / n_new) * (X.T @ X)
        self._n_folded[idx] = n_new
        self.folds += 1
        self.fold_counts.append((n_old, n_new))

    def _copy_folded(self, idx, src, src_idx):
        self._H[idx].copy_(src._H[src_idx])
        self._n_folded[idx] = src._n_folded[src_idx]

    def _settle(self, idx):
        n, nf = self._n[idx], self._n_folded[idx]
        if n != nf and n > 0:
            self._H[idx] *= nf / n
            self._n_folded[idx] = n
            self.rescales += 1

    def H(self):
        self._flush_all()
        return self._H[0]


@pytest.fixture
def cpu_staging(monkeypatch):
    def stage_tokens(buf, row0, x, sub=None):
        buf[row0:row0 + x.shape[0]].copy_(x)
    monkeypatch.setattr(ops, "stage_tokens", stage_tokens)
    monkeypatch.setattr(_engine, "STAGE_TOKENS", 8)   # small windows: many folds


def run(pattern, share, monkeypatch, C=6):
    """``pattern``: list of (object index, tensor) calls; returns the
    objects' Hessians (after a flush of each) and the total number of folds."""
    monkeypatch.setattr(_engine, "SHARE_FOLDS", share)
    n_obj = 1 + max(i for i, _ in pattern)
    objs = [FakeObj(C) for _ in range(n_obj)]
    for i, x in pattern:
        objs[i].add_batch(0, x)
    Hs = [o.H().clone() for o in objs]
    run.objs = objs
    return Hs, sum(o.folds for o in objs)


def inputs(n, C=6, T=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(1, T, C, generator=g) for _ in range(n)]


def check(pattern, monkeypatch):
    H1, f1 = run(pattern, True, monkeypatch)
    H0, f0 = run(pattern, False, monkeypatch)
    for a, b in zip(H1, H0):
        assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)
    return f1, f0


def test_lockstep_objects_fold_once(cpu_staging, monkeypatch):
    """Same Hessians with a third of the folds, and the folds use the sample
    counts a lone object uses (so the GPU results are bit-identical)."""
    xs = inputs(9)
    pattern = [(o, x) for x in xs for o in range(3)]        # q, k, v per sample
    _, f1 = run(pattern, True, monkeypatch)
    shared = run.objs
    _, f0 = run(pattern, False, monkeypatch)
    alone = run.objs
    assert f1 * 3 == f0
    assert shared[0].fold_counts == alone[0].fold_counts == [(0, 5), (5, 9), (9, 9)][:len(
        alone[0].fold_counts)]
    for a, b in zip(shared, alone):
        assert torch.equal(a._H, b._H) and a.rescales == 0 and a._n_folded == b._n_folded


def test_two_groups_side_by_side(cpu_staging, monkeypatch):
    a, b = inputs(7, seed=1), inputs(7, seed=2)
    pattern = []
    for xa, xb in zip(a, b):
        pattern += [(0, xa), (1, xa), (2, xb), (3, xb), (4, xa)]
    f1, f0 = check(pattern, monkeypatch)
    assert f1 * 5 == f0 * 2


def test_member_diverges_mid_window(cpu_staging, monkeypatch):
    xs, other = inputs(6), inputs(3, seed=5)
    pattern = [(o, x) for x in xs[:2] for o in range(3)]
    pattern += [(0, xs[2]), (1, other[0]), (2, xs[2])]
    pattern += [(o, x) for x in xs[3:] for o in (0, 2)] + [(1, other[1]), (1, other[2])]
    check(pattern, monkeypatch)


def test_member_lags_across_windows(cpu_staging, monkeypatch):
    xs = inputs(12)
    pattern = [(0, x) for x in xs[:6]] + [(1, x) for x in xs[:3]] + [(0, x) for x in xs[6:]]
    pattern += [(1, x) for x in xs[3:]]
    check(pattern, monkeypatch)


def test_flush_of_a_lagging_member(cpu_staging, monkeypatch):
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    xs = inputs(5)
    a, b = FakeObj(6), FakeObj(6)
    for x in xs[:3]:
        a.add_batch(0, x)
        b.add_batch(0, x)
    a.add_batch(0, xs[3])
    Hb = b.H().clone()                         # b lags a by one call, then reads H
    for x in xs[3:]:
        b.add_batch(0, x)
    a.add_batch(0, xs[4])
    monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
    ref = FakeObj(6)
    for x in xs[:3]:
        ref.add_batch(0, x)
    assert torch.allclose(Hb, ref.H(), rtol=1e-12, atol=1e-12)
    for x in xs[3:]:
        ref.add_batch(0, x)
    assert torch.allclose(a.H(), ref.H(), rtol=1e-12, atol=1e-12)
    assert torch.allclose(b.H(), ref.H(), rtol=1e-12, atol=1e-12)


def test_in_place_write_between_calls_is_not_shared(cpu_staging, monkeypatch):
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    x = inputs(1)[0]
    a, b = FakeObj(6), FakeObj(6)
    a.add_batch(0, x)
    x.mul_(2.0)                                 # bumps the version counter
    b.add_batch(0, x)
    assert torch.allclose(b.H(), 2.0 * x[0].double().T @ x[0].double())
    assert not torch.allclose(a.H(), b.H())


def test_same_storage_different_sample_count_is_not_folded_together(cpu_staging, monkeypatch):
    x = inputs(1, T=4)[0]
    pattern = [(0, x), (1, x.reshape(2, 2, 6)), (0, x), (1, x.reshape(2, 2, 6))]
    check(pattern, monkeypatch)


def test_late_object_does_not_join_a_folded_group(cpu_staging, monkeypatch):
    xs = inputs(10)
    pattern = [(0, x) for x in xs] + [(1, x) for x in xs]
    f1, f0 = check(pattern, monkeypatch)
    assert f1 == f0


@pytest.mark.gpu
def test_shared_folds_bit_identical_on_gpu(monkeypatch):
    """q/k/v-style objects fed one tensor: Hessians and quantized weights
    bit-identical with and without sharing."""
    from g2ptq_b200.gptq_utils import gptq_utils, common_utils
    from g2ptq_b200.utils.quant_utils import WeightQuantizer

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    C, seqs = 512, 12
    X = torch.randn(seqs, 2048, C, device=dev, generator=g).to(torch.bfloat16)
    Ws = [torch.randn(r, C, device=dev, generator=g) * 0.02 for r in (512, 128, 128)]

    def build(share):
        monkeypatch.setattr(_engine, "SHARE_FOLDS", share)
        objs = []
        for W in Ws:
            lin = torch.nn.Linear(C, W.shape[0], bias=False, device=dev)
            lin.weight.data = W.clone()
            o = gptq_utils.GPTQ([lin])
            q = WeightQuantizer()
            q.configure(4, perchannel=True, sym=True)
            o.quantizer = common_utils.make_group_quantizers(q, C, 128)
            objs.append(o)
        for s in range(seqs):
            xs = X[s:s + 1]
            for o in objs:
                o.add_batch(0, xs, None)
        Hs = [o.H.clone() for o in objs]
        for o in objs:
            o.fasterquant(blocksize=128, percdamp=0.01, groupsize=128, actorder=True,
                          static_groups=True)
        return Hs, [o.layers[0].weight.data.clone() for o in objs]

    H1, Q1 = build(True)
    H0, Q0 = build(False)
    for a, b in zip(H1 + Q1, H0 + Q0):
        assert torch.equal(a, b)


def test_member_left_behind_by_a_triggered_fold(cpu_staging, monkeypatch):
    """a's fifth call folds the full window (its count includes that call);
    b, one call behind, reads H at once: it leaves with nothing pending and
    rescales to its own count."""
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    xs = inputs(6)
    a, b = FakeObj(6), FakeObj(6)
    for x in xs[:4]:
        a.add_batch(0, x)
        b.add_batch(0, x)
    a.add_batch(0, xs[4])
    Hb = b.H().clone()
    b.add_batch(0, xs[5])
    monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
    r4, r5 = FakeObj(6), FakeObj(6)
    for x in xs[:4]:
        r4.add_batch(0, x)
    for x in xs[:5]:
        r5.add_batch(0, x)
    rb = FakeObj(6)
    for x in xs[:4] + [xs[5]]:
        rb.add_batch(0, x)
    assert torch.allclose(Hb, r4.H(), rtol=1e-12, atol=1e-12)
    assert torch.allclose(a.H(), r5.H(), rtol=1e-12, atol=1e-12)
    assert torch.allclose(b.H(), rb.H(), rtol=1e-12, atol=1e-12)


def test_call_without_tokens_rescales_like_the_reference(cpu_staging, monkeypatch):
    """gptq_utils.py:119-126 with an empty input: H <- H n/(n+1), nothing added."""
    monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
    x = inputs(1)[0]
    o = FakeObj(6)
    o.add_batch(0, x)
    H1 = o.H().clone()
    o.add_batch(0, torch.zeros(1, 0, 6))
    assert torch.allclose(o.H(), H1 / 2, rtol=1e-12, atol=1e-12)


class _RoleObj:
    _share_factor = True

    def __init__(self, group, exposed=False, layers=1):
        self._groups = [group] * layers
        self._h_exposed = exposed
        self.num_layers = layers


def test_layers_of_multi_layer_objects_share(cpu_staging, monkeypatch):
    """Layer 1 of one object and layer 0 of another, fed the same tensors,
    share; layer 0 of the first, fed others, stays alone."""
    def go(share):
        monkeypatch.setattr(_engine, "SHARE_FOLDS", share)
        xs, ys = inputs(9, seed=3), inputs(9, seed=4)
        a, b = FakeObj(6, layers=2), FakeObj(6)
        for x, y in zip(xs, ys):
            a.add_batch(0, y)
            a.add_batch(1, x)
            b.add_batch(0, x)
        a._flush_all()
        b._flush_all()
        return a._H.clone(), b._H.clone(), a.folds + b.folds
    Ha1, Hb1, f1 = go(True)
    Ha0, Hb0, f0 = go(False)
    assert torch.equal(Ha1, Ha0) and torch.equal(Hb1, Hb0)
    assert f0 - f1 == 3      # the shared pair folds once per window instead of twice


def test_member_leaving_mid_window_keeps_the_others_exact(cpu_staging, monkeypatch):
    """One member leaves (its statistics handed out and dropped, as fasterquant
    does) in the middle of a window; the remaining members go on sharing."""
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    xs = inputs(7)
    objs = [FakeObj(6) for _ in range(3)]
    for x in xs[:3]:
        for o in objs:
            o.add_batch(0, x)
    H_left = objs[0].H().clone()
    objs[0]._leave_groups()
    for x in xs[3:]:
        for o in objs[1:]:
            o.add_batch(0, x)
    monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
    r3, r7 = FakeObj(6), FakeObj(6)
    for x in xs[:3]:
        r3.add_batch(0, x)
    for x in xs:
        r7.add_batch(0, x)
    assert torch.allclose(H_left, r3.H(), rtol=1e-12, atol=1e-12)
    for o in objs[1:]:
        assert torch.allclose(o.H(), r7.H(), rtol=1e-12, atol=1e-12)


def test_factor_roles(monkeypatch):
    """One owner per fold group; members whose H was handed out, groupless or
    multi-layer objects, and groups with one eligible member share nothing."""
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    g1, g2, g3 = object(), object(), object()
    objs = [_RoleObj(None), _RoleObj(g1), _RoleObj(g2), _RoleObj(g1), _RoleObj(g1, exposed=True),
            _RoleObj(g3), _RoleObj(g2, layers=2), _RoleObj(g1)]
    roles = _engine.factor_roles(objs)
    assert sorted(roles) == [1, 3, 7]
    assert roles[1][0] == "factor_out" and roles[3][0] == roles[7][0] == "factor_in"
    assert roles[1][1] is roles[3][1] is roles[7][1]
    monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
    assert _engine.factor_roles(objs) == {}


@pytest.mark.gpu
def test_shared_factor_in_fasterquant_all(monkeypatch):
    """fasterquant_all over q/k/v-style objects fed one tensor factors their
    (bit-identical) Hessian once; quantized weights and export buffers are
    bit-identical to the run without sharing, which factors it three times."""
    from g2ptq_b200.gptq_utils import gptq_utils, common_utils
    from g2ptq_b200.utils.quant_utils import WeightQuantizer

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    C, seqs = 512, 10
    X = torch.randn(seqs, 2048, C, device=dev, generator=g).to(torch.bfloat16)
    Ws = [torch.randn(r, C, device=dev, generator=g) * 0.02 for r in (512, 128, 128, 256)]
    calls = []
    chol = ops.chol_upper_inverse

    def counting(*a, **k):
        calls.append(1)
        return chol(*a, **k)
    monkeypatch.setattr(ops, "chol_upper_inverse", counting)

    def build(share):
        monkeypatch.setattr(_engine, "SHARE_FOLDS", share)
        objs = []
        for W in Ws:
            lin = torch.nn.Linear(C, W.shape[0], bias=False, device=dev)
            lin.weight.data = W.clone()
            o = gptq_utils.GPTQ([lin])
            q = WeightQuantizer()
            q.configure(4, perchannel=True, sym=True)
            o.quantizer = common_utils.make_group_quantizers(q, C, 128)
            objs.append(o)
        for s in range(seqs):
            xs = X[s:s + 1]
            for o in objs[:3]:
                o.add_batch(0, xs, None)
            objs[3].add_batch(0, xs.float() * 0.5, None)   # its own input
        calls.clear()
        gptq_utils.fasterquant_all(objs, blocksize=128, percdamp=0.01, groupsize=128,
                                   actorder=True, static_groups=True,
                                   export_compressed_tensors=True)
        torch.cuda.synchronize()
        return len(calls), [(o.layers[0].weight.data.clone(),
                             o.layers[0]._export_qparams["weight_packed"].clone()) for o in objs]

    n1, out1 = build(True)
    n0, out0 = build(False)
    assert (n1, n0) == (2, 4)
    for (w1, p1), (w0, p0) in zip(out1, out0):
        assert torch.equal(w1, w0) and torch.equal(p1, p0)


@pytest.mark.gpu
def test_shared_factor_damp_retry(monkeypatch):
    """The shared Hessian is made indefinite (rank-deficient Gram minus a
    multiple of the identity, written identically into every member), so the
    first damped factorization fails and the damp auto-increment runs: the
    owner re-factors, the followers re-run their compensation with its U.
    Weights and final damps equal those of the unshared run, where each object
    retries on its own."""
    from g2ptq_b200.gptq_utils import gptq_utils, common_utils
    from g2ptq_b200.utils.quant_utils import WeightQuantizer

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    C = 512
    X = torch.randn(2, 32, C, device=dev, generator=g).to(torch.bfloat16)  # rank 64 < C
    Ws = [torch.randn(r, C, device=dev, generator=g) * 0.02 for r in (256, 128, 128)]

    def build(share):
        monkeypatch.setattr(_engine, "SHARE_FOLDS", share)
        objs = []
        for W in Ws:
            lin = torch.nn.Linear(C, W.shape[0], bias=False, device=dev)
            lin.weight.data = W.clone()
            o = gptq_utils.GPTQ([lin])
            q = WeightQuantizer()
            q.configure(4, perchannel=True, sym=True)
            o.quantizer = common_utils.make_group_quantizers(q, C, 128)
            objs.append(o)
        for s in range(2):
            for o in objs:
                o.add_batch(0, X[s:s + 1], None)
        for o in objs:
            o._flush_all()
            H = o._H[0]
            H -= 0.02 * torch.diagonal(H).mean() * torch.eye(C, device=dev)
        gptq_utils.fasterquant_all(objs, blocksize=128, percdamp=0.01, groupsize=128,
                                   actorder=False, static_groups=False)
        torch.cuda.synchronize()
        return [o.layers[0].weight.data.clone() for o in objs], [o._last_damps for o in objs]

    W1, d1 = build(True)
    W0, d0 = build(False)
    assert d1 == d0 and d0[0][0] > 0.02
    for a, b in zip(W1, W0):
        assert torch.equal(a, b)


def test_dropped_members_release_the_window(cpu_staging, monkeypatch):
    """Members dropped without free() leave the group; the others keep their
    exact statistics, and the window's tensors go with the last member, with
    no cycle left for the garbage collector."""
    import gc
    import weakref
    monkeypatch.setattr(_engine, "SHARE_FOLDS", True)
    xs = inputs(7)
    objs = [FakeObj(6) for _ in range(3)]
    gc_was = gc.isenabled()
    gc.disable()
    try:
        for x in xs[:3]:
            for o in objs:
                o.add_batch(0, x)
        group = weakref.ref(objs[0]._groups[0])
        del objs[1:]                                  # dropped mid-window, no free()
        for x in xs[3:]:
            objs[0].add_batch(0, x)
        monkeypatch.setattr(_engine, "SHARE_FOLDS", False)
        ref = FakeObj(6)
        for x in xs:
            ref.add_batch(0, x)
        assert torch.allclose(objs[0].H(), ref.H(), rtol=1e-12, atol=1e-12)
        assert len(group().members) == 1
        del objs
        assert group() is None    # collected by reference counting alone
    finally:
        if gc_was:
            gc.enable()
