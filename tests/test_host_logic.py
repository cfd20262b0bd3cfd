"""Host-side logic: chunking, owner assignment, staged-fold arithmetic and the
multi-rank statistics exchange (gloo, CPU ranks)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from g2ptq_b200.gptq_utils import common_utils
from oracle import hessian as ohess


class FakeModule:
    def __init__(self, rows, cols):
        self.weight = torch.zeros(rows, cols)


def test_build_chunk_specs_groups_by_shape():
    subset = {"q": FakeModule(64, 32), "k": FakeModule(16, 32), "v": FakeModule(16, 32),
              "o": FakeModule(32, 64)}
    specs = common_utils.build_chunk_specs(subset, 1)
    assert [s.chunk_names for s in specs] == [("q",), ("k",), ("v",), ("o",)]
    specs = common_utils.build_chunk_specs(subset, 8)
    assert [s.chunk_names for s in specs] == [("q",), ("k", "v"), ("o",)]
    assert specs[1].num_layers == 2 and specs[1].rows == 16


def test_moe_expert_chunking():
    subset = {f"experts.{e}.gate_proj": FakeModule(768, 2048) for e in range(128)}
    specs = common_utils.build_chunk_specs(subset, 64)
    assert len(specs) == 2 and all(s.num_layers == 64 for s in specs)


def test_partition_layers_lpt():
    class G:
        def __init__(self, n, r, c):
            self.num_layers, self.rows, self.columns = n, r, c
    gs = [G(1, 4096, 4096), G(1, 1024, 4096), G(1, 1024, 4096), G(1, 4096, 4096),
          G(1, 14336, 4096), G(1, 14336, 4096), G(1, 4096, 14336)]
    ordered, bins, owner = common_utils.partition_layers(gs, 4)
    loads = sorted(sum(g.rows * g.columns for g in bins[b]) for b in range(4))
    assert sum(loads) == sum(g.rows * g.columns for g in gs)
    assert ordered[0].rows * ordered[0].columns == 14336 * 4096
    assert set(owner.values()) <= {0, 1, 2, 3}
    # every object assigned exactly once
    assert sum(len(v) for v in bins.values()) == len(gs)


def test_staged_fold_matches_per_call_update():
    """Folding pending calls with alpha = n_old/n_new, beta = 2/n_new equals the
    reference's call-by-call update for any split into folds."""
    rng = np.random.default_rng(3)
    calls = [rng.standard_normal((b, 16, 24)).astype(np.float32) for b in (1, 2, 1, 3, 1)]
    H_ref, n = np.zeros((24, 24), np.float32), 0
    for x in calls:
        H_ref, n = ohess.gptq_add_batch(H_ref, n, x)
    for split in ([2, 3], [1, 1, 1, 1, 1], [5], [4, 1]):
        H = np.zeros((24, 24), np.float64)
        n_fold, n_now, i = 0, 0, 0
        for k in split:
            X = np.concatenate([c.reshape(-1, 24) for c in calls[i:i + k]])
            n_now += sum(c.shape[0] for c in calls[i:i + k])
            H = H * (n_fold / n_now) + (2.0 / n_now) * (X.T.astype(np.float64) @ X)
            n_fold = n_now
            i += k
        np.testing.assert_allclose(H, H_ref, rtol=2e-5, atol=1e-4)


def test_g2ptq_token_weights_match_per_call_update():
    rng = np.random.default_rng(4)
    C, G = 20, 4
    xs = [rng.standard_normal((t, C)).astype(np.float32) for t in (10, 7, 13)]
    ss = [rng.random((t, G)).astype(np.float32) for t in (10, 7, 13)]
    H_ref, a, k, t = np.zeros((G, C, C), np.float32), np.zeros(C, np.float32), 0, 0
    for x, s in zip(xs, ss):
        H_ref, a, k, t = ohess.g2ptq_add_batch(H_ref, a, k, t, x, s)
    X = np.concatenate(xs).astype(np.float64)
    Wt = np.concatenate([s / s.shape[0] for s in ss]).astype(np.float64)
    H = np.einsum("ni,nj,ng->gij", X, X, Wt) / len(xs)
    np.testing.assert_allclose(H, H_ref, rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------------------
# two CPU ranks: reduce_to_target_rank semantics
# ---------------------------------------------------------------------------

class HostGPTQ:
    """CPU stand-in carrying the attributes reduce_to_target_rank touches."""

    def __init__(self, H, n):
        import contextlib
        self.num_layers = H.shape[0]
        self._H = H
        self.nsamples = torch.tensor(n)
        self._n = list(n)
        self._n_folded = list(n)
        self._maybe_onload_hessian = contextlib.nullcontext

    @property
    def H(self):
        return self._H

    def _leave_groups(self):
        pass


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from g2ptq_b200.gptq_utils.gptq_utils import reduce_to_target_rank
    torch.manual_seed(rank)
    H = torch.rand(2, 8, 8)
    n = [3 + rank, 0]  # second layer never saw data on any rank
    obj = HostGPTQ(H.clone(), n)
    reduce_to_target_rank([obj], {obj: 1})
    q.put((rank, H, n, obj.H.clone(), obj.nsamples.clone()))
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_to_target_rank_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, H, n, Hout, nout = q.get(timeout=120)
        res[r] = (H, n, Hout, nout)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (H0, n0, _, _), (H1, n1, Hout1, nout1) = res[0], res[1]
    total = n0[0] + n1[0]
    expect = H0[0] * n0[0] / total + H1[0] * n1[0] / total
    torch.testing.assert_close(Hout1[0], expect)
    assert torch.count_nonzero(Hout1[1]) == 0       # no samples anywhere -> zeros
    assert nout1.tolist() == [total, 0]


def test_lazy_counter_applies_increments_on_read():
    """add_batch counters: increments recorded on the host appear at the next
    read; edits made in place through a read survive later increments."""
    from g2ptq_b200.gptq_utils import _engine

    class Obj:
        nsamples = _engine.lazy_counter("nsamples")

    o = Obj()
    o.nsamples = torch.zeros(2, dtype=torch.long)
    for _ in range(5):
        _engine.bump(o, "nsamples", 1, 3)
    _engine.bump(o, "nsamples", 0, 1)
    assert o.nsamples.tolist() == [1, 15]
    o.nsamples[0] = 7
    _engine.bump(o, "nsamples", 0, 2)
    assert o.nsamples.tolist() == [9, 15]
    o.nsamples = None
    assert o.nsamples is None


def test_weight_quantizer_deepcopy_is_independent():
    """make_group_quantizers' copies: configuration carried over, buffers and
    module containers distinct, the status word not shared."""
    import copy
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers

    q = WeightQuantizer()
    q.configure(3, perchannel=True, sym=False, mse=True, grid=20, weight_groupsize=-1)
    q._status = torch.zeros(1, dtype=torch.int32)
    qs = make_group_quantizers(q, 300, 128)
    assert len(qs) == 3
    for c in qs:
        assert (c.bits, c.sym, c.mse, c.grid, c.maxq, c.minq) == (3, False, True, 20, 3, -4)
        assert c._status is None and not c.ready()
        assert c._buffers is not q._buffers and c._modules is not q._modules
        assert set(c.state_dict()) == {"scale", "zero"}
    qs[0].scale.fill_(5.0)
    assert float(q.scale) == 0.0 and float(qs[1].scale) == 0.0
    c = copy.deepcopy(qs[0])
    assert float(c.scale) == 5.0 and c.scale is not qs[0].scale
