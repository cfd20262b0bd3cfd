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

def cpu_pack_upper(H, scale=1.0, out=None):
    """CPU stand-in of ops.pack_upper (row-major upper triangle)."""
    Hb = H if H.dim() == 3 else H[None]
    C = Hb.shape[-1]
    iu = torch.triu_indices(C, C)
    vals = (Hb[:, iu[0], iu[1]] * scale).reshape(-1)
    if out is None:
        return vals
    out.copy_(vals)
    return out


def cpu_unpack_upper(H, packed, mirror=True):
    """CPU stand-in of ops.unpack_upper."""
    Hb = H if H.dim() == 3 else H[None]
    C = Hb.shape[-1]
    iu = torch.triu_indices(C, C)
    vals = packed.view(Hb.shape[0], -1)
    Hb[:, iu[0], iu[1]] = vals
    Hb[:, iu[1], iu[0]] = vals if mirror else 0.0
    Hb[:, iu[0], iu[1]] = vals
    return H


class HostGPTQ:
    """CPU stand-in carrying the attributes reduce_to_target_rank touches."""

    def __init__(self, H, n):
        import contextlib
        self.num_layers = H.shape[0]
        self.dev = torch.device("cpu")
        self.offload_hessians = False
        self._H = H
        self.nsamples = torch.tensor(n)
        self._n = list(n)
        self._n_folded = list(n)
        self._maybe_onload_hessian = contextlib.nullcontext

    @property
    def H(self):
        return self._H

    def _hessian(self):
        return self._H

    def _leave_groups(self):
        pass


class HostLayer:
    def __init__(self, rows, cols, fill):
        self.weight = torch.nn.Parameter(torch.full((rows, cols), float(fill),
                                                    dtype=torch.bfloat16),
                                         requires_grad=False)


class HostQuantized:
    """Stand-in of a quantized object for broadcast_quantized_param: layers,
    the group quantizers' bit width and count."""

    def __init__(self, layers, bits, groups):
        from types import SimpleNamespace
        self.layers = layers
        self.num_layers = len(layers)
        self.quantizer = [SimpleNamespace(bits=bits) for _ in range(groups)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from g2ptq_b200.gptq_utils import collectives
    collectives.pack_upper = cpu_pack_upper
    collectives.unpack_upper = cpu_unpack_upper


class _Reply:
    """A rank's channel to the parent: ``put`` hands over the rank's result
    and returns once the parent holds every rank's result.  Tensors cross
    the queue as shared file descriptors that the sending process must keep
    open until the parent has rebuilt them, so no rank may exit before."""

    def __init__(self, q, done):
        self.q, self.done = q, done

    def put(self, item):
        self.q.put(item)
        self.done.wait(120)


def _run_ranks(target, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, _Reply(q, done)))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, payload = q.get(timeout=120)
            res[r] = payload
    finally:
        done.set()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def _rank_reduce(rank, world, port, q):
    _init(rank, world, port)
    from g2ptq_b200.gptq_utils.gptq_utils import reduce_to_target_rank
    torch.manual_seed(rank)
    H = torch.rand(2, 8, 8)
    H = H + H.transpose(1, 2)  # symmetric, as every Hessian is
    H2 = torch.rand(1, 6, 6)
    H2 = H2 + H2.transpose(1, 2)
    n = [3 + rank, 0]  # second layer never saw data on any rank
    obj = HostGPTQ(H.clone(), n)
    obj2 = HostGPTQ(H2.clone(), [5])
    reduce_to_target_rank([obj, obj2], {obj: 1, obj2: 0})
    q.put((rank, (H, n, obj.H.clone(), obj.nsamples.clone(), H2, obj2.H.clone(),
                  obj2.nsamples.clone())))
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_to_target_rank_two_ranks():
    """Two objects owned by different ranks in one coalesced exchange: each
    owner gets the sample-share weighted sum and the global counts."""
    res = _run_ranks(_rank_reduce)
    (H0, n0, _, _, H20, _, _), (H1, n1, Hout1, nout1, H21, _, _) = res[0], res[1]
    total = n0[0] + n1[0]
    expect = H0[0] * n0[0] / total + H1[0] * n1[0] / total
    torch.testing.assert_close(Hout1[0], expect)
    assert torch.count_nonzero(Hout1[1]) == 0       # no samples anywhere -> zeros
    assert nout1.tolist() == [total, 0]
    # the second object is owned by rank 0: equal shares of 5 samples each
    torch.testing.assert_close(res[0][5][0], (H20[0] + H21[0]) / 2)
    assert res[0][6].tolist() == [10]


def _rank_broadcast(rank, world, port, q):
    _init(rank, world, port)
    from g2ptq_b200.gptq_utils.common_utils import broadcast_quantized_param
    # 3-bit layer first: its 2-byte scales leave the next int64 weight_shape
    # at a byte offset that is not a multiple of 8 inside the buffer
    objs = [HostQuantized([HostLayer(8, 40, 10 * rank + k) for k in range(2)], 4, 2),
            HostQuantized([HostLayer(17, 24, 100 + rank)], 3, 1)]
    owner = {objs[0]: 1, objs[1]: 0}
    for o in objs:
        if owner[o] != rank:
            continue
        for k, layer in enumerate(o.layers):
            rows, cols = layer.weight.shape
            bits = o.quantizer[0].bits
            layer._export_qparams = {
                "weight_packed": torch.full((rows, -(-cols // (32 // bits))), 7 + k,
                                            dtype=torch.int32),
                "weight_scale": torch.full((rows, len(o.quantizer)), 0.5 + k,
                                           dtype=torch.bfloat16),
                "weight_shape": torch.tensor([rows, cols])}
    staged = broadcast_quantized_param(objs, owner, export_compressed_tensors=True)
    out = [[(l.weight.data.float().clone(), {k: v.clone() for k, v in l._export_qparams.items()})
            for l in o.layers] for o in objs]
    q.put((rank, (out, len(staged))))
    dist.barrier()
    dist.destroy_process_group()


def test_broadcast_quantized_param_two_ranks():
    """Every rank ends with the owner's weights and export buffers, without
    any metadata exchange: non-owners derive the buffer shapes."""
    res = _run_ranks(_rank_broadcast)
    for r in (0, 1):
        out, n_staged = res[r]
        assert n_staged == 3
        for k in range(2):  # object 0 owned by rank 1
            w, qp = out[0][k]
            assert torch.all(w == 10 + k)
            assert qp["weight_packed"].shape == (8, 5)
            assert torch.all(qp["weight_packed"] == 7 + k)
            assert torch.all(qp["weight_scale"].float() == 0.5 + k)
            assert qp["weight_shape"].tolist() == [8, 40]
        w, qp = out[1][0]  # object 1 owned by rank 0, 3-bit: 10 codes per word
        assert torch.all(w == 100)
        assert qp["weight_packed"].shape == (17, 3) and qp["weight_scale"].shape == (17, 1)
        assert qp["weight_shape"].tolist() == [17, 24]


def test_broadcast_quantized_param_with_an_idle_rank():
    """Three ranks for two objects (one LPT bin stays empty, as with seven
    linears on eight GPUs): the rank that owns nothing still ends with every
    owner's weights and export buffers."""
    res = _run_ranks(_rank_broadcast, world=3)
    for r in (0, 1, 2):
        out, n_staged = res[r]
        assert n_staged == 3
        for k in range(2):
            w, qp = out[0][k]
            assert torch.all(w == 10 + k)
            assert torch.all(qp["weight_packed"] == 7 + k)
        w, qp = out[1][0]
        assert torch.all(w == 100)
        assert qp["weight_shape"].tolist() == [17, 24]


def _rank_gather(rank, world, port, q):
    _init(rank, world, port)
    from g2ptq_b200.gptq_utils import collectives
    full_a = torch.zeros(10, 3)
    full_b = torch.zeros(7, dtype=torch.int32)
    a_rows = [(0, 6), (6, 10)][rank]   # ragged slices
    b_rows = [(0, 2), (2, 7)][rank]
    part_a = (torch.arange(30, dtype=torch.float32).view(10, 3) + 0.5)[a_rows[0]:a_rows[1]]
    part_b = torch.arange(7, dtype=torch.int32)[b_rows[0]:b_rows[1]] * 3
    collectives.all_gather_rows([(part_a.contiguous(), full_a), (part_b.contiguous(), full_b)],
                                torch.device("cpu"))
    q.put((rank, (full_a, full_b)))
    dist.barrier()
    dist.destroy_process_group()


def test_all_gather_rows_two_ranks():
    res = _run_ranks(_rank_gather)
    for r in (0, 1):
        a, b = res[r]
        torch.testing.assert_close(a, torch.arange(30, dtype=torch.float32).view(10, 3) + 0.5)
        assert b.tolist() == [3 * i for i in range(7)]


def test_cpu_pack_stand_in_layout():
    """The CPU stand-in packs in the kernel's documented layout: element
    (i, j), i <= j, at i C - i(i-1)/2 + j - i."""
    C = 5
    H = torch.arange(C * C, dtype=torch.float32).view(C, C)
    p = cpu_pack_upper(H)
    for i in range(C):
        for j in range(i, C):
            assert p[i * C - i * (i - 1) // 2 + j - i] == H[i, j]


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
