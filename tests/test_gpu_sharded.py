"""Multi-GPU quantization paths (GPU).

* Row slices of the row-sharded path against the single-GPU pipeline on one
  GPU: any split of the rows gives bit-identical weights, codes and scales.
* The packed upper-triangle exchange format (pack / unpack kernels).
* With two or more GPUs: ``fasterquant_rows`` and the reference's owner flow
  (``reduce_to_target_rank`` + owner ``fasterquant`` + ``broadcast_quantized_param``)
  over NCCL against the single-GPU result, for GPTQ and (owner flow, with
  G2PTQ's reduction of block-wise Hessians, gradients and squared
  activations) for G2PTQ.  Every rank feeds the same tokens,
  so the reduced statistics equal each rank's own exactly (x/2 + x/2 = x in
  fp32) and the results must match bit for bit.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

from g2ptq_b200 import ops  # noqa: E402
from g2ptq_b200.gptq_utils import _engine, gptq_utils, sharded  # noqa: E402
from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers  # noqa: E402
from g2ptq_b200.utils.quant_utils import WeightQuantizer  # noqa: E402

DEV = torch.device("cuda", 0)


def _layer(rows, cols, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    lin = torch.nn.Linear(cols, rows, bias=False, device=dev, dtype=torch.bfloat16)
    lin.weight.data = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    return lin


def _tokens(cols, seqs, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(seqs):
        x = torch.randn(1, 1024, cols, device=dev, generator=g)
        x[..., :4] *= 20
        out.append(x.to(torch.bfloat16))
    return out


def _quantizers(bits, sym, C, gs):
    q = WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=False)
    return make_group_quantizers(q, C, gs)


def test_pack_unpack_upper_roundtrip():
    g = torch.Generator(device=DEV).manual_seed(1)
    for C in (1, 31, 32, 33, 200):
        A = torch.randn(3, C, C, device=DEV, generator=g)
        H = A + A.transpose(1, 2)
        p = ops.pack_upper(H, 0.5)
        iu = torch.triu_indices(C, C, device=DEV)
        torch.testing.assert_close(p.view(3, -1), 0.5 * H[:, iu[0], iu[1]], rtol=0, atol=0)
        out = torch.full_like(H, 7.0)
        ops.unpack_upper(out, p)
        torch.testing.assert_close(out, 0.5 * H, rtol=0, atol=0)
        U = torch.triu(A)
        out.fill_(7.0)
        ops.unpack_upper(out, ops.pack_upper(U), mirror=False)
        torch.testing.assert_close(out, U, rtol=0, atol=0)


@pytest.mark.parametrize("gs,act,static,export", [(128, True, True, True),
                                                   (128, False, False, False),
                                                   (-1, False, False, True)])
def test_row_slices_bit_identical_to_single_gpu(gs, act, static, export, monkeypatch):
    rows, cols = 608, 1024  # splits into 16-row multiples with a ragged last slice
    lin = _layer(rows, cols, 3, DEV)
    W0 = lin.weight.data.clone()
    obj = gptq_utils.GPTQ([lin])
    obj.quantizer = _quantizers(4, True, cols, gs)
    for x in _tokens(cols, 4, 5, DEV):
        obj.add_batch(0, x, None)
    H = obj.H.clone()
    captured = {}
    orig = _engine.Pending.finish

    def finish(self_):
        out = orig(self_)
        captured["U"] = self_.U.clone()
        captured["scale"] = self_.params.scale.clone()
        return out
    monkeypatch.setattr(_engine.Pending, "finish", finish)
    obj.fasterquant(blocksize=128, percdamp=0.01, groupsize=gs, actorder=act,
                    static_groups=static, export_compressed_tensors=export)
    full_w = lin.weight.data.clone()
    full_qp = dict(lin.__dict__.get("_export_qparams") or {})

    # the factor owner's outputs, rebuilt from the same Hessian
    shared = {"diag": torch.diagonal(H, dim1=-2, dim2=-1).clone()}
    Hp = H.clone()
    ops.prepare_hessian(Hp)
    if act:
        shared["perm"], _ = _engine.act_order_perm(ops.mean_diag(Hp))
    lin2 = _layer(rows, cols, 3, DEV)
    assert torch.equal(lin2.weight.data, W0)
    obj2 = gptq_utils.GPTQ([lin2])
    obj2.quantizer = _quantizers(4, True, cols, gs)
    for world in (2, 3, 5):
        outs, packed, scales = [], [], []
        for r0, r1 in sharded.row_ranges(rows, world):
            w = sharded._Rows(obj2, captured["U"], shared, r0, r1, 128, gs, act, static, export)
            if w.n:
                outs.append(w.outs[0])
                scales.append(w.params.scale)
                if export:
                    packed.append(w.packed[0])
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(outs), full_w), world
        assert torch.equal(torch.cat(scales), captured["scale"]), world
        if export:
            assert torch.equal(torch.cat(packed), full_qp["weight_packed"]), world


# ---------------------------------------------------------------------------
# two or more GPUs
# ---------------------------------------------------------------------------

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(dev):
    """q/k fed one tensor (a fold group), down fed another; W4 sym g128."""
    layers = {"q": _layer(512, 1024, 11, dev), "k": _layer(256, 1024, 12, dev),
              "down": _layer(1024, 1536, 13, dev)}
    objs = {n: gptq_utils.GPTQ([l]) for n, l in layers.items()}
    for n, o in objs.items():
        o.quantizer = _quantizers(4, True, layers[n].weight.shape[1], 128)
    xa = _tokens(1024, 3, 21, dev)
    xd = _tokens(1536, 3, 22, dev)
    for s in range(3):
        objs["q"].add_batch(0, xa[s], None)
        objs["k"].add_batch(0, xa[s], None)
        objs["down"].add_batch(0, xd[s], None)
    return layers, objs


FQ = dict(blocksize=128, percdamp=0.01, groupsize=128, actorder=True, static_groups=True,
          export_compressed_tensors=True)
FQ_G2 = dict(blocksize=128, percdamp=0.01, groupsize=128, actorder=False, static_groups=False,
             enable_gradient_update=True, alpha=1.0, export_compressed_tensors=True)


def _build_g2ptq(dev):
    """Two G2PTQ linears (W3 asym, four row groups) with saliencies and
    gradients from seeded synthetic output gradients."""
    from g2ptq_b200.gptq_utils import g2ptq_utils
    layers = {"a": _layer(512, 1024, 31, dev), "b": _layer(256, 768, 32, dev)}
    objs = {}
    for n, lin in layers.items():
        rows, cols = lin.weight.shape
        xs = _tokens(cols, 3, 33 + cols, dev)
        g = torch.Generator(device=dev).manual_seed(34 + rows)
        sal, grad = [], torch.zeros(rows, cols, device=dev)
        for x in xs:
            go = (torch.randn(x.shape[1], rows, device=dev, generator=g) * 1e-3).to(
                torch.bfloat16)
            sal.append((go.float() ** 2).reshape(-1, 4, rows // 4).mean(-1))
            grad += (go.T @ x[0]).float() / x.shape[1]
        o = g2ptq_utils.G2PTQ([lin], [sal], [grad / len(xs)], num_groups=4)
        o.quantizer = _quantizers(3, False, cols, 128)
        for x in xs:
            o.add_batch(0, x, None)
        objs[n] = o
    return layers, objs


def _rank_main(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from g2ptq_b200.gptq_utils import common_utils
        # single-GPU result on this rank's own copy
        ref_layers, ref_objs = _build(dev)
        gptq_utils.fasterquant_all(list(ref_objs.values()), **FQ)
        ref = {n: (l.weight.data.clone(), l._export_qparams["weight_packed"].clone(),
                   l._export_qparams["weight_scale"].clone()) for n, l in ref_layers.items()}
        # row-sharded
        layers, objs = _build(dev)
        sharded.fasterquant_rows(list(objs.values()), **FQ)
        ok_rows = all(torch.equal(layers[n].weight.data, ref[n][0]) and
                      torch.equal(layers[n]._export_qparams["weight_packed"], ref[n][1]) and
                      torch.equal(layers[n]._export_qparams["weight_scale"], ref[n][2])
                      for n in ref)
        # the reference's owner flow
        layers, objs = _build(dev)
        specs = list(objs.values())
        _, _, owner = common_utils.partition_layers(specs, world)
        gptq_utils.reduce_to_target_rank(specs, owner)
        gptq_utils.fasterquant_all([o for o in specs if owner[o] == rank], **FQ)
        common_utils.broadcast_quantized_param(specs, owner, export_compressed_tensors=True)
        ok_owner = all(torch.equal(layers[n].weight.data, ref[n][0]) and
                       torch.equal(layers[n]._export_qparams["weight_packed"], ref[n][1])
                       for n in ref)
        # G2PTQ through its own coalesced reduction and the owner flow
        from g2ptq_b200.gptq_utils import g2ptq_utils
        g2_ref = _build_g2ptq(dev)
        gptq_utils.fasterquant_all(list(g2_ref[1].values()), **FQ_G2)
        g2_lay, g2_objs = _build_g2ptq(dev)
        specs = list(g2_objs.values())
        _, _, owner = common_utils.partition_layers(specs, world)
        g2ptq_utils.reduce_to_target_rank(specs, owner)
        gptq_utils.fasterquant_all([o for o in specs if owner[o] == rank], **FQ_G2)
        common_utils.broadcast_quantized_param(specs, owner, export_compressed_tensors=True)
        ok_owner = ok_owner and all(
            torch.equal(g2_lay[n].weight.data, g2_ref[0][n].weight.data) and
            torch.equal(g2_lay[n]._export_qparams["weight_packed"],
                        g2_ref[0][n]._export_qparams["weight_packed"]) for n in g2_lay)
        torch.cuda.synchronize()
        q.put((rank, ok_rows, ok_owner, None))
    except Exception as e:  # reported to the parent; the group is torn down below
        q.put((rank, False, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_gpu_paths_match_single_gpu():
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, ok_rows, ok_owner, err in res:
        assert err is None, (rank, err)
        assert ok_rows, f"rank {rank}: row-sharded result differs from the single-GPU one"
        assert ok_owner, f"rank {rank}: owner-flow result differs from the single-GPU one"
    assert all(p.exitcode == 0 for p in procs)
