"""compressed-tensors export (utils/compressed_tensors_utils.py of the reference)
against tests/golden/export.json, written by the reference's own
save_to_compressed_tensors from a seeded tiny Llama (tests/golden/make_golden.py).

CPU: the ignore-list expansion and the checkpoint writer on parameters staged
with the oracle's packing.  GPU: the whole path, packing in the CUDA kernel.
Bar: the quantization config identical and every tensor of the checkpoint
byte-identical (sha256).
"""

import importlib.util
import json
import os
import tempfile

import numpy as np
import pytest
import torch

from g2ptq_b200.utils import compressed_tensors_utils as ctu
from oracle.export import pack_to_int32

HERE = os.path.dirname(os.path.abspath(__file__))


def _golden_module():
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def fixture():
    with open(os.path.join(HERE, "golden", "export.json")) as f:
        return json.load(f)


def test_expand_ignore_list(fixture):
    for case, expected in fixture["ignore_cases"]:
        assert ctu.expand_ignore_list(case) == expected


def _save_and_compare(model, cfg, mg, fixture):
    with tempfile.TemporaryDirectory() as d:
        ctu.save_to_compressed_tensors("tiny", cfg, model, mg._Saver(), mg._Saver(), d, bits=4,
                                       group_size=mg.EXPORT_GS, sym=True)
        table = mg.export_table(d)
        with open(os.path.join(d, "config.json")) as f:
            qcfg = json.load(f)["quantization_config"]
    assert qcfg == fixture["quantization_config"]
    assert table == {k: [v[0], v[1], v[2]] for k, v in fixture["tensors"].items()}


def test_checkpoint_from_staged_parameters(fixture):
    """register_qparam_buffers + save_to_compressed_tensors on parameters staged
    with the oracle's packing (host code only)."""
    mg = _golden_module()
    cfg, model = mg.export_tiny_model()
    codes = np.load(os.path.join(HERE, "golden", "export.npz"))
    layer = model.model.layers[0]
    mods = []
    for name in mg.EXPORT_LINEARS:
        mod = layer.get_submodule(name)
        mod._export_qparams = {
            "weight_packed": torch.from_numpy(pack_to_int32(codes[name + "__codes"], 4)),
            "weight_scale": torch.from_numpy(codes[name + "__scale"]).to(mod.weight.dtype),
            "weight_shape": torch.tensor(mod.weight.shape),
        }
        mods.append(mod)
    ctu.register_qparam_buffers(mods)
    _save_and_compare(model, cfg, mg, fixture)


@pytest.mark.gpu
def test_checkpoint_through_compress_on_gpu(fixture):
    """compress (int32 packing in the CUDA kernel) + registration + writer."""
    mg = _golden_module()
    cfg, model = mg.export_tiny_model()
    model = model.to("cuda")
    codes = np.load(os.path.join(HERE, "golden", "export.npz"))
    layer = model.model.layers[0]
    mods = []
    for name in mg.EXPORT_LINEARS:
        mod = layer.get_submodule(name)
        c = torch.from_numpy(codes[name + "__codes"]).cuda()
        sc = torch.from_numpy(codes[name + "__scale"]).cuda()
        ctu.compress(mod, sc.repeat_interleave(mg.EXPORT_GS, dim=1), c.float(), 4, mg.EXPORT_GS)
        mods.append(mod)
    ctu.register_qparam_buffers(mods)
    _save_and_compare(model, cfg, mg, fixture)


# ---------------------------------------------------------------------------
# MoE expert stacking (utils/models/mixins.py:93-144)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("packed", [True, False])
def test_stack_experts_matches_reference(packed):
    """The 3-D expert parameters equal, bit for bit, those the reference's own
    ``MoEMixin.stack_experts`` made from the same per-expert tensors
    (tests/golden/stack_experts.npz), and the per-expert submodules are gone."""
    mg = _golden_module()
    z = np.load(os.path.join(HERE, "golden", "stack_experts.npz"))
    experts = mg.stack_container(z, packed)
    ctu.stack_experts(experts, weight_packed=packed)
    names = (["gate_up_proj_packed", "down_proj_packed", "gate_up_proj_scale",
              "down_proj_scale", "gate_up_proj_shape", "down_proj_shape"] if packed
             else ["gate_up_proj", "down_proj"])
    for n in names:
        t = getattr(experts, n).detach()
        got = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy()
        want = z[f"out_{n}"]
        assert got.dtype == want.dtype and got.shape == want.shape, n
        assert np.array_equal(got, want), n
    assert len(experts._modules) == int(z[f"left_{int(packed)}"]) == 0
    if packed:
        assert isinstance(experts.gate_up_proj_packed, torch.nn.Parameter)
        assert not experts.gate_up_proj_packed.requires_grad
