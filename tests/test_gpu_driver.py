"""The calibration driver (``gptq_utils.driver``) against the reference's own
flow of ``gptq_fwrd`` (gptq_utils/gptq_utils.py:455-595): for every
sequential group a whole forward of the layer with forward hooks calling
``add_batch(idx, inp[0].data, out)``, the group quantized, and a final forward
propagating the layer's output.  The driver computes the group inputs
incrementally instead; on a tiny two-layer Llama the quantized weights of
every linear and the propagated hidden states must be identical (GPU)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def tiny(layers=2, seed=42):
    import argparse
    import calibrate
    args = argparse.Namespace(layers=layers, seqs=6, seq_len=128, bsz=2, hidden=256,
                              intermediate=512, heads=4, kv_heads=2, head_dim=64, vocab=1000)
    cfg = calibrate.llama_config(args)
    model = calibrate.build_layers(torch, cfg, layers, DEV, seed=seed)
    inps = calibrate.calibration_inputs(torch, cfg, args, 0, 1, DEV)
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    rope = LlamaRotaryEmbedding(cfg, device=DEV)
    pe = rope(inps[0], torch.arange(args.seq_len, device=DEV)[None])
    return model, inps, pe


@torch.no_grad()
def hooked_flow(cal, layers, inps, pe):
    """The reference's flow, every group through hooks on whole forwards."""
    from g2ptq_b200.gptq_utils import driver, gptq_utils, g2ptq_utils
    from g2ptq_b200.gptq_utils.common_utils import make_group_quantizers
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    for li, layer in enumerate(layers):
        for names in driver.SEQUENTIAL_GROUPS:
            mods = {n: driver._module(layer, n) for n in names}
            captured = {n: [] for n in names}
            handles = [m.register_forward_hook(
                lambda m, inp, out, n=n: captured[n].append(inp[0].data.clone()))
                for n, m in mods.items()]
            for x in inps:
                layer(x, position_embeddings=pe)
            for h in handles:
                h.remove()
            if cal.method == "g2ptq":
                sal, grad = driver._synthetic_g2ptq_inputs(cal, list(names), mods,
                                                           captured[names[0]], li)
            objs = []
            for n in names:
                if cal.method == "g2ptq":
                    o = g2ptq_utils.G2PTQ([mods[n]], [list(sal[n])], [grad[n]],
                                          num_groups=cal.num_groups)
                else:
                    o = gptq_utils.GPTQ([mods[n]])
                q = WeightQuantizer()
                q.configure(cal.w_bits, perchannel=True, sym=not cal.w_asym, mse=False)
                o.quantizer = make_group_quantizers(q, mods[n].weight.shape[1], cal.w_groupsize)
                for x in captured[n]:
                    o.add_batch(0, x, None)
                objs.append(o)
            kw = dict(blocksize=128, percdamp=0.01, groupsize=cal.w_groupsize,
                      actorder=cal.act_order, static_groups=cal.act_order)
            if cal.method == "g2ptq":
                kw.update(enable_gradient_update=True, alpha=cal.alpha)
            gptq_utils.fasterquant_all(objs, **kw)
        for k, x in enumerate(inps):
            inps[k] = layer(x, position_embeddings=pe)
    return inps


@pytest.mark.parametrize("method", ["gptq", "g2ptq"])
def test_driver_matches_hooked_reference_flow(method):
    from g2ptq_b200.gptq_utils import driver
    if method == "gptq":
        cal = driver.Calibration(method="gptq", w_bits=4, act_order=True, bsz=2)
    else:
        cal = driver.Calibration(method="g2ptq", w_bits=3, w_asym=True, act_order=False, bsz=2,
                                 alpha=1.0)
    layers_a, inps_a, pe = tiny()
    layers_b, inps_b, _ = tiny()
    driver.calibrate(cal, layers_a, inps_a, pe)
    out_b = hooked_flow(cal, layers_b, [x.clone() for x in inps_b], pe)
    for la, lb in zip(layers_a, layers_b):
        for name in [n for g in driver.SEQUENTIAL_GROUPS for n in g]:
            wa = driver._module(la, name).weight
            wb = driver._module(lb, name).weight
            assert torch.equal(wa, wb), name
    for a, b in zip(inps_a, out_b):
        assert torch.equal(a, b)
        assert torch.isfinite(a).all()
