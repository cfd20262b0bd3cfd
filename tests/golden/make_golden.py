"""Generate golden fixtures by running the reference G2PTQ code on CPU.

Usage (needs a checkout of the reference; not available on GPU boxes)::

    python tests/golden/make_golden.py --reference <path-to-G2PTQ-checkout>

The reference's quantizer modules import third-party packages that are not
installed here (fast_hadamard_transform, llmcompressor, accelerate and
compressed_tensors.distributed).  None of them takes part in the arithmetic
captured below, so they are replaced by empty module stubs.  The CUDA-only
tensor validator and ``torch.cuda.synchronize`` are neutralised and the
shared-offload write-back is replaced by a plain ``weight.data.copy_`` so the
reference's torch path runs unchanged on CPU.

Each fixture file holds the inputs and the reference's outputs for one family
of calls; ``tests/test_oracle_golden.py`` replays the inputs through the numpy
oracle and the GPU tests replay them through the CUDA library.
"""

import argparse
import contextlib
import copy
import importlib.machinery
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _stub(name, **attrs):
    m = types.ModuleType(name)
    m.__spec__ = importlib.machinery.ModuleSpec(name, None)
    m.__dict__.update(attrs)
    sys.modules[name] = m
    return m


def import_reference(root):
    sys.path.insert(0, root)
    import transformers  # noqa: F401  (must precede the llmcompressor stubs)
    _stub("fast_hadamard_transform", hadamard_transform=lambda *a, **k: None)
    _stub("compressed_tensors.distributed", greedy_bin_packing=None,
          wait_for_comms=lambda c: [x.wait() for x in c],
          is_distributed=lambda: False, is_source_process=lambda: True)
    for n in ["llmcompressor", "llmcompressor.utils", "llmcompressor.modeling",
              "llmcompressor.modeling.moe"]:
        _stub(n)
    _stub("llmcompressor.utils.dev", skip_weights_initialize=None)
    _stub("llmcompressor.modeling.moe.conversion_mappings", ARCH_TO_2D_MAPPINGS={},
          get_linearize_load_mappings=None, has_linearize_load_mappings=None,
          set_save_conversion_mapping=None)
    _stub("llmcompressor.modeling.moe.linear_experts", LinearExperts2D=None)
    _stub("llmcompressor.modeling.moe.linearize", linearize_moe=None)
    _stub("accelerate", dispatch_model=None, infer_auto_device_map=None)
    _stub("accelerate.utils", get_balanced_memory=None)
    import compressed_tensors.offload.utils as _u
    import compressed_tensors.offload.load as _l
    _u.as_single_threaded = getattr(_u, "as_single_threaded", contextlib.nullcontext)
    for n in ["_get_cpu_memory", "_get_device_memory", "_estimate_tensor_count"]:
        if not hasattr(_l, n):
            setattr(_l, n, None)
    from utils import dist_utils  # noqa: F401
    from gptq_utils import gptq_utils, g2ptq_utils, gptaq_utils, gptq_guided_utils
    from utils import quant_utils, offload_utils
    torch.cuda.synchronize = lambda *a, **k: None
    offload_utils.update_shared_offload_parameter = (
        lambda layer, name, data, **k: layer.weight.data.copy_(data))
    for m in (gptq_utils, g2ptq_utils, gptaq_utils, gptq_guided_utils):
        m.validate_tensors = lambda *a, **k: None
        m.offload_utils = offload_utils
    return types.SimpleNamespace(gptq=gptq_utils, g2ptq=g2ptq_utils, gptaq=gptaq_utils,
                                 guided=gptq_guided_utils, quant=quant_utils)


def npy(t):
    return t.detach().cpu().numpy().copy()


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print("wrote", path, sum(a.nbytes for a in arrays.values()) // 1024, "KB")


def activations(gen, shape, outliers=(), outlier_scale=20.0):
    x = torch.randn(shape, generator=gen)
    for c in outliers:
        x[..., c] *= outlier_scale
    return x


# ---------------------------------------------------------------------------
# add_batch families
# ---------------------------------------------------------------------------

def gen_hessians(ref):
    gen = torch.Generator().manual_seed(43)
    C, R = 96, 32
    out = {}
    # GPTQ: three 3-D calls (b=1,2,1) then one 2-D call; BF16 and FP32 inputs.
    for tag, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        lin = torch.nn.Linear(C, R, bias=False)
        g = ref.gptq.GPTQ([lin])
        calls = [activations(gen, (1, 40, C), outliers=(3, 50)),
                 activations(gen, (2, 40, C), outliers=(3, 50)),
                 activations(gen, (1, 24, C)),
                 activations(gen, (56, C))]
        for i, x in enumerate(calls):
            x = x.to(dtype)
            g.add_batch(0, x, None)
            out[f"gptq_{tag}_x{i}"] = npy(x.float())
        out[f"gptq_{tag}_H"] = npy(g.H[0])
        out[f"gptq_{tag}_n"] = np.array(int(g.nsamples[0]))
    # G2PTQ: per-call [t, C] input with [t, 4] saliency.
    lin = torch.nn.Linear(C, R, bias=False)
    sals = [torch.rand(48, 4, generator=gen) for _ in range(3)]
    g2 = ref.g2ptq.G2PTQ([lin], [list(sals)], [torch.zeros(R, C)], num_groups=4)
    for i in range(3):
        x = activations(gen, (48, C), outliers=(7,))
        g2.add_batch(0, x, None)
        out[f"g2ptq_x{i}"] = npy(x)
        out[f"g2ptq_s{i}"] = npy(sals[i])
    out["g2ptq_H"] = npy(g2.H[0])
    out["g2ptq_act_square"] = npy(g2.act_square[0])
    out["g2ptq_index"] = np.array(int(g2.index[0]))
    out["g2ptq_total_tokens"] = np.array(int(g2.total_tokens[0]))
    # GPTAQ: quantized-path input plus FP input per call.
    lin = torch.nn.Linear(C, R, bias=False)
    ga = ref.gptaq.GPTAQ([lin])
    for i in range(3):
        x = activations(gen, (1, 32, C))
        xf = x + 0.05 * torch.randn(x.shape, generator=gen)
        ga.fp_inp[0].append(xf[0])
        ga.add_batch(0, x, None)
        out[f"gptaq_x{i}"] = npy(x)
        out[f"gptaq_fp{i}"] = npy(xf)
    out["gptaq_H"] = npy(ga.H[0])
    out["gptaq_dXXT"] = npy(ga.dXXT[0])
    out["gptaq_n"] = np.array(int(ga.nsamples[0]))
    # GuidedQuant: saliency [N, S, G] sliced by index.
    lin = torch.nn.Linear(C, R, bias=False)
    sal = torch.rand(3, 16, 4, generator=gen)
    gq = ref.guided.GPTQGuided([lin], [sal], num_groups=4)
    xs = [activations(gen, (1, 16, C)), activations(gen, (2, 16, C))]
    for i, x in enumerate(xs):
        gq.add_batch(0, x, None)
        out[f"guided_x{i}"] = npy(x)
    out["guided_sal"] = npy(sal)
    out["guided_H"] = npy(gq.H[0])
    out["guided_act_square"] = npy(gq.act_square[0])
    save("hessians.npz", **out)


# ---------------------------------------------------------------------------
# Compensation block kernels (the reference's kernel boundary ``run_eager``)
# ---------------------------------------------------------------------------

BLOCK_CASES = (
    # name, batch, columns, rows, maxq, asymmetric, seed  (the reference's CASES)
    ("symmetric_2bit_tail", 1, 7, 37, 1, False, 101),
    ("asymmetric_2bit_tail", 1, 7, 37, 1, True, 102),
    ("symmetric_4bit_batched", 2, 16, 193, 7, False, 201),
    ("asymmetric_4bit_batched", 2, 16, 193, 7, True, 202),
    ("symmetric_8bit_small", 3, 5, 11, 127, False, 301),
    ("asymmetric_8bit_small", 3, 5, 11, 127, True, 302),
    ("asymmetric_3bit_fullblock", 1, 128, 72, 3, True, 401),
    ("symmetric_4bit_fullblock", 1, 128, 40, 7, False, 402),
)


def block_inputs(batch, columns, rows, maxq, asymmetric, seed):
    """Same construction as the reference test fixture (away from ties)."""
    gen = torch.Generator().manual_seed(seed)
    shape = (batch, columns, rows)
    minq = -(maxq + 1)
    scale = torch.rand(shape, generator=gen).mul_(0.15).add_(0.05)
    zero = (torch.randint(minq, maxq + 1, shape, generator=gen).float() if asymmetric
            else torch.zeros(shape))
    target = torch.randint(minq, maxq + 1, shape, generator=gen).float()
    frac = torch.randint(0, 2, shape, generator=gen).float().mul_(0.5).sub_(0.25)
    weight = (target - zero + frac) * scale
    hinv = torch.triu(torch.randn(batch, columns, columns, generator=gen).mul_(0.002), 1)
    torch.diagonal(hinv, dim1=1, dim2=2).copy_(
        torch.rand(batch, columns, generator=gen).mul_(0.5).add_(0.75))
    z = torch.randn(shape, generator=gen).mul_(scale * 0.002)
    ghinv = torch.randn(shape, generator=gen).mul_(scale * 0.002)
    p = torch.triu(torch.randn(batch, columns, columns, generator=gen).mul_(0.002), 1)
    return weight, hinv, scale, zero, z, ghinv, p


def gen_blocks(ref):
    out = {}
    for name, batch, columns, rows, maxq, asym, seed in BLOCK_CASES:
        weight, hinv, scale, zero, z, ghinv, p = block_inputs(batch, columns, rows, maxq,
                                                              asym, seed)
        for k, v in (("weight", weight), ("hinv", hinv), ("scale", scale), ("zero", zero),
                     ("z", z), ("ghinv", ghinv), ("p", p)):
            out[f"{name}__{k}"] = npy(v)
        out[f"{name}__maxq"] = np.array(maxq)
        w, qi, err = weight.clone(), torch.empty_like(weight), torch.empty_like(weight)
        ref.gptq._run_torch_compensation(w, hinv.clone(), scale, zero, qi, err, maxq)
        out[f"{name}__gptq_q"], out[f"{name}__gptq_int"], out[f"{name}__gptq_err"] = \
            npy(w), npy(qi), npy(err)
        w, gh = weight.clone(), ghinv.clone()
        qi, err = torch.empty_like(weight), torch.empty_like(weight)
        ref.g2ptq._run_torch_compensation(w, hinv.clone(), scale, zero, z.clone(), gh, qi,
                                          err, maxq)
        out[f"{name}__g2ptq_q"], out[f"{name}__g2ptq_int"] = npy(w), npy(qi)
        out[f"{name}__g2ptq_err"], out[f"{name}__g2ptq_ghinv"] = npy(err), npy(gh)
        w = weight.clone()
        cw = torch.empty(batch, rows)
        qi, err = torch.empty_like(weight), torch.empty_like(weight)
        ref.gptaq._run_torch_compensation(w, hinv.clone(), p.clone(), scale, zero, cw, qi,
                                          err, maxq)
        out[f"{name}__gptaq_q"], out[f"{name}__gptaq_int"], out[f"{name}__gptaq_err"] = \
            npy(w), npy(qi), npy(err)
    save("blocks.npz", **out)


APPROX_BETA = 0.3


def gen_approx(ref):
    """G2PTQ's ``--approx_grad`` ablation (``approx_beta`` != 0): the block
    cases through the reference's torch compensation with a raw-weight
    snapshot, and whole ``fasterquant`` runs with ``approx_grad_beta``."""
    out = {"beta": np.array(APPROX_BETA, np.float32)}
    for name, batch, columns, rows, maxq, asym, seed in BLOCK_CASES:
        weight, hinv, scale, zero, z, ghinv, p = block_inputs(batch, columns, rows, maxq,
                                                              asym, seed)
        gen = torch.Generator().manual_seed(seed + 7)
        raw = weight + torch.randn(weight.shape, generator=gen) * scale * 0.3
        w, gh = weight.clone(), ghinv.clone()
        qi, err = torch.empty_like(weight), torch.empty_like(weight)
        ref.g2ptq._run_torch_compensation(w, hinv.clone(), scale, zero, z.clone(), gh, qi, err,
                                          maxq, weight_raw=raw.clone(), approx_beta=APPROX_BETA)
        out[f"{name}__raw"] = npy(raw)
        out[f"{name}__q"], out[f"{name}__int"] = npy(w), npy(qi)
        out[f"{name}__err"], out[f"{name}__ghinv"] = npy(err), npy(gh)
    gen = torch.Generator().manual_seed(46)
    for name, bits, sym, gs, act, B, R, C, blk in FQ_CASES[1:3]:
        layers = [torch.nn.Linear(C, R, bias=False) for _ in range(B)]
        for l in layers:
            l.weight.data = torch.randn(R, C, generator=gen) * 0.02
        W0 = torch.stack([l.weight.data.clone() for l in layers])
        G = 4
        sal = [[torch.rand(300, G, generator=gen)] for _ in range(B)]
        grads = [torch.randn(R, C, generator=gen) * 1e-3 for _ in range(B)]
        g2 = ref.g2ptq.G2PTQ(layers, [list(s) for s in sal], grads, num_groups=G,
                             approx_grad_beta=APPROX_BETA)
        g2.quantizer = make_quantizers(ref, bits, sym, C, gs)
        for b in range(B):
            g2.add_batch(b, hessian_from(gen, C, 300), None)
        out[f"{name}__W"] = npy(W0)
        out[f"{name}__grad"] = npy(torch.stack(grads))
        out[f"{name}__H"] = npy(g2.H)
        out[f"{name}__act_square"] = npy(g2.act_square)
        g2.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                       static_groups=act, enable_gradient_update=True, alpha=1.0)
        out[f"{name}__Q"] = npy(torch.stack([l.weight.data for l in layers]))
    save("approx.npz", **out)


# ---------------------------------------------------------------------------
# Whole fasterquant pipelines
# ---------------------------------------------------------------------------

FQ_CASES = (
    # name, bits, sym, groupsize, actorder(=static_groups), B, R, C, blocksize
    ("w4_sym_ungrouped", 4, True, -1, False, 2, 32, 160, 128),
    ("w4_sym_g40_actorder", 4, True, 40, True, 1, 32, 160, 128),
    ("w3_asym_g40_dynamic", 3, False, 40, False, 1, 32, 160, 64),
    ("w2_asym_g64_dynamic", 2, False, 64, False, 1, 32, 192, 128),
    ("w4_asym_g128_actorder", 4, False, 128, True, 1, 32, 256, 128),
)


def make_quantizers(ref, bits, sym, C, groupsize, mse=False, hclip=False):
    q = ref.quant.WeightQuantizer()
    q.configure(bits, perchannel=True, sym=sym, mse=mse, hclip=hclip)
    from gptq_utils.common_utils import make_group_quantizers
    return make_group_quantizers(q, C, groupsize)


def hessian_from(gen, C, T, dead=()):
    x = activations(gen, (T, C), outliers=(1, C // 2))
    x[:, list(dead)] = 0
    return x


def gen_fasterquant(ref):
    out = {}
    gen = torch.Generator().manual_seed(42)
    for name, bits, sym, gs, act, B, R, C, blk in FQ_CASES:
        layers = [torch.nn.Linear(C, R, bias=False) for _ in range(B)]
        for l in layers:
            l.weight.data = torch.randn(R, C, generator=gen) * 0.02
        W0 = torch.stack([l.weight.data.clone() for l in layers])
        # -- GPTQ
        g = ref.gptq.GPTQ(layers)
        g.quantizer = make_quantizers(ref, bits, sym, C, gs)
        xs = []
        for b in range(B):
            x = hessian_from(gen, C, 300, dead=(5,) if b == 0 else ())
            xs.append(x)
            g.add_batch(b, x.unsqueeze(0), None)
        H = g.H.clone()
        g.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                      static_groups=act)
        out[f"{name}__W"] = npy(W0)
        out[f"{name}__H"] = npy(H)
        out[f"{name}__gptq_Q"] = npy(torch.stack([l.weight.data for l in layers]))
        # capture codes/scales through the export staging hook
        for l, w in zip(layers, W0):
            l.weight.data = w.clone()
        g = ref.gptq.GPTQ(layers)
        g.quantizer = make_quantizers(ref, bits, sym, C, gs)
        g.H = H.clone()
        g.nsamples = torch.ones(B, dtype=torch.long)
        cap = {}
        orig = ref.gptq.compressed_tensors_utils.compress

        def grab(layer, Scale, W_int, bits, groupsize, cap=cap):
            cap.setdefault("Scale", []).append(Scale.clone())
            cap.setdefault("W_int", []).append(W_int.clone())

        ref.gptq.compressed_tensors_utils.compress = grab
        try:
            g.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                          static_groups=act, export_compressed_tensors=True)
        finally:
            ref.gptq.compressed_tensors_utils.compress = orig
        out[f"{name}__gptq_W_int"] = npy(torch.stack(cap["W_int"]))
        out[f"{name}__gptq_Scale"] = npy(torch.stack(cap["Scale"]))
        # -- GPTAQ (same H, synthetic dXXT from a perturbed FP input)
        for l, w in zip(layers, W0):
            l.weight.data = w.clone()
        ga = ref.gptaq.GPTAQ(layers)
        ga.quantizer = make_quantizers(ref, bits, sym, C, gs)
        for b in range(B):
            xf = xs[b] + 0.05 * torch.randn(xs[b].shape, generator=gen)
            ga.fp_inp[b].append(xf)
            ga.add_batch(b, xs[b].unsqueeze(0), None)
        assert torch.equal(ga.H, H), "GPTAQ H differs from GPTQ H on the same inputs"
        out[f"{name}__gptaq_dXXT"] = npy(ga.dXXT)
        ga.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                       static_groups=act)
        out[f"{name}__gptaq_Q"] = npy(torch.stack([l.weight.data for l in layers]))
        # -- G2PTQ (4 row groups, saliency-weighted Hessians, gradients, alpha 1.0)
        for l, w in zip(layers, W0):
            l.weight.data = w.clone()
        G = 4
        sal = [[torch.rand(300, G, generator=gen)] for _ in range(B)]
        grads = [torch.randn(R, C, generator=gen) * 1e-3 for _ in range(B)]
        g2 = ref.g2ptq.G2PTQ(layers, [list(s) for s in sal], grads, num_groups=G)
        g2.quantizer = make_quantizers(ref, bits, sym, C, gs)
        for b in range(B):
            g2.add_batch(b, xs[b], None)
        out[f"{name}__g2_sal"] = npy(torch.stack([s[0] for s in sal]))
        out[f"{name}__g2_grad"] = npy(torch.stack(grads))
        out[f"{name}__g2_H"] = npy(g2.H)
        out[f"{name}__g2_act_square"] = npy(g2.act_square)
        g2.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                       static_groups=act, enable_gradient_update=True, alpha=1.0)
        out[f"{name}__g2ptq_Q"] = npy(torch.stack([l.weight.data for l in layers]))
        # -- GuidedQuant
        for l, w in zip(layers, W0):
            l.weight.data = w.clone()
        gsal = [torch.rand(1, 300, G, generator=gen) for _ in range(B)]
        gq = ref.guided.GPTQGuided(layers, gsal, num_groups=G)
        gq.quantizer = make_quantizers(ref, bits, sym, C, gs)
        for b in range(B):
            gq.add_batch(b, xs[b].unsqueeze(0), None)
        out[f"{name}__guided_sal"] = npy(torch.stack(gsal))
        out[f"{name}__guided_H"] = npy(gq.H)
        out[f"{name}__guided_act_square"] = npy(gq.act_square)
        gq.fasterquant(blocksize=blk, percdamp=0.01, groupsize=gs, actorder=act,
                       static_groups=act)
        out[f"{name}__guided_Q"] = npy(torch.stack([l.weight.data for l in layers]))
    save("fasterquant.npz", **out)


# ---------------------------------------------------------------------------
# find_params, Cholesky chain, export packing
# ---------------------------------------------------------------------------

def gen_misc(ref):
    from compressed_tensors.compressors import pack_to_int32
    out = {}
    gen = torch.Generator().manual_seed(44)
    x = torch.randn(24, 64, generator=gen) * 0.02
    x[3] = 0.0
    x[3, 5] = 0.01
    x[4] = x[4].abs()
    out["fp_x"] = npy(x)
    hd = torch.rand(4, 64, generator=gen) + 0.5
    out["fp_hdiag"] = npy(hd)
    for bits in (2, 3, 4, 8):
        for sym in (True, False):
            for mse, hclip in ((False, False), (True, False), (True, True)):
                if mse and bits == 8:
                    continue
                q = ref.quant.WeightQuantizer()
                q.configure(bits, perchannel=True, sym=sym, mse=mse, hclip=hclip)
                q.find_params(x, hd.repeat_interleave(6, 0) if hclip else None)
                tag = f"fp_b{bits}_{'sym' if sym else 'asym'}_{int(mse)}{int(hclip)}"
                out[tag + "_scale"] = npy(q.scale)
                out[tag + "_zero"] = npy(q.zero)
                fq, qi, _ = q.fake_quantize(x)
                out[tag + "_fq"] = npy(fq)
                out[tag + "_q"] = npy(qi)
    # Cholesky chain: a well-conditioned H and a rank-deficient one that
    # needs the damp auto-increment.
    for tag, T in (("pd", 400), ("lowrank", 12)):
        xx = torch.randn(T, 80, generator=gen)
        H = (2 / T) * xx.t() @ xx
        if tag == "lowrank":
            H[7, :] = 0
            H[:, 7] = 0
            H -= 1e-3 * torch.eye(80) * H.diag().mean()
        out[f"chol_{tag}_H"] = npy(H)
        damp = 0.01
        while 1 > damp > 0:
            try:
                Ht = H.clone()
                Ht.diagonal().add_(damp * torch.mean(torch.diag(H)))
                L = torch.linalg.cholesky(Ht)
                Hinv = torch.cholesky_inverse(L)
                U = torch.linalg.cholesky(Hinv, upper=True)
                if torch.isnan(U).any():
                    raise torch._C._LinAlgError
                break
            except torch._C._LinAlgError:
                damp += 0.0015
        out[f"chol_{tag}_U"] = npy(U)
        out[f"chol_{tag}_damp"] = np.array(damp)
    for bits in (2, 3, 4, 8):
        lo, hi = -(2 ** (bits - 1)), 2 ** (bits - 1) - 1
        codes = torch.randint(lo, hi + 1, (6, 37), generator=gen).to(torch.int8)
        out[f"pack_b{bits}_codes"] = npy(codes)
        out[f"pack_b{bits}_packed"] = npy(pack_to_int32(codes, bits))
    save("misc.npz", **out)


# ---------------------------------------------------------------------------
# compressed-tensors export (utils/compressed_tensors_utils.py)
# ---------------------------------------------------------------------------

EXPORT_IGNORE_CASES = [
    ["re:^mtp.*", "lm_head"],
    ["model.layers.0.self_attn.q_proj", "model.layers.3.self_attn.v_proj", "lm_head"],
    ["model.layers.1.linear_attn.in_proj_qkv", "model.layers.1.linear_attn.in_proj_b",
     "model.layers.1.linear_attn.in_proj_z", "model.layers.2.mlp.gate"],
]
EXPORT_LINEARS = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                  "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"]
EXPORT_GS = 32


def export_tiny_model():
    """The tiny Llama the export fixture is written from (seeded, CPU)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(1234)
    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=1,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=128,
                      max_position_embeddings=64)
    return cfg, LlamaForCausalLM(cfg).to(torch.bfloat16)


def export_codes(model):
    """Seeded int4 codes and group scales for every linear of the decoder layer."""
    gen = torch.Generator().manual_seed(99)
    out = {}
    layer = model.model.layers[0]
    for name in EXPORT_LINEARS:
        mod = layer.get_submodule(name)
        R, C = mod.weight.shape
        out[name + "__codes"] = torch.randint(-8, 8, (R, C), generator=gen, dtype=torch.int8)
        out[name + "__scale"] = torch.rand(R, C // EXPORT_GS, generator=gen) * 0.01 + 1e-3
    return out


class _Saver:
    def save_pretrained(self, path):
        pass


def export_table(path):
    """{tensor name: [dtype, shape, sha256 of the bytes]} of a saved checkpoint."""
    import hashlib
    import glob
    from safetensors.torch import load_file
    table = {}
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        for k, v in load_file(f).items():
            b = v.contiguous().view(torch.uint8).numpy().tobytes()
            table[k] = [str(v.dtype), list(v.shape), hashlib.sha256(b).hexdigest()]
    return table


def gen_export(ref_root):
    import json
    import tempfile
    from utils import compressed_tensors_utils as ctu
    cases = [[c, ctu.expand_ignore_list(c)] for c in EXPORT_IGNORE_CASES]
    cfg, model = export_tiny_model()
    codes = export_codes(model)
    layer = model.model.layers[0]
    mods = []
    for name in EXPORT_LINEARS:
        mod = layer.get_submodule(name)
        R, C = mod.weight.shape
        scale = codes[name + "__scale"].repeat_interleave(EXPORT_GS, dim=1)
        ctu.compress(mod, scale, codes[name + "__codes"].float(), 4, EXPORT_GS)
        mods.append(mod)
    ctu.register_qparam_buffers(mods)
    with tempfile.TemporaryDirectory() as d:
        ctu.save_to_compressed_tensors("tiny", cfg, model, _Saver(), _Saver(), d, bits=4,
                                       group_size=EXPORT_GS, sym=True)
        table = export_table(d)
        with open(os.path.join(d, "config.json")) as f:
            qcfg = json.load(f)["quantization_config"]
    with open(os.path.join(HERE, "export.json"), "w") as f:
        json.dump({"ignore_cases": cases, "quantization_config": qcfg, "tensors": table}, f,
                  indent=1, sort_keys=True)
    save("export.npz", **{k: npy(v) for k, v in codes.items()})
    print("wrote", os.path.join(HERE, "export.json"), len(table), "tensors")

# ---------------------------------------------------------------------------
# G2PTQ refresh step: saliency / gradient caches and the block-loss heads
# ---------------------------------------------------------------------------

REFRESH_D, REFRESH_HID, REFRESH_V, REFRESH_G = 16, 32, 40, 4
# (loss type, head, kl_topk, seed offset, retain_graph) per batch, in call order
REFRESH_CALLS = [("block", "kl", 0, 100, True), ("topk", "kl", 8, 300, True),
                 ("patch", "mse", 0, 200, False)]
REFRESH_WEIGHTS = {"block": 1.0, "topk": 0.25, "patch": 0.5}
REFRESH_BATCHES = 2


def refresh_block(params):
    """The two-linear block ``b(relu(a(x)))`` and the logit head of the
    refresh fixtures, built from the arrays in ``params``."""
    nn = torch.nn
    a = nn.Linear(REFRESH_D, REFRESH_HID)
    b = nn.Linear(REFRESH_HID, REFRESH_D)
    head = nn.Linear(REFRESH_D, REFRESH_V, bias=False)
    with torch.no_grad():
        a.weight.copy_(torch.as_tensor(params["Wa"]))
        a.bias.copy_(torch.as_tensor(params["ba"]))
        b.weight.copy_(torch.as_tensor(params["Wb"]))
        b.bias.copy_(torch.as_tensor(params["bb"]))
        head.weight.copy_(torch.as_tensor(params["Wh"]))
    head.weight.requires_grad_(False)
    return a, b, head


def gen_refresh(ref):
    """The reference's SaliencyCache / GradientCache and its two loss
    functions over a seeded two-linear block (g2ptq_utils.py:586-766 and
    969-1035), replayed as in its per-layer loop (:1263-1383).  The labels,
    top-k indices and noise each call drew are re-drawn from the same seed and
    stored, so the oracle can replay the calls without the generator."""
    g2 = ref.g2ptq
    g2.offload_utils.zero_onloaded_grads = lambda: None
    gen = torch.Generator().manual_seed(11)
    params = {
        "Wa": torch.randn(REFRESH_HID, REFRESH_D, generator=gen) * 0.3,
        "ba": torch.randn(REFRESH_HID, generator=gen) * 0.1,
        "Wb": torch.randn(REFRESH_D, REFRESH_HID, generator=gen) * 0.3,
        "bb": torch.randn(REFRESH_D, generator=gen) * 0.1,
        "Wh": torch.randn(REFRESH_V, REFRESH_D, generator=gen),
    }
    a, b, head = refresh_block(params)
    full = {"a": a, "b": b}
    sc = g2.SaliencyCache(["a", "b"], REFRESH_G)
    sc.set_forward_hook(full)
    gc = g2.GradientCache(["a", "b"], REFRESH_G)
    gc.set_forward_hook(full)
    out = {k: npy(v) for k, v in params.items()}
    for j in range(REFRESH_BATCHES):
        x = torch.randn(2, 5, REFRESH_D, generator=gen)
        hfp = torch.randn(2, 5, REFRESH_D, generator=gen)
        out[f"x{j}"], out[f"hfp{j}"] = npy(x), npy(hfp)
        with torch.enable_grad():
            h = b(torch.relu(a(x)))
            for loss_type, kind, topk, seed, retain in REFRESH_CALLS:
                args = types.SimpleNamespace(kl_topk=topk)
                torch.manual_seed(seed + j)
                if kind == "kl":
                    logits, logits_fp = head(h), head(hfp)
                    loss = g2.compute_kl_grad_hessian(logits, logits_fp, sc, gc, full, args,
                                                      loss_type=loss_type,
                                                      retain_graph=retain)
                    lf = logits_fp.detach()
                    if topk > 0:
                        lf, idx = lf.topk(topk, dim=-1, sorted=False)
                        out[f"idx{j}_{loss_type}"] = npy(idx)
                    torch.manual_seed(seed + j)
                    out[f"labels{j}_{loss_type}"] = npy(
                        torch.distributions.Categorical(logits=lf).sample())
                else:
                    loss = g2.compute_mse_grad_hessian(h, hfp, sc, gc, full, args,
                                                       loss_type=loss_type,
                                                       retain_graph=retain)
                    torch.manual_seed(seed + j)
                    out[f"noise{j}_{loss_type}"] = npy(torch.distributions.Normal(
                        loc=torch.zeros_like(h), scale=float(np.sqrt(REFRESH_D))).sample())
                out[f"loss{j}_{loss_type}"] = np.float32(float(loss))
    sc.clear_hook()
    gc.clear_hook()
    weights = g2.normalize_loss_weights(dict(REFRESH_WEIGHTS))
    sc.summarize_saliency(weights)
    gc.summarize_gradients(weights)
    for name in ("a", "b"):
        for j, s in enumerate(sc.saliency_cache[name]):
            out[f"sal_{name}{j}"] = npy(s)
        out[f"grad_{name}"] = npy(gc.gradients_cache[name])

    # the two cache hooks on their own, at shapes the block does not reach
    sc2 = g2.SaliencyCache(["s"], 3)
    sc2.hooks_enabled = True
    gs = torch.randn(3, 5, 12, generator=gen)
    sc2.grad_hook(gs, name="s", loss_type="block")
    out["sal_in"], out["sal_out"] = npy(gs), npy(sc2.saliency_cache["s"]["block"][0])
    gc2 = g2.GradientCache(["w"], 4)
    gc2.hooks_enabled = True
    for i, n_tok in enumerate((10, 4, 7)):
        gw = torch.randn(6, 7, generator=gen)
        gc2.current_batch_tokens["w"] = n_tok
        gc2.cache_gradient(gw, name="w", loss_type="block")
        out[f"rm_in{i}"] = npy(gw)
    out["rm_out"] = npy(gc2.gradients_cache["w"]["block"])
    save("refresh.npz", **{k: np.asarray(v) for k, v in out.items()})


# ---------------------------------------------------------------------------
# MoE expert stacking before export
# ---------------------------------------------------------------------------

STACK_E, STACK_HID, STACK_INTER = 3, 16, 8


def stack_container(arrays, packed):
    """An experts container (``num_experts``, submodules "0".."E-1" with
    gate/up/down linears) holding the per-expert tensors in ``arrays``:
    compressed buffers (``weight_packed`` / ``weight_scale`` / ``weight_shape``)
    when ``packed``, else bf16 weights.  bf16 arrays are stored as int16 bits."""
    nn = torch.nn
    experts = nn.ModuleList()
    experts.num_experts = STACK_E
    for i in range(STACK_E):
        e = nn.Module()
        for part, (rows, cols) in (("gate_proj", (STACK_INTER, STACK_HID)),
                                   ("up_proj", (STACK_INTER, STACK_HID)),
                                   ("down_proj", (STACK_HID, STACK_INTER))):
            lin = nn.Linear(cols, rows, bias=False)
            if packed:
                del lin.weight
                lin.register_buffer("weight_packed",
                                    torch.as_tensor(arrays[f"{part}{i}_packed"]))
                lin.register_buffer("weight_scale", torch.as_tensor(
                    arrays[f"{part}{i}_scale"]).view(torch.bfloat16))
                lin.register_buffer("weight_shape", torch.tensor([rows, cols]))
            else:
                lin.weight = nn.Parameter(torch.as_tensor(
                    arrays[f"{part}{i}_weight"]).view(torch.bfloat16), requires_grad=False)
            setattr(e, part, lin)
        experts.append(e)
    return experts


def gen_stack():
    """The reference's ``MoEMixin.stack_experts`` (utils/models/mixins.py:93-144)
    on a seeded container, with and without packed weights."""
    from utils.models import mixins
    gen = torch.Generator().manual_seed(21)
    arrays = {}
    for i in range(STACK_E):
        for part, (rows, cols) in (("gate_proj", (STACK_INTER, STACK_HID)),
                                   ("up_proj", (STACK_INTER, STACK_HID)),
                                   ("down_proj", (STACK_HID, STACK_INTER))):
            arrays[f"{part}{i}_packed"] = npy(torch.randint(
                -2 ** 31, 2 ** 31 - 1, (rows, cols // 8), generator=gen, dtype=torch.int64
            ).to(torch.int32))
            arrays[f"{part}{i}_scale"] = npy((torch.rand(rows, cols // 8, generator=gen) + 0.1)
                                             .to(torch.bfloat16).view(torch.int16))
            arrays[f"{part}{i}_weight"] = npy(torch.randn(rows, cols, generator=gen)
                                              .to(torch.bfloat16).view(torch.int16))
    out = dict(arrays)
    for packed in (True, False):
        experts = stack_container(arrays, packed)
        mixins.MoEMixin.stack_experts(None, experts, weight_packed=packed)
        names = (["gate_up_proj_packed", "down_proj_packed", "gate_up_proj_scale",
                  "down_proj_scale", "gate_up_proj_shape", "down_proj_shape"] if packed
                 else ["gate_up_proj", "down_proj"])
        for n in names:
            t = getattr(experts, n).detach()
            out[f"out_{n}"] = npy(t.view(torch.int16) if t.dtype == torch.bfloat16 else t)
        out[f"left_{int(packed)}"] = np.asarray(len(experts._modules))
    save("stack_experts.npz", **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default=None,
                    help="one fixture family: export, refresh, stack or approx")
    args = ap.parse_args()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    ref = import_reference(os.path.abspath(args.reference))
    if args.only == "export":
        gen_export(os.path.abspath(args.reference))
        return
    if args.only == "refresh":
        gen_refresh(ref)
        return
    if args.only == "stack":
        gen_stack()
        return
    if args.only == "approx":
        gen_approx(ref)
        return
    gen_hessians(ref)
    gen_blocks(ref)
    gen_fasterquant(ref)
    gen_misc(ref)
    gen_export(os.path.abspath(args.reference))
    gen_refresh(ref)
    gen_stack()
    gen_approx(ref)


if __name__ == "__main__":
    main()
