"""End-to-end calibration pass of the Llama-3-8B architecture: the target of
BASELINE configs[1] (GPTQ W4 sym g128, act-order) and configs[2] (G2PTQ W3
asym g128, four row groups, trust radius 1.0, gradients N(0, 1e-3)).

32 random-init decoder layers (hidden 4096, intermediate 14336, 32 / 8 heads
of head_dim 128; linear weights N(0, 0.02) BF16, norms 1), 128 sequences x
2048 uniform random token ids embedded by a random-init 128256-entry table,
calibrated and quantized layer after layer with each layer's quantized
output propagated to the next (``g2ptq_b200.gptq_utils.driver``).  The
calibration set is split by sequences over the ranks of a torchrun job.
Prints one JSON line (seconds of the whole pass, max over ranks, and its
forward / quantization split).

    python calibrate.py [--layers 32] [--method gptq|g2ptq] [--multi owner|rows]
    python -m torch.distributed.run --nproc-per-node 8 calibrate.py ...
"""

import argparse
import json
import os
import time

HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM, VOCAB = 4096, 14336, 32, 8, 128, 128256


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seqs", type=int, default=128)
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--bsz", type=int, default=8, help="sequences per forward batch")
    ap.add_argument("--method", default="gptq", choices=["gptq", "g2ptq"])
    ap.add_argument("--multi", default="owner", choices=["owner", "rows"])
    ap.add_argument("--hidden", type=int, default=HIDDEN)
    ap.add_argument("--intermediate", type=int, default=INTER)
    ap.add_argument("--heads", type=int, default=HEADS)
    ap.add_argument("--kv-heads", type=int, default=KV_HEADS)
    ap.add_argument("--head-dim", type=int, default=HEAD_DIM)
    ap.add_argument("--vocab", type=int, default=VOCAB)
    return ap.parse_args()


def llama_config(args):
    from transformers import LlamaConfig
    cfg = LlamaConfig(hidden_size=args.hidden, intermediate_size=args.intermediate,
                      num_attention_heads=args.heads, num_key_value_heads=args.kv_heads,
                      head_dim=args.head_dim, num_hidden_layers=args.layers,
                      vocab_size=args.vocab, rms_norm_eps=1e-5, rope_theta=500000.0,
                      max_position_embeddings=max(8192, args.seq_len))
    cfg._attn_implementation = "sdpa"
    return cfg


def build_layers(torch, cfg, n_layers, dev, seed=42):
    """Random-init decoder layers in BF16: linears N(0, 0.02), norms 1."""
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for i in range(n_layers):
        layer = LlamaDecoderLayer(cfg, layer_idx=i).to(device=dev, dtype=torch.bfloat16)
        for m in layer.modules():
            if isinstance(m, torch.nn.Linear):
                m.weight.data = (torch.randn(m.weight.shape, device=dev, generator=g) * 0.02
                                 ).to(torch.bfloat16)
        layer.eval()
        layers.append(layer)
    return layers


def calibration_inputs(torch, cfg, args, rank, world, dev, seed=43):
    """This rank's share of the embedded calibration set, in batches of
    ``bsz`` sequences (every rank draws the same token ids)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (args.seqs, args.seq_len), device=dev, generator=g)
    table = (torch.randn(cfg.vocab_size, cfg.hidden_size, device=dev, generator=g) * 0.02).to(
        torch.bfloat16)
    lo, hi = args.seqs * rank // world, args.seqs * (rank + 1) // world
    batches = [table[ids[s:min(s + args.bsz, hi)]] for s in range(lo, hi, args.bsz)]
    del table
    return batches


def main():
    args = parse()
    import torch
    import torch.distributed as dist
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    from g2ptq_b200 import _lib
    from g2ptq_b200.gptq_utils import driver
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)
    _lib.load()
    cfg = llama_config(args)
    layers = build_layers(torch, cfg, args.layers, dev)
    inps = calibration_inputs(torch, cfg, args, rank, world, dev)
    rope = LlamaRotaryEmbedding(cfg, device=dev)
    pos = torch.arange(args.seq_len, device=dev)[None]
    cos, sin = rope(inps[0], pos)
    if args.method == "g2ptq":
        cal = driver.Calibration(method="g2ptq", w_bits=3, w_asym=True, w_groupsize=128,
                                 act_order=False, multi=args.multi, bsz=args.bsz, alpha=1.0)
    else:
        cal = driver.Calibration(method="gptq", w_bits=4, w_asym=False, w_groupsize=128,
                                 act_order=True, multi=args.multi, bsz=args.bsz)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    times = driver.calibrate(cal, layers, inps, (cos, sin))
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    finite = all(bool(torch.isfinite(x).all()) for x in inps)
    vals = torch.tensor([secs, times.get("forward", 0.0), times.get("quantize", 0.0)],
                        device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    secs, fwd, quant = vals.tolist()
    if rank == 0:
        label = ("GPTQ W4 sym g128 act-order" if args.method == "gptq" else
                 "G2PTQ W3 asym g128, 4 row groups, trust radius 1.0, gradients N(0, 1e-3)")
        print(json.dumps({
            "metric": "end-to-end calibration seconds", "value": round(secs, 3), "unit": "s",
            "higher_is_better": False, "n_gpus": world, "layers": args.layers,
            "linears_per_s": round(7 * args.layers / secs, 3),
            "seconds_forward_max_rank": round(fwd, 3),
            "seconds_quantize_max_rank": round(quant, 3),
            "outputs_finite": finite,
            "config": {"workload": f"Llama-3-8B architecture, {args.layers} layers, {label}, "
                                   f"{args.seqs}x{args.seq_len} random token ids",
                       "forward_batch": args.bsz, "multi_gpu": args.multi if world > 1 else None,
                       "data": "synthetic (random-init weights and embedding table)"}}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
