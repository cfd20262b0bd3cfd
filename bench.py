"""Benchmark of the per-layer quantization hot path (see the driver contract).

Workload: one Llama-3-8B decoder layer -- q/k/v/o/gate/up/
down linears (4096x4096, 1024x4096 x2, 4096x4096, 14336x4096 x2, 4096x14336),
GPTQ W4 symmetric, group 128, damp 0.01, act-order with static groups,
compressed-tensors export on, calibrated on 128 sequences x 2048 tokens.  One
step = every ``add_batch`` call of the calibration pass (one per sequence and
linear, ``--bsz 1``) followed by ``fasterquant`` of all seven linears (their
device work overlapped on a small stream pool by ``fasterquant_all``).
Activations are seeded synthetic BF16 hidden states N(0, 1) with 4 outlier
channels x20 per linear input (the stand-in for the model forward over
uniform random token ids); weights are random N(0, 0.02) BF16.

Metric: linear layers quantized per second (whole job); ``config`` also
reports the implied end-to-end calibration seconds of the 32-layer model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
"""

import argparse
import json
import os
import subprocess
import threading
import time

import numpy as np

HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM, N_LAYERS = 4096, 14336, 32, 8, 128, 32
LINEARS = [  # name, rows, columns, input group
    ("self_attn.q_proj", HEADS * HEAD_DIM, HIDDEN, "attn"),
    ("self_attn.k_proj", KV_HEADS * HEAD_DIM, HIDDEN, "attn"),
    ("self_attn.v_proj", KV_HEADS * HEAD_DIM, HIDDEN, "attn"),
    ("self_attn.o_proj", HIDDEN, HEADS * HEAD_DIM, "o"),
    ("mlp.gate_proj", INTER, HIDDEN, "mlp"),
    ("mlp.up_proj", INTER, HIDDEN, "mlp"),
    ("mlp.down_proj", HIDDEN, INTER, "down"),
]
GROUP_COLS = {"attn": HIDDEN, "o": HEADS * HEAD_DIM, "mlp": HIDDEN, "down": INTER}
BITS, GROUPSIZE, PERCDAMP, BLOCKSIZE = 4, 128, 0.01, 128
METRIC = "linear layers quantized/sec"
# BASELINE configs[1] (GPTQ, the headline) and configs[2] (G2PTQ)
METHODS = {
    "gptq": dict(bits=4, sym=True, label="GPTQ W4 sym g128 act-order",
                 fq=dict(groupsize=GROUPSIZE, actorder=True, static_groups=True)),
    "g2ptq": dict(bits=3, sym=False, label="G2PTQ W3 asym g128, 4 row groups, trust radius 1.0",
                  fq=dict(groupsize=GROUPSIZE, actorder=False, static_groups=False,
                          enable_gradient_update=True, alpha=1.0)),
}
G2_GROUPS = 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--seqs", type=int, default=128)
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--precision", type=int, default=None,
                    help="0: fp32 CUDA-core products, 1: tcgen05 tensor cores")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--method", default="gptq", choices=sorted(METHODS),
                    help="gptq: BASELINE configs[1] (default); g2ptq: configs[2]")
    ap.add_argument("--model", default="llama3-8b", choices=["llama3-8b", "qwen3-moe"],
                    help="llama3-8b: one decoder layer's 7 linears (configs[1] / [2]); "
                         "qwen3-moe: one Qwen3-30B-A3B MoE layer's 128 experts x 3 projections "
                         "(configs[3])")
    ap.add_argument("--moe-bsz", type=int, default=32,
                    help="sequences per forward batch of the MoE workload (one add_batch call "
                         "per hit expert and batch)")
    ap.add_argument("--multi", default="owner", choices=["rows", "owner"],
                    help="N>1: owner = the reference's flow over the coalesced collectives "
                         "(reduce to owners, each owner quantizes its layers, one broadcast "
                         "per owner; the default, measured faster at N=2 and 4); rows = "
                         "fasterquant_rows (the largest factorization shared, its rows split "
                         "over all ranks, one gather)")
    return ap.parse_args()


def load_peaks():
    """HBM GB/s and the dense bf16 TFLOP/s a kernel timed inside a long step can
    reach (the sustained figure: the Gram launches run back to back for seconds)."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1400.0, "fallback"


# DRAM traffic of one Gram fold at the bench's 4096-column fold shape (16384 BF16
# tokens): dram__bytes_read.sum + dram__bytes_write.sum of the CTA-pair kernel in
# one ncu capture of `kernel_cases.py gram --tokens 16384 --columns 4096`.  A
# static figure (the bench runs without a profiler); the algorithmic bytes of
# that launch are 268.4 MB (X once, H read and written once).
GRAM_FOLD_TRAFFIC_BYTES = 317.06e6
# device buffers (one calibration sequence each) of the host-input copy ring
E2E_RING = 48
GRAM_FOLD_ALGORITHMIC_BYTES = 268.44e6


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _run(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 2 + i and s[2 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# native arm
# ---------------------------------------------------------------------------

def make_inputs(torch, dev, rank, world, seqs, seq_len):
    """Per-rank shard of the calibration activations (the reference splits the
    calibration set by rank, gptq_utils/main.py:32-37)."""
    lo, hi = seqs * rank // world, seqs * (rank + 1) // world
    n = hi - lo
    g = torch.Generator(device=dev).manual_seed(43 + rank)
    acts = {}
    for grp, C in GROUP_COLS.items():
        out = torch.empty(n, seq_len, C, device=dev, dtype=torch.bfloat16)
        idx = torch.randperm(C, device=dev, generator=g)[:4]
        for s in range(0, n, 8):
            x = torch.randn(min(8, n - s), seq_len, C, device=dev, generator=g)
            x[..., idx] *= 20.0
            out[s:s + 8] = x.to(torch.bfloat16)
        acts[grp] = out
    return acts, n


def make_g2ptq_inputs(torch, dev, acts, n_local, seq_len, seed):
    """Saliency and gradient inputs of G2PTQ from synthetic per-token
    output gradients N(0, 1e-3) BF16 [tokens, rows] of every linear:
    s[n, g] = mean over the rows of group g of grad_out[n, r]^2 (the saliency
    cache, g2ptq_utils.py:611-618) and the weight gradient = mean over sequences of
    grad_out^T X / tokens (g2ptq_utils.py:704-714).  Made once, outside the timed
    region (the reference's refresh step that produces them is not on the path)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    sal, grad = {}, {}
    for name, rows, cols, grp in LINEARS:
        sal[name] = []
        acc = torch.zeros(rows, cols, device=dev, dtype=torch.float32)
        for s in range(n_local):
            go = (torch.randn(seq_len, rows, device=dev, generator=g) * 1e-3).to(torch.bfloat16)
            gf = go.float()
            sal[name].append((gf * gf).reshape(seq_len, G2_GROUPS, rows // G2_GROUPS).mean(-1))
            acc += (go.T @ acts[grp][s]).float() / seq_len
        grad[name] = acc / n_local
    return {"sal": sal, "grad": grad}


def make_layers(torch, dev):
    g = torch.Generator(device=dev).manual_seed(42)
    layers = {}
    for name, rows, cols, _ in LINEARS:
        lin = torch.nn.Linear(cols, rows, bias=False, device=dev, dtype=torch.bfloat16)
        lin.weight.data = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(
            torch.bfloat16)
        layers[name] = lin
    return layers


def one_step(torch, layers, acts, n_local, world, rank, dist, method="gptq", g2=None,
             marks=None, multi="rows", phases=None):
    """add_batch over the rank's sequences, reduce to owners, fasterquant, broadcast.

    ``marks``: optional list that receives a CUDA event at the end of the
    calibration phase (every add_batch call and the pending Gram folds, which
    fasterquant_all would run first anyway) and one at the end of the step."""
    from g2ptq_b200.gptq_utils import gptq_utils, g2ptq_utils, common_utils
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    cfg = METHODS[method]
    mod = g2ptq_utils if method == "g2ptq" else gptq_utils
    objs = {}
    for name, rows, cols, grp in LINEARS:
        if method == "g2ptq":
            obj = g2ptq_utils.G2PTQ([layers[name]], [list(g2["sal"][name])],
                                    [g2["grad"][name]], num_groups=G2_GROUPS)
        else:
            obj = gptq_utils.GPTQ([layers[name]])
        q = WeightQuantizer()
        q.configure(cfg["bits"], perchannel=True, sym=cfg["sym"], mse=False)
        obj.quantizer = common_utils.make_group_quantizers(q, cols, GROUPSIZE)
        objs[name] = obj
    for s in range(n_local):
        xs = acts(s) if callable(acts) else {g: acts[g][s:s + 1] for g in acts}
        for name, rows, cols, grp in LINEARS:
            objs[name].add_batch(0, xs[grp], None)
    if marks is not None:
        for o in objs.values():
            o._flush_all()
        marks.append(torch.cuda.Event(enable_timing=True))
        marks[-1].record()
    if world > 1 and multi == "rows" and method == "gptq":
        from g2ptq_b200.gptq_utils import sharded
        sharded.fasterquant_rows(list(objs.values()), blocksize=BLOCKSIZE, percdamp=PERCDAMP,
                                 export_compressed_tensors=True, marks=phases, **cfg["fq"])
    else:
        def mark(name):
            if phases is not None and world > 1:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                phases.append((name, ev))
        owners = objs
        if world > 1:
            specs = list(objs.values())
            _, _, obj2rank = common_utils.partition_layers(specs, world)
            mod.reduce_to_target_rank(specs, obj2rank)
            owners = {k: o for k, o in objs.items() if obj2rank[o] == rank}
            mark("reduce")
        gptq_utils.fasterquant_all(list(owners.values()), blocksize=BLOCKSIZE,
                                   percdamp=PERCDAMP, export_compressed_tensors=True,
                                   **cfg["fq"])
        mark("owner_fasterquant")
        if world > 1:
            common_utils.broadcast_quantized_param(list(objs.values()), obj2rank,
                                                   export_compressed_tensors=True)
            mark("broadcast")
    for o in objs.values():
        o.free()
    if marks is not None:
        marks.append(torch.cuda.Event(enable_timing=True))
        marks[-1].record()
    return objs


class GramTimer:
    """CUDA-event time and algorithmic flops of every Hessian (Gram) launch."""

    def __init__(self, torch):
        self.torch = torch
        self.events = []
        self.flops = 0.0

    def install(self):
        from g2ptq_b200 import ops
        orig = ops.gram_update
        orig_grouped = ops.gram_update_grouped
        timer = self

        def timed_grouped(D, X, scales, alpha=1.0, beta=1.0, precision=0):
            s = timer.torch.cuda.Event(enable_timing=True)
            e = timer.torch.cuda.Event(enable_timing=True)
            s.record()
            orig_grouped(D, X, scales, alpha, beta, precision)
            e.record()
            G, C, _ = D.shape
            timer.flops += G * X.shape[0] * C * (C + 1)
            timer.events.append((s, e))

        def timed(D, A, B=None, row_scale=None, alpha=1.0, beta=1.0, symmetric=None,
                  precision=0):
            s = timer.torch.cuda.Event(enable_timing=True)
            e = timer.torch.cuda.Event(enable_timing=True)
            s.record()
            orig(D, A, B, row_scale, alpha, beta, symmetric, precision)
            e.record()
            T, M = A.shape
            N = (B if B is not None else A).shape[1]
            sym = symmetric if symmetric is not None else (B is None or B is A)
            # algorithmic work: T*C*(C+1) for the symmetric update, 2*T*M*N otherwise
            timer.flops += T * M * (M + 1) if sym else 2.0 * T * M * N
            timer.events.append((s, e))

        ops.gram_update = timed
        ops.gram_update_grouped = timed_grouped
        self._orig = orig
        self._orig_grouped = orig_grouped

    def uninstall(self):
        from g2ptq_b200 import ops
        ops.gram_update = self._orig
        ops.gram_update_grouped = self._orig_grouped

    def total_ms(self):
        return sum(s.elapsed_time(e) for s, e in self.events)


def native(args):
    import torch
    import torch.distributed as dist
    from g2ptq_b200 import _lib
    from g2ptq_b200.gptq_utils import _engine
    if args.precision is not None:
        _engine.PRECISION = args.precision
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)
    lib = _lib.load()
    layers = make_layers(torch, dev)
    acts, n_local = make_inputs(torch, dev, rank, world, args.seqs, args.seq_len)
    g2 = (make_g2ptq_inputs(torch, dev, acts, n_local, args.seq_len, 44 + rank)
          if args.method == "g2ptq" else None)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_step(torch, layers, acts, n_local, world, rank, dist, args.method, g2,
                 multi=args.multi)
    barrier()
    timer = GramTimer(torch)
    timer.install()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = lib.g2q_launch_count()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    marks = [t0]
    phases = []  # per step: the row-sharded path's phase boundaries
    torch.cuda.nvtx.range_push("timed")  # lets a profiler capture exactly the timed steps
    for _ in range(args.steps):
        step_phases = []
        one_step(torch, layers, acts, n_local, world, rank, dist, args.method, g2, marks,
                 multi=args.multi, phases=step_phases)
        phases.append(step_phases)
    torch.cuda.nvtx.range_pop()
    t1.record()
    barrier()
    clk = clocks.stop()
    timer.uninstall()
    launches = lib.g2q_launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    # phase split of this rank's steps: calibration (add_batch + Gram folds) and
    # the rest (reduce, factorization, compensation, export, broadcast)
    calib_ms = sum(marks[2 * i].elapsed_time(marks[2 * i + 1])
                   for i in range(args.steps)) / args.steps
    quant_ms = sum(marks[2 * i + 1].elapsed_time(marks[2 * i + 2])
                   for i in range(args.steps)) / args.steps
    # the quantization phase split at the row-sharded path's events, every rank
    split = {}
    if phases and phases[0]:
        for i, step_marks in enumerate(phases):
            prev = marks[2 * i + 1]
            for name, ev in step_marks:
                split[name] = split.get(name, 0.0) + prev.elapsed_time(ev) / args.steps
                prev = ev
            split["export_and_free"] = (split.get("export_and_free", 0.0) +
                                        prev.elapsed_time(marks[2 * i + 2]) / args.steps)
        split = {k: round(v, 3) for k, v in split.items()}
    per_rank = None
    if world > 1:
        keys = ["add_batch_and_folds"] + (list(split) if split else ["quantize"])
        mine = [calib_ms] + ([split[k] for k in keys[1:]] if split else [quant_ms])
        t = torch.tensor(mine, device=dev, dtype=torch.float64)
        table = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(table, t)
        per_rank = [{k: round(float(v), 3) for k, v in zip(keys, row.tolist())}
                    for row in table]
    gram_ms = timer.total_ms() / args.steps
    gram_tflops = timer.flops / args.steps / (gram_ms * 1e-3) / 1e12 if gram_ms > 0 else 0.0

    e2e = e2e_dev = None
    if not args.no_e2e:
        e2e = native_e2e(torch, dist, args, layers, world, rank, dev, n_local, acts, g2)
        e2e_dev = native_e2e(torch, dist, args, layers, world, rank, dev, n_local, acts, g2,
                             host_inputs=False)
    del acts
    hbm, bf16, peak_kind = load_peaks()
    value = len(LINEARS) / (ms * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "linears/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16-in/f32", "data": "synthetic",
        "config": {
            "workload": f"Llama-3-8B decoder layer (7 linears) {METHODS[args.method]['label']}, "
                        f"{args.seqs}x{args.seq_len} calibration tokens",
            "parallelism": (f"tokens dp{world} + factor ownership (LPT) + row-sharded "
                            "compensation + one all_gather"
                            if world > 1 and args.multi == "rows" and args.method == "gptq"
                            else f"tokens dp{world} + linear ownership (LPT)"),
            "calibration_seconds_32_layers": round(N_LAYERS * ms * 1e-3, 3),
            "phase_ms_rank0": {"add_batch_and_folds": round(calib_ms, 3),
                               "reduce_factor_compensate_export": round(quant_ms, 3),
                               **({"split": split} if split else {})},
            **({"phase_ms_per_rank": per_rank} if per_rank else {}),
            "precision": "tcgen05" if _engine.PRECISION == 1 else "fp32-cuda-core",
            "l2": "inputs larger than L2 (GBs of activations per step)",
        },
        "gpu_launches": int(launches // args.steps) * args.steps,
        "clocks": clk,
        "roofline": {
            "kernel": "Hessian Gram update (g2q_gram_update)",
            "bound": "tensor", "achieved": round(gram_tflops, 2),
            "peak": bf16, "unit": "TFLOP/s",
            "frac": round(gram_tflops / bf16, 4), "traffic": GRAM_FOLD_TRAFFIC_BYTES,
            "traffic_per": "launch, C=4096 x T=16384 fold "
                           f"(algorithmic {GRAM_FOLD_ALGORITHMIC_BYTES:.4g} B)",
            "traffic_source": "static: one ncu capture of the fold kernel, not this run",
            "peak_kind": f"{peak_kind} bf16 dense sustained",
            "share_of_step": round(gram_ms / ms, 3) if ms else None,
        },
    }
    if e2e is not None:
        line["e2e"] = e2e
        # the same API path with the activations already on the device (where a
        # calibration forward produces them) and the results read back
        line["e2e_activations_on_device"] = e2e_dev
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.method == "gptq":
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def native_e2e(torch, dist, args, layers, world, rank, dev, n_local, dev_acts, g2=None,
               host_inputs=True):
    """Same steps through the public API with host-resident inputs: every step
    copies its activations from pinned host memory and reads the quantized
    weights and packed codes back to the host.  The copies stream through a ring
    of sequence buffers on a side stream (as the reference's prefetch_generator
    overlaps its H2D copies), running ahead into the next step's sequences while
    the current step factors and compensates.  ``host_inputs=False``: the
    activations stay where a calibration forward leaves them, on the device,
    and only the results cross to the host."""
    if not host_inputs:
        def device_feed(s):
            return {grp: x[s:s + 1] for grp, x in dev_acts.items()}
    host = ({grp: torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
             for grp, x in dev_acts.items()} if host_inputs else {})
    for grp in host:
        host[grp].copy_(dev_acts[grp])
    side = torch.cuda.Stream(device=dev)
    ring = max(2, min(n_local, E2E_RING)) if host_inputs else 0
    bufs = [{grp: torch.empty(1, args.seq_len, C, dtype=torch.bfloat16, device=dev)
             for grp, C in GROUP_COLS.items()} for _ in range(ring)]
    ready = [torch.cuda.Event() for _ in range(ring)]
    free_ev = [torch.cuda.Event() for _ in range(ring)]
    h2d_bytes = sum(h.numel() * h.element_size() for h in host.values())
    outs = {name: torch.empty(rows, cols, dtype=torch.bfloat16, pin_memory=True)
            for name, rows, cols, _ in LINEARS}
    packed = {}  # pinned host copies of the packed codes, shaped on first use
    state = {"issued": 0, "consumed": 0}  # sequences copied / handed to add_batch so far

    def prefetch_upto(g_end):
        while state["issued"] < g_end:
            g = state["issued"]
            k, s = g % ring, g % n_local
            with torch.cuda.stream(side):
                side.wait_event(free_ev[k])
                for grp in GROUP_COLS:
                    bufs[k][grp].copy_(host[grp][s:s + 1], non_blocking=True)
                ready[k].record(side)
            state["issued"] += 1

    def feed(s):
        g = state["consumed"]
        if g > 0:
            free_ev[(g - 1) % ring].record()  # users of the previous buffer are enqueued
        prefetch_upto(g + ring)  # the slot of g - 1 is free again
        torch.cuda.current_stream().wait_event(ready[g % ring])
        state["consumed"] += 1
        return bufs[g % ring]

    def step():
        one_step(torch, layers, feed if host_inputs else device_feed, n_local, world, rank,
                 dist, args.method, g2, multi=args.multi)
        if host_inputs:
            # free the last buffer and keep the copies running into the next step
            free_ev[(state["consumed"] - 1) % ring].record()
            prefetch_upto(state["consumed"] + ring)
        d2h = 0
        for name, rows, cols, _ in LINEARS:
            outs[name].copy_(layers[name].weight.data, non_blocking=True)
            qp = layers[name].__dict__.get("_export_qparams")
            d2h += rows * cols * 2
            if qp is not None:
                src = qp["weight_packed"]
                if name not in packed:
                    packed[name] = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
                packed[name].copy_(src, non_blocking=True)
                d2h += packed[name].numel() * packed[name].element_size()
        return d2h

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    d2h = 0
    for _ in range(args.steps):
        d2h = step()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    return {"value": round(len(LINEARS) / (ms * 1e-3), 4), "unit": "linears/s",
            "ms_per_step": round(ms, 3), "h2d_bytes_per_step": int(h2d_bytes),
            "d2h_bytes_per_step": int(d2h)}


# ---------------------------------------------------------------------------
# MoE workload: one Qwen3-30B-A3B MoE layer's experts
# ---------------------------------------------------------------------------

MOE_HIDDEN, MOE_INTER, MOE_EXPERTS, MOE_TOPK, MOE_LAYER_BSZ = 2048, 768, 128, 8, 64


def make_moe(torch, dev, rank, world, args):
    """Random-init experts (N(0, 0.02) BF16), a router N(0, 0.02), and this
    rank's share of the calibration tokens routed top-8: per forward batch of
    ``moe_bsz`` sequences the hidden states (BF16 N(0, 1), 4 outlier channels
    x20) gathered into expert order, one contiguous row range per expert, and
    the down projections' inputs (BF16 N(0, 1), the stand-in for
    act(gate) * up).  Made outside the timed region, like the Llama
    workload's activations."""
    g = torch.Generator(device=dev).manual_seed(42)
    experts = {}
    for proj, (rows, cols) in (("gate_proj", (MOE_INTER, MOE_HIDDEN)),
                               ("up_proj", (MOE_INTER, MOE_HIDDEN)),
                               ("down_proj", (MOE_HIDDEN, MOE_INTER))):
        for e in range(MOE_EXPERTS):
            lin = torch.nn.Linear(cols, rows, bias=False, device=dev, dtype=torch.bfloat16)
            lin.weight.data = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(
                torch.bfloat16)
            experts[(proj, e)] = lin
    router = torch.randn(MOE_EXPERTS, MOE_HIDDEN, device=dev, generator=g) * 0.02
    lo, hi = args.seqs * rank // world, args.seqs * (rank + 1) // world
    gx = torch.Generator(device=dev).manual_seed(43 + rank)
    idx_out = torch.randperm(MOE_HIDDEN, device=dev, generator=gx)[:4]
    batches = []
    for s in range(lo, hi, args.moe_bsz):
        n = min(args.moe_bsz, hi - s)
        x = torch.randn(n * args.seq_len, MOE_HIDDEN, device=dev, generator=gx)
        x[:, idx_out] *= 20.0
        x = x.to(torch.bfloat16)
        top = torch.topk(x.float() @ router.T, MOE_TOPK, dim=-1).indices.reshape(-1)
        order = torch.argsort(top, stable=True)
        counts = torch.bincount(top, minlength=MOE_EXPERTS).tolist()
        routed = x[order // MOE_TOPK].contiguous()
        down_in = torch.randn(routed.shape[0], MOE_INTER, device=dev, generator=gx).to(
            torch.bfloat16)
        bounds, c0 = [], 0
        for c in counts:
            bounds.append((c0, c0 + c))
            c0 += c
        batches.append((routed, down_in, bounds))
    return experts, batches


def moe_step(torch, experts, batches, world, rank, dist, marks=None):
    """add_batch of every hit expert per forward batch (gate and up share each
    call's routed tokens), the objects of ``layer_bsz`` = 64 same-shape experts
    (common_utils.build_chunk_specs order), then fasterquant of all of them;
    with several ranks the reference's owner flow."""
    from g2ptq_b200.gptq_utils import gptq_utils, common_utils
    from g2ptq_b200.utils.quant_utils import WeightQuantizer
    objs, where = [], {}
    for proj in ("up_proj", "gate_proj", "down_proj"):
        for c0 in range(0, MOE_EXPERTS, MOE_LAYER_BSZ):
            ids = list(range(c0, min(c0 + MOE_LAYER_BSZ, MOE_EXPERTS)))
            obj = gptq_utils.GPTQ([experts[(proj, e)] for e in ids])
            q = WeightQuantizer()
            q.configure(BITS, perchannel=True, sym=True, mse=False)
            obj.quantizer = common_utils.make_group_quantizers(
                q, experts[(proj, ids[0])].weight.shape[1], GROUPSIZE)
            objs.append(obj)
            for k, e in enumerate(ids):
                where[(proj, e)] = (obj, k)
    for routed, down_in, bounds in batches:
        for e, (a, b) in enumerate(bounds):
            if b == a:
                continue  # the reference calls only the hit experts
            x = routed[a:b]
            for proj in ("up_proj", "gate_proj"):
                o, k = where[(proj, e)]
                o.add_batch(k, x, None)
            o, k = where[("down_proj", e)]
            o.add_batch(k, down_in[a:b], None)
    if marks is not None:
        for o in objs:
            o._flush_all()
        marks.append(torch.cuda.Event(enable_timing=True))
        marks[-1].record()
    kw = dict(blocksize=BLOCKSIZE, percdamp=PERCDAMP, groupsize=GROUPSIZE, actorder=True,
              static_groups=True, export_compressed_tensors=True)
    if world > 1:
        _, _, owner = common_utils.partition_layers(objs, world)
        gptq_utils.reduce_to_target_rank(objs, owner)
        gptq_utils.fasterquant_all([o for o in objs if owner[o] == rank], **kw)
        common_utils.broadcast_quantized_param(objs, owner, export_compressed_tensors=True)
    else:
        gptq_utils.fasterquant_all(objs, **kw)
    for o in objs:
        o.free()
    if marks is not None:
        marks.append(torch.cuda.Event(enable_timing=True))
        marks[-1].record()


def native_moe(args):
    import torch
    import torch.distributed as dist
    from g2ptq_b200 import _lib
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)
    lib = _lib.load()
    experts, batches = make_moe(torch, dev, rank, world, args)
    routed_rows = sum(r.shape[0] for r, _, _ in batches)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        moe_step(torch, experts, batches, world, rank, dist)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = lib.g2q_launch_count()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    marks = [t0]
    torch.cuda.nvtx.range_push("timed")  # lets a profiler capture exactly the timed steps
    for _ in range(args.steps):
        moe_step(torch, experts, batches, world, rank, dist, marks)
    torch.cuda.nvtx.range_pop()
    t1.record()
    barrier()
    clk = clocks.stop()
    launches = lib.g2q_launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    calib = sum(marks[2 * i].elapsed_time(marks[2 * i + 1]) for i in range(args.steps))
    quant = sum(marks[2 * i + 1].elapsed_time(marks[2 * i + 2]) for i in range(args.steps))
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    n_lin = 3 * MOE_EXPERTS
    line = {
        "metric": "expert linear layers quantized/sec", "value": round(n_lin / (ms * 1e-3), 3),
        "unit": "linears/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16-in/f32", "data": "synthetic",
        "config": {
            "workload": "Qwen3-30B-A3B MoE layer: 128 experts x (gate 768x2048, up 768x2048, "
                        "down 2048x768), top-8 routing, GPTQ W4 sym g128 act-order, "
                        f"{args.seqs}x{args.seq_len} tokens, layer_bsz 64",
            "routed_rows_rank0": routed_rows, "forward_batch": args.moe_bsz,
            "add_batch_calls_rank0_per_step": sum(
                3 * sum(1 for a, b in bd if b > a) for _, _, bd in batches),
            "seconds_48_layers": round(48 * ms * 1e-3, 3),
            "phase_ms_rank0": {"add_batch_and_folds": round(calib / args.steps, 3),
                               "reduce_factor_compensate_export": round(quant / args.steps, 3)},
            "parallelism": f"tokens dp{world} + expert-chunk ownership (LPT)",
        },
        "gpu_launches": int(launches), "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's torch path on the host cores
# ---------------------------------------------------------------------------

SAMPLE_ROWS = 4096


def cpu_threads():
    """All host threads this process may use, set explicitly (torchrun exports
    OMP_NUM_THREADS=1 to its workers)."""
    import torch
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_sample():
    """Time the reference's torch operations (``oracle/torch_port.py``) on the
    host cores at the step's two column counts: one 2048-token ``add_batch``
    call at C = 4096 and at C = 14336, and ``fasterquant`` (W4 sym g128,
    act-order, static groups) of a 4096-row linear on each resulting Hessian.
    The step is assembled from the stages: 768 add_batch calls at C = 4096
    (q/k/v/o/gate/up x 128 sequences) and 128 at C = 14336 (down), one
    factorization per linear, the compensation scaled by rows (38912 rows at
    C = 4096, 4096 at C = 14336), the rest of fasterquant (parameters, dead
    columns, permutations) once per linear.  -> (seconds per step, parts)."""
    import torch
    from oracle import torch_port as tp
    threads = cpu_threads()
    g = torch.Generator().manual_seed(0)
    parts, wall0 = {}, time.perf_counter()
    for C in (HIDDEN, INTER):
        X = torch.randn(1, 2048, C, generator=g)
        X[..., :4] *= 20.0
        X = X.to(torch.bfloat16)
        t0 = time.perf_counter()
        H, _ = tp.add_batch(torch.zeros(C, C), 0, X)
        parts[f"add_batch_c{C}"] = time.perf_counter() - t0
        W = (torch.randn(1, SAMPLE_ROWS, C, generator=g) * 0.02).to(torch.bfloat16)
        tim = {}
        t0 = time.perf_counter()
        tp.fasterquant(W, H[None], BITS, True, GROUPSIZE, True, True, PERCDAMP, BLOCKSIZE,
                       timings=tim)
        total = time.perf_counter() - t0
        parts[f"factor_c{C}"] = tim["factor"]
        parts[f"compensate_r{SAMPLE_ROWS}_c{C}"] = tim["compensate"]
        parts[f"other_c{C}"] = total - tim["factor"] - tim["compensate"]
    step = 0.0
    seqs = 128
    for name, rows, cols, _ in LINEARS:
        step += seqs * parts[f"add_batch_c{cols}"]
        step += parts[f"factor_c{cols}"] + parts[f"other_c{cols}"]
        step += parts[f"compensate_r{SAMPLE_ROWS}_c{cols}"] * rows / SAMPLE_ROWS
    return step, parts, time.perf_counter() - wall0, threads


def cpu_warmup():
    """An untimed warm-up step of the CPU arm: the same torch operations at
    C = 1024 (thread pools and allocator warmed in well under a second; the
    full-size sample of a timed step takes tens of seconds)."""
    import torch
    from oracle import torch_port as tp
    cpu_threads()
    g = torch.Generator().manual_seed(1)
    X = torch.randn(1, 2048, 1024, generator=g).to(torch.bfloat16)
    H, _ = tp.add_batch(torch.zeros(1024, 1024), 0, X)
    W = (torch.randn(1, 256, 1024, generator=g) * 0.02).to(torch.bfloat16)
    tp.fasterquant(W, H[None], BITS, True, GROUPSIZE, True, True, PERCDAMP, BLOCKSIZE)


def _sample_text(parts, wall):
    p = ", ".join(f"{k} {v:.3f} s" for k, v in parts.items())
    return (f"reference torch ops on the host (oracle/torch_port.py): one 2048-token add_batch "
            f"call and fasterquant of a 4096-row linear at C=4096 and C=14336 ({wall:.1f} s: "
            f"{p}); step = 128 add_batch calls per linear + one fasterquant per linear, "
            f"compensation scaled by rows")


def cpu_baseline():
    step_s, parts, wall, threads = cpu_sample()
    return {"value": round(len(LINEARS) / step_s, 6), "unit": "linears/s",
            "cores": threads, "kind": "port", "sample": _sample_text(parts, wall)}


def reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_warmup()
    vals, parts, wall, threads = [], None, 0.0, 1
    for _ in range(args.steps):
        s, parts, wall, threads = cpu_sample()
        vals.append(s)
    step_s = float(np.mean(vals))
    value = len(LINEARS) / step_s
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 6),
            "unit": "linears/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(step_s * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "Llama-3-8B decoder layer (7 linears) GPTQ W4 sym g128 "
                                   "act-order, 128x2048 calibration tokens"},
            "cpu_baseline": {"value": round(value, 6), "unit": "linears/s", "cores": threads,
                             "kind": "port", "sample": _sample_text(parts, wall)},
            "e2e": {"value": round(value, 6), "unit": "linears/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        reference(a)
    elif a.model == "qwen3-moe":
        native_moe(a)
    else:
        native(a)
