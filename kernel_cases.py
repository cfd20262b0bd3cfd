"""Single-kernel cases of the quantization hot path, for timing and profiling.

    python kernel_cases.py gram --tokens 16384 --columns 4096
    python kernel_cases.py gram_weighted --tokens 16384 --columns 4096
    python kernel_cases.py gram_grouped --tokens 16384 --columns 4096
    python kernel_cases.py chol --columns 4096 [--batch 64]
    python kernel_cases.py compensate --rows 4096 --columns 4096 [--bits 4 --groupsize 128]
    python kernel_cases.py sweep [--tokens 262144]
    python kernel_cases.py block_loss --tokens 2048 --vocab 128256 --loss kl
    python kernel_cases.py saliency --tokens 8192 --rows 14336
    python kernel_cases.py running_mean --rows 14336 --columns 4096

Each case builds seeded synthetic inputs of one fold / one factorization /
one compensation pass of a Llama-3-8B linear on ``cuda:0``, runs ``--warmup``
untimed repetitions and ``--reps`` timed ones (CUDA events on the launching
stream), and prints one JSON line with the average duration and the
algorithmic work per repetition.  Used as the workload of the profiler
captures: ``-k`` selects the kernel, ``-s`` skips the warm-up launches.
"""

import argparse
import json

import torch

from g2ptq_b200 import ops, _lib


def _time(fn, warmup, reps):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    torch.cuda.nvtx.range_push("timed")  # profilers can restrict a capture to these launches
    for _ in range(reps):
        fn()
    torch.cuda.nvtx.range_pop()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def gram(args, g):
    """One add_batch fold: H <- a H + b X^T X over T staged BF16 tokens."""
    T, C = args.tokens or 16384, args.columns
    X = torch.randn(T, C, device="cuda", generator=g)
    X[:, :4] *= 20
    X = X.to(torch.bfloat16)
    H = torch.zeros(C, C, device="cuda")
    ms = _time(lambda: ops.gram_update(H, X, alpha=0.5, beta=2.0 / T, precision=1),
               args.warmup, args.reps)
    flops = T * C * (C + 1)          # upper triangle incl. diagonal, 2 flops per MAC
    bytes_ = T * C * 2 + 2 * C * C * 4
    return dict(case="gram", tokens=T, columns=C, ms=ms, tflops=flops / ms / 1e9,
                algorithmic_bytes=bytes_, flops=flops)


def gram_weighted(args, g):
    """One G2PTQ fold: H[k] <- a H[k] + b X^T diag(s_k) X for the four row groups
    (per-token saliency weights s, BF16 tokens)."""
    T, C = args.tokens or 16384, args.columns
    X = torch.randn(T, C, device="cuda", generator=g)
    X[:, :4] *= 20
    X = X.to(torch.bfloat16)
    S = torch.rand(T, 4, device="cuda", generator=g)
    H = torch.zeros(4, C, C, device="cuda")

    def run():
        for k in range(4):
            ops.gram_update(H[k], X, X, row_scale=S[:, k], alpha=0.5, beta=1.0 / T,
                            symmetric=True, precision=1)

    ms = _time(run, args.warmup, args.reps)
    flops = 4 * T * C * (C + 1)
    return dict(case="gram_weighted", tokens=T, columns=C, ms=ms, tflops=flops / ms / 1e9,
                flops=flops)


def _hessian(C, g, batch=1):
    H = torch.zeros(batch, C, C, device="cuda")
    for b in range(batch):
        X = torch.randn(2 * C, C, device="cuda", generator=g).to(torch.bfloat16)
        ops.gram_update(H[b], X, alpha=0.0, beta=1.0 / (2 * C), precision=1)
    return H


def gram_grouped(args, g):
    """One G2PTQ fold as the quantizer object runs it: the four row groups'
    Grams H[k] <- a H[k] + b X^T diag(s_k) X in one grouped launch (one split
    pass of X into the scaled bf16 pairs of all groups, one batched CTA-pair
    launch).  Algorithmic work: four upper-triangle Grams."""
    T, C = args.tokens or 16384, args.columns
    X = torch.randn(T, C, device="cuda", generator=g)
    X[:, :4] *= 20
    X = X.to(torch.bfloat16)
    S = torch.rand(T, 4, device="cuda", generator=g)
    H = torch.zeros(4, C, C, device="cuda")
    ms = _time(lambda: ops.gram_update_grouped(H, X, S, alpha=0.5, beta=1.0 / T, precision=1),
               args.warmup, args.reps)
    flops = 4 * T * C * (C + 1)
    return dict(case="gram_grouped", tokens=T, columns=C, ms=ms, tflops=flops / ms / 1e9,
                flops=flops)


def chol(args, g):
    """Damped inverse-Cholesky factors of ``batch`` C x C Hessians in one call
    (a layer-batched object's factorization)."""
    C, B = args.columns, args.batch
    H = _hessian(C, g, B)
    ms = _time(lambda: ops.chol_upper_inverse(H, 0.01, precision=1), args.warmup, args.reps)
    flops = B * 2 * C ** 3 / 3
    return dict(case="chol", columns=C, batch=B, ms=ms, tflops=flops / ms / 1e9, flops=flops)


def _compensate_pass(R, C, bits, gs, U, g, warmup, reps, dynamic=False):
    """One GPTQ compensation pass (symmetric, groups of ``gs``) of an R x C
    weight with the factor U: average ms over ``reps``.  Static groups take
    their parameters before the pass; dynamic groups (act-order off, the
    reference's default) find them inside it at each group's first column."""
    W = torch.randn(1, R, C, device="cuda", generator=g) * 0.02
    ng = C // gs
    scale = torch.empty(R, ng, device="cuda")
    zero = torch.empty_like(scale)
    if not dynamic:
        for gi in range(ng):
            ops.find_params(scale, zero, W[0][:, gi * gs:(gi + 1) * gs], bits, True,
                            param_col=gi)
    colgroup = (torch.arange(C, device="cuda") // gs).to(torch.int32)
    codes = torch.empty(1, R, C, dtype=torch.int8, device="cuda")
    Wp = W.clone()

    def run():
        Wp.copy_(W)
        # block size 128, as the reference
        ops.compensate(_lib.METHOD_GPTQ, Wp, U, scale, zero, colgroup, dynamic, gs, bits, True,
                       128, codes, precision=1)

    return _time(run, warmup, reps)


def _compensate_units(R, C):
    # 11 B per weight (read W fp32, write Q bf16, code int8, error fp32) and the
    # trailing updates: sum over blocks of 2 R * 128 * (C - i2) = R C (C - 128) flop
    return 11 * R * C, R * C * (C - 128)


def compensate(args, g):
    """One GPTQ compensation pass (sym, static groups) over R x C."""
    R, C = args.rows, args.columns
    U, _ = ops.chol_upper_inverse(_hessian(C, g), 0.01, precision=1)
    ms = _compensate_pass(R, C, args.bits, args.groupsize, U, g, args.warmup, args.reps)
    b, flops = _compensate_units(R, C)
    return dict(case="compensate", rows=R, columns=C, bits=args.bits, groupsize=args.groupsize,
                ms=ms, gbs=b / ms / 1e6, tflops=flops / ms / 1e9, flops=flops)


SWEEP_SHAPES = [(4096, 4096), (4096, 14336), (8192, 8192), (8192, 28672), (14336, 4096),
                (28672, 8192)]  # (columns, rows)


def _heavy_tailed_tokens(T, C, g, heavy):
    """T tokens ~N(0, 1) in fp32 whose ``heavy`` channels are Student-t (nu = 3)."""
    X = torch.randn(T, C, device="cuda", generator=g)
    z = torch.randn(T, heavy.numel(), device="cuda", generator=g)
    chi2 = (torch.randn(3, T, heavy.numel(), device="cuda", generator=g) ** 2).sum(0)
    X[:, heavy] = z / torch.sqrt(chi2 / 3.0)
    return X


def sweep(args, g):
    """The operator sweep: per column count, the Hessian of ``tokens`` fp32
    tokens (~N(0, 1), 1% Student-t channels) folded chunk by chunk (Gram
    TFLOP/s), its damped inverse-Cholesky factor (ms), and GPTQ compensation
    passes (act-order off: groups found inside the pass) at bits 2/3/4 x group
    64/128 for each row count of the column count (GB/s of the 11 B per
    weight, and the trailing updates' TFLOP/s).  One JSON line per
    measurement."""
    T, chunk = args.tokens or 262144, 16384
    out = []
    for C in sorted({c for c, _ in SWEEP_SHAPES}):
        heavy = torch.randperm(C, device="cuda", generator=g)[:max(1, C // 100)]
        H = torch.zeros(C, C, device="cuda")
        X = _heavy_tailed_tokens(chunk, C, g, heavy)
        ops.gram_update(H, X, alpha=0.0, beta=1.0, precision=1)  # untimed first fold
        n = 0
        fold_ms = 0.0
        for t0 in range(0, T, chunk):
            if t0:
                X = _heavy_tailed_tokens(chunk, C, g, heavy)
            torch.cuda.synchronize()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            ops.gram_update(H, X, alpha=n / (n + chunk), beta=2.0 / (n + chunk), precision=1)
            e.record()
            torch.cuda.synchronize()
            fold_ms += s.elapsed_time(e)
            n += chunk
        del X
        gflops = T * C * (C + 1)
        line = dict(case="sweep_gram", columns=C, tokens=T, dtype="f32", ms=fold_ms,
                    tflops=gflops / fold_ms / 1e9)
        print(json.dumps(line), flush=True)
        out.append(line)
        H = H[None].contiguous()
        ms = _time(lambda: ops.chol_upper_inverse(H, 0.01, precision=1), 1, 2)
        U, info = ops.chol_upper_inverse(H, 0.01, precision=1)
        cf = 2 * C ** 3 / 3
        line = dict(case="sweep_chol", columns=C, ms=ms, tflops=cf / ms / 1e9,
                    info=int(info[0].item()))
        print(json.dumps(line), flush=True)
        out.append(line)
        del H
        for c2, R in SWEEP_SHAPES:
            if c2 != C:
                continue
            for bits in (2, 3, 4):
                for gs in (64, 128):
                    ms = _compensate_pass(R, C, bits, gs, U, g, 1, 3, dynamic=True)
                    b, flops = _compensate_units(R, C)
                    line = dict(case="sweep_compensate", columns=C, rows=R, bits=bits,
                                groupsize=gs, groups="dynamic", ms=ms, gbs=b / ms / 1e6,
                                tflops=flops / ms / 1e9)
                    print(json.dumps(line), flush=True)
                    out.append(line)
        del U
        torch.cuda.empty_cache()
    return dict(case="sweep", lines=len(out))


def block_loss(args, g):
    """One G2PTQ refresh loss head over ``tokens`` rows of ``vocab`` BF16 logits
    (KL to a second set of logits, cross entropy against sampled labels, or
    the squared error to a target): the forward and the backward kernel,
    timed apart.  Algorithmic bytes: forward reads x (and the target), the
    backward reads them again and writes the gradient."""
    N, V = args.tokens or 16384, args.vocab
    kind = {"kl": _lib.LOSS_KL, "nll": _lib.LOSS_NLL, "mse": _lib.LOSS_MSE}[args.loss]
    x = (torch.randn(N, V, device="cuda", generator=g) * 3).to(torch.bfloat16)
    t = labels = None
    if kind == _lib.LOSS_NLL:
        labels = torch.randint(0, V, (N,), device="cuda", generator=g)
    else:
        t = (x.float() + 0.3 * torch.randn(N, V, device="cuda", generator=g)).to(torch.bfloat16)
    _, stats, x2, t2, lab = ops.block_loss_forward(kind, x, t, labels)
    fwd = _time(lambda: ops.block_loss_forward(kind, x, t, labels), args.warmup, args.reps)
    bwd = _time(lambda: ops.block_loss_backward(kind, stats, x2, t2, lab), args.warmup, args.reps)
    n_in = 1 if kind == _lib.LOSS_NLL else 2
    fb, bb = n_in * N * V * 2, (n_in + 1) * N * V * 2
    return dict(case="block_loss", loss=args.loss, tokens=N, vocab=V, fwd_ms=fwd, bwd_ms=bwd,
                fwd_bytes=fb, bwd_bytes=bb, fwd_gbs=fb / fwd / 1e6, bwd_gbs=bb / bwd / 1e6)


def saliency(args, g):
    """SaliencyCache.grad_hook over a ``tokens`` x ``rows`` BF16 output gradient."""
    T, R = args.tokens or 16384, args.rows
    grad = (torch.randn(T, R, device="cuda", generator=g) * 1e-3).to(torch.bfloat16)
    out = torch.empty(T, 4, device="cuda")
    ms = _time(lambda: ops.saliency(grad, 4, out=out), args.warmup, args.reps)
    b = T * R * 2 + T * 4 * 4
    return dict(case="saliency", tokens=T, rows=R, ms=ms, bytes=b, gbs=b / ms / 1e6)


def running_mean(args, g):
    """GradientCache.cache_gradient over a ``rows`` x ``columns`` BF16 weight gradient."""
    R, C = args.rows, args.columns
    grad = (torch.randn(R, C, device="cuda", generator=g) * 1e-3).to(torch.bfloat16)
    cache = torch.zeros(R, C, device="cuda")
    ms = _time(lambda: ops.running_mean(cache, grad, 0.5, 1.0 / 4096, False), args.warmup,
               args.reps)
    b = R * C * (2 + 4 + 4)
    return dict(case="running_mean", rows=R, columns=C, ms=ms, bytes=b, gbs=b / ms / 1e6)


CASES = {"gram": gram, "gram_weighted": gram_weighted, "gram_grouped": gram_grouped,
         "chol": chol,
         "compensate": compensate, "block_loss": block_loss, "saliency": saliency,
         "running_mean": running_mean, "sweep": sweep}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens of a fold / loss / saliency case (16384), of the sweep's "
                         "Hessians (262144)")
    ap.add_argument("--columns", type=int, default=4096)
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--loss", choices=["kl", "nll", "mse"], default="kl")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--groupsize", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    print(json.dumps(CASES[args.case](args, g)), flush=True)


if __name__ == "__main__":
    main()
