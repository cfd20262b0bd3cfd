"""Single-kernel cases of the quantization hot path, for timing and profiling.

    python -m g2ptq_b200.kernel_cases gram --tokens 16384 --columns 4096
    python -m g2ptq_b200.kernel_cases gram_weighted --tokens 16384 --columns 4096
    python -m g2ptq_b200.kernel_cases chol --columns 4096
    python -m g2ptq_b200.kernel_cases compensate --rows 4096 --columns 4096

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

from . import ops, _lib


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
    T, C = args.tokens, args.columns
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
    T, C = args.tokens, args.columns
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


def chol(args, g):
    """Damped inverse-Cholesky factor of one C x C Hessian."""
    C = args.columns
    X = torch.randn(2 * C, C, device="cuda", generator=g).to(torch.bfloat16)
    H = torch.zeros(C, C, device="cuda")
    ops.gram_update(H, X, alpha=0.0, beta=1.0 / (2 * C), precision=1)
    H = H[None].contiguous()
    ms = _time(lambda: ops.chol_upper_inverse(H, 0.01, precision=1), args.warmup, args.reps)
    flops = 2 * C ** 3 / 3
    return dict(case="chol", columns=C, ms=ms, tflops=flops / ms / 1e9, flops=flops)


def compensate(args, g):
    """One GPTQ compensation pass (W4 sym, group 128, static groups) over R x C."""
    R, C = args.rows, args.columns
    X = torch.randn(2 * C, C, device="cuda", generator=g).to(torch.bfloat16)
    H = torch.zeros(C, C, device="cuda")
    ops.gram_update(H, X, alpha=0.0, beta=1.0 / (2 * C), precision=1)
    U, _ = ops.chol_upper_inverse(H[None].contiguous(), 0.01, precision=1)
    W = torch.randn(1, R, C, device="cuda", generator=g) * 0.02
    ng = C // 128
    scale = torch.empty(R, ng, device="cuda")
    zero = torch.empty_like(scale)
    for gi in range(ng):
        ops.find_params(scale, zero, W[0][:, gi * 128:(gi + 1) * 128], 4, True, param_col=gi)
    colgroup = (torch.arange(C, device="cuda") // 128).to(torch.int32)
    codes = torch.empty(1, R, C, dtype=torch.int8, device="cuda")
    Wp = W.clone()

    def run():
        Wp.copy_(W)
        ops.compensate(_lib.METHOD_GPTQ, Wp, U, scale, zero, colgroup, False, 128, 4, True, 128,
                       codes, precision=1)

    ms = _time(run, args.warmup, args.reps)
    flops = R * C * C  # trailing updates: sum over blocks of 2 R * blk * (C - i2)
    return dict(case="compensate", rows=R, columns=C, ms=ms, tflops=flops / ms / 1e9,
                flops=flops)


CASES = {"gram": gram, "gram_weighted": gram_weighted, "chol": chol,
         "compensate": compensate}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--columns", type=int, default=4096)
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    print(json.dumps(CASES[args.case](args, g)), flush=True)


if __name__ == "__main__":
    main()
