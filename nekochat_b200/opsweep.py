"""Operator sweep on a B200 (the engine's operator set as single C-ABI calls): dequant matmul over
M in {1, 8, 64, 512} x (K, N) in {(1024, 3072), (3072, 1024), (2048, 6144), (2560, 9728), (9728, 2560),
(1024, 151936)} x {FP8, FP4}; RMSNorm and softmax over widths {1024, 2048, 2560, 151936} x rows {1, 64, 4096}.

Inputs are synthetic (seed 0): weights N(0, 0.02) quantized on the GPU by the engine's codec, activations N(0, 1)
fp32. Each launch is timed alone with CUDA events on the launching stream, after 3 warm-up launches, with the
L2 flushed (a 256 MB write) before every timed launch, and the median reported. Bytes are algorithmic:
  matmul  N * rowBytes(K) + M * K * 4 + M * N * 4     (flops 2 * M * N * K)
  norm    8 * rows * C + 4 * C
  softmax 8 * rows * C
Usage: python -m nekochat_b200.opsweep [--quick] [--out FILE.jsonl]
"""
import argparse
import json
import statistics

import numpy as np

MATMUL_SHAPES = [(1024, 3072), (3072, 1024), (2048, 6144), (2560, 9728), (9728, 2560), (1024, 151936)]
MS = [1, 8, 64, 512]
WIDTHS = [1024, 2048, 2560, 151936]
ROWS = [1, 64, 4096]


def timed(fn, flush, reps):
    import torch
    for _ in range(3):
        fn()
    times = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(reps):
        flush.zero_()
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    return statistics.median(times)


def main():
    import torch
    from . import ops
    from .ops import row_bytes

    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="M in {1, 64}, two matrix shapes, rows {1, 4096}")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    shapes = MATMUL_SHAPES[:2] + MATMUL_SHAPES[-1:] if args.quick else MATMUL_SHAPES
    ms = [1, 64] if args.quick else MS
    rows_list = [1, 4096] if args.quick else ROWS
    lines = []

    def emit(d):
        lines.append(d)
        print(json.dumps(d), flush=True)

    for fmt, fname in ((1, "fp8"), (2, "fp4")):
        for K, N in shapes:
            w = torch.randn((N, K), generator=g, device="cuda").mul_(0.02)
            q = ops.quantize(fmt, w)
            del w
            for M in ms:
                x = torch.randn((M, K), generator=g, device="cuda")
                y = torch.empty((M, N), device="cuda")
                reps = args.reps if M * N * K < 2e10 else 3
                t = timed(lambda: ops.matmul(fmt, x, q, K, y=y), flush, reps)
                nbytes = N * row_bytes(fmt, K) + M * K * 4 + M * N * 4
                emit({"op": "matmul", "fmt": fname, "M": M, "K": K, "N": N, "us": t * 1e6,
                      "GB_s": nbytes / t / 1e9, "TFLOP_s": 2.0 * M * N * K / t / 1e12})
            del q
    for C in WIDTHS:
        for rows in rows_list:
            x = torch.randn((rows, C), generator=g, device="cuda")
            gam = torch.ones(C, device="cuda")
            t = timed(lambda: ops.norm(x, gam), flush, args.reps)
            emit({"op": "rmsnorm", "C": C, "rows": rows, "us": t * 1e6, "GB_s": (8 * rows * C + 4 * C) / t / 1e9})
            t = timed(lambda: ops.softmax(x), flush, args.reps)
            emit({"op": "softmax", "C": C, "rows": rows, "us": t * 1e6, "GB_s": 8 * rows * C / t / 1e9})
    if args.out:
        with open(args.out, "w") as f:
            for d in lines:
                f.write(json.dumps(d) + "\n")


if __name__ == "__main__":
    main()
