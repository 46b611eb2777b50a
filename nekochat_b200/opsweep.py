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

Single workloads for profiling one kernel with ncu (a few warm-up launches, then a few timed ones, CUDA-event
times printed):
    python -m nekochat_b200.opsweep --matmul FMT M K N [--reps R]
        neko_op_matmul on synthetic FP8 (1) / FP4 (2) weights N(0, 0.02) and activations N(0, 1): 2 warm-up
        calls, then R timed ones (default 3). Under ncu the first timed launch of the matmul kernel is the
        third (`-s 2 -c 1`).
    python -m nekochat_b200.opsweep --decode B [--steps S] [--context C] [--pos P]
        Qwen3-0.6B FP8 decode steps of B sequences at position P (default 512) through the native runner, with
        random weights and a zero KV cache (the same bytes are read as after a real prompt): 3 warm-up steps,
        then S timed ones (default 5). Prints ms per step and launches per step.
"""
import argparse
import json
import statistics
import time

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


def one_matmul(fmt, M, K, N, reps):
    import torch
    from . import ops
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn((N, K), generator=g, device="cuda").mul_(0.02)
    q = ops.quantize(fmt, w)
    del w
    x = torch.randn((M, K), generator=g, device="cuda")
    y = torch.empty((M, N), device="cuda")
    for _ in range(2):
        ops.matmul(fmt, x, q, K, y=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(reps):
        ops.matmul(fmt, x, q, K, y=y)
    e1.record()
    e1.synchronize()
    t1 = time.perf_counter()
    print(f"matmul fmt={fmt} M={M} K={K} N={N}: {e0.elapsed_time(e1) / reps * 1e3:.1f} us/call "
          f"(host {1e6 * (t1 - t0) / reps:.1f} us)", flush=True)


def one_decode(B, steps, context, pos):
    import torch
    from . import model as nmodel, workload
    s = workload.shape("qwen3-0.6b")
    m = nmodel.Model(s, 1, context=context, max_seqs=B, max_rows=64)
    m.load_random_device(seed=0)
    slots = np.arange(B, dtype=np.int32)
    m.stage(slots, np.arange(B, dtype=np.int32) + 7, np.full(B, pos, np.int32))
    st = torch.cuda.Stream()
    for k in range(3):
        m.step(B, pos + k, st.cuda_stream)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for k in range(steps):
        m.step(B, pos + 3 + k, st.cuda_stream)
    e1.record(st)
    e1.synchronize()
    print(f"decode B={B} pos={pos}: {e0.elapsed_time(e1) / steps:.3f} ms/step, "
          f"launches/step {m.step_launches(B)}", flush=True)
    m.close()


def main():
    import torch
    from . import ops
    from .ops import row_bytes

    ap = argparse.ArgumentParser(prog="python -m nekochat_b200.opsweep")
    ap.add_argument("--quick", action="store_true", help="M in {1, 64}, two matrix shapes, rows {1, 4096}")
    ap.add_argument("--reps", type=int, default=None, help="timed launches (sweep: 10, --matmul: 3)")
    ap.add_argument("--out", default=None)
    ap.add_argument("--matmul", type=int, nargs=4, metavar=("FMT", "M", "K", "N"),
                    help="one matmul shape only (2 warm-up calls, then --reps timed ones)")
    ap.add_argument("--decode", type=int, metavar="B", help="Qwen3-0.6B FP8 decode steps of B sequences only")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--context", type=int, default=768)
    ap.add_argument("--pos", type=int, default=512)
    args = ap.parse_args()
    if args.matmul:
        one_matmul(*args.matmul, reps=args.reps or 3)
        return
    if args.decode:
        if args.context <= args.pos + args.steps + 8:
            ap.error("context must exceed pos + steps + 8")
        one_decode(args.decode, args.steps, args.context, args.pos)
        return
    args.reps = args.reps or 10
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
