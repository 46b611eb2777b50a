"""Small, repeatable workloads for profiling single kernels with ncu (each runs a few warm-up launches, then a
few timed ones, and prints CUDA-event times).

    python -m nekochat_b200.probe matmul FMT M K N [--reps R]
        neko_op_matmul on synthetic FP8 (1) / FP4 (2) weights N(0, 0.02) and activations N(0, 1): 2 warm-up
        calls, then R timed ones (default 3). Under ncu the first timed launch of the matmul kernel is the
        third (`-s 2 -c 1`).
    python -m nekochat_b200.probe decode B [--steps S] [--context C] [--pos P]
        Qwen3-0.6B FP8 decode steps of B sequences at position P (default 512) through the native runner, with
        random weights and a zero KV cache (the same bytes are read as after a real prompt): 3 warm-up steps,
        then S timed ones (default 5). Prints ms per step and launches per step.
"""
import argparse
import sys
import time


def matmul(args):
    import torch
    from . import ops
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn((args.N, args.K), generator=g, device="cuda").mul_(0.02)
    q = ops.quantize(args.fmt, w)
    del w
    x = torch.randn((args.M, args.K), generator=g, device="cuda")
    y = torch.empty((args.M, args.N), device="cuda")
    for _ in range(2):
        ops.matmul(args.fmt, x, q, args.K, y=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(args.reps):
        ops.matmul(args.fmt, x, q, args.K, y=y)
    e1.record()
    e1.synchronize()
    t1 = time.perf_counter()
    print(f"matmul fmt={args.fmt} M={args.M} K={args.K} N={args.N}: {e0.elapsed_time(e1) / args.reps * 1e3:.1f} "
          f"us/call (host {1e6 * (t1 - t0) / args.reps:.1f} us)", flush=True)


def decode(args):
    import numpy as np
    import torch
    from . import model as nmodel, workload
    s = workload.shape("qwen3-0.6b")
    m = nmodel.Model(s, 1, context=args.context, max_seqs=args.B, max_rows=64)
    m.load_random_device(seed=0)
    slots = np.arange(args.B, dtype=np.int32)
    pos = np.full(args.B, args.pos, np.int32)
    m.stage(slots, np.arange(args.B, dtype=np.int32) + 7, pos)
    st = torch.cuda.Stream()
    for k in range(3):
        m.step(args.B, args.pos + k, st.cuda_stream)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for k in range(args.steps):
        m.step(args.B, args.pos + 3 + k, st.cuda_stream)
    e1.record(st)
    e1.synchronize()
    print(f"decode B={args.B} pos={args.pos}: {e0.elapsed_time(e1) / args.steps:.3f} ms/step, "
          f"launches/step {m.step_launches(args.B)}", flush=True)
    m.close()


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m nekochat_b200.probe")
    sub = ap.add_subparsers(dest="what", required=True)
    a = sub.add_parser("matmul")
    a.add_argument("fmt", type=int)
    a.add_argument("M", type=int)
    a.add_argument("K", type=int)
    a.add_argument("N", type=int)
    a.add_argument("--reps", type=int, default=3)
    d = sub.add_parser("decode")
    d.add_argument("B", type=int)
    d.add_argument("--steps", type=int, default=5)
    d.add_argument("--context", type=int, default=768)
    d.add_argument("--pos", type=int, default=512)
    args = ap.parse_args(argv)
    if args.what == "decode" and args.context <= args.pos + args.steps + 8:
        ap.error("context must exceed pos + steps + 8")
    (matmul if args.what == "matmul" else decode)(args)


if __name__ == "__main__":
    main(sys.argv[1:])
