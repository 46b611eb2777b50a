"""Decode throughput of the B200 backend on the headline workload: Qwen3-0.6B shape, FP8 weights in the
engine's format, a 512-token random prompt, then greedy decode.

A step is one greedy decode step of every sequence on the GPU (batch 1 by default, --batch 64 for the batched
variant). One process per GPU; sequences are independent, so N GPUs run N replicas with the same per-GPU work
(weak scaling, no collective on the data path).

Printed line (rank 0): value = decode tok/s of the device-resident loop (tokens, positions and argmax stay in
HBM; one CUDA graph per step); e2e = the same through the engine-facing host API (neko_model_decode: host token
ids in, host logits out every step, like Model::forward); roofline = the dequant GEMV over every weight matrix of
one step, timed with CUDA events; cpu_baseline = the reference engine's CPU backend (compiled from its sources in
oracle/_ref) on this host's cores.

    python bench.py [--gpus N --steps K --warmup W --batch B --impl ours|reference --model M]

--model selects another benchmark configuration: gpt2-fp8 (GPT-2 small, FP8, 32-token prompt), qwen3-1.7b-fp4
(Qwen3-1.7B shape, the engine's FP4 weights, a 1024-token prompt), qwen3-4b-fp8 / qwen3-4b-fp4 (the per-GPU
batch of the data-parallel Qwen3-4B configuration: run with --batch 512); the default is the headline
configuration above.
"""
import argparse
import json
import os
import statistics
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# --model: the headline configuration and the other measured configurations
MODELS = {"qwen3-0.6b-fp8": ("qwen3-0.6b", 1, 512, "Qwen3-0.6B FP8 decode tok/s"),
          "gpt2-fp8": ("gpt2", 1, 32, "GPT-2 small FP8 decode tok/s"),
          "qwen3-1.7b-fp4": ("qwen3-1.7b", 2, 1024, "Qwen3-1.7B FP4 decode tok/s"),
          # the data-parallel Qwen3-4B configuration: 512 sequences of a 256-token prompt + 128 steps per GPU
          "qwen3-4b-fp8": ("qwen3-4b", 1, 256, "Qwen3-4B FP8 decode tok/s"),
          "qwen3-4b-fp4": ("qwen3-4b", 2, 256, "Qwen3-4B FP4 decode tok/s")}
SHAPE, FMT, PROMPT, METRIC = MODELS["qwen3-0.6b-fp8"]
FMT_NAME = {1: "FP8", 2: "FP4"}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--model", choices=sorted(MODELS), default="qwen3-0.6b-fp8",
                   help="qwen3-0.6b-fp8 (512-token prompt, the headline), gpt2-fp8 (32-token prompt), "
                        "qwen3-1.7b-fp4 (1024-token prompt), "
                        "qwen3-4b-fp8 / qwen3-4b-fp4 (256-token prompt; measured at --batch 512 "
                        "--steps 128)")
    p.add_argument("--prompt", type=int, default=None,
                   help="prompt tokens (default: the model's, 512 / 1024 / 256; 32 with --profile)")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--profile", action="store_true", help="small case for ncu: short prompt, few steps, no extras")
    return p.parse_args()


# ---------------------------------------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """Samples SM clock and throttle reasons every few ms on a thread while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index):
        self.samples, self.reasons, self.stop_ev = [], set(), threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self.stop_ev.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop_ev.set()
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------- helpers
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s for a kernel timed inside a long step: MEASURED_PEAKS.json's sustained figure, else the
    profiling recipe's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (bf16_tflops_sustained)"
    except Exception:
        return 1400.0, "fallback (sustained figure of the profiling recipe)"


def matmul_macs_per_token(s):
    """Multiply-adds of one token's matmuls (every layer matrix and the LM head; attention excluded)."""
    C, L, V = s["embd"], s["layers"], s["vocab"]
    if s["arch"] == "qwen3":
        H, KV, hd, F = s["heads"], s["kv_heads"], s["head_dim"], s["ff"]
        per = (H + 2 * KV) * hd * C + C * H * hd + 2 * F * C + C * F
    else:
        F = s["ff"]
        per = 3 * C * C + C * C + 2 * F * C
    return L * per + V * C


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def prompt_seed(rank, i):
    """The seed of sequence i's prompt on a rank: replicas decode disjoint sequences (i < 100000)."""
    return 1 + rank * 100000 + i


def reduce_max(x, world):
    """The largest x over the ranks (the job's time is its slowest rank's); on the GPU under NCCL, on the host
    under gloo."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if "nccl" in str(dist.get_backend()) else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def gemv_roofline(model, s, stream, reps=3):
    """Every packed weight matrix of one decode step (28 layers x {qkv, o, gate|up, down} + LM head, 633 MB for
    FP8 at 0.6B: far above the 126 MB L2, so each launch streams from HBM) through the GEMV kernel at M = 1,
    launched back to back with programmatic dependent launch as in the step. Returns (algorithmic bytes per
    launch, mean launch time in s, launches)."""
    import torch
    from nekochat_b200 import ops, workload
    mats = []
    for l in range(s["layers"]):
        for w in ("wqkv", "wo", "wgu", "wdown"):
            mats.append(model.matrix(f"layers.{l}.{w}"))
    mats.append(model.matrix("head"))
    kmax = max(c for _, _, c, _ in mats)
    nmax = max(r for _, r, _, _ in mats)
    x = torch.randn(kmax, device="cuda")
    y = torch.empty(nmax, device="cuda")
    lib = __import__("nekochat_b200").lib()
    import ctypes as C
    nbytes = 0
    for p, r, c, f in mats:
        nbytes += r * workload.row_bytes(f, c) + c * 4 + r * 4
    def run():
        for p, r, c, f in mats:
            rc = lib.neko_op_matmul(f, C.c_void_p(x.data_ptr()), 1, c, C.c_void_p(p), r, None,
                                    C.c_void_p(y.data_ptr()), r, 0, 256, C.c_void_p(stream.cuda_stream))
            if rc:
                raise RuntimeError(lib.neko_last_error().decode())
    # the chain is captured once as a CUDA graph so host launch overhead does not enter the timing
    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        capture = torch.cuda.current_stream()
        for p, r, c, f in mats:
            rc = lib.neko_op_matmul(f, C.c_void_p(x.data_ptr()), 1, c, C.c_void_p(p), r, None,
                                    C.c_void_p(y.data_ptr()), r, 0, 256, C.c_void_p(capture.cuda_stream))
            if rc:
                raise RuntimeError(lib.neko_last_error().decode())
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / (reps * len(mats))
    del graph
    # the LM head alone (the step's largest matrix), 20 launches back to back in one graph
    p, r, c, f = mats[-1]
    hgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(hgraph, stream=stream):
        capture = torch.cuda.current_stream()
        for _ in range(20):
            rc = lib.neko_op_matmul(f, C.c_void_p(x.data_ptr()), 1, c, C.c_void_p(p), r, None,
                                    C.c_void_p(y.data_ptr()), r, 0, 256, C.c_void_p(capture.cuda_stream))
            if rc:
                raise RuntimeError(lib.neko_last_error().decode())
    hgraph.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        hgraph.replay()
        e1.record(stream)
    e1.synchronize()
    t_head = e0.elapsed_time(e1) / 1e3 / 20
    del hgraph
    head_bytes = r * workload.row_bytes(f, c) + c * 4 + r * 4
    return nbytes / len(mats), t, reps * len(mats), head_bytes, t_head


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            return next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), "unknown")
    except OSError:
        return "unknown"


def reference_decode(s, h16, tmpdir, prompt_len, warm, steps, budget_s=20.0):
    """The reference engine's CPU backend on this host, on the GPU arm's workload: loadModel (CPU backend, the
    timing build for this host's ISA level, all host threads up to the engine's pool cap of 16) of an f16
    checkpoint of `h16`, the same `prompt_len`-token prompt fed in chunks of 64 (Model::kMaxBatch, as
    Engine::generate feeds it), `warm` untimed greedy steps, then greedy steps at the GPU arm's positions,
    timed until `steps` are done or `budget_s` has passed (a bounded sample; at least 2 steps). Returns
    (tok/s, timed steps, description)."""
    from nekochat_b200 import workload
    from oracle.checkpoint import write_model
    from oracle.oracle import Reference, native_build
    ref = Reference(native=True)
    folder = write_model(os.path.join(tmpdir, "ckpt"), s, h16, dtype=np.float16)
    threads = min(16, os.cpu_count() or 1)
    m = ref.load_model(folder, FMT, threads=threads)
    toks = workload.prompt(s, prompt_len)
    for i in range(0, prompt_len, 64):
        logits = m.forward(toks[i:i + 64], i)
    tok, pos = int(np.argmax(logits)), prompt_len
    for _ in range(warm):
        logits = m.forward(np.array([tok], np.int32), pos)
        tok, pos = int(np.argmax(logits)), pos + 1
    p0 = pos
    k = 0
    t0 = time.perf_counter()
    while k < steps and (k < 2 or time.perf_counter() - t0 < budget_s):
        logits = m.forward(np.array([tok], np.int32), pos)
        tok, pos = int(np.argmax(logits)), pos + 1
        k += 1
    dt = time.perf_counter() - t0
    m.close()
    build = native_build()[1]
    desc = (f"reference CPU engine (oracle/_ref/{ref.build}: {build}; x86 portable matmulGeneric path) on "
            f"{threads} threads of '{cpu_model()}' ({os.cpu_count()} logical CPUs), batch 1, the GPU arm's "
            f"{prompt_len}-token prompt prefilled in chunks of 64, {warm} warm-up steps, then {k} timed greedy "
            f"decode steps at positions {p0}..{pos - 1} (a bounded sample of {budget_s:.0f} s at most of the "
            f"{steps}-step run); the engine runs sequences one at a time, so this is also its aggregate rate")
    return k / dt, k, threads, desc


def random_h16(s, seed=0):
    """N(0, 0.02) f16 weights from torch's seeded CPU generator (numpy's is ~10x slower here), gains 1, biases 0."""
    import torch
    from nekochat_b200 import workload
    g = torch.Generator().manual_seed(seed)
    out = []
    for name, shp, kind in workload.tensor_specs(s):
        if kind == "w":
            a = (torch.randn(shp, generator=g) * 0.02).half().numpy()
        else:
            a = (np.ones if kind == "g" else np.zeros)(shp, np.float16)
        out.append((name, a))
    return out


# ---------------------------------------------------------------------------------------------- reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from nekochat_b200 import workload
    s = workload.shape(SHAPE)
    prompt_len = args.prompt or PROMPT
    with tempfile.TemporaryDirectory() as tmp:
        v, k, threads, sample = reference_decode(s, random_h16(s), tmp, prompt_len, args.warmup, args.steps)
    B = args.batch
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": k,
        "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{SHAPE} {FMT_NAME[FMT].lower()} (engine {FMT_NAME[FMT]} format), {prompt_len}-token "
                               f"random prompt, greedy decode, batch {B} per GPU", "batch": B, "prompt": prompt_len,
                   "positions": [prompt_len + args.warmup, prompt_len + args.warmup + k]},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    from nekochat_b200 import model as nmodel, workload
    world, rank, local = dist_setup(args)
    s = workload.shape(SHAPE)
    B = args.batch
    prompt_len = args.prompt or (32 if args.profile else PROMPT)
    steps, warm = (4, 3) if args.profile else (args.steps, args.warmup)
    e2e_on = not (args.no_e2e or args.profile)
    context = prompt_len + 2 * (warm + steps) + 8
    context = (context + 255) // 256 * 256
    cpu_on = (rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile
              and os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libneko_ref.so")))
    cpu = None
    if cpu_on:
        # First, before the GPU work starts threads of its own on this host: the same routine, weights
        # generator, prompt and positions as --impl reference, so the two CPU figures measure the same thing.
        with tempfile.TemporaryDirectory() as tmp:
            try:
                v, k, threads, sample = reference_decode(s, random_h16(s), tmp, prompt_len, warm, steps)
                cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample}
            except Exception as e:  # the baseline is reported, never required
                cpu = {"value": None, "unit": "tok/s", "error": str(e)[:200]}
    m = nmodel.Model(s, FMT, context=context, max_seqs=B, max_rows=max(64, B), device=local)
    m.load_random_device(seed=0)

    # prefill every sequence (different prompts per rank and sequence)
    first = np.zeros(B, np.int32)
    for i in range(B):
        p = workload.prompt(s, prompt_len, seed=prompt_seed(rank, i))
        first[i] = int(np.argmax(m.prefill(p, slot=i)))
    slots = np.arange(B, dtype=np.int32)
    pos = np.full(B, prompt_len, np.int32)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream()
    m.stage(slots, first, pos)
    for k in range(warm):
        m.step(B, prompt_len + k, stream.cuda_stream)
    stream.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for k in range(steps):
            m.step(B, prompt_len + warm + k, stream.cuda_stream)
        e1.record(stream)
        e1.synchronize()
    barrier(world)
    t = reduce_max(e0.elapsed_time(e1) / 1e3, world)
    value = world * B * steps / t
    launches = m.step_launches(B) * steps

    # end to end through the host API (host token ids in, host logits out, every step)
    e2e = None
    if e2e_on:
        # the same positions (and so the same greedy chain) as the device-resident leg: restart at the prompt's end
        m.tokens(B)
        toks, p0 = first.copy(), pos.copy()
        h2d = B * 3 * 4
        d2h = B * s["vocab"] * 4 + B * 4
        tok = toks.copy()
        lg_host = m.host_logits(B)  # one (pinned) host logits buffer, reused like the engine's
        for k in range(warm):
            _, tok = m.decode(slots, tok, p0 + k, out=lg_host)
        barrier(world)
        t0 = time.perf_counter()
        for k in range(steps):
            lg, tok = m.decode(slots, tok, p0 + warm + k, out=lg_host)
        t_e2e = reduce_max(time.perf_counter() - t0, world)
        e2e = {"value": world * B * steps / t_e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h,
               "positions": "the device-resident leg's (the same greedy chain from the prompt's end)",
               "path": "neko_model_decode: pinned-staged H2D of token/slot/position (one copy), CUDA graph step, "
                       "D2H of the full logits into one reused pinned host buffer and the greedy token, host "
                       "synchronisation, every step"}

    roof = None
    if rank == 0 and not args.profile:
        peak, src = peaks()
        psrc = f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else \
            "fallback (MEASURED_PEAKS.json absent: the profiling recipe's 6650 GB/s)"
        # algorithmic bytes of one step: every weight byte once, each sequence's KV cache up to its position
        # (mean over the timed steps), the activations are a few KB
        mean_pos = prompt_len + warm + (steps - 1) / 2
        bytes_step = workload.weight_stream_bytes(s, FMT) + B * workload.kv_bytes_per_position(s) * (mean_pos + 1)
        nl = nmodel.decode_kernel_launches(s, FMT)
        single = m.step_launches(B) == nl
        ach = bytes_step / (t / steps) / 1e9
        dk = f"decode_kernel<{FMT_NAME[FMT]},{1 if B == 1 else 4}>"
        roof = {"bound": "hbm",
                "kernel": (f"{dk} (a whole decode step, one launch)" if nl == 1 else
                           f"{dk} (every layer, one launch) + gemv_fp8_tc_kernel (final norm, LM head, greedy argmax "
                           "and token / position finalize): the step's two launches, timed together")
                if single else "decode step as a kernel chain (tc_gemm_kernel and attention_tc_kernel dominant)",
                "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "peak_source": psrc, "traffic": None, "bytes_per_launch": bytes_step if single and nl == 1 else None,
                "bytes_per_step": bytes_step, "launch_us": t / steps * 1e6 if single and nl == 1 else None,
                "step_us": t / steps * 1e6,
                "timing": "CUDA events on the launch stream around the timed steps (graph replays back to back)"}
        if B >= 128:  # layer matmuls and LM head on tcgen05 (128+ rows): the step is bound by the tensor pipe
            tpk, tsrc = tensor_peak()
            tfl = 2 * matmul_macs_per_token(s) * B / (t / steps) / 1e12
            roof.update({"bound": "tensor", "kernel": "decode step as a kernel chain (umma_gemm_kernel dominant)",
                         "achieved": round(tfl, 1), "peak": tpk, "unit": "TFLOP/s", "frac": round(tfl / tpk, 4),
                         "peak_source": tsrc, "hbm_achieved_gbs": round(ach, 1),
                         "flops_note": "2 x (layer + LM-head weights) x batch per step, useful FLOPs; the kernels "
                                       "issue 3 f16 MMAs per product (hi / lo split operands)"})
        tf = os.path.join(ROOT, "profiles", "traffic.json")
        key = f"decode_{FMT_NAME[FMT].lower()}_b{B}" + ("" if SHAPE == "qwen3-0.6b" else "_" + SHAPE)
        if single and os.path.exists(tf):
            try:
                rec = json.load(open(tf)).get(key)
                if rec:  # ncu DRAM bytes of one launch, scaled from the captured position to this run's mean
                    roof["traffic"] = round(rec["dram_bytes"] * bytes_step / rec["algorithmic_bytes"])
                    what = rec.get("launches", "one launch")
                    roof["traffic_note"] = (f"ncu dram__bytes_read+write of {what} at position {rec['position']} "
                                            f"({rec['dram_bytes']} B vs {rec['algorithmic_bytes']} B algorithmic), "
                                            "scaled by the algorithmic bytes to the mean timed position")
            except Exception:
                pass
        # the same weight matrices as single GEMV launches (the operator the step is built from), for reference
        per_launch, t_launch, n, head_bytes, t_head = gemv_roofline(m, s, stream)
        gk = "gemv_fp8_tc_kernel" if FMT == 1 else f"gemv_stream_kernel<{FMT_NAME[FMT]},1>"
        roof["gemv_op"] = {"kernel": f"{gk} (M=1, every weight matrix of a step, one launch each, CUDA graph with "
                                     "programmatic dependent launch)",
                           "achieved": round(per_launch / t_launch / 1e9, 1), "bytes_per_launch": per_launch,
                           "launch_us": t_launch * 1e6, "frac": round(per_launch / t_launch / 1e9 / peak, 4),
                           "lm_head": {"achieved": round(head_bytes / t_head / 1e9, 1), "bytes_per_launch": head_bytes,
                                       "launch_us": t_head * 1e6,
                                       "frac": round(head_bytes / t_head / 1e9 / peak, 4),
                                       "timing": "20 launches back to back in one CUDA graph (the head is above L2)"}}

    m.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": t / steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{SHAPE} {FMT_NAME[FMT].lower()} (engine {FMT_NAME[FMT]} format), {prompt_len}-token "
                                   f"random prompt, greedy decode, batch {B} per GPU", "batch": B, "prompt": prompt_len,
                       "positions": [prompt_len + warm, prompt_len + warm + steps],
                       "weights": f"N(0,0.02) random init, quantized on the GPU by the engine's {FMT_NAME[FMT]} codec",
                       "l2": f"no flush needed: each step streams "
                             f"{workload.weight_stream_bytes(s, FMT) / 1e6:.0f} MB of weights (> 126 MB L2)",
                       "parallelism": f"dp{world} (independent replicas)"},
            "gpu_launches": launches,
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    global SHAPE, FMT, PROMPT, METRIC
    args = parse()
    SHAPE, FMT, PROMPT, METRIC = MODELS[args.model]
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
