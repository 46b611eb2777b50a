"""The reference engine itself, unchanged, on the B200 backend: the drop-in path.

``oracle/_ref/libneko_ref_cuda.so`` is the reference's own engine (model loading, Qwen3Model / Gpt2Model, the
sampler) compiled from its sources, with the B200 backend (``nekochat_b200/csrc/cuda_compute.cpp`` over
``libneko_cuda.so``) in the first GPU slot that ``Model::startGpu`` tries (shared/cpp/model.cpp:137-173). So
``loadModel(..., backend=Auto)`` runs the engine's own compatibility check, its ``gpu::selfTest``, its GPU
loader and every ``forwardGpu`` dispatch (qwen3/cpp/qwen3_model.cpp:278-341, gpt2/cpp/gpt2_model.cpp:220-278)
on CUDA. Its logits are compared with the same engine's CPU backend (``backend=CPU``, forwardCpu) reading the
same checkpoint, at the engine's GPU-vs-CPU tolerance (max-abs 2e-2, rel 1e-2 + 2e-3), with the greedy tokens
teacher-forced from the CPU side and checked margin-aware.
"""
import os
import tempfile
import time

import numpy as np
import pytest

from nekochat_b200 import workload
from oracle.checkpoint import write_model
from oracle.oracle import FP4, FP8, Reference

pytestmark = pytest.mark.gpu
LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "libneko_ref_cuda.so")
THREADS = min(16, os.cpu_count() or 1)
AUTO, CPU = 0, 3


def close(got, want, what):
    d = np.abs(got - want)
    assert d.max() <= 2e-2, f"{what}: max-abs {d.max():.3g}"
    assert np.all(d <= 1e-2 * np.abs(want) + 2e-3), f"{what}: rel error {d.max():.3g}"
    return float(d.max())


def engines(s, fmt, seed, tmp):
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libneko_ref_cuda.so not built")
    folder = write_model(os.path.join(tmp, "ckpt"), s, workload.weights(s, seed=seed, perturb=True),
                         dtype=np.float16)
    ref = Reference(cuda=True)
    gpu = ref.load_model(folder, fmt, threads=THREADS, backend=AUTO)
    cpu = ref.load_model(folder, fmt, threads=THREADS, backend=CPU)
    return gpu, cpu


@pytest.mark.parametrize("name,fmt", [("qwen3-tiny", FP8), ("qwen3-tiny", FP4), ("gpt2-tiny", FP8),
                                      ("qwen3-0.6b", FP8), ("gpt2", FP8)])
def test_engine_forward_gpu_matches_forward_cpu(name, fmt):
    """loadModel(Auto) picks the CUDA backend; a prompt in the engine's 64-token chunks, then 16 greedy steps
    through forwardGpu, match forwardCpu. Prints the per-token time of the engine's own dispatch path."""
    s = workload.shape(name)
    with tempfile.TemporaryDirectory() as tmp:
        gpu, cpu = engines(s, fmt, seed=17, tmp=tmp)
        try:
            assert gpu.backend().split("\n")[0] == "CUDA", gpu.backend()
            assert cpu.backend().split("\n")[0] == "CPU"
            prompt = workload.prompt(s, 40, seed=18)
            want = cpu.forward(prompt, 0)
            got = gpu.forward(prompt, 0)
            close(got, want, f"{name} prompt")
            pos, steps, t_gpu = len(prompt), 16, 0.0
            for k in range(steps):
                tok = int(np.argmax(want))
                want = cpu.forward(np.array([tok], np.int32), pos)
                t0 = time.perf_counter()
                got = gpu.forward(np.array([tok], np.int32), pos)
                t_gpu += time.perf_counter() - t0
                err = close(got, want, f"{name} step {k}")
                if int(np.argmax(got)) != int(np.argmax(want)):
                    srt = np.sort(want)
                    assert srt[-1] - srt[-2] <= 2 * err, f"{name} step {k}: greedy token differs"
                pos += 1
            print(f"\n[drop-in] {name} fmt {fmt}: engine forwardGpu on CUDA {1e3 * t_gpu / steps:.2f} ms/token "
                  f"(host logits download included)")
        finally:
            gpu.close()
            cpu.close()
