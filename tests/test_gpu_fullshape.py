"""Model-level parity at the benchmarked models' own shapes, against the reference engine compiled from its sources.

The benchmarked kernels run here at the shapes they are timed on:
* Qwen3-0.6B FP8 (the headline configuration) at batch 1 and 4 -- the persistent ``decode_kernel`` (head_dim 128, GQA
  group 2, 148-CTA row partition of the 151,936-row LM head, split-KV attention with the ticket merge once the
  position passes 64) -- and at batch 64 (the tensor-core kernel chain of the batched line);
* Qwen3-1.7B FP4 at batch 1 and 32;
* GPT-2 small FP8: 32-token prompt, 128 greedy steps;
* the Qwen3-4B layer shapes (C 2560, 32 Q / 8 KV heads, F 9728) at 512 sequences, the tcgen05 path,
  with 4 of its 36 layers so the CPU side stays within seconds (every matrix shape is the full model's).

The checker is ``oracle/_ref/libneko_ref.so``: the reference's own C++ engine (``loadModel`` with the CPU backend,
``Model::forward``, qwen3_model.cpp:232-276 / gpt2_model.cpp:179-218, cpu_ops.cpp:442-575) reading an f16
safetensors checkpoint of exactly the weights the runner was given. Weights are N(0, 0.02) from a seeded
generator (norm gains 1, biases 0), rounded through f16 on both sides.

Tolerance (the engine's GPU-vs-CPU bound): every logit within max-abs 2e-2 and within rel 1e-2 (+2e-3 absolute for
logits near zero) of the reference, and the same greedy token at every step. Steps are teacher-forced with the
reference's own greedy tokens; a greedy mismatch only counts when the reference's top-1 / top-2 margin exceeds
twice the observed logit error (random-init weights produce near-ties).
"""
import os
import tempfile

import numpy as np
import pytest

from nekochat_b200 import model as nmodel
from nekochat_b200 import workload
from oracle.checkpoint import write_model
from oracle.oracle import FP4, FP8, Reference

pytestmark = pytest.mark.gpu
REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libneko_ref.so")
THREADS = min(16, os.cpu_count() or 1)


def check_logits(got, want, what):
    d = np.abs(got - want)
    assert d.max() <= 2e-2, f"{what}: max-abs {d.max():.3g}"
    bad = d > 1e-2 * np.abs(want) + 2e-3
    assert not bad.any(), f"{what}: rel error at logit {int(np.argmax(bad))} ({d[np.argmax(bad)]:.3g})"
    return float(d.max())


def check_greedy(got_tok, want_logits, err, what):
    want_tok = int(np.argmax(want_logits))
    if int(got_tok) != want_tok:
        s = np.sort(want_logits)
        assert s[-1] - s[-2] <= 2 * err, f"{what}: greedy token {got_tok} != {want_tok} (margin {s[-1] - s[-2]:.3g})"


class Pair:
    """The B200 runner and the reference CPU engine holding the same f16-exact random weights."""

    def __init__(self, s, fmt, context, max_seqs, max_rows, seed=0):
        if not os.path.exists(REF_LIB):
            pytest.skip("oracle/_ref/libneko_ref.so not built")
        self.s = s
        h16 = []
        self.m = nmodel.Model(s, fmt, context=context, max_seqs=max_seqs, max_rows=max_rows)
        self.m.load_random_device(seed=seed, host_copy=lambda n, a: h16.append((n, a)), f16_exact=True)
        self.tmp = tempfile.TemporaryDirectory()
        folder = write_model(os.path.join(self.tmp.name, "ckpt"), s, h16, dtype=np.float16)
        del h16
        self.ref = Reference().load_model(folder, fmt, threads=THREADS)
        self.tmp.cleanup()

    def record(self, prompt, steps):
        """The reference's prompt logits and `steps` greedy steps: (tokens fed at each step, logits [steps+1][V]).
        The prompt goes in chunks of at most 64 tokens, Model::kMaxBatch (model.h:66), as Engine::generate feeds
        it (engine.cpp:98-112)."""
        for i in range(0, len(prompt), 64):
            lg = self.ref.forward(prompt[i:i + 64], i)
        want = [lg]
        toks, pos = [], len(prompt)
        for _ in range(steps):
            toks.append(int(np.argmax(want[-1])))
            want.append(self.ref.forward(np.array([toks[-1]], np.int32), pos))
            pos += 1
        return toks, want

    def close(self):
        self.m.close()
        self.ref.close()


def run_batch(pair, prompts, steps, checked, what):
    """Prefills every slot, then `steps` batched decode steps. Slots in `checked` are fed the reference's greedy
    tokens and compared with it at every step; the others are fed seeded random tokens."""
    s, m = pair.s, pair.m
    n = len(prompts)
    rec = {i: pair.record(prompts[i], steps) for i in checked}
    rng = np.random.default_rng(99)
    feed = np.zeros((steps, n), np.int32)
    for i in range(n):
        if i in rec:
            feed[:, i] = rec[i][0]
        else:
            feed[:, i] = rng.integers(0, s["vocab"], steps)
    for i, p in enumerate(prompts):
        got = m.prefill(p, slot=i)
        if i in rec:
            check_logits(got, rec[i][1][0], f"{what} slot {i} prompt")
    slots = np.arange(n, dtype=np.int32)
    pos = np.array([len(p) for p in prompts], np.int32)
    worst = 0.0
    for k in range(steps):
        lg, am = m.decode(slots, feed[k], pos + k)
        for i in rec:
            want = rec[i][1][k + 1]
            err = check_logits(lg[i], want, f"{what} slot {i} step {k}")
            check_greedy(am[i], want, err, f"{what} slot {i} step {k}")
            worst = max(worst, err)
    return worst


# ---------------------------------------------------------------------------------------------- Qwen3-0.6B FP8
@pytest.fixture(scope="module")
def q06():
    p = Pair(workload.shape("qwen3-0.6b"), FP8, context=256, max_seqs=64, max_rows=64)
    yield p
    p.close()


def test_qwen3_06b_fp8_b1_decode_kernel(q06):
    """Qwen3-0.6B FP8 at batch 1: a 120-token prompt, then 32 greedy steps on the persistent decode kernel, whose
    attention crosses from 2 to 3 key splits at position 128 (the ticket merge)."""
    assert q06.m.set_decode_kernel(True) and q06.m.step_launches(1) == nmodel.decode_kernel_launches(q06.s, FP8) == 2
    prompt = workload.prompt(q06.s, 120, seed=1)
    run_batch(q06, [prompt], 32, [0], "qwen3-0.6b fp8 b1")


def test_qwen3_06b_fp8_b4_decode_kernel(q06):
    """Four sequences in one decode_kernel<FP8, 4> launch, at different positions (1, 2 and 3 key splits)."""
    assert q06.m.step_launches(4) == 2
    prompts = [workload.prompt(q06.s, n, seed=10 + i) for i, n in enumerate((40, 70, 100, 150))]
    run_batch(q06, prompts, 12, [0, 3], "qwen3-0.6b fp8 b4")


def test_qwen3_06b_fp8_b64_chain(q06):
    """Qwen3-0.6B FP8 at batch 64: the batched kernel chain (tensor-core matmuls, fused decode attention)."""
    assert q06.m.step_launches(64) > 1
    rng = np.random.default_rng(5)
    prompts = [workload.prompt(q06.s, int(n), seed=200 + i) for i, n in enumerate(rng.integers(8, 130, 64))]
    run_batch(q06, prompts, 10, [3, 40], "qwen3-0.6b fp8 b64")


# ---------------------------------------------------------------------------------------------- Qwen3-1.7B FP4
@pytest.fixture(scope="module")
def q17():
    p = Pair(workload.shape("qwen3-1.7b"), FP4, context=192, max_seqs=32, max_rows=64)
    yield p
    p.close()


def test_qwen3_17b_fp4_b1_decode_kernel(q17):
    """Qwen3-1.7B FP4 at batch 1 (FP4 nibbles + f16 block scales, C 2048, F 6144): 70-token prompt, 32 steps."""
    assert q17.m.set_decode_kernel(True) and q17.m.step_launches(1) == nmodel.decode_kernel_launches(q17.s, FP4) == 1
    prompt = workload.prompt(q17.s, 70, seed=1)
    run_batch(q17, [prompt], 32, [0], "qwen3-1.7b fp4 b1")


def test_qwen3_17b_fp4_b32_chain(q17):
    """Qwen3-1.7B FP4 at batch 32."""
    rng = np.random.default_rng(6)
    prompts = [workload.prompt(q17.s, int(n), seed=300 + i) for i, n in enumerate(rng.integers(8, 90, 32))]
    run_batch(q17, prompts, 6, [7], "qwen3-1.7b fp4 b32")


# ---------------------------------------------------------------------------------------------- GPT-2 small FP8
def test_gpt2_small_fp8_128_steps():
    """The CPU-runnable configuration exactly: GPT-2 small, FP8, 32-token prompt, 128 greedy steps (decode kernel, head_dim 64)."""
    p = Pair(workload.shape("gpt2"), FP8, context=256, max_seqs=1, max_rows=64)
    try:
        assert p.m.set_decode_kernel(True) and p.m.step_launches(1) == nmodel.decode_kernel_launches(p.s, FP8) == 2
        prompt = workload.prompt(p.s, 32, seed=1)
        run_batch(p, [prompt], 128, [0], "gpt2 small fp8")
    finally:
        p.close()


# ---------------------------------------------------------------------------------------------- Qwen3-4B shapes
@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_qwen3_4b_shapes_512_sequences(fmt):
    """The data-parallel Qwen3-4B configuration's per-GPU batch: 512 sequences in one step (tcgen05 matmuls at 512 rows), on 4 layers of the
    Qwen3-4B shape (every matrix at its full size; 4 layers keep the CPU reference to seconds per token)."""
    s = workload.shape("qwen3-4b")
    s["layers"] = 4
    p = Pair(s, fmt, context=96, max_seqs=512, max_rows=512)
    try:
        rng = np.random.default_rng(7)
        prompts = [workload.prompt(s, int(n), seed=400 + i) for i, n in enumerate(rng.integers(4, 60, 512))]
        run_batch(p, prompts, 4, [0, 511], f"qwen3-4b x4 layers {'fp8' if fmt == FP8 else 'fp4'} b512")
    finally:
        p.close()
