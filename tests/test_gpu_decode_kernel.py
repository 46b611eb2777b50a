"""The single-kernel decode step (k_decode.cu) against the per-operator kernel chain and the reference CPU forward.

Decode steps of 1..4 sequences run as one persistent kernel by default; neko_model_set_decode_kernel(0) switches
a model to the kernel chain. Both compute the same dot products in the same order; attention differs only in how
the keys are split (tolerance 1e-4). Parity with the reference is the model tolerance (max-abs 2e-2, rel 1e-2).
"""
import numpy as np
import pytest

import nekochat_b200 as nb
from nekochat_b200 import model as nmodel
from nekochat_b200 import workload
from oracle import models as omodels
from oracle.oracle import FP4, FP8, Restatement

pytestmark = pytest.mark.gpu

# GPT-2 with head_dim 64 like GPT-2 small (gpt2-tiny has 32, which the single kernel does not take)
GPT2_64 = dict(arch="gpt2", vocab=1000, embd=256, layers=2, heads=4, kv_heads=4, head_dim=64, ff=512, max_pos=256,
               eps=1e-5, rope_theta=0.0)


def shape_of(name):
    return dict(GPT2_64) if name == "gpt2-64" else workload.shape(name)


def pair(name, fmt, context, seqs, seed):
    s = shape_of(name)
    tensors = list(workload.weights(s, seed=seed, perturb=True))
    a = nmodel.Model(s, fmt, context=context, max_seqs=seqs, max_rows=32).load(tensors)
    b = nmodel.Model(s, fmt, context=context, max_seqs=seqs, max_rows=32).load(tensors)
    assert a.set_decode_kernel(True)
    b.set_decode_kernel(False)
    return s, tensors, a, b


def test_single_kernel_availability():
    m = nmodel.build("qwen3-tiny", FP8, context=64, max_seqs=4, max_rows=8)
    assert m.set_decode_kernel(True)
    n = nmodel.decode_kernel_launches(workload.shape("qwen3-tiny"), FP8)
    assert n == 2 and m.step_launches(1) == n and m.step_launches(4) == n
    m.set_decode_kernel(False)
    assert m.step_launches(1) > 10
    m.close()
    g = nmodel.build("gpt2-tiny", FP8, context=64, max_seqs=1, max_rows=8)  # head_dim 32: kernel chain only
    assert not g.set_decode_kernel(True)
    assert g.step_launches(1) > 1
    g.close()


@pytest.mark.parametrize("name,fmt", [("qwen3-tiny", FP8), ("qwen3-tiny", FP4), ("gpt2-64", FP8)])
@pytest.mark.parametrize("n", [1, 2, 4])
def test_single_kernel_matches_chain(name, fmt, n):
    """Same logits and greedy tokens as the kernel chain, over prompts long enough for several attention splits
    (ticket merge) and one short enough for a single split."""
    s, _, a, b = pair(name, fmt, context=256, seqs=4, seed=11 + n)
    lens = [7, 45, 130, 200][:n]
    toks = []
    for slot, L in enumerate(lens):
        p = workload.prompt(s, L, seed=30 + slot)
        la = a.prefill(p, slot)
        lb = b.prefill(p, slot)
        np.testing.assert_array_equal(la, lb)  # prefill is the same chain on both
        toks.append(int(np.argmax(la)))
    slots = np.arange(n, dtype=np.int32)
    pos = np.array(lens, np.int32)
    for step in range(6):
        la, ama = a.decode(slots, toks, pos + step)
        lb, amb = b.decode(slots, toks, pos + step)
        np.testing.assert_allclose(la, lb, rtol=1e-4, atol=1e-4)
        for i in range(n):
            if ama[i] != amb[i]:
                srt = np.sort(lb[i])
                assert srt[-1] - srt[-2] <= 2e-4, f"greedy token differs (step {step}, seq {i})"
        toks = list(ama)
    a.close()
    b.close()


@pytest.mark.parametrize("name,fmt", [("gpt2-64", FP8), ("qwen3-tiny", FP8)])
def test_single_kernel_vs_reference_teacher_forced(name, fmt):
    """Logit-level agreement with the reference CPU forward (restatement) for 12 greedy steps, teacher-forced."""
    R = Restatement()
    s = shape_of(name)
    tensors = list(workload.weights(s, seed=7, perturb=True))
    ref = omodels.make(s, tensors, fmt, 128, R)
    m = nmodel.Model(s, fmt, context=128, max_seqs=1, max_rows=64).load(tensors)
    assert m.set_decode_kernel(True)
    prompt = workload.prompt(s, 40, seed=8)
    want = ref.forward(prompt, 0)
    got = m.prefill(prompt, 0)
    assert np.abs(got - want).max() <= 2e-2
    tok, pos = int(np.argmax(want)), 40
    for _ in range(12):
        lg, am = m.decode([0], [tok], [pos])
        want = ref.forward(np.array([tok], np.int32), pos)
        d = np.abs(lg[0] - want)
        assert d.max() <= 2e-2 and np.all(d <= 1e-2 * np.abs(want) + 2e-3), f"max-abs {d.max()}"
        if int(am[0]) != int(np.argmax(want)):
            srt = np.sort(want)
            assert srt[-1] - srt[-2] <= 2 * d.max()
        tok, pos = int(np.argmax(want)), pos + 1
    m.close()


def test_single_kernel_wait_timeout_reports_and_recovers():
    """A wait that nothing satisfies gives up after its limit: the step reports a device error, and the next
    step runs normally (counters, tickets and keys were reset)."""
    s, _, a, b = pair("qwen3-tiny", FP8, context=128, seqs=1, seed=21)
    p = workload.prompt(s, 50, seed=22)
    tok = int(np.argmax(a.prefill(p, 0)))
    b.prefill(p, 0)
    a.set_decode_kernel(2)
    with pytest.raises(nb.NekoError, match="device error"):
        a.decode([0], [tok], [50])
    assert a.set_decode_kernel(True)
    la, ama = a.decode([0], [tok], [50])
    lb, amb = b.decode([0], [tok], [50])
    np.testing.assert_allclose(la, lb, rtol=1e-4, atol=1e-4)
    a.close()
    b.close()


def test_single_kernel_device_loop_matches_chain():
    """stage + step (greedy token and position advanced inside the kernel, graph replay) on both paths."""
    s, _, a, b = pair("qwen3-tiny", FP8, context=96, seqs=3, seed=23)
    n = 3
    toks = []
    for i in range(n):
        p = workload.prompt(s, 20 + 9 * i, seed=40 + i)
        toks.append(int(np.argmax(a.prefill(p, i))))
        b.prefill(p, i)
    slots = np.arange(n, dtype=np.int32)
    pos = np.array([20 + 9 * i for i in range(n)], np.int32)
    for m in (a, b):
        m.stage(slots, toks, pos)
        for k in range(12):
            m.step(n, int(pos.max()) + k)
    ta, pa = a.tokens(n)
    tb, pb = b.tokens(n)
    assert np.array_equal(pa, pos + 12) and np.array_equal(pb, pos + 12)
    assert np.array_equal(ta, tb)
    a.close()
    b.close()
