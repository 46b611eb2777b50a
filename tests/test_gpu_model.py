"""Model-level parity of the native runner (neko_model_*) with the reference CPU forward.

Tolerance (the engine's GPU-vs-CPU bound): logits within max-abs 2e-2 and rel 1e-2 of the reference CPU backend on the
same seeded inputs, and identical greedy tokens. Greedy identity is checked teacher-forced: both sides are fed
the reference's token, and a step only counts as a mismatch when the reference's top-1/top-2 margin exceeds the
observed logit error (random-init weights give near-ties; ties are reported, not counted).
"""
import os

import numpy as np
import pytest

import nekochat_b200 as nb
from nekochat_b200 import workload
from nekochat_b200 import model as nmodel
from oracle import models as omodels
from oracle.oracle import FP4, FP8, Restatement

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def logits_close(got, want):
    d = np.abs(got - want)
    assert d.max() <= 2e-2, f"max-abs {d.max()}"
    assert np.all(d <= 1e-2 * np.abs(want) + 2e-3), f"rel error at {np.argmax(d - 1e-2 * np.abs(want))}"
    return d.max()


def margin(l):
    s = np.sort(l)
    return s[-1] - s[-2]


@pytest.mark.parametrize("tag,name,fmt", [("qwen3_fp8", "qwen3-tiny", FP8), ("qwen3_fp4", "qwen3-tiny", FP4),
                                          ("gpt2_fp8", "gpt2-tiny", FP8)])
def test_tiny_models_vs_reference_golden(tag, name, fmt):
    """Prompt + 4 greedy steps against the reference engine's own logits (tests/golden/models.npz)."""
    g = np.load(os.path.join(GOLD, "models.npz"))
    s = workload.shape(name)
    m = nmodel.build(name, fmt, context=256, max_seqs=2, max_rows=16, seed=0, perturb=True)
    want = g[f"{tag}_logits"]
    logits_close(m.forward(g[f"{tag}_prompt"], 0, slot=1), want[0])
    pos = 8
    for i, t in enumerate(g[f"{tag}_tokens"]):
        lg, am = m.decode([1], [t], [pos])
        logits_close(lg[0], want[i + 1])
        if margin(want[i + 1]) > 4e-2:
            assert int(am[0]) == int(np.argmax(want[i + 1]))
        pos += 1
    m.close()


@pytest.mark.parametrize("name,fmt", [("qwen3-tiny", FP8), ("gpt2-tiny", FP8), ("qwen3-tiny", FP4)])
def test_greedy_32_steps_teacher_forced(name, fmt):
    R = Restatement()
    s = workload.shape(name)
    tensors = list(workload.weights(s, seed=3, perturb=True))
    ref = omodels.make(s, tensors, fmt, 128, R)
    m = nmodel.Model(s, fmt, context=128, max_seqs=1, max_rows=64).load(tensors)
    prompt = workload.prompt(s, 20, seed=4)
    want = ref.forward(prompt, 0)
    logits_close(m.forward(prompt, 0), want)
    tok, pos, ties, errs = int(np.argmax(want)), 20, 0, []
    for _ in range(32):
        lg, am = m.decode([0], [tok], [pos])
        want = ref.forward(np.array([tok], np.int32), pos)
        errs.append(logits_close(lg[0], want))
        if int(am[0]) != int(np.argmax(want)):
            ties += 1
            assert margin(want) <= 2 * max(errs), f"greedy token differs with margin {margin(want)}"
        tok, pos = int(np.argmax(want)), pos + 1  # teacher-forced: the reference's token
    m.close()
    assert ties <= 2


def test_batched_decode_matches_single_sequence():
    """b sequences in one step == each sequence decoded alone (slots are independent). Six sequences run on the
    tensor-core matmul and one on the single-kernel step: different summation orders, so they agree to the
    fp32 rounding level, not bit for bit."""
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=5, perturb=True))
    m = nmodel.Model(s, FP8, context=96, max_seqs=6, max_rows=32).load(tensors)
    rng = np.random.default_rng(9)
    prompts = [workload.prompt(s, int(n), seed=10 + i) for i, n in enumerate(rng.integers(3, 40, 6))]
    first = []
    for slot, p in enumerate(prompts):
        first.append(int(np.argmax(m.prefill(p, slot))))
    slots = np.arange(6, dtype=np.int32)
    pos = np.array([len(p) for p in prompts], np.int32)
    lg_b, am_b = m.decode(slots, first, pos)
    # redo each sequence alone into a second model instance
    m2 = nmodel.Model(s, FP8, context=96, max_seqs=6, max_rows=32).load(tensors)
    for slot, p in enumerate(prompts):
        m2.prefill(p, slot)
        lg, am = m2.decode([slot], [first[slot]], [pos[slot]])
        np.testing.assert_allclose(lg_b[slot], lg[0], rtol=1e-4, atol=1e-4)
        if am_b[slot] != am[0]:
            srt = np.sort(lg[0])
            assert srt[-1] - srt[-2] <= 2e-4, "greedy token differs beyond a near-tie"
    m.close()
    m2.close()


def test_device_greedy_loop_matches_host_loop():
    """stage + step (argmax and position advance on the device, CUDA-graph replay) == decode with host feedback."""
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=6, perturb=True))
    n, steps = 4, 10
    prompts = [workload.prompt(s, 16, seed=20 + i) for i in range(n)]
    a = nmodel.Model(s, FP8, context=64, max_seqs=n, max_rows=16).load(tensors)
    b = nmodel.Model(s, FP8, context=64, max_seqs=n, max_rows=16).load(tensors)
    toks = []
    for i, p in enumerate(prompts):
        toks.append(int(np.argmax(a.prefill(p, i))))
        b.prefill(p, i)
    slots = np.arange(n, dtype=np.int32)
    pos = np.full(n, 16, np.int32)
    a.stage(slots, toks, pos)
    for k in range(steps):
        a.step(n, 16 + k)
    dev_tokens, dev_pos = a.tokens(n)
    host = np.array(toks, np.int32)
    for k in range(steps):
        _, am = b.decode(slots, host, pos + k, want_logits=False)
        host = am
    assert np.array_equal(dev_tokens, host)
    assert np.array_equal(dev_pos, pos + steps)
    a.close()
    b.close()


def test_forward_rejects_bad_input():
    s = workload.shape("qwen3-tiny")
    m = nmodel.build("qwen3-tiny", FP8, context=32, max_seqs=1, max_rows=8)
    import nekochat_b200 as nb
    with pytest.raises(nb.NekoError):
        m.forward([s["vocab"]], 0)          # token id out of range (Model::checkBatch)
    with pytest.raises(nb.NekoError):
        m.forward([1] * 9, 0)               # batch above max_rows
    with pytest.raises(nb.NekoError):
        m.forward([1, 2], 31)               # context overflow
    m.close()


def test_device_tensor_on_another_device_is_refused():
    """Weights in another GPU's memory are refused by the host with an error (a kernel would fault on them)."""
    import ctypes as C
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    m = nmodel.build("qwen3-tiny", FP8, context=32, max_seqs=1, max_rows=8, device=0)
    t = torch.zeros((4, 4), device="cuda:1")
    rc = nb.lib().neko_model_set_tensor_device(m.h, b"embed_tokens.weight", C.c_void_p(t.data_ptr()), 4, 4)
    assert rc != 0 and "device" in nb.lib().neko_model_last_error(m.h).decode()
    with pytest.raises(nb.NekoError, match="cuda:1"):
        m.set_tensor_device("embed_tokens.weight", t)
    m.close()


def test_step_launch_count_matches_captured_graph():
    """neko_model_step_launches (the bench's gpu_launches) == the kernel nodes of the captured step graph, on the
    single-kernel step (1, 4 sequences), the kernel chain with chained matmuls (8, 40, 64 sequences; 72 with the
    argmax and the token advance as kernels of their own) and without (130 rows: tcgen05 matmuls)."""
    s = workload.shape("qwen3-tiny")
    m = nmodel.build("qwen3-tiny", FP8, context=64, max_seqs=130, max_rows=130, seed=1)
    rng = np.random.default_rng(2)
    for n in (1, 4, 8, 40, 64, 72, 130):
        slots = np.arange(n, dtype=np.int32)
        m.stage(slots, rng.integers(0, s["vocab"], n).astype(np.int32), np.full(n, 5, np.int32))
        m.step(n, 5)
        assert m.graph_kernels() == m.step_launches(n), n
    m.close()


def test_device_greedy_loop_past_64_sequences():
    """stage + step for 72 sequences (greedy argmax and the token / position advance as separate kernels past
    64 output rows) == decode with host feedback."""
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=8, perturb=True))
    n, steps = 72, 4
    a = nmodel.Model(s, FP8, context=48, max_seqs=n, max_rows=n).load(tensors)
    b = nmodel.Model(s, FP8, context=48, max_seqs=n, max_rows=n).load(tensors)
    toks = []
    for i in range(n):
        p = workload.prompt(s, 8, seed=40 + i)
        toks.append(int(np.argmax(a.prefill(p, i))))
        b.prefill(p, i)
    slots = np.arange(n, dtype=np.int32)
    pos = np.full(n, 8, np.int32)
    a.stage(slots, toks, pos)
    for k in range(steps):
        a.step(n, 8 + k)
    dev_tokens, dev_pos = a.tokens(n)
    host = np.array(toks, np.int32)
    for k in range(steps):
        _, host = b.decode(slots, host, pos + k, want_logits=False)
    assert np.array_equal(dev_tokens, host)
    assert np.array_equal(dev_pos, pos + steps)
    a.close()
    b.close()


@pytest.mark.parametrize("n", [40, 100])
def test_chained_batch_matches_single_sequence(n):
    """n sequences in one step (matmuls chained: each epilogue writes the next matmul's split activations, the
    RMSNorms applied as row scales; 100 rows take two 64-row tiles) == each sequence decoded alone on the
    single-kernel step, to the fp32 rounding level."""
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=7, perturb=True))
    m = nmodel.Model(s, FP8, context=48, max_seqs=n, max_rows=n).load(tensors)
    m2 = nmodel.Model(s, FP8, context=48, max_seqs=n, max_rows=n).load(tensors)
    rng = np.random.default_rng(11)
    prompts = [workload.prompt(s, int(k), seed=30 + i) for i, k in enumerate(rng.integers(2, 30, n))]
    first = [int(np.argmax(m.prefill(p, slot))) for slot, p in enumerate(prompts)]
    slots = np.arange(n, dtype=np.int32)
    pos = np.array([len(p) for p in prompts], np.int32)
    lg_b, am_b = m.decode(slots, first, pos)
    for slot, p in enumerate(prompts):
        m2.prefill(p, slot)
        lg, am = m2.decode([slot], [first[slot]], [pos[slot]])
        np.testing.assert_allclose(lg_b[slot], lg[0], rtol=1e-4, atol=1e-4)
        if am_b[slot] != am[0]:
            srt = np.sort(lg[0])
            assert srt[-1] - srt[-2] <= 2e-4, "greedy token differs beyond a near-tie"
    m.close()
    m2.close()


def test_generate_reuses_the_cached_prefix_and_stops():
    """nekochat_b200.generate (Engine::generate semantics): a second turn whose prompt extends the first reuses the
    slot's cache (all but the last sampled token, which was never run) and samples from logits that match a fresh
    run of the whole prompt; a stop id ends generation before it; a full context ends it with reason 3."""
    from nekochat_b200.generate import SlotGenerator
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=12, perturb=True))
    p1 = [int(t) for t in workload.prompt(s, 20, seed=50)]
    a = nmodel.Model(s, FP8, context=96, max_seqs=1, max_rows=16).load(tensors)
    ga = SlotGenerator(a)
    out1, st1 = ga.generate(p1, 6)
    assert st1["reused_tokens"] == 0 and st1["generated_tokens"] == 6 and st1["stop_reason"] == 0
    p2 = p1 + out1 + [7, 8, 9]
    out2, st2 = ga.generate(p2, 4, keep_logits=True)
    assert st2["reused_tokens"] == len(p1) + len(out1) - 1
    b = nmodel.Model(s, FP8, context=96, max_seqs=1, max_rows=16).load(tensors)
    out_b, stb = SlotGenerator(b).generate(p2, 4, keep_logits=True)
    assert stb["reused_tokens"] == 0
    np.testing.assert_allclose(st2["logits"][0], stb["logits"][0], rtol=1e-4, atol=1e-4)
    # stop id: the token a plain run produces third ends generation after two tokens
    c = nmodel.Model(s, FP8, context=32, max_seqs=1, max_rows=16).load(tensors)
    plain, _ = SlotGenerator(c).generate(p1, 5)
    if plain[2] not in plain[:2]:
        stopped, stc = SlotGenerator(c, stop_ids=[plain[2]]).generate(p1, 5)
        assert stopped == plain[:2] and stc["stop_reason"] == 1
    # a full context: 20 prompt tokens + 12 decoded fill the 32 positions
    full, stf = SlotGenerator(c).generate(p1, 40)
    assert stf["stop_reason"] == 3 and len(full) == 32 - 20 + 1
    for mm in (a, b, c):
        mm.close()


@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_fp8_checkpoint_weights_load_like_f32(fmt):
    """A Qwen3-*-FP8 style checkpoint (every layer matrix as E4M3 codes with 128 x 128 block scales, ragged
    edges included) loaded through neko_model_set_tensor_fp8 gives the same logits, bit for bit, as the same
    weights dequantized by the reference loader's rule (tensor_store.cpp:543-571) on the host and loaded as f32."""
    from oracle.checkpoint import fp8_block_dequant
    s = workload.shape("qwen3-tiny")
    rng = np.random.default_rng(6)
    as_fp8, as_f32 = [], []
    for name, a in workload.weights(s, seed=5):
        if a.ndim == 2 and name.startswith("layers."):
            R, Cn = a.shape
            codes = (rng.integers(0x08, 0x48, (R, Cn)) | (rng.integers(0, 2, (R, Cn)) << 7)).astype(np.uint8)
            sc = (rng.random(((R + 127) // 128, (Cn + 127) // 128)) * 0.004 + 0.001).astype(np.float32)
            as_fp8.append((name, codes, sc))
            as_f32.append((name, fp8_block_dequant(codes, sc)))
        else:
            as_fp8.append((name, a))
            as_f32.append((name, a))
    a = nmodel.Model(s, fmt, context=64, max_seqs=1, max_rows=64).load(as_f32)
    b = nmodel.Model(s, fmt, context=64, max_seqs=1, max_rows=64).load(as_fp8)
    prompt = workload.prompt(s, 12, seed=7)
    la, lb = a.forward(prompt, 0), b.forward(prompt, 0)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    with pytest.raises(nb.NekoError):  # the weight's shape is checked after the dequantization
        b.set_tensor_fp8("layers.0.mlp.down_proj.weight", np.zeros((8, 8), np.uint8), np.ones((1, 1), np.float32))
    a.close()
    b.close()


def engine_turn(stream, stops, max_new):
    """Engine::generate's loop (engine.cpp:120-134) over a greedy token stream: (tokens, stop reason)."""
    out = []
    for t in stream:
        if t in stops:
            return out, 1
        out.append(t)
        if len(out) == max_new:
            return out, 0
    return out, -1


def test_device_loop_stop_ids_follow_engine_rules():
    """neko_model_set_stop: the device greedy loop logs each sequence's tokens and ends it at a stop id (the
    staged first token included) or after max_new tokens, exactly as the engine's loop would over the same greedy
    streams; finished sequences stay at their token and position while the others keep decoding."""
    s = workload.shape("qwen3-tiny")
    m = nmodel.Model(s, FP8, context=128, max_seqs=4, max_rows=64).load(workload.weights(s, seed=8))
    n, K, max_new = 3, 14, 9
    prompts = [workload.prompt(s, 10 + 3 * i, seed=20 + i) for i in range(n)]
    pos0 = [len(p) for p in prompts]

    def prefill():
        return [int(np.argmax(m.forward(p, 0, slot=i))) for i, p in enumerate(prompts)]

    first = prefill()
    m.stage(list(range(n)), first, pos0)
    streams = [[t] for t in first]
    for _ in range(K):
        m.step(n, max(pos0) + K)
        t, _ = m.tokens(n)
        for i in range(n):
            streams[i].append(int(t[i]))
    stops = sorted({streams[0][5], first[2]})
    m.set_stop(stops, max_new)
    assert prefill() == first
    m.stage(list(range(n)), first, pos0)
    for _ in range(K):
        m.step(n, max(pos0) + K)
    got, reasons = m.generated(n)
    for i in range(n):
        want, why = engine_turn(streams[i], set(stops), max_new)
        assert got[i].tolist() == want, f"sequence {i}"
        assert reasons[i] == why, f"sequence {i}"
    assert reasons[0] == 1 and reasons[2] == 1 and len(got[2]) == 0
    t, p = m.tokens(n)
    assert int(t[2]) == first[2] and int(p[2]) == pos0[2]  # frozen at its staged token and position
    m.set_stop([], 0)
    with pytest.raises(nb.NekoError):
        m.generated(n)
    m.close()


def test_batch_generator_engine_semantics():
    """BatchGenerator: three slots decoding together on the device give each slot exactly the engine's turn over
    the plain greedy stream of the same batch (stop ids, max_new); a slot near the end of its context finishes on
    the host with the engine's context-full stop; a second turn reuses each slot's cached prefix."""
    from nekochat_b200.generate import BatchGenerator
    s = workload.shape("qwen3-tiny")
    tensors = list(workload.weights(s, seed=14, perturb=True))
    prompts = {i: [int(t) for t in workload.prompt(s, 12 + 5 * i, seed=60 + i)] for i in range(3)}
    K, max_new = 12, 10
    # the plain streams: same batch, plain device steps read back one by one
    from nekochat_b200.generate import prefill_chunks
    b = nmodel.Model(s, FP8, context=96, max_seqs=3, max_rows=16).load(tensors)
    first = []
    for i in range(3):  # the generator's chunks, so the KV cache is bit-identical
        for lo, hi in prefill_chunks(0, len(prompts[i]), 16):
            lg = b.forward(np.array(prompts[i][lo:hi], np.int32), lo, slot=i)
        first.append(int(np.argmax(lg)))
    pos0 = [len(prompts[i]) for i in range(3)]
    b.stage([0, 1, 2], first, pos0)
    streams = [[t] for t in first]
    for k in range(K):
        b.step(3, max(pos0) + k)
        t, _ = b.tokens(3)
        for i in range(3):
            streams[i].append(int(t[i]))
    b.close()
    stops = [streams[1][4]] if streams[1][4] not in streams[1][:4] else []
    a = nmodel.Model(s, FP8, context=96, max_seqs=3, max_rows=16).load(tensors)
    g = BatchGenerator(a, stop_ids=stops)
    res = g.generate(prompts, max_new)
    for i in range(3):
        want, why = engine_turn(streams[i], set(stops), max_new)
        out, st = res[i]
        assert out == want and st["stop_reason"] == why, f"slot {i}"
        assert st["reused_tokens"] == 0
    # second turn: each prompt extends the first turn's prompt and reply
    p2 = {i: prompts[i] + res[i][0] + [5, 6] for i in range(3)}
    res2 = g.generate(p2, 3)
    for i in range(3):
        out1, st1 = res[i]
        ran = len(out1) if st1["stop_reason"] == 1 else len(out1) - 1
        assert res2[i][1]["reused_tokens"] == len(prompts[i]) + ran
        assert len(res2[i][0]) == res2[i][1]["generated_tokens"] <= 3
    a.close()
    # context-full: a 40-position context and a 30-token prompt give 40 - 30 + 1 tokens, stop reason 3
    c = nmodel.Model(s, FP8, context=40, max_seqs=2, max_rows=16).load(tensors)
    res3 = BatchGenerator(c).generate({0: prompts[0], 1: [int(t) for t in workload.prompt(s, 30, seed=70)]}, 20)
    assert res3[1][1]["stop_reason"] == 3 and len(res3[1][0]) == 40 - 30 + 1
    assert res3[0][1]["stop_reason"] == 0 and len(res3[0][0]) == 20
    c.close()


def test_decode_into_the_pinned_host_logits_buffer():
    """decode with out = host_logits() (no second host copy) returns the same logits and tokens as decode into a
    fresh array; the view is overwritten by the next call."""
    s = workload.shape("qwen3-tiny")
    m = nmodel.Model(s, FP8, context=64, max_seqs=2, max_rows=16).load(workload.weights(s, seed=4))
    for i in range(2):
        m.prefill(workload.prompt(s, 10, seed=80 + i), i)
    buf = m.host_logits(2)
    la, aa = m.decode([0, 1], [3, 4], [10, 10])
    lb, ab = m.decode([0, 1], [3, 4], [10, 10], out=buf)
    assert lb.ctypes.data == buf.ctypes.data
    assert np.array_equal(la, lb) and np.array_equal(aa, ab)
    m.decode([0, 1], [5, 6], [10, 10], out=buf)
    assert not np.array_equal(buf, la)
    m.close()


def test_host_logits_view_outlives_close():
    """A host_logits view stays readable after close(): the runner is destroyed only once the last view is
    released; the closed model refuses to decode or hand out new views."""
    import gc
    s = workload.shape("qwen3-tiny")
    m = nmodel.Model(s, FP8, context=64, max_seqs=1, max_rows=16).load(workload.weights(s, seed=4))
    m.prefill(workload.prompt(s, 10, seed=80), 0)
    buf = m.host_logits(1)
    want, _ = m.decode([0], [3], [10], out=buf)
    want = want.copy()
    m.close()
    assert np.array_equal(buf, want)  # still the runner's pinned buffer, not freed memory
    with pytest.raises(nb.NekoError, match="closed"):
        m.decode([0], [3], [10], out=buf)
    with pytest.raises(nb.NekoError, match="closed"):
        m.host_logits(1)
    del buf
    gc.collect()  # the last view is gone: the deferred destroy has run
