"""The oracle (my C restatement, oracle/neko_oracle.c) pinned to the reference engine.

1. Against the golden fixtures the reference itself produced (tests/golden/make_golden.py): bit-exact.
2. Live against the compiled reference (oracle/_ref/libneko_ref.so) on fresh seeded inputs, when it is built.
3. A planted mistake in the oracle's output is caught by the same comparison (the checks are not vacuous).
"""
import os

import numpy as np
import pytest

from oracle import models as omodels
from oracle.oracle import ACCUMULATE, FP4, FP8, F16, GELU, Reference, Restatement
from nekochat_b200 import workload
from tests.golden.make_golden import attention_case

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REF_SO = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libneko_ref.so")


@pytest.fixture(scope="module")
def R():
    return Restatement()


@pytest.fixture(scope="module")
def g():
    return {k: dict(np.load(os.path.join(GOLD, k + ".npz"))) for k in ("codec", "ops", "models")}


def bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32) if a.dtype == np.float32 else a,
                                                 b.view(np.uint32) if b.dtype == np.float32 else b)


@pytest.mark.parametrize("tag,fmt", [("fp8", FP8), ("fp4", FP4)])
def test_codec_golden(R, g, tag, fmt):
    c = g["codec"]
    q = R.quantize(fmt, c[f"{tag}_w"])
    assert np.array_equal(q, c[f"{tag}_q"]), "quantizeMatrix bytes differ from the reference"
    assert bits_equal(R.dequantize(fmt, c[f"{tag}_q"], 96), c[f"{tag}_deq"])
    assert bits_equal(R.dequantize(fmt, c[f"{tag}_raw"], 256), c[f"{tag}_raw_deq"])


def test_row_bytes(R):
    # quantRowBytes values for the benchmarked models' K dimensions
    for K, f8, f4 in ((1024, 1088, 576), (2048, 2176, 1152), (3072, 3264, 1728), (768, 816, 432),
                      (2560, 2720, 1440), (9728, 10336, 5472)):
        assert R.row_bytes(FP8, K) == f8 == workload.row_bytes(FP8, K)
        assert R.row_bytes(FP4, K) == f4 == workload.row_bytes(FP4, K)


@pytest.mark.parametrize("tag,fmt", [("fp8", FP8), ("fp4", FP4)])
@pytest.mark.parametrize("K", [96, 1024])
def test_matmul_golden(R, g, tag, fmt, K):
    o = g["ops"]
    p = f"mm_{tag}_{K}_"
    y = R.matmul(fmt, o[p + "x"], o[p + "q"], K, o[p + "b"], o[p + "y0"].copy(), 42, ACCUMULATE, 3)
    assert bits_equal(y, o[p + "y"])
    yg = R.matmul(fmt, o[p + "x"], o[p + "q"], K, o[p + "b"], None, None, GELU)
    assert bits_equal(yg, o[p + "ygelu"])


def test_f16_matmul_golden(R, g):
    o = g["ops"]
    assert bits_equal(R.matmul(F16, o["mm_f16_x"], o["mm_f16_q"], 64, o["mm_f16_b"], None, None, GELU), o["mm_f16_y"])


def test_norms_rope_act_golden(R, g):
    o = g["ops"]
    assert bits_equal(R.layer_norm(o["norm_x"], o["norm_g"], o["norm_b"], 1e-5), o["ln_y"])
    assert bits_equal(R.rms_norm(o["norm_x"], o["norm_g"], 1e-6), o["rms_y"])
    r = o["rope_x"].copy()
    R.rope(r, 3, 64, o["rope_cs"])
    assert bits_equal(r, o["rope_y"])
    assert bits_equal(R.silu_mul(o["silu_h"], 100), o["silu_y"])
    assert bits_equal(np.array([R.gelu(float(v)) for v in o["gelu_x"]], np.float32), o["gelu_y"])


def test_kv_attention_golden(R, g):
    o = g["ops"]
    H, KV, hd, T, pos0, qkv, kc, vc = attention_case()
    stride, kvW = (H + 2 * KV) * hd, KV * hd
    R.store_kv(qkv[:, H * hd:], qkv[:, (H + KV) * hd:], stride, kc, vc, kvW, T, pos0)
    assert np.array_equal(kc[pos0:pos0 + T], o["att_k_new"]) and np.array_equal(vc[pos0:pos0 + T], o["att_v_new"])
    assert bits_equal(R.attention(qkv, stride, kc, vc, T, H, KV, hd, pos0), o["att_y"])


@pytest.mark.parametrize("tag,name,fmt", [("qwen3_fp8", "qwen3-tiny", FP8), ("qwen3_fp4", "qwen3-tiny", FP4),
                                          ("gpt2_fp8", "gpt2-tiny", FP8)])
def test_models_golden(R, g, tag, name, fmt):
    """Model-level restatement (oracle/models.py) == the reference's Model::forward, bit for bit."""
    m = g["models"]
    s = workload.shape(name)
    om = omodels.make(s, workload.weights(s, seed=0, perturb=True), fmt, 256, R)
    logits = [om.forward(m[f"{tag}_prompt"], 0)]
    pos = 8
    for t in m[f"{tag}_tokens"]:
        logits.append(om.forward(np.array([t], np.int32), pos))
        pos += 1
    assert bits_equal(np.stack(logits), m[f"{tag}_logits"])
    assert [int(np.argmax(l)) for l in logits[:-1]] == list(m[f"{tag}_tokens"])


def test_planted_mistake_is_caught(R, g):
    """Flip one mantissa bit of one oracle output: the bit-exact comparison must reject it."""
    o = g["ops"]
    y = R.layer_norm(o["norm_x"], o["norm_g"], o["norm_b"], 1e-5)
    y.view(np.uint32)[1, 7] ^= 1
    assert not bits_equal(y, o["ln_y"])
    q = R.quantize(FP8, g["codec"]["fp8_w"])
    q[3, 5] ^= 0x10
    assert not np.array_equal(q, g["codec"]["fp8_q"])


needs_ref = pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref not built (needs the reference source)")


@needs_ref
@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_live_codec_vs_reference(R, fmt):
    F = Reference()
    rng = np.random.default_rng(100 + fmt)
    for rows, cols, scale in ((64, 1024, 0.02), (16, 3072, 1.0), (7, 96, 300.0), (5, 64, 1e-6)):
        w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
        q = R.quantize(fmt, w)
        assert np.array_equal(q, F.quantize(fmt, w))
        assert bits_equal(R.dequantize(fmt, q, cols), F.dequantize(fmt, q, cols))


@needs_ref
def test_live_ops_vs_reference(R):
    F = Reference()
    rng = np.random.default_rng(7)
    for fmt in (FP8, FP4):
        for K, N, T in ((96, 37, 5), (2048, 24, 3), (3072, 9, 1)):
            w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
            x = (rng.standard_normal((T, K)) * 20).astype(np.float32)
            q = R.quantize(fmt, w)
            assert bits_equal(R.matmul(fmt, x, q, K), F.matmul(fmt, x, q, K))
    x = (rng.standard_normal((4, 1024)) * 3).astype(np.float32)
    gm = rng.standard_normal(1024).astype(np.float32)
    assert bits_equal(R.rms_norm(x, gm, 1e-6), F.rms_norm(x, gm, 1e-6))
    assert bits_equal(R.layer_norm(x, gm, gm, 1e-5), F.layer_norm(x, gm, gm, 1e-5))
