"""The fused forms of the decode step as single operators, and the model bisected layer by layer.

* norm prologue + matmul == cpu::rmsNorm / cpu::layerNorm then cpu::matmul (qwen3_model.cpp:245-247,
  gpt2_model.cpp:196-198), tolerance 2e-3 (1 + |cpu|) like the engine's self-test matmuls;
* SwiGLU pair == cpu::matmul into [gate | up] then cpu::siluMul (qwen3_model.cpp:263-265);
* neko_model_set_debug(n) (Model::setDebugLayers, the engine's `--bisect`): hidden states after n layers against
  the oracle forward stopped at n layers.
"""
import numpy as np
import pytest

from nekochat_b200 import model as nmodel, workload
from oracle import models as omodels
from oracle.oracle import ACCUMULATE, FP4, FP8, F16, GELU, Restatement

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def R():
    return Restatement()


def close(a, b, tol=2e-3):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    d = np.abs(a - b)
    ok = d <= tol * (1 + np.abs(b))
    assert ok.all(), f"max err {d.max()} at {np.unravel_index(np.argmax(~ok), a.shape)}: {a.flat[np.argmax(~ok)]} vs {b.flat[np.argmax(~ok)]}"


def cu(torch, a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M,K", [(1, 256), (3, 256), (8, 512), (10, 256)])  # up to M * K = 4096, 40 KB FP4
@pytest.mark.parametrize("kind", ["rms", "ln"])
def test_norm_prologue_matmul(torch, R, fmt, M, K, kind):
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + 10 * fmt)
    N = 300
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    q = R.quantize(fmt, (rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    if kind == "rms":
        xn, y = R.rms_norm(x, g, 1e-6), ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, N, 1, cu(torch, g), None, 1e-6)
        want = R.matmul(fmt, xn, q, K)
    else:
        xn = R.layer_norm(x, g, b, 1e-5)
        y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, N, 2, cu(torch, g), cu(torch, b), 1e-5,
                             bias=cu(torch, bias), flags=GELU)
        want = R.matmul(fmt, xn, q, K, bias, None, None, GELU)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), want)


@pytest.mark.parametrize("fmt", [FP8, FP4, F16])
@pytest.mark.parametrize("M", [1, 2, 7, 10])
@pytest.mark.parametrize("norm", [0, 1])
def test_swiglu_pair(torch, R, fmt, M, norm):
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 3 + fmt + 7 * norm)
    K, F = 256, 320
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    q = R.quantize(fmt, w) if fmt != F16 else w.astype(np.float16).view(np.uint8).reshape(2 * F, 2 * K)
    xin = R.rms_norm(x, g, 1e-6) if norm else x
    h = R.matmul(fmt, xin, q, K)
    want = R.silu_mul(h, F)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, norm, cu(torch, g) if norm else None, None, 1e-6,
                         swiglu=True)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), want)


@pytest.mark.parametrize("K,N", [(9728, 2560), (9728, 40)])
def test_wide_rows_plan(torch, R, K, N):
    """K = 9728 (Qwen3-4B down_proj): rows so wide that fewer rows than warps fit per ring stage."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(K + N)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, K)).astype(np.float32)
    for fmt in (FP8, FP4):
        q = R.quantize(fmt, w)
        y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
        torch.cuda.synchronize()
        close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


STAGES = {"qwen3": [(2, "qkv"), (3, "qk-norm+rope"), (4, "attn"), (5, "o_proj+res"), (8, "silu*up"),
                    (9, "down+res")],
          "gpt2": [(2, "qkv"), (3, "attn"), (4, "proj+res"), (6, "fc+gelu"), (7, "fc2+res")]}


@pytest.mark.parametrize("name,fmt,T", [("qwen3-tiny", FP8, 8), ("qwen3-tiny", FP8, 1), ("gpt2-tiny", FP8, 20),
                                        ("gpt2-tiny", FP8, 8), ("qwen3-tiny", FP4, 8)])
def test_bisect_layers(name, fmt, T):
    """Every dumpable stage of every layer for one prefill chunk (the engine's --bisect, cli_main.cpp:402-442)."""
    s = workload.shape(name)
    tensors = list(workload.weights(s, seed=0, perturb=True))
    prompt = workload.prompt(s, T, seed=2)
    ref = omodels.make(s, tensors, fmt, 64, Restatement())
    m = nmodel.Model(s, fmt, context=64, max_seqs=1, max_rows=32).load(tensors)
    failures = []
    for n in range(s["layers"] + 1):
        for st, label in [(0, "hidden")] + (STAGES[s["arch"]] if n < s["layers"] else []):
            want = omodels.make(s, tensors, fmt, 64, ref.R).forward(prompt, 0, stop_layer=n, stage=st)
            m.set_debug(n, st)
            got = m.hidden(prompt, 0, width=want.shape[1])
            d = np.abs(got - want)
            if not d.max() <= 1e-3 * (1 + np.abs(want).max()):
                failures.append(f"layer {n} stage {st} ({label}): max err {d.max():.4g} |x| {np.abs(want).max():.4g} "
                                f"at {np.unravel_index(np.argmax(d), d.shape)}")
    m.close()
    assert not failures, "\n".join(failures)
