"""The warp-specialised tcgen05 matmul (k_umma_ws.cu: 5..64 activation rows, the weights as the UMMA's 128-row M
side) against the oracle's cpu::matmul, through the operator API.

The op API splits the activations into f16 hi / lo first whenever 8+ column tiles share them (or the call has a
norm prologue, or 64 rows), and those calls take this kernel; the shapes below are chosen to do so. Weights enter
as w = code x scale split into f16 hi + lo, activations as f16 hi + lo, fp32 accumulation in TMEM: held to the
fp32 kernels' bound |gpu - cpu| <= 2e-3 (1 + |cpu|).
"""
import numpy as np
import pytest

from oracle.oracle import ACCUMULATE, FP4, FP8, GELU, Restatement

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def R():
    return Restatement()


def close(a, b, tol=TOL):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    d = np.abs(a - b)
    ok = d <= tol * (1 + np.abs(b))
    assert ok.all(), f"max err {d.max()} at {np.unravel_index(np.argmax(~ok), a.shape)}"


def cu(torch, a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M", [5, 17, 32, 33, 64])
@pytest.mark.parametrize("K,N", [(1024, 4096), (2048, 1024), (3072, 1024), (64, 600), (1344, 520), (192, 1000)])
def test_ws_matmul_shapes(torch, R, fmt, M, K, N):
    """N = 32 / 64 activation columns (rows past M zero), partial last weight tiles, a single K stage, K stage
    counts the splits do not divide evenly, scale groups that end inside a row's padding (K = 192)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 11 + K + N + fmt)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("flags", [0, GELU, ACCUMULATE, GELU | ACCUMULATE])
def test_ws_matmul_epilogues(torch, R, fmt, flags):
    """bias, GELU, residual accumulate into a wider output (y_stride, n_off), like the model's layers."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(flags + 10 * fmt)
    M, K, N, ys, off = 24, 2048, 700, 760, 37
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    y0 = rng.standard_normal((M, ys)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = cu(torch, y0.copy())
    ops.matmul(fmt, cu(torch, x), cu(torch, q), K, bias=cu(torch, bias), y=y, y_stride=ys, n_off=off, flags=flags)
    torch.cuda.synchronize()
    want = y0.copy()
    R.matmul(fmt, x, q, K, bias, want, ys, flags, off)
    close(y.cpu().numpy(), want)


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M,F", [(8, 320), (40, 3072), (64, 1000)])
def test_ws_swiglu_pair(torch, R, fmt, M, F):
    """gate | up rows in one call (64 gate + 64 up rows per CTA): silu(gate . x) * (up . x)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + F + fmt)
    K = 1024
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, 0, None, None, 1e-6, swiglu=True)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.silu_mul(R.matmul(fmt, x, q, K), F))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("norm", [1, 2])
def test_ws_norm_prologue(torch, R, fmt, norm):
    """RMSNorm (1) / LayerNorm (2) applied by the activation split, then this kernel (the op API's norm prologue
    takes T * K <= 4096)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(norm + 3 * fmt)
    M, K, N = 5, 768, 1536
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = (rng.standard_normal((M, K)) * 3 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, N, norm, cu(torch, g), cu(torch, b), 1e-5)
    torch.cuda.synchronize()
    xn = R.rms_norm(x, g, 1e-5) if norm == 1 else R.layer_norm(x, g, b, 1e-5)
    close(y.cpu().numpy(), R.matmul(fmt, xn, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_ws_matmul_deterministic(torch, R, fmt):
    """The K splits' partials are summed in split order: repeated calls give bit-identical results."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(7 + fmt)
    M, K, N = 48, 3072, 1024
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    xt = cu(torch, rng.standard_normal((M, K)).astype(np.float32))
    qt = cu(torch, R.quantize(fmt, w))
    first = ops.matmul(fmt, xt, qt, K).cpu().numpy()
    for _ in range(4):
        assert np.array_equal(ops.matmul(fmt, xt, qt, K).cpu().numpy(), first)


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M", [17, 64])
def test_ws_two_per_sm(torch, R, fmt, M):
    """More weight tiles than two waves and no K split (the LM-head shape class): two CTAs per SM, the receive
    buffer over the drained rings."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + 100 * fmt)
    K, N = 1024, 40000
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_ws_two_per_sm_swiglu(torch, R, fmt):
    """The SwiGLU pair at more than two waves of tiles (64 gate + 64 up rows each), two CTAs per SM."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(9 + fmt)
    M, K, F = 40, 1024, 20000
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, 0, None, None, 1e-6, swiglu=True)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.silu_mul(R.matmul(fmt, x, q, K), F))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M", [17, 64])
def test_ws_two_per_sm_split(torch, R, fmt, M):
    """A single wave of tiles that two CTAs per SM let split K further (one raw stage of 4 K stages per split,
    4 splits): the split two-per-SM layout, partials pushed into a receive buffer of its own."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + 200 * fmt)
    K, N = 1024, 8192
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K, bias=cu(torch, bias), flags=GELU)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K, bias, None, None, GELU))
