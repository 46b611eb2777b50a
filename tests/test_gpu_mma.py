"""The tensor-core matmul (k_mma.cu, 5+ activation rows) against the oracle's cpu::matmul.

Weights enter as exact codes with the block scale applied in fp32, activations as two f16 halves (hi + lo), so
the results are held to the fp32 kernels' bound: the engine's matmul self-test form |gpu - cpu| <= tol * (1 +
|cpu|) with tol = 2e-3.
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
@pytest.mark.parametrize("M", [5, 16, 64, 100])
@pytest.mark.parametrize("K,N", [(1024, 300), (3072, 1024), (9728, 40)])
def test_tc_matmul_shapes(torch, R, fmt, M, K, N):
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 7 + K + fmt)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("flags", [GELU, ACCUMULATE, GELU | ACCUMULATE])
def test_tc_matmul_epilogues(torch, R, fmt, flags):
    """bias + GELU / residual accumulate into a wider output (y_stride, n_off), like the model's layers."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(flags + 10 * fmt)
    M, K, N, ys, off = 24, 2048, 200, 260, 37
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
@pytest.mark.parametrize("M", [8, 64])
def test_tc_swiglu_pair(torch, R, fmt, M):
    """gate | up rows in one call: silu(gate . x) * (up . x) (cpu::matmul into [gate|up] then cpu::siluMul)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + fmt)
    K, F = 1024, 320
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, 0, None, None, 1e-6, swiglu=True)
    torch.cuda.synchronize()
    h = R.matmul(fmt, x, q, K)
    want = R.silu_mul(h, F)
    close(y.cpu().numpy(), want)


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M,K,N", [(7, 1344, 300), (64, 1344, 520), (130, 4096, 96), (9, 64, 2000)])
def test_tc_matmul_uneven_k_splits(torch, R, fmt, M, K, N):
    """K stage counts that the splits do not divide evenly (a short last split), a single K stage, row blocks
    past 64 and split activations (8+ column tiles)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + K + N + fmt)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_tc_matmul_deterministic(torch, R, fmt):
    """Split-K partial tiles are summed in split order by whichever CTA finishes last: repeated calls give
    bit-identical results."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(5 + fmt)
    M, K, N = 48, 3072, 1024
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    xt = cu(torch, rng.standard_normal((M, K)).astype(np.float32))
    qt = cu(torch, R.quantize(fmt, w))
    first = ops.matmul(fmt, xt, qt, K).cpu().numpy()
    for _ in range(4):
        assert np.array_equal(ops.matmul(fmt, xt, qt, K).cpu().numpy(), first)


# ------------------------------------------------------------------------------------------- tcgen05 (128+ rows)
@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M,K,N", [(128, 1024, 3072), (200, 3072, 1024), (256, 2048, 700), (129, 64, 96)])
def test_umma_matmul_shapes(torch, R, fmt, M, K, N):
    """The tcgen05 path: scale-folded hi/lo f16 weights, hi/lo activations, TMEM accumulation over all of K;
    several row blocks, partial row blocks, K split over clusters (small N), a single K stage."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 3 + K + N + fmt)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("flags", [GELU, ACCUMULATE])
def test_umma_epilogues(torch, R, fmt, flags):
    from nekochat_b200 import ops
    rng = np.random.default_rng(flags + 20 * fmt)
    M, K, N, ys, off = 160, 1024, 200, 260, 37
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
def test_umma_swiglu_pair(torch, R, fmt):
    from nekochat_b200 import ops
    rng = np.random.default_rng(40 + fmt)
    M, K, F = 192, 1024, 320
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, 0, None, None, 1e-6, swiglu=True)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.silu_mul(R.matmul(fmt, x, q, K), F))


def test_umma_deterministic(torch, R):
    """Cluster split-K partial tiles are summed in split order: repeated calls give bit-identical results."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(9)
    M, K, N = 128, 3072, 1024
    xt = cu(torch, rng.standard_normal((M, K)).astype(np.float32))
    qt = cu(torch, R.quantize(FP8, (rng.standard_normal((N, K)) * 0.02).astype(np.float32)))
    first = ops.matmul(FP8, xt, qt, K).cpu().numpy()
    for _ in range(3):
        assert np.array_equal(ops.matmul(FP8, xt, qt, K).cpu().numpy(), first)


# ---------------------------------------------------------------------- dequantise, then tcgen05 GEMM (256+ rows)
@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("M,K,N", [(256, 1024, 3072), (300, 2048, 700), (512, 3072, 1024), (384, 64, 200)])
def test_dq_gemm_shapes(torch, R, fmt, M, K, N):
    """256+ rows: the weights dequantised once into hi / lo f16 rows, then the TMA-fed tcgen05 GEMM; partial row
    and column tiles (zero-filled tensor copies past the matrices), K split over clusters, a single K stage."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 5 + K + N + fmt)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul(fmt, cu(torch, x), cu(torch, q), K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("flags", [GELU, ACCUMULATE])
def test_dq_gemm_epilogues(torch, R, fmt, flags):
    from nekochat_b200 import ops
    rng = np.random.default_rng(flags + 30 * fmt)
    M, K, N, ys, off = 320, 1024, 200, 260, 37
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
def test_dq_gemm_swiglu_pair(torch, R, fmt):
    from nekochat_b200 import ops
    rng = np.random.default_rng(50 + fmt)
    M, K, F = 300, 1024, 320
    w = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(fmt, w)
    y = ops.matmul_fused(fmt, cu(torch, x), cu(torch, q), K, F, 0, None, None, 1e-6, swiglu=True)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.silu_mul(R.matmul(fmt, x, q, K), F))


def test_dq_gemm_deterministic(torch, R):
    """Repeated calls (cluster split-K summed in split order) give bit-identical results."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(19)
    M, K, N = 512, 3072, 1024
    xt = cu(torch, rng.standard_normal((M, K)).astype(np.float32))
    qt = cu(torch, R.quantize(FP8, (rng.standard_normal((N, K)) * 0.02).astype(np.float32)))
    first = ops.matmul(FP8, xt, qt, K).cpu().numpy()
    for _ in range(2):
        assert np.array_equal(ops.matmul(FP8, xt, qt, K).cpu().numpy(), first)
