"""The direct-load tensor-core GEMV (FP8 weights, 1..4 activation rows; nekochat_b200/csrc/k_gemv_fp8tc.cu) through
the C ABI: both phases of its plan (whole tiles per warp; leftover tiles split over K 1..16 ways), the norm
prologue, the SwiGLU pair, the bias / GELU / accumulate epilogues with an output offset, and activations whose
magnitudes span many decades (f16 hi / lo pairs under one power-of-two scale per activation row). Checked against
the oracle's cpu::matmul (tolerance 2e-3 (1 + |cpu|), the engine's self-test bound) and, where the oracle's
sequential sum is too slow, against an fp64 product of the exactly dequantized weights at 1e-4 (1 + |ref|)."""
import numpy as np
import pytest

from oracle.oracle import ACCUMULATE, FP8, GELU, Restatement

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
    assert ok.all(), f"max err {d.max()} at {np.unravel_index(np.argmax(~ok), a.shape)}"


def cu(torch, a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


def fp64_ref(torch, x, q, K):
    from nekochat_b200 import ops
    deq = ops.dequantize(FP8, q, K).double()
    return (x.double() @ deq.T).float()


# tiles (16 rows) 19 / 148 / 296 / 592 / 1250 / 2600: K split 16, 16, 8, 4, 1 ways, and 2600 = one full round
# of whole tiles (148 SMs x 16 warps) plus 232 tiles split 8 ways; 300, 20000 and 41593 end in a partial tile
@pytest.mark.parametrize("N", [300, 2368, 4736, 9472, 20000, 41593])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("K", [1024, 3072])
def test_plans_against_fp64(torch, M, K, N):
    from nekochat_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(N + 7 * K + M)
    w = torch.randn((N, K), generator=g, device="cuda") * 0.02
    x = torch.randn((M, K), generator=g, device="cuda")
    q = ops.quantize(FP8, w)
    y = ops.matmul(FP8, x, q, K)
    ref = fp64_ref(torch, x, q, K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), ref.cpu().numpy(), 1e-4)


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_small_shapes_against_oracle(torch, R, M):
    rng = np.random.default_rng(40 + M)
    for K, N in ((128, 5), (256, 17), (1024, 300), (2048, 1031)):
        w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        q = R.quantize(FP8, w)
        from nekochat_b200 import ops
        y = ops.matmul(FP8, cu(torch, x), cu(torch, q), K)
        torch.cuda.synchronize()
        close(y.cpu().numpy(), R.matmul(FP8, x, q, K))


CASES = ["decades", "tiny", "huge", "zeros", "one_hot", "row_scales_differ"]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("M", [1, 2, 4])
def test_activation_ranges(torch, case, M):
    """The power-of-two scale and the hi / lo split: magnitudes over 1e-30 .. 1e30, zero rows, a single non-zero."""
    from nekochat_b200 import ops
    K, N = 2048, 1500
    rng = np.random.default_rng(10 * CASES.index(case) + M)
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randn((N, K), generator=g, device="cuda") * 0.02
    q = ops.quantize(FP8, w)
    if case == "decades":
        x = rng.standard_normal((M, K)) * 10.0 ** rng.uniform(-8, 4, (M, K))
    elif case == "tiny":
        x = rng.standard_normal((M, K)) * 1e-30
    elif case == "huge":
        x = rng.standard_normal((M, K)) * 1e30
    elif case == "zeros":
        x = np.zeros((M, K))
    elif case == "one_hot":
        x = np.zeros((M, K))
        x[:, 777] = -3.25
    else:
        x = rng.standard_normal((M, K)) * (10.0 ** np.linspace(-20, 20, M))[:, None]
    xt = cu(torch, x.astype(np.float32))
    y = ops.matmul(FP8, xt, q, K)
    ref = fp64_ref(torch, xt, q, K)
    deq = ops.dequantize(FP8, q, K).double()
    mag = (xt.double().abs() @ deq.abs().T).cpu().numpy()  # sum_k |x_k w_k|
    torch.cuda.synchronize()
    y, ref = y.cpu().numpy(), ref.cpu().numpy()
    assert np.isfinite(y).all()
    # hi + lo: about 2^-22 of each product, plus 2^-38 of the row's largest activation per weight (loose bound)
    ws = deq.abs().sum(dim=1).cpu().numpy()
    for m in range(M):
        bound = 2.0 ** -14 * mag[m] + 2.0 ** -27 * np.abs(x[m]).max() * ws + 1e-37
        d = np.abs(y[m].astype(np.float64) - ref[m])
        assert (d <= bound).all(), f"row {m}: max err {d.max():.3g}, worst ratio {(d / bound).max():.3g}"


@pytest.mark.parametrize("M", [1, 2, 4])
@pytest.mark.parametrize("F", [320, 20000, 40000])
@pytest.mark.parametrize("norm", [0, 1])
def test_swiglu_pair(torch, R, M, F, norm):
    """Gate and up rows of the same tile (F = 320: K split 16 ways; 20000: 1250 tiles, one warp each; 40000: a
    full round of whole tiles and 132 tiles split 16 ways)."""
    from nekochat_b200 import ops
    rng = np.random.default_rng(M * 3 + F + norm)
    K = 1024
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    gt = torch.Generator(device="cuda").manual_seed(F + M)
    w = torch.randn((2 * F, K), generator=gt, device="cuda") * 0.03
    q = ops.quantize(FP8, w)
    y = ops.matmul_fused(FP8, cu(torch, x), q, K, F, norm, cu(torch, g) if norm else None, None, 1e-6, swiglu=True)
    xin = R.rms_norm(x, g, 1e-6) if norm else x
    h = fp64_ref(torch, cu(torch, xin), q, K).cpu().numpy()
    want = R.silu_mul(h, F)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), want)


@pytest.mark.parametrize("M", [1, 3])
@pytest.mark.parametrize("flags", [ACCUMULATE, GELU, GELU | ACCUMULATE])
def test_epilogues(torch, R, M, flags):
    from nekochat_b200 import ops
    rng = np.random.default_rng(flags + 10 * M)
    K, N, NS, off = 1024, 200, 211, 7
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y0 = rng.standard_normal((M, NS)).astype(np.float32)
    q = R.quantize(FP8, w)
    y = ops.matmul(FP8, cu(torch, x), cu(torch, q), K, cu(torch, b), cu(torch, y0.copy()), NS, off, flags)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), R.matmul(FP8, x, q, K, b, y0.copy(), NS, flags, off))


@pytest.mark.parametrize("kind", ["rms", "ln"])
@pytest.mark.parametrize("M", [1, 2])
def test_norm_prologue(torch, R, kind, M):
    from nekochat_b200 import ops
    rng = np.random.default_rng(M + (kind == "ln"))
    K, N = 2048, 700
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(K)).astype(np.float32)
    q = R.quantize(FP8, (rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    if kind == "rms":
        y = ops.matmul_fused(FP8, cu(torch, x), cu(torch, q), K, N, 1, cu(torch, g), None, 1e-6)
        want = R.matmul(FP8, R.rms_norm(x, g, 1e-6), q, K)
    else:
        y = ops.matmul_fused(FP8, cu(torch, x), cu(torch, q), K, N, 2, cu(torch, g), cu(torch, b), 1e-5)
        want = R.matmul(FP8, R.layer_norm(x, g, b, 1e-5), q, K)
    torch.cuda.synchronize()
    close(y.cpu().numpy(), want)
