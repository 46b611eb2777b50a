"""Operator parity through the C ABI (neko_op_*) against the oracle: dequant matmul over the benchmarked shapes and
odd shapes (tolerance |gpu - cpu| <= 2e-3 (1 + |cpu|), the engine's self-test bound for matmuls), norms,
softmax, argmax and attention."""
import numpy as np
import pytest

from oracle.oracle import ACCUMULATE, FP4, FP8, F16, GELU, Restatement

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


def run_matmul(torch, fmt, x, q, K, bias=None, y0=None, y_stride=None, n_off=0, flags=0):
    from nekochat_b200 import ops
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    y = ops.matmul(fmt, t(x), t(q), K, t(bias), t(y0), y_stride, n_off, flags)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("fmt", [FP8, FP4, F16])
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 13])
@pytest.mark.parametrize("K,N", [(96, 37), (1024, 300), (3072, 129), (2048, 1024)])
def test_matmul_shapes(torch, R, fmt, M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N + fmt)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = (rng.standard_normal((M, K))).astype(np.float32)
    q = R.quantize(fmt, w) if fmt != F16 else w.astype(np.float16).view(np.uint8).reshape(N, 2 * K)
    close(run_matmul(torch, fmt, x, q, K), R.matmul(fmt, x, q, K))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("flags", [ACCUMULATE, GELU, GELU | ACCUMULATE])
def test_matmul_epilogues(torch, R, fmt, flags):
    rng = np.random.default_rng(flags)
    K, N, M, NS, off = 1024, 200, 4, 211, 7
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y0 = rng.standard_normal((M, NS)).astype(np.float32)
    q = R.quantize(fmt, w)
    close(run_matmul(torch, fmt, x, q, K, b, y0.copy(), NS, off, flags),
          R.matmul(fmt, x, q, K, b, y0.copy(), NS, flags, off))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("K,N", [(1024, 3072), (3072, 1024), (2048, 6144), (2560, 9728), (9728, 2560), (1024, 151936)])
def test_matmul_baseline_sweep_m1(torch, R, fmt, K, N):
    """The reference's operator sweep shapes at M = 1 (decode), weights quantized on the GPU, checked against an
    fp64 product of the exactly dequantized weights (the oracle's sequential sum is too slow at 152K rows)."""
    from nekochat_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(K * 7 + N)
    w = torch.randn((N, K), generator=g, device="cuda") * 0.02
    x = torch.randn((1, K), generator=g, device="cuda")
    q = ops.quantize(fmt, w)
    y = ops.matmul(fmt, x, q, K)
    deq = ops.dequantize(fmt, q, K).double()
    ref = (x.double() @ deq.T).float()
    torch.cuda.synchronize()
    close(y.cpu().numpy(), ref.cpu().numpy(), 1e-4)
    # spot-check rows against the oracle's exact sequential sum
    rows = np.linspace(0, N - 1, 16).astype(int)
    qh = q[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    close(y.cpu().numpy()[:, rows], R.matmul(fmt, x.cpu().numpy(), qh, K))


@pytest.mark.parametrize("M", [16, 64])
def test_matmul_many_rows(torch, R, M):
    """Prefill-sized activations (x read from global memory, several passes over each staged row block)."""
    rng = np.random.default_rng(M)
    K, N = 1024, 512
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = R.quantize(FP8, w)
    close(run_matmul(torch, FP8, x, q, K), R.matmul(FP8, x, q, K))


# (151936, 1..2) and (20000, 100): wide rows, fewer than the SMs, split over CTAs (RMSNorm; LayerNorm keeps one
# CTA per row, or a cluster per row past the row cache); (16384, 150): one CTA per row; (1024, 300),
# (2500, 400): a warp per row; (40000, 160): a cluster of 2 CTAs per row
@pytest.mark.parametrize("C,rows", [(96, 3), (1024, 7), (2560, 2), (151936, 2), (151936, 1), (20000, 100),
                                    (16384, 150), (1024, 300), (2500, 400), (40000, 160)])
def test_norms(torch, R, C, rows):
    from nekochat_b200 import ops
    rng = np.random.default_rng(C)
    x = (rng.standard_normal((rows, C)) * 5).astype(np.float32)
    g = rng.standard_normal(C).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    tx, tg, tb = (torch.from_numpy(a).cuda() for a in (x, g, b))
    close(ops.norm(tx, tg, None, 1e-6).cpu().numpy(), R.rms_norm(x, g, 1e-6), 1e-5)
    close(ops.norm(tx, tg, tb, 1e-5).cpu().numpy(), R.layer_norm(x, g, b, 1e-5), 1e-5)


@pytest.mark.parametrize("C,rows", [(1024, 5), (2048, 3), (2560, 1), (151936, 2), (1000, 4), (151936, 1),
                                    (20000, 100), (16384, 150), (1000, 300), (40000, 160)])
def test_softmax_argmax(torch, R, C, rows):
    from nekochat_b200 import ops
    rng = np.random.default_rng(C + 1)
    x = (rng.standard_normal((rows, C)) * 4).astype(np.float32)
    x[0, C // 3] = x[0].max() + 1  # a clear winner
    if rows > 1:
        x[1, 5] = x[1, 9] = x[1].max() + 1  # tie: the first index wins (std::max_element)
    tx = torch.from_numpy(x).cuda()
    got = ops.softmax(tx).cpu().numpy()
    # against an fp64 softmax (tight), and against the oracle, whose sequential float sum over up to 152K terms
    # carries its own relative error of order 1e-4
    e = np.exp(x.astype(np.float64) - x.max(1, keepdims=True))
    close(got, (e / e.sum(1, keepdims=True)).astype(np.float32), 2e-6)
    d = np.abs(got - R.softmax_rows(x))
    assert np.all(d <= 1e-6 + 5e-4 * np.abs(got))
    am = ops.argmax(tx).cpu().numpy()
    assert [int(a) for a in am] == [R.argmax(r) for r in x]


@pytest.mark.parametrize("H,KV,hd,T,pos0", [(16, 8, 128, 1, 700), (4, 2, 64, 3, 1030), (12, 12, 64, 5, 0),
                                            (32, 8, 128, 1, 4000), (8, 8, 128, 64, 200), (32, 4, 128, 3, 63),
                                            (8, 1, 64, 2, 127), (4, 4, 32, 4, 90)])
def test_attention_op(torch, R, H, KV, hd, T, pos0):
    from nekochat_b200 import ops
    rng = np.random.default_rng(pos0 + T)
    ctx = pos0 + T
    stride = (H + 2 * KV) * hd
    q = rng.uniform(-1, 1, (T, stride)).astype(np.float32)
    kc = rng.uniform(-1, 1, (ctx, KV * hd)).astype(np.float16).view(np.uint16)
    vc = rng.uniform(-1, 1, (ctx, KV * hd)).astype(np.float16).view(np.uint16)
    ref = R.attention(q, stride, kc, vc, T, H, KV, hd, pos0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16) if a.dtype == np.uint16 else a).cuda()
    got = ops.attention(t(q), stride, t(kc), t(vc), T, H, KV, hd, pos0).cpu().numpy()
    close(got, ref, 2e-3)


SAMPLE_PARAMS = [(0.8, 40, 0.95, 1.1, 64), (1.0, 1, 1.0, 1.0, 0), (0.7, 1024, 0.9, 1.3, 32), (1.5, 0, 0.5, 1.0, 64),
                 (0.0, 40, 0.95, 1.1, 64)]


@pytest.mark.parametrize("params", SAMPLE_PARAMS)
@pytest.mark.parametrize("V", [1000, 151936])
def test_sample_matches_reference_sampler(torch, params, V):
    """neko_op_sample against the reference's own Sampler::sample (compiled from its sources) with the same
    seeds: the device takes each seed's uniform draw as input. Same token, same penalised logits."""
    import nekochat_b200 as nb
    from nekochat_b200 import ops
    from oracle.oracle import Reference
    R = Reference()
    rng = np.random.default_rng(V + params[1])
    rows, S = 4, 80
    x = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    hist = rng.integers(0, V, (rows, S)).astype(np.int32)
    hist[:, -3:] = np.argmax(x, axis=1)[:, None]  # the top token repeated: the penalty moves it
    hlen = np.array([S, 50, 10, 0], np.int32)
    seeds = [5000 + i for i in range(rows)]
    u = np.array([R.sampler_draw(sd) for sd in seeds])
    tx = torch.from_numpy(x.copy()).cuda()
    args = (torch.from_numpy(u).cuda(),) + params
    kw = dict(history=torch.from_numpy(hist).cuda(), hist_len=torch.from_numpy(hlen).cuda())
    if params[0] > 0 and (params[1] if params[1] > 0 else V) > 1024:
        with pytest.raises(nb.NekoError):
            ops.sample(tx, *args, **kw)
        return
    out = ops.sample(tx, *args, **kw).cpu().numpy()
    got_x = tx.cpu().numpy()
    for i in range(rows):
        want, px = R.sample(x[i], hist[i, :hlen[i]], *params, seeds[i])
        assert int(out[i]) == want, (i, params)
        np.testing.assert_array_equal(got_x[i], px)
