"""The ComputeBackend contract on CUDA: every case of the engine's own gpu::selfTest
(app/architecture/shared/cpp/gpu/compute.cpp:32-290), restated through the C ABI dispatch with the same shapes,
parameter blocks and tolerances (|gpu - cpu| <= tol * (1 + |cpu|)), the CPU side computed by the oracle.
When oracle/_ref/libneko_ref_cuda.so exists, the reference's own selfTest also runs unmodified on the backend.
"""
import math
import os

import numpy as np
import pytest

import nekochat_b200 as nb
from nekochat_b200 import Kernel, float_bits
from oracle.oracle import ACCUMULATE, FP4, FP8, F16, GELU, Restatement

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def close(a, b, tol):
    a, b = np.asarray(a, np.float32).reshape(-1), np.asarray(b, np.float32).reshape(-1)
    d = np.abs(a - b)
    bad = ~(d <= tol * (1 + np.abs(b)))
    assert not bad.any(), f"mismatch at {np.argmax(bad)}: gpu {a[np.argmax(bad)]} cpu {b[np.argmax(bad)]}"


@pytest.fixture(scope="module")
def be():
    b = nb.ComputeBackend(0)
    yield b
    b.close()


@pytest.fixture(scope="module")
def R():
    return Restatement()


@pytest.fixture()
def rnd():
    rng = np.random.default_rng(1234)
    return lambda *shape: rng.uniform(-1, 1, shape).astype(np.float32)


def halves(v):
    h = v.astype(np.float16)
    return h.view(np.uint16), h.astype(np.float32)


def test_name_and_device(be):
    assert be.name() == "CUDA"
    assert "sm_10" in be.device_name()
    assert be.max_buffer_bytes() > 100 << 30


def test_matmul_f16_bias_gelu_partial_tile(be, R, rnd):
    # compute.cpp:63-82: K=64, N=37, T=5, bias + gelu
    K, N, T = 64, 37, 5
    x, bias, wf = rnd(T, K), rnd(N), rnd(N, K)
    wh, wf = halves(wf)
    ref = np.array([[R.gelu(float(bias[n] + np.dot(x[t].astype(np.float64), wf[n]))) for n in range(N)]
                    for t in range(T)], np.float32)
    by = be.create(ref.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.Matmul, [be.create_from(x), be.create_from(wh), be.create_from(bias), by], [K, N, T, 4 | 1],
                N, (T + 3) // 4)
    be.submit_and_wait()
    close(be.download(by, 0, ref.nbytes), ref, 2e-3)


def test_matmul_768_rowoffset_accumulate_coloffset(be, rnd):
    # compute.cpp:84-104
    BK, BN, BT, row0, noff = 768, 96, 6, 1, 5
    NS = BN + 8
    bx, bb, bwf, y0 = rnd(BT + row0, BK), rnd(BN), rnd(BN, BK), rnd(BT, NS)
    bw, bwf = halves(bwf)
    ref = y0.copy()
    ref[:, noff:noff + BN] += (bx[row0:].astype(np.float64) @ bwf.T.astype(np.float64) + bb).astype(np.float32)
    by = be.create_from(y0, readback=True)
    be.begin()
    be.dispatch(Kernel.Matmul, [be.create_from(bx), be.create_from(bw), be.create_from(bb), by],
                [BK, NS, BT, 4 | 2, row0, noff], BN, (BT + 3) // 4)
    be.submit_and_wait()
    close(be.download(by, 0, y0.nbytes), ref, 2e-3)


def test_embed_plain_and_chunked(be, rnd):
    # compute.cpp:106-132
    EV, EC, EP, ET, epos, split = 10, 64, 4, 3, 1, 6
    hte, wte = halves(rnd(EV, EC))
    hpe, wpe = halves(rnd(EP, EC))
    toks = np.array([3, 7, 9], np.int32)
    ref = wte[toks] + wpe[epos:epos + ET]
    bt = be.create_from(toks)
    out = be.create(ref.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.Embed, [bt, be.create_from(hte), be.create_from(hpe), out], [ET, EC, epos, 1, 0, EV], 1, ET)
    be.submit_and_wait()
    close(be.download(out, 0, ref.nbytes), ref, 1e-5)
    c0, c1 = be.create_from(hte[:split]), be.create_from(hte[split:])
    be.begin()
    be.dispatch(Kernel.Embed, [bt, c0, None, out], [ET, EC, 0, 0, 0, split], 1, ET)
    be.dispatch(Kernel.Embed, [bt, c1, None, out], [ET, EC, 0, 0, split, EV - split], 1, ET)
    be.submit_and_wait()
    close(be.download(out, 0, ref.nbytes), wte[toks], 1e-5)


def test_layernorm_rmsnorm_and_chained_matmul(be, R, rnd):
    # compute.cpp:134-176 (the chained case catches missing ordering between dispatches)
    C, Rn = 96, 3
    lx, g, b = rnd(C * Rn) * 20, rnd(C), rnd(C)
    lref, rref = R.layer_norm(lx.reshape(Rn, C), g, b, 1e-5), R.rms_norm(lx.reshape(Rn, C), g, 1e-6)
    blx, bg, bbb = be.create_from(lx), be.create_from(g), be.create_from(b)
    bly = be.create(lx.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.LayerNorm, [blx, bly, bg, bbb], [C, float_bits(1e-5), 0, 0], Rn, 1)
    be.submit_and_wait()
    close(be.download(bly, 0, lx.nbytes), lref, 1e-3)
    be.begin()
    be.dispatch(Kernel.LayerNorm, [blx, bly, bg, None], [C, float_bits(1e-6), 0, 1], Rn, 1)
    be.submit_and_wait()
    close(be.download(bly, 0, lx.nbytes), rref, 1e-3)
    CN = 3072
    chw, cw = halves(rnd(CN, C))
    cref = (lref.astype(np.float64) @ cw.T.astype(np.float64)).astype(np.float32)
    bcy, bln = be.create(cref.nbytes, readback=True), be.create(lx.nbytes)
    be.begin()
    be.dispatch(Kernel.LayerNorm, [blx, bln, bg, bbb], [C, float_bits(1e-5), 0, 0], Rn, 1)
    be.dispatch(Kernel.Matmul, [bln, be.create_from(chw), None, bcy], [C, CN, Rn, 0], CN, 1)
    be.submit_and_wait()
    close(be.download(bcy, 0, cref.nbytes), cref, 5e-3)


def test_layernorm_row_offset(be, R, rnd):
    # the final norm runs on the last row only (qwen3_model.cpp:337: rowOffset = T - 1)
    C, T = 1024, 5
    x, g = rnd(T, C) * 3, rnd(C)
    by = be.create(C * 4, readback=True)
    be.begin()
    be.dispatch(Kernel.LayerNorm, [be.create_from(x), by, be.create_from(g), None], [C, float_bits(1e-6), T - 1, 1], 1, 1)
    be.submit_and_wait()
    close(be.download(by, 0, C * 4), R.rms_norm(x[T - 1:], g, 1e-6), 1e-3)


def test_qk_norm_rope(be, R, rnd):
    # compute.cpp:178-202
    H, KV, hd, T, pos0 = 2, 1, 64, 2, 3
    stride = (H + 2 * KV) * hd
    qkv, wn = rnd(T, stride), rnd(2 * hd)
    cs = np.zeros(((pos0 + T), hd), np.float32)
    for p in range(pos0 + T):
        for i in range(hd // 2):
            a = p * math.pow(10000.0, -2.0 * i / hd)
            cs[p, 2 * i], cs[p, 2 * i + 1] = math.cos(a), math.sin(a)
    ref = qkv.copy()
    for t in range(T):
        r = ref[t]
        r[:H * hd] = R.rms_norm(r[:H * hd].reshape(H, hd), wn[:hd], 1e-6).reshape(-1)
        r[H * hd:(H + KV) * hd] = R.rms_norm(r[H * hd:(H + KV) * hd].reshape(KV, hd), wn[hd:], 1e-6).reshape(-1)
        R.rope(r, H + KV, hd, cs[pos0 + t])
    bq = be.create_from(qkv, readback=True)
    be.begin()
    be.dispatch(Kernel.Rope, [bq, be.create_from(wn), be.create_from(cs)], [stride, H, hd, pos0, float_bits(1e-6), 1],
                H + KV, T)
    be.submit_and_wait()
    close(be.download(bq, 0, qkv.nbytes), ref, 1e-3)


def test_swiglu(be, R, rnd):
    # compute.cpp:204-216
    T, I = 2, 100
    h = rnd(T, 2 * I) * 6
    ref = R.silu_mul(h, I)
    bo = be.create(ref.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.SiluMul, [be.create_from(h), bo], [T, I], (I + 63) // 64, T)
    be.submit_and_wait()
    close(be.download(bo, 0, ref.nbytes), ref, 1e-4)


@pytest.mark.parametrize("fmt,kernel", [(FP8, Kernel.MatmulQ8), (FP4, Kernel.MatmulQ4)])
@pytest.mark.parametrize("K", [96, 1024])
def test_quantized_matmul_bias_accumulate_offset(be, R, rnd, fmt, kernel, K):
    # compute.cpp:218-244
    N, T, noff = 37, 5, 3
    NS = N + 5
    x, bias, wf, y0 = rnd(T, K), rnd(N), rnd(N, K), rnd(T, NS)
    q = R.quantize(fmt, wf)
    ref = R.matmul(fmt, x, q, K, bias, y0.copy(), NS, ACCUMULATE, noff)
    by = be.create_from(y0, readback=True)
    be.begin()
    be.dispatch(kernel, [be.create_from(x), be.create_from(q), be.create_from(bias), by], [K, NS, T, 4 | 2, 0, noff], N,
                (T + 3) // 4)
    be.submit_and_wait()
    close(be.download(by, 0, y0.nbytes), ref, 2e-3)


@pytest.mark.parametrize("fmt", [FP8, FP4])
def test_quantized_embed(be, R, rnd, fmt):
    # compute.cpp:245-259
    EV, EC, ET = 10, 64, 3
    q = R.quantize(fmt, rnd(EV, EC))
    toks = np.array([3, 7, 9], np.int32)
    ref = R.dequantize(fmt, q, EC)[toks]
    out = be.create(ref.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.Embed, [be.create_from(toks), be.create_from(q), None, out],
                [ET, EC, 0, 2 if fmt == FP8 else 4, 0, EV, q.shape[1] // 4], 1, ET)
    be.submit_and_wait()
    got = be.download(out, 0, ref.nbytes)
    assert np.array_equal(got.view(np.uint32), ref.reshape(-1).view(np.uint32))  # exact dequant


def test_kvstore_attention_crossing_1024(be, R):
    # compute.cpp:262-284: pos0 = 1030 crosses the shaders' 1024-key tile
    from tests.golden.make_golden import attention_case
    H, KV, hd, T, pos0, qkv, kc, vc = attention_case()
    stride, kvW, kOff, vOff = (H + 2 * KV) * hd, KV * hd, H * hd, (H + KV) * hd
    kcr, vcr = kc.copy(), vc.copy()
    R.store_kv(qkv[:, kOff:], qkv[:, vOff:], stride, kcr, vcr, kvW, T, pos0)
    ref = R.attention(qkv, stride, kcr, vcr, T, H, KV, hd, pos0)
    bq, bk, bv = be.create_from(qkv), be.create_from(kc, True), be.create_from(vc, True)
    bo = be.create(ref.nbytes, readback=True)
    be.begin()
    be.dispatch(Kernel.KvStore, [bq, bk, bv], [T, kvW, pos0, 0, stride, kOff, vOff], (kvW // 2 + 63) // 64, T)
    be.dispatch(Kernel.Attention, [bq, bk, bv, bo], [T, stride, H, pos0, hd, float_bits(1 / math.sqrt(hd)), kvW], H, T)
    be.submit_and_wait()
    close(be.download(bo, 0, ref.nbytes), ref, 2e-3)
    got_k = be.download(bk, 0, kc.nbytes, np.uint16).reshape(kc.shape)
    assert np.array_equal(got_k, kcr)  # f16 round-to-nearest-even, bit-exact
    assert np.array_equal(be.download(bv, 0, vc.nbytes, np.uint16).reshape(vc.shape), vcr)


def test_dispatch_rejects_bad_sizes(be, rnd):
    """Out-of-range bindings fail like the engine's fail(): an exception, no launch."""
    x = be.create_from(rnd(4, 64))
    with pytest.raises(nb.NekoError):
        be.dispatch(Kernel.MatmulQ8, [x, be.create(16), None, be.create(64)], [64, 8, 4, 0], 8, 1)
    with pytest.raises(nb.NekoError):
        be.dispatch(99, [x, None, None, None], [0] * 8, 1, 1)


REF_CUDA = os.path.join(ROOT, "oracle", "_ref", "libneko_ref_cuda.so")


@pytest.mark.skipif(not os.path.exists(REF_CUDA), reason="reference engine with the CUDA backend not built")
def test_reference_selftest_unmodified():
    """gpu::selfTest (compute.cpp:32) of the reference engine, compiled from its sources, on CudaBackend."""
    from oracle.oracle import Reference
    rc, msg = Reference(cuda=True).selftest_cuda()
    assert rc == 0, msg
