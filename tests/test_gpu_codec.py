"""GPU weight codec: the on-device quantizer must be byte-identical to the engine's quantizeMatrix
(quant.cpp:255-279) and the device dequant bit-exact to QMatrix::dequantizeRow (quant.cpp:230-253)."""
import os

import numpy as np
import pytest

from oracle.oracle import FP4, FP8, F16, Restatement

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    return t


@pytest.fixture(scope="module")
def R():
    return Restatement()


def gpu_quant(torch, fmt, w, transpose=False):
    from nekochat_b200 import ops
    q = ops.quantize(fmt, torch.from_numpy(np.ascontiguousarray(w)).cuda(), transpose_f16=transpose)
    torch.cuda.synchronize()
    return q.cpu().numpy()


@pytest.mark.parametrize("tag,fmt", [("fp8", FP8), ("fp4", FP4)])
def test_quantize_golden(torch, tag, fmt):
    c = np.load(os.path.join(GOLD, "codec.npz"))
    assert np.array_equal(gpu_quant(torch, fmt, c[f"{tag}_w"]), c[f"{tag}_q"])


@pytest.mark.parametrize("tag,fmt", [("fp8", FP8), ("fp4", FP4)])
def test_dequantize_golden_all_codes(torch, tag, fmt):
    from nekochat_b200 import ops
    c = np.load(os.path.join(GOLD, "codec.npz"))
    for key, cols in ((f"{tag}_q", 96), (f"{tag}_raw", 256)):
        d = ops.dequantize(fmt, torch.from_numpy(c[key]).cuda(), cols).cpu().numpy()
        want = c[f"{tag}_deq"] if key.endswith("_q") else c[f"{tag}_raw_deq"]
        assert np.array_equal(d.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", [FP8, FP4])
@pytest.mark.parametrize("rows,cols,scale", [(4096, 1024, 0.02), (300, 3072, 1.0), (33, 96, 1e3), (64, 2560, 1e-5)])
def test_quantize_random_matches_oracle(torch, R, fmt, rows, cols, scale):
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    w[0, :17] = 0.0
    q = gpu_quant(torch, fmt, w)
    assert np.array_equal(q, R.quantize(fmt, w))
    from nekochat_b200 import ops
    d = ops.dequantize(fmt, torch.from_numpy(q).cuda(), cols).cpu().numpy()
    assert np.array_equal(d.view(np.uint32), R.dequantize(fmt, q, cols).view(np.uint32))


@pytest.mark.parametrize("fmt", [FP8, FP4, F16])
def test_conv1d_transpose_path(torch, R, fmt):
    """GPT-2 Conv1D weights [in][out] -> [out][in] through f16 (gpt2_model.cpp:78-82) before quantizing."""
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((128, 384)) * 0.02).astype(np.float32)  # [in=C][out=3C]
    q = gpu_quant(torch, fmt, w, transpose=True)
    want = R.quantize(fmt, np.ascontiguousarray(w.T).astype(np.float16).astype(np.float32))
    assert np.array_equal(q, want)


def test_fp8_checkpoint_dequant_golden(torch):
    """neko_op_fp8_block_dequant bit-exact to the reference loader's TensorStore::toF32 (tensor_store.cpp:543-571)
    on every golden case, through the four-codes-per-thread path and, with codes one byte off alignment, the
    scalar one."""
    from nekochat_b200 import ops
    g = np.load(os.path.join(GOLD, "fp8ckpt.npz"))
    n = len([k for k in g.files if k.endswith("_codes")])
    for i in range(n):
        codes, sc, want = g[f"c{i}_codes"], g[f"c{i}_scales"], g[f"c{i}_f32"]
        d_sc = torch.from_numpy(np.ascontiguousarray(sc)).cuda()
        got = ops.fp8_block_dequant(torch.from_numpy(codes).cuda(), d_sc).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"case {i}"
        buf = torch.zeros(codes.size + 1, dtype=torch.uint8, device="cuda")
        buf[1:] = torch.from_numpy(codes.ravel()).cuda()
        got = ops.fp8_block_dequant(buf[1:].view(codes.shape), d_sc).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"case {i}, unaligned codes"
