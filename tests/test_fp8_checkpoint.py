"""FP8 (E4M3) checkpoint weights (Qwen3-*-FP8): the restatement of the reference loader's dequantization
(TensorStore::rows, tensor_store.cpp:543-571) against golden vectors from the reference's own TensorStore, and,
where the compiled reference is present, against it live on fresh files."""
import os
import tempfile

import numpy as np
import pytest

from oracle.checkpoint import e4m3fn_table, fp8_block_dequant, fp8_block_of, write_safetensors

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REF_SO = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libneko_ref.so")


def cases():
    g = np.load(os.path.join(GOLD, "fp8ckpt.npz"))
    n = len([k for k in g.files if k.endswith("_codes")])
    return [(g[f"c{i}_codes"], g[f"c{i}_scales"], g[f"c{i}_f32"]) for i in range(n)]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_table_known_values():
    t = e4m3fn_table()
    assert t[0x00] == 0.0 and np.signbit(t[0x80])
    assert t[0x38] == 1.0 and t[0xB8] == -1.0       # e = 7, m = 0
    assert t[0x01] == 2.0 ** -9                      # smallest subnormal
    assert t[0x08] == 2.0 ** -6                      # smallest normal
    assert t[0x7E] == 448.0 and t[0x7F] == 480.0     # no NaN code in the reference's table
    assert t[0xFF] == -480.0


def test_block_lengths():
    assert fp8_block_of(300, 3) == 128   # ceil(300 / 128) scales: 128-element blocks, ragged last one
    assert fp8_block_of(96, 4) == 24     # otherwise the shape split evenly
    assert fp8_block_of(10, 20) == 1
    assert fp8_block_of(77, 1) == 77     # one scale: the whole axis


def test_restatement_matches_reference_golden():
    for codes, scales, want in cases():
        assert np.array_equal(bits(fp8_block_dequant(codes, scales)), bits(want))


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="compiled reference (oracle/_ref) not built")
def test_restatement_matches_reference_live():
    from oracle.oracle import Reference
    ref = Reference()
    rng = np.random.default_rng(41)
    with tempfile.TemporaryDirectory() as d:
        for (R, Cn), sh, sdt in (((257, 130), (3, 2), np.float32), ((64, 200), (1, 2), np.float32),
                                 ((33, 17), (33, 17), np.float32), ((50, 40), (), np.float16)):
            codes = rng.integers(0, 256, (R, Cn), dtype=np.uint8)
            sc = (rng.random(sh) * 0.02 + 1e-3).astype(sdt) if sh else np.asarray(0.0071, sdt)
            p = os.path.join(d, "w.safetensors")
            write_safetensors(p, [("m.weight", codes, "F8_E4M3"), ("m.weight_scale", sc)])
            got = ref.tensor_f32(p, "m.weight", R * Cn).reshape(R, Cn)
            assert np.array_equal(bits(fp8_block_dequant(codes, sc.astype(np.float32))), bits(got))
