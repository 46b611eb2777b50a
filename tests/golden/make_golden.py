"""Generates the golden fixtures in this folder by running the reference engine itself.

The reference publishes no golden vectors for its hot path, so these are produced from its own C++ CPU code,
compiled from its sources by oracle/Makefile into oracle/_ref/libneko_ref.so (built without FMA contraction).
Each fixture stores seeded inputs and the reference's outputs; tests/test_oracle.py checks the restatement in
oracle/neko_oracle.c against them bit for bit, and the GPU parity tests reuse the inputs.

Run from the repository root after `make -C oracle`:  python tests/golden/make_golden.py
"""
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.checkpoint import write_model, write_safetensors  # noqa: E402
from oracle.oracle import ACCUMULATE, FP4, FP8, F16, GELU, Reference  # noqa: E402
from nekochat_b200 import workload  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def codec(ref):
    """quantizeMatrix / dequantizeRow (quant.cpp:255-279, 230-253) on awkward blocks."""
    rng = np.random.default_rng(11)
    out = {}
    for fmt, tag in ((FP8, "fp8"), (FP4, "fp4")):
        w = (rng.standard_normal((24, 96)) * 0.05).astype(np.float32)
        w[0, :32] = 0.0                                # all-zero block -> scale 0
        w[1, 5] = 1.5                                  # outlier
        w[2, :] = np.linspace(-3, 3, 96, dtype=np.float32)
        w[3, 7] = -70000.0                             # beyond f16 range after scaling
        w[4, :32] = np.float32(1e-7)                   # f16-subnormal scale
        w[5, :] = np.float32(448.0) * np.sign(w[5, :])  # exact max code
        w[6, 0:32] = np.float32(6.0)                   # FP4 max exactly
        w[7, 1::2] = -w[7, 1::2] * 40                  # mixed magnitudes
        w[8, :] = np.float32(0.25)                     # FP4 rounding tie (0.25 * scale)
        w[9, 3] = np.float32(-0.0)
        q = ref.quantize(fmt, w)
        out[f"{tag}_w"] = w
        out[f"{tag}_q"] = q
        out[f"{tag}_deq"] = ref.dequantize(fmt, q, 96)
        # all 256 codes of one FP8 block / all 16 nibbles of FP4, decoded by the reference
        raw = np.zeros((8, ref.row_bytes(fmt, 256)), np.uint8)
        nb = 256 if fmt == FP8 else 128
        raw[:, :nb] = np.arange(nb * 8, dtype=np.int64).reshape(8, nb).astype(np.uint8)
        scales = np.array([0x3C00, 0x3800, 0x0001, 0x7BFF, 0x2E66, 0x0400, 0x3555, 0x4000], np.uint16)  # f16
        sv = raw[:, nb:nb + 16].view(np.uint16)
        sv[:, :8] = scales
        raw_deq = ref.dequantize(fmt, raw, 256)
        out[f"{tag}_raw"] = raw
        out[f"{tag}_raw_deq"] = raw_deq
    return out


def attention_case():
    """The self-test's attention shape (compute.cpp:262-268): H=4, KV=2, hd=64, T=3 new tokens at pos0=1030,
    f16 caches of uniform(-1, 1) values from default_rng(1030)."""
    H, KV, hd, T, pos0 = 4, 2, 64, 3, 1030
    rng = np.random.default_rng(1030)
    qkv = rng.uniform(-1, 1, (T, (H + 2 * KV) * hd)).astype(np.float32)
    kc = rng.uniform(-1, 1, (pos0 + T, KV * hd)).astype(np.float16).view(np.uint16)
    vc = rng.uniform(-1, 1, (pos0 + T, KV * hd)).astype(np.float16).view(np.uint16)
    return H, KV, hd, T, pos0, qkv, kc, vc


def ops(ref):
    """cpu::matmul, layerNorm, rmsNorm, rope, siluMul, gelu, storeKv, attention (cpu_ops.cpp)."""
    rng = np.random.default_rng(12)
    out = {}
    for fmt, tag in ((FP8, "fp8"), (FP4, "fp4")):
        for K in (96, 1024):
            N, T, noff = 37, 5, 3
            NS = N + 5
            w = rng.uniform(-1, 1, (N, K)).astype(np.float32)
            x = rng.uniform(-1, 1, (T, K)).astype(np.float32)
            b = rng.uniform(-1, 1, N).astype(np.float32)
            y0 = rng.uniform(-1, 1, (T, NS)).astype(np.float32)
            q = ref.quantize(fmt, w)
            y = ref.matmul(fmt, x, q, K, b, y0.copy(), NS, ACCUMULATE, noff)
            yg = ref.matmul(fmt, x, q, K, b, None, None, GELU)
            out.update({f"mm_{tag}_{K}_q": q, f"mm_{tag}_{K}_x": x, f"mm_{tag}_{K}_b": b, f"mm_{tag}_{K}_y0": y0,
                        f"mm_{tag}_{K}_y": y, f"mm_{tag}_{K}_ygelu": yg})
    # F16 weights (matmulF16 path)
    w = rng.uniform(-1, 1, (37, 64)).astype(np.float32)
    h = w.astype(np.float16).view(np.uint16).view(np.uint8).reshape(37, 128)
    x = rng.uniform(-1, 1, (5, 64)).astype(np.float32)
    b = rng.uniform(-1, 1, 37).astype(np.float32)
    out.update(mm_f16_q=h, mm_f16_x=x, mm_f16_b=b, mm_f16_y=ref.matmul(F16, x, h, 64, b, None, None, GELU))
    # norms
    x = (rng.uniform(-1, 1, (3, 96)) * 20).astype(np.float32)
    g = rng.uniform(-1, 1, 96).astype(np.float32)
    bb = rng.uniform(-1, 1, 96).astype(np.float32)
    out.update(norm_x=x, norm_g=g, norm_b=bb, ln_y=ref.layer_norm(x, g, bb, 1e-5), rms_y=ref.rms_norm(x, g, 1e-6))
    # rope (table rows as the self-test builds them, compute.cpp:182-188)
    hd, nh = 64, 3
    v = rng.uniform(-1, 1, nh * hd).astype(np.float32)
    i = np.arange(hd // 2)
    a = 5 * np.power(10000.0, -2.0 * i / hd)
    cs = np.stack([np.cos(a), np.sin(a)], 1).reshape(-1).astype(np.float32)
    r = v.copy()
    ref.rope(r, nh, hd, cs)
    out.update(rope_x=v, rope_cs=cs, rope_y=r)
    hh = (rng.uniform(-1, 1, (2, 200)) * 6).astype(np.float32)
    out.update(silu_h=hh, silu_y=ref.silu_mul(hh, 100))
    gx = (rng.standard_normal(64) * 4).astype(np.float32)
    out.update(gelu_x=gx, gelu_y=np.array([ref.gelu(float(t)) for t in gx], np.float32))
    # kv store + attention at pos0 = 1030 (compute.cpp:262-284); the caches are regenerated by
    # attention_case() in the tests, so only the stored rows and the output are kept
    H, KV, hd, T, pos0, qkv, kc, vc = attention_case()
    stride, kvW = (H + 2 * KV) * hd, KV * hd
    kc2, vc2 = kc.copy(), vc.copy()
    ref.store_kv(qkv[:, H * hd:], qkv[:, (H + KV) * hd:], stride, kc2, vc2, kvW, T, pos0)
    att = ref.attention(qkv, stride, kc2, vc2, T, H, KV, hd, pos0)
    out.update(att_k_new=kc2[pos0:pos0 + T], att_v_new=vc2[pos0:pos0 + T], att_y=att)
    return out


def models(ref, tmp):
    """Tiny GPT-2 / Qwen3 through loadModel + Model::forward on the CPU backend (model.cpp:187-193)."""
    out = {}
    for name, fmt, tag in (("qwen3-tiny", FP8, "qwen3_fp8"), ("qwen3-tiny", FP4, "qwen3_fp4"),
                           ("gpt2-tiny", FP8, "gpt2_fp8")):
        s = workload.shape(name)
        folder = write_model(os.path.join(tmp, tag), s, workload.weights(s, seed=0, perturb=True))
        m = ref.load_model(folder, fmt, threads=1)
        prompt = workload.prompt(s, 9)
        logits = [m.forward(prompt[:8], 0)]
        toks = []
        nxt = int(np.argmax(logits[-1]))
        pos = 8
        for _ in range(4):  # greedy continuation, one token per forward (Engine::generate decode loop)
            toks.append(nxt)
            logits.append(m.forward(np.array([nxt], np.int32), pos))
            pos += 1
            nxt = int(np.argmax(logits[-1]))
        m.close()
        out[f"{tag}_prompt"] = prompt[:8]
        out[f"{tag}_tokens"] = np.array(toks, np.int32)
        out[f"{tag}_logits"] = np.stack(logits)
    return out


# (rows, cols), scale shape: 128 x 128 blocks with ragged edges, an even split, a per-tensor 0-d scale, a 1-D
# scale (rows only), more scale rows than weight rows, a 1 x 1 scale, odd columns
FP8CKPT_CASES = (((136, 260), (2, 3)), ((96, 64), (4, 2)), ((40, 33), ()), ((140, 40), (2,)), ((10, 24), (20, 3)),
                 ((8, 32), (1, 1)), ((129, 7), (2, 1)))


def fp8ckpt(ref, tmp):
    """FP8 (E4M3) checkpoint weights as the reference loader reads them (TensorStore::toF32 through
    tensor_store.cpp:543-571), from safetensors files with F8_E4M3 weights and f32 "_scale_inv" tensors. Every
    case holds all 256 codes."""
    rng = np.random.default_rng(29)
    out = {}
    for i, ((R, Cn), sh) in enumerate(FP8CKPT_CASES):
        codes = rng.integers(0, 256, (R, Cn), dtype=np.uint8)
        codes.flat[:256] = np.arange(256, dtype=np.uint8)[:codes.size]
        sc = (rng.random(sh) * 0.01 + 1e-4).astype(np.float32) if sh else np.float32(0.0137)
        path = os.path.join(tmp, f"fp8_{i}.safetensors")
        write_safetensors(path, [("w.weight", codes, "F8_E4M3"), ("w.weight_scale_inv", np.asarray(sc, np.float32))])
        out[f"c{i}_codes"] = codes
        out[f"c{i}_scales"] = np.asarray(sc, np.float32)
        out[f"c{i}_f32"] = ref.tensor_f32(path, "w.weight", R * Cn).reshape(R, Cn)
    return out


def main(which=("codec", "ops", "models", "fp8ckpt")):
    """Writes the named fixtures (all by default): python tests/golden/make_golden.py [name ...]"""
    ref = Reference()
    if "codec" in which:
        np.savez_compressed(os.path.join(HERE, "codec.npz"), **codec(ref))
    if "ops" in which:
        np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops(ref))
    with tempfile.TemporaryDirectory() as tmp:
        if "models" in which:
            np.savez_compressed(os.path.join(HERE, "models.npz"), **models(ref, tmp))
        if "fp8ckpt" in which:
            np.savez_compressed(os.path.join(HERE, "fp8ckpt.npz"), **fp8ckpt(ref, tmp))
    for f in which:
        print(f + ".npz", os.path.getsize(os.path.join(HERE, f + ".npz")))


if __name__ == "__main__":
    main(tuple(sys.argv[1:]) or ("codec", "ops", "models", "fp8ckpt"))
