"""Model shapes and seeded synthetic weights/prompts for the benchmark configurations.

No checkpoints or datasets exist on the GPU box, so every run uses random-init weights of the named
architecture: N(0, 0.02) from numpy ``default_rng(seed)`` (PCG64) drawn in the fixed tensor order of
:func:`tensor_specs`, norm gains 1, norm biases and linear biases 0; prompts are token ids uniform in [0, vocab)
from ``default_rng(1)``. Shapes follow the HF configs the engine reads (gpt2_model.cpp:17-32,
qwen3_model.cpp:16-40).
"""
import numpy as np

SHAPES = {
    # GPT-2 small (the CPU-runnable benchmark configuration)
    "gpt2": dict(arch="gpt2", vocab=50257, embd=768, layers=12, heads=12, kv_heads=12, head_dim=64, ff=3072,
                 max_pos=1024, eps=1e-5, rope_theta=0.0),
    # Qwen3 shapes (the other benchmark configurations)
    "qwen3-0.6b": dict(arch="qwen3", vocab=151936, embd=1024, layers=28, heads=16, kv_heads=8, head_dim=128,
                       ff=3072, max_pos=40960, eps=1e-6, rope_theta=1e6),
    "qwen3-1.7b": dict(arch="qwen3", vocab=151936, embd=2048, layers=28, heads=16, kv_heads=8, head_dim=128,
                       ff=6144, max_pos=40960, eps=1e-6, rope_theta=1e6),
    "qwen3-4b": dict(arch="qwen3", vocab=151936, embd=2560, layers=36, heads=32, kv_heads=8, head_dim=128,
                     ff=9728, max_pos=40960, eps=1e-6, rope_theta=1e6),
    # small shapes for parity tests (same code paths, oracle-sized)
    "qwen3-tiny": dict(arch="qwen3", vocab=1000, embd=256, layers=2, heads=4, kv_heads=2, head_dim=64, ff=512,
                       max_pos=4096, eps=1e-6, rope_theta=1e6),
    "gpt2-tiny": dict(arch="gpt2", vocab=1000, embd=128, layers=2, heads=4, kv_heads=4, head_dim=32, ff=512,
                      max_pos=256, eps=1e-5, rope_theta=0.0),
}


def shape(name):
    return dict(SHAPES[name])


def tensor_specs(s):
    """[(checkpoint name, shape, kind)] in generation order; kind is 'w' (N(0, 0.02)), 'g' (ones) or 'b' (zeros).
    Names are the HF checkpoint names the engine loads (prefix-less)."""
    C, V, L = s["embd"], s["vocab"], s["layers"]
    out = []
    if s["arch"] == "qwen3":
        H, KV, hd, F = s["heads"], s["kv_heads"], s["head_dim"], s["ff"]
        out.append(("embed_tokens.weight", (V, C), "w"))
        for l in range(L):
            p = f"layers.{l}."
            out += [(p + "input_layernorm.weight", (C,), "g"),
                    (p + "self_attn.q_proj.weight", (H * hd, C), "w"),
                    (p + "self_attn.k_proj.weight", (KV * hd, C), "w"),
                    (p + "self_attn.v_proj.weight", (KV * hd, C), "w"),
                    (p + "self_attn.o_proj.weight", (C, H * hd), "w"),
                    (p + "self_attn.q_norm.weight", (hd,), "g"),
                    (p + "self_attn.k_norm.weight", (hd,), "g"),
                    (p + "post_attention_layernorm.weight", (C,), "g"),
                    (p + "mlp.gate_proj.weight", (F, C), "w"),
                    (p + "mlp.up_proj.weight", (F, C), "w"),
                    (p + "mlp.down_proj.weight", (C, F), "w")]
        out.append(("norm.weight", (C,), "g"))
    else:
        F, P = s["ff"], s["max_pos"]
        out += [("wte.weight", (V, C), "w"), ("wpe.weight", (P, C), "w")]
        for l in range(L):
            p = f"h.{l}."
            out += [(p + "ln_1.weight", (C,), "g"), (p + "ln_1.bias", (C,), "b"),
                    (p + "attn.c_attn.weight", (C, 3 * C), "w"), (p + "attn.c_attn.bias", (3 * C,), "b"),
                    (p + "attn.c_proj.weight", (C, C), "w"), (p + "attn.c_proj.bias", (C,), "b"),
                    (p + "ln_2.weight", (C,), "g"), (p + "ln_2.bias", (C,), "b"),
                    (p + "mlp.c_fc.weight", (C, F), "w"), (p + "mlp.c_fc.bias", (F,), "b"),
                    (p + "mlp.c_proj.weight", (F, C), "w"), (p + "mlp.c_proj.bias", (C,), "b")]
        out += [("ln_f.weight", (C,), "g"), ("ln_f.bias", (C,), "b")]
    return out


def weights(s, seed=0, perturb=False):
    """Yields (name, float32 array) in generation order. perturb=True also randomises norm gains (1 + N(0, 0.1))
    and biases (N(0, 0.02)) so parity tests exercise those code paths."""
    rng = np.random.default_rng(seed)
    for name, shp, kind in tensor_specs(s):
        if kind == "w":
            a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        elif kind == "g":
            a = np.ones(shp, np.float32)
            if perturb:
                a += rng.standard_normal(shp, dtype=np.float32) * np.float32(0.1)
        else:
            a = np.zeros(shp, np.float32)
            if perturb:
                a += rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        yield name, a


def prompt(s, n, seed=1):
    return np.random.default_rng(seed).integers(0, s["vocab"], size=n, dtype=np.int64).astype(np.int32)


def row_bytes(fmt, cols):
    """quantRowBytes (quant.cpp:199-208): codes, then cols/32 f16 scales padded to 16 bytes."""
    scales = (cols // 32 * 2 + 15) // 16 * 16
    return 2 * cols if fmt == 0 else (cols + scales if fmt == 1 else cols // 2 + scales)


def param_count(s):
    return sum(int(np.prod(shp)) for _, shp, _ in tensor_specs(s))


def weight_stream_bytes(s, fmt):
    """Packed weight bytes one decode step streams from HBM: every layer matrix plus the tied LM head
    (the embedding gather reads one row per token)."""
    C, L = s["embd"], s["layers"]
    if s["arch"] == "qwen3":
        H, KV, hd, F = s["heads"], s["kv_heads"], s["head_dim"], s["ff"]
        per = ((H + 2 * KV) * hd * row_bytes(fmt, C) + C * row_bytes(fmt, H * hd) + 2 * F * row_bytes(fmt, C)
               + C * row_bytes(fmt, F))
    else:
        F = s["ff"]
        per = 3 * C * row_bytes(fmt, C) + C * row_bytes(fmt, C) + F * row_bytes(fmt, C) + C * row_bytes(fmt, F)
    return L * per + s["vocab"] * row_bytes(fmt, C)


def kv_bytes_per_position(s):
    """f16 K and V bytes of one cached position across all layers (Model kvBytesPerToken_)."""
    return s["layers"] * 2 * s["kv_heads"] * s["head_dim"] * 2
