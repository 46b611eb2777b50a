"""Writes a synthetic model folder (config.json + model.safetensors) that the reference engine's loader reads
(TensorStore::loadSafetensors, app/architecture/shared/cpp/tensor_store.cpp:98-119; config keys of
gpt2_model.cpp:17-32 and qwen3_model.cpp:16-40). TEST INFRASTRUCTURE ONLY: it feeds the compiled reference
(oracle/_ref) the same seeded weights the B200 runner gets."""
import json
import os
import struct

import numpy as np

_DT = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}


def write_safetensors(path, tensors):
    """tensors: list of (name, array) or (name, array, dtype tag). Arrays are written as stored (F32 or F16);
    a tag names the stored type of raw bytes, e.g. (name, uint8 codes, "F8_E4M3") for an FP8 checkpoint weight."""
    header, blobs, off = {}, [], 0
    for item in tensors:
        name, a = item[0], np.ascontiguousarray(item[1])
        tag = item[2] if len(item) > 2 else _DT[a.dtype]
        header[name] = {"dtype": tag, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a)
        off += a.nbytes
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for a in blobs:
            f.write(a.tobytes())


def config_json(s):
    if s["arch"] == "qwen3":
        return {"model_type": "qwen3", "architectures": ["Qwen3ForCausalLM"], "vocab_size": s["vocab"],
                "max_position_embeddings": s["max_pos"], "hidden_size": s["embd"],
                "num_hidden_layers": s["layers"], "num_attention_heads": s["heads"],
                "num_key_value_heads": s["kv_heads"], "head_dim": s["head_dim"], "intermediate_size": s["ff"],
                "rms_norm_eps": s["eps"], "rope_theta": s["rope_theta"], "tie_word_embeddings": True,
                "attention_bias": False}
    return {"model_type": "gpt2", "architectures": ["GPT2LMHeadModel"], "vocab_size": s["vocab"],
            "n_positions": s["max_pos"], "n_embd": s["embd"], "n_layer": s["layers"], "n_head": s["heads"],
            "layer_norm_epsilon": s["eps"]}


def write_model(folder, s, tensors, dtype=np.float32):
    """tensors: iterable of (prefix-less name, float32 array). Qwen3 names get the HF "model." prefix."""
    os.makedirs(folder, exist_ok=True)
    pre = "model." if s["arch"] == "qwen3" else ""
    items = [(pre + n, np.asarray(a, dtype=dtype)) for n, a in tensors]
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(config_json(s), f)
    write_safetensors(os.path.join(folder, "model.safetensors"), items)
    return folder


def e4m3fn_table():
    """The reference's FP8 checkpoint decode table (tensor_store.cpp:558-563): OCP E4M3, bias 7, no infinities
    and no NaN code (0x7F / 0xFF give +-480); code 0x80 is -0.0."""
    c = np.arange(256)
    e, m = (c >> 3) & 15, c & 7
    mag = np.where(e == 0, np.ldexp(m / 8.0, -6), np.ldexp(1.0 + m / 8.0, e - 7)).astype(np.float32)
    return np.where(c & 0x80, -mag, mag).astype(np.float32)


def fp8_block_of(n, parts):
    """Block length along an axis of n elements with `parts` scales (tensor_store.cpp:550-554)."""
    if parts <= 1:
        return n
    if (n + 127) // 128 == parts:
        return 128
    return (n + parts - 1) // parts


def fp8_block_dequant(codes, scales):
    """TensorStore::rows for an F8_E4M3 weight (tensor_store.cpp:543-571): table[code] * scale of its block, one
    f32 multiply. codes uint8 [R][C]; scales as stored (0-d, [sR] or [sR][sC])."""
    codes = np.asarray(codes, np.uint8)
    s = np.asarray(scales, np.float32)
    sR = s.shape[0] if s.ndim >= 1 else 1
    sC = s.shape[1] if s.ndim >= 2 else 1
    s = s.reshape(sR, sC)
    R, Cn = codes.shape
    bR, bC = fp8_block_of(R, sR), fp8_block_of(Cn, sC)
    ri, ci = np.arange(R) // bR, np.arange(Cn) // bC
    return (e4m3fn_table()[codes] * s[ri][:, ci]).astype(np.float32)
