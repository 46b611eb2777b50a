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
    """tensors: list of (name, array). Arrays are written as stored (F32 or F16)."""
    header, blobs, off = {}, [], 0
    for name, a in tensors:
        a = np.ascontiguousarray(a)
        header[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
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
