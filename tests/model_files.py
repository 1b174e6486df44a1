"""Writes model.safetensors files for the load tests: the reference's
tensor names (generator.cpp:364-434) holding the library's synthetic
weights, so a loaded generator equals Generator.synthetic(cfg, seed)."""
from __future__ import annotations

import json
import struct

import numpy as np


def write_safetensors(path, tensors):
    header, offset, blobs = {}, 0, []
    for name, arr in tensors.items():
        data = np.ascontiguousarray(arr, dtype=np.float32).tobytes()
        header[name] = {"dtype": "F32", "shape": list(arr.shape),
                        "data_offsets": [offset, offset + len(data)]}
        offset += len(data)
        blobs.append(data)
    raw = json.dumps(header).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)


def write_synthetic_model(path, cfg, seed, native):
    """Tensor ids as in the library's synthetic weights: text 1, audio
    embeddings 2, heads 3, layer l: 64 (l + 1) + {q 0, k 1, v 2, o 3,
    gate 4, up 5, down 6}; norms 1."""
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim

    def syn(tensor, *shape):
        out = np.empty(int(np.prod(shape)), np.float32)
        native.ov_synthetic_fill_host(out.ctypes.data, out.size, seed, tensor, 0.02, 0)
        return out.reshape(shape)

    t = {"llm.embed_tokens.weight": syn(1, cfg.vocab_size, H),
         "audio_embeddings.weight": syn(2, 8 * 1025, H),
         "audio_heads.weight": syn(3, 8 * 1025, H), "llm.norm.weight": np.ones(H)}
    for l in range(cfg.layers):
        b, p = 64 * (l + 1), f"llm.layers.{l}."
        t[p + "self_attn.q_proj.weight"] = syn(b, cfg.heads * D, H)
        t[p + "self_attn.k_proj.weight"] = syn(b + 1, cfg.kv_heads * D, H)
        t[p + "self_attn.v_proj.weight"] = syn(b + 2, cfg.kv_heads * D, H)
        t[p + "self_attn.o_proj.weight"] = syn(b + 3, H, cfg.heads * D)
        t[p + "mlp.gate_proj.weight"] = syn(b + 4, I, H)
        t[p + "mlp.up_proj.weight"] = syn(b + 5, I, H)
        t[p + "mlp.down_proj.weight"] = syn(b + 6, H, I)
        for n in ("input_layernorm", "post_attention_layernorm"):
            t[p + n + ".weight"] = np.ones(H)
        t[p + "self_attn.q_norm.weight"] = np.ones(D)
        t[p + "self_attn.k_norm.weight"] = np.ones(D)
    write_safetensors(path, t)
