"""Independent architecture check of the oracle (CPU): transformers'
Qwen3Model in float32 with a block-diagonal bidirectional mask, as the
reference's fixture generator builds its CFG batch
(tools/reference/generator_golden.py:40-54), must give the same logits as
the oracle's restatement of generator.cpp:262-301 up to the half roundings
the reference applies to activations."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")

from conftest import oracle_config_from, small_config  # noqa: E402


def synthetic(native, tensor, count, seed=5, first=0):
    """Values [first, first + count) of synthetic tensor `tensor`."""
    out = np.empty(count, np.float32)
    assert native.ov_synthetic_fill_host(out.ctypes.data, count, seed, tensor, 0.02, first) == 0
    return out


def half(a):
    return a.astype(np.float16).astype(np.float32)


def build_hf(native, cfg, seed):
    from transformers import Qwen3Config, Qwen3Model
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    # The model is fed embeddings (inputs_embeds): its own table is unused.
    hf = Qwen3Config(vocab_size=16, hidden_size=H, intermediate_size=I,
                     num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                     num_key_value_heads=cfg.kv_heads, head_dim=D, rms_norm_eps=cfg.rms_norm_eps,
                     rope_theta=cfg.rope_theta, max_position_embeddings=4096,
                     attn_implementation="eager")
    model = Qwen3Model(hf).eval()
    sd = model.state_dict()
    qh, kvh = cfg.heads * D, cfg.kv_heads * D

    def lin(tensor, rows, cols):
        return torch.from_numpy(half(synthetic(native, tensor, rows * cols, seed)).reshape(rows, cols))

    for l in range(cfg.layers):
        base = 64 * (l + 1)
        p = f"layers.{l}."
        sd[p + "self_attn.q_proj.weight"] = lin(base + 0, qh, H)
        sd[p + "self_attn.k_proj.weight"] = lin(base + 1, kvh, H)
        sd[p + "self_attn.v_proj.weight"] = lin(base + 2, kvh, H)
        sd[p + "self_attn.o_proj.weight"] = lin(base + 3, H, qh)
        sd[p + "mlp.gate_proj.weight"] = lin(base + 4, I, H)
        sd[p + "mlp.up_proj.weight"] = lin(base + 5, I, H)
        sd[p + "mlp.down_proj.weight"] = lin(base + 6, H, I)
        for name in ("input_layernorm", "post_attention_layernorm"):
            sd[p + name + ".weight"] = torch.ones(H)
        sd[p + "self_attn.q_norm.weight"] = torch.ones(D)
        sd[p + "self_attn.k_norm.weight"] = torch.ones(D)
    sd["norm.weight"] = torch.ones(H)
    model.load_state_dict(sd)
    return model


def _compare(native, oracle_lib, cfg, seed, ids, start, F):
    """Oracle logits against transformers' Qwen3Model on the same weights and
    packed CFG batch (conditional rows then the unconditional copy of the
    target frames, each block attending only within itself)."""
    L = ids.shape[1]
    model = oracle_lib.OracleModel(oracle_config_from(cfg), seed)
    got = model.forward(ids, start, F)
    model.close()

    H = cfg.hidden_size
    audio = synthetic(native, 2, 8 * 1025 * H, seed).reshape(8 * 1025, H)
    heads = half(synthetic(native, 3, 8 * 1025 * H, seed).reshape(8 * 1025, H))
    R = L + F
    packed = np.concatenate([ids, ids[:, L - F:]], axis=1)
    emb = np.zeros((R, H), np.float32)
    for r in range(R):
        if r < start:  # the text table's row of this id
            emb[r] = synthetic(native, 1, H, seed, int(packed[0, r]) * H)
        else:
            for c in range(8):
                emb[r] += audio[c * 1025 + packed[c, r]]
    pos = np.concatenate([np.arange(L), np.arange(F)])
    allowed = np.zeros((R, R), bool)
    allowed[:L, :L] = True
    allowed[L:, L:] = True
    mask = torch.where(torch.from_numpy(allowed), 0.0, float("-inf"))[None, None]
    hf = build_hf(native, cfg, seed)
    with torch.no_grad():
        h = hf(inputs_embeds=torch.from_numpy(emb)[None], attention_mask=mask,
               position_ids=torch.from_numpy(pos)[None]).last_hidden_state[0].numpy()
    del hf
    rows = np.concatenate([np.arange(L - F, L), np.arange(L, L + F)])
    want = half(h[rows]) @ heads.T
    diff = np.abs(got - want)
    agree = (got.reshape(2 * F, 8, 1025).argmax(-1) == want.reshape(2 * F, 8, 1025).argmax(-1)).mean()
    print(f"max |d logit| {diff.max():.3e}, mean {diff.mean():.3e}, argmax agreement {agree:.4f}")
    return diff, agree


def test_oracle_forward_matches_transformers_qwen3(native, oracle_lib):
    cfg = small_config()
    rng = np.random.default_rng(0)
    L, F, start = 48, 20, 12
    ids = rng.integers(0, 1024, size=(8, L)).astype(np.int32)
    ids[:, start:] = rng.integers(0, 1024, size=(8, L - start))
    ids[:, L - F:] = 1024
    ids[:, L - F:L - F + 5] = rng.integers(0, 1024, size=(8, 5))
    text = rng.integers(0, cfg.vocab_size, size=start).astype(np.int32)
    ids[:, :start] = text[None, :]
    diff, agree = _compare(native, oracle_lib, cfg, 5, ids, start, F)
    assert diff.max() < 2e-2, diff.max()
    assert agree >= 0.95, agree


def test_oracle_full_width_config1_matches_transformers_qwen3(native, oracle_lib):
    """The same check on the real model's widths (hidden 1024, 16/8 heads of
    128, intermediate 3072, vocabulary 151936; random init of seed 0) with
    BASELINE config 1's conditional input at the oracle's first generation
    step (every target frame masked, tests/golden/generation_golden.npz).
    One layer by default, to keep the CPU suite short (building the float32
    transformers model dominates); OV_ORACLE_HF_LAYERS=28 runs the full
    depth (about 12 minutes on this suite's CPU host)."""
    import os
    from pathlib import Path
    from omnivoice_b200 import model_config
    cfg = model_config()
    cfg.layers = int(os.environ.get("OV_ORACLE_HF_LAYERS", "1"))
    data = np.load(Path(__file__).resolve().parent / "golden" / "generation_golden.npz")
    ids = np.ascontiguousarray(data["c1_step_ids"][0])
    start, F, _ = (int(v) for v in data["c1_meta"])
    diff, agree = _compare(native, oracle_lib, cfg, 0, ids, start, F)
    assert diff.max() < 2e-2, diff.max()
    assert agree >= 0.95, agree
