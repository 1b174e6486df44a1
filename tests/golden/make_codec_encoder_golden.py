"""Generates tests/golden/codec_encoder_golden.json: codes from Hugging Face
transformers' HiggsAudioV2TokenizerModel.encode (the published
implementation the reference's codec_encoder.cpp ports: torchaudio's
resampler, HubertModel's averaged hidden states, the semantic encoder, the
DAC encoder, fc and the residual vector quantizer,
modeling_higgs_audio_v2_tokenizer.py:489-579) in float64 on the seeded
synthetic weights of oracle/codec_encoder.py, and checks the oracle's codes
and features against it.

Run from the repository root (CPU only):
    python tests/golden/make_codec_encoder_golden.py

transformers 5.5.0 and torchaudio 2.11 (installed in this image) provide the
modules; the weights and samples come from seeds, so the tests regenerate
them instead of storing them.
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import codec_encoder as oe  # noqa: E402

SMALL = dict(codebook_size=64, codebook_dim=8, hidden=32, intermediate=64, heads=4, layers=2,
             position_kernel=16, position_groups=4, conv_channels=[16, 16, 16, 16],
             conv_kernels=[10, 4, 4, 4], conv_strides=[5, 4, 4, 4], encoder_channels=4,
             latent_channels=32, downsampling_ratios=[8, 5, 4, 2, 3])
MID = dict(codebook_size=256, codebook_dim=16, hidden=64, intermediate=128, heads=4, layers=3,
           position_kernel=32, position_groups=8, conv_channels=[32] * 7, encoder_channels=8,
           latent_channels=64)
CASES = [
    # name, shape kwargs, weight seed, seconds, sample seed
    ("small", SMALL, 31, 1.0, 32),
    ("mid", MID, 41, 2.0, 42),
]


def hf_model(cfg: oe.EncoderShape, weights: dict):
    from transformers import HiggsAudioV2TokenizerConfig, HiggsAudioV2TokenizerModel

    bw = cfg.codebooks * math.log2(cfg.codebook_size) * (cfg.sample_rate / cfg.frame_samples) / 1000
    tok = HiggsAudioV2TokenizerConfig(
        acoustic_model_config=dict(encoder_hidden_size=cfg.encoder_channels,
                                   downsampling_ratios=list(cfg.downsampling_ratios),
                                   decoder_hidden_size=64, upsampling_ratios=list(cfg.downsampling_ratios),
                                   hidden_size=cfg.latent_channels),
        semantic_model_config=dict(hidden_size=cfg.hidden, num_hidden_layers=cfg.layers,
                                   num_attention_heads=cfg.heads, intermediate_size=cfg.intermediate,
                                   conv_dim=list(cfg.conv_channels), conv_kernel=list(cfg.conv_kernels),
                                   conv_stride=list(cfg.conv_strides),
                                   num_conv_pos_embeddings=cfg.position_kernel,
                                   num_conv_pos_embedding_groups=cfg.position_groups,
                                   feat_extract_norm="group", conv_bias=False,
                                   do_stable_layer_norm=False, feat_proj_layer_norm=True,
                                   layer_norm_eps=cfg.layer_norm_eps, hidden_act="gelu"),
        codebook_size=cfg.codebook_size, codebook_dim=cfg.codebook_dim,
        sample_rate=cfg.sample_rate, semantic_sample_rate=cfg.semantic_rate,
        downsample_factor=cfg.semantic_frame, target_bandwidths=[bw])
    model = HiggsAudioV2TokenizerModel(tok)
    sd = model.state_dict()
    missing = [k for k in weights if k not in sd]
    assert not missing, missing[:5]
    for k, v in weights.items():
        sd[k] = torch.from_numpy(v.reshape(sd[k].shape))
    model.load_state_dict(sd)
    return model.double().eval(), bw


def main():
    out = {"source": "transformers " + __import__("transformers").__version__ +
                     " HiggsAudioV2TokenizerModel.encode in float64; weights "
                     "oracle.codec_encoder.synthetic_weights",
           "cases": []}
    for name, kw, wseed, seconds, sseed in CASES:
        cfg = oe.EncoderShape(**kw)
        weights = oe.synthetic_weights(cfg, wseed)
        n = int(seconds * cfg.sample_rate) // cfg.frame_samples * cfg.frame_samples
        samples = (0.3 * np.random.default_rng(sseed).standard_normal(n)).astype(np.float32)
        model, bw = hf_model(cfg, weights)
        with torch.no_grad():
            x = torch.from_numpy(samples.astype(np.float64))[None, None, :]
            hf_codes = model.encode(x, bandwidth=bw, return_dict=False)[0].numpy()  # [codebooks][frames]
            feats = model._extract_semantic_features(x)[0].numpy()
        mine, f = oe.encode(weights, cfg, samples, return_features=True)
        sem_err = float(np.abs(f["hubert"][::cfg.semantic_stride][:feats.shape[0]] - feats).max())
        agree = float((mine == hf_codes).mean())
        print(f"{name}: {hf_codes.shape[1]} frames, oracle code agreement {agree:.4f}, "
              f"semantic features max |d| {sem_err:.2e}")
        assert hf_codes.shape == mine.shape and agree == 1.0, "oracle codes disagree with transformers"
        assert sem_err < 1e-5, "oracle semantic features disagree with transformers"
        out["cases"].append({"name": name, "shape": kw, "weight_seed": wseed, "seconds": seconds,
                             "sample_seed": sseed, "codes": hf_codes.tolist(),
                             "semantic_feature_max_error": sem_err})
    path = Path(__file__).with_name("codec_encoder_golden.json")
    path.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    main()
