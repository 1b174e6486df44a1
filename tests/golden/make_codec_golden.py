"""Generates tests/golden/codec_golden.json: audio decoded by Hugging Face
transformers' HiggsAudioV2Tokenizer decoder path (the published
implementation the reference's codec.cpp ports: RVQ decode,
HiggsAudioV2TokenizerModel.decode's fc2, and transformers' DacDecoder
with the tokenizer's stride-parity output padding and no final tanh,
modeling_higgs_audio_v2_tokenizer.py:476-489,564-584) on the seeded
synthetic weights of oracle/codec.py, and checks the oracle against it.

Run from the repository root (CPU only):  python tests/golden/make_codec_golden.py

transformers 5.5.0 (installed in this image) provides the modules; the
weights come from oracle.codec.synthetic_weights, so the tests regenerate
them instead of storing them.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import codec as oc  # noqa: E402

CASES = [
    # name, shape, weight seed, frames, code seed, stored sample stride
    ("small", oc.CodecShape(codebook_dim=8, semantic_hidden=24, latent_channels=16,
                            decoder_channels=64), 11, 6, 12, 1),
    ("default", oc.CodecShape(), 21, 3, 22, 3),
]


def hf_decoder(cfg: oc.CodecShape, weights: dict, dtype):
    from transformers import DacConfig
    from transformers.models.dac.modeling_dac import DacDecoder
    from transformers.models.higgs_audio_v2_tokenizer import modeling_higgs_audio_v2_tokenizer as M
    from transformers.models.higgs_audio_v2_tokenizer.configuration_higgs_audio_v2_tokenizer import (
        HiggsAudioV2TokenizerConfig)

    acoustic = DacConfig(decoder_hidden_size=cfg.decoder_channels,
                         upsampling_ratios=list(cfg.upsampling_ratios),
                         downsampling_ratios=list(cfg.upsampling_ratios),
                         hidden_size=cfg.latent_channels)
    tok = HiggsAudioV2TokenizerConfig(
        acoustic_model_config=acoustic.to_dict(),
        semantic_model_config=dict(hidden_size=cfg.semantic_hidden, num_hidden_layers=1,
                                   num_attention_heads=1, intermediate_size=8),
        codebook_size=cfg.codebook_size, codebook_dim=cfg.codebook_dim)
    decoder = DacDecoder(acoustic)
    M.HiggsAudioV2TokenizerModel._adjust_dac_decoder(decoder)
    quantizer = M.HiggsAudioV2TokenizerResidualVectorQuantization(tok)
    assert len(quantizer.quantizers) >= cfg.codebooks
    fc2 = torch.nn.Linear(cfg.hidden, cfg.latent_channels)

    def load(module, prefix):
        sd = module.state_dict()
        for name in sd:
            key = prefix + name
            if key in weights:
                sd[name] = torch.from_numpy(weights[key].reshape(sd[name].shape))
        module.load_state_dict(sd)
        return module.to(dtype).eval()

    decoder = load(decoder, "acoustic_decoder.")
    quantizer = load(quantizer, "quantizer.")
    fc2 = load(fc2, "fc2.")

    def run(codes):
        with torch.no_grad():
            c = torch.from_numpy(np.asarray(codes, np.int64))[:, None, :]  # [codebooks][1][frames]
            q = quantizer.decode(c)                                        # [1][hidden][frames]
            lat = fc2(q.transpose(1, 2)).transpose(1, 2)
            return decoder(lat)[0, 0].double().numpy()
    return run


def main():
    out = {"source": "transformers " + __import__("transformers").__version__ +
                     " HiggsAudioV2Tokenizer decode path; weights oracle.codec.synthetic_weights",
           "cases": []}
    for name, cfg, wseed, frames, cseed, stride in CASES:
        weights = oc.synthetic_weights(cfg, wseed)
        codes = np.random.default_rng(cseed).integers(0, cfg.codebook_size, (cfg.codebooks, frames))
        ref64 = hf_decoder(cfg, weights, torch.float64)(codes)
        ref32 = hf_decoder(cfg, weights, torch.float32)(codes)
        mine = oc.decode(weights, cfg, codes)
        scale = float(np.sqrt(np.mean(ref64 ** 2)))
        err_oracle = float(np.abs(mine - ref64).max())
        err_fp32 = float(np.abs(ref32 - ref64).max())
        print(f"{name}: {len(ref64)} samples rms {scale:.4f}; oracle vs fp64 {err_oracle:.3e}; "
              f"fp32 vs fp64 {err_fp32:.3e}")
        assert err_oracle <= 1e-9 * max(1.0, scale), "oracle disagrees with transformers"
        out["cases"].append({
            "name": name,
            "shape": {"codebooks": cfg.codebooks, "codebook_size": cfg.codebook_size,
                      "codebook_dim": cfg.codebook_dim, "semantic_hidden": cfg.semantic_hidden,
                      "latent_channels": cfg.latent_channels,
                      "decoder_channels": cfg.decoder_channels,
                      "upsampling_ratios": list(cfg.upsampling_ratios)},
            "weight_seed": wseed, "codes": codes.tolist(), "length": len(ref64),
            "rms": scale, "stride": stride,
            "samples": [float("%.9g" % v) for v in ref64[::stride]],
            "fp32_max_error": err_fp32,
        })
    path = Path(__file__).with_name("codec_golden.json")
    path.write_text(json.dumps(out, indent=1))
    print("wrote", path)


if __name__ == "__main__":
    main()
