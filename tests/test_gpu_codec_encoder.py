"""The CUDA codec encoder (include/ov_codec.h, ov_codec_encode) against the
encoder's CPU restatement (oracle/codec_encoder.py) on the same seeded
weights, written to a safetensors file with the reference's tensor names,
and the same samples: codes [codebooks][frames] equal (float32 against the
float64 restatement; a code may only differ where two entries are within
float32 rounding of each other, so the bar is 99 % of codes per case),
plus the reference's error behaviour."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).parent))
from model_files import write_safetensors  # noqa: E402
from omnivoice_b200.codec import CodecError, Encoder, EncoderConfig  # noqa: E402
from oracle import codec_encoder as oe  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(codebook_size=64, codebook_dim=8, hidden=32, intermediate=64, heads=4, layers=2,
             position_kernel=16, position_groups=4, conv_channels=[16, 16, 16, 16],
             conv_kernels=[10, 4, 4, 4], conv_strides=[5, 4, 4, 4], encoder_channels=4,
             latent_channels=32, downsampling_ratios=[8, 5, 4, 2, 3])
SHAPES = {"small": SMALL, "default": {}}


def config_of(shape: oe.EncoderShape) -> EncoderConfig:
    return EncoderConfig(sample_rate=shape.sample_rate, codebooks=shape.codebooks,
                         codebook_size=shape.codebook_size, codebook_dim=shape.codebook_dim,
                         semantic_sample_rate=shape.semantic_rate, hidden_size=shape.hidden,
                         intermediate_size=shape.intermediate, heads=shape.heads, layers=shape.layers,
                         position_kernel=shape.position_kernel, position_groups=shape.position_groups,
                         layer_norm_eps=shape.layer_norm_eps, conv_channels=list(shape.conv_channels),
                         conv_kernels=list(shape.conv_kernels), conv_strides=list(shape.conv_strides),
                         encoder_channels=shape.encoder_channels, latent_channels=shape.latent_channels,
                         downsampling_ratios=list(shape.downsampling_ratios))


def build(name, tmp_path, seed):
    shape = oe.EncoderShape(**SHAPES[name])
    weights = oe.synthetic_weights(shape, seed)
    path = tmp_path / f"{name}.safetensors"
    write_safetensors(path, weights)
    return shape, weights, Encoder.load(config_of(shape), str(path))


@pytest.mark.parametrize("name,seconds", [("small", 1.0), ("small", 2.2), ("default", 1.0)])
def test_encode_matches_oracle(cuda_device, native, tmp_path, name, seconds):
    shape, weights, enc = build(name, tmp_path, seed=int(seconds * 10))
    rng = np.random.default_rng(int(seconds * 10))
    n = int(seconds * shape.sample_rate) // shape.frame_samples * shape.frame_samples
    samples = (0.3 * rng.standard_normal(n)).astype(np.float32)
    got = enc.encode(samples)
    enc.close()
    want = oe.encode(weights, shape, samples)
    assert got.shape == want.shape
    agree = float((got == want).mean())
    print(f"{name} {seconds}s: {got.shape[1]} frames, code agreement {agree:.4f}, "
          f"per codebook {[float((got[c] == want[c]).mean()) for c in range(shape.codebooks)]}")
    assert agree >= 0.99


def test_encode_rejects_partial_frames(cuda_device, native, tmp_path):
    shape, _, enc = build("small", tmp_path, seed=1)
    samples = np.zeros(shape.frame_samples * 25 - 1, np.float32)
    with pytest.raises(CodecError, match="^OmniVoice encode: reference audio must be a whole number of frames"):
        enc.encode(samples)
    enc.close()


def test_encoder_load_reports_missing_tensor(cuda_device, native, tmp_path):
    shape = oe.EncoderShape(**SMALL)
    weights = oe.synthetic_weights(shape, 2)
    del weights["fc.bias"]
    path = tmp_path / "broken.safetensors"
    write_safetensors(path, weights)
    with pytest.raises(CodecError, match="^OmniVoice audio tokenizer: .*fc.bias"):
        Encoder.load(config_of(shape), str(path))


def test_synthetic_encoder_produces_codes(cuda_device, native):
    enc = Encoder.synthetic(EncoderConfig(), seed=3)
    rng = np.random.default_rng(3)
    samples = (0.3 * rng.standard_normal(24000 * 2)).astype(np.float32)
    codes = enc.encode(samples)
    enc.close()
    assert codes.shape == (8, 50)
    assert (codes >= 0).all() and (codes < 1024).all()
    assert len(set(codes[0].tolist())) > 5


def test_cpp_dropin_encode(cuda_device, native, tmp_path):
    """tests/cpp/codec_encoder_dropin_test.cpp: the reference-facing C++ class
    loads a checkpoint holding decoder and encoder tensors, Codec::Encode
    gives the oracle's codes and Codec::Decode takes them back to audio."""
    import subprocess

    from oracle import codec as oc
    exe = Path(__file__).resolve().parents[1] / "omnivoice_b200" / "_build" / "codec_encoder_dropin_test"
    if not exe.exists():
        pytest.skip("codec_encoder_dropin_test not built (python -m omnivoice_b200.build)")
    shape = oe.EncoderShape(**SMALL)
    weights = oc.synthetic_weights(oc.CodecShape(codebook_size=shape.codebook_size,
                                                 codebook_dim=shape.codebook_dim,
                                                 semantic_hidden=shape.hidden,
                                                 latent_channels=shape.latent_channels), 4)
    weights.update(oe.synthetic_weights(shape, 4))  # the quantizer's shared tensors: the encoder's
    (tmp_path / "audio_tokenizer").mkdir()
    write_safetensors(tmp_path / "audio_tokenizer" / "model.safetensors", weights)
    samples = (0.3 * np.random.default_rng(4).standard_normal(960 * 30)).astype(np.float32)
    samples.tofile(tmp_path / "samples.f32")
    out = subprocess.run([str(exe), str(tmp_path), str(tmp_path / "samples.f32"), str(samples.size),
                          str(tmp_path / "codes.i32")], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout + out.stderr
    got = np.fromfile(tmp_path / "codes.i32", np.int32).reshape(8, 30)
    assert (got == oe.encode(weights, shape, samples)).mean() >= 0.99


@pytest.mark.parametrize("case", ["small", "mid"])
def test_encode_matches_transformers_golden(cuda_device, native, tmp_path, case):
    """The CUDA encoder on the cases of tests/golden/codec_encoder_golden.json
    (codes of transformers' HiggsAudioV2TokenizerModel.encode in float64)."""
    import json
    g = {c["name"]: c for c in json.loads((Path(__file__).parent / "golden" /
                                           "codec_encoder_golden.json").read_text())["cases"]}[case]
    shape = oe.EncoderShape(**g["shape"])
    weights = oe.synthetic_weights(shape, g["weight_seed"])
    write_safetensors(tmp_path / "w.safetensors", weights)
    enc = Encoder.load(config_of(shape), str(tmp_path / "w.safetensors"))
    n = int(g["seconds"] * shape.sample_rate) // shape.frame_samples * shape.frame_samples
    samples = (0.3 * np.random.default_rng(g["sample_seed"]).standard_normal(n)).astype(np.float32)
    got = enc.encode(samples)
    enc.close()
    assert (got == np.array(g["codes"])).mean() >= 0.99
