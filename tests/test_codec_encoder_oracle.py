"""The encoder's CPU restatement (oracle/codec_encoder.py): the resampler
pinned to the reference's torchaudio golden vectors
(tests/golden/resample_golden.json, extracted by make_resample_golden.py),
and the encoder's structure on a small shape (frame counts, code ranges,
determinism, the quantizer against the decoder restatement's tables)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import codec as dec
from oracle import codec_encoder as enc

GOLDEN = Path(__file__).parent / "golden" / "resample_golden.json"

# A small encoder: HuBERT strides multiply to 320 (50 frames per second at
# 16 kHz), DAC strides to 960 (25 frames per second at 24 kHz).
SMALL = dict(codebook_size=64, codebook_dim=8, hidden=32, intermediate=64, heads=4, layers=2,
             position_kernel=16, position_groups=4, conv_channels=[16, 16, 16, 16],
             conv_kernels=[10, 4, 4, 4], conv_strides=[5, 4, 4, 4], encoder_channels=4,
             latent_channels=32, downsampling_ratios=[8, 5, 4, 2, 3])


def generate(spec, rate, seed):
    """The reference audio test's integer signal generator (audio_test.cpp
    Generate): a 31-bit LCG driving noise and a triangle tone, PCM16 / 32768."""
    state = seed
    out = []
    for ms, kind, amplitude in spec:
        noise_amplitude = min(amplitude, 64)
        for n in range(ms * rate // 1000):
            state = (state * 1103515245 + 12345) & 0x7FFFFFFF
            if kind == "tone":
                period = 55
                phase = n % period
                noise = (state >> 8) % (2 * noise_amplitude + 1) - noise_amplitude
                value = (4 * amplitude * abs(2 * phase - period)) // (2 * period) - amplitude + noise
            else:
                value = (state >> 8) % (2 * amplitude + 1) - amplitude
            value = min(max(value, -32768), 32767)
            out.append(np.float32(value) / np.float32(32768.0))
    return np.array(out, dtype=np.float32)


@pytest.mark.parametrize("case", range(6))
def test_resample_matches_reference_golden(case):
    g = json.loads(GOLDEN.read_text())
    e = g["cases"][case]
    sig = e["signal"]
    got = enc.resample(generate(sig["spec"], sig["rate"], sig["seed"]), sig["rate"], e["target"])
    assert got.size == e["length"]
    want = np.array(e["samples"], dtype=np.float64)
    diff = np.abs(got[::g["stride"]][:want.size].astype(np.float64) - want)
    assert diff.max() <= g["tolerance"], diff.max()


def small_case(seconds=1.0, seed=0):
    cfg = enc.EncoderShape(**SMALL)
    weights = enc.synthetic_weights(cfg, seed)
    rng = np.random.default_rng(seed + 100)
    n = int(seconds * cfg.sample_rate) // cfg.frame_samples * cfg.frame_samples
    samples = (0.3 * rng.standard_normal(n)).astype(np.float32)
    return cfg, weights, samples


def test_encode_small_shape_frames_and_ranges():
    cfg, weights, samples = small_case(1.0)
    assert cfg.semantic_stride == 2
    codes, feats = enc.encode(weights, cfg, samples, return_features=True)
    frames = samples.size // cfg.frame_samples
    assert codes.shape == (cfg.codebooks, frames)
    assert (codes >= 0).all() and (codes < cfg.codebook_size).all()
    assert feats["acoustic"].shape == (frames, cfg.latent_channels)
    assert feats["semantic"].shape == (frames, cfg.hidden)
    assert np.isfinite(feats["fc"]).all()
    # Not degenerate: several entries used per codebook.
    assert min(len(set(row)) for row in codes.tolist()) > 3
    assert np.array_equal(codes, enc.encode(weights, cfg, samples))


def test_quantizer_tables_are_the_decoders():
    cfg, weights, _ = small_case(0.2)
    shape = dec.CodecShape(codebooks=cfg.codebooks, codebook_size=cfg.codebook_size,
                           codebook_dim=cfg.codebook_dim, semantic_hidden=cfg.hidden,
                           latent_channels=cfg.latent_channels)
    for a, b in zip(enc.decode_tables(weights, cfg), dec.rvq_tables(weights, shape)):
        assert np.array_equal(a, b)


def test_quantize_recovers_codes_of_a_decoded_sum():
    """A residual that is exactly the sum of one entry per codebook, with
    project_in the pseudo-inverse direction of project_out, quantizes back
    to those entries (each stage removes its entry)."""
    cfg, weights, _ = small_case(0.2)
    rng = np.random.default_rng(5)
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        w_out = weights[p + "project_out.weight"].astype(np.float64)
        weights[p + "project_in.weight"] = np.linalg.pinv(w_out).astype(np.float32)
        weights[p + "project_in.bias"] = (-np.linalg.pinv(w_out) @ weights[p + "project_out.bias"]).astype(np.float32)
    tables = enc.decode_tables(weights, cfg)
    want = rng.integers(0, cfg.codebook_size, (cfg.codebooks, 6))
    residual = sum(tables[c][want[c]] for c in range(cfg.codebooks))
    # Only codebook 0 sees the others' entries as noise; a large first entry
    # scale keeps its choice unambiguous.
    got = enc.quantize(weights, cfg, residual)
    assert (got[0] == want[0]).mean() >= 0.5


def test_rejects_partial_frames():
    cfg, weights, samples = small_case(0.2)
    with pytest.raises(ValueError, match="whole number of frames"):
        enc.encode(weights, cfg, samples[:-1])


ENC_GOLDEN = Path(__file__).parent / "golden" / "codec_encoder_golden.json"


@pytest.mark.parametrize("case", ["small", "mid"])
def test_encode_matches_transformers_golden(case):
    """Codes of transformers' HiggsAudioV2TokenizerModel.encode (float64, the
    published implementation the reference ports) on the seeded weights,
    stored by tests/golden/make_codec_encoder_golden.py: the restatement
    reproduces them exactly."""
    g = {c["name"]: c for c in json.loads(ENC_GOLDEN.read_text())["cases"]}[case]
    cfg = enc.EncoderShape(**g["shape"])
    weights = enc.synthetic_weights(cfg, g["weight_seed"])
    n = int(g["seconds"] * cfg.sample_rate) // cfg.frame_samples * cfg.frame_samples
    samples = (0.3 * np.random.default_rng(g["sample_seed"]).standard_normal(n)).astype(np.float32)
    assert np.array_equal(enc.encode(weights, cfg, samples), np.array(g["codes"]))
