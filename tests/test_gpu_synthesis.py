"""Chunked synthesis of a long text on the B200 (omnivoice_b200/synthesis.py):
chunk 0 alone, the remaining chunks as one packed batch, each decoded by
the codec, against the reference's chunk-by-chunk order
(synthesizer.cpp:180-207) on the same generator and codec."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import small_config  # noqa: E402
from omnivoice_b200 import ConditionalInput, DecodingConfig, Generator  # noqa: E402
from omnivoice_b200.codec import Codec, CodecConfig  # noqa: E402
from omnivoice_b200.synthesis import synthesize_chunks, synthesize_chunks_sequential  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("count,has_ref", [(4, False), (3, True)])
def test_batched_chunks_match_chunk_by_chunk(cuda_device, native, count, has_ref):
    cfg = small_config()
    gen = Generator.synthetic(cfg, weight_seed=5)
    codec = Codec.synthetic(CodecConfig(codebook_dim=8, semantic_hidden=32, latent_channels=32,
                                        decoder_channels=256, upsampling_ratios=[2, 3, 4]), seed=5)
    rng = np.random.default_rng(count)
    texts = [rng.integers(0, cfg.vocab_size, 8 + 5 * i).tolist() for i in range(count)]
    frames = [20 + 7 * i for i in range(count)]
    caller_ref = rng.integers(0, 1024, (8, 15)).astype(np.int32) if has_ref else None

    def build(i, voice):
        if voice is not None:  # chunk 0's text and codes lead the prompt
            return ConditionalInput.build(texts[voice.index] + texts[i], voice.codes, frames[i])
        return ConditionalInput.build(texts[i], caller_ref, frames[i])

    dec = DecodingConfig()
    got = synthesize_chunks(gen, codec, count, build, dec, seed=11, has_reference=has_ref)
    want = synthesize_chunks_sequential(gen, codec, count, build, dec, seed=11,
                                        has_reference=has_ref)
    for a, b in zip(got, want):
        assert a.codes.shape == (8, frames[a.index])
        assert (a.codes == b.codes).mean() >= 0.995
        if np.array_equal(a.codes, b.codes):
            assert np.array_equal(a.audio, b.audio)
        assert a.audio.shape == (frames[a.index] * 24,) and np.isfinite(a.audio).all()
    gen.close()
    codec.close()


def test_cloned_voice_prompts_the_chunks(cuda_device, native, tmp_path):
    """Voice cloning end to end: a recording encoded once by the CUDA codec
    encoder through the runner's voice cache (its codes equal the encoder
    oracle's), then used as the caller's reference voice for every chunk."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).parent))
    from model_files import write_safetensors
    from omnivoice_b200.codec import Encoder, EncoderConfig
    from omnivoice_b200.synthesis import VoiceCache
    from oracle import codec_encoder as oe

    shape = oe.EncoderShape(codebook_size=64, codebook_dim=8, hidden=32, intermediate=64, heads=4,
                            layers=2, position_kernel=16, position_groups=4,
                            conv_channels=[16, 16, 16, 16], conv_kernels=[10, 4, 4, 4],
                            conv_strides=[5, 4, 4, 4], encoder_channels=4, latent_channels=32)
    weights = oe.synthetic_weights(shape, 6)
    write_safetensors(tmp_path / "enc.safetensors", weights)
    enc = Encoder.load(EncoderConfig(codebook_size=64, codebook_dim=8, hidden_size=32,
                                     intermediate_size=64, heads=4, layers=2, position_kernel=16,
                                     position_groups=4, conv_channels=[16, 16, 16, 16],
                                     conv_kernels=[10, 4, 4, 4], conv_strides=[5, 4, 4, 4],
                                     encoder_channels=4, latent_channels=32),
                       str(tmp_path / "enc.safetensors"))
    recording = (0.3 * np.random.default_rng(6).standard_normal(960 * 20)).astype(np.float32)
    cache = VoiceCache(enc)
    voice = cache.get(recording, "a reference transcript")
    assert cache.get(recording, "a reference transcript") is voice and len(cache) == 1
    assert np.array_equal(voice.codes, oe.encode(weights, shape, recording))
    enc.close()

    cfg = small_config()
    gen = Generator.synthetic(cfg, weight_seed=6)
    rng = np.random.default_rng(7)
    texts = [rng.integers(0, cfg.vocab_size, 10).tolist() for _ in range(3)]

    def build(i, carried):
        assert carried is None  # the caller's voice: no carry-over
        return ConditionalInput.build(texts[i], voice.codes, 24)

    out = synthesize_chunks(gen, None, 3, build, DecodingConfig(steps=8), seed=3, has_reference=True)
    gen.close()
    assert [r.codes.shape for r in out] == [(8, 24)] * 3
    assert all(((r.codes >= 0) & (r.codes < 1024)).all() for r in out)


def test_gufo_runner_over_the_library(cuda_device, native, tmp_path):
    """tests/cpp/gufo_runner_test.cpp: a provider/runner translation unit in
    the shape of the reference's provider.cpp and runner.cpp, built against
    the Gufo SDK stand-in headers and this library, creates its runner
    through the registered provider and synthesises a three-chunk request;
    its codes must match the reference's chunk-by-chunk order."""
    import subprocess

    from model_files import write_safetensors, write_synthetic_model
    from omnivoice_b200.build import build_test_programs
    from oracle import codec as oc
    exe = [p for p in build_test_programs() if p.name == "gufo_runner_test"][0]
    cfg = small_config()
    write_synthetic_model(tmp_path / "model.safetensors", cfg, 3, native)
    shape = oc.CodecShape(codebook_dim=8, semantic_hidden=32, latent_channels=32,
                          decoder_channels=256, upsampling_ratios=[2, 3, 4])
    (tmp_path / "audio_tokenizer").mkdir()
    write_safetensors(tmp_path / "audio_tokenizer" / "model.safetensors",
                      oc.synthetic_weights(shape, 2))
    out = tmp_path / "out"
    out.mkdir()
    args = [str(exe), str(tmp_path), str(out), str(cfg.vocab_size), str(cfg.hidden_size),
            str(cfg.intermediate_size), str(cfg.layers), str(cfg.heads), str(cfg.kv_heads),
            "8", "32", "32", "256", "2", "3", "4"]
    run = subprocess.run(args, capture_output=True, text=True, timeout=600)
    print(run.stdout)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
    samples = np.fromfile(out / "samples.f32", np.float32)
    assert samples.shape == (3 * 24 * 24,) and np.isfinite(samples).all()
