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
