"""Chunk scheduling of a long text (omnivoice_b200/synthesis.py) on the
host, with a fake generator and codec: the voice carry-over of
synthesizer.cpp:196-200 and the batching of the independent chunks."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest

from omnivoice_b200 import synthesis
from omnivoice_b200.synthesis import (synthesize_chunks, synthesize_chunks_sequential)


@dataclass
class FakeInput:
    index: int
    voice: object
    frames: int


@dataclass
class FakeResult:
    codes: np.ndarray


class FakeGenerator:
    """Codes depend only on (chunk, carried voice, seed), like a real
    generation of that prompt."""

    def __init__(self):
        self.calls = []

    def generate_batch(self, inputs, decoding, seeds, noise="device"):
        self.calls.append([i.index for i in inputs])
        out = []
        for inp, seed in zip(inputs, seeds):
            v = 0 if inp.voice is None else int(inp.voice.codes.sum()) % 97
            codes = np.full((8, inp.frames), (inp.index * 31 + v + seed) % 1024, np.int32)
            out.append(FakeResult(codes))
        return out


class FakeCodec:
    def __init__(self):
        self.decoded = 0

    def decode(self, codes):
        self.decoded += 1
        return codes[0].astype(np.float32).repeat(4)


def builder(frames):
    return lambda i, voice: FakeInput(i, voice, frames[i])


@pytest.mark.parametrize("count,has_ref", [(1, False), (2, False), (5, False), (4, True)])
def test_batched_chunks_equal_the_reference_order(count, has_ref):
    frames = [10 + 3 * i for i in range(count)]
    gen, codec = FakeGenerator(), FakeCodec()
    got = synthesize_chunks(gen, codec, count, builder(frames), None, seed=7, has_reference=has_ref)
    if count > 1 and not has_ref:
        assert gen.calls == [[0], list(range(1, count))]  # chunk 0, then one batch
    else:
        assert gen.calls == [list(range(count))]         # nothing carried: one batch
    assert codec.decoded == count
    want = synthesize_chunks_sequential(FakeGenerator(), FakeCodec(), count, builder(frames), None,
                                        seed=7, has_reference=has_ref)
    assert [r.index for r in got] == list(range(count))
    for a, b in zip(got, want):
        assert np.array_equal(a.codes, b.codes)
        assert np.array_equal(a.audio, b.audio)
        assert a.codes.shape == (8, frames[a.index])


def test_later_chunks_carry_chunk_zero_voice():
    seen = []

    def build(i, voice):
        seen.append((i, None if voice is None else voice.index))
        return FakeInput(i, voice, 5)

    synthesize_chunks(FakeGenerator(), None, 3, build, None, seed=0)
    assert seen == [(0, None), (1, 0), (2, 0)]


def test_batch_override_and_errors():
    calls = []

    def runner(inputs, decoding, seeds):
        calls.append(len(inputs))
        return [FakeResult(np.zeros((8, i.frames), np.int32)) for i in inputs]

    out = synthesize_chunks(None, None, 3, builder([4, 4, 4]), None, seed=0, batch=runner)
    assert calls == [1, 2] and all(r.audio is None for r in out)
    with pytest.raises(ValueError):
        synthesize_chunks(None, None, 0, builder([]), None, seed=0, batch=runner)
    with pytest.raises(RuntimeError, match="results"):
        synthesize_chunks(None, None, 3, builder([4, 4, 4]), None, seed=0,
                          batch=lambda inputs, d, s: [])


# ------------------------------------------------------------ voice cloning

class CountingEncoder:
    """Stands in for omnivoice_b200.codec.Encoder: codes from the samples'
    mean, and a count of the encodes."""

    def __init__(self):
        self.calls = 0

    def encode(self, samples):
        self.calls += 1
        samples = np.asarray(samples, np.float32)
        if samples.size == 0 or samples.size % 960:
            raise ValueError("OmniVoice encode: reference audio must be a whole number of frames")
        frames = samples.size // 960
        return np.full((8, frames), int(abs(samples.mean()) * 1000) % 1024, np.int32)


def test_clone_voice_needs_a_transcript_and_encodes_once():
    enc = CountingEncoder()
    with pytest.raises(ValueError, match="needs the reference transcript"):
        synthesis.clone_voice(enc, np.zeros(960, np.float32), "  ")
    voice = synthesis.clone_voice(enc, np.full(960 * 3, 0.25, np.float32), "hello")
    assert voice.frames == 3 and voice.text == "hello" and enc.calls == 1


def test_fingerprint_is_fnv1a_over_samples_and_text():
    # FNV-1a 64 of the empty input is the offset basis; one byte moves it.
    assert synthesis.fingerprint(np.zeros(0, np.float32), "") == 1469598103934665603
    a = synthesis.fingerprint(np.zeros(4, np.float32), "x")
    assert a != synthesis.fingerprint(np.zeros(4, np.float32), "y")
    assert a == synthesis.fingerprint(np.zeros(4, np.float32), "x")


def test_voice_cache_encodes_each_recording_once_and_evicts_lru():
    enc = CountingEncoder()
    cache = synthesis.VoiceCache(enc, capacity=2)
    rec = [np.full(960, v, np.float32) for v in (0.1, 0.2, 0.3)]
    cache.get(rec[0], "a")
    cache.get(rec[1], "b")
    cache.get(rec[0], "a")          # hit, moves to the front
    assert enc.calls == 2
    cache.get(rec[2], "c")          # evicts rec[1] (least recently used)
    assert len(cache) == 2
    cache.get(rec[0], "a")
    assert enc.calls == 3
    cache.get(rec[1], "b")          # evicted: encoded again
    assert enc.calls == 4
