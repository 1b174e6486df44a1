"""Chunk scheduling of a long text (omnivoice_b200/synthesis.py) on the
host, with a fake generator and codec: the voice carry-over of
synthesizer.cpp:196-200 and the batching of the independent chunks."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest

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
