"""Generation and decoding of the chunks of one long text (row f2).

The reference synthesises a long text chunk by chunk, each chunk one
32-step generation followed by a codec decode, strictly one after the other
(synthesizer.cpp:163-207).  The only dependency between chunks is the voice
carry-over: without a caller-supplied reference voice, chunk 0's text and
codes become the reference of every later chunk (synthesizer.cpp:196-200).
So chunks 1..n-1 are independent of each other once chunk 0 is done (and
all n are independent when the caller gives a reference).  This module
keeps the reference's results and runs them as:

  1. chunk 0 alone when its codes carry the voice;
  2. every remaining chunk in one packed batch (Generator.generate_batch,
     one shared unmasking loop), or through the runner the caller passes as
     `batch` (for instance one that spreads the chunks over several GPUs
     with scheduler.generate_data_parallel);
  3. each chunk's codes decoded by the codec (chunks are separate signals:
     the decoder's convolutions must not see across chunk boundaries).

Text chunking, prompt building and tokenisation (synthesizer.cpp:166-178,
prompt.cpp) stay with the caller: `build_input(index, voice)` returns the
ConditionalInput of chunk `index` given the reference voice `voice` (None,
or the carried Voice of chunk 0).  Cross-fading and post-processing of the
pieces (synthesizer.cpp:202-206) are the caller's too.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np


@dataclass
class Voice:
    """A reference voice carried from chunk `index` (synthesizer.cpp:196-200):
    its codes [codebooks][frames]."""
    index: int
    codes: np.ndarray

    @property
    def frames(self) -> int:
        return int(self.codes.shape[1])


@dataclass
class ChunkResult:
    index: int
    codes: np.ndarray      # [codebooks][frames]
    audio: np.ndarray | None


def synthesize_chunks(generator, codec, count: int,
                      build_input: Callable[[int, Voice | None], object], decoding, seed: int,
                      has_reference: bool = False, noise: str = "device",
                      batch: Callable[[list, object, list], list] | None = None
                      ) -> list[ChunkResult]:
    """Generates and decodes `count` chunks; returns them in chunk order.

    `has_reference`: the caller's prompt already carries a reference voice,
    so there is no carry-over and all chunks run in one batch.  Every chunk
    uses `seed` (the reference passes the same options to each chunk).
    `batch(inputs, decoding, seeds)` overrides the batched generation (for
    instance a data-parallel runner over several GPUs); by default it is
    `generator.generate_batch(..., noise=noise)`.  `codec` may be None to
    skip decoding."""
    if count < 1:
        raise ValueError("no chunks")
    run = batch or (lambda inputs, dec, seeds: generator.generate_batch(inputs, dec, seeds,
                                                                      noise=noise))

    def generate(indices, voice):
        inputs = [build_input(i, voice) for i in indices]
        outs = run(inputs, decoding, [seed] * len(indices))
        if len(outs) != len(indices):
            raise RuntimeError("batch returned %d results for %d chunks" % (len(outs), len(indices)))
        return outs

    results: list[ChunkResult | None] = [None] * count
    voice = None
    first = 0
    if not has_reference and count > 1:
        res0 = generate([0], None)[0]
        results[0] = ChunkResult(0, res0.codes, None)
        voice = Voice(0, res0.codes)
        first = 1
    rest = list(range(first, count))
    for i, out in zip(rest, generate(rest, voice)):
        results[i] = ChunkResult(i, out.codes, None)
    if codec is not None:
        for r in results:
            r.audio = codec.decode(r.codes)
    return results


def synthesize_chunks_sequential(generator, codec, count: int,
                                 build_input: Callable[[int, Voice | None], object], decoding,
                                 seed: int, has_reference: bool = False, noise: str = "device"
                                 ) -> list[ChunkResult]:
    """The reference's order (synthesizer.cpp:180-207): one generation and
    one decode per chunk, the voice carried from chunk 0.  The checker of
    synthesize_chunks and the baseline it is timed against."""
    results = []
    voice = None
    for i in range(count):
        out = generator.generate_batch([build_input(i, voice)], decoding, [seed], noise=noise)[0]
        results.append(ChunkResult(i, out.codes, codec.decode(out.codes) if codec else None))
        if not has_reference and i == 0 and count > 1:
            voice = Voice(0, out.codes)
    return results


def chunk_seconds(results: Sequence[ChunkResult], frame_rate: float = 25.0) -> float:
    return sum(r.codes.shape[1] for r in results) / frame_rate


@dataclass
class ClonedVoice:
    """A reference voice encoded for cloning (synthesizer.cpp:111-130's
    ReferenceVoice): its codes [codebooks][frames] and transcript."""
    codes: np.ndarray
    text: str

    @property
    def frames(self) -> int:
        return int(self.codes.shape[1])


def clone_voice(encoder, samples, text: str) -> ClonedVoice:
    """Synthesizer::CloneVoice's encode step (synthesizer.cpp:111-130): the
    transcript is required and the prepared 24 kHz mono samples are encoded
    by the codec encoder (`encoder.encode`, omnivoice_b200.codec.Encoder).
    Preparing the recording (downmix, resampling to 24 kHz, level, silence
    removal and the trim to whole frames, audio.cpp PrepareReference) is the
    caller's; samples that are not a whole number of frames raise the
    encoder's error."""
    if not text.strip():
        raise ValueError("OmniVoice: voice cloning needs the reference transcript")
    return ClonedVoice(np.asarray(encoder.encode(samples)), text)


def fingerprint(samples, text: str) -> int:
    """64-bit FNV-1a over the samples' bytes and the transcript's, the key of
    the runner's voice cache (runner.cpp:22-35)."""
    h = 1469598103934665603
    for data in (np.ascontiguousarray(samples, dtype=np.float32).tobytes(), text.encode()):
        for b in data:
            h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class VoiceCache:
    """The runner's cache of cloned voices (runner.cpp:143-172): the
    `capacity` most recently used recordings and transcripts, each encoded
    once; a hit moves to the front, the least recently used falls out."""

    def __init__(self, encoder, capacity: int = 8):
        self.encoder = encoder
        self.capacity = capacity
        self._entries: list[tuple[int, ClonedVoice]] = []  # most recent first

    def __len__(self) -> int:
        return len(self._entries)

    def get(self, samples, text: str) -> ClonedVoice:
        key = fingerprint(samples, text)
        for i, (k, voice) in enumerate(self._entries):
            if k == key:
                self._entries.insert(0, self._entries.pop(i))
                return voice
        voice = clone_voice(self.encoder, samples, text)
        self._entries.insert(0, (key, voice))
        del self._entries[self.capacity:]
        return voice
