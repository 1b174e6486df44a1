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
pieces (synthesizer.cpp:208-212) are the caller's too.
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
