"""Data-parallel generation over several GPUs, one process (rank) per GPU.

Each rank holds a full replica of the generator (the 0.6 B backbone fits
any B200 many times over); one generation is never split across GPUs,
because every unmasking step depends on the previous one.  A batch of
utterances is partitioned on the host by longest-processing-time first
(LPT) over the hot path's cost model, each rank generates its share as
packed batches through its own generator, and the codes are gathered to
rank 0 in host memory.  There is no collective on the data path: the one
exchange is the gather of the finished codes.

The reference serves one request at a time per GPU worker
(gufo-extensions/omnivoice README.md:78, synthesizer.cpp:163-201); this
module is the scheduler that batching across utterances and GPUs needs.

Failures are detected on the host: a rank whose generation raises reports
the error in its gathered payload and rank 0 raises WorkerFailed naming
it; a rank that never reports ends the gather with the process group's
timeout, which rank 0 also turns into WorkerFailed.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

# Algorithmic FLOPs of one forward step: R rows through the 28 layers'
# linear layers, attention over each sequence, and the audio heads on the
# 2F target rows (Qwen3-0.6B shape: hidden 1024, 16/8 heads of 128,
# intermediate 3072, 8 x 1025 audio logits).
FLOPS_PER_ROW = 28 * 2 * (1024 * 4096 + 2048 * 1024 + 1024 * 6144 + 3072 * 1024)
FLOPS_PER_KEY_PAIR = 28 * 4 * 128 * 16
FLOPS_PER_TARGET_ROW = 2 * 1024 * 8200


def utterance_cost(length: int, frames: int, steps: int = 32) -> float:
    """FLOPs of one full generation: conditional sequence of `length` rows
    and unconditional sequence of `frames` rows, `steps` forward passes."""
    rows = length + frames
    return steps * (rows * FLOPS_PER_ROW + FLOPS_PER_KEY_PAIR * (length * length + frames * frames)
                    + 2 * frames * FLOPS_PER_TARGET_ROW)


def lpt_partition(costs: Sequence[float], workers: int) -> tuple[list[list[int]], list[float]]:
    """Longest-processing-time-first assignment of items to `workers`.

    Items are taken in decreasing cost (ties by index) and each goes to the
    least-loaded worker (ties by worker index), so the result depends only
    on the costs.  Returns the item indices of each worker (in assignment
    order) and each worker's total cost."""
    if workers < 1:
        raise ValueError("workers must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * workers
    parts: list[list[int]] = [[] for _ in range(workers)]
    for i in order:
        w = min(range(workers), key=lambda k: (load[k], k))
        parts[w].append(i)
        load[w] += costs[i]
    return parts, load


def pack_by_frames(indices: Sequence[int], frames: Sequence[int], rows: Sequence[int],
                   max_rows: int) -> list[list[int]]:
    """Splits one worker's utterances into packed batches of at most
    `max_rows` packed rows (a single larger utterance forms its own pack),
    grouping similar frame counts so the packs' unmasking schedules stay
    aligned."""
    order = sorted(indices, key=lambda i: (-frames[i], i))
    packs: list[list[int]] = []
    current: list[int] = []
    used = 0
    for i in order:
        if current and used + rows[i] > max_rows:
            packs.append(current)
            current, used = [], 0
        current.append(i)
        used += rows[i]
    if current:
        packs.append(current)
    return packs


class WorkerFailed(RuntimeError):
    def __init__(self, rank: int, message: str):
        super().__init__(f"rank {rank}: {message}")
        self.rank = rank


@dataclass
class _Payload:
    rank: int
    ok: bool
    error: str
    results: list  # [(index, result)]


def generate_data_parallel(inputs: Sequence, decoding, seeds: Sequence[int],
                           runner: Callable[[list, object, list], list],
                           group=None, max_rows: int = 1 << 17) -> list | None:
    """Generates every input across the ranks of `group` (the default
    torch.distributed group; a single process when torch.distributed is
    not initialised).

    `runner(inputs, decoding, seeds)` generates one packed batch on this
    rank's GPU and returns one result per input (Generator.generate_batch).
    Every rank calls this with the same arguments.  Rank 0 returns the
    results in input order; the other ranks return None."""
    import torch.distributed as dist

    distributed = dist.is_available() and dist.is_initialized()
    rank = dist.get_rank(group) if distributed else 0
    world = dist.get_world_size(group) if distributed else 1
    if len(seeds) != len(inputs):
        raise ValueError("one seed per input")
    lengths = [inp.length for inp in inputs]
    frames = [inp.target_frames for inp in inputs]
    costs = [utterance_cost(L, F, decoding.steps) for L, F in zip(lengths, frames)]
    parts, _ = lpt_partition(costs, world)
    rows = [L + F for L, F in zip(lengths, frames)]

    payload = _Payload(rank=rank, ok=True, error="", results=[])
    try:
        for pack in pack_by_frames(parts[rank], frames, rows, max_rows):
            out = runner([inputs[i] for i in pack], decoding, [seeds[i] for i in pack])
            if len(out) != len(pack):
                raise RuntimeError("runner returned %d results for %d inputs" % (len(out), len(pack)))
            payload.results.extend(zip(pack, out))
    except Exception as failure:  # reported to rank 0, never raised across ranks
        payload = _Payload(rank=rank, ok=False, error=f"{type(failure).__name__}: {failure}",
                           results=[])

    if not distributed:
        if not payload.ok:
            raise WorkerFailed(0, payload.error)
        return _ordered(payload.results, len(inputs))

    gathered = [None] * world if rank == 0 else None
    try:
        dist.gather_object(payload, gathered, dst=0, group=group)
    except Exception as failure:
        if rank == 0:
            raise WorkerFailed(-1, f"a worker did not report: {failure}") from failure
        raise
    if rank != 0:
        return None
    collected = []
    for p in gathered:
        if not p.ok:
            raise WorkerFailed(p.rank, p.error)
        collected.extend(p.results)
    return _ordered(collected, len(inputs))


def _ordered(pairs, count):
    out = [None] * count
    for index, result in pairs:
        out[index] = result
    missing = [i for i, r in enumerate(out) if r is None]
    if missing:
        raise WorkerFailed(-1, f"no result for inputs {missing[:8]}")
    return out
