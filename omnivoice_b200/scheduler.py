"""Data-parallel generation over several GPUs, one process (rank) per GPU.

Each rank holds a full replica of the generator (the 0.6 B backbone fits
any B200 many times over); one generation is never split across GPUs,
because every unmasking step depends on the previous one.  A batch of
utterances is partitioned on the host by longest-processing-time first
(LPT) over the hot path's cost model, each rank generates its share as
packed batches through its own generator, and the finished codes come back
to rank 0 through host memory: the key-value store the processes already
share for their rendezvous (torch.distributed's TCPStore).  There is no
collective and no NCCL anywhere on this path.

The reference serves one request at a time per GPU worker
(gufo-extensions/omnivoice README.md:78, synthesizer.cpp:163-201, and the
runner's per-request loop, runner.cpp:78-114); this module is the scheduler
that batching across utterances and GPUs needs.

Failures are detected on the host and the work of a failed rank is
re-queued to the survivors.  Every rank beats a heartbeat counter in the
store while it works; rank 0 coordinates.  A rank whose generation raises
reports the error (and any packs it finished); a rank whose heartbeat
stops (it exited or was killed) is failed by rank 0 after
`heartbeat_timeout` seconds.  Rank 0 then partitions the unfinished
utterances over the surviving ranks (LPT again) and publishes that plan as
the next round; the failed ranks take no further part.  WorkerFailed is
raised only when no rank survives (or rank 0 itself disappears, which the
other ranks notice from its heartbeat).
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
    results: list  # [(index, result)] of the packs that finished


_calls = 0  # generate_data_parallel calls made by this process (the same on every rank)


class _Heartbeat:
    """Adds 1 to this rank's heartbeat counter in the store every `period`
    seconds from a daemon thread while the call runs."""

    def __init__(self, store, key: str, period: float):
        import threading
        self.store, self.key, self.period = store, key, period
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._beat, daemon=True)

    def _beat(self):
        while not self.stop.is_set():
            try:
                self.store.add(self.key, 1)
            except Exception:  # the store went away: nothing left to tell
                return
            self.stop.wait(self.period)

    def __enter__(self):
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)


def _counter(store, key: str) -> int:
    return int(store.add(key, 0))


def _wait_for(store, key: str, beat_key: str, heartbeat_timeout: float, poll: float = 0.01):
    """Polls until `key` is in the store (True) or the heartbeat counter at
    `beat_key` has not moved for `heartbeat_timeout` seconds (False)."""
    import time
    last = _counter(store, beat_key)
    moved = time.monotonic()
    while True:
        if store.check([key]):
            return True
        now = time.monotonic()
        beat = _counter(store, beat_key)
        if beat != last:
            last, moved = beat, now
        elif now - moved > heartbeat_timeout:
            return store.check([key])
        time.sleep(poll)


def _run_share(rank, items, inputs, decoding, seeds, runner, frames, rows, max_rows) -> _Payload:
    payload = _Payload(rank=rank, ok=True, error="", results=[])
    try:
        for pack in pack_by_frames(items, frames, rows, max_rows):
            out = runner([inputs[i] for i in pack], decoding, [seeds[i] for i in pack])
            if len(out) != len(pack):
                raise RuntimeError("runner returned %d results for %d inputs" % (len(out), len(pack)))
            payload.results.extend(zip(pack, out))
    except Exception as failure:  # reported to rank 0, never raised across ranks
        payload.ok = False
        payload.error = f"{type(failure).__name__}: {failure}"
    return payload


def generate_data_parallel(inputs: Sequence, decoding, seeds: Sequence[int],
                           runner: Callable[[list, object, list], list],
                           group=None, max_rows: int = 1 << 17, store=None,
                           heartbeat_timeout: float = 30.0, heartbeat_period: float = 0.25,
                           failures: list | None = None) -> list | None:
    """Generates every input across the ranks of `group` (the default
    torch.distributed group; a single process when torch.distributed is
    not initialised).

    `runner(inputs, decoding, seeds)` generates one packed batch on this
    rank's GPU and returns one result per input (Generator.generate_batch).
    Every rank calls this with the same arguments, the same number of times
    and in the same order.  Rank 0 returns the results in input order; the
    other ranks return None.  `store` is the host key-value store the ranks
    share (default: the process group's rendezvous store).  On rank 0,
    `failures` (a list) receives one (rank, message) per failed rank."""
    import pickle

    import torch.distributed as dist

    global _calls
    distributed = dist.is_available() and dist.is_initialized()
    rank = dist.get_rank(group) if distributed else 0
    world = dist.get_world_size(group) if distributed else 1
    if len(seeds) != len(inputs):
        raise ValueError("one seed per input")
    lengths = [inp.length for inp in inputs]
    frames = [inp.target_frames for inp in inputs]
    costs = [utterance_cost(L, F, decoding.steps) for L, F in zip(lengths, frames)]
    rows = [L + F for L, F in zip(lengths, frames)]

    if not distributed or world == 1:
        parts, _ = lpt_partition(costs, 1)
        payload = _run_share(0, parts[0], inputs, decoding, seeds, runner, frames, rows, max_rows)
        if not payload.ok:
            raise WorkerFailed(0, payload.error)
        return _ordered(payload.results, len(inputs))

    if store is None:
        from torch.distributed import distributed_c10d
        store = distributed_c10d._get_default_store()
    _calls += 1
    prefix = f"ov_dp/{_calls}"
    beat = [f"{prefix}/hb/{r}" for r in range(world)]
    alive = list(range(world))
    pending = list(range(len(inputs)))
    done: dict[int, object] = {}
    with _Heartbeat(store, beat[rank], heartbeat_period):
        for round_ in range(world + 1):
            sub, _ = lpt_partition([costs[i] for i in pending], len(alive))
            share = {r: [pending[j] for j in part] for r, part in zip(alive, sub)}
            if rank in share:
                payload = _run_share(rank, share[rank], inputs, decoding, seeds, runner, frames,
                                     rows, max_rows)
                store.set(f"{prefix}/r{round_}/{rank}", pickle.dumps(payload))
            plan_key = f"{prefix}/plan{round_}"
            if rank != 0:
                if not _wait_for(store, plan_key, beat[0], heartbeat_timeout):
                    raise WorkerFailed(0, "the coordinating rank stopped beating")
                plan = pickle.loads(store.get(plan_key))
                if plan["done"]:
                    return None
                alive, pending = plan["alive"], plan["pending"]
                continue
            # Rank 0: collect this round's reports.
            failed = []
            for r in alive:
                key = f"{prefix}/r{round_}/{r}"
                if r != 0 and not _wait_for(store, key, beat[r], heartbeat_timeout):
                    failed.append((r, "stopped beating without reporting"))
                    continue
                got = pickle.loads(store.get(key))
                done.update(got.results)
                if not got.ok:
                    failed.append((r, got.error))
            if failures is not None:
                failures.extend(failed)
            alive = [r for r in alive if r not in {f for f, _ in failed}]
            pending = [i for i in pending if i not in done]
            if not pending:
                store.set(plan_key, pickle.dumps({"done": True}))
                return _ordered(list(done.items()), len(inputs))
            if not alive:
                store.set(plan_key, pickle.dumps({"done": True}))
                r, message = failed[0]
                raise WorkerFailed(r, message)
            store.set(plan_key, pickle.dumps({"done": False, "alive": alive, "pending": pending}))
    raise WorkerFailed(-1, "work left after every round")  # unreachable: a round loses a rank


def _ordered(pairs, count):
    out = [None] * count
    for index, result in pairs:
        out[index] = result
    missing = [i for i, r in enumerate(out) if r is None]
    if missing:
        raise WorkerFailed(-1, f"no result for inputs {missing[:8]}")
    return out
