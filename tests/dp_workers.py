"""Rank bodies for the multi-process scheduler tests (gloo on CPU).

Each rank runs generate_data_parallel with a fake runner that stands in
for a GPU generator: it returns, per input, the rank that produced it and
a code array derived from the seed, so rank 0 can check both the
partition and the order of the gathered results."""
from __future__ import annotations

import datetime
import os
import sys
import traceback
from dataclasses import dataclass
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


@dataclass
class FakeInput:
    length: int
    target_frames: int


@dataclass
class FakeDecoding:
    steps: int = 32


def make_inputs():
    frames = [50, 750, 300, 120, 640, 75, 410, 222, 90, 505]
    return [FakeInput(length=int(f * 1.6), target_frames=f) for f in frames]


def _init(rank, world, port, timeout_s):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def worker(rank, world, port, mode, out_dir):
    """mode: "ok" | "raise" (rank 1's runner fails) | "vanish" (the last
    rank exits without reporting) | "partial" (rank 1 fails on its second
    pack) | "all_raise" (every runner fails).  Rank 0 writes its outcome to
    out_dir/rank0.txt: "ok", then per input its index and producing rank,
    then a line per failed rank; or "failed <rank> <message>"."""
    import numpy as np

    from omnivoice_b200.scheduler import WorkerFailed, generate_data_parallel
    dist = _init(rank, world, port, 60)
    inputs = make_inputs()
    seeds = [100 + i for i in range(len(inputs))]
    calls = []

    def runner(batch, decoding, batch_seeds):
        calls.append(len(batch))
        if mode == "all_raise" or (mode == "raise" and rank == 1):
            raise RuntimeError("injected failure")
        if mode == "partial" and rank == 1 and len(calls) == 2:
            raise RuntimeError("injected failure on the second pack")
        return [(rank, np.full((8, inp.target_frames), s % 1024, np.int32))
                for inp, s in zip(batch, batch_seeds)]

    if mode == "vanish" and rank == world - 1:
        os._exit(0)  # leaves between steps, before reporting
    outcome = ""
    failures = []
    try:
        res = generate_data_parallel(inputs, FakeDecoding(), seeds, runner, max_rows=1500,
                                     heartbeat_timeout=3.0, failures=failures)
        if rank == 0:
            lines = []
            for i, (r, codes) in enumerate(res):
                assert codes.shape == (8, inputs[i].target_frames)
                assert int(codes[0, 0]) == seeds[i] % 1024
                lines.append(f"{i} {r}")
            lines += [f"failure {r} {m}" for r, m in failures]
            outcome = "ok\n" + "\n".join(lines)
        else:
            assert res is None
    except WorkerFailed as failure:
        outcome = f"failed {failure.rank} {failure}"
    except Exception:
        outcome = "error " + traceback.format_exc()
    if rank == 0:
        Path(out_dir, "rank0.txt").write_text(outcome)
    if mode != "vanish":
        dist.destroy_process_group()
