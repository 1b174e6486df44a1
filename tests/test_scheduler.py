"""Host side of the multi-GPU path: the LPT partition, packing, and the
gather of results across ranks, with failures injected on the host (a rank
whose generation raises, a rank that leaves without reporting).  The ranks
are gloo processes on the CPU."""
import socket

import pytest
import torch.multiprocessing as mp

import dp_workers
from omnivoice_b200.scheduler import (FLOPS_PER_ROW, lpt_partition, pack_by_frames,
                                      utterance_cost)


def test_cost_model_matches_the_flop_count():
    # R * 880.80 M + 229,376 * sum L_s^2 + 2F * 16.79 M per step.
    assert FLOPS_PER_ROW == 880_803_840
    L, F = 370, 250
    per_step = utterance_cost(L, F, steps=1)
    expected = 620 * 880_803_840 + 229_376 * (370 ** 2 + 250 ** 2) + 2 * 250 * 2 * 1024 * 8200
    assert per_step == expected
    assert abs(per_step / 1e9 - 600.2) < 0.1  # config 2: 600.2 GFLOP per step


def test_lpt_partition_covers_every_item_once_and_balances():
    costs = [utterance_cost(int(1.6 * f), f) for f in
             [50, 750, 300, 120, 640, 75, 410, 222, 90, 505, 333, 610, 58, 700]]
    for workers in (1, 2, 4, 8):
        parts, load = lpt_partition(costs, workers)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(costs)))
        assert abs(sum(load) - sum(costs)) < 1e-6 * sum(costs)
        for p, l in zip(parts, load):
            assert abs(sum(costs[i] for i in p) - l) < 1e-6 * l + 1
        # LPT bound: makespan <= 4/3 of optimal; optimal >= max(mean, largest item).
        lower = max(sum(costs) / workers, max(costs))
        assert max(load) <= 4 / 3 * lower + 1e-6 * lower
    assert lpt_partition(costs, 4) == lpt_partition(costs, 4)  # deterministic


def test_lpt_partition_rejects_no_workers():
    with pytest.raises(ValueError):
        lpt_partition([1.0], 0)


def test_pack_by_frames_respects_the_row_budget():
    frames = [50, 750, 300, 120, 640, 75]
    rows = [int(2.6 * f) for f in frames]
    packs = pack_by_frames(range(6), frames, rows, max_rows=2000)
    assert sorted(i for p in packs for i in p) == list(range(6))
    for p in packs:
        assert len(p) == 1 or sum(rows[i] for i in p) <= 2000
        # frames non-increasing inside and across packs
    order = [i for p in packs for i in p]
    assert [frames[i] for i in order] == sorted(frames, reverse=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(mode, tmp_path, world=2):
    ctx = mp.start_processes(dp_workers.worker, args=(world, _free_port(), mode, str(tmp_path)),
                             nprocs=world, join=False, start_method="spawn")
    while not ctx.join(timeout=120):
        pass
    return (tmp_path / "rank0.txt").read_text()


def test_two_ranks_gather_results_in_input_order(tmp_path):
    out = _run("ok", tmp_path)
    assert out.startswith("ok"), out
    rows = [line.split() for line in out.splitlines()[1:]]
    assert [int(i) for i, _ in rows] == list(range(10))
    producers = {int(i): int(r) for i, r in rows}
    inputs = dp_workers.make_inputs()
    costs = [utterance_cost(x.length, x.target_frames) for x in inputs]
    parts, _ = lpt_partition(costs, 2)
    for rank, part in enumerate(parts):
        assert all(producers[i] == rank for i in part)
    assert set(producers.values()) == {0, 1}


def test_a_failing_rank_is_reported_by_rank_zero(tmp_path):
    out = _run("raise", tmp_path)
    assert out.startswith("failed 1"), out
    assert "injected failure" in out


def test_a_rank_that_never_reports_ends_in_an_error(tmp_path):
    out = _run("vanish", tmp_path)
    assert out.startswith("failed -1"), out
