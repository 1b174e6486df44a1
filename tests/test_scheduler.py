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


def _parse(out):
    assert out.startswith("ok"), out
    lines = out.splitlines()[1:]
    producers = {int(a): int(b) for a, b in (l.split() for l in lines if not l.startswith("failure"))}
    failed = [int(l.split()[1]) for l in lines if l.startswith("failure")]
    assert sorted(producers) == list(range(10))
    return producers, failed


def _parts(world):
    inputs = dp_workers.make_inputs()
    costs = [utterance_cost(x.length, x.target_frames) for x in inputs]
    return lpt_partition(costs, world)[0], costs


def test_two_ranks_gather_results_in_input_order(tmp_path):
    producers, failed = _parse(_run("ok", tmp_path))
    assert failed == []
    parts, _ = _parts(2)
    for rank, part in enumerate(parts):
        assert all(producers[i] == rank for i in part)
    assert set(producers.values()) == {0, 1}


def test_a_failing_rank_is_requeued_to_the_survivors(tmp_path):
    producers, failed = _parse(_run("raise", tmp_path))
    assert failed == [1]
    # Every utterance of the failed rank was generated again by rank 0.
    assert set(producers.values()) == {0}


def test_a_rank_that_never_reports_is_requeued(tmp_path):
    producers, failed = _parse(_run("vanish", tmp_path))
    assert failed == [1]
    assert set(producers.values()) == {0}


def test_finished_packs_of_a_failing_rank_are_kept(tmp_path):
    producers, failed = _parse(_run("partial", tmp_path))
    assert failed == [1]
    parts, _ = _parts(2)
    mine = [i for i in parts[1] if producers[i] == 1]
    assert mine and len(mine) < len(parts[1])  # the first pack's results survive
    assert all(producers[i] == 0 for i in parts[0])


def test_three_ranks_share_the_work_of_one_that_vanished(tmp_path):
    producers, failed = _parse(_run("vanish", tmp_path, world=3))
    assert failed == [2]
    parts, costs = _parts(3)
    lost = parts[2]
    # Re-partitioned by LPT over the two survivors.
    again, _ = lpt_partition([costs[i] for i in lost], 2)
    for rank, part in enumerate(again):
        assert all(producers[lost[j]] == rank for j in part)
    for rank in (0, 1):
        assert all(producers[i] == rank for i in parts[rank])


def test_no_survivor_ends_in_worker_failed(tmp_path):
    out = _run("all_raise", tmp_path)
    assert out.startswith("failed "), out
    assert "injected failure" in out
