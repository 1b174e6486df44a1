"""Decoding parity pins (CPU): the reference's golden vectors
(tests/decoding_test.cpp:40-80 over tests/fixtures/generator_golden.json),
checked for the product's host code, for the oracle, and for the
reference's own decoding.cpp compiled from its sources (oracle/_ref)."""
from __future__ import annotations

import numpy as np
import pytest

from omnivoice_b200 import ConditionalInput, unmask_schedule


def test_schedule_matches_golden(decoding_golden, native, oracle_lib):
    cfg = decoding_golden["config"]
    for entry in decoding_golden["generate"]:
        total = 8 * entry["target"]
        want = entry["schedule"]
        assert unmask_schedule(total, cfg["num_step"], cfg["t_shift"]) == want
        assert oracle_lib.schedule(total, cfg["num_step"], cfg["t_shift"]) == want
        ref = oracle_lib.reference_decoding()
        if ref is not None:
            out = np.empty(cfg["num_step"], np.uint64)
            ref.ref_unmask_schedule(total, cfg["num_step"], cfg["t_shift"], out.ctypes.data)
            assert [int(x) for x in out] == want


def test_conditional_input_matches_golden(decoding_golden, native):
    for entry in decoding_golden["generate"]:
        ids = np.array(entry["input_ids"], np.int32)
        start = entry["audio_start"]
        ref = entry["reference_codes"]
        ref = None if ref is None else np.array(ref, np.int32)
        inp = ConditionalInput.build(ids[0, :start].tolist(), ref, entry["target"], 8, 1024)
        assert inp.length == ids.shape[1]
        assert inp.audio_start == start
        assert np.array_equal(inp.ids, ids)


def test_greedy_position_choice(oracle_lib):
    # tests/decoding_test.cpp:67-80: two codebooks of three frames, codebook
    # 1 pays a penalty of 5, temperature 0.
    codes = np.array([[1024, 7, 1024], [1024, 1024, 1024]], np.int32)
    pred = np.array([[10, 11, 12], [13, 14, 15]], np.int32)
    conf = np.array([[-0.5, -0.1, -2.0], [-0.2, -0.3, -9.0]], np.float32)
    out, chosen = oracle_lib.select(2, pred, conf, codes, temperature=0.0)
    assert chosen == [0, 2]
    assert out.tolist() == [[10, 7, 12], [1024, 1024, 1024]]


@pytest.mark.parametrize("seed", [0, 1, 7, 12345])
def test_schedules_agree_with_reference_sources(oracle_lib, seed):
    ref = oracle_lib.reference_decoding()
    rng = np.random.default_rng(seed)
    for _ in range(50):
        total = int(rng.integers(1, 20000))
        steps = int(rng.integers(1, 65))
        shift = float(rng.choice([0.1, 0.5, 1.0, 0.05]))
        mine = unmask_schedule(total, steps, shift)
        assert sum(mine) == total
        assert oracle_lib.schedule(total, steps, shift) == mine
        if ref is not None:
            out = np.empty(steps, np.uint64)
            ref.ref_unmask_schedule(total, steps, shift, out.ctypes.data)
            assert [int(x) for x in out] == mine


@pytest.mark.parametrize("seed", [0, 3, 99])
def test_selector_matches_reference_fill_bit_exact(oracle_lib, seed):
    """oracle select + the reference's mt19937_64 Gumbel stream == the
    reference's PositionSelector::Fill over a whole multi-step run,
    including ties, already-unmasked slots and greedy mode."""
    ref = oracle_lib.reference_decoding()
    if ref is None:
        pytest.skip("reference decoding.cpp not built (no reference tree)")
    rng = np.random.default_rng(seed)
    for temperature in (5.0, 0.0):
        c, f = 8, int(rng.integers(3, 90))
        n = c * f
        codes_ref = np.full(n, 1024, np.int32)
        codes_me = codes_ref.copy()
        sched = oracle_lib.schedule(n, 32, 0.1)
        stream = oracle_lib.reference_gumbel(seed, n * 32)
        used = 0
        first = True
        for step, count in enumerate(sched):
            if count == 0:
                continue
            pred = rng.integers(0, 1024, size=n).astype(np.int32)
            conf = rng.normal(-2, 1, size=n).astype(np.float32)
            conf[rng.integers(0, n, size=n // 5)] = -1.0  # exact ties
            chosen_ref = np.empty(n, np.uint64)
            k = ref.ref_fill(1 if first else 0, seed, 5.0, temperature, count, c, f,
                             pred.ctypes.data, conf.ctypes.data, 1024, codes_ref.ctypes.data,
                             chosen_ref.ctypes.data)
            first = False
            g = None
            if temperature > 0:
                g = stream[used:used + n]
                used += n
            out, chosen = oracle_lib.select(count, pred.reshape(c, f), conf.reshape(c, f),
                                            codes_me.reshape(c, f), temperature=temperature,
                                            gumbel=g)
            codes_me = out.reshape(-1)
            assert chosen == [int(x) for x in chosen_ref[:k]]
            assert np.array_equal(codes_me, codes_ref)
        assert (codes_me != 1024).all()
