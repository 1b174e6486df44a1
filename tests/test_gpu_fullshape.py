"""Generator parity on the full model shape (28 layers, hidden 1024, 16/8
heads, vocabulary 151936, random-init weights of seed 0) at BASELINE.json's
configurations, in the shape of the reference's tests/generator_test.cpp
(:76-175, driving Generator::Generate of generator.cpp:486-543 on the real
model shape):

  * config 1: the full 32-step CFG generation with the reference's noise
    stream, against the oracle's generation stored in
    tests/golden/generation_golden.npz (made by make_generation_golden.py);
  * configs 1, 2 and 3 (with reference codes): step by step on the oracle's
    own 32-step trajectory (the same ids into both forwards at every step);
  * configs 2, 3 and 5: one CFG forward each against the oracle's forward
    (computed here), logits within 2e-2 absolute; the scores of those
    logits with exact argmax outside the float32 tie band;
  * config 4: six of its utterances generated as one packed batch
    (ov_generator_generate_batch) against the stored oracle generations.

The bars.  Logits within 2e-2 of the fp32-accumulated fp16 restatement
(north star).  For codes: at random init the 32-step generation is
chaotic, since near-flat logits make the choice of positions and classes
flip on float32 rounding, and one early flip changes every later step's
input.  The fixture measures this on the oracle itself: the same
restatement with its linear layers' float32 sums in the opposite order
(just as valid: hipBLAS leaves the order unspecified) agrees with the
oracle on 68 % of config 1's codes, and on 61-100 % of the config-4
utterances'.  A free-running comparison therefore says where two
trajectories part, not how close the arithmetic is, so it is reported
(next to the reversed-sum restatement's figure) and asserted only on
what does not depend on the trajectory: valid codes and every step
unmasking exactly its scheduled count.  The parity bar is asserted step
by step on the oracle's own config-1, 2 and 3 trajectories (the same ids
into both forwards at every step): predictions at the masked positions at
least as close as the reversed-sum restatement's, or 99 %, and 99 % of the
chosen positions.  Every comparison prints its figure.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from conftest import check_argmax_exact, oracle_config_from
from omnivoice_b200 import ConditionalInput, DecodingConfig, Generator, model_config

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2
VOCAB = 151936
GOLDEN = Path(__file__).resolve().parent / "golden" / "generation_golden.npz"


@pytest.fixture(scope="module")
def full(cuda_device, native):
    gen = Generator.synthetic(model_config(), weight_seed=0)
    yield gen
    gen.close()


@pytest.fixture(scope="module")
def golden_data():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def golden(golden_data):
    data = golden_data
    out = {}
    for name in data["names"]:
        name = str(name)
        audio_start, frames, seed = (int(v) for v in data[f"{name}_meta"])
        ids = data[f"{name}_ids"]
        inp = ConditionalInput(8, ids.shape[1], audio_start, frames, np.ascontiguousarray(ids))
        out[name] = (inp, seed, data[f"{name}_codes"], data[f"{name}_unmasked_at"])
    return out


def _agreement(name, res, codes, when):
    """Prints the agreement of a free-running generation with the oracle's
    and asserts what holds on any trajectory: valid codes, and each step
    unmasking exactly its scheduled count (decoding.cpp:12-40)."""
    from oracle import binding
    same_codes = float((res.codes == codes).mean())
    same_when = float((res.unmasked_at == when).mean())
    parted = [s for s in range(32) if not np.array_equal(res.unmasked_at == s, when == s)]
    print(f"{name}: codes {same_codes:.4f} equal, unmasked_at {same_when:.4f} equal "
          f"({int((res.codes != codes).sum())} of {codes.size} codes differ; first step "
          f"choosing other positions: {parted[0] if parted else 'none'})")
    assert ((res.codes >= 0) & (res.codes < 1024)).all()
    sched = binding.schedule(codes.size, 32, 0.1)
    assert [int((res.unmasked_at == s).sum()) for s in range(32)] == sched
    return same_codes, same_when


def test_generate_config1_full_model_matches_oracle(full, golden, golden_data):
    inp, seed, codes, when = golden["c1"]
    res = full.generate(inp, DecodingConfig(), seed, noise="reference")
    same_codes, same_when = _agreement("config 1", res, codes, when)
    v_codes, v_when = golden_data["c1_variant_agreement"][:2]
    print(f"config 1: the reversed-sum oracle agrees {v_codes:.4f} / {v_when:.4f}")


@pytest.mark.parametrize("case", ["c1", "c2", "c3"])
def test_steps_on_the_oracle_trajectory(full, golden, golden_data, case):
    """Every step of the oracle's config-1 / 2 / 3 generation, fed to the
    GPU with the oracle's ids: the predictions at the masked positions, and
    the positions the selection picks from the GPU's confidences with the
    step's reference noise, against the oracle's."""
    from oracle import binding
    inp, seed, _, _ = golden[case]
    step_ids = golden_data[f"{case}_step_ids"]
    step_pred = golden_data[f"{case}_step_prediction"]
    step_conf = golden_data[f"{case}_step_confidence"]
    F = inp.target_frames
    total = 8 * F
    sched = binding.schedule(total, 32, 0.1)
    gumbel = binding.reference_gumbel(seed, total * sum(1 for c in sched if c > 0))
    same_pred = masked_total = same_pick = picked_total = 0
    draw = 0
    for step, count in enumerate(sched):
        if count == 0:
            continue
        ids = step_ids[step]
        step_inp = ConditionalInput(8, inp.length, inp.audio_start, F, np.ascontiguousarray(ids))
        pred, conf = full.score(step_inp, 2.0)
        codes = ids[:, inp.length - F:]
        masked = codes == 1024
        same_pred += int((pred == step_pred[step])[masked].sum())
        masked_total += int(masked.sum())
        g = gumbel[draw * total:(draw + 1) * total]
        draw += 1
        _, mine = binding.select(count, pred, conf, codes, gumbel=g)
        _, want = binding.select(count, step_pred[step], step_conf[step], codes, gumbel=g)
        same_pick += len(set(mine) & set(want))
        picked_total += len(want)
    pred_agree = same_pred / masked_total
    pick_agree = same_pick / picked_total
    variant = float(golden_data[f"{case}_variant_agreement"][2])
    print(f"{case} step by step: predictions {pred_agree:.4f} equal at masked positions "
          f"({masked_total - same_pred} of {masked_total} differ), chosen positions "
          f"{pick_agree:.4f}; the reversed-sum oracle's predictions {variant:.4f}")
    assert pred_agree >= min(0.99, variant)
    assert pick_agree >= 0.99


def test_generate_config4_subset_batch_matches_oracle(full, golden, golden_data):
    names = sorted(n for n in golden if n.startswith("c4_"))
    assert len(names) == 6
    inputs = [golden[n][0] for n in names]
    seeds = [golden[n][1] for n in names]
    results = full.generate_batch(inputs, DecodingConfig(), seeds, noise="reference")
    total = same = 0
    v_same = 0.0
    for name, res in zip(names, results):
        _, _, codes, when = golden[name]
        c, w = _agreement(f"config 4 {name}", res, codes, when)
        v_codes, v_when = golden_data[f"{name}_variant_agreement"][:2]
        print(f"  the reversed-sum oracle agrees {v_codes:.4f} / {v_when:.4f}")
        total += codes.size
        same += int((res.codes == codes).sum())
        v_same += v_codes * codes.size
    print(f"config 4 subset: {same / total:.4f} of {total} codes equal "
          f"(reversed-sum oracle {v_same / total:.4f})")


def _config_input(text, ref, target, seed):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, VOCAB, size=text).tolist()
    codes = rng.integers(0, 1024, size=(8, ref)).astype(np.int32) if ref else None
    inp = ConditionalInput.build(ids, codes, target)
    # Part of the target already unmasked, as in the middle of a generation.
    tail = inp.ids[:, inp.length - target:]
    tail[:, ::3] = rng.integers(0, 1024, size=tail[:, ::3].shape)
    return inp


@pytest.mark.parametrize("name,text,ref,target,seed", [
    ("config 2", 120, 0, 250, 1),
    ("config 3", 180, 150, 375, 2),
    ("config 5", 300, 375, 750, 3),
])
def test_forward_full_model_matches_oracle(full, oracle_lib, name, text, ref, target, seed):
    inp = _config_input(text, ref, target, seed)
    got = full.forward(inp)
    oracle = oracle_lib.OracleModel(oracle_config_from(model_config()), 0)
    want = oracle.forward(inp.ids, inp.audio_start, target)
    oracle.close()
    diff = np.abs(got - want)
    print(f"{name} forward (L={inp.length}, F={target}): max |d logit| {diff.max():.3e}, "
          f"mean {diff.mean():.3e}")
    assert diff.max() < LOGIT_TOL
    pred, conf = full.score(inp, 2.0)
    check_argmax_exact(pred, got, target)
    want_p, want_c = oracle_lib.score(got, target)
    assert np.abs(conf - want_c).max() < 1e-4
