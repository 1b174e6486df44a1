"""End-to-end parity of the generator on the B200 against the CPU oracle,
through the generator C-ABI (ov_generator.h), in the shape of the
reference's tests/generator_test.cpp: forward logits, the scoring step and
full generations, plus batching, cancellation and error reporting.

Tolerances (north star): logits within 2e-2 absolute of the oracle's
fp32-accumulated fp16 restatement; predictions and position choices bit
exact given identical logits / scores and noise; final codes >= 99.5 %
equal with the same injected noise."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import check_argmax_exact, oracle_config_from, small_config
from model_files import write_synthetic_model
from omnivoice_b200 import (Cancelled, ConditionalInput, DecodingConfig, Generator,
                            GeneratorError, model_config)

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


def make_input(rng, text, ref_frames, target, vocab=151936):
    text_ids = rng.integers(0, vocab, size=text).tolist()
    ref = rng.integers(0, 1024, size=(8, ref_frames)).astype(np.int32) if ref_frames else None
    return ConditionalInput.build(text_ids, ref, target)


@pytest.fixture(scope="module")
def small(cuda_device, native, oracle_lib):
    cfg = small_config()
    gen = Generator.synthetic(cfg, weight_seed=3)
    oracle = oracle_lib.OracleModel(oracle_config_from(cfg), 3)
    yield cfg, gen, oracle
    gen.close()
    oracle.close()


def test_forward_matches_oracle_small(small):
    cfg, gen, oracle = small
    rng = np.random.default_rng(0)
    for text, ref, target in [(10, 0, 20), (30, 40, 64), (1, 0, 1), (50, 100, 130)]:
        inp = make_input(rng, text, ref, target, cfg.vocab_size)
        # Partly unmasked target, as the reference's forward fixture.
        inp.ids[:, inp.length - target::3] = rng.integers(0, 1024, size=inp.ids[:, inp.length - target::3].shape)
        got = gen.forward(inp)
        want = oracle.forward(inp.ids, inp.audio_start, target)
        assert np.abs(got - want).max() < LOGIT_TOL


def test_score_is_exact_on_identical_logits(small, oracle_lib):
    cfg, gen, _ = small
    rng = np.random.default_rng(1)
    inp = make_input(rng, 20, 0, 90, cfg.vocab_size)
    logits = gen.forward(inp)
    pred, conf = gen.score(inp, 2.0)
    want_p, want_c = oracle_lib.score(logits, 90)
    check_argmax_exact(pred, logits, 90)
    assert np.abs(conf - want_c).max() < 1e-4


def test_generate_matches_oracle_with_reference_noise(small):
    cfg, gen, oracle = small
    rng = np.random.default_rng(2)
    for text, ref, target, temperature, seed in [(12, 0, 40, 5.0, 0), (20, 30, 60, 5.0, 7),
                                                 (8, 0, 25, 0.0, 0)]:
        inp = make_input(rng, text, ref, target, cfg.vocab_size)
        dec = DecodingConfig(position_temperature=temperature)
        res = gen.generate(inp, dec, seed, noise="reference")
        codes, when = oracle.generate(inp.ids, inp.audio_start, target, temperature=temperature,
                                      seed=seed)
        assert ((res.codes >= 0) & (res.codes < 1024)).all()
        assert (res.codes == codes).mean() >= 0.995
        assert (res.unmasked_at == when).mean() >= 0.995


def test_generate_is_deterministic_and_device_noise_valid(small):
    cfg, gen, _ = small
    rng = np.random.default_rng(3)
    inp = make_input(rng, 16, 0, 50, cfg.vocab_size)
    dec = DecodingConfig()
    a = gen.generate(inp, dec, 11, noise="device")
    b = gen.generate(inp, dec, 11, noise="device")
    c = gen.generate(inp, dec, 12, noise="device")
    assert np.array_equal(a.codes, b.codes) and np.array_equal(a.unmasked_at, b.unmasked_at)
    assert not np.array_equal(a.unmasked_at, c.unmasked_at)
    from omnivoice_b200 import unmask_schedule
    sched = unmask_schedule(8 * 50, 32, 0.1)
    for step, count in enumerate(sched):
        assert (a.unmasked_at == step).sum() == count


def test_batch_matches_single_generations(small):
    cfg, gen, _ = small
    rng = np.random.default_rng(4)
    inputs = [make_input(rng, t, r, f, cfg.vocab_size) for t, r, f in
              [(10, 0, 30), (25, 50, 80), (5, 0, 12)]]
    seeds = [1, 2, 3]
    dec = DecodingConfig()
    batch = gen.generate_batch(inputs, dec, seeds, noise="reference")
    for inp, seed, res in zip(inputs, seeds, batch):
        single = gen.generate(inp, dec, seed, noise="reference")
        assert (single.codes == res.codes).mean() >= 0.995


def test_cancellation_reports_cancelled(small):
    cfg, gen, _ = small
    rng = np.random.default_rng(5)
    inp = make_input(rng, 10, 0, 30, cfg.vocab_size)
    calls = []

    def cancelled():
        calls.append(1)
        return len(calls) > 3

    with pytest.raises(Cancelled) as e:
        gen.generate(inp, DecodingConfig(), 0, cancelled=cancelled)
    assert str(e.value) == "cancelled"
    # The generator stays usable after a cancellation.
    assert gen.generate(inp, DecodingConfig(), 0).codes.shape == (8, 30)


def test_errors_carry_reference_prefixes(small):
    cfg, gen, _ = small
    inp = ConditionalInput.build([cfg.vocab_size + 5], None, 4)
    with pytest.raises(GeneratorError) as e:
        gen.forward(inp)
    assert str(e.value) == "OmniVoice forward: text token outside the vocabulary"
    with pytest.raises(GeneratorError) as e:
        gen.score(inp, 2.0)
    assert str(e.value).startswith("OmniVoice score: ")


def test_safetensors_load_equals_synthetic(small, native, tmp_path):
    cfg, gen, _ = small
    H, I = cfg.hidden_size, cfg.intermediate_size
    path = tmp_path / "model.safetensors"
    write_synthetic_model(path, cfg, 3, native)
    loaded = Generator.load(cfg, str(path))
    rng = np.random.default_rng(6)
    inp = make_input(rng, 9, 10, 33, cfg.vocab_size)
    assert np.array_equal(loaded.forward(inp), gen.forward(inp))
    loaded.close()
    with pytest.raises(GeneratorError) as e:
        Generator.load(model_config(layers=cfg.layers + 1, vocab_size=cfg.vocab_size,
                                    hidden_size=H, intermediate_size=I, heads=cfg.heads,
                                    kv_heads=cfg.kv_heads), str(path))
    assert str(e.value).startswith("OmniVoice generator: missing tensor")


def test_forward_full_model_config1_matches_oracle(cuda_device, native, oracle_lib):
    """BASELINE config 1 shape (40 text + 100 target, 28 layers, full
    vocabulary) for one CFG forward, against the oracle."""
    cfg = model_config()
    gen = Generator.synthetic(cfg, weight_seed=0)
    rng = np.random.default_rng(0)
    inp = make_input(rng, 40, 0, 100)
    got = gen.forward(inp)
    gen.close()
    oracle = oracle_lib.OracleModel(oracle_config_from(cfg), 0)
    want = oracle.forward(inp.ids, inp.audio_start, 100)
    oracle.close()
    diff = np.abs(got - want)
    print(f"config-1 forward: max |d logit| {diff.max():.3e}, mean {diff.mean():.3e}")
    assert diff.max() < LOGIT_TOL
