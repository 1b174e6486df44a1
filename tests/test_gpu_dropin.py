"""The C++ drop-in API (csrc/host/generator.hpp and gemm.hpp, the
reference's generator.hpp:16-56 and gemm.hpp:12-71) on the B200.

tests/cpp/dropin_test.cpp loads a model.safetensors through
Generator::Load, runs Forward, Score, Generate and GenerateBatch, checks
error prefixes, cancellation and HalfGemm against a float64 host product,
and writes its results; here they must equal, bit for bit, what the C-ABI
generator (the Python mirror) computes on the same weights and input."""
from __future__ import annotations

import subprocess

import numpy as np
import pytest

from conftest import small_config
from model_files import write_synthetic_model
from omnivoice_b200 import ConditionalInput, DecodingConfig, Generator

pytestmark = pytest.mark.gpu


def test_cpp_dropin_matches_the_c_abi(cuda_device, native, tmp_path):
    from omnivoice_b200.build import build_test_programs
    exe = [p for p in build_test_programs() if p.name == "dropin_test"][0]
    cfg = small_config()
    write_synthetic_model(tmp_path / "model.safetensors", cfg, 3, native)
    out = tmp_path / "out"
    out.mkdir()
    run = subprocess.run([str(exe), str(tmp_path), str(out), str(cfg.vocab_size),
                          str(cfg.hidden_size), str(cfg.intermediate_size), str(cfg.layers),
                          str(cfg.heads), str(cfg.kv_heads)],
                         capture_output=True, text=True, timeout=600)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr

    length, audio_start, frames = np.fromfile(out / "meta.i32", np.int32).tolist()
    ids = np.fromfile(out / "ids.i32", np.int32).reshape(8, length)
    inp = ConditionalInput(codebooks=8, length=length, audio_start=audio_start,
                           target_frames=frames, ids=ids)
    gen = Generator.synthetic(cfg, weight_seed=3)
    try:
        logits = gen.forward(inp)
        assert np.array_equal(np.fromfile(out / "forward.f32", np.float32), logits.ravel())
        pred, conf = gen.score(inp, 2.0)
        assert np.array_equal(np.fromfile(out / "prediction.i32", np.int32), pred.ravel())
        assert np.array_equal(np.fromfile(out / "confidence.f32", np.float32), conf.ravel())
        res = gen.generate(inp, DecodingConfig(), 7, noise="reference")
        assert np.array_equal(np.fromfile(out / "codes.i32", np.int32), res.codes.ravel())
        assert np.array_equal(np.fromfile(out / "unmasked.i32", np.int32),
                              res.unmasked_at.ravel())
    finally:
        gen.close()
