"""The codec decoder oracle (oracle/codec.py) against the golden audio
that transformers' HiggsAudioV2Tokenizer decoder path produced on the same
seeded weights (tests/golden/make_codec_golden.py), plus the reference's
input checks (codec.cpp:207-214)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import codec as oc

GOLDEN = json.loads((Path(__file__).parent / "golden" / "codec_golden.json").read_text())


def shape_of(case):
    return oc.CodecShape(**case["shape"])


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=lambda c: c["name"])
def test_oracle_matches_transformers_golden(case):
    cfg = shape_of(case)
    weights = oc.synthetic_weights(cfg, case["weight_seed"])
    audio = oc.decode(weights, cfg, np.array(case["codes"]))
    assert len(audio) == case["length"] == len(case["codes"][0]) * cfg.frame_samples
    got = audio[::case["stride"]]
    want = np.array(case["samples"])
    # Stored with 9 significant digits.
    assert (np.abs(got - want) <= 1e-8 * np.abs(want) + 1e-9 * case["rms"]).all()
    assert abs(np.sqrt(np.mean(audio ** 2)) - case["rms"]) <= 1e-9 * case["rms"]


def test_oracle_rejects_bad_codes():
    cfg = shape_of(GOLDEN["cases"][0])
    weights = oc.synthetic_weights(cfg, 1)
    with pytest.raises(ValueError, match="outside the codebook"):
        oc.decode(weights, cfg, np.full((8, 2), 1024))
    with pytest.raises(ValueError, match="doesn't match"):
        oc.decode(weights, cfg, np.zeros((7, 2), np.int64))


def test_transposed_convolution_keeps_length_times_stride():
    rng = np.random.default_rng(0)
    for stride in (2, 3, 4, 5, 8):
        x = rng.standard_normal((3, 7))
        w = rng.standard_normal((3, 2, 2 * stride))
        y = oc.conv_transpose1d(x, w, np.zeros(2), stride)
        assert y.shape == (2, 7 * stride)
        # Direct definition: y[o][t] = sum_{i,j,k: t = j s + k - ceil(s/2)} w[i][o][k] x[i][j].
        pad = (stride + 1) // 2
        ref = np.zeros_like(y)
        for j in range(7):
            for k in range(2 * stride):
                t = j * stride + k - pad
                if 0 <= t < 7 * stride:
                    ref[:, t] += w[:, :, k].T @ x[:, j]
        assert np.allclose(y, ref)
