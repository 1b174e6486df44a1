"""The C-ABI library loads and exports every entry point include/*.h
declares, and its host-only helpers behave as documented (no GPU needed)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"\b(ov_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_every_declared_symbol_is_exported(native):
    missing = [n for n in sorted(declared_functions()) if not hasattr(native, n)]
    assert not missing, missing


def test_binding_covers_every_declaration():
    from omnivoice_b200 import _native
    assert declared_functions() - {"ov_cancel_fn"} <= set(_native.SIGNATURES)


def test_binding_constants_match_the_headers():
    """Every enumerator the headers define with a plain integer has the same
    value in the Python binding."""
    from omnivoice_b200 import _native
    seen = 0
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"\b(OV_[A-Z0-9_]+)\s*=\s*(\d+)\b", text):
            if hasattr(_native, m.group(1)):
                assert getattr(_native, m.group(1)) == int(m.group(2)), m.group(1)
                seen += 1
    assert seen >= 10


def test_last_error_is_empty_initially(native):
    from omnivoice_b200 import _native
    assert _native.last_error() == "" or isinstance(_native.last_error(), str)


def test_rope_tables_follow_hf_default(native):
    d, n, theta = 128, 64, 1e6
    cos = np.empty((n, d // 2), np.float32)
    sin = np.empty((n, d // 2), np.float32)
    assert native.ov_rope_tables(theta, d, n, cos.ctypes.data, sin.ctypes.data) == 0
    i = np.arange(d // 2, dtype=np.float32)
    inv = (1.0 / np.power(np.float32(theta), (2 * i) / np.float32(d))).astype(np.float32)
    ang = (np.arange(n, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    # One float32 ulp of inv_freq moves angles near 64 rad by ~4e-6.
    np.testing.assert_allclose(cos, np.cos(ang), atol=1e-5)
    np.testing.assert_allclose(sin, np.sin(ang), atol=1e-5)


def test_synthetic_weights_match_the_oracle_restatement(native, oracle_lib):
    for tensor, first, count in [(1, 0, 4096), (2, 12345, 1000), (64 + 4, 7, 3000)]:
        mine = np.empty(count, np.float32)
        assert native.ov_synthetic_fill_host(mine.ctypes.data, count, 7, tensor, 0.02, first) == 0
        theirs = np.empty(count, np.float32)
        oracle_lib.oracle().oc_synthetic_values(7, tensor, 0.02, first, count, theirs.ctypes.data)
        assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))


def test_synthetic_weights_are_roughly_normal(native):
    n = 1 << 18
    w = np.empty(n, np.float32)
    native.ov_synthetic_fill_host(w.ctypes.data, n, 0, 64 + 0, 0.02, 0)
    assert abs(w.mean()) < 2e-4
    assert abs(w.std() - 0.02) < 3e-4
    assert np.abs(w).max() < 0.02 * 3.5


def test_interleave_gate_up(native):
    width, cols = 128, 8
    g = np.arange(2 * width * cols, dtype=np.uint16).reshape(2 * width, cols)
    out = np.empty_like(g)
    assert native.ov_interleave_gate_up(g.ctypes.data, width, cols, out.ctypes.data) == 0
    G = 64
    for j in range(width):
        grp, r = divmod(j, G)
        assert np.array_equal(out[2 * grp * G + r], g[j])
        assert np.array_equal(out[2 * grp * G + G + r], g[width + j])


def test_gumbel_from_uniform(native):
    for u in [0.0, 0.25, 0.5, 0.999]:
        want = np.float32(-np.log(-np.log(np.float32(u) + np.float32(1e-10)) + np.float32(1e-10)))
        assert abs(native.ov_gumbel_from_uniform(u) - want) <= 1e-5 * max(1, abs(want))


def test_generator_errors_without_gpu_are_reported(native):
    from omnivoice_b200 import _native
    import torch
    if torch.cuda.is_available():
        return
    h = ctypes.c_void_p()
    cfg = _native.default_model_config()
    status = native.ov_generator_create_synthetic(ctypes.byref(cfg), 0, 0, ctypes.byref(h))
    assert status != 0
    assert _native.last_error().startswith("OmniVoice generator: ")
