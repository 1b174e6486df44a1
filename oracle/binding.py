"""ctypes binding of the CPU oracle (oracle/liboracle.so) and of the
reference's own decoding.cpp (oracle/_ref/libref_decoding.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the omnivoice_b200 package.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_float, c_int, c_int32, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libref_decoding.so"


class OracleConfig(ctypes.Structure):
    _fields_ = [("vocab_size", c_size_t), ("hidden_size", c_size_t),
                ("intermediate_size", c_size_t), ("layers", c_size_t), ("heads", c_size_t),
                ("kv_heads", c_size_t), ("head_dim", c_size_t), ("max_positions", c_size_t),
                ("rms_norm_eps", c_float), ("rope_theta", c_float),
                ("audio_codebooks", c_size_t), ("audio_vocab_size", c_size_t),
                ("audio_mask_id", c_uint32)]


_P = c_void_p
_SIG = {
    "oc_set_threads": (None, [c_int]),
    "oc_get_threads": (c_int, []),
    "oc_model_synthetic": (c_void_p, [POINTER(OracleConfig), c_uint64]),
    "oc_model_free": (None, [_P]),
    "oc_synthetic_values": (None, [c_uint64, c_uint64, c_float, c_uint64, c_size_t, _P]),
    "oc_forward": (c_int, [_P, _P, c_size_t, c_size_t, c_size_t, _P, c_int, _P]),
    "oc_score": (c_int, [_P, c_size_t, c_size_t, c_size_t, c_size_t, c_uint32, c_float, _P, _P]),
    "oc_schedule": (None, [c_size_t, c_size_t, c_float, _P]),
    "oc_build_input": (None, [_P, c_size_t, _P, c_size_t, c_size_t, c_size_t, c_uint32, _P]),
    "oc_reference_gumbel": (None, [c_uint64, c_size_t, _P]),
    "oc_select": (c_size_t, [c_size_t, c_size_t, c_size_t, _P, _P, c_uint32, c_float, c_float,
                             _P, _P, _P]),
    "oc_generate": (c_int, [_P, _P, c_size_t, c_size_t, c_size_t, c_size_t, c_float, c_float,
                            c_float, c_float, c_uint64, _P, _P, _P]),
    "oc_generate_traced": (c_int, [_P, _P, c_size_t, c_size_t, c_size_t, c_size_t, c_float,
                                   c_float, c_float, c_float, c_uint64, _P, _P, _P, _P, _P, _P]),
    "oc_set_accumulation_order": (None, [c_int]),
}
_REF_SIG = {
    "ref_unmask_schedule": (None, [c_size_t, c_size_t, c_float, _P]),
    "ref_build_input": (c_size_t, [_P, c_size_t, _P, c_size_t, c_size_t, c_size_t, c_uint32, _P]),
    "ref_fill": (c_size_t, [c_int, c_uint64, c_float, c_float, c_size_t, c_size_t, c_size_t, _P,
                            _P, c_uint32, _P, _P]),
}

_oracle = None
_ref = None


def reference_tree() -> str | None:
    """Where the reference sources are: $OV_REF_DIR, else the
    `reference_path` that BASELINE.json at the repository root records;
    None when neither names an existing directory."""
    import json
    import os
    path = os.environ.get("OV_REF_DIR")
    if not path:
        baseline = HERE.parent / "BASELINE.json"
        try:
            path = json.loads(baseline.read_text()).get("reference_path")
        except (OSError, ValueError):
            path = None
    return path if path and Path(path).is_dir() else None


def build() -> None:
    """Builds liboracle.so (and oracle/_ref when the reference tree exists)."""
    cmd = ["make", "-s", "-C", str(HERE)]
    ref = reference_tree()
    if ref is not None:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_PATH.exists():
            build()
        h = ctypes.CDLL(str(ORACLE_PATH))
        for name, (res, args) in _SIG.items():
            getattr(h, name).restype = res
            getattr(h, name).argtypes = args
        _oracle = h
    return _oracle


def reference_decoding() -> ctypes.CDLL | None:
    """The reference's decoding.cpp, or None when it was not built here."""
    global _ref
    if _ref is None and REF_PATH.exists():
        h = ctypes.CDLL(str(REF_PATH))
        for name, (res, args) in _REF_SIG.items():
            getattr(h, name).restype = res
            getattr(h, name).argtypes = args
        _ref = h
    return _ref


def config(**kw) -> OracleConfig:
    base = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, layers=28, heads=16,
                kv_heads=8, head_dim=128, max_positions=40960, rms_norm_eps=1e-6,
                rope_theta=1e6, audio_codebooks=8, audio_vocab_size=1025, audio_mask_id=1024)
    base.update(kw)
    return OracleConfig(**base)


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class OracleModel:
    """The synthetic random-init model on the CPU."""

    def __init__(self, cfg: OracleConfig, seed: int):
        self.cfg = cfg
        self.h = oracle().oc_model_synthetic(ctypes.byref(cfg), seed)

    def close(self):
        if self.h:
            oracle().oc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, ids: np.ndarray, audio_start: int, frames: int, layers: int = -1,
                want_hidden: bool = False):
        """Logits after `layers` layers (all when negative) and the final
        norm and head; with want_hidden also the residual stream."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        length = ids.shape[1]
        cv = self.cfg.audio_codebooks * self.cfg.audio_vocab_size
        logits = np.empty((2 * frames, cv), np.float32)
        hidden = np.empty((length + frames, self.cfg.hidden_size), np.float32) if want_hidden else None
        status = oracle().oc_forward(self.h, ptr(ids), length, audio_start, frames, ptr(logits),
                                     layers, ptr(hidden) if want_hidden else None)
        if status != 0:
            raise RuntimeError(f"oc_forward failed with {status}")
        return (logits, hidden) if want_hidden else logits

    def generate_traced(self, ids: np.ndarray, audio_start: int, frames: int, steps=32,
                        seed=0):
        """generate() with the default decoding settings that also returns,
        per step, the ids the forward pass saw and the scoring's
        predictions and confidences."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        c = self.cfg.audio_codebooks
        codes = np.empty((c, frames), np.int32)
        when = np.empty((c, frames), np.int32)
        step_ids = np.zeros((steps, c, ids.shape[1]), np.int32)
        step_pred = np.zeros((steps, c, frames), np.int32)
        step_conf = np.zeros((steps, c, frames), np.float32)
        status = oracle().oc_generate_traced(self.h, ptr(ids), ids.shape[1], audio_start, frames,
                                             steps, 2.0, 0.1, 5.0, 5.0, seed, None, ptr(codes),
                                             ptr(when), ptr(step_ids), ptr(step_pred),
                                             ptr(step_conf))
        if status != 0:
            raise RuntimeError(f"oc_generate_traced failed with {status}")
        return codes, when, step_ids, step_pred, step_conf

    def generate(self, ids: np.ndarray, audio_start: int, frames: int, steps=32, guidance=2.0,
                 t_shift=0.1, layer_penalty=5.0, temperature=5.0, seed=0, gumbel=None):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        c = self.cfg.audio_codebooks
        codes = np.empty((c, frames), np.int32)
        when = np.empty((c, frames), np.int32)
        g = None if gumbel is None else np.ascontiguousarray(gumbel, dtype=np.float32)
        status = oracle().oc_generate(self.h, ptr(ids), ids.shape[1], audio_start, frames, steps,
                                      guidance, t_shift, layer_penalty, temperature, seed,
                                      ptr(g) if g is not None else None, ptr(codes), ptr(when))
        if status != 0:
            raise RuntimeError(f"oc_generate failed with {status}")
        return codes, when


def score(logits: np.ndarray, frames: int, codebooks=8, vocab=1025, mask=1024, guidance=2.0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    pred = np.empty((codebooks, frames), np.int32)
    conf = np.empty((codebooks, frames), np.float32)
    oracle().oc_score(ptr(logits), logits.shape[1], frames, codebooks, vocab, mask, guidance,
                      ptr(pred), ptr(conf))
    return pred, conf


def schedule(total: int, steps: int, t_shift: float) -> list[int]:
    out = np.empty(steps, np.uint64)
    oracle().oc_schedule(total, steps, t_shift, ptr(out))
    return [int(x) for x in out]


def reference_gumbel(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    oracle().oc_reference_gumbel(seed, count, ptr(out))
    return out


def select(count, prediction, confidence, codes, mask=1024, layer_penalty=5.0, temperature=5.0,
           gumbel=None):
    """PositionSelector::Fill; returns (codes_out, chosen list)."""
    prediction = np.ascontiguousarray(prediction, dtype=np.int32)
    confidence = np.ascontiguousarray(confidence, dtype=np.float32)
    c, f = prediction.shape
    out = np.ascontiguousarray(codes, dtype=np.int32).copy()
    chosen = np.empty(c * f, np.uint64)
    g = None if gumbel is None else np.ascontiguousarray(gumbel, dtype=np.float32)
    n = oracle().oc_select(count, c, f, ptr(prediction), ptr(confidence), mask, layer_penalty,
                           temperature, ptr(g) if g is not None else None, ptr(out), ptr(chosen))
    return out, [int(x) for x in chosen[:n]]
