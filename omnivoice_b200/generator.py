"""Python mirror of the reference's generator interface over the C-ABI.

Names, argument meanings and error behaviour follow
gufo::models::omnivoice (generator.hpp:20-56, decoding.hpp:14-77):
  Generator.load / Generator.synthetic   <- Generator::Load
  Generator.forward                      <- Generator::Forward
  Generator.score                        <- Generator::Score
  Generator.generate                     <- Generator::Generate
  ConditionalInput.build                 <- ConditionalInput::Build
  unmask_schedule                        <- UnmaskSchedule
Failures raise GeneratorError carrying the reference's message prefixes
("OmniVoice forward: ..."); cancellation raises Cancelled("cancelled").
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np

from . import _native as N


class GeneratorError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Cancelled(GeneratorError):
    pass


def _check(status: int) -> None:
    if status == N.OV_OK:
        return
    message = N.last_error()
    if status == N.OV_ERR_CANCELLED:
        raise Cancelled(status, message)
    raise GeneratorError(status, message)


@dataclass
class DecodingConfig:
    steps: int = 32
    guidance: float = 2.0
    t_shift: float = 0.1
    layer_penalty: float = 5.0
    position_temperature: float = 5.0

    def c(self) -> N.DecodingConfigC:
        return N.DecodingConfigC(self.steps, self.guidance, self.t_shift, self.layer_penalty,
                                 self.position_temperature)


@dataclass
class ConditionalInput:
    codebooks: int
    length: int
    audio_start: int
    target_frames: int
    ids: np.ndarray  # int32 [codebooks][length]

    @staticmethod
    def build(text_ids: Sequence[int], reference_codes: np.ndarray | None,
              target_frames: int, codebooks: int = 8, mask_id: int = 1024) -> "ConditionalInput":
        text = np.ascontiguousarray(np.asarray(text_ids, dtype=np.uint32))
        if reference_codes is None:
            ref = np.zeros((codebooks, 0), dtype=np.int32)
        else:
            ref = np.ascontiguousarray(np.asarray(reference_codes, dtype=np.int32))
        frames_ref = ref.shape[1]
        length = len(text) + frames_ref + target_frames
        ids = np.empty((codebooks, length), dtype=np.int32)
        got = N.lib().ov_build_conditional_input(
            text.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), len(text),
            ref.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), frames_ref, target_frames,
            codebooks, mask_id, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
        assert got == length
        return ConditionalInput(codebooks, length, len(text), target_frames, ids)

    def c(self) -> N.ConditionalInputC:
        ids = np.ascontiguousarray(self.ids, dtype=np.int32)
        self._keep = ids  # keep the buffer alive while the struct is used
        return N.ConditionalInputC(self.codebooks, self.length, self.audio_start,
                                   self.target_frames,
                                   ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))


@dataclass
class GenerationResult:
    codes: np.ndarray = field(default_factory=lambda: np.zeros((0, 0), np.int32))
    unmasked_at: np.ndarray = field(default_factory=lambda: np.zeros((0, 0), np.int32))


def unmask_schedule(total: int, steps: int, t_shift: float) -> list[int]:
    out = (ctypes.c_size_t * steps)()
    _check(N.lib().ov_unmask_schedule(total, steps, t_shift, out))
    return list(out)


def model_config(**overrides) -> N.ModelConfig:
    cfg = N.default_model_config()
    for key, value in overrides.items():
        setattr(cfg, key, value)
    return cfg


NOISE = {"reference": N.OV_GEN_NOISE_REFERENCE, "device": N.OV_GEN_NOISE_DEVICE}


class Generator:
    """One replica of the backbone on one GPU.  Not thread-safe."""

    def __init__(self, handle: int, config: N.ModelConfig):
        self._h = handle
        self.config = config

    @classmethod
    def load(cls, config: N.ModelConfig, safetensors_path: str, device: int = 0) -> "Generator":
        h = ctypes.c_void_p()
        _check(N.lib().ov_generator_load(ctypes.byref(config), str(safetensors_path).encode(),
                                         device, ctypes.byref(h)))
        return cls(h.value, config)

    @classmethod
    def synthetic(cls, config: N.ModelConfig | None = None, weight_seed: int = 0,
                  device: int = 0) -> "Generator":
        config = config or N.default_model_config()
        h = ctypes.c_void_p()
        _check(N.lib().ov_generator_create_synthetic(ctypes.byref(config), weight_seed, device,
                                                     ctypes.byref(h)))
        return cls(h.value, config)

    def close(self) -> None:
        if self._h:
            N.lib().ov_generator_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _vocab(self) -> int:
        return self.config.audio_codebooks * self.config.audio_vocab_size

    def forward(self, inp: ConditionalInput) -> np.ndarray:
        logits = np.empty((2 * inp.target_frames, self._vocab()), dtype=np.float32)
        c = inp.c()
        _check(N.lib().ov_generator_forward(self._h, ctypes.byref(c), logits.ctypes.data))
        return logits

    def score(self, inp: ConditionalInput, guidance: float) -> tuple[np.ndarray, np.ndarray]:
        shape = (inp.codebooks, inp.target_frames)
        pred = np.empty(shape, dtype=np.int32)
        conf = np.empty(shape, dtype=np.float32)
        c = inp.c()
        _check(N.lib().ov_generator_score(self._h, ctypes.byref(c), guidance, pred.ctypes.data,
                                          conf.ctypes.data))
        return pred, conf

    def generate(self, inp: ConditionalInput, decoding: DecodingConfig, seed: int,
                 cancelled: Callable[[], bool] | None = None,
                 noise: str = "reference") -> GenerationResult:
        shape = (inp.codebooks, inp.target_frames)
        codes = np.empty(shape, dtype=np.int32)
        steps = np.empty(shape, dtype=np.int32)
        c, d = inp.c(), decoding.c()
        cb = N.CANCEL_FN(lambda _user: 1 if cancelled() else 0) if cancelled else N.CANCEL_FN()
        _check(N.lib().ov_generator_generate(self._h, ctypes.byref(c), ctypes.byref(d), seed,
                                             NOISE[noise], cb, None, codes.ctypes.data,
                                             steps.ctypes.data))
        return GenerationResult(codes, steps)

    def _batch_args(self, inputs, decoding, seeds):
        n = len(inputs)
        cs = (N.ConditionalInputC * n)(*[i.c() for i in inputs])
        sd = (ctypes.c_uint64 * n)(*seeds)
        return n, cs, decoding.c(), sd

    def generate_batch(self, inputs: Sequence[ConditionalInput], decoding: DecodingConfig,
                       seeds: Sequence[int], cancelled: Callable[[], bool] | None = None,
                       noise: str = "device") -> list[GenerationResult]:
        n, cs, d, sd = self._batch_args(inputs, decoding, seeds)
        results = [GenerationResult(np.empty((i.codebooks, i.target_frames), np.int32),
                                    np.empty((i.codebooks, i.target_frames), np.int32))
                   for i in inputs]
        codes = (ctypes.c_void_p * n)(*[r.codes.ctypes.data for r in results])
        steps = (ctypes.c_void_p * n)(*[r.unmasked_at.ctypes.data for r in results])
        cb = N.CANCEL_FN(lambda _user: 1 if cancelled() else 0) if cancelled else N.CANCEL_FN()
        _check(N.lib().ov_generator_generate_batch(self._h, cs, n, ctypes.byref(d), sd,
                                                   NOISE[noise], cb, None, codes, steps))
        return results

    # Split form used for device-resident timing.
    def prepare(self, inputs: Sequence[ConditionalInput], decoding: DecodingConfig,
                seeds: Sequence[int], noise: str = "device") -> None:
        n, cs, d, sd = self._batch_args(inputs, decoding, seeds)
        self._prepared = list(inputs)
        _check(N.lib().ov_generator_prepare(self._h, cs, n, ctypes.byref(d), sd, NOISE[noise]))

    def run(self) -> None:
        _check(N.lib().ov_generator_run(self._h, N.CANCEL_FN(), None))

    def fetch(self) -> list[GenerationResult]:
        inputs = self._prepared
        results = [GenerationResult(np.empty((i.codebooks, i.target_frames), np.int32),
                                    np.empty((i.codebooks, i.target_frames), np.int32))
                   for i in inputs]
        n = len(inputs)
        codes = (ctypes.c_void_p * n)(*[r.codes.ctypes.data for r in results])
        steps = (ctypes.c_void_p * n)(*[r.unmasked_at.ctypes.data for r in results])
        _check(N.lib().ov_generator_fetch(self._h, codes, steps))
        return results

    def stats(self) -> N.GeneratorStats:
        st = N.GeneratorStats()
        _check(N.lib().ov_generator_stats_get(self._h, ctypes.byref(st)))
        return st

    def profile_step(self) -> list[dict]:
        """Device time per kernel class of one step of the prepared batch."""
        times = (N.KernelTime * 32)()
        count = ctypes.c_size_t()
        _check(N.lib().ov_generator_profile_step(self._h, times, 32, ctypes.byref(count)))
        return [{"name": t.name.decode(), "ms": t.ms, "launches": t.launches,
                 "flops": t.flops, "bytes": t.bytes} for t in times[:count.value]]
