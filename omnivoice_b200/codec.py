"""Python mirror of the reference's audio tokenizer over the C-ABI
(include/ov_codec.h).

Names, argument meanings and error behaviour follow
gufo::models::omnivoice::Codec (codec.hpp:17-43):
  Codec.load / Codec.synthetic   <- Codec::Load   (decoder tensors)
  Codec.decode                   <- Codec::Decode: codes [codebook][frame] ->
                                    frames * frame_samples float32 samples
  Codec.decode_device            codes and audio as CUDA tensors, no host copy
  Encoder.load / Encoder.synthetic <- Codec::Load (encoder tensors)
  Encoder.encode                 <- Codec::Encode: 24 kHz samples (whole
                                    frames) -> codes [codebook][frame]
Failures raise CodecError carrying the reference's prefixes
("OmniVoice decode: ...", "OmniVoice encode: ...",
"OmniVoice audio tokenizer: ...").
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _native as N


class CodecError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _check(status: int) -> None:
    if status != N.OV_OK:
        raise CodecError(status, N.last_error())


@dataclass
class CodecConfig:
    """The decoder's part of CodecConfig (config.hpp:41-72)."""
    codebooks: int = 8
    codebook_size: int = 1024
    codebook_dim: int = 64
    semantic_hidden: int = 768
    latent_channels: int = 256
    decoder_channels: int = 1024
    upsampling_ratios: list = field(default_factory=lambda: [8, 5, 4, 2, 3])
    sample_rate: int = 24000

    @property
    def frame_samples(self) -> int:
        return int(np.prod(self.upsampling_ratios))

    def c(self) -> N.CodecConfigC:
        out = N.CodecConfigC()
        out.codebooks, out.codebook_size = self.codebooks, self.codebook_size
        out.codebook_dim, out.semantic_hidden = self.codebook_dim, self.semantic_hidden
        out.latent_channels, out.decoder_channels = self.latent_channels, self.decoder_channels
        if not 1 <= len(self.upsampling_ratios) <= 8:
            raise ValueError("1 to 8 upsampling blocks")
        for i, r in enumerate(self.upsampling_ratios):
            out.upsampling_ratios[i] = r
        out.num_upsampling = len(self.upsampling_ratios)
        out.sample_rate = self.sample_rate
        return out


class Codec:
    """One decoder on one GPU (not thread-safe, codec.hpp:16)."""

    def __init__(self, handle: int, config: CodecConfig):
        self._h = ctypes.c_void_p(handle)
        self.config = config

    @classmethod
    def load(cls, config: CodecConfig, safetensors_path: str, device: int = 0) -> "Codec":
        out = ctypes.c_void_p()
        _check(N.lib().ov_codec_load(ctypes.byref(config.c()), str(safetensors_path).encode(),
                                     device, ctypes.byref(out)))
        return cls(out.value, config)

    @classmethod
    def synthetic(cls, config: CodecConfig, seed: int = 0, device: int = 0) -> "Codec":
        out = ctypes.c_void_p()
        _check(N.lib().ov_codec_create_synthetic(ctypes.byref(config.c()), seed, device,
                                                 ctypes.byref(out)))
        return cls(out.value, config)

    def close(self) -> None:
        if self._h:
            N.lib().ov_codec_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def frame_samples(self) -> int:
        return int(N.lib().ov_codec_frame_samples(self._h))

    def decode(self, codes) -> np.ndarray:
        """codes: int [codebooks][frames] -> float32 [frames * frame_samples]."""
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        if codes.ndim != 2 or codes.shape[0] != self.config.codebooks:
            raise CodecError(N.OV_ERR_INVALID,
                             "OmniVoice decode: code count doesn't match the frames")
        frames = codes.shape[1]
        audio = np.empty(frames * self.frame_samples, np.float32)
        _check(N.lib().ov_codec_decode(self._h, codes.ctypes.data, frames, audio.ctypes.data))
        return audio

    def decode_device(self, codes, audio, stream: int = 0) -> None:
        """codes: CUDA int32 [codebooks][frames]; audio: CUDA float32
        [frames * frame_samples]; enqueued on `stream` (0: the codec's)."""
        frames = codes.shape[1]
        _check(N.lib().ov_codec_decode_device(self._h, codes.data_ptr(), frames,
                                              audio.data_ptr(), stream or None))


@dataclass
class EncoderConfig:
    """The encoder's part of CodecConfig (config.hpp:30-72): the codec's rate
    and quantizer, HuBERT (SemanticEncoderConfig) and the DAC encoder
    (AcousticConfig)."""
    sample_rate: int = 24000
    codebooks: int = 8
    codebook_size: int = 1024
    codebook_dim: int = 64
    semantic_sample_rate: int = 16000
    hidden_size: int = 768
    intermediate_size: int = 3072
    heads: int = 12
    layers: int = 12
    position_kernel: int = 128
    position_groups: int = 16
    layer_norm_eps: float = 1e-5
    conv_channels: list = field(default_factory=lambda: [512] * 7)
    conv_kernels: list = field(default_factory=lambda: [10, 3, 3, 3, 3, 2, 2])
    conv_strides: list = field(default_factory=lambda: [5, 2, 2, 2, 2, 2, 2])
    encoder_channels: int = 64
    latent_channels: int = 256
    downsampling_ratios: list = field(default_factory=lambda: [8, 5, 4, 2, 3])

    @property
    def frame_samples(self) -> int:
        return int(np.prod(self.downsampling_ratios))

    def c(self) -> N.CodecEncoderConfigC:
        out = N.CodecEncoderConfigC()
        for name in ("sample_rate", "codebooks", "codebook_size", "codebook_dim",
                     "semantic_sample_rate", "hidden_size", "intermediate_size", "heads", "layers",
                     "position_kernel", "position_groups", "layer_norm_eps", "encoder_channels",
                     "latent_channels"):
            setattr(out, name, getattr(self, name))
        if not (len(self.conv_channels) == len(self.conv_kernels) == len(self.conv_strides)
                and 1 <= len(self.conv_channels) <= 8):
            raise ValueError("1 to 8 feature-extractor convolutions, one channel / kernel / stride each")
        if not 1 <= len(self.downsampling_ratios) <= 8:
            raise ValueError("1 to 8 downsampling blocks")
        for i, (ch, k, st) in enumerate(zip(self.conv_channels, self.conv_kernels, self.conv_strides)):
            out.conv_channels[i], out.conv_kernels[i], out.conv_strides[i] = ch, k, st
        out.num_convs = len(self.conv_channels)
        for i, r in enumerate(self.downsampling_ratios):
            out.downsampling_ratios[i] = r
        out.num_downsampling = len(self.downsampling_ratios)
        return out


class Encoder:
    """One encoder on one GPU (not thread-safe, codec.hpp:16)."""

    def __init__(self, handle: int, config: EncoderConfig):
        self._h = ctypes.c_void_p(handle)
        self.config = config

    @classmethod
    def load(cls, config: EncoderConfig, safetensors_path: str, device: int = 0) -> "Encoder":
        out = ctypes.c_void_p()
        _check(N.lib().ov_codec_encoder_load(ctypes.byref(config.c()), str(safetensors_path).encode(),
                                             device, ctypes.byref(out)))
        return cls(out.value, config)

    @classmethod
    def synthetic(cls, config: EncoderConfig, seed: int = 0, device: int = 0) -> "Encoder":
        out = ctypes.c_void_p()
        _check(N.lib().ov_codec_encoder_create_synthetic(ctypes.byref(config.c()), seed, device,
                                                         ctypes.byref(out)))
        return cls(out.value, config)

    def close(self) -> None:
        if self._h:
            N.lib().ov_codec_encoder_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def frame_samples(self) -> int:
        return int(N.lib().ov_codec_encoder_frame_samples(self._h))

    def encode(self, samples) -> np.ndarray:
        """float32 samples at sample_rate (a whole number of frames) ->
        int32 codes [codebooks][frames]."""
        samples = np.ascontiguousarray(samples, dtype=np.float32)
        frames_max = samples.size // max(self.frame_samples, 1)
        codes = np.empty(self.config.codebooks * max(frames_max, 1), np.int32)
        frames = ctypes.c_size_t()
        _check(N.lib().ov_codec_encode(self._h, samples.ctypes.data, samples.size, codes.ctypes.data,
                                       codes.size, ctypes.byref(frames)))
        return codes[:self.config.codebooks * frames.value].reshape(self.config.codebooks, frames.value)
