"""CPU restatement of the OmniVoice audio tokenizer's decoder: RVQ codes
to 24 kHz samples (the reference's Codec::Decode).

TEST INFRASTRUCTURE ONLY: the checker of the CUDA decoder, imported by
tests/ and by bench.py's CPU-baseline leg, never by the omnivoice_b200
package.

Follows, step by step (paths within the reference tree):
  codec.cpp:136-160       RVQ decode tables: project_out(codebook) + bias
  codec.cpp:197-262       Decode: codebook sum, fc2 into the input
                          convolution's padded buffer, input conv, the
                          upsampling blocks, final snake, output conv (no tanh)
  codec_state.hpp:217-239 Apply: Conv1d as one product per tap, + bias
  codec_state.hpp:241-263 Residual: snake1, conv1 (k 7, dilation d), snake2,
                          conv2 (k 1) added into the signal, + bias
  codec_state.hpp:265-289 Block: snake, ConvTranspose1d (kernel 2 s,
                          padding ceil(s / 2), output padding s % 2) as one
                          product into columns + col2im, the three units
  kernels/codec_kernels.hip:11-79  Snake, Col2Im, CodebookSum
The reference computes in float32 (hipblasSgemm); this restatement keeps
the same operations in float64, so it is the exact result the float32
paths approximate.  Signals are channel-major [channels][time] as in the
reference.

Weights are a dict keyed by the reference's safetensors names (float32
arrays), `cfg` a CodecShape.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

RESIDUAL_KERNEL = 7          # codec_state.hpp:26
DILATIONS = (1, 3, 9)        # codec_state.hpp:27


@dataclass
class CodecShape:
    """The decoder's part of CodecConfig (reference config.hpp:41-72)."""
    codebooks: int = 8
    codebook_size: int = 1024
    codebook_dim: int = 64
    semantic_hidden: int = 768
    latent_channels: int = 256
    decoder_channels: int = 1024
    upsampling_ratios: list = field(default_factory=lambda: [8, 5, 4, 2, 3])

    @property
    def hidden(self) -> int:  # codec.cpp:121-122
        return self.semantic_hidden + self.latent_channels

    @property
    def frame_samples(self) -> int:
        return int(np.prod(self.upsampling_ratios))


def snake(x, alpha):
    """codec_kernels.hip:11-27: x + sin(a x)^2 / (a + 1e-9), per channel."""
    a = alpha.reshape(-1, 1).astype(np.float64)
    return x + (1.0 / (a + 1e-9)) * np.sin(a * x) ** 2


def conv1d(x, weight, bias, dilation=1):
    """codec_state.hpp:217-239: 'same' Conv1d, padding (k - 1) d / 2 zeros
    on both sides; weight [out][in][k]."""
    k = weight.shape[2]
    pad = (k - 1) * dilation // 2
    length = x.shape[1]
    xp = np.pad(x, ((0, 0), (pad, pad)))
    w = weight.astype(np.float64)
    out = np.zeros((w.shape[0], length))
    for tap in range(k):
        out += w[:, :, tap] @ xp[:, tap * dilation: tap * dilation + length]
    return out + bias.astype(np.float64).reshape(-1, 1)


def conv_transpose1d(x, weight, bias, stride):
    """codec_state.hpp:265-283 + Col2Im (codec_kernels.hip:45-65): columns
    [k][out][j] = W[:, :, k]^T x[:, j], then output[t] = bias + sum over
    t = j s + k - pad, pad = ceil(s / 2), t < length * s; weight
    [in][out][2 s]."""
    kernel = 2 * stride
    pad = (stride + 1) // 2
    length = x.shape[1]
    out_len = length * stride
    w = weight.astype(np.float64)
    out = np.zeros((w.shape[1], out_len)) + bias.astype(np.float64).reshape(-1, 1)
    j = np.arange(length)
    for k in range(kernel):
        cols = w[:, :, k].T @ x  # [out][length]
        t = j * stride + k - pad
        ok = (t >= 0) & (t < out_len)
        out[:, t[ok]] += cols[:, ok]
    return out


def rvq_tables(weights, cfg: CodecShape):
    """codec.cpp:136-160: table[c][e] = project_out_c(embed_c[e])."""
    tables = []
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        embed = weights[p + "codebook.embed"].astype(np.float64)
        proj = weights[p + "project_out.weight"].astype(np.float64)
        bias = weights[p + "project_out.bias"].astype(np.float64)
        tables.append(embed @ proj.T + bias)
    return tables


def decode(weights, cfg: CodecShape, codes):
    """codec.cpp:197-262.  codes: int [codebooks][frames]; returns float64
    [frames * frame_samples] samples."""
    codes = np.asarray(codes)
    if codes.shape[0] != cfg.codebooks:
        raise ValueError("code count doesn't match the frames")
    if (codes < 0).any() or (codes >= cfg.codebook_size).any():
        raise ValueError("code outside the codebook")
    tables = rvq_tables(weights, cfg)
    quantized = sum(tables[c][codes[c]] for c in range(cfg.codebooks))  # [frames][hidden]
    latent = (weights["fc2.weight"].astype(np.float64) @ quantized.T
              + weights["fc2.bias"].astype(np.float64).reshape(-1, 1))  # [latent][frames]
    x = conv1d(latent, weights["acoustic_decoder.conv1.weight"],
               weights["acoustic_decoder.conv1.bias"])
    for i, stride in enumerate(cfg.upsampling_ratios):
        p = f"acoustic_decoder.block.{i}."
        x = conv_transpose1d(snake(x, weights[p + "snake1.alpha"]), weights[p + "conv_t1.weight"],
                             weights[p + "conv_t1.bias"], stride)
        for u, dilation in enumerate(DILATIONS):
            q = p + f"res_unit{u + 1}."
            y = conv1d(snake(x, weights[q + "snake1.alpha"]), weights[q + "conv1.weight"],
                       weights[q + "conv1.bias"], dilation)
            y = conv1d(snake(y, weights[q + "snake2.alpha"]), weights[q + "conv2.weight"],
                       weights[q + "conv2.bias"])
            x = x + y
    x = snake(x, weights["acoustic_decoder.snake1.alpha"])
    y = conv1d(x, weights["acoustic_decoder.conv2.weight"], weights["acoustic_decoder.conv2.bias"])
    return y[0]


def tensor_shapes(cfg: CodecShape) -> dict:
    """Every tensor the decoder reads, with the shape the reference expects
    (codec.cpp:26-106,131-188)."""
    s = {}
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        s[p + "codebook.embed"] = (cfg.codebook_size, cfg.codebook_dim)
        s[p + "project_out.weight"] = (cfg.hidden, cfg.codebook_dim)
        s[p + "project_out.bias"] = (cfg.hidden,)
    s["fc2.weight"] = (cfg.latent_channels, cfg.hidden)
    s["fc2.bias"] = (cfg.latent_channels,)
    ch = cfg.decoder_channels
    s["acoustic_decoder.conv1.weight"] = (ch, cfg.latent_channels, RESIDUAL_KERNEL)
    s["acoustic_decoder.conv1.bias"] = (ch,)
    for i, stride in enumerate(cfg.upsampling_ratios):
        p = f"acoustic_decoder.block.{i}."
        out = ch // 2
        s[p + "snake1.alpha"] = (1, ch, 1)
        s[p + "conv_t1.weight"] = (ch, out, 2 * stride)
        s[p + "conv_t1.bias"] = (out,)
        for u in range(3):
            q = p + f"res_unit{u + 1}."
            s[q + "snake1.alpha"] = (1, out, 1)
            s[q + "snake2.alpha"] = (1, out, 1)
            s[q + "conv1.weight"] = (out, out, RESIDUAL_KERNEL)
            s[q + "conv1.bias"] = (out,)
            s[q + "conv2.weight"] = (out, out, 1)
            s[q + "conv2.bias"] = (out,)
        ch = out
    s["acoustic_decoder.snake1.alpha"] = (1, ch, 1)
    s["acoustic_decoder.conv2.weight"] = (1, ch, RESIDUAL_KERNEL)
    s["acoustic_decoder.conv2.bias"] = (1,)
    return s


def synthetic_weights(cfg: CodecShape, seed: int) -> dict:
    """Seeded float32 weights of every decoder tensor (numpy PCG64, the same
    on every machine): convolutions N(0, 1 / fan_in) scaled so the residual
    stream keeps its size through the blocks, snake alphas U(0.5, 2),
    codebooks N(0, 1)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in tensor_shapes(cfg).items():
        if name.endswith("alpha"):
            v = rng.uniform(0.5, 2.0, shape)
        elif name.endswith("codebook.embed"):
            v = rng.standard_normal(shape)
        elif name.endswith("bias"):
            v = 0.05 * rng.standard_normal(shape)
        elif "conv_t1" in name:
            fan_in = shape[0] * 2  # two taps reach each output
            v = rng.standard_normal(shape) / np.sqrt(fan_in)
        else:
            fan_in = int(np.prod(shape[1:]))
            gain = 0.5 if "res_unit" in name else 1.0
            v = gain * rng.standard_normal(shape) / np.sqrt(fan_in)
        out[name] = v.astype(np.float32)
    return out
