"""CPU restatement of the OmniVoice audio tokenizer's encoder: 24 kHz samples
to residual-vector-quantized codes (the reference's Codec::Encode, voice
cloning).

TEST INFRASTRUCTURE ONLY: the checker of the CUDA encoder, imported by
tests/ and by bench.py's CPU-baseline leg, never by the omnivoice_b200
package.

Follows, step by step (paths within the reference tree):
  audio.cpp:265-321          Resample: torchaudio's windowed-sinc resampler
                             (Hann window, 6 zero crossings, rolloff 0.99),
                             kernel built in float32, sums in float64
  codec_encoder.cpp:249-309  HuBERT feature extractor (bias-free strided
                             convolutions, per-channel group norm + GELU on
                             the first, GELU on the others), layer norm and
                             projection, weight-normed grouped positional
                             convolution + GELU added to the states, encoder
                             layer norm
  codec_encoder.cpp:310-368  post-norm HuBERT layers (attention, out
                             projection added, layer norm, GELU MLP added,
                             final layer norm); the features average the
                             layer input and every layer output
  codec_encoder.cpp:369-398  every semantic_stride-th frame, the semantic
                             encoder (bias-free k3 convolution, blocks of ELU
                             residual units and a k3 convolution)
  codec_encoder.cpp:399-424  DAC encoder (k7 input convolution, blocks of
                             three snake residual units, snake, strided
                             convolution doubling the width), snake, k3
                             output convolution
  codec_encoder.cpp:425-458  fc over [acoustic latent | semantic], then per
                             codebook: project_in, the nearest entry by
                             -(|h|^2 - 2 h.e + |e|^2) (lowest index on ties),
                             and the entry's decoded vector subtracted
  kernels/encoder_kernels.hip:41-229  GELU (erf form), group / layer norm,
                             ELU, softmax, nearest entry
The reference computes in float32 (hipblasSgemm); this restatement keeps
the same operations in float64 (the resampler's kernel excepted: float32
operation by operation, as the reference builds it).  Signals are
time-major [time][channels].

Weights are a dict keyed by the reference's safetensors names (float32
arrays), `cfg` an EncoderShape.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
from scipy.special import erf

from oracle.codec import DILATIONS, RESIDUAL_KERNEL, snake

GROUP_NORM_EPS = 1e-5   # encoder_kernels.hip GroupNormGelu's epsilon (codec_encoder.cpp:286)
HUBERT_PAD = 160        # zero samples on both sides at 16 kHz (codec_encoder.cpp:262-263)


@dataclass
class EncoderShape:
    """The encoder's part of CodecConfig (reference config.hpp:30-72)."""
    sample_rate: int = 24000
    codebooks: int = 8
    codebook_size: int = 1024
    codebook_dim: int = 64
    # HuBERT (SemanticEncoderConfig)
    semantic_rate: int = 16000
    hidden: int = 768
    intermediate: int = 3072
    heads: int = 12
    layers: int = 12
    position_kernel: int = 128
    position_groups: int = 16
    layer_norm_eps: float = 1e-5
    conv_channels: list = field(default_factory=lambda: [512] * 7)
    conv_kernels: list = field(default_factory=lambda: [10, 3, 3, 3, 3, 2, 2])
    conv_strides: list = field(default_factory=lambda: [5, 2, 2, 2, 2, 2, 2])
    # DAC encoder (AcousticConfig)
    encoder_channels: int = 64
    latent_channels: int = 256
    downsampling_ratios: list = field(default_factory=lambda: [8, 5, 4, 2, 3])

    @property
    def frame_samples(self) -> int:
        return int(np.prod(self.downsampling_ratios))

    @property
    def semantic_frame(self) -> int:  # HuBERT samples per frame at semantic_rate
        return int(np.prod(self.conv_strides))

    @property
    def semantic_stride(self) -> int:  # config.cpp:260-266
        return (self.semantic_rate // self.semantic_frame) // (self.sample_rate // self.frame_samples)

    @property
    def joint(self) -> int:  # the quantizer's hidden size
        return self.hidden + self.latent_channels


# ----------------------------------------------------------------- resample

def resample(samples, from_rate: int, to_rate: int) -> np.ndarray:
    """audio.cpp:265-321.  Returns float32."""
    x = np.asarray(samples, dtype=np.float32)
    if from_rate == to_rate or x.size == 0:
        return x.copy()
    zero_crossings, rolloff = 6, 0.99
    g = math.gcd(from_rate, to_rate)
    frm, to = from_rate // g, to_rate // g
    base = min(frm, to) * rolloff
    width = int(math.ceil(zero_crossings * frm / base))
    taps = 2 * width + frm
    f32 = np.float32
    base_f, pi_f = f32(base), f32(math.pi)
    scale_f = f32(base / frm)
    idx = (np.arange(taps, dtype=np.int64) - width).astype(f32) / f32(frm)
    kernel = np.empty((to, taps), dtype=f32)
    for phase in range(to):
        t = f32(-phase) / f32(to) + idx
        t = t * base_f
        t = np.clip(t, f32(-zero_crossings), f32(zero_crossings))
        cosine = np.cos(t * pi_f / f32(zero_crossings) / f32(2.0))
        window = cosine * cosine
        t = t * pi_f
        with np.errstate(invalid="ignore", divide="ignore"):
            sinc = np.where(t == 0, f32(1.0), np.sin(t) / t).astype(f32)
        kernel[phase] = sinc * (window * scale_f)
    length = x.size
    out_len = int(math.ceil(to * length / frm))
    # conv1d over the input padded by `width` before and `width + frm` after.
    padded = np.concatenate([np.zeros(width), x.astype(np.float64), np.zeros(width + frm + taps)])
    out = np.empty(out_len, dtype=np.float32)
    kd = kernel.astype(np.float64)
    for o in range(out_len):
        block, phase = divmod(o, to)
        origin = block * frm  # in padded coordinates
        out[o] = np.float32(np.dot(kd[phase], padded[origin:origin + taps]))
    return out


# ------------------------------------------------------------- primitives

def gelu(x):
    """encoder_kernels.hip:41-43: 0.5 x (1 + erf(x / sqrt 2))."""
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def elu(x):
    return np.where(x > 0, x, np.expm1(np.minimum(x, 0.0)))


def layer_norm(x, w, b, eps):
    """Rows [T][C] over C (encoder_kernels.hip LayerNormKernel)."""
    mean = x.mean(axis=1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * w.astype(np.float64) + b.astype(np.float64)


def conv(x, weight, bias=None, stride=1, dilation=1, pad=0, groups=1):
    """Strided Conv1d on time-major x [T][Cin]; weight [Cout][Cin / groups][K];
    output length (T + 2 pad - dilation (K - 1) - 1) / stride + 1
    (codec_state.hpp:83-85)."""
    w = weight.astype(np.float64)
    cout, cin_g, k = w.shape
    length = x.shape[0]
    out_len = (length + 2 * pad - dilation * (k - 1) - 1) // stride + 1
    xp = np.pad(x, ((pad, pad), (0, 0)))
    cout_g = cout // groups
    out = np.zeros((out_len, cout))
    for g in range(groups):
        xs = xp[:, g * cin_g:(g + 1) * cin_g]
        for tap in range(k):
            start = tap * dilation
            rows = xs[start:start + stride * (out_len - 1) + 1:stride]  # [out_len][cin_g]
            out[:, g * cout_g:(g + 1) * cout_g] += rows @ w[g * cout_g:(g + 1) * cout_g, :, tap].T
    if bias is not None:
        out += bias.astype(np.float64)
    return out


def linear(x, weights, prefix):
    return x @ weights[prefix + ".weight"].astype(np.float64).T + weights[prefix + ".bias"].astype(np.float64)


def position_weight(weights, cfg: EncoderShape):
    """codec_encoder.cpp:103-137: the weight norm folded, g_k v / |v_k| with
    the norm over all but the tap axis (dim = 2)."""
    p = "semantic_model.encoder.pos_conv_embed.conv.parametrizations.weight."
    g = weights[p + "original0"].astype(np.float64).reshape(-1)
    v = weights[p + "original1"].astype(np.float64)
    norms = np.sqrt((v ** 2).sum(axis=(0, 1)))
    return v * (g / norms)


# ------------------------------------------------------------------ HuBERT

def hubert(weights, cfg: EncoderShape, samples16):
    """codec_encoder.cpp:256-368: HuBERT states averaged over the layer
    input and every layer's output, [steps][hidden]."""
    x = np.concatenate([np.zeros(HUBERT_PAD), np.asarray(samples16, np.float64), np.zeros(HUBERT_PAD)])
    x = x.reshape(-1, 1)
    for i, (k, s) in enumerate(zip(cfg.conv_kernels, cfg.conv_strides)):
        x = conv(x, weights[f"semantic_model.feature_extractor.conv_layers.{i}.conv.weight"], stride=s)
        if i == 0:  # per-channel group norm over time, then GELU
            p = "semantic_model.feature_extractor.conv_layers.0.layer_norm."
            mean = x.mean(axis=0, keepdims=True)
            var = ((x - mean) ** 2).mean(axis=0, keepdims=True)
            x = (x - mean) / np.sqrt(var + GROUP_NORM_EPS) * weights[p + "weight"] + weights[p + "bias"]
        x = gelu(x)
    eps = cfg.layer_norm_eps
    p = "semantic_model.feature_projection."
    x = layer_norm(x, weights[p + "layer_norm.weight"], weights[p + "layer_norm.bias"], eps)
    h = linear(x, weights, p + "projection")
    # Positional convolution: kernel K, padding K / 2, the last output of an
    # even kernel dropped (only `steps` outputs are computed).
    steps = h.shape[0]
    kk = cfg.position_kernel
    pos = conv(h, position_weight(weights, cfg), weights["semantic_model.encoder.pos_conv_embed.conv.bias"],
               pad=kk // 2, groups=cfg.position_groups)[:steps]
    h = h + gelu(pos)
    p = "semantic_model.encoder.layer_norm."
    h = layer_norm(h, weights[p + "weight"], weights[p + "bias"], eps)
    total = h.copy()
    d = cfg.hidden // cfg.heads
    for layer in range(cfg.layers):
        p = f"semantic_model.encoder.layers.{layer}."
        q = linear(h, weights, p + "attention.q_proj")
        k = linear(h, weights, p + "attention.k_proj")
        v = linear(h, weights, p + "attention.v_proj")
        att = np.empty_like(h)
        for head in range(cfg.heads):
            sl = slice(head * d, (head + 1) * d)
            s = q[:, sl] @ k[:, sl].T / math.sqrt(d)
            s = np.exp(s - s.max(axis=1, keepdims=True))
            att[:, sl] = (s / s.sum(axis=1, keepdims=True)) @ v[:, sl]
        h = h + linear(att, weights, p + "attention.out_proj")
        h = layer_norm(h, weights[p + "layer_norm.weight"], weights[p + "layer_norm.bias"], eps)
        m = gelu(linear(h, weights, p + "feed_forward.intermediate_dense"))
        h = h + linear(m, weights, p + "feed_forward.output_dense")
        h = layer_norm(h, weights[p + "final_layer_norm.weight"], weights[p + "final_layer_norm.bias"], eps)
        total = total + h
    return total / (cfg.layers + 1)


def semantic_encoder(weights, x):
    """codec_encoder.cpp:379-398 on [frames][hidden]."""
    b = conv(x, weights["encoder_semantic.conv.weight"], pad=1)
    for blk in range(2):
        p = f"encoder_semantic.conv_blocks.{blk}."
        for u in range(2):
            q = p + f"res_units.{u}."
            c = conv(elu(b), weights[q + "conv1.weight"], pad=1)
            b = b + conv(elu(c), weights[q + "conv2.weight"])
        b = conv(b, weights[p + "conv.weight"], weights[p + "conv.bias"], pad=1)
    return b


def dac_encoder(weights, cfg: EncoderShape, samples):
    """codec_encoder.cpp:399-424 (residual units as codec_state.hpp:241-263)."""
    x = conv(np.asarray(samples, np.float64).reshape(-1, 1), weights["acoustic_encoder.conv1.weight"],
             weights["acoustic_encoder.conv1.bias"], pad=3)
    for i, stride in enumerate(cfg.downsampling_ratios):
        p = f"acoustic_encoder.block.{i}."
        for u, dil in enumerate(DILATIONS):
            q = p + f"res_unit{u + 1}."
            y = conv(snake(x.T, weights[q + "snake1.alpha"]).T, weights[q + "conv1.weight"],
                     weights[q + "conv1.bias"], dilation=dil, pad=(RESIDUAL_KERNEL - 1) * dil // 2)
            y = conv(snake(y.T, weights[q + "snake2.alpha"]).T, weights[q + "conv2.weight"],
                     weights[q + "conv2.bias"])
            x = x + y
        x = conv(snake(x.T, weights[p + "snake1.alpha"]).T, weights[p + "conv1.weight"],
                 weights[p + "conv1.bias"], stride=stride, pad=(stride + 1) // 2)
    x = snake(x.T, weights["acoustic_encoder.snake1.alpha"]).T
    return conv(x, weights["acoustic_encoder.conv2.weight"], weights["acoustic_encoder.conv2.bias"], pad=1)


def decode_tables(weights, cfg: EncoderShape):
    """codec.cpp:136-160: entry e of codebook c in the quantizer's hidden
    space, project_out_c(embed_c[e])."""
    out = []
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        out.append(weights[p + "codebook.embed"].astype(np.float64) @
                   weights[p + "project_out.weight"].astype(np.float64).T +
                   weights[p + "project_out.bias"].astype(np.float64))
    return out


def quantize(weights, cfg: EncoderShape, residual):
    """codec_encoder.cpp:425-458: codes [codebooks][frames]."""
    tables = decode_tables(weights, cfg)
    residual = residual.copy()
    codes = np.empty((cfg.codebooks, residual.shape[0]), dtype=np.int64)
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        h = linear(residual, weights, p + "project_in")
        emb = weights[p + "codebook.embed"].astype(np.float64)
        dist = -(((h ** 2).sum(axis=1, keepdims=True) - 2.0 * h @ emb.T) + (emb ** 2).sum(axis=1))
        idx = np.argmax(dist, axis=1)  # first maximum: the lowest index on ties
        codes[c] = idx
        residual = residual - tables[c][idx]
    return codes


def encode(weights, cfg: EncoderShape, samples, return_features=False):
    """codec_encoder.cpp:249-458: 24 kHz samples (a whole number of frames)
    to codes [codebooks][frames]."""
    samples = np.asarray(samples, dtype=np.float32)
    if samples.size == 0 or samples.size % cfg.frame_samples:
        raise ValueError("reference audio must be a whole number of frames")
    count = samples.size // cfg.frame_samples
    feats = hubert(weights, cfg, resample(samples, cfg.sample_rate, cfg.semantic_rate))
    if feats.shape[0] < count * cfg.semantic_stride:
        raise ValueError("reference audio is too short for the semantic encoder")
    semantic = semantic_encoder(weights, feats[::cfg.semantic_stride][:count])
    acoustic = dac_encoder(weights, cfg, samples)
    if acoustic.shape[0] != count:
        raise ValueError("acoustic and semantic frame counts differ")
    joint = np.concatenate([acoustic, semantic], axis=1)
    residual = linear(joint, weights, "fc")
    codes = quantize(weights, cfg, residual)
    if return_features:
        return codes, {"hubert": feats, "semantic": semantic, "acoustic": acoustic, "fc": residual}
    return codes


# ------------------------------------------------------------- tensors

def tensor_shapes(cfg: EncoderShape) -> dict:
    """Every tensor the encoder reads, with the shape the reference expects
    (codec_encoder.cpp:72-247; the quantizer's project_out for the decoded
    entries, codec.cpp:136-160)."""
    s = {}
    cin = 1
    for i, (ch, k) in enumerate(zip(cfg.conv_channels, cfg.conv_kernels)):
        s[f"semantic_model.feature_extractor.conv_layers.{i}.conv.weight"] = (ch, cin, k)
        cin = ch
    c0 = cfg.conv_channels[0]
    s["semantic_model.feature_extractor.conv_layers.0.layer_norm.weight"] = (c0,)
    s["semantic_model.feature_extractor.conv_layers.0.layer_norm.bias"] = (c0,)
    s["semantic_model.feature_projection.layer_norm.weight"] = (cin,)
    s["semantic_model.feature_projection.layer_norm.bias"] = (cin,)
    h = cfg.hidden
    s["semantic_model.feature_projection.projection.weight"] = (h, cin)
    s["semantic_model.feature_projection.projection.bias"] = (h,)
    p = "semantic_model.encoder.pos_conv_embed.conv."
    s[p + "parametrizations.weight.original0"] = (1, 1, cfg.position_kernel)
    s[p + "parametrizations.weight.original1"] = (h, h // cfg.position_groups, cfg.position_kernel)
    s[p + "bias"] = (h,)
    s["semantic_model.encoder.layer_norm.weight"] = (h,)
    s["semantic_model.encoder.layer_norm.bias"] = (h,)
    for layer in range(cfg.layers):
        p = f"semantic_model.encoder.layers.{layer}."
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            s[p + f"attention.{name}.weight"] = (h, h)
            s[p + f"attention.{name}.bias"] = (h,)
        for name in ("layer_norm", "final_layer_norm"):
            s[p + f"{name}.weight"] = (h,)
            s[p + f"{name}.bias"] = (h,)
        s[p + "feed_forward.intermediate_dense.weight"] = (cfg.intermediate, h)
        s[p + "feed_forward.intermediate_dense.bias"] = (cfg.intermediate,)
        s[p + "feed_forward.output_dense.weight"] = (h, cfg.intermediate)
        s[p + "feed_forward.output_dense.bias"] = (h,)
    s["encoder_semantic.conv.weight"] = (h, h, 3)
    for blk in range(2):
        p = f"encoder_semantic.conv_blocks.{blk}."
        for u in range(2):
            s[p + f"res_units.{u}.conv1.weight"] = (h, h, 3)
            s[p + f"res_units.{u}.conv2.weight"] = (h, h, 1)
        s[p + "conv.weight"] = (h, h, 3)
        s[p + "conv.bias"] = (h,)
    ch = cfg.encoder_channels
    s["acoustic_encoder.conv1.weight"] = (ch, 1, RESIDUAL_KERNEL)
    s["acoustic_encoder.conv1.bias"] = (ch,)
    for i, stride in enumerate(cfg.downsampling_ratios):
        p = f"acoustic_encoder.block.{i}."
        for u in range(3):
            q = p + f"res_unit{u + 1}."
            s[q + "snake1.alpha"] = (1, ch, 1)
            s[q + "snake2.alpha"] = (1, ch, 1)
            s[q + "conv1.weight"] = (ch, ch, RESIDUAL_KERNEL)
            s[q + "conv1.bias"] = (ch,)
            s[q + "conv2.weight"] = (ch, ch, 1)
            s[q + "conv2.bias"] = (ch,)
        s[p + "snake1.alpha"] = (1, ch, 1)
        s[p + "conv1.weight"] = (2 * ch, ch, 2 * stride)
        s[p + "conv1.bias"] = (2 * ch,)
        ch *= 2
    s["acoustic_encoder.snake1.alpha"] = (1, ch, 1)
    s["acoustic_encoder.conv2.weight"] = (cfg.latent_channels, ch, 3)
    s["acoustic_encoder.conv2.bias"] = (cfg.latent_channels,)
    j = cfg.joint
    s["fc.weight"] = (j, j)
    s["fc.bias"] = (j,)
    for c in range(cfg.codebooks):
        p = f"quantizer.quantizers.{c}."
        s[p + "project_in.weight"] = (cfg.codebook_dim, j)
        s[p + "project_in.bias"] = (cfg.codebook_dim,)
        s[p + "codebook.embed"] = (cfg.codebook_size, cfg.codebook_dim)
        s[p + "project_out.weight"] = (j, cfg.codebook_dim)
        s[p + "project_out.bias"] = (j,)
    return s


def synthetic_weights(cfg: EncoderShape, seed: int) -> dict:
    """Seeded float32 weights of every encoder tensor (numpy PCG64):
    projections and convolutions N(0, 1 / fan_in) (residual branches scaled
    by 0.5), norm weights 1 + N(0, 0.1), biases N(0, 0.05), snake alphas
    U(0.5, 2), codebooks N(0, 1), the positional convolution's direction
    N(0, 1) and per-tap gains U(0.5, 1.5)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in tensor_shapes(cfg).items():
        if name.endswith("alpha"):
            v = rng.uniform(0.5, 2.0, shape)
        elif name.endswith("codebook.embed"):
            v = rng.standard_normal(shape)
        elif name.endswith("original0"):
            v = rng.uniform(0.5, 1.5, shape)
        elif name.endswith("original1"):
            v = rng.standard_normal(shape)
        elif "norm" in name and name.endswith("weight"):
            v = 1.0 + 0.1 * rng.standard_normal(shape)
        elif name.endswith("bias"):
            v = 0.05 * rng.standard_normal(shape)
        else:
            fan_in = int(np.prod(shape[1:]))
            gain = 0.5 if ("res_unit" in name or "output_dense" in name or "out_proj" in name) else 1.0
            v = gain * rng.standard_normal(shape) / np.sqrt(fan_in)
        out[name] = v.astype(np.float32)
    return out
