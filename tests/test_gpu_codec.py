"""The CUDA codec decoder (include/ov_codec.h) against the float64 oracle
(oracle/codec.py, itself pinned to transformers' decoder) on the same
seeded weights, written to a safetensors file with the reference's tensor
names and loaded through ov_codec_load.

Tolerance: the reference's own codec test bar (tests/codec_test.cpp:
66-67), relative to the signal: max |sample error| <= 1e-3 * rms and
|rms error| <= 1e-4 * rms; the split-operand tf32 products keep float32
accuracy, so the measured errors sit orders of magnitude below it."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from model_files import write_safetensors  # noqa: E402
from omnivoice_b200.codec import Codec, CodecConfig, CodecError  # noqa: E402
from oracle import codec as oc  # noqa: E402

pytestmark = pytest.mark.gpu

SHAPES = {
    # every width >= 32 (the tensor-core convolutions); strides even and odd
    "narrow": dict(codebook_dim=8, semantic_hidden=32, latent_channels=32, decoder_channels=256,
                   upsampling_ratios=[2, 3, 4]),
    "wide": dict(codebook_dim=16, semantic_hidden=96, latent_channels=64, decoder_channels=512,
                 upsampling_ratios=[8, 5, 2, 3]),
    "default": {},
}


def build(name, tmp_path, seed):
    shape = oc.CodecShape(**SHAPES[name])
    weights = oc.synthetic_weights(shape, seed)
    path = tmp_path / f"{name}.safetensors"
    write_safetensors(path, weights)
    cfg = CodecConfig(**{k: getattr(shape, k) for k in (
        "codebooks", "codebook_size", "codebook_dim", "semantic_hidden", "latent_channels",
        "decoder_channels")}, upsampling_ratios=list(shape.upsampling_ratios))
    return shape, weights, Codec.load(cfg, str(path))


def check(audio, want):
    rms = float(np.sqrt(np.mean(want ** 2)))
    err = np.abs(audio.astype(np.float64) - want)
    assert audio.shape == want.shape
    assert np.isfinite(audio).all()
    assert err.max() <= 1e-3 * rms, (err.max(), rms)
    assert abs(np.sqrt(np.mean(audio.astype(np.float64) ** 2)) - rms) <= 1e-4 * rms
    return err.max() / rms


@pytest.mark.parametrize("name,frames", [("narrow", 1), ("narrow", 37), ("wide", 5), ("wide", 130),
                                         ("default", 3)])
def test_decode_matches_oracle(cuda_device, native, tmp_path, name, frames):
    shape, weights, codec = build(name, tmp_path, seed=frames)
    rng = np.random.default_rng(frames)
    codes = rng.integers(0, shape.codebook_size, (shape.codebooks, frames))
    audio = codec.decode(codes)
    rel = check(audio, oc.decode(weights, shape, codes))
    print(f"{name} frames={frames}: max error {rel:.2e} of rms")
    codec.close()


def test_decode_device_and_repeat_and_frame_changes(cuda_device, native, tmp_path):
    shape, weights, codec = build("narrow", tmp_path, seed=4)
    rng = np.random.default_rng(4)
    results = {}
    for frames in (9, 2, 9):  # the plan changes size and comes back
        codes = rng.integers(0, shape.codebook_size, (shape.codebooks, frames))
        host = codec.decode(codes)
        check(host, oc.decode(weights, shape, codes))
        dev_codes = torch.from_numpy(codes.astype(np.int32)).cuda()
        dev_audio = torch.empty(frames * shape.frame_samples, device="cuda")
        codec.decode_device(dev_codes, dev_audio, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert np.array_equal(dev_audio.cpu().numpy(), host)  # same kernels, same order
        results.setdefault(frames, []).append(host)
    codec.close()


def test_decode_rejects_bad_codes_with_reference_messages(cuda_device, native, tmp_path):
    shape, _, codec = build("narrow", tmp_path, seed=1)
    with pytest.raises(CodecError, match="^OmniVoice decode: code outside the codebook"):
        codec.decode(np.full((shape.codebooks, 3), shape.codebook_size))
    with pytest.raises(CodecError, match="^OmniVoice decode: code count"):
        codec.decode(np.zeros((shape.codebooks - 1, 3), np.int64))
    assert codec.decode(np.zeros((shape.codebooks, 0), np.int64)).shape == (0,)
    codec.close()


def test_load_reports_missing_tensor(cuda_device, native, tmp_path):
    shape = oc.CodecShape(**SHAPES["narrow"])
    weights = oc.synthetic_weights(shape, 1)
    del weights["acoustic_decoder.block.1.res_unit2.conv1.bias"]
    path = tmp_path / "broken.safetensors"
    write_safetensors(path, weights)
    cfg = CodecConfig(codebook_dim=8, semantic_hidden=32, latent_channels=32,
                      decoder_channels=256, upsampling_ratios=[2, 3, 4])
    with pytest.raises(CodecError, match="^OmniVoice audio tokenizer: .*res_unit2.conv1.bias"):
        Codec.load(cfg, str(path))


def test_synthetic_default_decodes_finite_audio(cuda_device, native):
    codec = Codec.synthetic(CodecConfig(), seed=3)
    codes = np.random.default_rng(3).integers(0, 1024, (8, 25))
    audio = codec.decode(codes)
    assert audio.shape == (25 * 960,) and np.isfinite(audio).all() and audio.std() > 0
    codec.close()


def test_cpp_dropin_codec_matches_oracle(cuda_device, native, tmp_path):
    """The reference's C++ Codec interface (host/codec.hpp) built against
    the library: Load from <root>/audio_tokenizer/model.safetensors, Decode,
    the reference's error messages."""
    import subprocess
    from pathlib import Path
    exe = Path(__file__).resolve().parents[1] / "omnivoice_b200" / "_build" / "codec_dropin_test"
    if not exe.exists():
        pytest.skip("codec_dropin_test not built (python -m omnivoice_b200.build)")
    shape = oc.CodecShape(**SHAPES["wide"])
    weights = oc.synthetic_weights(shape, 9)
    (tmp_path / "audio_tokenizer").mkdir()
    write_safetensors(tmp_path / "audio_tokenizer" / "model.safetensors", weights)
    frames = 11
    codes = np.random.default_rng(9).integers(0, 1024, (8, frames)).astype(np.int32)
    codes.tofile(tmp_path / "codes.i32")
    out = subprocess.run([str(exe), str(tmp_path), str(tmp_path / "codes.i32"), str(frames),
                          str(tmp_path / "audio.f32"), str(shape.codebook_dim),
                          str(shape.semantic_hidden), str(shape.latent_channels),
                          str(shape.decoder_channels)] + [str(r) for r in shape.upsampling_ratios],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout + out.stderr
    audio = np.fromfile(tmp_path / "audio.f32", np.float32)
    check(audio, oc.decode(weights, shape, codes))
