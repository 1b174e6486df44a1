// Exercises Codec::Encode of the C++ drop-in (codec.hpp) on a B200.
//
// usage: codec_encoder_dropin_test <model_root> <samples.f32> <count> <codes.i32>
//
// Loads <model_root>/audio_tokenizer/model.safetensors (decoder and encoder
// tensors of the small test tokenizer below) through Codec::Load, encodes
// the <count> samples of <samples.f32> with Codec::Encode and writes the
// [8][frames] codes to <codes.i32> for the Python test to compare with the
// oracle; checks in place the partial-frame message and that Decode takes
// the codes back to frames * 960 samples.  Prints "ok" and exits 0 when
// every check holds.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include "codec.hpp"

using namespace gufo::models::omnivoice;

namespace {

int failures = 0;

void Require(bool ok, const std::string& what) {
  if (!ok) {
    std::printf("FAIL %s\n", what.c_str());
    ++failures;
  }
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 5) {
    std::printf("usage: %s model_root samples count codes\n", argv[0]);
    return 2;
  }
  const size_t count = std::strtoul(argv[3], nullptr, 10);
  // The small tokenizer of tests/test_gpu_codec_encoder.py (SMALL): HuBERT
  // 32 wide, 2 layers of 4 heads; DAC encoder from 4 channels; 8 x 64 codes
  // of width 8; the decoder from 1024 channels.
  Config config;
  CodecConfig& c = config.codec;
  c.sample_rate = 24000;
  c.frame_samples = 960;
  c.codebooks = 8;
  c.codebook_size = 64;
  c.codebook_dim = 8;
  c.semantic_stride = 2;
  SemanticEncoderConfig& s = c.semantic;
  s.sample_rate = 16000;
  s.frame_samples = 320;
  s.hidden_size = 32;
  s.intermediate_size = 64;
  s.heads = 4;
  s.layers = 2;
  s.position_kernel = 16;
  s.position_groups = 4;
  s.layer_norm_eps = 1e-5F;
  s.conv_channels = {16, 16, 16, 16};
  s.conv_kernels = {10, 4, 4, 4};
  s.conv_strides = {5, 4, 4, 4};
  c.acoustic.encoder_channels = 4;
  c.acoustic.decoder_channels = 1024;
  c.acoustic.latent_channels = 32;
  c.acoustic.downsampling_ratios = {8, 5, 4, 2, 3};
  c.acoustic.upsampling_ratios = {8, 5, 4, 2, 3};
  std::string error;
  auto codec = Codec::Load(config, argv[1], &error);
  if (codec == nullptr) {
    std::printf("FAIL load: %s\n", error.c_str());
    return 1;
  }
  std::vector<float> samples(count);
  std::ifstream(argv[2], std::ios::binary)
      .read(reinterpret_cast<char*>(samples.data()), static_cast<std::streamsize>(count * 4));
  std::vector<int32_t> codes;
  size_t frames = 0;
  Require(codec->Encode(samples, &codes, &frames, &error), "encode: " + error);
  Require(frames == count / 960 && codes.size() == 8 * frames, "encoded frame count");
  std::ofstream(argv[4], std::ios::binary)
      .write(reinterpret_cast<const char*>(codes.data()),
             static_cast<std::streamsize>(codes.size() * 4));
  std::vector<int32_t> unused;
  size_t unused_frames = 0;
  std::vector<float> partial(samples.begin(), samples.end() - 1);
  Require(!codec->Encode(partial, &unused, &unused_frames, &error) &&
              error == "OmniVoice encode: reference audio must be a whole number of frames",
          "partial frame message: " + error);
  std::vector<float> audio;
  Require(codec->Decode(codes, frames, &audio, &error) && audio.size() == frames * 960,
          "decode of the encoded codes: " + error);
  if (failures == 0) std::printf("ok\n");
  return failures == 0 ? 0 : 1;
}
