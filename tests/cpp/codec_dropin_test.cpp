// Exercises the C++ drop-in Codec (codec.hpp) on a B200.
//
// usage: codec_dropin_test <model_root> <codes.i32> <frames> <audio.f32>
//          <codebook_dim> <semantic_hidden> <latent> <decoder_channels> <ratio>...
//
// Loads <model_root>/audio_tokenizer/model.safetensors through Codec::Load,
// decodes the [8][frames] codes read from <codes.i32> with Codec::Decode and
// writes the samples to <audio.f32> for the Python test to compare with the
// oracle; checks in place the reference's error messages (code count, code
// range, missing checkpoint) and that Encode, with no encoder in the config,
// reports it.
// Prints "ok" and exits 0 when every check holds.
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

bool StartsWith(const std::string& s, const std::string& p) { return s.rfind(p, 0) == 0; }

}  // namespace

int main(int argc, char** argv) {
  if (argc < 10) {
    std::printf("usage: %s model_root codes frames audio dim semantic latent decoder ratios...\n",
                argv[0]);
    return 2;
  }
  const size_t frames = std::strtoul(argv[3], nullptr, 10);
  Config config;
  CodecConfig& c = config.codec;
  c.sample_rate = 24000;
  c.codebooks = 8;
  c.codebook_size = 1024;
  c.codebook_dim = std::strtoul(argv[5], nullptr, 10);
  c.semantic.hidden_size = std::strtoul(argv[6], nullptr, 10);
  c.acoustic.latent_channels = std::strtoul(argv[7], nullptr, 10);
  c.acoustic.decoder_channels = std::strtoul(argv[8], nullptr, 10);
  c.frame_samples = 1;
  for (int i = 9; i < argc; ++i) {
    c.acoustic.upsampling_ratios.push_back(std::strtoul(argv[i], nullptr, 10));
    c.frame_samples *= c.acoustic.upsampling_ratios.back();
  }
  std::string error;
  Require(Codec::Load(config, "/nonexistent-model-root", &error) == nullptr &&
              StartsWith(error, "OmniVoice audio tokenizer: "),
          "missing checkpoint: " + error);
  auto codec = Codec::Load(config, argv[1], &error);
  if (codec == nullptr) {
    std::printf("FAIL load: %s\n", error.c_str());
    return 1;
  }
  std::vector<int32_t> codes(8 * frames);
  std::ifstream(argv[2], std::ios::binary)
      .read(reinterpret_cast<char*>(codes.data()), static_cast<std::streamsize>(codes.size() * 4));
  std::vector<float> audio;
  Require(codec->Decode(codes, frames, &audio, &error), "decode: " + error);
  Require(audio.size() == frames * c.frame_samples, "decoded length");
  std::ofstream(argv[4], std::ios::binary)
      .write(reinterpret_cast<const char*>(audio.data()),
             static_cast<std::streamsize>(audio.size() * 4));
  std::vector<float> unused;
  Require(!codec->Decode(std::vector<int32_t>(8 * frames + 1, 0), frames, &unused, &error) &&
              error == "OmniVoice decode: code count doesn't match the frames",
          "count message: " + error);
  std::vector<int32_t> bad(8 * frames, 0);
  if (!bad.empty()) bad.back() = 1024;
  Require(frames == 0 || (!codec->Decode(bad, frames, &unused, &error) &&
                          error == "OmniVoice decode: code outside the codebook"),
          "range message: " + error);
  std::vector<int32_t> enc;
  size_t enc_frames = 0;
  Require(!codec->Encode(std::vector<float>(960, 0.0f), &enc, &enc_frames, &error) &&
              StartsWith(error, "OmniVoice encode: "),
          "encode message: " + error);
  if (failures == 0) std::printf("ok\n");
  return failures == 0 ? 0 : 1;
}
