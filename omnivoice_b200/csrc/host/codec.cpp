// The reference's Codec (codec.hpp:17-43) over ov_codec.h.
#include "codec.hpp"

#include <cuda_runtime.h>

#include <algorithm>

#include "ov_codec.h"
#include "ov_runtime.h"

namespace gufo::models::omnivoice {

struct Codec::State {
  ov_codec* codec = nullptr;
  CodecConfig config;
  ~State() { ov_codec_free(codec); }
};

namespace {

std::string LastError() {
  char buf[1024];
  ov_last_error(buf, sizeof(buf));
  return buf;
}

void SetError(std::string* error, const std::string& message) {
  if (error != nullptr) *error = message;
}

}  // namespace

Codec::Codec(std::unique_ptr<State> state) : state_(std::move(state)) {}
Codec::~Codec() = default;

std::unique_ptr<Codec> Codec::Load(const Config& config, const std::filesystem::path& model_root,
                                   std::string* error) {
  const CodecConfig& c = config.codec;
  ov_codec_config cc{};
  cc.codebooks = c.codebooks;
  cc.codebook_size = c.codebook_size;
  cc.codebook_dim = c.codebook_dim;
  cc.semantic_hidden = c.semantic.hidden_size;
  cc.latent_channels = c.acoustic.latent_channels;
  cc.decoder_channels = c.acoustic.decoder_channels;
  if (c.acoustic.upsampling_ratios.empty() || c.acoustic.upsampling_ratios.size() > 8) {
    SetError(error, "OmniVoice audio tokenizer: 1 to 8 upsampling blocks are supported");
    return nullptr;
  }
  for (size_t i = 0; i < c.acoustic.upsampling_ratios.size(); ++i)
    cc.upsampling_ratios[i] = c.acoustic.upsampling_ratios[i];
  cc.num_upsampling = c.acoustic.upsampling_ratios.size();
  cc.sample_rate = c.sample_rate;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) device = 0;
  auto state = std::make_unique<State>();
  state->config = c;
  const std::string path = (model_root / "audio_tokenizer" / "model.safetensors").string();
  if (ov_codec_load(&cc, path.c_str(), device, &state->codec) != OV_OK) {
    SetError(error, LastError());
    return nullptr;
  }
  if (c.frame_samples != 0 && ov_codec_frame_samples(state->codec) != c.frame_samples) {
    SetError(error, "OmniVoice audio tokenizer: the upsampling ratios don't multiply to hop_length");
    return nullptr;
  }
  return std::unique_ptr<Codec>(new Codec(std::move(state)));
}

// codec.cpp:195-262.
bool Codec::Decode(const std::vector<std::int32_t>& codes, std::size_t frames,
                   std::vector<float>* audio, std::string* error) {
  if (codes.size() != state_->config.codebooks * frames) {
    SetError(error, "OmniVoice decode: code count doesn't match the frames");
    return false;
  }
  std::vector<float> out(frames * ov_codec_frame_samples(state_->codec));
  if (ov_codec_decode(state_->codec, codes.data(), frames, out.data()) != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  *audio = std::move(out);
  return true;
}

bool Codec::Encode(const std::vector<float>&, std::vector<std::int32_t>*, std::size_t*,
                   std::string* error) {
  SetError(error, "OmniVoice encode: not available in this build");
  return false;
}

}  // namespace gufo::models::omnivoice
