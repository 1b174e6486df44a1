// The reference's Codec (codec.hpp:17-43) over ov_codec.h.
#include "codec.hpp"

#include <cuda_runtime.h>

#include <algorithm>

#include "ov_codec.h"
#include "ov_runtime.h"

namespace gufo::models::omnivoice {

struct Codec::State {
  ov_codec* codec = nullptr;
  ov_codec_encoder* encoder = nullptr;  // null: the config describes no encoder
  CodecConfig config;
  ~State() {
    ov_codec_free(codec);
    ov_codec_encoder_free(encoder);
  }
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
  // The encoder (codec.cpp:188, LoadEncoder) when the config describes it.
  const SemanticEncoderConfig& sem = c.semantic;
  if (!sem.conv_channels.empty()) {
    ov_codec_encoder_config ec{};
    ec.sample_rate = c.sample_rate;
    ec.codebooks = c.codebooks;
    ec.codebook_size = c.codebook_size;
    ec.codebook_dim = c.codebook_dim;
    ec.semantic_sample_rate = sem.sample_rate;
    ec.hidden_size = sem.hidden_size;
    ec.intermediate_size = sem.intermediate_size;
    ec.heads = sem.heads;
    ec.layers = sem.layers;
    ec.position_kernel = sem.position_kernel;
    ec.position_groups = sem.position_groups;
    ec.layer_norm_eps = sem.layer_norm_eps;
    const std::vector<size_t>& ratios = c.acoustic.downsampling_ratios;
    if (sem.conv_channels.size() > 8 || sem.conv_kernels.size() != sem.conv_channels.size() ||
        sem.conv_strides.size() != sem.conv_channels.size() || ratios.empty() || ratios.size() > 8) {
      SetError(error, "OmniVoice audio tokenizer: 1 to 8 feature-extractor convolutions and "
                      "downsampling blocks are supported");
      return nullptr;
    }
    for (size_t i = 0; i < sem.conv_channels.size(); ++i) {
      ec.conv_channels[i] = sem.conv_channels[i];
      ec.conv_kernels[i] = sem.conv_kernels[i];
      ec.conv_strides[i] = sem.conv_strides[i];
    }
    ec.num_convs = sem.conv_channels.size();
    ec.encoder_channels = c.acoustic.encoder_channels;
    ec.latent_channels = c.acoustic.latent_channels;
    for (size_t i = 0; i < ratios.size(); ++i) ec.downsampling_ratios[i] = ratios[i];
    ec.num_downsampling = ratios.size();
    if (ov_codec_encoder_load(&ec, path.c_str(), device, &state->encoder) != OV_OK) {
      SetError(error, LastError());
      return nullptr;
    }
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

// codec_encoder.cpp:249-458.
bool Codec::Encode(const std::vector<float>& samples, std::vector<std::int32_t>* codes,
                   std::size_t* frames, std::string* error) {
  if (state_->encoder == nullptr) {
    SetError(error, "OmniVoice encode: the config describes no encoder (semantic_model_config)");
    return false;
  }
  std::vector<std::int32_t> out(state_->config.codebooks *
                                (samples.size() / std::max<size_t>(
                                                      ov_codec_encoder_frame_samples(state_->encoder), 1) +
                                 1));
  size_t count = 0;
  if (ov_codec_encode(state_->encoder, samples.data(), samples.size(), out.data(), out.size(),
                      &count) != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  out.resize(state_->config.codebooks * count);
  *codes = std::move(out);
  *frames = count;
  return true;
}

}  // namespace gufo::models::omnivoice
