// The part of the reference's model configuration (config.hpp:14-80) that
// the generator and the codec decoder read: the backbone shape, the audio
// codebook layout and the audio tokenizer's decoder shape.
// In the reference tree the reference's own config.hpp (which has these
// members and the codec's) is used instead; the drop-in generator reads
// only the members declared here.
#ifndef GUFO_MODELS_OMNIVOICE_CONFIG_HPP_
#define GUFO_MODELS_OMNIVOICE_CONFIG_HPP_

#include <cstddef>
#include <cstdint>
#include <vector>

namespace gufo::models::omnivoice {

struct BackboneConfig {
  std::size_t vocab_size = 0;
  std::size_t hidden_size = 0;
  std::size_t intermediate_size = 0;
  std::size_t layers = 0;
  std::size_t heads = 0;
  std::size_t kv_heads = 0;
  std::size_t head_dim = 0;
  std::size_t max_positions = 0;
  float rms_norm_eps = 0.0F;
  float rope_theta = 0.0F;
};

/// config.hpp:28-43: of the semantic (HuBERT) encoder the decoder reads
/// only the width, which with the acoustic latent width makes the RVQ's
/// hidden size.
struct SemanticEncoderConfig {
  std::uint32_t sample_rate = 0;
  std::size_t frame_samples = 0;
  std::size_t hidden_size = 0;
  std::size_t intermediate_size = 0;
  std::size_t heads = 0;
  std::size_t layers = 0;
  std::size_t position_kernel = 0;
  std::size_t position_groups = 0;
  float layer_norm_eps = 0.0F;
  std::vector<std::size_t> conv_channels;
  std::vector<std::size_t> conv_kernels;
  std::vector<std::size_t> conv_strides;
};

/// config.hpp:45-52 (DAC encoder and decoder of the acoustic branch).
struct AcousticConfig {
  std::size_t encoder_channels = 0;
  std::size_t decoder_channels = 0;
  std::size_t latent_channels = 0;
  std::vector<std::size_t> downsampling_ratios;
  std::vector<std::size_t> upsampling_ratios;
};

/// config.hpp:54-72 (Higgs Audio v2 tokenizer).
struct CodecConfig {
  std::uint32_t sample_rate = 0;
  std::size_t frame_samples = 0;
  std::size_t codebooks = 0;
  std::size_t codebook_size = 0;
  std::size_t codebook_dim = 0;
  std::size_t semantic_stride = 0;
  SemanticEncoderConfig semantic;
  AcousticConfig acoustic;

  [[nodiscard]] std::uint32_t FrameRate() const {
    return frame_samples == 0 ? 0 : sample_rate / static_cast<std::uint32_t>(frame_samples);
  }
};

struct Config {
  BackboneConfig backbone;
  /// Codebooks the backbone embeds and predicts per audio frame.
  std::size_t audio_codebooks = 0;
  /// Entries per codebook, including the mask.
  std::size_t audio_vocab_size = 0;
  std::uint32_t audio_mask_id = 0;
  CodecConfig codec;
};

}  // namespace gufo::models::omnivoice

#endif  // GUFO_MODELS_OMNIVOICE_CONFIG_HPP_
