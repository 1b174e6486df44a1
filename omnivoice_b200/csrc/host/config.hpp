// The part of the reference's model configuration (config.hpp:14-80) that
// the generator reads: the backbone shape and the audio codebook layout.
// In the reference tree the reference's own config.hpp (which has these
// members and the codec's) is used instead; the drop-in generator reads
// only the members declared here.
#ifndef GUFO_MODELS_OMNIVOICE_CONFIG_HPP_
#define GUFO_MODELS_OMNIVOICE_CONFIG_HPP_

#include <cstddef>
#include <cstdint>

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

struct Config {
  BackboneConfig backbone;
  /// Codebooks the backbone embeds and predicts per audio frame.
  std::size_t audio_codebooks = 0;
  /// Entries per codebook, including the mask.
  std::size_t audio_vocab_size = 0;
  std::uint32_t audio_mask_id = 0;
};

}  // namespace gufo::models::omnivoice

#endif  // GUFO_MODELS_OMNIVOICE_CONFIG_HPP_
