// Drop-in for the reference's audio tokenizer class (codec.hpp:17-43): the
// same class and signatures, with Load, Decode and Encode implemented on the
// B200 C-ABI (ov_codec.h).  Load also loads the encoder when the config
// describes one (semantic.conv_channels set, as the reference's config
// parser always does); without it Encode returns false with an
// "OmniVoice encode: " message.
#ifndef GUFO_MODELS_OMNIVOICE_CODEC_HPP_
#define GUFO_MODELS_OMNIVOICE_CODEC_HPP_

#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <memory>
#include <string>
#include <vector>

#include "config.hpp"

namespace gufo::models::omnivoice {

/// The Higgs Audio v2 tokenizer on one B200: RVQ codes to 24 kHz audio and
/// back.  Uses the GPU current at Load.  Not thread-safe.
class Codec {
 public:
  /// Reads model_root / "audio_tokenizer" / "model.safetensors" (float32,
  /// the reference's tensor names).  Failures return nullptr with
  /// "OmniVoice audio tokenizer: ..." in *error.
  [[nodiscard]] static std::unique_ptr<Codec> Load(const Config& config,
                                                   const std::filesystem::path& model_root,
                                                   std::string* error = nullptr);
  ~Codec();
  Codec(const Codec&) = delete;
  Codec& operator=(const Codec&) = delete;

  /// `codes` is [codebook][frame]; yields frames * frame_samples samples.
  [[nodiscard]] bool Decode(const std::vector<std::int32_t>& codes, std::size_t frames,
                            std::vector<float>* audio, std::string* error = nullptr);

  /// `samples` at sample_rate, a whole number of frames; yields
  /// [codebook][frame] codes and the frame count.
  [[nodiscard]] bool Encode(const std::vector<float>& samples, std::vector<std::int32_t>* codes,
                            std::size_t* frames, std::string* error = nullptr);

 private:
  struct State;
  explicit Codec(std::unique_ptr<State> state);
  std::unique_ptr<State> state_;
};

}  // namespace gufo::models::omnivoice

#endif  // GUFO_MODELS_OMNIVOICE_CODEC_HPP_
