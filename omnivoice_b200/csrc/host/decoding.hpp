// Drop-in replacement of the reference's decoding.hpp (decoding.hpp:14-77):
// the host side of OmniVoice's iterative unmasking.  Same names, fields,
// signatures and semantics; the generator runs the per-step selection on
// the device and uses these for the schedule, the conditional input layout
// and the reference-compatible noise stream.
#ifndef OMNIVOICE_B200_HOST_DECODING_HPP_
#define OMNIVOICE_B200_HOST_DECODING_HPP_

#include <cstddef>
#include <cstdint>
#include <random>
#include <vector>

namespace gufo::models::omnivoice {

/// OmniVoiceGenerationConfig's decoding parameters (decoding.hpp:14-21).
struct DecodingConfig {
  std::size_t steps = 32;
  float guidance = 2.0F;
  float t_shift = 0.1F;
  float layer_penalty = 5.0F;
  /// Gumbel noise on the position scores; 0 selects positions greedily.
  float position_temperature = 5.0F;
};

/// Codes to unmask per step: ceil(total * (t[s+1] - t[s])) of the shifted
/// float32 linear schedule, the remainder at the last step (decoding.cpp:12-40).
[[nodiscard]] std::vector<std::size_t> UnmaskSchedule(std::size_t total, std::size_t steps,
                                                      float t_shift);

/// [text tokens | reference frames | target frames] in `codebooks` rows of
/// `length` ids (decoding.hpp:32-47).
struct ConditionalInput {
  std::size_t codebooks = 0;
  std::size_t length = 0;
  std::size_t audio_start = 0;
  std::size_t target_frames = 0;
  /// [codebook][position].
  std::vector<std::int32_t> ids;

  /// `reference_codes` is [codebook][frame] (decoding.cpp:42-62).
  [[nodiscard]] static ConditionalInput Build(const std::vector<std::uint32_t>& text_ids,
                                              const std::vector<std::int32_t>& reference_codes,
                                              std::size_t reference_frames,
                                              std::size_t target_frames, std::size_t codebooks,
                                              std::uint32_t mask_id);
};

struct GenerationResult {
  /// [codebook][frame].
  std::vector<std::int32_t> codes;
  /// The step that unmasked each code, [codebook][frame].
  std::vector<std::int32_t> unmasked_at;
};

/// The host position choice of one step (decoding.cpp:64-107).  The B200
/// generator runs the same choice on the device; this class keeps the
/// reference's host API for callers that use it directly.
class PositionSelector {
 public:
  PositionSelector(const DecodingConfig& config, std::uint64_t seed);

  /// Returns the flat indices it filled, best first.
  std::vector<std::size_t> Fill(std::size_t count, std::size_t codebooks, std::size_t frames,
                                const std::vector<std::int32_t>& prediction,
                                const std::vector<float>& confidence, std::uint32_t mask_id,
                                std::vector<std::int32_t>* codes);

 private:
  float layer_penalty_;
  float temperature_;
  std::mt19937_64 random_;
};

/// The Gumbel values PositionSelector draws for `draws` consecutive slots
/// from `random` (u = (x >> 40) * 2^-24, -log(-log(u + 1e-10) + 1e-10)).
void DrawGumbel(std::mt19937_64* random, std::size_t draws, float* out);

}  // namespace gufo::models::omnivoice

#endif  // OMNIVOICE_B200_HOST_DECODING_HPP_
