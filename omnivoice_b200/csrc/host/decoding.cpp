// Host decoding helpers of the generator (see decoding.hpp).  The schedule
// follows OmniVoice's _get_time_steps: torch.linspace(0, 1, steps + 1) in
// float32 (which fills the first half upward from 0 and the second half
// downward from 1), the shift t' = s t / (1 + (s - 1) t), and per-step
// counts ceil(total * (t[i+1] - t[i])) evaluated in double, clamped to what
// remains, with the remainder at the final step.
#include "decoding.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <numeric>

namespace gufo::models::omnivoice {

std::vector<std::size_t> UnmaskSchedule(std::size_t total, std::size_t steps, float t_shift) {
  std::vector<float> t(steps + 1);
  const float delta = 1.0F / static_cast<float>(steps);
  const std::size_t upper = (steps + 1) / 2;
  for (std::size_t i = 0; i <= steps; ++i) {
    const float linear = i < upper ? delta * static_cast<float>(i)
                                   : 1.0F - delta * static_cast<float>(steps - i);
    t[i] = t_shift * linear / (1.0F + (t_shift - 1.0F) * linear);
  }
  std::vector<std::size_t> counts(steps, 0);
  std::size_t left = total;
  for (std::size_t i = 0; i < steps; ++i) {
    std::size_t n = left;
    if (i + 1 < steps) {
      const double span = static_cast<double>(t[i + 1]) - static_cast<double>(t[i]);
      n = std::min(left, static_cast<std::size_t>(std::ceil(static_cast<double>(total) * span)));
    }
    counts[i] = n;
    left -= n;
  }
  return counts;
}

ConditionalInput ConditionalInput::Build(const std::vector<std::uint32_t>& text_ids,
                                         const std::vector<std::int32_t>& reference_codes,
                                         std::size_t reference_frames, std::size_t target_frames,
                                         std::size_t codebooks, std::uint32_t mask_id) {
  ConditionalInput in;
  in.codebooks = codebooks;
  in.audio_start = text_ids.size();
  in.target_frames = target_frames;
  in.length = text_ids.size() + reference_frames + target_frames;
  in.ids.assign(codebooks * in.length, static_cast<std::int32_t>(mask_id));
  for (std::size_t c = 0; c < codebooks; ++c) {
    auto row = in.ids.begin() + static_cast<std::ptrdiff_t>(c * in.length);
    std::transform(text_ids.begin(), text_ids.end(), row,
                   [](std::uint32_t id) { return static_cast<std::int32_t>(id); });
    std::copy_n(reference_codes.begin() + static_cast<std::ptrdiff_t>(c * reference_frames),
                reference_frames, row + static_cast<std::ptrdiff_t>(text_ids.size()));
  }
  return in;
}

void DrawGumbel(std::mt19937_64* random, std::size_t draws, float* out) {
  for (std::size_t i = 0; i < draws; ++i) {
    const float u = static_cast<float>((*random)() >> 40) * 0x1.0p-24F;
    out[i] = -std::log(-std::log(u + 1e-10F) + 1e-10F);
  }
}

PositionSelector::PositionSelector(const DecodingConfig& config, std::uint64_t seed)
    : layer_penalty_(config.layer_penalty),
      temperature_(config.position_temperature),
      random_(seed) {}

std::vector<std::size_t> PositionSelector::Fill(std::size_t count, std::size_t codebooks,
                                                std::size_t frames,
                                                const std::vector<std::int32_t>& prediction,
                                                const std::vector<float>& confidence,
                                                std::uint32_t mask_id,
                                                std::vector<std::int32_t>* codes) {
  const std::size_t total = codebooks * frames;
  std::vector<float> noise(temperature_ > 0.0F ? total : 0);
  if (!noise.empty()) DrawGumbel(&random_, total, noise.data());
  std::vector<float> score(total);
  for (std::size_t i = 0; i < total; ++i) {
    const float penalty = static_cast<float>(i / frames) * layer_penalty_;
    float s = confidence[i] - penalty;
    if (temperature_ > 0.0F) s = s / temperature_ + noise[i];
    score[i] = (*codes)[i] == static_cast<std::int32_t>(mask_id)
                   ? s
                   : -std::numeric_limits<float>::infinity();
  }
  count = std::min(count, total);
  std::vector<std::size_t> order(total);
  std::iota(order.begin(), order.end(), std::size_t{0});
  const auto better = [&score](std::size_t a, std::size_t b) {
    return score[a] != score[b] ? score[a] > score[b] : a < b;
  };
  std::partial_sort(order.begin(), order.begin() + static_cast<std::ptrdiff_t>(count),
                    order.end(), better);
  order.resize(count);
  for (const std::size_t i : order) (*codes)[i] = prediction[i];
  return order;
}

}  // namespace gufo::models::omnivoice
