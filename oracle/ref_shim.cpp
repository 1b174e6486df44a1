// C entry points over the reference's own decoding.cpp (compiled from the
// reference tree by oracle/Makefile into oracle/_ref/libref_decoding.so).
// TEST INFRASTRUCTURE ONLY: used by tests/ to pin the oracle's decoding
// restatement against the reference implementation itself.
#include <cstddef>
#include <cstdint>
#include <vector>

#include "decoding.hpp"

namespace ov = gufo::models::omnivoice;

extern "C" {

void ref_unmask_schedule(size_t total, size_t steps, float t_shift, size_t* out) {
  const std::vector<size_t> s = ov::UnmaskSchedule(total, steps, t_shift);
  for (size_t i = 0; i < s.size(); ++i) out[i] = s[i];
}

size_t ref_build_input(const uint32_t* text, size_t text_count, const int32_t* reference,
                       size_t reference_frames, size_t target_frames, size_t codebooks,
                       uint32_t mask_id, int32_t* ids_out) {
  const std::vector<uint32_t> t(text, text + text_count);
  const std::vector<int32_t> r(reference, reference + codebooks * reference_frames);
  const ov::ConditionalInput in =
      ov::ConditionalInput::Build(t, r, reference_frames, target_frames, codebooks, mask_id);
  for (size_t i = 0; i < in.ids.size(); ++i) ids_out[i] = in.ids[i];
  return in.length;
}

// One PositionSelector per call sequence: `seed` starts a new selector when
// `reset` is nonzero, so successive calls consume the same mt19937_64 stream
// as successive steps of Generator::Generate.
size_t ref_fill(int reset, uint64_t seed, float layer_penalty, float temperature, size_t count,
                size_t codebooks, size_t frames, const int32_t* prediction,
                const float* confidence, uint32_t mask_id, int32_t* codes, size_t* chosen) {
  static ov::PositionSelector* selector = nullptr;
  if (reset || selector == nullptr) {
    delete selector;
    ov::DecodingConfig config;
    config.layer_penalty = layer_penalty;
    config.position_temperature = temperature;
    selector = new ov::PositionSelector(config, seed);
  }
  const size_t n = codebooks * frames;
  const std::vector<int32_t> p(prediction, prediction + n);
  const std::vector<float> c(confidence, confidence + n);
  std::vector<int32_t> out(codes, codes + n);
  const std::vector<size_t> order =
      selector->Fill(count, codebooks, frames, p, c, mask_id, &out);
  for (size_t i = 0; i < n; ++i) codes[i] = out[i];
  for (size_t i = 0; i < order.size(); ++i) chosen[i] = order[i];
  return order.size();
}

}  // extern "C"
