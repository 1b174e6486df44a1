// C exports of the host decoding helpers (ov_generator.h).
#include <algorithm>
#include <vector>

#include "decoding.hpp"
#include "ov_generator.h"

namespace ov = gufo::models::omnivoice;

extern "C" {

int ov_unmask_schedule(size_t total, size_t steps, float t_shift, size_t* counts) {
  if (steps == 0 || counts == nullptr) return OV_ERR_INVALID;
  const std::vector<size_t> s = ov::UnmaskSchedule(total, steps, t_shift);
  std::copy(s.begin(), s.end(), counts);
  return OV_OK;
}

size_t ov_build_conditional_input(const uint32_t* text_ids, size_t text_count,
                                  const int32_t* reference_codes, size_t reference_frames,
                                  size_t target_frames, size_t codebooks, uint32_t mask_id,
                                  int32_t* ids) {
  const std::vector<uint32_t> text(text_ids, text_ids + text_count);
  const std::vector<int32_t> reference(
      reference_codes, reference_codes + (reference_codes ? codebooks * reference_frames : 0));
  const ov::ConditionalInput in = ov::ConditionalInput::Build(
      text, reference, reference_codes ? reference_frames : 0, target_frames, codebooks, mask_id);
  std::copy(in.ids.begin(), in.ids.end(), ids);
  return in.length;
}

}  // extern "C"
