// Device-side description of a packed batch of utterances, shared by the
// score and selection kernels and the generator host code.
//
// Utterance u occupies packed rows [row_base, row_base + length) for its
// conditional sequence and [row_base + length, row_base + length + frames)
// for its unconditional one (the reference packs one utterance the same
// way, generator.cpp:175-258).  Its logits rows start at logit_row
// (conditional frames, then unconditional), and its [codebook][frame] slots
// start at slot_base in the code / prediction / confidence arrays.
#pragma once

#include <cstdint>

namespace ovb {

struct UttDesc {
  int32_t row_base;
  int32_t length;
  int32_t frames;
  int32_t audio_start;
  int32_t frame_base;  // sum of the frames of earlier utterances
  int32_t logit_row;   // 2 * frame_base
  int32_t slot_base;   // codebooks * frame_base
  int32_t gumbel_stride;  // floats per step in `gumbel` (codebooks * frames)
  uint64_t noise_seed;
  const float* gumbel;    // [steps][codebooks * frames] Gumbel values, or null
  const int32_t* counts;  // [steps] codes to unmask per step, or null
};

// Step bookkeeping that lets one recorded CUDA graph serve every step: the
// selection kernel reads the step it runs from step_list[launch[u]] and
// advances launch[u] when done.
struct StepControl {
  const int32_t* step_list;  // real step numbers of the launched steps
  int32_t* launch;           // per utterance launch counter
};

}  // namespace ovb
