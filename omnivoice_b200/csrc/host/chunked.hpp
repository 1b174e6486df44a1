// Generation and decoding of the chunks of one long text, the part of the
// reference's Synthesizer::Synthesize (synthesizer.cpp:163-201) that runs on
// the GPU, over one or several GPUs.
//
// The reference generates and decodes the chunks strictly one after the
// other.  The only dependency between chunks is the voice carry-over:
// without a caller-supplied reference voice, chunk 0's text and codes become
// the reference of every later chunk (synthesizer.cpp:196-200).  So chunks
// 1..n-1 are independent once chunk 0 is done (all n are when the caller
// gives a reference).  ChunkedSynthesis keeps the reference's results and
// runs them as: chunk 0 alone when its codes carry the voice; the remaining
// chunks spread over the generators (one per GPU, longest-processing-time
// first on the rows each chunk packs), each generator's share as one packed
// batch (Generator::GenerateBatch) on its own host thread; every chunk then
// decoded by the codec of the GPU that generated it (chunks are separate
// signals: a decoder's convolutions must not see across chunk boundaries).
//
// Text chunking, prompt building and tokenisation (synthesizer.cpp:166-178,
// prompt.cpp) stay with the caller: `build(index, voice, &input)` makes the
// conditional input of chunk `index` given the carried voice (null, or
// chunk 0's codes).  Cross-fading and post-processing of the pieces
// (synthesizer.cpp:202-206) are the caller's too.
#ifndef OMNIVOICE_B200_CHUNKED_HPP_
#define OMNIVOICE_B200_CHUNKED_HPP_

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

#include "codec.hpp"
#include "decoding.hpp"
#include "generator.hpp"

namespace gufo::models::omnivoice {

/// The voice chunk 0 hands to the later chunks: its codes
/// ([codebook][frame]) and the index of the chunk whose text they speak.
struct CarriedVoice {
  std::size_t index = 0;
  std::vector<std::int32_t> codes;
  std::size_t frames = 0;
};

/// One generated (and decoded) chunk.
struct SynthesizedChunk {
  std::vector<std::int32_t> codes;  // [codebook][frame]
  std::size_t frames = 0;
  std::vector<float> audio;         // empty without a codec
};

class ChunkedSynthesis {
 public:
  using BuildInput = std::function<bool(std::size_t index, const CarriedVoice* voice,
                                        ConditionalInput* input, std::string* error)>;

  /// generators[g] (and codecs[g], when given) belong to GPU g; `codecs` may
  /// be empty to skip decoding, else it has one codec per generator.  The
  /// objects stay owned by the caller and must outlive this one.
  ChunkedSynthesis(std::vector<Generator*> generators, std::vector<Codec*> codecs);

  /// Generates (and decodes) `count` chunks into *chunks, in chunk order.
  /// `has_reference`: the caller's prompts already carry a reference voice,
  /// so there is no carry-over and every chunk runs in the spread batch.
  /// Every chunk uses `seed` (the reference passes the same options to each
  /// chunk).  `cancelled` is polled before every unmasking step of every
  /// generator; cancelling returns false with *error "cancelled".
  [[nodiscard]] bool Run(std::size_t count, const BuildInput& build, bool has_reference,
                         const DecodingConfig& decoding, std::uint64_t seed,
                         const std::function<bool()>& cancelled,
                         std::vector<SynthesizedChunk>* chunks, std::string* error = nullptr);

 private:
  std::vector<Generator*> generators_;
  std::vector<Codec*> codecs_;
};

}  // namespace gufo::models::omnivoice

#endif  // OMNIVOICE_B200_CHUNKED_HPP_
