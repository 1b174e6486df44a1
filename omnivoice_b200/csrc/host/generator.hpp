// Drop-in for the reference's generator (generator.hpp:16-56): the same
// class, members and semantics, implemented on the B200 C-ABI
// (ov_generator.h).  A caller built against the reference's generator.hpp
// links against libomnivoice_b200.so instead of generator.cpp, gemm.cpp
// and the HIP kernels.  GenerateBatch is an addition: several utterances
// packed into one varlen batch that shares the unmasking loop.
#ifndef GUFO_MODELS_OMNIVOICE_GENERATOR_HPP_
#define GUFO_MODELS_OMNIVOICE_GENERATOR_HPP_

#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "config.hpp"
#include "decoding.hpp"

namespace gufo::models::omnivoice {

/// The bidirectional Qwen3 backbone with its audio embeddings and heads on
/// one B200, and OmniVoice's iterative unmasking with classifier-free
/// guidance, every step on the device.  Uses the GPU current at Load.  Not
/// thread-safe: one instance per GPU worker.
class Generator {
 public:
  /// Reads model_root / "model.safetensors" (the reference's tensor names).
  /// Failures return nullptr with "OmniVoice generator: ..." in *error.
  [[nodiscard]] static std::unique_ptr<Generator> Load(const Config& config,
                                                       const std::filesystem::path& model_root,
                                                       std::string* error = nullptr);
  ~Generator();
  Generator(const Generator&) = delete;
  Generator& operator=(const Generator&) = delete;

  /// Runs the unmasking loop from `input`'s masked target.  `cancelled` is
  /// polled before every step; cancelling returns false with *error
  /// "cancelled".  Position noise is the reference's std::mt19937_64(seed)
  /// stream, so results match the reference's host selection.
  [[nodiscard]] bool Generate(const ConditionalInput& input, const DecodingConfig& decoding,
                              std::uint64_t seed, const std::function<bool()>& cancelled,
                              GenerationResult* result, std::string* error = nullptr);

  /// Generate for several inputs packed into one batch (seeds[i] for
  /// inputs[i]); results[i] matches a single Generate of inputs[i].
  [[nodiscard]] bool GenerateBatch(const std::vector<ConditionalInput>& inputs,
                                   const DecodingConfig& decoding,
                                   const std::vector<std::uint64_t>& seeds,
                                   const std::function<bool()>& cancelled,
                                   std::vector<GenerationResult>* results,
                                   std::string* error = nullptr);

  /// One forward pass of the CFG batch; `logits` receives the target
  /// frames' rows, conditional then unconditional, [2 * frames][codebooks *
  /// vocab].
  [[nodiscard]] bool Forward(const ConditionalInput& input, std::vector<float>* logits,
                             std::string* error = nullptr);

  /// Forward plus the scoring step: per [codebook][frame] the guided
  /// argmax and its log-probability.
  [[nodiscard]] bool Score(const ConditionalInput& input, float guidance,
                           std::vector<std::int32_t>* prediction, std::vector<float>* confidence,
                           std::string* error = nullptr);

 private:
  struct State;
  explicit Generator(std::unique_ptr<State> state);
  std::unique_ptr<State> state_;
};

}  // namespace gufo::models::omnivoice

#endif  // GUFO_MODELS_OMNIVOICE_GENERATOR_HPP_
