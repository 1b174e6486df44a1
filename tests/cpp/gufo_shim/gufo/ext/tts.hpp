// Minimal stand-in for the Gufo SDK's speech-synthesis extension interface
// (gufo-org/gufo, not in this tree): only the types and members that the
// OmniVoice provider (provider.cpp:8-19) and runner (runner.cpp:44-141,
// runner.hpp) use, with their names and meanings, so a provider/runner
// translation unit of this shape compiles and links against
// libomnivoice_b200.so here.  A Gufo build uses the SDK's own header.
#ifndef GUFO_EXT_TTS_HPP_
#define GUFO_EXT_TTS_HPP_

#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <functional>
#include <memory>
#include <optional>
#include <span>
#include <string>
#include <string_view>
#include <vector>

namespace gufo::ext {

/// Interleaved float samples.
struct TtsAudioBuffer {
  std::uint32_t sample_rate = 0;
  std::uint32_t channels = 0;
  std::vector<float> samples;
};

struct SamplingOptions {
  bool sample = true;
  std::uint64_t seed = 0;
};

struct SynthesisRequest {
  std::string text;
  std::string language;
  std::string instruct;
  std::size_t max_new_tokens = 0;
  SamplingOptions sampling;
  TtsAudioBuffer reference_audio;
  std::string reference_text;
  bool speaker_embedding_only = false;
  /// Streaming: called with each piece of audio; false stops the request.
  std::function<bool(std::span<const float>)> on_audio;
};

struct SynthesisResult {
  std::uint32_t sample_rate = 0;
  /// Codebooks per frame of `codes` ([frame][codebook]).
  std::uint32_t code_groups = 0;
  std::vector<std::int32_t> codes;
  std::size_t sample_count = 0;
  std::vector<float> samples;
};

using CancellationCheck = std::function<bool()>;

enum class TtsVariant { kBase };
enum class TtsConditioningMode { kNone, kOptional, kRequired };

struct TtsConditioningCapabilities {
  bool unconditioned = false;
  bool require_voice = false;
  std::string default_voice;
  TtsConditioningMode reference_audio = TtsConditioningMode::kNone;
  bool reference_presets = false;
  TtsConditioningMode instructions = TtsConditioningMode::kNone;
};

struct TtsRunnerOptions {
  std::filesystem::path model_root;
};

class TtsRunner {
 public:
  virtual ~TtsRunner() = default;
  virtual bool Synthesize(const SynthesisRequest& request, const CancellationCheck& is_cancelled,
                          SynthesisResult* result, std::string* error) = 0;
  virtual std::vector<std::string> Voices() const = 0;
  virtual TtsVariant Variant() const = 0;
  virtual std::uint32_t SampleRate() const = 0;
  virtual TtsConditioningCapabilities Conditioning() const = 0;
  virtual std::string ModelId() const = 0;
};

/// A speech-synthesis provider as Registry::AddTtsProvider takes it.
struct TtsProvider {
  std::string id;
  bool (*probe)(std::string_view model_root) = nullptr;
  bool (*resolve)(std::string_view model_root, std::string* error) = nullptr;
  std::unique_ptr<TtsRunner> (*create)(const std::filesystem::path& model_root,
                                       std::string* error) = nullptr;
  std::unique_ptr<TtsRunner> (*create_with_options)(const TtsRunnerOptions& options,
                                                    std::string* error) = nullptr;
};

}  // namespace gufo::ext

#endif  // GUFO_EXT_TTS_HPP_
