// A Gufo speech provider and runner built on this library, in the shape of
// the reference's provider.cpp:8-19 and runner.cpp:44-141, compiled against
// the Gufo SDK stand-in headers of tests/cpp/gufo_shim (the SDK itself is
// not in this tree) and linked against libomnivoice_b200.so.
//
// What is OmniVoice-specific and outside the generator path stays out:
// there is no tokenizer, text normalisation, prompt builder or audio
// post-processing here, so this runner takes its request text as token ids
// already chunked ("12 7 99|5 1 2": chunks separated by '|') and returns the
// chunks' decoded audio one after another.  Everything on the GPU is the
// library's: the C++ Generator and Codec drop-ins and ChunkedSynthesis
// (chunk 0 first, its voice carried to the others, the remaining chunks
// spread over the generators as packed batches).
//
// usage:
//   gufo_runner_test
//       registers the provider into a Registry and checks what it received
//       (no GPU needed);
//   gufo_runner_test <model_root> <out_dir> <vocab> <hidden> <intermediate>
//       <layers> <heads> <kv_heads> <codebook_dim> <semantic_hidden> <latent>
//       <decoder_channels> <ratio>...
//       also writes <model_root>/b200_shape.txt (the stand-in for the
//       checkpoint's config.json), creates the runner through the provider,
//       synthesises a three-chunk request and checks it against the
//       reference's chunk-by-chunk order (Generator::Generate and
//       Codec::Decode per chunk, the voice carried from chunk 0); writes the
//       samples and codes to <out_dir>.
// Prints "ok" and exits 0 when every check holds.
#include <gufo/ext/generated/omnivoice_constants.hpp>
#include <gufo/ext/registry.hpp>
#include <gufo/ext/tts.hpp>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "chunked.hpp"
#include "codec.hpp"
#include "decoding.hpp"
#include "generator.hpp"

namespace fs = std::filesystem;
using namespace gufo::models::omnivoice;

namespace b200_runner {

constexpr std::size_t kCodebooks = 8;

// <model_root>/b200_shape.txt: the backbone and codec sizes, one line.
bool ReadShape(const fs::path& root, Config* config) {
  std::ifstream in(root / "b200_shape.txt");
  if (!in) return false;
  Config c;
  BackboneConfig& b = c.backbone;
  std::size_t dim = 0, semantic = 0, latent = 0, decoder = 0, ratios = 0;
  in >> b.vocab_size >> b.hidden_size >> b.intermediate_size >> b.layers >> b.heads >>
      b.kv_heads >> dim >> semantic >> latent >> decoder >> ratios;
  if (!in) return false;
  b.head_dim = 128;
  b.max_positions = 40960;
  b.rms_norm_eps = 1e-6F;
  b.rope_theta = 1e6F;
  c.audio_codebooks = kCodebooks;
  c.audio_vocab_size = 1025;
  c.audio_mask_id = 1024;
  CodecConfig& k = c.codec;
  k.sample_rate = 24000;
  k.codebooks = kCodebooks;
  k.codebook_size = 1024;
  k.codebook_dim = dim;
  k.semantic.hidden_size = semantic;
  k.acoustic.latent_channels = latent;
  k.acoustic.decoder_channels = decoder;
  k.frame_samples = 1;
  for (std::size_t i = 0; i < ratios; ++i) {
    std::size_t r = 0;
    in >> r;
    k.acoustic.upsampling_ratios.push_back(r);
    k.frame_samples *= r;
  }
  if (!in) return false;
  *config = c;
  return true;
}

bool Probe(std::string_view model_root) {
  std::error_code code;
  const fs::path root(model_root);
  Config config;
  return fs::is_regular_file(root / "model.safetensors", code) && ReadShape(root, &config);
}

bool Resolve(std::string_view model_root, std::string* error) {
  const fs::path root(model_root);
  std::error_code code;
  for (const char* file : {"model.safetensors", "audio_tokenizer/model.safetensors"}) {
    if (!fs::is_regular_file(root / file, code)) {
      if (error != nullptr) *error = "OmniVoice model directory lacks " + std::string(file);
      return false;
    }
  }
  Config config;
  if (!ReadShape(root, &config)) {
    if (error != nullptr) *error = "OmniVoice model directory lacks b200_shape.txt";
    return false;
  }
  return true;
}

std::vector<std::vector<std::uint32_t>> ParseChunks(const std::string& text) {
  std::vector<std::vector<std::uint32_t>> chunks(1);
  std::string token;
  auto flush = [&] {
    if (!token.empty()) chunks.back().push_back(static_cast<std::uint32_t>(std::stoul(token)));
    token.clear();
  };
  for (const char ch : text) {
    if (ch == '|') {
      flush();
      chunks.emplace_back();
    } else if (ch == ' ') {
      flush();
    } else {
      token.push_back(ch);
    }
  }
  flush();
  return chunks;
}

class Runner final : public gufo::ext::TtsRunner {
 public:
  Runner(Config config, std::unique_ptr<Generator> generator, std::unique_ptr<Codec> codec)
      : config_(std::move(config)), generator_(std::move(generator)), codec_(std::move(codec)) {}

  bool Synthesize(const gufo::ext::SynthesisRequest& request,
                  const gufo::ext::CancellationCheck& is_cancelled,
                  gufo::ext::SynthesisResult* result, std::string* error) override {
    if (!request.reference_audio.samples.empty()) {
      if (error != nullptr) *error = "this runner takes no reference audio";
      return false;
    }
    const auto chunks = ParseChunks(request.text);
    const std::size_t frames = request.max_new_tokens > 0 ? request.max_new_tokens : 50;
    DecodingConfig decoding;
    if (!request.sampling.sample) decoding.position_temperature = 0.0F;
    // Chunk i's prompt: its own text, or (with chunk 0's voice carried)
    // chunk 0's text and codes in front of it (synthesizer.cpp:196-200).
    const auto build = [&](std::size_t i, const CarriedVoice* voice, ConditionalInput* input,
                           std::string*) {
      std::vector<std::uint32_t> text;
      std::vector<std::int32_t> codes;
      std::size_t ref_frames = 0;
      if (voice != nullptr) {
        text = chunks[voice->index];
        codes = voice->codes;
        ref_frames = voice->frames;
      }
      text.insert(text.end(), chunks[i].begin(), chunks[i].end());
      *input = ConditionalInput::Build(text, codes, ref_frames, frames, kCodebooks,
                                       config_.audio_mask_id);
      return true;
    };
    ChunkedSynthesis synthesis({generator_.get()}, {codec_.get()});
    std::vector<SynthesizedChunk> out;
    const auto cancelled = [&] { return is_cancelled && is_cancelled(); };
    if (!synthesis.Run(chunks.size(), build, false, decoding, request.sampling.seed, cancelled,
                       &out, error))
      return false;
    result->sample_rate = SampleRate();
    result->code_groups = static_cast<std::uint32_t>(kCodebooks);
    result->codes.clear();
    result->samples.clear();
    for (const SynthesizedChunk& c : out) {
      for (std::size_t f = 0; f < c.frames; ++f)
        for (std::size_t k = 0; k < kCodebooks; ++k) result->codes.push_back(c.codes[k * c.frames + f]);
      result->samples.insert(result->samples.end(), c.audio.begin(), c.audio.end());
    }
    result->sample_count = result->samples.size();
    return true;
  }

  std::vector<std::string> Voices() const override { return {"auto"}; }
  gufo::ext::TtsVariant Variant() const override { return gufo::ext::TtsVariant::kBase; }
  std::uint32_t SampleRate() const override { return config_.codec.sample_rate; }
  gufo::ext::TtsConditioningCapabilities Conditioning() const override {
    gufo::ext::TtsConditioningCapabilities c;
    c.unconditioned = true;
    c.default_voice = "auto";
    return c;
  }
  std::string ModelId() const override { return "omnivoice"; }

 private:
  Config config_;
  std::unique_ptr<Generator> generator_;
  std::unique_ptr<Codec> codec_;
};

std::unique_ptr<gufo::ext::TtsRunner> Create(const gufo::ext::TtsRunnerOptions& options,
                                             std::string* error) {
  Config config;
  if (!ReadShape(options.model_root, &config)) {
    if (error != nullptr) *error = "OmniVoice model directory lacks b200_shape.txt";
    return nullptr;
  }
  auto generator = Generator::Load(config, options.model_root, error);
  if (generator == nullptr) return nullptr;
  auto codec = Codec::Load(config, options.model_root, error);
  if (codec == nullptr) return nullptr;
  return std::make_unique<Runner>(config, std::move(generator), std::move(codec));
}

}  // namespace b200_runner

// provider.cpp:8-19's registration, with this library's runner.
void omnivoice_provider_register(gufo::ext::Registry& registry) {
  registry.AddProvider(gufo::ext::generated::extension_omnivoice::kProvider_omnivoice);
  registry.AddTtsProvider({
      .id = "omnivoice",
      .probe = &b200_runner::Probe,
      .resolve = &b200_runner::Resolve,
      .create = nullptr,
      .create_with_options = &b200_runner::Create,
  });
}

namespace {

int failures = 0;

void Require(bool ok, const std::string& what) {
  if (!ok) {
    std::printf("FAIL %s\n", what.c_str());
    ++failures;
  }
}

}  // namespace

int main(int argc, char** argv) {
  gufo::ext::Registry registry;
  omnivoice_provider_register(registry);
  Require(registry.providers.size() == 1 &&
              std::string(registry.providers[0].id) == "omnivoice",
          "provider registered");
  Require(registry.tts.size() == 1 && registry.tts[0].id == "omnivoice" &&
              registry.tts[0].create == nullptr && registry.tts[0].create_with_options != nullptr,
          "speech provider registered");
  Require(!registry.tts[0].probe("/nonexistent-model-root"), "probe of a missing directory");
  std::string error;
  Require(!registry.tts[0].resolve("/nonexistent-model-root", &error) &&
              error.rfind("OmniVoice model directory lacks ", 0) == 0,
          "resolve message: " + error);
  if (argc == 1) {
    if (failures == 0) std::printf("ok\n");
    return failures == 0 ? 0 : 1;
  }
  if (argc < 14) {
    std::printf("usage: %s [model_root out_dir vocab hidden intermediate layers heads kv_heads "
                "codebook_dim semantic latent decoder ratio...]\n", argv[0]);
    return 2;
  }
  const fs::path root = argv[1];
  const fs::path out = argv[2];
  {
    std::ofstream shape(root / "b200_shape.txt");
    for (int i = 3; i < 13; ++i) shape << argv[i] << ' ';
    shape << (argc - 13);
    for (int i = 13; i < argc; ++i) shape << ' ' << argv[i];
    shape << '\n';
  }
  Require(registry.tts[0].probe(root.string()), "probe of the model directory");
  Require(registry.tts[0].resolve(root.string(), &error), "resolve: " + error);
  auto runner = registry.tts[0].create_with_options({root}, &error);
  if (runner == nullptr) {
    std::printf("FAIL create: %s\n", error.c_str());
    return 1;
  }
  Require(runner->ModelId() == "omnivoice" && runner->SampleRate() == 24000, "runner identity");

  gufo::ext::SynthesisRequest request;
  request.text = "17 3 99 250 4|8 1200 77|5 6 7 8 9 10";
  request.max_new_tokens = 24;
  request.sampling.seed = 11;
  gufo::ext::SynthesisResult result;
  Require(runner->Synthesize(request, nullptr, &result, &error), "synthesize: " + error);

  // The reference's order: chunk by chunk, the voice carried from chunk 0.
  Config config;
  Require(b200_runner::ReadShape(root, &config), "shape");
  auto generator = Generator::Load(config, root, &error);
  auto codec = Codec::Load(config, root, &error);
  const auto chunks = b200_runner::ParseChunks(request.text);
  std::vector<std::int32_t> codes0, want_codes;
  std::vector<float> want_samples;
  for (std::size_t i = 0; i < chunks.size(); ++i) {
    std::vector<std::uint32_t> text;
    if (i > 0) text = chunks[0];
    text.insert(text.end(), chunks[i].begin(), chunks[i].end());
    const ConditionalInput input = ConditionalInput::Build(
        text, i > 0 ? codes0 : std::vector<std::int32_t>{}, i > 0 ? 24 : 0, 24, 8, 1024);
    GenerationResult g;
    Require(generator->Generate(input, DecodingConfig(), 11, nullptr, &g, &error),
            "reference-order generate: " + error);
    if (i == 0) codes0 = g.codes;
    for (std::size_t f = 0; f < 24; ++f)
      for (std::size_t k = 0; k < 8; ++k) want_codes.push_back(g.codes[k * 24 + f]);
    std::vector<float> piece;
    Require(codec->Decode(g.codes, 24, &piece, &error), "decode: " + error);
    want_samples.insert(want_samples.end(), piece.begin(), piece.end());
  }
  Require(result.codes.size() == want_codes.size() && result.samples.size() == want_samples.size(),
          "result sizes");
  std::size_t same = 0;
  for (std::size_t i = 0; i < want_codes.size() && i < result.codes.size(); ++i)
    same += result.codes[i] == want_codes[i];
  const double agreement = want_codes.empty() ? 0.0 : static_cast<double>(same) / want_codes.size();
  std::printf("codes equal to the chunk-by-chunk order: %.4f\n", agreement);
  Require(agreement >= 0.995, "code agreement");
  std::ofstream(out / "samples.f32", std::ios::binary)
      .write(reinterpret_cast<const char*>(result.samples.data()),
             static_cast<std::streamsize>(result.samples.size() * 4));
  std::ofstream(out / "codes.i32", std::ios::binary)
      .write(reinterpret_cast<const char*>(result.codes.data()),
             static_cast<std::streamsize>(result.codes.size() * 4));
  if (failures == 0) std::printf("ok\n");
  return failures == 0 ? 0 : 1;
}
