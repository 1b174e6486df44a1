// gufo::models::omnivoice::Generator on the B200 C-ABI.  Reference
// semantics (generator.cpp:364-543): Load reads model_root /
// "model.safetensors"; failures return false / nullptr with the
// reference's message prefixes, which the C-ABI already produces
// ("OmniVoice generator: ", "OmniVoice forward: ", "OmniVoice score: ",
// "OmniVoice generation: "); a cancelled generation reports "cancelled".
#include "generator.hpp"

#include <string>
#include <utility>

#include "ov_generator.h"

namespace gufo::models::omnivoice {
namespace {

void SetError(std::string* error, std::string message) {
  if (error != nullptr) *error = std::move(message);
}

std::string LastError() {
  char buffer[2048];
  ov_last_error(buffer, sizeof(buffer));
  return buffer;
}

ov_conditional_input View(const ConditionalInput& in) {
  ov_conditional_input v;
  v.codebooks = in.codebooks;
  v.length = in.length;
  v.audio_start = in.audio_start;
  v.target_frames = in.target_frames;
  v.ids = in.ids.data();
  return v;
}

ov_decoding_config View(const DecodingConfig& d) {
  ov_decoding_config v;
  v.steps = d.steps;
  v.guidance = d.guidance;
  v.t_shift = d.t_shift;
  v.layer_penalty = d.layer_penalty;
  v.position_temperature = d.position_temperature;
  return v;
}

int PollCancelled(void* user) {
  const auto* cancelled = static_cast<const std::function<bool()>*>(user);
  return (*cancelled && (*cancelled)()) ? 1 : 0;
}

bool InputShapeOk(const ConditionalInput& in, std::string* error, const char* prefix) {
  if (in.ids.size() != in.codebooks * in.length) {
    SetError(error, std::string(prefix) + "input ids do not match codebooks x length");
    return false;
  }
  return true;
}

}  // namespace

struct Generator::State {
  ov_generator* handle = nullptr;
  std::size_t codebooks = 0;
  std::size_t vocab = 0;
  ~State() {
    if (handle != nullptr) ov_generator_destroy(handle);
  }
};

Generator::Generator(std::unique_ptr<State> state) : state_(std::move(state)) {}
Generator::~Generator() = default;

std::unique_ptr<Generator> Generator::Load(const Config& config,
                                           const std::filesystem::path& model_root,
                                           std::string* error) {
  ov_model_config c;
  ov_default_model_config(&c);
  const BackboneConfig& b = config.backbone;
  c.vocab_size = b.vocab_size;
  c.hidden_size = b.hidden_size;
  c.intermediate_size = b.intermediate_size;
  c.layers = b.layers;
  c.heads = b.heads;
  c.kv_heads = b.kv_heads;
  c.head_dim = b.head_dim;
  if (b.max_positions != 0) c.max_positions = b.max_positions;
  c.rms_norm_eps = b.rms_norm_eps;
  c.rope_theta = b.rope_theta;
  c.audio_codebooks = config.audio_codebooks;
  c.audio_vocab_size = config.audio_vocab_size;
  c.audio_mask_id = config.audio_mask_id;
  int device = 0;
  if (ov_get_device(&device) != OV_OK) {
    SetError(error, "OmniVoice generator: " + LastError());
    return nullptr;
  }
  auto state = std::make_unique<State>();
  state->codebooks = c.audio_codebooks;
  state->vocab = c.audio_vocab_size;
  const std::string path = (model_root / "model.safetensors").string();
  if (ov_generator_load(&c, path.c_str(), device, &state->handle) != OV_OK) {
    SetError(error, LastError());
    return nullptr;
  }
  return std::unique_ptr<Generator>(new Generator(std::move(state)));
}

bool Generator::Generate(const ConditionalInput& input, const DecodingConfig& decoding,
                         std::uint64_t seed, const std::function<bool()>& cancelled,
                         GenerationResult* result, std::string* error) {
  if (!InputShapeOk(input, error, "OmniVoice generation: ")) return false;
  const ov_conditional_input in = View(input);
  const ov_decoding_config dec = View(decoding);
  GenerationResult out;
  out.codes.assign(input.codebooks * input.target_frames, 0);
  out.unmasked_at.assign(input.codebooks * input.target_frames, 0);
  const int status = ov_generator_generate(
      state_->handle, &in, &dec, seed, OV_GEN_NOISE_REFERENCE, cancelled ? PollCancelled : nullptr,
      const_cast<std::function<bool()>*>(&cancelled), out.codes.data(), out.unmasked_at.data());
  if (status != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  if (result != nullptr) *result = std::move(out);
  return true;
}

bool Generator::GenerateBatch(const std::vector<ConditionalInput>& inputs,
                              const DecodingConfig& decoding,
                              const std::vector<std::uint64_t>& seeds,
                              const std::function<bool()>& cancelled,
                              std::vector<GenerationResult>* results, std::string* error) {
  if (seeds.size() != inputs.size()) {
    SetError(error, "OmniVoice generation: one seed per input");
    return false;
  }
  std::vector<ov_conditional_input> views;
  std::vector<GenerationResult> out(inputs.size());
  std::vector<std::int32_t*> codes, unmasked;
  for (std::size_t i = 0; i < inputs.size(); ++i) {
    if (!InputShapeOk(inputs[i], error, "OmniVoice generation: ")) return false;
    views.push_back(View(inputs[i]));
    const std::size_t slots = inputs[i].codebooks * inputs[i].target_frames;
    out[i].codes.assign(slots, 0);
    out[i].unmasked_at.assign(slots, 0);
    codes.push_back(out[i].codes.data());
    unmasked.push_back(out[i].unmasked_at.data());
  }
  const ov_decoding_config dec = View(decoding);
  const int status = ov_generator_generate_batch(
      state_->handle, views.data(), views.size(), &dec, seeds.data(), OV_GEN_NOISE_REFERENCE,
      cancelled ? PollCancelled : nullptr, const_cast<std::function<bool()>*>(&cancelled),
      codes.data(), unmasked.data());
  if (status != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  if (results != nullptr) *results = std::move(out);
  return true;
}

bool Generator::Forward(const ConditionalInput& input, std::vector<float>* logits,
                        std::string* error) {
  if (!InputShapeOk(input, error, "OmniVoice forward: ")) return false;
  const ov_conditional_input in = View(input);
  std::vector<float> out(2 * input.target_frames * state_->codebooks * state_->vocab);
  if (ov_generator_forward(state_->handle, &in, out.data()) != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  if (logits != nullptr) *logits = std::move(out);
  return true;
}

bool Generator::Score(const ConditionalInput& input, float guidance,
                      std::vector<std::int32_t>* prediction, std::vector<float>* confidence,
                      std::string* error) {
  if (!InputShapeOk(input, error, "OmniVoice score: ")) return false;
  const ov_conditional_input in = View(input);
  std::vector<std::int32_t> pred(state_->codebooks * input.target_frames);
  std::vector<float> conf(pred.size());
  if (ov_generator_score(state_->handle, &in, guidance, pred.data(), conf.data()) != OV_OK) {
    SetError(error, LastError());
    return false;
  }
  if (prediction != nullptr) *prediction = std::move(pred);
  if (confidence != nullptr) *confidence = std::move(conf);
  return true;
}

}  // namespace gufo::models::omnivoice
