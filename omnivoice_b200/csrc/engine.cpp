// The generator engine (engine.hpp) and the ov_generator.h C-ABI.
//
// Per step, for a packed batch of R rows (generator.cpp:262-301 with the
// element-wise kernels fused into their producers):
//   embed+norm, 28 x { [norm], QKV GEMM (+QK-norm/RoPE), attention,
//   o GEMM (+residual), norm, gate/up GEMM (+SwiGLU), down GEMM (+residual) },
//   gather+final norm, head GEMM, score, select/scatter.
// The whole step is recorded once as a CUDA graph and replayed for every
// non-empty step; nothing returns to the host between steps (the reference
// synchronises and selects on the host each step, generator.cpp:517-535).
#include "engine.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <random>
#include <sstream>

#include "decoding.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "safetensors.hpp"
#include "synthetic.hpp"

namespace ovb {
namespace {

constexpr float kInitStd = 0.02f;

size_t RoundUp(size_t x, size_t m) { return (x + m - 1) / m * m; }

// Copies host arrays through one pinned staging area so the uploads are
// true asynchronous DMA transfers.
class Uploader {
 public:
  Uploader(uint8_t* staging, cudaStream_t stream) : staging_(staging), stream_(stream) {}
  template <typename T>
  void Add(T* dst, const T* src, size_t count) {
    if (count == 0) return;
    const size_t bytes = count * sizeof(T);
    std::memcpy(staging_ + offset_, src, bytes);
    Check(cudaMemcpyAsync(dst, staging_ + offset_, bytes, cudaMemcpyHostToDevice, stream_),
          "upload batch");
    offset_ += RoundUp(bytes, 256);
    total_ += bytes;
  }
  template <typename T>
  void Add(DeviceBuffer<T>& dst, const std::vector<T>& src) {
    Add(dst.get(), src.data(), src.size());
  }
  size_t total() const { return total_; }
  static size_t Need(size_t bytes) { return RoundUp(bytes, 256); }

 private:
  uint8_t* staging_;
  cudaStream_t stream_;
  size_t offset_ = 0;
  size_t total_ = 0;
};

}  // namespace

Engine::Engine(const ov_model_config& config, int device) : cfg_(config), device_(device) {
  Activate();
  CheckConfig();
  sms_ = SmCount();
  (void)DeviceErrorWord();
  ConfigureGemmKernels();
  ConfigureAttentionKernel();
  ConfigureSelectKernel();
  Check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  for (auto& e : step_done_)
    Check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  H_ = cfg_.hidden_size;
  I_ = cfg_.intermediate_size;
  D_ = cfg_.head_dim;
  QH_ = cfg_.heads * D_;
  QKVW_ = (cfg_.heads + 2 * cfg_.kv_heads) * D_;
  C_ = cfg_.audio_codebooks;
  V_ = cfg_.audio_vocab_size;
  CV_ = C_ * V_;
  ldl_ = RoundUp(CV_, 32);
  AllocateWeights();
}

Engine::~Engine() {
  cudaSetDevice(device_);
  DestroyGraph();
  for (auto& e : step_done_)
    if (e != nullptr) cudaEventDestroy(e);
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
  if (staging_ != nullptr) cudaFreeHost(staging_);
}

void Engine::Activate() const { Check(cudaSetDevice(device_), "cudaSetDevice"); }

// config.cpp:340-355 (IsSupported) plus the shapes these kernels implement.
void Engine::CheckConfig() const {
  const ov_model_config& c = cfg_;
  auto need = [](bool ok, const char* what) {
    if (!ok) throw Error(OV_ERR_UNSUPPORTED, std::string("unsupported model: ") + what);
  };
  need(c.head_dim == 128, "head_dim must be 128");
  need(c.heads > 0 && c.kv_heads > 0 && c.heads % c.kv_heads == 0, "heads / kv_heads");
  const size_t hv = c.hidden_size / 128;
  need(c.hidden_size % 128 == 0 && (hv == 1 || hv == 2 || hv == 4 || hv == 8 || hv == 16),
       "hidden_size must be 128, 256, 512, 1024 or 2048");
  need(c.intermediate_size % 128 == 0 && c.intermediate_size > 0, "intermediate_size % 128");
  need(c.layers > 0, "layers");
  need(c.audio_codebooks > 0 && c.audio_vocab_size > 0 && c.audio_vocab_size <= 1056,
       "audio vocab must be at most 1056");
  need(c.audio_mask_id < c.audio_vocab_size, "mask id");
  need(c.vocab_size > 0, "vocab");
  need(c.audio_codebooks * c.audio_vocab_size % 4 == 0, "codebooks * vocab must be a multiple of 4");
}

void Engine::AllocateWeights() {
  const size_t L = cfg_.layers;
  text_ = DeviceBuffer<float>(cfg_.vocab_size * H_);
  audio_emb_ = DeviceBuffer<float>(CV_ * H_);
  heads_ = DeviceBuffer<uint16_t>(CV_ * H_);
  final_norm_ = DeviceBuffer<float>(H_);
  qkv_w_ = DeviceBuffer<uint16_t>(L * QKVW_ * H_);
  o_w_ = DeviceBuffer<uint16_t>(L * H_ * QH_);
  gu_w_ = DeviceBuffer<uint16_t>(L * 2 * I_ * H_);
  down_w_ = DeviceBuffer<uint16_t>(L * H_ * I_);
  norms_ = DeviceBuffer<float>(L * (2 * H_ + 2 * D_));
}

float* Engine::LayerNorms(size_t layer) const { return norms_.get() + layer * (2 * H_ + 2 * D_); }

void Engine::LoadSynthetic(uint64_t seed) {
  Activate();
  const size_t KV = cfg_.kv_heads * D_;
  const size_t biggest = std::max({QH_ * H_, H_ * QH_, I_ * H_, H_ * I_, CV_ * H_});
  DeviceBuffer<float> tmp(biggest);
  cudaStream_t s = stream_;
  LaunchSyntheticFill(text_.get(), cfg_.vocab_size * H_, seed, kTextEmbeddings, kInitStd, s);
  LaunchSyntheticFill(audio_emb_.get(), CV_ * H_, seed, kAudioEmbeddings, kInitStd, s);
  LaunchSyntheticFill(tmp.get(), CV_ * H_, seed, kAudioHeads, kInitStd, s);
  LaunchToHalfRows(tmp.get(), heads_.get(), CV_, H_, 0, 0, s);
  LaunchFill(final_norm_.get(), H_, 1.0f, s);
  LaunchFill(norms_.get(), cfg_.layers * (2 * H_ + 2 * D_), 1.0f, s);
  for (size_t l = 0; l < cfg_.layers; ++l) {
    uint16_t* qkv = qkv_w_.get() + l * QKVW_ * H_;
    LaunchSyntheticFill(tmp.get(), QH_ * H_, seed, LayerTensor(l, kLayerQ), kInitStd, s);
    LaunchToHalfRows(tmp.get(), qkv, QH_, H_, 0, 0, s);
    LaunchSyntheticFill(tmp.get(), KV * H_, seed, LayerTensor(l, kLayerK), kInitStd, s);
    LaunchToHalfRows(tmp.get(), qkv + QH_ * H_, KV, H_, 0, 0, s);
    LaunchSyntheticFill(tmp.get(), KV * H_, seed, LayerTensor(l, kLayerV), kInitStd, s);
    LaunchToHalfRows(tmp.get(), qkv + (QH_ + KV) * H_, KV, H_, 0, 0, s);
    LaunchSyntheticFill(tmp.get(), H_ * QH_, seed, LayerTensor(l, kLayerO), kInitStd, s);
    LaunchToHalfRows(tmp.get(), o_w_.get() + l * H_ * QH_, H_, QH_, 0, 0, s);
    uint16_t* gu = gu_w_.get() + l * 2 * I_ * H_;
    LaunchSyntheticFill(tmp.get(), I_ * H_, seed, LayerTensor(l, kLayerGate), kInitStd, s);
    LaunchToHalfRows(tmp.get(), gu, I_, H_, OV_SWIGLU_GROUP, 0, s);
    LaunchSyntheticFill(tmp.get(), I_ * H_, seed, LayerTensor(l, kLayerUp), kInitStd, s);
    LaunchToHalfRows(tmp.get(), gu, I_, H_, OV_SWIGLU_GROUP, OV_SWIGLU_GROUP, s);
    LaunchSyntheticFill(tmp.get(), H_ * I_, seed, LayerTensor(l, kLayerDown), kInitStd, s);
    LaunchToHalfRows(tmp.get(), down_w_.get() + l * H_ * I_, H_, I_, 0, 0, s);
  }
  Check(cudaStreamSynchronize(s), "synthetic weights");
  loaded_ = true;
}

// generator.cpp:364-434 (Load): the reference's tensor names and shapes.
void Engine::LoadSafetensors(const std::string& path) {
  Activate();
  SafetensorsFile file(path);
  const size_t KV = cfg_.kv_heads * D_;
  const size_t biggest = std::max({QH_ * H_, H_ * QH_, I_ * H_, H_ * I_, CV_ * H_});
  DeviceBuffer<float> tmp(biggest);
  cudaStream_t s = stream_;
  auto copy = [&](float* dst, const float* src, size_t count) {
    Check(cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyHostToDevice, s),
          "upload weights");
    Check(cudaStreamSynchronize(s), "upload weights");
  };
  auto half = [&](const std::string& name, size_t rows, size_t cols, uint16_t* dst, int group,
                  int offset) {
    copy(tmp.get(), file.ExpectF32(name, {rows, cols}), rows * cols);
    LaunchToHalfRows(tmp.get(), dst, static_cast<int64_t>(rows), static_cast<int64_t>(cols),
                     group, offset, s);
  };
  copy(text_.get(), file.ExpectF32("llm.embed_tokens.weight", {cfg_.vocab_size, H_}),
       cfg_.vocab_size * H_);
  copy(audio_emb_.get(), file.ExpectF32("audio_embeddings.weight", {CV_, H_}), CV_ * H_);
  half("audio_heads.weight", CV_, H_, heads_.get(), 0, 0);
  copy(final_norm_.get(), file.ExpectF32("llm.norm.weight", {H_}), H_);
  for (size_t l = 0; l < cfg_.layers; ++l) {
    const std::string p = "llm.layers." + std::to_string(l) + ".";
    uint16_t* qkv = qkv_w_.get() + l * QKVW_ * H_;
    half(p + "self_attn.q_proj.weight", QH_, H_, qkv, 0, 0);
    half(p + "self_attn.k_proj.weight", KV, H_, qkv + QH_ * H_, 0, 0);
    half(p + "self_attn.v_proj.weight", KV, H_, qkv + (QH_ + KV) * H_, 0, 0);
    half(p + "self_attn.o_proj.weight", H_, QH_, o_w_.get() + l * H_ * QH_, 0, 0);
    uint16_t* gu = gu_w_.get() + l * 2 * I_ * H_;
    half(p + "mlp.gate_proj.weight", I_, H_, gu, OV_SWIGLU_GROUP, 0);
    half(p + "mlp.up_proj.weight", I_, H_, gu, OV_SWIGLU_GROUP, OV_SWIGLU_GROUP);
    half(p + "mlp.down_proj.weight", H_, I_, down_w_.get() + l * H_ * I_, 0, 0);
    float* n = LayerNorms(l);
    copy(n, file.ExpectF32(p + "input_layernorm.weight", {H_}), H_);
    copy(n + H_, file.ExpectF32(p + "post_attention_layernorm.weight", {H_}), H_);
    copy(n + 2 * H_, file.ExpectF32(p + "self_attn.q_norm.weight", {D_}), D_);
    copy(n + 2 * H_ + D_, file.ExpectF32(p + "self_attn.k_norm.weight", {D_}), D_);
  }
  Check(cudaStreamSynchronize(s), "weights");
  loaded_ = true;
}

void Engine::EnsureRope(size_t positions) {
  if (positions <= rope_positions_) return;
  const size_t n = std::max<size_t>(RoundUp(positions, 1024), 4096);
  std::vector<float> cs(n * D_ / 2), sn(n * D_ / 2);
  CheckStatus(ov_rope_tables(cfg_.rope_theta, D_, n, cs.data(), sn.data()));
  rope_cos_ = DeviceBuffer<float>(cs.size());
  rope_sin_ = DeviceBuffer<float>(sn.size());
  Check(cudaMemcpy(rope_cos_.get(), cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope");
  Check(cudaMemcpy(rope_sin_.get(), sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope");
  rope_positions_ = n;
  signature_.clear();  // plans hold the table pointers
}

void Engine::Prepare(const ov_conditional_input* inputs, size_t count,
                     const ov_decoding_config* decoding, const uint64_t* seeds, int noise_mode) {
  Activate();
  if (!loaded_) throw Error(OV_ERR_INVALID, "weights are not loaded");
  OV_REQUIRE(count > 0 && inputs != nullptr, "no inputs");
  OV_REQUIRE(decoding == nullptr || decoding->steps > 0, "decoding steps must be positive");
  const size_t n = count;
  utts_.assign(n, UttDesc{});
  frames_.assign(n, 0);
  R_ = 0;
  total_frames_ = 0;
  max_seqlen_ = 0;
  max_slots_ = 0;
  std::ostringstream sig;
  sig << n << ':';
  for (size_t u = 0; u < n; ++u) {
    const ov_conditional_input& in = inputs[u];
    OV_REQUIRE(in.codebooks == C_, "input codebooks do not match the model");
    OV_REQUIRE(in.length > 0 && in.target_frames > 0 && in.target_frames <= in.length,
               "target frames must be in [1, length]");
    OV_REQUIRE(in.audio_start <= in.length - in.target_frames,
               "text tokens must precede the target frames");
    OV_REQUIRE(in.ids != nullptr, "input ids missing");
    UttDesc& d = utts_[u];
    d.row_base = static_cast<int32_t>(R_);
    d.length = static_cast<int32_t>(in.length);
    d.frames = static_cast<int32_t>(in.target_frames);
    d.audio_start = static_cast<int32_t>(in.audio_start);
    d.frame_base = static_cast<int32_t>(total_frames_);
    d.logit_row = static_cast<int32_t>(2 * total_frames_);
    d.slot_base = static_cast<int32_t>(C_ * total_frames_);
    d.gumbel_stride = static_cast<int32_t>(C_ * in.target_frames);
    frames_[u] = in.target_frames;
    R_ += in.length + in.target_frames;
    total_frames_ += in.target_frames;
    max_seqlen_ = std::max(max_seqlen_, in.length);
    max_slots_ = std::max(max_slots_, C_ * in.target_frames);
    sig << in.length << ',' << in.target_frames << ';';
  }
  OV_REQUIRE(R_ < (1u << 30), "batch too large");
  n_seqs_ = 2 * n;
  // Host images of the per-row arrays (generator.cpp:218-258).
  std::vector<int32_t> positions(R_), row_text(R_, -1), ids(C_ * R_), cu(n_seqs_ + 1);
  std::vector<int32_t> targets(2 * total_frames_), frame_utt(total_frames_);
  for (size_t u = 0; u < n; ++u) {
    const ov_conditional_input& in = inputs[u];
    const UttDesc& d = utts_[u];
    const size_t L = in.length, F = in.target_frames, base = static_cast<size_t>(d.row_base);
    for (size_t t = 0; t < in.audio_start; ++t) {
      const int32_t id = in.ids[t];
      if (id < 0 || static_cast<size_t>(id) >= cfg_.vocab_size)
        throw Error(OV_ERR_INVALID, "text token outside the vocabulary");
      row_text[base + t] = id;
    }
    for (size_t c = 0; c < C_; ++c)
      for (size_t t = in.audio_start; t < L; ++t) {
        const int32_t id = in.ids[c * L + t];
        if (id < 0 || static_cast<size_t>(id) >= V_)
          throw Error(OV_ERR_INVALID, "audio code outside the codebook");
      }
    for (size_t r = 0; r < L; ++r) positions[base + r] = static_cast<int32_t>(r);
    for (size_t f = 0; f < F; ++f) positions[base + L + f] = static_cast<int32_t>(f);
    for (size_t c = 0; c < C_; ++c) {
      std::copy(in.ids + c * L, in.ids + (c + 1) * L, &ids[c * R_ + base]);
      std::copy(in.ids + c * L + L - F, in.ids + (c + 1) * L, &ids[c * R_ + base + L]);
    }
    cu[2 * u] = static_cast<int32_t>(base);
    cu[2 * u + 1] = static_cast<int32_t>(base + L);
    for (size_t f = 0; f < F; ++f) {
      targets[d.logit_row + f] = static_cast<int32_t>(base + L - F + f);
      targets[d.logit_row + F + f] = static_cast<int32_t>(base + L + f);
      frame_utt[d.frame_base + f] = static_cast<int32_t>(u);
    }
  }
  cu[n_seqs_] = static_cast<int32_t>(R_);
  EnsureRope(max_seqlen_);
  // Attention work list: every (sequence, pair of 128-query tiles), longest
  // sequences first so that the long CTAs start in the first wave.
  std::vector<int32_t> seq_order(n_seqs_);
  for (size_t q = 0; q < n_seqs_; ++q) seq_order[q] = static_cast<int32_t>(q);
  std::stable_sort(seq_order.begin(), seq_order.end(), [&](int32_t a, int32_t b) {
    return cu[a + 1] - cu[a] > cu[b + 1] - cu[b];
  });
  // A CTA takes two 128-query tiles that share each K/V tile (two softmax
  // groups ping-ponging on the tensor core); batches short enough that one
  // tile per CTA still fits in one wave take single tiles (twice the CTAs,
  // each tile's softmax split over four warpgroups).
  size_t pairs = 0, singles = 0;
  for (size_t q = 0; q < n_seqs_; ++q) {
    const size_t len = static_cast<size_t>(cu[q + 1] - cu[q]);
    pairs += (len + 255) / 256;
    singles += (len + 127) / 128;
  }
  single_tiles_ = pairs * cfg_.heads < static_cast<size_t>(sms_) &&
                  singles * cfg_.heads <= static_cast<size_t>(sms_);
  const bool single_tiles = single_tiles_;
  const int32_t per_item = single_tiles ? 1 : 2;
  std::vector<int32_t> items;
  for (const int32_t q : seq_order) {
    const int32_t len = cu[q + 1] - cu[q];
    for (int32_t tile = 0; tile * 128 < len; tile += per_item) {
      items.push_back(q);
      items.push_back(tile | (per_item << 24));
    }
  }
  n_items_ = items.size() / 2;

  // Decoding state: per-utterance schedules, the union of non-empty steps,
  // and for the reference noise the host mt19937_64 stream of each seed.
  decode_ready_ = decoding != nullptr;
  std::vector<int32_t> counts;
  std::vector<float> gumbel;
  step_list_.clear();
  size_t gumbel_floats = 0;
  if (decode_ready_) {
    const size_t steps = decoding->steps;
    guidance_ = decoding->guidance;
    layer_penalty_ = decoding->layer_penalty;
    temperature_ = decoding->position_temperature;
    noise_ = temperature_ <= 0.0f ? OV_NOISE_NONE
             : noise_mode == OV_GEN_NOISE_DEVICE ? OV_NOISE_DEVICE
                                                 : OV_NOISE_BUFFER;
    counts.assign(n * steps, 0);
    std::vector<char> any(steps, 0);
    for (size_t u = 0; u < n; ++u) {
      const std::vector<size_t> s =
          gufo::models::omnivoice::UnmaskSchedule(C_ * frames_[u], steps, decoding->t_shift);
      for (size_t i = 0; i < steps; ++i) {
        counts[u * steps + i] = static_cast<int32_t>(s[i]);
        if (s[i] > 0) any[i] = 1;
      }
    }
    for (size_t i = 0; i < steps; ++i)
      if (any[i]) step_list_.push_back(static_cast<int32_t>(i));
    if (noise_ == OV_NOISE_BUFFER) {
      for (size_t u = 0; u < n; ++u) gumbel_floats += steps * C_ * frames_[u];
      gumbel.assign(gumbel_floats, 0.0f);
      size_t offset = 0;
      for (size_t u = 0; u < n; ++u) {
        const size_t slots = C_ * frames_[u];
        std::mt19937_64 random(seeds != nullptr ? seeds[u] : 0);
        for (size_t i = 0; i < steps; ++i)
          if (counts[u * steps + i] > 0)
            gufo::models::omnivoice::DrawGumbel(&random, slots, &gumbel[offset + i * slots]);
        offset += steps * slots;
      }
    }
    sig << "d" << steps << ',' << noise_ << ',' << guidance_ << ',' << layer_penalty_ << ','
        << temperature_;
  }

  // Buffers (grow-only); any reallocation invalidates plans and the graph.
  bool moved = false;
  moved |= ids_.Reserve(C_ * R_);
  moved |= ids_init_.Reserve(C_ * R_);
  moved |= positions_.Reserve(R_);
  moved |= row_text_.Reserve(R_);
  moved |= cu_seqlens_.Reserve(n_seqs_ + 1);
  moved |= attn_items_.Reserve(std::max<size_t>(items.size(), 2));
  moved |= targets_.Reserve(2 * total_frames_);
  moved |= frame_utt_.Reserve(total_frames_);
  moved |= utts_d_.Reserve(n);
  moved |= launch_.Reserve(n);
  moved |= counts_.Reserve(std::max<size_t>(counts.size(), 1));
  moved |= step_list_d_.Reserve(std::max<size_t>(step_list_.size(), 1));
  moved |= gumbel_.Reserve(std::max<size_t>(gumbel_floats, 1));
  moved |= hidden_.Reserve(R_ * H_);
  moved |= normed_.Reserve(R_ * H_);
  moved |= qkv_.Reserve(R_ * QKVW_);
  moved |= attn_.Reserve(R_ * QH_);
  moved |= act_.Reserve(R_ * I_);
  moved |= final_.Reserve(2 * total_frames_ * H_);
  moved |= logits_.Reserve(2 * total_frames_ * ldl_);
  moved |= pred_.Reserve(C_ * total_frames_);
  moved |= conf_.Reserve(C_ * total_frames_);
  moved |= codes_.Reserve(C_ * total_frames_);
  moved |= unmasked_.Reserve(C_ * total_frames_);
  const size_t ws = std::max(
      GemmWorkspaceBytes(static_cast<int>(R_), static_cast<int>(H_), static_cast<int>(QH_),
                         OV_EPI_ACCUM_F32, sms_),
      GemmWorkspaceBytes(static_cast<int>(R_), static_cast<int>(H_), static_cast<int>(I_),
                         OV_EPI_ACCUM_F32, sms_));
  if (gemm_ws_.Reserve(std::max<size_t>(ws, 256))) {
    moved = true;
    Check(cudaMemset(gemm_ws_.get(), 0, gemm_ws_.size()), "clear GEMM workspace");
  }
  gemm_ws_bytes_ = ws;

  // Device pointers inside the descriptors.
  size_t goff = 0;
  for (size_t u = 0; u < n; ++u) {
    UttDesc& d = utts_[u];
    d.noise_seed = seeds != nullptr ? seeds[u] : 0;
    d.counts = decode_ready_ ? counts_.get() + u * decoding->steps : nullptr;
    d.gumbel = noise_ == OV_NOISE_BUFFER && decode_ready_ ? gumbel_.get() + goff : nullptr;
    if (decode_ready_) goff += decoding->steps * C_ * frames_[u];
  }
  cudaStream_t s = stream_;
  const size_t need =
      Uploader::Need(positions.size() * 4) + Uploader::Need(row_text.size() * 4) +
      Uploader::Need(ids.size() * 4) + Uploader::Need(cu.size() * 4) +
      Uploader::Need(targets.size() * 4) + Uploader::Need(frame_utt.size() * 4) +
      Uploader::Need(n * sizeof(UttDesc)) + Uploader::Need(counts.size() * 4) +
      Uploader::Need(step_list_.size() * 4) + Uploader::Need(gumbel.size() * 4) +
      Uploader::Need(items.size() * 4);
  if (need > staging_bytes_) {
    if (staging_ != nullptr) Check(cudaFreeHost(staging_), "free staging");
    staging_ = nullptr;
    staging_bytes_ = 0;
    void* p = nullptr;
    Check(cudaMallocHost(&p, need), "allocate pinned staging");
    staging_ = static_cast<uint8_t*>(p);
    staging_bytes_ = need;
  }
  Uploader up(staging_, s);
  up.Add(positions_, positions);
  up.Add(row_text_, row_text);
  up.Add(ids_init_, ids);
  up.Add(cu_seqlens_, cu);
  up.Add(attn_items_, items);
  up.Add(targets_, targets);
  up.Add(frame_utt_, frame_utt);
  up.Add(utts_d_.get(), utts_.data(), n);
  up.Add(counts_, counts);
  up.Add(step_list_d_, step_list_);
  up.Add(gumbel_, gumbel);
  h2d_bytes_ = up.total();
  EnqueueReset(s);
  // The host vectors above go out of scope: wait for the copies.
  Check(cudaStreamSynchronize(s), "upload batch");

  const std::string signature = sig.str() + "|" + std::to_string(rope_positions_);
  if (moved || signature != signature_) {
    DestroyGraph();
    BuildPlans();
    signature_ = signature;
  }
}

void Engine::BuildPlans() {
  const int R = static_cast<int>(R_);
  const int L = static_cast<int>(cfg_.layers);
  plans_.assign(cfg_.layers, LayerPlans{});
  for (int l = 0; l < L; ++l) {
    ov_epilogue_args ea{};
    ea.q_norm = LayerNorms(l) + 2 * H_;
    ea.k_norm = LayerNorms(l) + 2 * H_ + D_;
    ea.positions = positions_.get();
    ea.rope_cos = rope_cos_.get();
    ea.rope_sin = rope_sin_.get();
    ea.max_positions = static_cast<int32_t>(rope_positions_);
    ea.heads = static_cast<int32_t>(cfg_.heads);
    ea.kv_heads = static_cast<int32_t>(cfg_.kv_heads);
    ea.head_dim = static_cast<int32_t>(D_);
    ea.epsilon = cfg_.rms_norm_eps;
    LayerPlans& p = plans_[l];
    PlanGemm(&p.qkv, normed_.get(), H_, qkv_w_.get(), L * QKVW_, l * QKVW_, qkv_.get(), QKVW_, R,
             QKVW_, H_, OV_EPI_QKNORM_ROPE_F16, &ea, nullptr, 0, sms_);
    PlanGemm(&p.o, attn_.get(), QH_, o_w_.get(), L * H_, l * H_, hidden_.get(), H_, R, H_, QH_,
             OV_EPI_ACCUM_F32, nullptr, gemm_ws_.get(), gemm_ws_bytes_, sms_);
    PlanGemm(&p.gate_up, normed_.get(), H_, gu_w_.get(), L * 2 * I_, l * 2 * I_, act_.get(), I_,
             R, 2 * I_, H_, OV_EPI_SWIGLU_F16, nullptr, nullptr, 0, sms_);
    PlanGemm(&p.down, act_.get(), I_, down_w_.get(), L * H_, l * H_, hidden_.get(), H_, R, H_, I_,
             OV_EPI_ACCUM_F32, nullptr, gemm_ws_.get(), gemm_ws_bytes_, sms_);
  }
  PlanGemm(&head_plan_, final_.get(), H_, heads_.get(), CV_, 0, logits_.get(), ldl_,
           static_cast<int>(2 * total_frames_), CV_, H_, OV_EPI_STORE_F32, nullptr, nullptr, 0,
           sms_);
  EncodeQkvMap(&qkv_map_, qkv_.get(), QKVW_, R_, QKVW_);
  EncodeAttnOutMap(&attn_out_map_, attn_.get(), QH_, R_, QH_);
}

void Engine::EnqueueForward(cudaStream_t s, Marker* m) {
  const float eps = cfg_.rms_norm_eps;
  const float scale = 1.0f / std::sqrt(static_cast<float>(D_));
  const double R = static_cast<double>(R_);
  const double H = static_cast<double>(H_);
  const double F2 = 2.0 * static_cast<double>(total_frames_);
  double attn_flops = 0.0;
  for (const UttDesc& d : utts_)
    attn_flops += 4.0 * static_cast<double>(D_) * cfg_.heads *
                  (static_cast<double>(d.length) * d.length + static_cast<double>(d.frames) * d.frames);
  double text_rows = 0.0;
  for (const UttDesc& d : utts_) text_rows += d.audio_start;
  auto mark = [&](int kind, double flops, double bytes) {
    if (m != nullptr) m->Mark(kind, flops, bytes);
  };
  size_t launches = 0;
  // Embed: gathered rows read, hidden written (fp32) and normed (fp16).
  mark(kEmbedNorm, 0.0,
       (text_rows + (R - text_rows) * C_) * H * 4 + R * H * 4 + R * H * 2 + C_ * R * 4);
  LaunchEmbed(text_.get(), cfg_.vocab_size, row_text_.get(), audio_emb_.get(), V_, ids_.get(), C_,
              R_, H_, hidden_.get(), LayerNorms(0), eps, normed_.get(), s);
  ++launches;
  const double norm_bytes = R * H * (4 + 2);
  for (size_t l = 0; l < cfg_.layers; ++l) {
    const LayerPlans& p = plans_[l];
    if (l > 0) {
      mark(kRmsNorm, 0.0, norm_bytes);
      LaunchRmsNorm(hidden_.get(), nullptr, R_, LayerNorms(l), normed_.get(), H_, eps, s);
      ++launches;
    }
    mark(kGemmQkv, 2.0 * R * H * QKVW_, 0.0);
    LaunchGemm(p.qkv, s);
    mark(kAttention, attn_flops, 0.0);
    LaunchAttention(qkv_map_, attn_out_map_, cu_seqlens_.get(), static_cast<int>(n_seqs_),
                    static_cast<int>(max_seqlen_), attn_items_.get(),
                    static_cast<int>(n_items_), static_cast<int>(cfg_.heads),
                    static_cast<int>(cfg_.kv_heads), scale,
                    reinterpret_cast<__half*>(attn_.get()), static_cast<int64_t>(QH_), s,
                    single_tiles_);
    mark(kGemmO, 2.0 * R * QH_ * H, 0.0);
    LaunchGemm(p.o, s);
    mark(kRmsNorm, 0.0, norm_bytes);
    LaunchRmsNorm(hidden_.get(), nullptr, R_, LayerNorms(l) + H_, normed_.get(), H_, eps, s);
    mark(kGemmGateUp, 2.0 * R * H * 2 * I_, 0.0);
    LaunchGemm(p.gate_up, s);
    mark(kGemmDown, 2.0 * R * I_ * H, 0.0);
    LaunchGemm(p.down, s);
    launches += 6;
  }
  mark(kGatherNorm, 0.0, F2 * H * (4 + 2) + F2 * 4);
  LaunchRmsNorm(hidden_.get(), targets_.get(), 2 * total_frames_, final_norm_.get(),
                final_.get(), H_, eps, s);
  mark(kGemmHead, 2.0 * F2 * H * CV_, 0.0);
  LaunchGemm(head_plan_, s);
  launches += 2;
  kernels_per_step_ = launches;
}

void Engine::EnqueueDecode(cudaStream_t s, Marker* m) {
  const double slots = static_cast<double>(C_ * total_frames_);
  if (m != nullptr) m->Mark(kScore, 0.0, 2.0 * total_frames_ * CV_ * 4 + slots * 8);
  LaunchScore(logits_.get(), static_cast<int64_t>(ldl_), static_cast<int>(total_frames_),
              static_cast<int>(C_), static_cast<int>(V_), cfg_.audio_mask_id, guidance_,
              utts_d_.get(), frame_utt_.get(), 0, pred_.get(), conf_.get(), s);
  StepControl ctl{step_list_d_.get(), launch_.get()};
  if (m != nullptr) m->Mark(kSelect, 0.0, slots * (4 + 4 + 4 + 4));
  LaunchSelect(pred_.get(), conf_.get(), static_cast<int>(C_), layer_penalty_, temperature_,
               noise_, cfg_.audio_mask_id, codes_.get(), unmasked_.get(), ids_.get(),
               static_cast<int64_t>(R_), UttDesc{}, utts_d_.get(), static_cast<int>(utts_.size()),
               ctl, static_cast<int>(max_slots_), 0, 0, 0, 0, s);
  kernels_per_step_ += 2;
}

namespace {

// Records a CUDA event before every kernel of a captured step.
struct EventMarker : Engine::Marker {
  explicit EventMarker(cudaStream_t s) : stream(s) {}
  ~EventMarker() override {
    for (cudaEvent_t e : events) cudaEventDestroy(e);
  }
  void Mark(int kind, double f, double b) override {
    cudaEvent_t e = nullptr;
    Check(cudaEventCreate(&e), "cudaEventCreate");
    events.push_back(e);
    // External: a timed event-record node in the captured graph.
    Check(cudaEventRecordWithFlags(e, stream, cudaEventRecordExternal), "cudaEventRecord");
    kinds.push_back(kind);
    flops.push_back(f);
    bytes.push_back(b);
  }
  cudaStream_t stream;
  std::vector<cudaEvent_t> events;
  std::vector<int> kinds;
  std::vector<double> flops, bytes;
};

const char* KindName(int kind) {
  static const char* names[] = {"embed_norm",      "rmsnorm",      "gemm_qkv_qknorm_rope",
                                "attention",       "gemm_o_residual", "gemm_gate_up_swiglu",
                                "gemm_down_residual", "gather_norm", "gemm_audio_head",
                                "score",           "select"};
  return names[kind];
}

}  // namespace

std::vector<ov_kernel_time> Engine::Profile() {
  Activate();
  OV_REQUIRE(!plans_.empty(), "no prepared batch");
  cudaStream_t s = stream_;
  EnqueueReset(s);
  Check(cudaStreamSynchronize(s), "profile");
  EventMarker marker(s);
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  Check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    const PdlScope no_pdl(false);  // event nodes sit between the kernels
    EnqueueForward(s, &marker);
    if (decode_ready_) EnqueueDecode(s, &marker);
    marker.Mark(-1, 0.0, 0.0);
  } catch (...) {
    (void)cudaStreamEndCapture(s, &graph);
    if (graph != nullptr) cudaGraphDestroy(graph);
    throw;
  }
  Check(cudaStreamEndCapture(s, &graph), "end capture");
  Check(cudaGraphInstantiate(&exec, graph, 0), "instantiate profile graph");
  Check(cudaGraphLaunch(exec, s), "launch profile graph");
  Check(cudaStreamSynchronize(s), "profile");
  std::vector<ov_kernel_time> out(kKinds);
  for (int k = 0; k < kKinds; ++k) {
    std::memset(&out[k], 0, sizeof(ov_kernel_time));
    std::strncpy(out[k].name, KindName(k), sizeof(out[k].name) - 1);
  }
  for (size_t i = 0; i + 1 < marker.events.size(); ++i) {
    float ms = 0.0f;
    Check(cudaEventElapsedTime(&ms, marker.events[i], marker.events[i + 1]), "event time");
    ov_kernel_time& t = out[marker.kinds[i]];
    t.ms += ms;
    t.launches += 1;
    t.flops += marker.flops[i];
    t.bytes += marker.bytes[i];
  }
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  EnqueueReset(s);
  Check(cudaStreamSynchronize(s), "profile");
  return out;
}

// generator.cpp:496-499: codes start as the mask, unmasked_at as -1, and
// the ids are the caller's conditional input.
void Engine::EnqueueReset(cudaStream_t s) {
  Check(cudaMemcpyAsync(ids_.get(), ids_init_.get(), C_ * R_ * sizeof(int32_t),
                        cudaMemcpyDeviceToDevice, s),
        "reset ids");
  LaunchFillInt(codes_.get(), C_ * total_frames_, static_cast<int32_t>(cfg_.audio_mask_id), s);
  LaunchFillInt(unmasked_.get(), C_ * total_frames_, -1, s);
  Check(cudaMemsetAsync(launch_.get(), 0, utts_.size() * sizeof(int32_t), s), "reset steps");
}

void Engine::CaptureGraph() {
  DestroyGraph();
  Check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    const PdlScope pdl(true);
    EnqueueForward(stream_);
    EnqueueDecode(stream_);
  } catch (...) {
    cudaGraph_t g = nullptr;
    (void)cudaStreamEndCapture(stream_, &g);
    if (g != nullptr) cudaGraphDestroy(g);
    throw;
  }
  Check(cudaStreamEndCapture(stream_, &graph_), "end capture");
  Check(cudaGraphInstantiate(&graph_exec_, graph_, 0), "instantiate step graph");
}

void Engine::DestroyGraph() {
  if (graph_exec_ != nullptr) cudaGraphExecDestroy(graph_exec_);
  if (graph_ != nullptr) cudaGraphDestroy(graph_);
  graph_exec_ = nullptr;
  graph_ = nullptr;
}

void Engine::Run(ov_cancel_fn cancelled, void* user) {
  Activate();
  OV_REQUIRE(decode_ready_, "batch was prepared without decoding settings");
  if (graph_exec_ == nullptr) CaptureGraph();
  EnqueueReset(stream_);
  const size_t n = step_list_.size();
  for (size_t k = 0; k < n; ++k) {
    if (cancelled != nullptr) {
      // Poll before every step (generator.cpp:508-511) with at most two
      // steps queued ahead of it.
      if (k >= 2) Check(cudaEventSynchronize(step_done_[k % 2]), "step");
      if (cancelled(user) != 0) {
        Check(cudaStreamSynchronize(stream_), "cancel");
        throw Error(OV_ERR_CANCELLED, "cancelled");
      }
    }
    Check(cudaGraphLaunch(graph_exec_, stream_), "launch step graph");
    if (cancelled != nullptr) Check(cudaEventRecord(step_done_[k % 2], stream_), "record step");
  }
}

void Engine::Fetch(int32_t** codes, int32_t** unmasked_at) {
  Activate();
  d2h_bytes_ = 0;
  for (size_t u = 0; u < utts_.size(); ++u) {
    const size_t off = static_cast<size_t>(utts_[u].slot_base);
    const size_t bytes = C_ * frames_[u] * sizeof(int32_t);
    if (codes != nullptr && codes[u] != nullptr) {
      Check(cudaMemcpyAsync(codes[u], codes_.get() + off, bytes, cudaMemcpyDeviceToHost, stream_),
            "download codes");
      d2h_bytes_ += bytes;
    }
    if (unmasked_at != nullptr && unmasked_at[u] != nullptr) {
      Check(cudaMemcpyAsync(unmasked_at[u], unmasked_.get() + off, bytes, cudaMemcpyDeviceToHost,
                            stream_),
            "download unmasked_at");
      d2h_bytes_ += bytes;
    }
  }
  Check(cudaStreamSynchronize(stream_), "generation");
  uint32_t flags = 0;
  CheckStatus(ov_take_device_errors(&flags, stream_));
  if (flags & kErrWaitTimeout) throw Error(OV_ERR_TIMEOUT, "a device-side wait timed out");
  if (flags & kErrBadArgument) throw Error(OV_ERR_INVALID, "a kernel rejected an argument");
}

void Engine::ForwardOnce(float* logits, float guidance, int32_t* prediction, float* confidence) {
  Activate();
  EnqueueReset(stream_);
  {
    const PdlScope pdl(true);
    EnqueueForward(stream_);
  }
  const size_t F = frames_[0];
  if (prediction != nullptr) {
    LaunchScore(logits_.get(), static_cast<int64_t>(ldl_), static_cast<int>(total_frames_),
                static_cast<int>(C_), static_cast<int>(V_), cfg_.audio_mask_id, guidance,
                utts_d_.get(), frame_utt_.get(), 0, pred_.get(), conf_.get(), stream_);
    Check(cudaMemcpyAsync(prediction, pred_.get(), C_ * F * sizeof(int32_t),
                          cudaMemcpyDeviceToHost, stream_),
          "download predictions");
    Check(cudaMemcpyAsync(confidence, conf_.get(), C_ * F * sizeof(float), cudaMemcpyDeviceToHost,
                          stream_),
          "download confidences");
  }
  if (logits != nullptr)
    Check(cudaMemcpy2DAsync(logits, CV_ * sizeof(float), logits_.get(), ldl_ * sizeof(float),
                            CV_ * sizeof(float), 2 * F, cudaMemcpyDeviceToHost, stream_),
          "download logits");
  Check(cudaStreamSynchronize(stream_), "forward");
  uint32_t flags = 0;
  CheckStatus(ov_take_device_errors(&flags, stream_));
  if (flags & kErrWaitTimeout) throw Error(OV_ERR_TIMEOUT, "a device-side wait timed out");
  if (flags & kErrBadArgument) throw Error(OV_ERR_INVALID, "a kernel rejected an argument");
}

void Engine::Stats(ov_generator_stats* st) const {
  st->rows = R_;
  st->steps_run = step_list_.size();
  double sum_sq = 0.0;
  for (const UttDesc& d : utts_)
    sum_sq += static_cast<double>(d.length) * d.length + static_cast<double>(d.frames) * d.frames;
  const double linear = 2.0 * cfg_.layers *
                        static_cast<double>(H_ * QKVW_ + QH_ * H_ + H_ * 2 * I_ + I_ * H_);
  st->flops_per_step = static_cast<double>(R_) * linear +
                       4.0 * cfg_.layers * static_cast<double>(D_) * cfg_.heads * sum_sq +
                       2.0 * static_cast<double>(2 * total_frames_) * H_ * CV_;
  st->kernels_per_step = kernels_per_step_;
  st->kernels_per_reset = kernels_per_reset_;
  st->h2d_bytes = h2d_bytes_;
  st->d2h_bytes = d2h_bytes_;
  st->stream = stream_;
}

}  // namespace ovb

// ------------------------------------------------------------------ C-ABI

struct ov_generator {
  std::unique_ptr<ovb::Engine> engine;
};

namespace {

// Runs body with the reference's error prefix, except that cancellation
// reports exactly "cancelled" (generator.cpp:509, synthesis_test.cpp:126-129).
template <typename Body>
int GuardGen(const char* prefix, Body&& body) {
  try {
    ovb::ClearError();
    body();
    return OV_OK;
  } catch (const ovb::Error& e) {
    if (e.status() == OV_ERR_CANCELLED) return ovb::Fail(OV_ERR_CANCELLED, "cancelled");
    return ovb::Fail(e.status(), std::string(prefix) + e.what());
  } catch (const std::bad_alloc&) {
    return ovb::Fail(OV_ERR_OOM, std::string(prefix) + "host allocation failed");
  } catch (const std::exception& e) {
    return ovb::Fail(OV_ERR_INVALID, std::string(prefix) + e.what());
  }
}

}  // namespace

extern "C" {

void ov_default_model_config(ov_model_config* c) {
  c->vocab_size = 151936;
  c->hidden_size = 1024;
  c->intermediate_size = 3072;
  c->layers = 28;
  c->heads = 16;
  c->kv_heads = 8;
  c->head_dim = 128;
  c->max_positions = 40960;
  c->rms_norm_eps = 1e-6f;
  c->rope_theta = 1000000.0f;
  c->audio_codebooks = 8;
  c->audio_vocab_size = 1025;
  c->audio_mask_id = 1024;
}

void ov_default_decoding_config(ov_decoding_config* d) {
  d->steps = 32;
  d->guidance = 2.0f;
  d->t_shift = 0.1f;
  d->layer_penalty = 5.0f;
  d->position_temperature = 5.0f;
}

int ov_generator_load(const ov_model_config* config, const char* path, int device,
                      ov_generator** generator) {
  *generator = nullptr;
  return GuardGen("OmniVoice generator: ", [&] {
    auto g = std::make_unique<ov_generator>();
    g->engine = std::make_unique<ovb::Engine>(*config, device);
    g->engine->LoadSafetensors(path);
    *generator = g.release();
  });
}

int ov_generator_create_synthetic(const ov_model_config* config, uint64_t seed, int device,
                                  ov_generator** generator) {
  *generator = nullptr;
  return GuardGen("OmniVoice generator: ", [&] {
    auto g = std::make_unique<ov_generator>();
    g->engine = std::make_unique<ovb::Engine>(*config, device);
    g->engine->LoadSynthetic(seed);
    *generator = g.release();
  });
}

void ov_generator_destroy(ov_generator* generator) { delete generator; }

int ov_generator_forward(ov_generator* g, const ov_conditional_input* input, float* logits) {
  return GuardGen("OmniVoice forward: ", [&] {
    g->engine->Prepare(input, 1, nullptr, nullptr, 0);
    g->engine->ForwardOnce(logits, 0.0f, nullptr, nullptr);
  });
}

int ov_generator_score(ov_generator* g, const ov_conditional_input* input, float guidance,
                       int32_t* prediction, float* confidence) {
  return GuardGen("OmniVoice score: ", [&] {
    g->engine->Prepare(input, 1, nullptr, nullptr, 0);
    g->engine->ForwardOnce(nullptr, guidance, prediction, confidence);
  });
}

int ov_generator_generate(ov_generator* g, const ov_conditional_input* input,
                          const ov_decoding_config* decoding, uint64_t seed, int noise_mode,
                          ov_cancel_fn cancelled, void* user, int32_t* codes,
                          int32_t* unmasked_at) {
  return GuardGen("OmniVoice generation: ", [&] {
    g->engine->Prepare(input, 1, decoding, &seed, noise_mode);
    g->engine->Run(cancelled, user);
    g->engine->Fetch(&codes, &unmasked_at);
  });
}

int ov_generator_generate_batch(ov_generator* g, const ov_conditional_input* inputs,
                                size_t count, const ov_decoding_config* decoding,
                                const uint64_t* seeds, int noise_mode, ov_cancel_fn cancelled,
                                void* user, int32_t** codes, int32_t** unmasked_at) {
  return GuardGen("OmniVoice generation: ", [&] {
    g->engine->Prepare(inputs, count, decoding, seeds, noise_mode);
    g->engine->Run(cancelled, user);
    g->engine->Fetch(codes, unmasked_at);
  });
}

int ov_generator_prepare(ov_generator* g, const ov_conditional_input* inputs, size_t count,
                         const ov_decoding_config* decoding, const uint64_t* seeds,
                         int noise_mode) {
  return GuardGen("OmniVoice generation: ", [&] {
    g->engine->Prepare(inputs, count, decoding, seeds, noise_mode);
  });
}

int ov_generator_run(ov_generator* g, ov_cancel_fn cancelled, void* user) {
  return GuardGen("OmniVoice generation: ", [&] { g->engine->Run(cancelled, user); });
}

int ov_generator_fetch(ov_generator* g, int32_t** codes, int32_t** unmasked_at) {
  return GuardGen("OmniVoice generation: ", [&] { g->engine->Fetch(codes, unmasked_at); });
}

int ov_generator_stats_get(ov_generator* g, ov_generator_stats* stats) {
  return GuardGen("OmniVoice generator: ", [&] { g->engine->Stats(stats); });
}

int ov_generator_profile_step(ov_generator* g, ov_kernel_time* times, size_t capacity,
                              size_t* count) {
  return GuardGen("OmniVoice generator: ", [&] {
    const std::vector<ov_kernel_time> t = g->engine->Profile();
    const size_t n = std::min(capacity, t.size());
    std::copy(t.begin(), t.begin() + static_cast<std::ptrdiff_t>(n), times);
    *count = n;
  });
}

}  // extern "C"
