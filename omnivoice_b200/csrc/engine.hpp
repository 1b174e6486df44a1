// The generator engine behind ov_generator.h: one replica of the OmniVoice
// backbone on one GPU (the reference's Generator::State,
// generator.cpp:87-304), extended to packed batches of utterances.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "device_buffer.hpp"
#include "gemm.hpp"
#include "ov_generator.h"
#include "pack.hpp"

namespace ovb {

class Engine {
 public:
  Engine(const ov_model_config& config, int device);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  void LoadSynthetic(uint64_t seed);
  void LoadSafetensors(const std::string& path);

  // Uploads a packed batch and (re)builds plans and the step graph when its
  // shape changed.  decoding == nullptr prepares a forward-only batch.
  void Prepare(const ov_conditional_input* inputs, size_t count, const ov_decoding_config* decoding,
               const uint64_t* seeds, int noise_mode);
  // Restores the prepared initial state and runs every non-empty step.
  void Run(ov_cancel_fn cancelled, void* user);
  // Copies codes / unmasked_at of each utterance to the host.
  void Fetch(int32_t** codes, int32_t** unmasked_at);

  // One forward of the prepared batch (no graph): logits of utterance 0
  // compacted into [2F][C*V]; with prediction != nullptr also the scores.
  void ForwardOnce(float* logits, float guidance, int32_t* prediction, float* confidence);

  void Stats(ov_generator_stats* stats) const;
  // Device time per kernel class of one step (ov_generator_profile_step).
  std::vector<ov_kernel_time> Profile();
  int device() const { return device_; }
  void Activate() const;

  // Kernel classes of a step, in launch order.
  enum Kind {
    kEmbedNorm, kRmsNorm, kGemmQkv, kAttention, kGemmO, kGemmGateUp, kGemmDown,
    kGatherNorm, kGemmHead, kScore, kSelect, kKinds
  };
  // Called before each launch when a step is profiled.
  struct Marker {
    virtual ~Marker() = default;
    virtual void Mark(int kind, double flops, double bytes) = 0;
  };

 private:
  struct LayerPlans {
    GemmPlan qkv, o, gate_up, down;
  };

  void CheckConfig() const;
  void AllocateWeights();
  void EnsureRope(size_t positions);
  void BuildPlans();
  void EnqueueForward(cudaStream_t stream, Marker* marker = nullptr);
  void EnqueueDecode(cudaStream_t stream, Marker* marker = nullptr);
  void EnqueueReset(cudaStream_t stream);
  void CaptureGraph();
  void DestroyGraph();
  float* LayerNorms(size_t layer) const;  // [input H | post H | q D | k D]

  ov_model_config cfg_;
  int device_ = 0;
  int sms_ = 148;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t step_done_[2] = {nullptr, nullptr};

  // Derived sizes.
  size_t H_, I_, D_, QH_, QKVW_, C_, V_, CV_, ldl_;

  // Weights.
  DeviceBuffer<float> text_;        // [vocab][H]
  DeviceBuffer<float> audio_emb_;   // [C*V][H]
  DeviceBuffer<uint16_t> heads_;    // [C*V][H]
  DeviceBuffer<float> final_norm_;  // [H]
  DeviceBuffer<uint16_t> qkv_w_;    // [layers][QKVW][H]
  DeviceBuffer<uint16_t> o_w_;      // [layers][H][QH]
  DeviceBuffer<uint16_t> gu_w_;     // [layers][2I][H], gate/up interleaved
  DeviceBuffer<uint16_t> down_w_;   // [layers][H][I]
  DeviceBuffer<float> norms_;       // [layers][2H + 2D]
  DeviceBuffer<float> rope_cos_, rope_sin_;
  size_t rope_positions_ = 0;
  bool loaded_ = false;

  // The prepared pack.
  std::vector<UttDesc> utts_;
  std::vector<size_t> frames_;   // per utterance
  std::vector<int32_t> step_list_;
  size_t R_ = 0, total_frames_ = 0, n_seqs_ = 0, max_seqlen_ = 0, max_slots_ = 0;
  std::string signature_;
  float guidance_ = 2.0f, layer_penalty_ = 5.0f, temperature_ = 0.0f;
  int noise_ = 0;
  bool decode_ready_ = false;

  // Pack inputs (device) and their pristine copies.
  DeviceBuffer<int32_t> ids_, ids_init_, positions_, row_text_, cu_seqlens_, targets_;
  DeviceBuffer<int32_t> frame_utt_, counts_, step_list_d_, launch_;
  DeviceBuffer<int32_t> attn_items_;  // [n_items][2] (sequence, query-tile pair)
  bool single_tiles_ = false;         // attention items are single query tiles
  size_t n_items_ = 0;
  DeviceBuffer<UttDesc> utts_d_;
  DeviceBuffer<float> gumbel_;
  // Activations.
  DeviceBuffer<float> hidden_, logits_, conf_;
  DeviceBuffer<uint16_t> normed_, qkv_, attn_, act_, final_;
  DeviceBuffer<int32_t> pred_, codes_, unmasked_;
  DeviceBuffer<uint8_t> gemm_ws_;
  size_t gemm_ws_bytes_ = 0;
  // Pinned host staging of the batch uploads.
  uint8_t* staging_ = nullptr;
  size_t staging_bytes_ = 0;
  size_t h2d_bytes_ = 0, d2h_bytes_ = 0;

  std::vector<LayerPlans> plans_;
  GemmPlan head_plan_;
  CUtensorMap qkv_map_;
  CUtensorMap attn_out_map_;
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t graph_exec_ = nullptr;
  size_t kernels_per_step_ = 0;
  size_t kernels_per_reset_ = 3;
};

}  // namespace ovb
