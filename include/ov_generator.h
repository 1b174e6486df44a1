/*
 * ov_generator.h - C-ABI of the OmniVoice generator on B200.
 *
 * The C entry points an FFI binds to drive the whole hot path: the
 * 32-step masked-unmasking loop with classifier-free guidance over the
 * bidirectional Qwen3 backbone.  They replace, one for one, the reference's
 * C++ class gufo::models::omnivoice::Generator (generator.hpp:20-56):
 *   ov_generator_load / _create_synthetic  <- Generator::Load      (generator.cpp:364-434)
 *   ov_generator_forward                    <- Generator::Forward   (generator.cpp:436-454)
 *   ov_generator_score                      <- Generator::Score     (generator.cpp:456-484)
 *   ov_generator_generate                   <- Generator::Generate  (generator.cpp:486-543)
 * and add a packed multi-utterance variant (ov_generator_generate_batch).
 * The C++ drop-in class with the reference's exact signatures lives in
 * omnivoice_b200/csrc/host/generator.hpp and is built on these functions'
 * implementation.  All array arguments here are HOST memory.
 *
 * A generator is not thread-safe (generator.hpp:17-19); use one per GPU.
 */
#ifndef OMNIVOICE_B200_OV_GENERATOR_H_
#define OMNIVOICE_B200_OV_GENERATOR_H_

#include <stddef.h>
#include <stdint.h>

#include "ov_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ov_generator ov_generator;

/* config.hpp:15-26 (BackboneConfig) and config.hpp:74-82 (Config). */
typedef struct {
  size_t vocab_size;
  size_t hidden_size;
  size_t intermediate_size;
  size_t layers;
  size_t heads;
  size_t kv_heads;
  size_t head_dim;
  size_t max_positions;
  float rms_norm_eps;
  float rope_theta;
  size_t audio_codebooks;
  size_t audio_vocab_size;
  uint32_t audio_mask_id;
} ov_model_config;

/* decoding.hpp:14-21 (DecodingConfig). */
typedef struct {
  size_t steps;
  float guidance;
  float t_shift;
  float layer_penalty;
  float position_temperature;
} ov_decoding_config;

/* decoding.hpp:32-47 (ConditionalInput): ids is [codebooks][length]. */
typedef struct {
  size_t codebooks;
  size_t length;
  size_t audio_start;
  size_t target_frames;
  const int32_t* ids;
} ov_conditional_input;

/* Noise of the position choice (decoding.cpp:82-87):
 *   OV_GEN_NOISE_REFERENCE - the reference's own stream: std::mt19937_64(seed),
 *     one draw per [codebook][frame] slot per non-empty step, u = (x >> 40) * 2^-24,
 *     Gumbel -log(-log(u + 1e-10) + 1e-10), drawn on the host and uploaded once;
 *   OV_GEN_NOISE_DEVICE - a counter-based Philox-4x32-10 stream on the device
 *     keyed by seed (no host work, different values from the reference's).
 * With position_temperature == 0 no noise is drawn in either mode. */
enum { OV_GEN_NOISE_REFERENCE = 0, OV_GEN_NOISE_DEVICE = 1 };

/* Returns nonzero to cancel; polled before every step (generator.cpp:508-511). */
typedef int (*ov_cancel_fn)(void* user);

/* Qwen3-0.6B-shaped OmniVoice defaults (vocab 151936, 28 layers, ...). */
void ov_default_model_config(ov_model_config* config);
void ov_default_decoding_config(ov_decoding_config* config);

/* Loads `model.safetensors`-format float32 weights with the reference's
 * tensor names (generator.cpp:381-425) onto `device`. */
int ov_generator_load(const ov_model_config* config, const char* safetensors_path, int device,
                      ov_generator** generator);
/* Random-init weights (ov_synthetic_fill, seed `weight_seed`) generated on the device. */
int ov_generator_create_synthetic(const ov_model_config* config, uint64_t weight_seed,
                                  int device, ov_generator** generator);
void ov_generator_destroy(ov_generator* generator);

/* logits: [2 * target_frames][codebooks * audio_vocab_size], conditional rows first. */
int ov_generator_forward(ov_generator* generator, const ov_conditional_input* input,
                         float* logits);
/* prediction / confidence: [codebooks][target_frames]. */
int ov_generator_score(ov_generator* generator, const ov_conditional_input* input,
                       float guidance, int32_t* prediction, float* confidence);
/* codes / unmasked_at: [codebooks][target_frames]. */
int ov_generator_generate(ov_generator* generator, const ov_conditional_input* input,
                          const ov_decoding_config* decoding, uint64_t seed, int noise_mode,
                          ov_cancel_fn cancelled, void* user, int32_t* codes,
                          int32_t* unmasked_at);
/* `count` independent utterances packed into one batch; codes[i] and
 * unmasked_at[i] are [codebooks][inputs[i].target_frames]. */
int ov_generator_generate_batch(ov_generator* generator, const ov_conditional_input* inputs,
                                size_t count, const ov_decoding_config* decoding,
                                const uint64_t* seeds, int noise_mode, ov_cancel_fn cancelled,
                                void* user, int32_t** codes, int32_t** unmasked_at);

/* Split form of generate_batch for timing: prepare uploads the inputs and
 * records the step graph, run executes every step on the device without
 * host synchronisation, fetch copies the results back. */
int ov_generator_prepare(ov_generator* generator, const ov_conditional_input* inputs,
                         size_t count, const ov_decoding_config* decoding,
                         const uint64_t* seeds, int noise_mode);
int ov_generator_run(ov_generator* generator, ov_cancel_fn cancelled, void* user);
int ov_generator_fetch(ov_generator* generator, int32_t** codes, int32_t** unmasked_at);

/* Host decoding helpers of the generator (decoding.hpp:23-47):
 * UnmaskSchedule (decoding.cpp:12-40) writes `steps` counts, and
 * ConditionalInput::Build (decoding.cpp:42-62) writes
 * [codebooks][text + reference + target] ids and returns the length. */
int ov_unmask_schedule(size_t total, size_t steps, float t_shift, size_t* counts);
size_t ov_build_conditional_input(const uint32_t* text_ids, size_t text_count,
                                  const int32_t* reference_codes, size_t reference_frames,
                                  size_t target_frames, size_t codebooks, uint32_t mask_id,
                                  int32_t* ids);

/* Timing and accounting of the last prepared batch. */
typedef struct {
  size_t rows;              /* packed GEMM rows per step, sum of L + F      */
  size_t steps_run;         /* non-empty steps                              */
  double flops_per_step;    /* algorithmic FLOPs of one forward             */
  size_t kernels_per_step;  /* kernels this library launches per step       */
  size_t kernels_per_reset; /* kernels launched to restore the initial state */
  size_t h2d_bytes;         /* host->device bytes of the last prepare       */
  size_t d2h_bytes;         /* device->host bytes of the last fetch         */
  ov_stream_t stream;       /* the generator's stream                       */
} ov_generator_stats;
int ov_generator_stats_get(ov_generator* generator, ov_generator_stats* stats);

/* Device time of one step of the prepared batch by kernel class, measured
 * with CUDA events recorded on the generator's stream between the
 * kernels of one eagerly launched step (forward + scoring + selection; the
 * batch's state is restored afterwards).  flops / bytes are the
 * algorithmic work of all launches of the class. */
typedef struct {
  char name[32];
  double ms;
  size_t launches;
  double flops;
  double bytes;
} ov_kernel_time;
int ov_generator_profile_step(ov_generator* generator, ov_kernel_time* times, size_t capacity,
                              size_t* count);

#ifdef __cplusplus
}
#endif

#endif /* OMNIVOICE_B200_OV_GENERATOR_H_ */
