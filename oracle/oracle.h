/*
 * oracle.h - CPU restatement of the OmniVoice generator hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the
 * checker / the timed CPU baseline; the product (omnivoice_b200) never
 * links or calls it.
 *
 * Restates, in plain scalar C++ with std::thread parallelism:
 *   oc_forward   generator.cpp:175-301 (Prepare + RunForward) with the
 *                kernels of kernels/generator_kernels.hip:62-209 and the
 *                fp16-operand / fp32-accumulate GEMM of gemm.cpp:248-262;
 *   oc_score     generator_kernels.hip:212-265 (ScoreKernel);
 *   oc_schedule  decoding.cpp:12-40 (UnmaskSchedule);
 *   oc_build_input decoding.cpp:42-62 (ConditionalInput::Build);
 *   oc_select    decoding.cpp:70-107 (PositionSelector::Fill);
 *   oc_generate  generator.cpp:486-543 (Generator::Generate).
 * Rounding points follow the reference: half at every RMSNorm output, at
 * q/k/v, at the softmax probabilities, at the merged heads and at the
 * SwiGLU output; float32 everywhere else.
 *
 * Parity pins: the decoding functions are checked against the reference's
 * own fixtures (tests/fixtures/generator_golden.json, committed as
 * tests/golden/decoding_golden.json) and against the reference's
 * decoding.cpp compiled from its sources (oracle/_ref).  The forward pass
 * has no reference fixture at random init (the reference's generator
 * fixtures need the real checkpoint, which is absent): forward parity is
 * pinned by this restatement only.
 */
#ifndef OMNIVOICE_B200_ORACLE_H_
#define OMNIVOICE_B200_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field layout as ov_model_config. */
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
} oc_config;

void oc_set_threads(int threads);
int oc_get_threads(void);

/* Order of the float32 sums of every linear layer: 0 (default) adds the
 * products in increasing input index, 1 in decreasing.  Both restate
 * gemm.cpp's float32 accumulation, whose order hipBLAS leaves unspecified;
 * the second one measures how far two valid restatements drift apart. */
void oc_set_accumulation_order(int reversed);

/* Synthetic random-init model (same tensors and values as the product's
 * synthetic checkpoint, restated from its published definition). */
void* oc_model_synthetic(const oc_config* config, uint64_t seed);
void oc_model_free(void* model);

/* `count` values of synthetic tensor `tensor` starting at element `first`
 * (the oracle's own restatement of the weight definition). */
void oc_synthetic_values(uint64_t seed, uint64_t tensor, float std, uint64_t first, size_t count,
                         float* out);

/* One CFG forward of one utterance: logits [2 frames][codebooks * vocab]
 * (conditional rows first).  layers_to_run < 0 runs every layer; when
 * hidden_out != NULL it receives the float32 residual stream [L + F][hidden]
 * after `layers_to_run` layers (then logits may be NULL). */
int oc_forward(void* model, const int32_t* ids, size_t length, size_t audio_start,
               size_t frames, float* logits, int layers_to_run, float* hidden_out);

int oc_score(const float* logits, size_t ld, size_t frames, size_t codebooks, size_t vocab,
             uint32_t mask_id, float guidance, int32_t* prediction, float* confidence);

void oc_schedule(size_t total, size_t steps, float t_shift, size_t* out);

/* ids_out: [codebooks][text + reference + target]. */
void oc_build_input(const uint32_t* text_ids, size_t text_count, const int32_t* reference_codes,
                    size_t reference_frames, size_t target_frames, size_t codebooks,
                    uint32_t mask_id, int32_t* ids_out);

/* The first `count` Gumbel values of the reference's std::mt19937_64(seed)
 * noise stream (decoding.cpp:84-85). */
void oc_reference_gumbel(uint64_t seed, size_t count, float* out);

/* PositionSelector::Fill with the noise given as Gumbel values per slot
 * (NULL when temperature <= 0).  Returns the number of chosen slots and
 * writes them to `chosen` (may be NULL) in (score desc, index asc) order. */
size_t oc_select(size_t count, size_t codebooks, size_t frames, const int32_t* prediction,
                 const float* confidence, uint32_t mask_id, float layer_penalty,
                 float temperature, const float* gumbel, int32_t* codes, size_t* chosen);

/* Generator::Generate.  gumbel_all: [steps][codebooks * frames] Gumbel
 * values indexed by step (NULL: draw the reference's mt19937_64(seed)
 * stream for every non-empty step, exactly as decoding.cpp does). */
int oc_generate(void* model, const int32_t* ids, size_t length, size_t audio_start,
                size_t frames, size_t steps, float guidance, float t_shift,
                float layer_penalty, float temperature, uint64_t seed,
                const float* gumbel_all, int32_t* codes, int32_t* unmasked_at);

/* oc_generate that also records, for every step, the ids the forward pass
 * saw ([steps][codebooks][length]) and the scoring's predictions and
 * confidences ([steps][codebooks][frames]); steps with nothing to unmask
 * are left untouched. */
int oc_generate_traced(void* model, const int32_t* ids, size_t length, size_t audio_start,
                       size_t frames, size_t steps, float guidance, float t_shift,
                       float layer_penalty, float temperature, uint64_t seed,
                       const float* gumbel_all, int32_t* codes, int32_t* unmasked_at,
                       int32_t* step_ids, int32_t* step_prediction, float* step_confidence);

#ifdef __cplusplus
}
#endif

#endif /* OMNIVOICE_B200_ORACLE_H_ */
