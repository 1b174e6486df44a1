/*
 * ov_kernels.h - C-ABI device kernels of omnivoice-b200 (sm_100a).
 *
 * Replaces the reference's kernels/generator_kernels.hpp:21-66 and
 * gemm.hpp:43-62.  Every pointer argument named like a tensor is DEVICE
 * memory; sizes are element counts; half-precision tensors are passed as
 * uint16_t so host translation units need no CUDA headers (the reference's
 * `Half = __half`, generator_kernels.hpp:17).  Every call is asynchronous on
 * `stream` and returns an OV_* status from ov_runtime.h.
 *
 * Row conventions follow generator_kernels.hpp:10-12: rows are token
 * positions of a packed batch of sequences.  Unlike the reference, several
 * utterances may be packed into one batch (see ov_utterance).
 */
#ifndef OMNIVOICE_B200_OV_KERNELS_H_
#define OMNIVOICE_B200_OV_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#include "ov_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- embed */

/* generator_kernels.hpp:19-24 (Embed) with the text-embedding gather moved
 * to the device (the reference gathers on the host, generator.cpp:204-217)
 * and the first layer's input RMSNorm fused in.
 *   row_text_ids[r] >= 0 : hidden[r] = text_table[row_text_ids[r]]
 *   row_text_ids[r] <  0 : hidden[r] = sum_c audio_table[c*audio_vocab + ids[c*rows + r]]
 * (codebooks summed in order c = 0..codebooks-1 from 0.0f, as the reference).
 * When norm_weight != NULL also writes normed[r] = half(w * (x * rsqrt(mean(x^2) + eps))). */
int ov_embed(const float* text_table, size_t text_vocab, const int32_t* row_text_ids,
             const float* audio_table, size_t audio_vocab, const int32_t* ids,
             size_t codebooks, size_t rows, size_t width, float* hidden,
             const float* norm_weight, float epsilon, uint16_t* normed, ov_stream_t stream);

/* generator_kernels.hpp:26-29 (RmsNorm): output = half(w * (x * rsqrt(mean(x^2) + eps))). */
int ov_rmsnorm(const float* input, const float* weight, uint16_t* output, size_t rows,
               size_t width, float epsilon, ov_stream_t stream);

/* generator_kernels.hpp:54-56 (GatherRows) fused with the final RmsNorm
 * (generator.cpp:295-298): output[i] = rmsnorm(input[indices[i]]). */
int ov_gather_rmsnorm(const float* input, const int32_t* indices, size_t count,
                      const float* weight, uint16_t* output, size_t width, float epsilon,
                      ov_stream_t stream);

/* ---------------------------------------------------------- QK norm/RoPE */

/* Host helper: Hugging Face default RoPE tables, inv_freq = 1 / theta^(2i/d)
 * in float32 and angle = position * inv_freq (generator_kernels.hip:209-214),
 * evaluated once on the host: cos_table/sin_table are [max_positions][head_dim/2]. */
int ov_rope_tables(float theta, size_t head_dim, size_t max_positions, float* cos_table,
                   float* sin_table);

/* generator_kernels.hpp:31-39 (QkNormRope) as a standalone kernel.  Input is
 * the float32 fused projection [rows][ (heads + 2 kv_heads) * head_dim ];
 * output is half in the SAME token-major layout (q heads, k heads, v heads),
 * with k and v stored once per kv head (the attention maps query head h to
 * kv head h / (heads / kv_heads) instead of repeating k and v).  The fused
 * GEMM epilogue OV_EPI_QKNORM_ROPE_F16 computes the same values. */
int ov_qknorm_rope(const float* qkv, size_t ld_in, const float* q_norm, const float* k_norm,
                   const int32_t* positions, const float* rope_cos, const float* rope_sin,
                   size_t max_positions, size_t rows, size_t heads, size_t kv_heads,
                   size_t head_dim, float epsilon, uint16_t* output, size_t ld_out,
                   ov_stream_t stream);

/* generator_kernels.hpp:50-52 (SwiGlu): out[r][i] = half(silu(g[r][i]) * g[r][width+i]). */
int ov_swiglu(const float* gate_up, size_t rows, size_t width, uint16_t* output,
              ov_stream_t stream);

/* ----------------------------------------------------------------- GEMM */

/* Epilogues of the tcgen05 GEMM.  OV_EPI_STORE_F32 / OV_EPI_ACCUM_F32 are
 * HalfGemm::Linear with accumulate false / true (gemm.hpp:41-42). */
enum {
  OV_EPI_STORE_F32 = 0,       /* y[r][n]  = acc                                */
  OV_EPI_ACCUM_F32 = 1,       /* y[r][n] += acc  (residual stream)             */
  OV_EPI_SWIGLU_F16 = 2,      /* y[r][j]  = half(silu(gate) * up)              */
  OV_EPI_QKNORM_ROPE_F16 = 3  /* y[r][n]  = ov_qknorm_rope of the projection   */
};

/* Gate/up interleave group of OV_EPI_SWIGLU_F16: w's rows come in groups
 * of 2 * OV_SWIGLU_GROUP, rows [2gG, 2gG+G) being gate rows [gG, gG+G) and
 * rows [2gG+G, 2gG+2G) the matching up rows (ov_interleave_gate_up builds
 * it from the reference's [gate | up] stacking, generator.cpp:411-414). */
#define OV_SWIGLU_GROUP 64

/* Extra operands of the fused epilogues.
 * SWIGLU: w interleaved as above, out a multiple of 128; y is [rows][out/2].
 * QKNORM_ROPE: the fields below describe the heads; head_dim must be 128. */
typedef struct {
  const float* q_norm;
  const float* k_norm;
  const int32_t* positions;
  const float* rope_cos;
  const float* rope_sin;
  int32_t max_positions;
  int32_t heads;
  int32_t kv_heads;
  int32_t head_dim;
  float epsilon;
} ov_epilogue_args;

/* y (+)= x[rows][in] * w[out][in]^T with float16 operands and float32
 * accumulation in tensor memory (gemm.hpp:41-42, gemm.cpp:248-262).
 * x, w are K-major with row strides ldx / in elements (multiples of 8);
 * y's row stride ldy is in elements of the output type.  Short-M products
 * with the residual or plain-store epilogue may be split along K across a
 * thread-block cluster; the splits' partials are summed in split order, so
 * results do not depend on timing.  `workspace` (optional, may be NULL,
 * 16-byte aligned) lets the splits exchange their partials through global
 * memory instead of distributed shared memory (faster), and allows a
 * serialised split-K whose splits add into y in split order behind one
 * order counter per output tile.  ov_gemm_workspace_bytes gives the size
 * the chosen shape needs (0: none); with a smaller workspace the call
 * chooses as if it had none.  Zero the workspace once before its first
 * use (every call leaves the counters zero again); calls sharing a
 * workspace must not overlap. */
int ov_gemm_f16(const uint16_t* x, size_t ldx, const uint16_t* w, void* y, size_t ldy,
                size_t rows, size_t in, size_t out, int epilogue,
                const ov_epilogue_args* args, void* workspace, size_t workspace_bytes,
                ov_stream_t stream);
size_t ov_gemm_workspace_bytes(size_t rows, size_t in, size_t out, int epilogue);
/* Host helper: interleave [gate(width) | up(width)] rows of a float16 weight
 * [2*width][in] into groups of OV_SWIGLU_GROUP rows (layout described above). */
int ov_interleave_gate_up(const uint16_t* gate_up, size_t width, size_t in, uint16_t* output);

/* ov_gemm_f16 for callers that cannot allocate device memory.  No
 * counterpart in the reference: it is an addition of this library.
 *
 * Some callers cannot call cudaMalloc: a host process that has handed all
 * of the GPU's memory to its own pool, or code on a latency-critical path
 * where cudaMalloc / cudaFree would block on or synchronise the device.
 * This entry point allocates nothing.  Its split-K scratch (per-tile order
 * counters) is a 64 KiB file-scope device array that every GPU loading the
 * library holds until the process exits; bounded waits report into a status
 * word kept with it, which ov_take_device_errors reads and clears together
 * with the library's other device error word.
 * Inputs and outputs are the caller's, as for ov_gemm_f16.
 *   - The first call on a device sets up that device (looks up the array's
 *     device address with that device current, clears it and the status
 *     word, and measures the cluster capacities the tile choice uses);
 *     make that first call before any stream capture.
 *   - Split-K here uses the scratch only for its per-tile order counters
 *     (the partial-slice exchange of ov_gemm_f16's workspace is not
 *     offered); a product that would need more than 64 KiB of counters is
 *     rejected with OV_ERR_INVALID (none does on a 148-SM B200).  A call
 *     that uses them clears them first (cudaMemsetAsync on `stream`), so a
 *     split whose wait timed out in an earlier call leaves no stale order
 *     behind.
 *   - Every call shares the array, which keeps the last call's contents:
 *     calls that overlap on the GPU (different streams, or different host
 *     threads on one device) race and must be serialised by the caller. */
int ov_gemm_f16_noalloc(const uint16_t* x, size_t ldx, const uint16_t* w, void* y, size_t ldy,
                        size_t rows, size_t in, size_t out, int epilogue,
                        const ov_epilogue_args* args, ov_stream_t stream);

/* General strided-batched product in the column-major BLAS convention of
 * HalfGemm::Matmul (gemm.hpp:16-36,56-57): for each batch b,
 * C_b[m][n] (+)= op(A_b)[m][k] * op(B_b)[k][n], element (i, j) of a
 * column-major matrix X at x[i + j * ldx], op(X) = X^T when transpose_x.
 * float16 operands, float32 accumulation and output.  Off the generator's
 * hot path (a plain CUDA-core kernel); any K and strides. */
typedef struct {
  int32_t transpose_a;
  int32_t transpose_b;
  size_t m, n, k;
  size_t lda, ldb, ldc;
  int64_t stride_a, stride_b, stride_c; /* elements between batches */
  size_t batch;
  int32_t accumulate;
} ov_matmul_shape;
int ov_matmul_f16(const ov_matmul_shape* shape, const uint16_t* a, const uint16_t* b, float* c,
                  ov_stream_t stream);

/* ------------------------------------------------------------ attention */

/* Bidirectional (non-causal) attention within each packed sequence,
 * replacing the reference's per-sequence Scores/Softmax/Values GEMMs and
 * MergeHeads (generator.cpp:122-172, generator_kernels.hpp:41-48).
 * qkv is half [rows][ld_qkv] holding heads q heads, then kv_heads k heads,
 * then kv_heads v heads, head_dim = 128 each; cu_seqlens (device, int32,
 * num_seqs + 1 entries) gives sequence boundaries; out is half
 * [rows][ld_out] with heads * head_dim columns (the merged heads).
 * Probabilities are rounded to half before the PV product, as the reference. */
int ov_attention_varlen(const uint16_t* qkv, size_t ld_qkv, size_t rows,
                        const int32_t* cu_seqlens, size_t num_seqs, size_t max_seqlen,
                        size_t heads, size_t kv_heads, size_t head_dim, float scale,
                        uint16_t* out, size_t ld_out, ov_stream_t stream);

/* ov_attention_varlen over an explicit work list, the generator's own form:
 * items (device, int32 [n_items][2], at most 65535) = (sequence, first
 * 128-query tile | tiles per item << 24) with 2 tiles per item (query-tile
 * pairs) or 1 (single tiles; every item must then have 1), one CTA per
 * (item, head), items started in list order.  Every query tile of every
 * sequence must be covered exactly once; an item naming a sequence outside
 * [0, num_seqs) is skipped and reported as OV_DEVICE_BAD_ARGUMENT by
 * ov_take_device_errors. */
int ov_attention_varlen_items(const uint16_t* qkv, size_t ld_qkv, size_t rows,
                              const int32_t* cu_seqlens, size_t num_seqs, size_t max_seqlen,
                              const int32_t* items, size_t n_items, int single_tiles,
                              size_t heads, size_t kv_heads, size_t head_dim, float scale,
                              uint16_t* out, size_t ld_out, ov_stream_t stream);

/* ------------------------------------------------------ decoding tail */

/* generator_kernels.hpp:58-66 (Score).  logits rows [0, frames) are
 * conditional, [frames, 2 frames) unconditional, row stride ld; per
 * [codebook][frame]: g = c + guidance * (c - u) of the log-softmaxed rows,
 * prediction = argmax over j != mask_id (lowest index on ties),
 * confidence = max - logsumexp(g). */
int ov_score(const float* logits, size_t ld, size_t frames, size_t codebooks, size_t vocab,
             uint32_t mask_id, float guidance, int32_t* prediction, float* confidence,
             ov_stream_t stream);

/* Noise sources of the position choice (decoding.cpp:82-87). */
enum {
  OV_NOISE_NONE = 0,    /* temperature 0: greedy position choice            */
  OV_NOISE_DEVICE = 1,  /* counter-based Philox-4x32-10 on the device       */
  OV_NOISE_BUFFER = 2   /* caller-supplied Gumbel values, e.g. the host
                           std::mt19937_64 stream of the reference          */
};

/* decoding.cpp:70-106 (PositionSelector::Fill) plus the code write-back of
 * generator.cpp:526-535, on the device, for one utterance:
 *   score = confidence - c * layer_penalty;  if temperature > 0:
 *   score = score / temperature + gumbel;  slots whose code is not mask_id
 *   get -inf; the `count` best slots by (score desc, index asc) take their
 *   prediction, record `step` in unmasked_at, and are written into
 *   ids[c*ids_rows + cond_row + f] and ids[c*ids_rows + uncond_row + f].
 * codes / unmasked_at / prediction / confidence are [codebook][frame].
 * noise: OV_NOISE_BUFFER -> gumbel points at codebooks*frames floats;
 *        OV_NOISE_DEVICE -> noise_seed and step select the Philox stream. */
int ov_select_positions(const int32_t* prediction, const float* confidence, size_t codebooks,
                        size_t frames, size_t count, float layer_penalty, float temperature,
                        int noise_mode, const float* gumbel, uint64_t noise_seed, int32_t step,
                        uint32_t mask_id, int32_t* codes, int32_t* unmasked_at, int32_t* ids,
                        size_t ids_rows, size_t cond_row, size_t uncond_row,
                        ov_stream_t stream);

/* Host helper: the Gumbel value the device path derives from a uniform u,
 * -log(-log(u + 1e-10) + 1e-10) in float32 (decoding.cpp:84-85). */
float ov_gumbel_from_uniform(float uniform);

/* -------------------------------------------------- synthetic weights */

/* Deterministic random-init weights, identical on host and device:
 * value(i) = (s - 131070) * (std / 37837.2269...), s the sum of the four
 * 16-bit lanes of splitmix64(seed ^ (tensor << 40) ^ i) (an Irwin-Hall(4)
 * approximation of N(0, std^2)).  Device fill: */
int ov_synthetic_fill(float* output, size_t count, uint64_t seed, uint64_t tensor, float std,
                      uint64_t first_index, ov_stream_t stream);
/* ... and the same values on the host. */
int ov_synthetic_fill_host(float* output, size_t count, uint64_t seed, uint64_t tensor,
                           float std, uint64_t first_index);

#ifdef __cplusplus
}
#endif

#endif /* OMNIVOICE_B200_OV_KERNELS_H_ */
