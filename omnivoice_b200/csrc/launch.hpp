// Internal kernel launchers shared between the C-ABI entry points and the
// generator engine.  All pointers are device memory; all launches are
// asynchronous on `stream` and throw ovb::Error on a launch failure.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>

#include "internal.hpp"
#include "pack.hpp"

namespace ovb {

// Programmatic dependent launch (PDL) for the kernels of a generator step:
// while a PdlScope(true) is alive on this thread, Launch() marks kernels so
// the next one may start (prologue, weight prefetch) before the previous one
// finishes; every kernel calls pdl_wait() before reading its inputs.
bool PdlEnabled();
class PdlScope {
 public:
  explicit PdlScope(bool on);
  ~PdlScope();
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;

 private:
  bool previous_;
};

// cluster_x > 1 launches thread-block clusters of cluster_x CTAs along x.
template <typename... KernelArgs, typename... Args>
void LaunchEx(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
              cudaStream_t stream, const char* what, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (PdlEnabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = n > 0 ? attr : nullptr;
  cfg.numAttrs = n;
  Check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

template <typename... KernelArgs, typename... Args>
void Launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
            cudaStream_t stream, const char* what, Args&&... args) {
  LaunchEx(kernel, grid, block, smem, stream, what, 1u, std::forward<Args>(args)...);
}

void LaunchEmbed(const float* text_table, size_t text_vocab, const int32_t* row_text_ids,
                 const float* audio_table, size_t audio_vocab, const int32_t* ids,
                 size_t codebooks, size_t rows, size_t width, float* hidden,
                 const float* norm_weight, float epsilon, uint16_t* normed, cudaStream_t stream);

// indices == nullptr: plain RMSNorm of `rows` rows.
void LaunchRmsNorm(const float* input, const int32_t* indices, size_t rows, const float* weight,
                   uint16_t* output, size_t width, float epsilon, cudaStream_t stream);

void EncodeQkvMap(CUtensorMap* map, const uint16_t* qkv, int64_t ld_qkv, int64_t rows,
                  int64_t width);
// Attention output [rows][width] fp16 as 128B-swizzled [128][64] boxes.
void EncodeAttnOutMap(CUtensorMap* map, const uint16_t* out, int64_t ld_out, int64_t rows,
                      int64_t width);
// items: device [n_items][2] (sequence, pair of 128-query tiles), longest
// sequences first; null covers ceil(max_seqlen / 256) pairs of every
// sequence (CTAs past a sequence's end exit at once).
void LaunchAttention(const CUtensorMap& map_qkv, const CUtensorMap& map_out,
                     const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                     const int32_t* items, int n_items, int heads, int kv_heads, float scale,
                     __half* out, int64_t ld_out, cudaStream_t stream, bool single = false);

void LaunchScore(const float* logits, int64_t ld, int total_frames, int codebooks, int vocab,
                 uint32_t mask_id, float guidance, const UttDesc* utts, const int32_t* frame_utt,
                 int single_frames, int32_t* prediction, float* confidence, cudaStream_t stream);

void LaunchSelect(const int32_t* prediction, const float* confidence, int codebooks,
                  float layer_penalty, float temperature, int noise_mode, uint32_t mask_id,
                  int32_t* codes, int32_t* unmasked_at, int32_t* ids, int64_t ids_rows,
                  const UttDesc& single, const UttDesc* table, int utterances, StepControl ctl,
                  int max_slots, int explicit_count, int explicit_step, int single_cond_row,
                  int single_uncond_row, cudaStream_t stream);

// Weight preparation (weights.cu).
// out[dst_row(j)][k] = half(src[j][k]) for a [rows][cols] float32 source,
// dst_row(j) = j, or with group > 0 the gate/up interleave
// (j / group) * 2 group + offset + j % group.
void LaunchToHalfRows(const float* src, uint16_t* out, int64_t rows, int64_t cols, int group,
                      int offset, cudaStream_t stream);
// Fills `count` floats with the synthetic checkpoint values of `tensor`.
void LaunchSyntheticFill(float* out, size_t count, uint64_t seed, uint64_t tensor, float std,
                         cudaStream_t stream);
void LaunchFill(float* out, size_t count, float value, cudaStream_t stream);
void LaunchFillInt(int32_t* out, size_t count, int32_t value, cudaStream_t stream);

// Sets the dynamic shared memory limit of `func` on the current device once.
void SetMaxDynamicSmem(const void* func, int bytes);
// Set every kernel's shared-memory limit on the current device up front,
// so no attribute call happens while a CUDA graph is being captured.
void ConfigureGemmKernels();
void ConfigureAttentionKernel();
void ConfigureSelectKernel();

}  // namespace ovb
