// Internal interface of the audio tokenizer's decoder kernels (codec.cu)
// and its engine (codec_engine.cpp).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "device_buffer.hpp"

namespace ovb {
namespace codec {

// A convolution's weights as the tensor cores read them: [taps][cout][cin]
// float32 split into tf32 hi and lo planes, plus the bias.
struct ConvWeights {
  DeviceBuffer<float> hi, lo, bias;
  int cin = 0;
  int cout = 0;
  int taps = 0;
};

// Per-launch arguments of conv_kernel (see codec.cu for the semantics).
struct ConvArgs {
  int m_count = 0;   // output positions (per phase for a transposed conv)
  int cin = 0;
  int cout = 0;
  int taps = 0;      // 1 or 7 (plain), 2 (a phase of a transposed conv)
  int dilation = 1;  // plain
  int pad = 0;       // plain: (kernel - 1) * dilation / 2; transposed: ceil(stride / 2)
  int stride = 0;    // 0: plain; else the transposed conv's stride (= phases)
  const float* bias = nullptr;
  const float* resid = nullptr;  // [rows_out][cout] added before the outputs, or null
  float* out_x = nullptr;        // [rows_out][cout] raw output, or null
  const float* alpha = nullptr;  // [cout] snake applied to the split planes, or null
  float* out_hi = nullptr;       // [rows_out][cout]
  float* out_lo = nullptr;
  uint32_t* err = nullptr;
};

struct ConvPlan {
  CUtensorMap map_a_hi, map_a_lo, map_b_hi, map_b_lo;
  ConvArgs args;
  dim3 grid;
  int bn = 128;
};

// Plans one convolution reading the split planes [rows_in][w.cin].
void PlanConv(ConvPlan* plan, const float* in_hi, const float* in_lo, int rows_in,
              const ConvWeights& w, int m_count, int phases, const ConvArgs& args);
void LaunchConv(const ConvPlan& plan, cudaStream_t stream);

void LaunchCodes(const float* table, const float* bias, const int32_t* codes, int codebooks,
                 int entries, int frames, int width, float* hi, float* lo, cudaStream_t stream);
void LaunchOutputConv(const float* hi, const float* lo, int rows, int channels,
                      const float* weight, const float* bias, float* out, cudaStream_t stream);
void LaunchDense(const float* A, const float* B, const float* bias, float* C, int M, int N, int K,
                 cudaStream_t stream);
void LaunchSplit(const float* src, float* hi, float* lo, int64_t n, cudaStream_t stream);

}  // namespace codec
}  // namespace ovb
