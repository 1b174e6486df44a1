// HBM-bound kernels of the generator step: the fused embedding gather +
// first RMSNorm, RMSNorm, target-row gather + final RMSNorm, and standalone
// forms of the QK-norm/RoPE and SwiGLU epilogues.  One warp owns one row;
// every lane moves float4 / 8-byte vectors so a warp touches whole 512-byte
// segments.  Reference kernels: kernels/generator_kernels.hip:62-209.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "norm_device.cuh"
#include "ptx.cuh"
#include "synthetic.hpp"

namespace ovb {
namespace {

constexpr int kRowsPerBlock = 4;  // warps per block, one row each

// generator_kernels.hip:62-83 (EmbedKernel) + :85-97 (RmsNormKernel).
template <int kVec>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    embed_kernel(const float* __restrict__ text_table, int64_t text_vocab,
                 const int32_t* __restrict__ row_text_ids, const float* __restrict__ audio_table,
                 int64_t audio_vocab, const int32_t* __restrict__ ids, int codebooks, int64_t rows,
                 float* __restrict__ hidden, const float* __restrict__ norm_weight,
                 float epsilon, __half* __restrict__ normed, uint32_t* err) {
  constexpr int width = 128 * kVec;
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  float4 x[kVec];
  const int32_t text_id = row_text_ids[row];
  if (text_id >= 0) {
    const int64_t id = text_id < text_vocab ? text_id : 0;
    if (text_id >= text_vocab && lane == 0) atomicOr(err, kErrBadArgument);
    const float* src = text_table + id * width;
#pragma unroll
    for (int i = 0; i < kVec; ++i) x[i] = *reinterpret_cast<const float4*>(src + (i * 32 + lane) * 4);
  } else {
#pragma unroll
    for (int i = 0; i < kVec; ++i) x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    // The codes first (independent loads), then each codebook's row loaded
    // while the previous one is added; the sum runs in codebook order.
    auto row_of = [&](int c) {
      int64_t code = ids[static_cast<int64_t>(c) * rows + row];
      if (code < 0 || code >= audio_vocab) {
        if (lane == 0) atomicOr(err, kErrBadArgument);
        code = 0;
      }
      return audio_table + (static_cast<int64_t>(c) * audio_vocab + code) * width;
    };
    constexpr int kPrefetch = 8;
    const float* srcs[kPrefetch];
#pragma unroll
    for (int c = 0; c < kPrefetch; ++c) srcs[c] = c < codebooks ? row_of(c) : nullptr;
    float4 cur[kVec], next[kVec];
    if (codebooks > 0) {
#pragma unroll
      for (int i = 0; i < kVec; ++i) cur[i] = *reinterpret_cast<const float4*>(srcs[0] + (i * 32 + lane) * 4);
    }
    auto step = [&](int c, const float* next_src) {
      if (next_src != nullptr) {
#pragma unroll
        for (int i = 0; i < kVec; ++i)
          next[i] = *reinterpret_cast<const float4*>(next_src + (i * 32 + lane) * 4);
      }
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        x[i].x += cur[i].x;
        x[i].y += cur[i].y;
        x[i].z += cur[i].z;
        x[i].w += cur[i].w;
        cur[i] = next[i];
      }
    };
#pragma unroll
    for (int c = 0; c < kPrefetch; ++c) {
      if (c >= codebooks) break;
      step(c, c + 1 >= codebooks ? nullptr : c + 1 < kPrefetch ? srcs[c + 1] : row_of(c + 1));
    }
    for (int c = kPrefetch; c < codebooks; ++c) step(c, c + 1 < codebooks ? row_of(c + 1) : nullptr);
  }
  float* dst = hidden + row * width;
#pragma unroll
  for (int i = 0; i < kVec; ++i) *reinterpret_cast<float4*>(dst + (i * 32 + lane) * 4) = x[i];
  if (norm_weight != nullptr) {
    const float scale = rms_scale(row_squares<kVec>(x), width, epsilon);
    norm_store_row<kVec>(x, norm_weight, normed + row * width, scale, lane);
  }
}

// generator_kernels.hip:85-97 (RmsNormKernel); with `indices` also
// :202-209 (GatherRowsKernel) in front of it.
template <int kVec>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    rmsnorm_kernel(const float* __restrict__ input, const int32_t* __restrict__ indices,
                   int64_t rows, const float* __restrict__ weight, __half* __restrict__ output,
                   float epsilon) {
  constexpr int width = 128 * kVec;
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t src_row = indices != nullptr ? static_cast<int64_t>(indices[row]) : row;
  const float* src = input + src_row * width;
  float4 x[kVec];
#pragma unroll
  for (int i = 0; i < kVec; ++i) x[i] = *reinterpret_cast<const float4*>(src + (i * 32 + lane) * 4);
  const float scale = rms_scale(row_squares<kVec>(x), width, epsilon);
  norm_store_row<kVec>(x, weight, output + row * width, scale, lane);
}

// One warp per (row, head slot); lane l owns d = l + 32 j, so the rotary
// pairs (d, d + 64) are lanes' own elements j and j + 2.
// generator_kernels.hip:102-159 (QkNormRopeKernel), without the GQA repeat.
__global__ void __launch_bounds__(256)
    qknorm_rope_kernel(const float* __restrict__ qkv, int64_t ld_in,
                       const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                       const int32_t* __restrict__ positions, const float* __restrict__ rope_cos,
                       const float* __restrict__ rope_sin, int max_positions, int64_t rows,
                       int heads, int kv_heads, float epsilon, __half* __restrict__ out,
                       int64_t ld_out, uint32_t* err) {
  const int slots = heads + 2 * kv_heads;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= rows * slots) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = item / slots;
  const int slot = static_cast<int>(item % slots);
  const float* in = qkv + row * ld_in + slot * 128;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = in[lane + 32 * j];
  __half* o = out + row * ld_out + slot * 128;
  if (slot < heads + kv_heads) {
    const float* w = slot < heads ? q_norm : k_norm;
    float s = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    s = warp_sum(s);
    const float scale = 1.0f / sqrtf(s / 128.0f + epsilon);
    int pos = positions[row];
    if (pos < 0 || pos >= max_positions) {
      if (lane == 0) atomicOr(err, kErrBadArgument);
      pos = 0;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;  // rotary pair (i, i + 64)
      const float a = w[i] * (v[j] * scale);
      const float b = w[i + 64] * (v[j + 2] * scale);
      const float c = rope_cos[static_cast<int64_t>(pos) * 64 + i];
      const float sn = rope_sin[static_cast<int64_t>(pos) * 64 + i];
      o[i] = __float2half_rn(a * c - b * sn);
      o[i + 64] = __float2half_rn(b * c + a * sn);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) o[lane + 32 * j] = __float2half_rn(v[j]);
  }
}

// generator_kernels.hip:191-200 (SwiGluKernel).
__global__ void swiglu_kernel(const float* __restrict__ gate_up, int64_t rows, int64_t width,
                              __half* __restrict__ out) {
  const int64_t total = rows * width;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / width;
    const int64_t c = i % width;
    const float g = gate_up[r * 2 * width + c];
    const float u = gate_up[r * 2 * width + width + c];
    out[i] = __float2half_rn(g / (1.0f + expf(-g)) * u);
  }
}

__global__ void synthetic_kernel(float* __restrict__ out, int64_t count, uint64_t base,
                                 float scale, uint64_t first) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = SyntheticValue(base, first + static_cast<uint64_t>(i), scale);
}

int Blocks(int64_t rows) { return static_cast<int>((rows + kRowsPerBlock - 1) / kRowsPerBlock); }

#define OV_VEC_DISPATCH(width, KERNEL_CALL)                 \
  switch ((width) / 128) {                                  \
    case 1: { constexpr int V = 1; KERNEL_CALL; break; }    \
    case 2: { constexpr int V = 2; KERNEL_CALL; break; }    \
    case 4: { constexpr int V = 4; KERNEL_CALL; break; }    \
    case 8: { constexpr int V = 8; KERNEL_CALL; break; }    \
    case 16: { constexpr int V = 16; KERNEL_CALL; break; }  \
    default: throw Error(OV_ERR_UNSUPPORTED, "row width must be 128, 256, 512, 1024 or 2048"); \
  }

}  // namespace

void LaunchEmbed(const float* text_table, size_t text_vocab, const int32_t* row_text_ids,
                 const float* audio_table, size_t audio_vocab, const int32_t* ids,
                 size_t codebooks, size_t rows, size_t width, float* hidden,
                 const float* norm_weight, float epsilon, uint16_t* normed,
                 cudaStream_t stream) {
  if (rows == 0) return;
  uint32_t* err = DeviceErrorWord();
  OV_VEC_DISPATCH(width, (Launch(embed_kernel<V>, dim3(Blocks(rows)), dim3(kRowsPerBlock * 32),
                                 0, stream, "embed kernel launch", text_table,
                                 static_cast<int64_t>(text_vocab), row_text_ids, audio_table,
                                 static_cast<int64_t>(audio_vocab), ids,
                                 static_cast<int>(codebooks), static_cast<int64_t>(rows), hidden,
                                 norm_weight, epsilon, reinterpret_cast<__half*>(normed), err)));
}

void LaunchRmsNorm(const float* input, const int32_t* indices, size_t rows,
                   const float* weight, uint16_t* output, size_t width, float epsilon,
                   cudaStream_t stream) {
  if (rows == 0) return;
  OV_VEC_DISPATCH(width, (Launch(rmsnorm_kernel<V>, dim3(Blocks(rows)), dim3(kRowsPerBlock * 32),
                                 0, stream, "rmsnorm kernel launch", input, indices,
                                 static_cast<int64_t>(rows), weight,
                                 reinterpret_cast<__half*>(output), epsilon)));
}

}  // namespace ovb

using namespace ovb;

extern "C" {

int ov_embed(const float* text_table, size_t text_vocab, const int32_t* row_text_ids,
             const float* audio_table, size_t audio_vocab, const int32_t* ids,
             size_t codebooks, size_t rows, size_t width, float* hidden,
             const float* norm_weight, float epsilon, uint16_t* normed, ov_stream_t stream) {
  return Guard("ov_embed: ", [&] {
    OV_REQUIRE(norm_weight == nullptr || normed != nullptr, "normed output missing");
    LaunchEmbed(text_table, text_vocab, row_text_ids, audio_table, audio_vocab, ids, codebooks,
                rows, width, hidden, norm_weight, epsilon, normed, AsStream(stream));
  });
}

int ov_rmsnorm(const float* input, const float* weight, uint16_t* output, size_t rows,
               size_t width, float epsilon, ov_stream_t stream) {
  return Guard("ov_rmsnorm: ", [&] {
    LaunchRmsNorm(input, nullptr, rows, weight, output, width, epsilon, AsStream(stream));
  });
}

int ov_gather_rmsnorm(const float* input, const int32_t* indices, size_t count,
                      const float* weight, uint16_t* output, size_t width, float epsilon,
                      ov_stream_t stream) {
  return Guard("ov_gather_rmsnorm: ", [&] {
    OV_REQUIRE(indices != nullptr, "indices missing");
    LaunchRmsNorm(input, indices, count, weight, output, width, epsilon, AsStream(stream));
  });
}

int ov_rope_tables(float theta, size_t head_dim, size_t max_positions, float* cos_table,
                   float* sin_table) {
  return Guard("ov_rope_tables: ", [&] {
    OV_REQUIRE(head_dim % 2 == 0 && head_dim > 0, "head_dim must be even");
    const size_t half = head_dim / 2;
    for (size_t i = 0; i < half; ++i) {
      const float inv_freq =
          1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
      for (size_t p = 0; p < max_positions; ++p) {
        const float angle = static_cast<float>(p) * inv_freq;
        cos_table[p * half + i] = std::cos(angle);
        sin_table[p * half + i] = std::sin(angle);
      }
    }
  });
}

int ov_qknorm_rope(const float* qkv, size_t ld_in, const float* q_norm, const float* k_norm,
                   const int32_t* positions, const float* rope_cos, const float* rope_sin,
                   size_t max_positions, size_t rows, size_t heads, size_t kv_heads,
                   size_t head_dim, float epsilon, uint16_t* output, size_t ld_out,
                   ov_stream_t stream) {
  return Guard("ov_qknorm_rope: ", [&] {
    OV_REQUIRE(head_dim == 128, "head_dim must be 128");
    if (rows == 0) return;
    const int64_t items = static_cast<int64_t>(rows) * static_cast<int64_t>(heads + 2 * kv_heads);
    qknorm_rope_kernel<<<static_cast<unsigned>((items + 7) / 8), 256, 0, AsStream(stream)>>>(
        qkv, static_cast<int64_t>(ld_in), q_norm, k_norm, positions, rope_cos, rope_sin,
        static_cast<int>(max_positions), static_cast<int64_t>(rows), static_cast<int>(heads),
        static_cast<int>(kv_heads), epsilon, reinterpret_cast<__half*>(output),
        static_cast<int64_t>(ld_out), DeviceErrorWord());
    Check(cudaGetLastError(), "qknorm_rope kernel launch");
  });
}

int ov_swiglu(const float* gate_up, size_t rows, size_t width, uint16_t* output,
              ov_stream_t stream) {
  return Guard("ov_swiglu: ", [&] {
    if (rows == 0 || width == 0) return;
    const int64_t total = static_cast<int64_t>(rows * width);
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    swiglu_kernel<<<blocks, 256, 0, AsStream(stream)>>>(gate_up, static_cast<int64_t>(rows),
                                                       static_cast<int64_t>(width),
                                                       reinterpret_cast<__half*>(output));
    Check(cudaGetLastError(), "swiglu kernel launch");
  });
}

int ov_synthetic_fill(float* output, size_t count, uint64_t seed, uint64_t tensor, float std,
                      uint64_t first_index, ov_stream_t stream) {
  return Guard("ov_synthetic_fill: ", [&] {
    if (count == 0) return;
    const int blocks = static_cast<int>(std::min<size_t>((count + 255) / 256, 148 * 32));
    synthetic_kernel<<<blocks, 256, 0, AsStream(stream)>>>(
        output, static_cast<int64_t>(count), SyntheticBase(seed, tensor), SyntheticScale(std),
        first_index);
    Check(cudaGetLastError(), "synthetic fill launch");
  });
}

int ov_synthetic_fill_host(float* output, size_t count, uint64_t seed, uint64_t tensor,
                           float std, uint64_t first_index) {
  return Guard("ov_synthetic_fill_host: ", [&] {
    const uint64_t base = SyntheticBase(seed, tensor);
    const float scale = SyntheticScale(std);
    for (size_t i = 0; i < count; ++i) output[i] = SyntheticValue(base, first_index + i, scale);
  });
}

}  // extern "C"
