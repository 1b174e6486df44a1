// Row RMSNorm arithmetic of the norm kernels (elementwise.cu): one warp per
// row of 128 * kVec floats, lane l holding float4 vectors l, l + 32, ...;
// the row's sum of squares is each lane's sum in vector order, then a
// butterfly over the warp (generator_kernels.hip:85-97).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ptx.cuh"

namespace ovb {
namespace {

// Sum of squares -> 1 / sqrt(mean + eps), IEEE sqrt and division so the
// host oracle can evaluate the same expression.
__device__ __forceinline__ float rms_scale(float squares, int width, float epsilon) {
  return 1.0f / sqrtf(squares / static_cast<float>(width) + epsilon);
}

template <int kVec>  // float4 vectors per lane; width = 128 * kVec
__device__ __forceinline__ void norm_store_row(const float4 (&x)[kVec], const float* weight,
                                               __half* out, float scale, int lane) {
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int col = (i * 32 + lane) * 4;
    const float4 w = *reinterpret_cast<const float4*>(weight + col);
    uint2 packed;
    packed.x = pack_half2(w.x * (x[i].x * scale), w.y * (x[i].y * scale));
    packed.y = pack_half2(w.z * (x[i].z * scale), w.w * (x[i].w * scale));
    *reinterpret_cast<uint2*>(out + col) = packed;
  }
}

template <int kVec>
__device__ __forceinline__ float row_squares(const float4 (&x)[kVec]) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    s += x[i].x * x[i].x;
    s += x[i].y * x[i].y;
    s += x[i].z * x[i].z;
    s += x[i].w * x[i].w;
  }
  return warp_sum(s);
}

}  // namespace
}  // namespace ovb
