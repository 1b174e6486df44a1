// General strided-batched half-precision product in the column-major BLAS
// convention of the reference's HalfGemm::Matmul (gemm.hpp:16-36,56-57):
// C[m][n] (+)= op(A)[m][k] * op(B)[k][n], fp16 operands, fp32 accumulation
// and output.  The generator's hot path does not use it (its products go
// through the tcgen05 GEMM of gemm.cu); it keeps the reference's API for
// callers and for the shapes the tiled kernel does not take (K not a
// multiple of 64, unaligned strides).  One 32 x 32 tile of C per CTA,
// k in steps of 32 through shared memory, fp32 FMA.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"

namespace ovb {
namespace {

constexpr int kTile = 32;

__global__ void __launch_bounds__(256) matmul_kernel(ov_matmul_shape s, const __half* a,
                                                     const __half* b, float* c) {
  __shared__ float as[kTile][kTile + 1];  // [i][l]
  __shared__ float bs[kTile][kTile + 1];  // [l][j]
  const int64_t batch = blockIdx.z;
  a += batch * s.stride_a;
  b += batch * s.stride_b;
  c += batch * s.stride_c;
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kTile;
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * kTile;
  const int tx = threadIdx.x & 31;   // column within the loaded tile
  const int ty = threadIdx.x >> 5;   // 0..7
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t l0 = 0; l0 < static_cast<int64_t>(s.k); l0 += kTile) {
    // op(A)(i, l): A is stored column-major; transposed means A holds k x m.
    for (int r = ty; r < kTile; r += 8) {
      const int64_t i = i0 + r, l = l0 + tx;
      float v = 0.f;
      if (i < static_cast<int64_t>(s.m) && l < static_cast<int64_t>(s.k))
        v = __half2float(s.transpose_a ? a[l + i * static_cast<int64_t>(s.lda)]
                                       : a[i + l * static_cast<int64_t>(s.lda)]);
      as[r][tx] = v;
      const int64_t lb = l0 + r, j = j0 + tx;
      float w = 0.f;
      if (lb < static_cast<int64_t>(s.k) && j < static_cast<int64_t>(s.n))
        w = __half2float(s.transpose_b ? b[j + lb * static_cast<int64_t>(s.ldb)]
                                       : b[lb + j * static_cast<int64_t>(s.ldb)]);
      bs[r][tx] = w;
    }
    __syncthreads();
#pragma unroll 8
    for (int l = 0; l < kTile; ++l) {
      const float bv = bs[l][tx];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf(as[ty + 8 * q][l], bv, acc[q]);
    }
    __syncthreads();
  }
  const int64_t j = j0 + tx;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t i = i0 + ty + 8 * q;
    if (i < static_cast<int64_t>(s.m) && j < static_cast<int64_t>(s.n)) {
      float* dst = c + i + j * static_cast<int64_t>(s.ldc);
      *dst = s.accumulate ? *dst + acc[q] : acc[q];
    }
  }
}

}  // namespace
}  // namespace ovb

using namespace ovb;

extern "C" int ov_matmul_f16(const ov_matmul_shape* shape, const uint16_t* a, const uint16_t* b,
                             float* c, ov_stream_t stream) {
  return Guard("ov_matmul_f16: ", [&] {
    OV_REQUIRE(shape != nullptr, "shape missing");
    const ov_matmul_shape& s = *shape;
    if (s.m == 0 || s.n == 0 || s.batch == 0) return;
    OV_REQUIRE(s.ldc >= s.m, "ldc < m");
    OV_REQUIRE(s.lda >= (s.transpose_a ? s.k : s.m) || s.k == 0, "lda too small");
    OV_REQUIRE(s.ldb >= (s.transpose_b ? s.n : s.k) || s.k == 0, "ldb too small");
    OV_REQUIRE(s.batch < 65536 && s.m < (size_t{1} << 31) && s.n < (size_t{1} << 31),
               "shape too large");
    const dim3 grid(static_cast<unsigned>((s.m + kTile - 1) / kTile),
                    static_cast<unsigned>((s.n + kTile - 1) / kTile),
                    static_cast<unsigned>(s.batch));
    OV_REQUIRE(grid.y < 65536, "n too large");
    Launch(matmul_kernel, grid, dim3(256), 0, AsStream(stream), "matmul kernel launch", s,
           reinterpret_cast<const __half*>(a), reinterpret_cast<const __half*>(b), c);
  });
}
