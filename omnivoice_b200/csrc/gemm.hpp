// Host interface of the tcgen05 GEMM (gemm.cu): a plan holds the TMA
// tensor maps and launch shape of one product so the generator can build
// plans once per packed-batch shape and replay them inside a CUDA graph.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "ov_kernels.h"

namespace ovb {

struct GemmArgs {
  int M = 0;        // rows of x and y
  int N = 0;        // output features (rows of w)
  int K = 0;        // input features
  int kblocks = 0;  // K / 64
  int splits = 1;   // split-K factor (OV_EPI_ACCUM_F32 only)
  int b_row_offset = 0;
  int64_t ldy = 0;  // y row stride in elements of the output type
  void* y = nullptr;
  float* partials = nullptr;     // split-K partial tiles
  uint32_t* counters = nullptr;  // split-K arrival counters, one per tile
  // OV_EPI_QKNORM_ROPE_F16
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  const int32_t* positions = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int max_positions = 0;
  int heads = 0;
  int kv_heads = 0;
  float epsilon = 0.0f;
  uint32_t* err = nullptr;
};

struct GemmPlan {
  CUtensorMap map_a;
  CUtensorMap map_b;
  GemmArgs args;
  dim3 grid;
  int bn = 128;
  int epilogue = OV_EPI_STORE_F32;
  size_t smem_bytes = 0;
};

struct GemmShapeChoice {
  int bn;
  int splits;
};

// Tile width and split-K factor for a product of this shape on `sms` SMs.
GemmShapeChoice ChooseGemmShape(int M, int N, int K, int epilogue, bool have_workspace, int sms);
// Workspace bytes a plan with this shape needs for split-K (0 if none).
size_t GemmWorkspaceBytes(int M, int N, int K, int epilogue, int sms);

// Builds a plan.  `w_rows` is the number of rows of the (possibly stacked)
// weight tensor w points at and b_row_offset the first row this product
// uses, so one tensor map can cover all layers.
// `err` is the word bounded waits report into (nullptr: the device error
// word of ov_take_device_errors).
void PlanGemm(GemmPlan* plan, const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t w_rows,
              int b_row_offset, void* y, int64_t ldy, int M, int N, int K, int epilogue,
              const ov_epilogue_args* epilogue_args, void* workspace, size_t workspace_bytes,
              int sms, uint32_t* err = nullptr);

void LaunchGemm(const GemmPlan& plan, cudaStream_t stream);

}  // namespace ovb
