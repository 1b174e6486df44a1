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
  int num_m = 0;    // 128-row tiles
  int num_n = 0;    // BN-column tiles
  int units = 0;    // num_m * num_n * splits work units
  int out_cols = 0; // columns of y (N, or N / 2 for SwiGLU)
  // Split-K order counters, one per tile: split s adds its partial into y
  // after splits 0..s-1 did, so the sum order is fixed.
  uint32_t* counters = nullptr;
  // 1: the splits of a tile run as one thread-block cluster (one unit per
  // CTA, split = rank in the cluster); rank r sums column slice r of the
  // splits' partials in split order.  The partials travel through `xchg`
  // (global memory, [tile][sender][slice][128 x BN / splits floats]) when
  // it is set, else through distributed shared memory; no counters.
  int cluster = 0;
  float* xchg = nullptr;
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
  CUtensorMap map_y;
  GemmArgs args;
  dim3 grid;
  int bn = 128;
  int epilogue = OV_EPI_STORE_F32;
  size_t smem_bytes = 0;
  unsigned cluster_x = 1;  // CTAs per thread-block cluster
  bool pair = false;       // 256-row tiles on CTA pairs (cta_group::2)
};

struct GemmShapeChoice {
  int bn;
  int splits;
  bool cluster = false;  // splits reduced inside a thread-block cluster
  bool pair = false;     // 256-row tiles on CTA pairs (cta_group::2 MMAs)
  bool xchg = false;     // cluster splits exchange partials through the workspace
};

// Tile width and split-K factor for a product of this shape on `sms` SMs.
// OV_GEMM_TILE=<bn>x<splits> (serialised split-K), <bn>c<splits> (cluster
// split-K) or <bn>p1 (CTA pairs) in the environment overrides the choice
// (tuning aid; ignored when the override is not valid for the product).
// OV_GEMM_XCHG=0 makes cluster split-K exchange its partials through
// distributed shared memory even when a workspace is given.
// allow_xchg false: with a workspace, only its order-counter use (serialised
// split-K) is considered, never the partial-slice exchange.
GemmShapeChoice ChooseGemmShape(int M, int N, int K, int epilogue, bool have_workspace, int sms,
                                bool allow_xchg = true);
// Workspace bytes a plan with this shape needs for split-K (0 if none):
// the order counters of serialised split-K or the partial slices of
// cluster split-K.
size_t GemmWorkspaceBytes(int M, int N, int K, int epilogue, int sms);

// Builds a plan.  `w_rows` is the number of rows of the (possibly stacked)
// weight tensor w points at and b_row_offset the first row this product
// uses, so one tensor map can cover all layers.  `err` is the word bounded
// waits report into (nullptr: the device error word of ov_take_device_errors).
void PlanGemm(GemmPlan* plan, const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t w_rows,
              int b_row_offset, void* y, int64_t ldy, int M, int N, int K, int epilogue,
              const ov_epilogue_args* epilogue_args, void* workspace, size_t workspace_bytes,
              int sms, uint32_t* err = nullptr, bool allow_xchg = true);

void LaunchGemm(const GemmPlan& plan, cudaStream_t stream);

}  // namespace ovb
