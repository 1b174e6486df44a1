// Host interface of the persistent layer kernel (layers.cu): the whole
// stack of decoder layers of one forward pass as one launch of one CTA per
// SM, each CTA working through a fixed share of a dependency-ordered task
// list (norm row chunks, GEMM output tiles, attention items).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

namespace ovb {

// Task kinds, in the order of a layer (also the counter stage index).
enum LayerTaskKind : uint8_t {
  kTaskNorm1 = 0,  // input RMSNorm of a row chunk (layers >= 1)
  kTaskQkv = 1,    // QKV output tile + QK-norm + RoPE
  kTaskAttn = 2,   // attention item (sequence, 1-2 query tiles, head)
  kTaskO = 3,      // o-projection tile split (+ residual)
  kTaskNorm2 = 4,  // post-attention RMSNorm of a row chunk
  kTaskGateUp = 5, // gate/up tile + SwiGLU
  kTaskDown = 6,   // down-projection tile split (+ residual)
  kTaskKinds = 7
};

// One task (32 bytes).  Counters are per (layer, kind, 128-row block m):
// a task waits until counter[wait_layer][wait_kind][m] >=
// target[wait_kind][m] for every m in [wait_lo, wait_hi] (none when
// wait_kind < 0), and adds 1 to counter[layer][kind][m] for m in
// [sig_lo, sig_hi] when its output is complete.
struct LayerTask {
  uint8_t kind;
  uint8_t layer;
  uint8_t split;     // GEMM split-K part; attention: query tiles (1 or 2)
  uint8_t splits;    // GEMM split-K parts
  int16_t m;         // GEMM: 128-row tile; norm: row block; attention: sequence
  int16_t n;         // GEMM: 256-column tile; attention: query head
  int8_t wait_kind;
  uint8_t wait_layer;
  int16_t wait_lo, wait_hi;
  int16_t sig_lo, sig_hi;
  int16_t pad1;
  int32_t row0;      // norm: first row; attention: first query row in the sequence
  int32_t rows;      // norm: rows of the chunk
  int32_t pad2;
};
static_assert(sizeof(LayerTask) == 32, "task layout");

struct LayerKernelParams {
  // Activations (A operands and outputs), 128B-swizzled boxes of 64 halves
  // (or 32 floats) x 128 rows.
  CUtensorMap map_normed;   // [R][H] half: A of QKV and gate/up
  CUtensorMap map_attn;     // [R][QH] half: attention output, A of o
  CUtensorMap map_act;      // [R][I] half: SwiGLU output, A of down
  CUtensorMap map_qkv[2];   // [R][QKVW] half, per layer parity: QKV output, attention input
  CUtensorMap map_hidden;   // [R][H] float32: residual stream (o / down reduce-add)
  // Weights stacked over layers, boxes of 64 halves x 256 rows.
  CUtensorMap map_w_qkv, map_w_o, map_w_gu, map_w_down;

  const LayerTask* tasks;
  int ntasks;
  int num_m;                // 128-row blocks
  uint32_t* counters;       // [layers][kTaskKinds][num_m], zero at launch
  const int32_t* targets;   // [kTaskKinds][num_m]
  uint32_t* xchg_counters;  // [layers][2][tiles], zero at launch
  float* xchg;              // split-K partial slices, [tile][splits][splits][128 x 256 / splits]
  uint32_t* abort;          // set by the first CTA that gives up; every wait then returns
  uint32_t* err;

  float* hidden;            // [R][H]
  uint16_t* normed;         // [R][H]
  uint16_t* qkv[2];         // [R][QKVW], even / odd layers
  uint16_t* act;            // [R][I]
  const float* norms;       // [layers][2H + 2D]: input, post-attention, q, k norm weights
  const int32_t* positions; // [R]
  const float* rope_cos;
  const float* rope_sin;
  int max_positions;
  const int32_t* cu_seqlens;
  uint16_t* attn_out;       // [R][QH]
  float scale_log2;
  float epsilon;
  int rows, hidden_size, heads, kv_heads, intermediate;
  int layers;
  int o_splits, down_splits;
};

// Builds the task list and the per-(kind, row block) targets of a packed
// batch: rows R, sequences given by cu_seqlens (host, n_seqs + 1 entries).
// o_splits / down_splits: split-K parts of the two residual products.
void BuildLayerTasks(int layers, int rows, int hidden, int heads, int kv_heads, int intermediate,
                     const std::vector<int32_t>& cu_seqlens, int o_splits, int down_splits,
                     std::vector<LayerTask>* tasks, std::vector<int32_t>* targets);

// Whether the layer kernel supports this model shape (head_dim 128; hidden,
// QKV width, 2 x intermediate and heads x 128 multiples of 256; hidden a
// multiple of 128 up to 1024 per norm row).
bool LayerKernelSupports(int hidden, int heads, int kv_heads, int head_dim, int intermediate);

// Split-K parts for a residual product of K input features.
int LayerKernelSplits(int k);

// Grid size (CTAs resident at once, one per SM) on the current device.
int LayerKernelGrid();

void ConfigureLayerKernel();
void LaunchLayerKernel(const LayerKernelParams& params, int grid, cudaStream_t stream);

}  // namespace ovb
