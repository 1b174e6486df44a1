// Bidirectional grouped-query attention over packed variable-length
// sequences on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-sequence attention (generator.cpp:122-172:
// a batched Q K^T GEMM into float32 scores [heads][L][L], SoftmaxKernel
// writing half probabilities, a batched P V GEMM and MergeHeadsKernel) with
// one flash-style kernel: scores never leave the SM.  The roles of a work
// item (softmax warpgroups, producer warp, MMA thread) are in
// attention_device.cuh; this kernel runs one work item per CTA:
//   attention_kernel<2>  320 threads: two softmax warpgroups (warps 0-7),
//                        producer warp 8, MMA warp 9; items of two query
//                        tiles (one per warpgroup) or one tile split in two;
//   attention_kernel<4>  576 threads: one query tile split over four
//                        softmax warpgroups (warps 0-15), producer warp 16,
//                        MMA warp 17.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "attention_device.cuh"
#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "ptx.cuh"

namespace ovb {
namespace {

// Softmax warpgroups per CTA: 2 (tile pairs, or one tile split in two
// key halves) or 4 (one tile split in four key quarters); plus a producer
// and an MMA warp.
constexpr int ThreadsOf(int wgs) { return 128 * wgs + 64; }
// Q0, Q1 | K, V ring of two stages | barriers, row-statistics exchange.
constexpr uint32_t kSmemBytes = 2 * kTile + 2 * 2 * kTile + 1024 + 8192;

template <int kWG>
__global__ void __launch_bounds__(ThreadsOf(kWG), 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_qkv,
                     const __grid_constant__ CUtensorMap map_out, const AttnArgs args) {
  constexpr int kProducerWarp = 4 * kWG;
  constexpr int kMmaWarp = 4 * kWG + 1;
  // The next kernel may start its prologue now; this one waits for its
  // inputs (q, k, v of the previous kernel) only after its own set-up.  The
  // work items and sequence bounds are uploaded before the step.
  pdl_trigger();
  int seq, tile, max_groups;
  if (args.items != nullptr) {
    // Work items: head blockIdx.x, item blockIdx.y, so the hardware starts
    // the items (longest first) in order across all heads.
    seq = args.items[2 * blockIdx.y];
    const int code = args.items[2 * blockIdx.y + 1];
    tile = code & 0xFFFFFF;
    max_groups = code >> 24;
  } else if (args.single) {
    seq = blockIdx.y;
    tile = blockIdx.x;
    max_groups = 1;
  } else {
    seq = blockIdx.y;
    tile = 2 * blockIdx.x;
    max_groups = 2;
  }
  if (kWG == 4) max_groups = 1;  // the four-warpgroup form takes single tiles only
  const int h = args.items != nullptr ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.z);
  const int start = args.cu_seqlens[seq];
  const int len = args.cu_seqlens[seq + 1] - start;
  const int q0 = tile * kQ;
  if (q0 >= len) return;  // uniform over the CTA, before any barrier
  const int groups = max_groups >= 2 && q0 + kQ < len ? 2 : 1;
  const int kvh = h / (args.heads / args.kv_heads);
  const int nt = (len + kKeys - 1) / kKeys;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;                  // [2 groups] x 32 KB
  uint8_t* k_s = q_s + 2 * kTile;       // [2 stages] x 32 KB
  uint8_t* v_s = k_s + 2 * kTile;       // [2 stages] x 32 KB
  uint64_t* bar_mem = reinterpret_cast<uint64_t*>(v_s + 2 * kTile);
  // K and V tiles have their own barriers: a K stage frees when its S
  // MMAs are done, well before the P V that frees the V stage, so the
  // next K tiles load ahead.
  AttnBars bars;
  bars.q_full = bar_mem;
  bars.k_full = bar_mem + 1;    // [2 stages]
  bars.k_empty = bar_mem + 3;   // [2]
  bars.v_full = bar_mem + 5;    // [2]
  bars.v_empty = bar_mem + 7;   // [2]
  bars.s_full = bar_mem + 9;    // [2 groups, or 2 S regions of one tile]
  bars.p_full = bar_mem + 11;   // [2]
  bars.o_done = bar_mem + 13;   // [2 groups]
  bars.pv_done = bar_mem + 15;  // one query tile: each P V complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mem + 16);
  float* xmax = reinterpret_cast<float*>(bar_mem + 18);  // [2 tiles][kWG warpgroups][128 rows]
  float* xsum = xmax + 2 * kWG * 128;                    // [kWG warpgroups][128 rows]
  const AttnPhase phase;  // fresh barriers: every phase count starts at 0

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    // One query tile: every softmax warpgroup arrives on p_full[i].
    InitAttnBars(bars, groups == 1 ? 128 * kWG : 128);
    fence_mbar_init();
    tma_prefetch_map(&map_qkv);
    tma_prefetch_map(&map_out);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, k, v of the previous kernel are complete

  if (warp == kProducerWarp) {
    AttnProduce(args, &map_qkv, bars, phase, q_s, k_s, v_s, lane, start, q0, groups, nt, h, kvh);
  } else if (warp == kMmaWarp) {
    if (lane == 0) (void)AttnIssue(args, tmem, bars, phase, q_s, k_s, v_s, groups, nt);
  } else if constexpr (kWG == 4) {
    SoftmaxRole<4>(args, &map_out, tmem, bars, phase, xmax, xsum, q_s, warp >> 2, warp & 3, lane,
                   len, nt, q0, start, h, 1, 1);
  } else {
    if (groups == 1)
      SoftmaxRole<2>(args, &map_out, tmem, bars, phase, xmax, xsum, q_s, warp >> 2, warp & 3,
                     lane, len, nt, q0, start, h, 1, 1);
    else
      SoftmaxRole<1>(args, &map_out, tmem, bars, phase, xmax, xsum, q_s, warp >> 2, warp & 3,
                     lane, len, nt, q0, start, h, 1, 1);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void ConfigureAttentionKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<2>),
                    static_cast<int>(kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<4>),
                    static_cast<int>(kSmemBytes));
}

// items: device [n_items][2] (sequence, first 128-query tile | max groups
// << 24); null to cover every sequence by tile pairs (ceil(max_seqlen /
// 256) per sequence) or, `single`, by single tiles (ceil(max_seqlen / 128)).
// single: every work item is one query tile, run by the four-warpgroup form.
void LaunchAttention(const CUtensorMap& map_qkv, const CUtensorMap& map_out,
                     const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                     const int32_t* items, int n_items, int heads, int kv_heads, float scale,
                     __half* out, int64_t ld_out, cudaStream_t stream, bool single) {
  if (num_seqs == 0 || max_seqlen == 0) return;
  AttnArgs a;
  a.cu_seqlens = cu_seqlens;
  a.items = items;
  a.out = out;
  a.ld_out = ld_out;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = DeviceErrorWord();
  a.single = single ? 1 : 0;
  const int per = single ? kQ : 2 * kQ;
  if (items != nullptr && n_items > 65535)
    throw Error(OV_ERR_UNSUPPORTED, "more than 65535 attention work items");
  const dim3 grid = items != nullptr
                        ? dim3(static_cast<unsigned>(heads), static_cast<unsigned>(n_items), 1)
                        : dim3(static_cast<unsigned>((max_seqlen + per - 1) / per),
                               static_cast<unsigned>(num_seqs), static_cast<unsigned>(heads));
  if (single) {
    SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<4>),
                      static_cast<int>(kSmemBytes));
    Launch(attention_kernel<4>, grid, dim3(ThreadsOf(4)), kSmemBytes, stream,
           "attention kernel launch", map_qkv, map_out, a);
  } else {
    SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<2>),
                      static_cast<int>(kSmemBytes));
    Launch(attention_kernel<2>, grid, dim3(ThreadsOf(2)), kSmemBytes, stream,
           "attention kernel launch", map_qkv, map_out, a);
  }
}

void EncodeAttnOutMap(CUtensorMap* map, const uint16_t* out, int64_t ld_out, int64_t rows,
                      int64_t width) {
  EncodeTensorMap2D(map, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<uint64_t>(width),
                    static_cast<uint64_t>(rows), static_cast<uint64_t>(ld_out) * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

void EncodeQkvMap(CUtensorMap* map, const uint16_t* qkv, int64_t ld_qkv, int64_t rows,
                  int64_t width) {
  EncodeTensorMap2D(map, qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<uint64_t>(width),
                    static_cast<uint64_t>(rows), static_cast<uint64_t>(ld_qkv) * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace ovb

using namespace ovb;


extern "C" int ov_attention_varlen(const uint16_t* qkv, size_t ld_qkv, size_t rows,
                                   const int32_t* cu_seqlens, size_t num_seqs,
                                   size_t max_seqlen, size_t heads, size_t kv_heads,
                                   size_t head_dim, float scale, uint16_t* out, size_t ld_out,
                                   ov_stream_t stream) {
  return Guard("ov_attention_varlen: ", [&] {
    OV_REQUIRE(head_dim == 128, "head_dim must be 128");
    OV_REQUIRE(kv_heads > 0 && heads % kv_heads == 0, "heads must be a multiple of kv_heads");
    OV_REQUIRE(ld_qkv % 8 == 0 && ld_qkv >= (heads + 2 * kv_heads) * head_dim, "qkv stride");
    OV_REQUIRE(ld_out % 8 == 0 && ld_out >= heads * head_dim, "out stride");
    if (rows == 0 || num_seqs == 0) return;
    OV_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0, "out must be 16-byte aligned");
    CUtensorMap map, map_out;
    EncodeQkvMap(&map, qkv, static_cast<int64_t>(ld_qkv), static_cast<int64_t>(rows),
                 static_cast<int64_t>((heads + 2 * kv_heads) * head_dim));
    EncodeAttnOutMap(&map_out, out, static_cast<int64_t>(ld_out), static_cast<int64_t>(rows),
                     static_cast<int64_t>(heads * head_dim));
    // Single query tiles (four softmax warpgroups each) when one tile per
    // CTA still fits the GPU in one wave, else tile pairs; OV_ATTN_FORM =
    // single | pair in the environment overrides (tuning and test aid).
    const size_t tiles = (max_seqlen + 127) / 128 * num_seqs * heads;
    bool single = tiles <= static_cast<size_t>(SmCount());
    if (const char* env = std::getenv("OV_ATTN_FORM")) {
      if (std::strcmp(env, "single") == 0) single = true;
      if (std::strcmp(env, "pair") == 0) single = false;
    }
    LaunchAttention(map, map_out, cu_seqlens, static_cast<int>(num_seqs), static_cast<int>(max_seqlen),
                    nullptr, 0, static_cast<int>(heads), static_cast<int>(kv_heads), scale,
                    reinterpret_cast<__half*>(out), static_cast<int64_t>(ld_out),
                    AsStream(stream), single);
  });
}
