// The decoder layer stack of one forward pass as one persistent kernel.
//
// Replaces the 7 launches per layer of the per-kernel step (RMSNorm, QKV +
// QK-norm + RoPE, attention, o-proj + residual, RMSNorm, gate/up + SwiGLU,
// down + residual; generator.cpp:262-294) for batches of a few thousand
// rows, where every launch's fixed cost (first operand loads after the
// wait for the previous grid, the last tile's epilogue, the grid's drain)
// is as long as its k loop.  Here one CTA per SM stays resident for the
// whole stack and works through its share of a task list ordered so that
// every task depends only on earlier ones:
//   norm chunks (32 rows), GEMM output tiles of 128 x 256 (the residual
//   products split along K, the splits exchanging partial slices through a
//   global workspace and each adding one column slice, in split order),
//   attention items (sequence, 1-2 query tiles, head).
// Task t runs on CTA t % gridDim.x.  Dependencies are counters per (layer,
// task kind, 128-row block) in global memory: a task's producer (or, for a
// norm chunk, its worker warps) waits with acquire loads until the row
// blocks it reads are complete, and a finished task adds 1 with a release
// after its writes are complete.  Every wait is bounded; the first CTA that
// gives up sets the abort word and every other wait then returns at once.
//
// Roles (320 threads), the same for every task kind:
//   warp 0   producer: TMA loads of a GEMM tile's k blocks into a 4-stage
//            ring (the weight tiles of the first stages before the
//            dependency wait), or an attention item's Q, K and V;
//   warp 1   tensor-memory owner (all 512 columns) and MMA issuer: two
//            accumulator buffers of 256 columns for GEMM tiles, or all of
//            tensor memory for an attention item;
//   warps 2-9  workers: the GEMM epilogues (gemm_device.cuh), the
//            attention softmax (attention_device.cuh), the norm rows
//            (norm_device.cuh).
// A CTA's roles run ahead of one another across tasks (the producer loads
// the next tile while the workers finish the previous epilogue) exactly as
// within the persistent GEMM kernel.  An attention item takes the whole
// operand ring and both accumulator buffers; the ring goes back to the
// producer once the item's output, staged in its query tiles, is stored.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "attention_device.cuh"
#include "gemm_device.cuh"
#include "internal.hpp"
#include "launch.hpp"
#include "layers.hpp"
#include "norm_device.cuh"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kLBN = 256;                 // GEMM tile width
constexpr int kLStages = kRingBytes / (kBM * kBK * 2 + kLBN * kBK * 2);  // 4
constexpr uint32_t kLABytes = kBM * kBK * 2;
constexpr uint32_t kLBBytes = kLBN * kBK * 2;
constexpr uint32_t kLStageBytes = kLABytes + kLBBytes;
constexpr int kNormRows = 16;             // rows of a norm task (8 warps x 2, loaded together)
constexpr uint32_t kAttnBarBase = 4;      // named barriers 4-6 (GEMM epilogues use 1-3)
static_assert(kLStages == 4, "ring of four 48 KB stages");

// Dynamic shared memory: ring | staging (2 x 16 KB); the barriers, the
// QK-norm weights and two words are static shared memory, whose addresses
// are constants (no registers hold them across the task loop).
constexpr size_t kLSmemBytes = kRingBytes + 2 * kStageTile + 1024;
static_assert(kLSmemBytes + 32 * 8 + 256 * 4 + 16 <= 232448, "shared memory budget");

__shared__ uint64_t s_bars[32];
__shared__ float s_norm_w[256];
__shared__ uint32_t s_words[4];  // tensor-memory base, abort decision

struct Bars {
  uint64_t* full;         // [4] ring stage filled
  uint64_t* empty;        // [4] ring stage consumed
  uint64_t* tfull;        // [2] accumulator buffer ready
  uint64_t* tempty;       // [2] accumulator buffer read (256 worker arrivals)
  uint64_t* ring_release; // attention output stored from the query tiles (256 arrivals)
  uint64_t* mma_done;     // every MMA of the CTA complete (teardown)
  AttnBars attn;
};

__device__ __forceinline__ bool Aborted(const LayerKernelParams& p) {
  return *reinterpret_cast<volatile const uint32_t*>(p.abort) != 0;
}

__device__ __forceinline__ void GiveUp(const LayerKernelParams& p) {
  atomicOr(p.err, kErrWaitTimeout);
  atomicExch(p.abort, 1u);
}

// mbarrier wait bounded by kWaitLimitNs that also returns (false) once any
// CTA has aborted.
__device__ __forceinline__ bool BarWait(uint64_t* bar, uint32_t parity, const LayerKernelParams& p) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63) {
      if (Aborted(p)) return false;
      if (global_timer_ns() - start > kWaitLimitNs) {
        GiveUp(p);
        return false;
      }
    }
  }
}

// Waits until *c >= target, then acquires.  Polls with relaxed loads: an
// acquire per poll would invalidate the SM's L1 each time, under the feet
// of the other warps of the CTA (their register spills live there).
__device__ __forceinline__ bool CounterWait(const uint32_t* c, uint32_t target,
                                            const LayerKernelParams& p) {
  if (ld_relaxed_gpu(c) < target) {
    const uint64_t start = global_timer_ns();
    while (true) {
      __nanosleep(64);
      if (ld_relaxed_gpu(c) >= target) break;
      if (Aborted(p)) return false;
      if (global_timer_ns() - start > kWaitLimitNs) {
        GiveUp(p);
        return false;
      }
    }
  }
  fence_acq_rel_gpu();
  return true;
}

__device__ __forceinline__ uint32_t* Counter(const LayerKernelParams& p, int layer, int kind, int m) {
  return p.counters + (static_cast<size_t>(layer) * kTaskKinds + kind) * p.num_m + m;
}

// The task's inputs are complete (its dependency range reached its targets).
__device__ __forceinline__ bool WaitDeps(const LayerKernelParams& p, const LayerTask& t) {
  if (t.wait_kind < 0) return true;
  const int32_t* target = p.targets + t.wait_kind * p.num_m;
  for (int m = t.wait_lo; m <= t.wait_hi; ++m)
    if (!CounterWait(Counter(p, t.wait_layer, t.wait_kind, m), static_cast<uint32_t>(target[m]), p))
      return false;
  return true;
}

// Called by one thread after a CTA barrier that followed every worker's
// writes of the task: the fence is cumulative over the writes the barrier
// ordered before it, and the release add publishes them.
__device__ __forceinline__ void Signal(const LayerKernelParams& p, const LayerTask& t) {
  fence_acq_rel_gpu();
  for (int m = t.sig_lo; m <= t.sig_hi; ++m) red_release_gpu_add(Counter(p, t.layer, t.kind, m), 1u);
}

// A GEMM task's operands and shape.
struct TileShape {
  const CUtensorMap* a;
  const CUtensorMap* b;
  const CUtensorMap* y;
  int kblocks;  // of the whole product
  int b_row;    // first weight row of the tile
  int n_tiles;  // 256-column tiles of the product
};

__device__ __forceinline__ TileShape ShapeOf(const LayerKernelParams& p, const LayerTask& t) {
  const int H = p.hidden_size, QH = p.heads * kD, I = p.intermediate;
  const int QKVW = (p.heads + 2 * p.kv_heads) * kD;
  TileShape s;
  switch (t.kind) {
    case kTaskQkv:
      s = {&p.map_normed, &p.map_w_qkv, &p.map_qkv[t.layer & 1], H / kBK, t.layer * QKVW, QKVW / kLBN};
      break;
    case kTaskO:
      s = {&p.map_attn, &p.map_w_o, &p.map_hidden, QH / kBK, t.layer * H, H / kLBN};
      break;
    case kTaskGateUp:
      s = {&p.map_normed, &p.map_w_gu, &p.map_act, H / kBK, t.layer * 2 * I, 2 * I / kLBN};
      break;
    default:  // kTaskDown
      s = {&p.map_act, &p.map_w_down, &p.map_hidden, I / kBK, t.layer * H, H / kLBN};
      break;
  }
  s.b_row += t.n * kLBN;
  return s;
}

__device__ __forceinline__ void SplitRange(const LayerTask& t, int kblocks, int& kb0, int& kb1) {
  kb0 = t.split * kblocks / t.splits;
  kb1 = (t.split + 1) * kblocks / t.splits;
}

// Epilogue arguments of a GEMM task (gemm_device.cuh reads these fields).
__device__ __forceinline__ GemmArgs EpilogueArgs(const LayerKernelParams& p, const LayerTask& t) {
  GemmArgs a{};
  a.M = p.rows;
  a.splits = t.splits;
  a.num_n = ShapeOf(p, t).n_tiles;
  a.out_cols = t.kind == kTaskGateUp ? p.intermediate : t.kind == kTaskQkv
                                                            ? (p.heads + 2 * p.kv_heads) * kD
                                                            : p.hidden_size;
  a.xchg = p.xchg;
  a.positions = p.positions;
  a.rope_cos = p.rope_cos;
  a.rope_sin = p.rope_sin;
  a.max_positions = p.max_positions;
  a.heads = p.heads;
  a.kv_heads = p.kv_heads;
  a.epsilon = p.epsilon;
  a.err = p.err;
  return a;
}

__device__ __forceinline__ AttnArgs AttentionArgs(const LayerKernelParams& p) {
  AttnArgs a{};
  a.cu_seqlens = p.cu_seqlens;
  a.items = nullptr;
  a.out = reinterpret_cast<__half*>(p.attn_out);
  a.ld_out = p.heads * kD;
  a.heads = p.heads;
  a.kv_heads = p.kv_heads;
  a.scale_log2 = p.scale_log2;
  a.err = p.err;
  a.single = 0;
  return a;
}

// ------------------------------------------------------------ producer

__device__ void ProducerRole(const LayerKernelParams& p, uint8_t* ring, const Bars& b) {
  const int lane = threadIdx.x & 31;
  uint8_t* sa = ring;
  uint8_t* sb = ring + kLStages * kLABytes;
  uint32_t k_iter = 0;  // ring positions filled so far
  AttnPhase aph;
  const AttnArgs aargs = AttentionArgs(p);
  bool ok = true;
  for (int ti = blockIdx.x; ok && ti < p.ntasks; ti += gridDim.x) {
    const LayerTask t = p.tasks[ti];
    if (t.kind == kTaskNorm1 || t.kind == kTaskNorm2) continue;
    if (t.kind == kTaskAttn) {
      // The item takes the whole ring: its four stages, in ring order.
      if (lane == 0) {
        for (int i = 0; ok && i < kLStages; ++i, ++k_iter) {
          const int s = static_cast<int>(k_iter % kLStages);
          if (k_iter >= static_cast<uint32_t>(kLStages))
            ok = BarWait(&b.empty[s], ((k_iter / kLStages) - 1) & 1u, p);
          if (ok) mbar_arrive(&b.full[s]);
        }
        ok = ok && WaitDeps(p, t);
        fence_proxy_async_global();  // the TMA loads below see the waited-for writes
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const int start = p.cu_seqlens[t.m];
      const int len = p.cu_seqlens[t.m + 1] - start;
      const int nt = (len + kKeys - 1) / kKeys;
      const int h = t.n;
      const int kvh = h / (p.heads / p.kv_heads);
      AttnProduce(aargs, &p.map_qkv[t.layer & 1], b.attn, aph, ring, ring + 2 * kTile,
                  ring + 4 * kTile, lane, start, t.row0, t.split, nt, h, kvh);
      aph.Advance(nt, t.split);
      __syncwarp();
      continue;
    }
    if (lane == 0) {
      const TileShape sh = ShapeOf(p, t);
      int kb0, kb1;
      SplitRange(t, sh.kblocks, kb0, kb1);
      const int a_row = t.m * kBM;
      const int pre = min(kLStages, kb1 - kb0);
      // The weight tiles of the first stages depend on nothing.
      for (int i = 0; ok && i < pre; ++i) {
        const uint32_t pos = k_iter + i;
        const int s = static_cast<int>(pos % kLStages);
        if (pos >= static_cast<uint32_t>(kLStages))
          ok = BarWait(&b.empty[s], ((pos / kLStages) - 1) & 1u, p);
        if (!ok) break;
        mbar_arrive_expect_tx(&b.full[s], kLStageBytes);
        tma_load_2d(sb + s * kLBBytes, sh.b, &b.full[s], (kb0 + i) * kBK, sh.b_row);
      }
      ok = ok && WaitDeps(p, t);
      fence_proxy_async_global();
      for (int kb = kb0; ok && kb < kb1; ++kb, ++k_iter) {
        const int s = static_cast<int>(k_iter % kLStages);
        if (kb - kb0 < pre) {
          tma_load_2d(sa + s * kLABytes, sh.a, &b.full[s], kb * kBK, a_row);
          continue;
        }
        if (k_iter >= static_cast<uint32_t>(kLStages) &&
            !(ok = BarWait(&b.empty[s], ((k_iter / kLStages) - 1) & 1u, p)))
          break;
        mbar_arrive_expect_tx(&b.full[s], kLStageBytes);
        tma_load_2d(sa + s * kLABytes, sh.a, &b.full[s], kb * kBK, a_row);
        tma_load_2d(sb + s * kLBBytes, sh.b, &b.full[s], kb * kBK, sh.b_row);
      }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
  }
  // Let the copies this thread started land before the CTA can exit.
  if (lane == 0) {
    const uint32_t first = k_iter > static_cast<uint32_t>(kLStages) ? k_iter - kLStages : 0u;
    for (uint32_t i = first; i < k_iter; ++i)
      (void)mbar_wait(&b.full[i % kLStages], (i / kLStages) & 1u, p.err);
  }
}

// ----------------------------------------------------------------- MMA

__device__ void MmaRole(const LayerKernelParams& p, uint8_t* ring, const Bars& b, uint32_t tmem) {
  uint8_t* sa = ring;
  uint8_t* sb = ring + kLStages * kLABytes;
  constexpr uint32_t idesc = idesc_f16_f32(kBM, kLBN);
  uint32_t k_iter = 0;
  int acc_iter = 0;
  uint32_t releases = 0;
  AttnPhase aph;
  const AttnArgs aargs = AttentionArgs(p);
  bool ok = true;
  auto acquire_buffer = [&](int it) {
    return it < 2 || BarWait(&b.tempty[it & 1], static_cast<uint32_t>((it >> 1) - 1) & 1u, p);
  };
  for (int ti = blockIdx.x; ok && ti < p.ntasks; ti += gridDim.x) {
    const LayerTask t = p.tasks[ti];
    if (t.kind == kTaskNorm1 || t.kind == kTaskNorm2) continue;
    if (t.kind == kTaskAttn) {
      ok = acquire_buffer(acc_iter) && acquire_buffer(acc_iter + 1);
      for (int i = 0; ok && i < kLStages; ++i)
        ok = BarWait(&b.full[(k_iter + i) % kLStages], ((k_iter + i) / kLStages) & 1u, p);
      if (!ok) break;
      tc_fence_after_sync();
      const int len = p.cu_seqlens[t.m + 1] - p.cu_seqlens[t.m];
      const int nt = (len + kKeys - 1) / kKeys;
      ok = AttnIssue(aargs, tmem, b.attn, aph, ring, ring + 2 * kTile, ring + 4 * kTile, t.split, nt);
      if (!ok) {
        GiveUp(p);
        break;
      }
      aph.Advance(nt, t.split);
      // Both accumulator buffers were used: their "ready" phases advance.
      umma_commit(&b.tfull[acc_iter & 1]);
      umma_commit(&b.tfull[(acc_iter + 1) & 1]);
      acc_iter += 2;
      // The ring returns once the output staged in the query tiles is stored.
      ok = BarWait(b.ring_release, releases & 1u, p);
      ++releases;
      for (int i = 0; i < kLStages; ++i, ++k_iter) mbar_arrive(&b.empty[k_iter % kLStages]);
      continue;
    }
    const TileShape sh = ShapeOf(p, t);
    int kb0, kb1;
    SplitRange(t, sh.kblocks, kb0, kb1);
    const int buf = acc_iter & 1;
    if (!(ok = acquire_buffer(acc_iter))) break;
    tc_fence_after_sync();
    const uint32_t d = tmem + static_cast<uint32_t>(buf * kLBN);
    for (int kb = kb0; kb < kb1; ++kb, ++k_iter) {
      const int s = static_cast<int>(k_iter % kLStages);
      if (!(ok = BarWait(&b.full[s], (k_iter / kLStages) & 1u, p))) break;
      tc_fence_after_sync();
      const uint32_t a0 = smem_u32(sa + s * kLABytes);
      const uint32_t b0 = smem_u32(sb + s * kLBBytes);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        umma_f16_ss(d, smem_desc_sw128(a0 + k * 32, 16, 1024), smem_desc_sw128(b0 + k * 32, 16, 1024),
                    idesc, (kb > kb0 || k > 0) ? 1u : 0u);
      umma_commit(&b.empty[s]);
    }
    if (!ok) break;
    umma_commit(&b.tfull[buf]);
    ++acc_iter;
  }
  // No MMA may be in flight when tensor memory is released.
  umma_commit(b.mma_done);
  (void)mbar_wait(b.mma_done, 0, p.err);
}

// ------------------------------------------------------------- workers

// Warp `wid` normalises rows row0 + wid and row0 + wid + 8 of the chunk
// (L2 reads: other SMs' adds just landed there).
template <int kVec>
__device__ __forceinline__ void NormRows(const LayerKernelParams& p, const LayerTask& t, int wid,
                                         int lane) {
  constexpr int width = 128 * kVec;
  const float* weight = p.norms + static_cast<size_t>(t.layer) * (2 * width + 2 * kD) +
                        (t.kind == kTaskNorm1 ? 0 : width);
  __half* out = reinterpret_cast<__half*>(p.normed);
  for (int r = t.row0 + wid; r < t.row0 + t.rows; r += 8) {
    float4 x[kVec];
#pragma unroll
    for (int i = 0; i < kVec; ++i)
      x[i] = __ldcg(reinterpret_cast<const float4*>(p.hidden + static_cast<size_t>(r) * width +
                                                    (i * 32 + lane) * 4));
    norm_store_row<kVec>(x, weight, out + static_cast<size_t>(r) * width,
                         rms_scale(row_squares<kVec>(x), width, p.epsilon), lane);
  }
}

template <int S>
__device__ __forceinline__ void SplitEpilogue(const LayerKernelParams& p, const LayerTask& t,
                                              const GemmArgs& a, const CUtensorMap* map_y,
                                              EpilogueCtx& c, uint32_t tacc, int tile, bool& ok) {
  XchgSend<kLBN, S>(a, tacc, c, tile, t.split);
  named_barrier(kEpiBarrier, 256);  // every partial slice of this split is written
  uint32_t* arrived = p.xchg_counters +
                      (static_cast<size_t>(t.layer) * 2 + (t.kind == kTaskDown ? 1 : 0)) *
                          static_cast<size_t>(p.num_m * (p.hidden_size / kLBN)) +
                      tile;
  if (c.ep == 0) {
    fence_acq_rel_gpu();
    red_release_gpu_add(arrived, 1u);
    ok = CounterWait(arrived, static_cast<uint32_t>(S), p);
  }
  // The peers' slices are in L2 (acquired by thread 0, ordered by the barrier).
  named_barrier(kEpiBarrier, 256);
  XchgReduce<kLBN, OV_EPI_ACCUM_F32, S, 1>(a, map_y, c, tacc, tile, t.m, t.n, t.split);
}

// Shared-memory layout of the layer kernel (1024-byte aligned base).
struct Smem {
  uint8_t* ring;      // kRingBytes
  uint8_t* staging;   // 2 x kStageTile
  float* norm_w;      // 256 floats
  Bars b;
  uint32_t* tmem_slot;
  uint32_t* flag;
};

__device__ __forceinline__ Smem SmemAt(uint8_t* base) {
  Smem m;
  m.ring = base;
  m.staging = base + kRingBytes;
  m.norm_w = s_norm_w;
  uint64_t* bar_mem = s_bars;
  m.b.full = bar_mem;
  m.b.empty = bar_mem + 4;
  m.b.tfull = bar_mem + 8;
  m.b.tempty = bar_mem + 10;
  m.b.ring_release = bar_mem + 12;
  m.b.mma_done = bar_mem + 13;
  m.b.attn.q_full = bar_mem + 14;
  m.b.attn.k_full = bar_mem + 15;
  m.b.attn.k_empty = bar_mem + 17;
  m.b.attn.v_full = bar_mem + 19;
  m.b.attn.v_empty = bar_mem + 21;
  m.b.attn.s_full = bar_mem + 23;
  m.b.attn.p_full = bar_mem + 25;
  m.b.attn.o_done = bar_mem + 27;
  m.b.attn.pv_done = bar_mem + 29;
  m.tmem_slot = &s_words[0];
  m.flag = &s_words[1];
  return m;
}

// The workers' part of each task kind; each ends with the task's
// completion signal.

__device__ __forceinline__ void WorkNorm(const LayerKernelParams& p, const LayerTask t) {
  const int lane = threadIdx.x & 31;
  const int wid = (threadIdx.x >> 5) - 2;
  bool ok = true;
  if (lane == 0) ok = WaitDeps(p, t);
  ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
  if (ok) {
    switch (p.hidden_size / 128) {
      case 8: NormRows<8>(p, t, wid, lane); break;
      case 4: NormRows<4>(p, t, wid, lane); break;
      case 2: NormRows<2>(p, t, wid, lane); break;
      default: NormRows<1>(p, t, wid, lane); break;
    }
  }
  named_barrier(kEpiBarrier, 256);
  if (threadIdx.x == 64 && !Aborted(p)) Signal(p, t);
}

__device__ __forceinline__ void WorkAttn(const LayerKernelParams& p, const LayerTask t, uint8_t* base,
                                      uint32_t tmem, int acc_iter, uint32_t phase_bits) {
  const Smem m = SmemAt(base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int wg = (warp - 2) >> 2;
  AttnPhase aph;
  aph.bits = phase_bits;
  const int start = p.cu_seqlens[t.m];
  const int len = p.cu_seqlens[t.m + 1] - start;
  const int nt = (len + kKeys - 1) / kKeys;
  // Row statistics of a split tile live in the staging tiles.
  float* xmax = reinterpret_cast<float*>(m.staging);
  float* xsum = xmax + 2 * 2 * 128;
  const AttnArgs aargs = AttentionArgs(p);
  if (t.split == 2)
    SoftmaxRole<1>(aargs, &p.map_attn, tmem, m.b.attn, aph, xmax, xsum, m.ring, wg, quarter, lane,
                   len, nt, t.row0, start, t.n, kAttnBarBase, 2);
  else
    SoftmaxRole<2>(aargs, &p.map_attn, tmem, m.b.attn, aph, xmax, xsum, m.ring, wg, quarter, lane,
                   len, nt, t.row0, start, t.n, kAttnBarBase, 1);
  tc_fence_before_sync();
  // Both accumulator buffers: keep their phases in step, then release.
  for (int j = 0; j < 2; ++j)
    (void)BarWait(&m.b.tfull[(acc_iter + j) & 1], static_cast<uint32_t>((acc_iter + j) >> 1) & 1u, p);
  for (int j = 0; j < 2; ++j) mbar_arrive(&m.b.tempty[(acc_iter + j) & 1]);
  // The query tiles' staged output has been read (by the storing threads,
  // inside SoftmaxRole): the ring may be refilled.
  mbar_arrive(m.b.ring_release);
  if (quarter == 0 && lane == 0) {  // the threads that issued TMA stores
    bulk_wait_group<0>();
    fence_proxy_async_global();
  }
  named_barrier(kEpiBarrier, 256);
  if (threadIdx.x == 64 && !Aborted(p)) Signal(p, t);
}

template <int KIND>
__device__ __forceinline__ void WorkGemm(const LayerKernelParams& p, const LayerTask t, uint8_t* base,
                                      uint32_t tmem, int acc_iter) {
  const Smem m = SmemAt(base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  EpilogueCtx c;
  c.staging = m.staging;
  c.ring = nullptr;  // the ring belongs to the next task's loads
  c.ep = threadIdx.x - 64;
  c.group = c.ep >> 7;
  c.gep = c.ep & 127;
  c.row = quarter * 32 + lane;
  c.chunk_iter = 0;
  c.joint_iter = 0;
  c.direct_rows = p.rows;
  // Outputs go straight from registers to global memory (no staging tile,
  // no wait for a TMA store to drain before the next chunk).
  if (KIND == kTaskQkv) {
    c.direct = reinterpret_cast<uint8_t*>(p.qkv[t.layer & 1]);
    c.direct_ld = static_cast<int64_t>(p.heads + 2 * p.kv_heads) * kD * 2;
    c.direct_elem = 2;
  } else if (KIND == kTaskGateUp) {
    c.direct = reinterpret_cast<uint8_t*>(p.act);
    c.direct_ld = static_cast<int64_t>(p.intermediate) * 2;
    c.direct_elem = 2;
  } else {
    c.direct = reinterpret_cast<uint8_t*>(p.hidden);
    c.direct_ld = static_cast<int64_t>(p.hidden_size) * 4;
    c.direct_elem = 4;
  }
  const GemmArgs a = EpilogueArgs(p, t);
  const TileShape sh = ShapeOf(p, t);
  const int buf = acc_iter & 1;
  RopeRow rope;
  if constexpr (KIND == kTaskQkv) {
    LoadRopeRow<OV_EPI_QKNORM_ROPE_F16>(a, t.m, c.row, c.group, rope);
    const float* n = p.norms + static_cast<size_t>(t.layer) * (2 * p.hidden_size + 2 * kD) +
                     2 * p.hidden_size;
    m.norm_w[c.ep] = n[c.ep];  // q norm (128) then k norm (128)
    named_barrier(kEpiBarrier, 256);
  }
  (void)BarWait(&m.b.tfull[buf], static_cast<uint32_t>(acc_iter >> 1) & 1u, p);
  __syncwarp();  // the tensor-memory loads below are warp-collective
  tc_fence_after_sync();
  const uint32_t tacc = tmem + static_cast<uint32_t>(buf * kLBN) + (static_cast<uint32_t>(quarter * 32) << 16);
  if constexpr (KIND == kTaskQkv) {
    EpilogueUnit<kLBN, OV_EPI_QKNORM_ROPE_F16>(a, sh.y, c, tacc, t.m, t.n, m.norm_w, rope);
  } else if constexpr (KIND == kTaskGateUp) {
    EpilogueUnit<kLBN, OV_EPI_SWIGLU_F16>(a, sh.y, c, tacc, t.m, t.n, m.norm_w, rope);
  } else {  // residual products
    const int tile = t.m * sh.n_tiles + t.n;
    bool ok = true;
    if (t.splits == 4)
      SplitEpilogue<4>(p, t, a, sh.y, c, tacc, tile, ok);
    else if (t.splits == 2)
      SplitEpilogue<2>(p, t, a, sh.y, c, tacc, tile, ok);
    else
      EpilogueUnit<kLBN, OV_EPI_ACCUM_F32>(a, sh.y, c, tacc, t.m, t.n, m.norm_w, rope);
  }
  tc_fence_before_sync();
  mbar_arrive(&m.b.tempty[buf]);
  named_barrier(kEpiBarrier, 256);
  if (c.ep == 0 && !Aborted(p)) Signal(p, t);
}

__device__ void WorkerRole(const LayerKernelParams& p, uint8_t* base, uint32_t tmem) {
  // Only the task index, the accumulator count and the attention phases
  // live across tasks.
  int acc_iter = 0;
  AttnPhase aph;
  uint32_t* flag = SmemAt(base).flag;
  for (int ti = blockIdx.x; ti < p.ntasks; ti += gridDim.x) {
    // The previous task's staging tiles, norm weights and row statistics
    // are free; every worker sees the same abort decision.
    if (threadIdx.x == 64) *flag = Aborted(p) ? 1u : 0u;
    named_barrier(kEpiBarrier, 256);
    if (*flag != 0) break;
    const LayerTask t = p.tasks[ti];
    switch (t.kind) {
      case kTaskNorm1:
      case kTaskNorm2:
        WorkNorm(p, t);
        break;
      case kTaskAttn: {
        WorkAttn(p, t, base, tmem, acc_iter, aph.bits);
        const int len = p.cu_seqlens[t.m + 1] - p.cu_seqlens[t.m];
        aph.Advance((len + kKeys - 1) / kKeys, t.split);
        acc_iter += 2;
        break;
      }
      case kTaskQkv:
        WorkGemm<kTaskQkv>(p, t, base, tmem, acc_iter);
        ++acc_iter;
        break;
      case kTaskGateUp:
        WorkGemm<kTaskGateUp>(p, t, base, tmem, acc_iter);
        ++acc_iter;
        break;
      default:
        WorkGemm<kTaskO>(p, t, base, tmem, acc_iter);
        ++acc_iter;
        break;
    }
  }
}

// 320 threads: ten warps, three on two of the four SM sub-partitions, whose
// 16K registers each cap a thread at 168.
__global__ void __launch_bounds__(kThreads, 1)
    layers_kernel(const __grid_constant__ LayerKernelParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const Smem m = SmemAt(base);
  const Bars& b = m.b;
  uint8_t* ring = m.ring;
  uint32_t* tmem_slot = m.tmem_slot;

  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLStages; ++s) {
      mbar_init(&b.full[s], 1);
      mbar_init(&b.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b.tfull[i], 1);
      mbar_init(&b.tempty[i], 256);
    }
    mbar_init(b.ring_release, 256);
    mbar_init(b.mma_done, 1);
    // p_full: 256 arrivals per key tile whatever the item's form (a tile
    // pair's 128 threads of a group arrive twice each).
    InitAttnBars(b.attn, 256);
    fence_mbar_init();
    const CUtensorMap* maps[] = {&p.map_normed, &p.map_attn, &p.map_act, &p.map_qkv[0],
                                 &p.map_qkv[1], &p.map_hidden, &p.map_w_qkv, &p.map_w_o,
                                 &p.map_w_gu, &p.map_w_down};
    for (const CUtensorMap* m : maps) tma_prefetch_map(m);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the embedding and first norm of the previous kernel are complete

  if (warp == 0) {
    ProducerRole(p, ring, b);
  } else if (warp == 1) {
    if ((threadIdx.x & 31) == 0) MmaRole(p, ring, b, tmem);
    __syncwarp();
  } else {
    WorkerRole(p, base, tmem);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool LayerKernelSupports(int hidden, int heads, int kv_heads, int head_dim, int intermediate) {
  const int qkvw = (heads + 2 * kv_heads) * head_dim;
  return head_dim == 128 && kv_heads > 0 && heads % kv_heads == 0 && hidden % 256 == 0 &&
         hidden <= 1024 && qkvw % 256 == 0 && (heads * head_dim) % 256 == 0 &&
         (2 * intermediate) % 256 == 0 && intermediate % 64 == 0;
}

int LayerKernelSplits(int k) {
  const int kblocks = k / kBK;
  return kblocks >= 16 ? 4 : kblocks >= 4 ? 2 : 1;
}

void BuildLayerTasks(int layers, int rows, int hidden, int heads, int kv_heads, int intermediate,
                     const std::vector<int32_t>& cu, int o_splits, int down_splits,
                     std::vector<LayerTask>* tasks, std::vector<int32_t>* targets) {
  const int num_m = (rows + kBM - 1) / kBM;
  const int qkv_tiles = (heads + 2 * kv_heads) * kD / kLBN;
  const int h_tiles = hidden / kLBN;
  const int gu_tiles = 2 * intermediate / kLBN;
  const int n_seqs = static_cast<int>(cu.size()) - 1;
  targets->assign(static_cast<size_t>(kTaskKinds) * num_m, 0);
  auto target = [&](int kind, int m) -> int32_t& { return (*targets)[kind * num_m + m]; };
  auto block_of = [](int row) { return row / kBM; };
  // Norm chunks of every row block.
  std::vector<std::pair<int, int>> chunks;  // (row0, rows)
  for (int m = 0; m < num_m; ++m)
    for (int r = m * kBM; r < std::min(rows, (m + 1) * kBM); r += kNormRows) {
      chunks.emplace_back(r, std::min(kNormRows, std::min(rows, (m + 1) * kBM) - r));
      ++target(kTaskNorm1, m);
      ++target(kTaskNorm2, m);
    }
  for (int m = 0; m < num_m; ++m) {
    target(kTaskQkv, m) = qkv_tiles;
    target(kTaskO, m) = h_tiles * o_splits;
    target(kTaskGateUp, m) = gu_tiles;
    target(kTaskDown, m) = h_tiles * down_splits;
  }
  // Attention items: longest sequences first, tile pairs (a sequence's odd
  // last tile alone), every head.
  std::vector<int> order(n_seqs);
  for (int s = 0; s < n_seqs; ++s) order[s] = s;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return cu[a + 1] - cu[a] > cu[b + 1] - cu[b]; });
  struct Item {
    int seq, q0, groups, lo, hi, sig_lo, sig_hi;
  };
  std::vector<Item> items;
  for (const int s : order) {
    const int start = cu[s], len = cu[s + 1] - cu[s];
    if (len <= 0) continue;
    for (int q0 = 0; q0 < len; q0 += 2 * kQ) {
      const int groups = q0 + kQ < len ? 2 : 1;
      const int q_end = std::min(len, q0 + groups * kQ);
      items.push_back({s, q0, groups, block_of(start), block_of(start + len - 1),
                       block_of(start + q0), block_of(start + q_end - 1)});
    }
  }
  for (const Item& it : items)
    for (int m = it.sig_lo; m <= it.sig_hi; ++m) target(kTaskAttn, m) += heads;

  tasks->clear();
  auto add = [&](uint8_t kind, int layer, int m, int n, int split, int splits, int wait_kind,
                 int wait_layer, int wait_lo, int wait_hi, int sig_lo, int sig_hi, int row0,
                 int nrows) {
    LayerTask t{};
    t.kind = kind;
    t.layer = static_cast<uint8_t>(layer);
    t.split = static_cast<uint8_t>(split);
    t.splits = static_cast<uint8_t>(splits);
    t.m = static_cast<int16_t>(m);
    t.n = static_cast<int16_t>(n);
    t.wait_kind = static_cast<int8_t>(wait_kind);
    t.wait_layer = static_cast<uint8_t>(std::max(wait_layer, 0));
    t.wait_lo = static_cast<int16_t>(wait_lo);
    t.wait_hi = static_cast<int16_t>(wait_hi);
    t.sig_lo = static_cast<int16_t>(sig_lo);
    t.sig_hi = static_cast<int16_t>(sig_hi);
    t.row0 = row0;
    t.rows = nrows;
    tasks->push_back(t);
  };
  for (int l = 0; l < layers; ++l) {
    // Layer 0's input norm is fused into the embedding kernel.
    if (l > 0)
      for (const auto& [r0, nr] : chunks)
        add(kTaskNorm1, l, block_of(r0), 0, 0, 1, kTaskDown, l - 1, block_of(r0), block_of(r0),
            block_of(r0), block_of(r0), r0, nr);
    for (int m = 0; m < num_m; ++m)
      for (int n = 0; n < qkv_tiles; ++n)
        add(kTaskQkv, l, m, n, 0, 1, l > 0 ? kTaskNorm1 : -1, l, m, m, m, m, 0, 0);
    for (const Item& it : items)
      for (int h = 0; h < heads; ++h)
        add(kTaskAttn, l, it.seq, h, it.groups, 1, kTaskQkv, l, it.lo, it.hi, it.sig_lo,
            it.sig_hi, it.q0, 0);
    for (int m = 0; m < num_m; ++m)
      for (int n = 0; n < h_tiles; ++n)
        for (int s = 0; s < o_splits; ++s)
          add(kTaskO, l, m, n, s, o_splits, kTaskAttn, l, m, m, m, m, 0, 0);
    for (const auto& [r0, nr] : chunks)
      add(kTaskNorm2, l, block_of(r0), 0, 0, 1, kTaskO, l, block_of(r0), block_of(r0),
          block_of(r0), block_of(r0), r0, nr);
    for (int m = 0; m < num_m; ++m)
      for (int n = 0; n < gu_tiles; ++n)
        add(kTaskGateUp, l, m, n, 0, 1, kTaskNorm2, l, m, m, m, m, 0, 0);
    for (int m = 0; m < num_m; ++m)
      for (int n = 0; n < h_tiles; ++n)
        for (int s = 0; s < down_splits; ++s)
          add(kTaskDown, l, m, n, s, down_splits, kTaskGateUp, l, m, m, m, m, 0, 0);
  }
}

int LayerKernelGrid() {
  int blocks = 0;
  Check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, layers_kernel, kThreads,
                                                      kLSmemBytes),
        "layer kernel occupancy");
  OV_REQUIRE(blocks >= 1, "the layer kernel does not fit an SM");
  return SmCount();
}

void ConfigureLayerKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(layers_kernel), static_cast<int>(kLSmemBytes));
}

void LaunchLayerKernel(const LayerKernelParams& params, int grid, cudaStream_t stream) {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(layers_kernel), static_cast<int>(kLSmemBytes));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kLSmemBytes;
  cfg.stream = stream;
  // Every CTA waits on others: all of them must be resident at once.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Check(cudaLaunchKernelEx(&cfg, layers_kernel, params), "layer kernel launch");
}

}  // namespace ovb
