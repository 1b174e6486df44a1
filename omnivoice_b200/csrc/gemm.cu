// y (+)= x * w^T on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the reference's hipBLASLt wrapper (gemm.cpp:80-288, HalfGemm)
// and fuses the element-wise kernels that follow each product in
// generator.cpp:272-300: SwiGLU (generator_kernels.hip:191-200), QK
// RMSNorm + RoPE (:102-159) and the residual add (beta = 1).
//
// Persistent kernel, one CTA per SM at most, looping over work units
// (128 x BN output tiles, times the split-K factor):
//   warp 0      TMA producer: 128x64 tiles of x and BNx64 tiles of w,
//               128-byte swizzled, into a STAGES-deep shared-memory ring
//               that runs continuously across units;
//   warp 1      owns 2 x BN tensor-memory columns (two accumulators) and,
//               from one thread, issues tcgen05.mma (M=128, N=BN, K=16)
//               into the accumulator of the current unit, releasing ring
//               slots with tcgen05.commit;
//   warps 2..5  epilogue: thread r owns accumulator row r (tensor-memory
//               lane r); it loads its row with tcgen05.ld, applies the fused
//               epilogue, writes 128-byte row pieces into a 128B-swizzled
//               shared-memory staging tile, and one thread stores the tile
//               with a TMA bulk store -- or, for the residual add, a TMA
//               bulk reduce-add into y (one writer per element: exact and
//               deterministic).  The epilogue of unit i overlaps the MMAs
//               of unit i+1 (double-buffered accumulators).
// Split-K (short M), always summed in split order so results do not depend
// on timing: the splits of a tile run as one thread-block cluster and
// exchange column slices of their partials (through the caller's workspace
// in global memory, or else through distributed shared memory); or, for
// the residual epilogue, they add into y one after another behind a
// per-tile order counter.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "gemm.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ptx.cuh"
#include "gemm_device.cuh"

namespace ovb {
namespace {

template <int BN, int EPI, int S>
__device__ __forceinline__ void XchgSplitK(const GemmArgs& a, const CUtensorMap* map_y,
                                           EpilogueCtx& c, uint32_t tacc, uint64_t* inbox_bar,
                                           int tile, int m_tile, int n_tile, int rank) {
  if constexpr (BN / S >= 32) {
    XchgSend<BN, S>(a, tacc, c, tile, rank);
    named_barrier(kEpiBarrier, 256);  // every partial slice is written
    if (c.ep == 0) {
      // The readers are this cluster's CTAs (acquire at cluster scope).
      fence_acq_rel_cluster();
      for (int j = 0; j < S; ++j)
        if (j != rank) mbar_arrive_cluster(mapa_shared(smem_u32(inbox_bar), static_cast<uint32_t>(j)));
    }
    (void)mbar_wait_cluster(inbox_bar, 0, a.err);
    __syncwarp();
    XchgReduce<BN, EPI, S>(a, map_y, c, tacc, tile, m_tile, n_tile, rank);
  }
}


template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_y, const GemmArgs args) {
  using Cfg = TileConfig<BN, EPI, PAIR>;
  constexpr int kStages = Cfg::kStages;
  constexpr bool kClusterSplit = !PAIR && (EPI == OV_EPI_ACCUM_F32 || EPI == OV_EPI_STORE_F32);
  // PAIR: units are 256-row tiles walked by CTA pairs; rank 0 issues the MMAs.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ustep = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sb = sa + kStages * Cfg::kABytes;
  uint8_t* staging = sb + kStages * Cfg::kBBytes;  // 1024-byte aligned
  float* norm_w = reinterpret_cast<float*>(staging + 2 * kStageTile);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(norm_w) + Cfg::kNormFloats * 4);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;  // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* inbox_bar = tempty + 2;   // cluster split-K: partials received
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(inbox_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // The next kernel may start its prologue (its CTAs find SMs only as this
  // grid's leave); every read of this kernel's inputs waits below.
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      // PAIR: one arrival from each CTA's epilogue (on rank 0's barrier).
      mbar_init(&tempty[b], PAIR ? 2 : 256);
    }
    // Global-memory exchange: one arrival per peer; else one arrival that
    // expects the peers' bulk-copy bytes.
    mbar_init(inbox_bar, args.xchg != nullptr ? static_cast<uint32_t>(args.splits - 1) : 1u);
    fence_mbar_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    tma_prefetch_map(&map_y);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 2 * BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 2 * BN);
      tmem_relinquish();
    }
  }
  if constexpr (EPI == OV_EPI_QKNORM_ROPE_F16) {
    if (warp >= 2) {
      const int i = threadIdx.x - 64;  // 0..255: q_norm then k_norm
      norm_w[i] = i < 128 ? args.q_norm[i] : args.k_norm[i - 128];
    }
  }
  tc_fence_before_sync();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
  else
    __syncthreads();
  tc_fence_after_sync();
  // Global-memory split-K exchange: the arrival half of the barrier that
  // makes every rank's inbox barrier visible before a peer signals it; the
  // wait half runs after the MMAs, by when every rank has long arrived.
  if (kClusterSplit && args.xchg != nullptr) cluster_arrive();
  const uint32_t tmem = *tmem_slot;
  if (!(warp == 0 && lane == 0)) pdl_wait();  // inputs of the previous kernel are ready

  if (warp == 0) {
    if (lane == 0) {
      // The weights do not depend on the previous kernel: start the weight
      // tiles of the first ring slots before waiting for it.
      //
      // PAIR: each CTA loads its A rows (256-row tile m: rows 256 m + 128
      // rank ..) and its half of the B rows into its own ring; all bytes
      // complete on rank 0's full barrier, which rank 0 arms for both.
      const uint32_t stage_tx = PAIR ? 2 * Cfg::kStageBytes : Cfg::kStageBytes;
      const bool arm = !PAIR || rank == 0;
      const int b_rows = PAIR ? BN / 2 : BN;
      auto bar_of = [&](int st) -> uint32_t {
        return PAIR ? mapa_shared(smem_u32(&full[st]), 0) : smem_u32(&full[st]);
      };
      auto load = [&](void* dst, const CUtensorMap* map, int st, int x, int y) {
        if constexpr (PAIR)
          tma_load_2d_pair(dst, map, bar_of(st), x, y);
        else
          tma_load_2d(dst, map, &full[st], x, y);
      };
      uint32_t pre = 0;
      if (unit0 < args.units) {
        int m_tile, n_tile, split;
        UnitCoords(args, unit0, m_tile, n_tile, split);
        const int kb0 = split * args.kblocks / args.splits;
        const int kb1 = (split + 1) * args.kblocks / args.splits;
        pre = static_cast<uint32_t>(min(kStages, kb1 - kb0));
        for (uint32_t i = 0; i < pre; ++i) {
          if (arm) mbar_arrive_expect_tx(&full[i], stage_tx);
          load(sb + i * Cfg::kBBytes, &map_b, static_cast<int>(i),
               (kb0 + static_cast<int>(i)) * kBK,
               args.b_row_offset + n_tile * BN + static_cast<int>(rank) * b_rows);
        }
      }
      pdl_wait();
      uint32_t k_iter = 0;
      bool ok = true;
      for (int u = unit0; ok && u < args.units; u += ustep) {
        int m_tile, n_tile, split;
        UnitCoords(args, u, m_tile, n_tile, split);
        const int a_row = (PAIR ? 2 * m_tile + static_cast<int>(rank) : m_tile) * kBM;
        const int kb0 = split * args.kblocks / args.splits;
        const int kb1 = (split + 1) * args.kblocks / args.splits;
        for (int kb = kb0; kb < kb1; ++kb, ++k_iter) {
          const int s = static_cast<int>(k_iter % kStages);
          const uint32_t phase = (k_iter / kStages) & 1u;
          if (k_iter < pre) {  // weight tile already on its way
            load(sa + s * Cfg::kABytes, &map_a, s, kb * kBK, a_row);
            continue;
          }
          if (k_iter >= static_cast<uint32_t>(kStages) &&
              !mbar_wait(&empty[s], phase ^ 1u, args.err)) {
            ok = false;
            break;
          }
          if (arm) mbar_arrive_expect_tx(&full[s], stage_tx);
          load(sa + s * Cfg::kABytes, &map_a, s, kb * kBK, a_row);
          load(sb + s * Cfg::kBBytes, &map_b, s, kb * kBK,
               args.b_row_offset + n_tile * BN + static_cast<int>(rank) * b_rows);
        }
      }
      // Let the copies this thread started land before the CTA can exit
      // (PAIR rank 1: its copies land on rank 0's barriers, which rank 0's
      // MMAs consume before this CTA's accumulators are complete).
      if (arm) {
        const uint32_t first = k_iter > static_cast<uint32_t>(kStages) ? k_iter - kStages : 0u;
        for (uint32_t i = first; i < k_iter; ++i)
          (void)mbar_wait(&full[i % kStages], (i / kStages) & 1u, args.err);
      }
    }
    if (kClusterSplit && args.cluster) {  // the barriers of the split-K reduction
      __syncwarp();
      if (args.xchg != nullptr) {
        cluster_wait();
      } else {
        cluster_sync();
        cluster_sync();
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // PAIR: rank 0 issues for both CTAs
      constexpr uint32_t idesc = idesc_f16_f32(PAIR ? 2 * kBM : kBM, BN);
      uint32_t k_iter = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int u = unit0; ok && u < args.units; u += ustep, ++acc_iter) {
        int m_tile, n_tile, split;
        UnitCoords(args, u, m_tile, n_tile, split);
        const int kb0 = split * args.kblocks / args.splits;
        const int kb1 = (split + 1) * args.kblocks / args.splits;
        const int buf = acc_iter & 1;
        if (acc_iter >= 2 &&
            !mbar_wait(&tempty[buf], static_cast<uint32_t>((acc_iter >> 1) - 1) & 1u, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++k_iter) {
          const int s = static_cast<int>(k_iter % kStages);
          const uint32_t phase = (k_iter / kStages) & 1u;
          if (!mbar_wait(&full[s], phase, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sa + s * Cfg::kABytes);
          const uint32_t b0 = smem_u32(sb + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + k * 32, 16, 1024);
            const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
            if constexpr (PAIR)
              umma_f16_ss_pair(d, ad, bd, idesc, acc);
            else
              umma_f16_ss(d, ad, bd, idesc, acc);
          }
          if constexpr (PAIR)
            umma_commit_pair(&empty[s], 0x3);  // both CTAs' slots are free
          else
            umma_commit(&empty[s]);
        }
        if constexpr (PAIR)
          umma_commit_pair(&tfull[buf], 0x3);
        else
          umma_commit(&tfull[buf]);
      }
    }
    if (kClusterSplit && args.cluster) {
      __syncwarp();
      if (args.xchg != nullptr) {
        cluster_wait();
      } else {
        cluster_sync();
        cluster_sync();
      }
    }
  } else {
    EpilogueCtx c;
    c.staging = staging;
    c.chunk_iter = 0;
    c.joint_iter = 0;
    c.ring = nullptr;
    c.ep = threadIdx.x - 64;
    c.group = c.ep >> 7;
    c.gep = c.ep & 127;
    const int quarter = warp & 3;  // tensor-memory lanes 32*quarter .. +31
    c.row = quarter * 32 + lane;
    // Global-memory split-K exchange: every rank's inbox barrier is
    // initialised before this rank signals it (the wait half of the
    // prologue's cluster barrier, taken while the MMAs run).
    if (kClusterSplit && args.xchg != nullptr) cluster_wait();
    int acc_iter = 0;
    for (int u = unit0; u < args.units; u += ustep, ++acc_iter) {
      int m_tile, n_tile, split;
      UnitCoords(args, u, m_tile, n_tile, split);
      if constexpr (PAIR) m_tile = 2 * m_tile + static_cast<int>(rank);  // this CTA's 128 rows
      const int buf = acc_iter & 1;
      RopeRow rope;
      LoadRopeRow<EPI>(args, m_tile, c.row, c.group, rope);
      // Every epilogue thread runs the epilogue even after a timed-out wait
      // (the error word is set) so the 256 threads stay in step.
      (void)mbar_wait(&tfull[buf], static_cast<uint32_t>(acc_iter >> 1) & 1u, args.err);
      __syncwarp();  // the tensor-memory loads below are warp-collective
      tc_fence_after_sync();
      if (args.cluster) break;  // one unit per CTA, reduced below
      const int tile = u / args.splits;
      if (EPI == OV_EPI_ACCUM_F32 && args.splits > 1) {
        // Earlier splits of this tile first; their adds are complete.
        if (c.ep == 0) {
          (void)wait_counter_equals(args.counters + tile, static_cast<uint32_t>(split), args.err);
        }
        named_barrier(kEpiBarrier, 256);
        if (c.gep == 0) fence_proxy_async_global();
      }
      const uint32_t tacc =
          tmem + static_cast<uint32_t>(buf * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      // This CTA's last unit: its loads are all consumed and its MMAs done.
      c.ring = u + ustep >= args.units ? smem : nullptr;
      EpilogueUnit<BN, EPI>(args, &map_y, c, tacc, m_tile, n_tile, norm_w, rope);
      tc_fence_before_sync();
      if constexpr (PAIR) {
        // Both CTAs' accumulators are read: one arrival per CTA on rank 0.
        named_barrier(kEpiBarrier, 256);
        if (c.ep == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
      } else {
        mbar_arrive(&tempty[buf]);
      }
      if (EPI == OV_EPI_ACCUM_F32 && args.splits > 1) {
        if (c.gep == 0) {  // both group leaders: their adds are complete
          bulk_wait_group<0>();
          fence_proxy_async_global();
        }
        named_barrier(kEpiBarrier, 256);
        if (c.ep == 0) {
          __threadfence();
          if (split == args.splits - 1)
            st_relaxed_gpu(args.counters + tile, 0u);  // ready for the next launch
          else
            red_release_gpu_add(args.counters + tile, 1u);
        }
      }
    }
    if constexpr (kClusterSplit) {
      if (args.cluster) {
        // Every CTA of the cluster has waited for its accumulator, so all
        // MMAs are complete and every operand ring is free.
        int m_tile, n_tile, split;
        UnitCoords(args, blockIdx.x, m_tile, n_tile, split);
        const uint32_t tacc = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        __syncwarp();
        if (args.xchg != nullptr) {
          c.ring = smem;  // all MMAs are complete: the idle ring stages the stores
          const int tile = static_cast<int>(blockIdx.x) / args.splits;
          switch (args.splits) {
            case 2:
              XchgSplitK<BN, EPI, 2>(args, &map_y, c, tacc, inbox_bar, tile, m_tile, n_tile, split);
              break;
            case 4:
              XchgSplitK<BN, EPI, 4>(args, &map_y, c, tacc, inbox_bar, tile, m_tile, n_tile, split);
              break;
            default:
              XchgSplitK<BN, EPI, 8>(args, &map_y, c, tacc, inbox_bar, tile, m_tile, n_tile, split);
              break;
          }
        } else {
          tc_fence_before_sync();
          cluster_sync();
          tc_fence_after_sync();
          if (c.ep == 0) {
            const uint32_t slot_bytes = static_cast<uint32_t>(kBM * (BN / args.splits) * 4);
            mbar_arrive_expect_tx(inbox_bar, static_cast<uint32_t>(args.splits - 1) * slot_bytes);
          }
          ClusterSend<BN>(tacc, smem, c, split, args.splits, inbox_bar);
          (void)mbar_wait(inbox_bar, 0, args.err);
          __syncwarp();
          ClusterReduce<BN, EPI>(args, &map_y, c, tacc, smem, m_tile, n_tile, split);
          // No CTA leaves while a peer's bulk copy may still read its outbox.
          __syncwarp();
          cluster_sync();
        }
      }
    }
    // Each group leader's stores have read their staging tiles before the
    // CTA's shared memory goes away; the writes complete with the grid.
    if (c.gep == 0) bulk_wait_group_read<0>();
  }
  tc_fence_before_sync();
  if constexpr (PAIR)
    cluster_sync();  // no CTA leaves while its peer may still signal it
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, 2 * BN);
    else
      tmem_dealloc(tmem, 2 * BN);
  }
}

// Every compiled (tile width, epilogue, CTA pair) instance.
#define OV_GEMM_INSTANCES(X)                 \
  X(64, OV_EPI_STORE_F32, false)             \
  X(128, OV_EPI_STORE_F32, false)            \
  X(256, OV_EPI_STORE_F32, false)            \
  X(64, OV_EPI_ACCUM_F32, false)             \
  X(128, OV_EPI_ACCUM_F32, false)            \
  X(256, OV_EPI_ACCUM_F32, false)            \
  X(128, OV_EPI_SWIGLU_F16, false)           \
  X(256, OV_EPI_SWIGLU_F16, false)           \
  X(128, OV_EPI_QKNORM_ROPE_F16, false)      \
  X(256, OV_EPI_QKNORM_ROPE_F16, false)      \
  X(256, OV_EPI_STORE_F32, true)             \
  X(256, OV_EPI_ACCUM_F32, true)             \
  X(256, OV_EPI_SWIGLU_F16, true)            \
  X(256, OV_EPI_QKNORM_ROPE_F16, true)

// Switch key of an instance.
constexpr int InstanceKey(int bn, int epilogue, bool pair) {
  return epilogue * 1000 + bn + (pair ? 100000 : 0);
}

template <int BN, int EPI, bool PAIR>
void LaunchTyped(const GemmPlan& p, cudaStream_t stream) {
  LaunchEx(gemm_kernel<BN, EPI, PAIR>, p.grid, dim3(kThreads),
           TileConfig<BN, EPI, PAIR>::kSmemBytes, stream,
           "gemm kernel launch", p.cluster_x, p.map_a, p.map_b, p.map_y, p.args);
}

int Tiles(int M, int N, int bn) { return ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn); }

bool ValidShape(int bn, int splits, bool cluster, int N, int K, int epilogue, bool xchg = false) {
  if (splits < 1 || splits > 8) return false;
  if (cluster) {
    // Split-K inside a thread-block cluster, each rank reducing a BN /
    // splits slice of the splits' partials.
    if (splits != 2 && splits != 4 && splits != 8) return false;
    if (epilogue != OV_EPI_ACCUM_F32 && epilogue != OV_EPI_STORE_F32) return false;
    if (bn / splits < 32 || (K / kBK) < splits) return false;
    // Distributed shared memory: inbox and outbox, (S - 1) slices each,
    // live in the 192 KB operand ring.
    if (!xchg && 2 * (splits - 1) * kBM * (bn / splits) * 4 > kRingBytes) return false;
    return bn == 64 || bn == 128 || bn == 256;
  }
  if (splits > 1 && (epilogue != OV_EPI_ACCUM_F32 || (K / kBK) / splits < 2)) return false;
  switch (epilogue) {
    case OV_EPI_QKNORM_ROPE_F16: return (bn == 128 || bn == 256) && N % bn == 0;
    case OV_EPI_SWIGLU_F16: return (bn == 128 || bn == 256) && N % bn == 0;
    default: return bn == 64 || bn == 128 || bn == 256;
  }
}

// Epilogues and widths the CTA-pair kernel is built for.
bool ValidPairShape(int bn, int N, int epilogue) {
  if (bn != 256) return false;
  switch (epilogue) {
    case OV_EPI_SWIGLU_F16:
    case OV_EPI_QKNORM_ROPE_F16: return N % 256 == 0;
    default: return true;
  }
}

// CTAs of one GEMM kernel that can be resident at once in clusters of
// 1, 2, 4 and 8 (index log2), measured per device by ConfigureGemmKernels;
// 0 until then (the chooser then assumes one cluster per 8 SMs).
int g_cluster_ctas[64][4];

int ClusterCapacity(int splits, int sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  const int idx = splits == 2 ? 1 : splits == 4 ? 2 : splits == 8 ? 3 : 0;
  const int v = g_cluster_ctas[dev][idx];
  return v > 0 ? v : (sms / 8) * 8;
}

}  // namespace

GemmShapeChoice ChooseGemmShape(int M, int N, int K, int epilogue, bool have_workspace, int sms,
                                bool allow_xchg) {
  // OV_GEMM_XCHG=0: cluster split-K exchanges through distributed shared
  // memory even when a workspace is given (comparison aid).
  if (const char* env = std::getenv("OV_GEMM_XCHG"); env != nullptr && std::strcmp(env, "0") == 0)
    allow_xchg = false;
  if (const char* env = std::getenv("OV_GEMM_TILE")) {
    int bn = 0, splits = 1;
    char sep = 'x';
    if (std::sscanf(env, "%d%c%d", &bn, &sep, &splits) >= 1) {
      const bool cluster = sep == 'c';
      if (sep == 'p') {
        if (ValidPairShape(bn, N, epilogue)) return {bn, 1, false, true};
      } else if (ValidShape(bn, splits, cluster, N, K, epilogue,
                            cluster && have_workspace && allow_xchg) &&
                 (splits == 1 || cluster || have_workspace)) {
        return {bn, splits, cluster && splits > 1, false,
                cluster && splits > 1 && have_workspace && allow_xchg};
      }
    }
  }
  // Cost in units of one 64-deep k block of one CTA (about 0.3 us on
  // B200, measured: the four tcgen05.mma of a k block take nearly the same
  // time for BN = 64, 128 and 256).  A persistent CTA runs
  // ceil(units / CTAs) units back to back; each kernel pays a fill
  // (prologue, first loads, last epilogue, about 5 us); serialised split-K
  // adds one tile reduction per extra split; cluster split-K one exchange
  // of (S - 1) slices, through the workspace in global memory when there
  // is one (written and read back at L2 speed), else through distributed
  // shared memory (about 25 GB/s per SM, measured).
  const int kblocks = K / kBK;
  auto per_kblock = [](int bn) { return bn == 256 ? 1.03 : 1.0; };
  constexpr double kFill = 17.0;
  GemmShapeChoice best{128, 1, false};
  double best_cost = 1e300;
  for (int bn : {64, 128, 256}) {
    for (int s = 1; s <= 8; s *= 2) {
      for (int cl = 0; cl < 2; ++cl) {
        const bool cluster = cl == 1;
        if (cluster && s == 1) continue;
        const bool xchg = cluster && have_workspace && allow_xchg;
        if (!ValidShape(bn, s, cluster, N, K, epilogue, xchg)) continue;
        if (s > 1 && !cluster && (!have_workspace || s > 4)) continue;
        const double units = static_cast<double>(Tiles(M, N, bn)) * s;
        const double ctas = cluster ? ClusterCapacity(s, sms) : sms;
        const double rounds = std::ceil(units / ctas);
        double cost = rounds * (static_cast<double>(kblocks) / s) * per_kblock(bn) + kFill;
        const double slice_bytes = (s - 1) * (kBM * (bn / s) * 4.0);
        if (s > 1 && !cluster) cost += (s - 1) * 18.0;
        if (s > 1 && cluster) cost += xchg ? 2.0 + 2.0 * slice_bytes / 49152.0 : 4.0 + slice_bytes / 8192.0;
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          best = {bn, s, cluster, false, xchg};
        }
      }
    }
  }
  // CTA pairs: 256 x 256 tiles; a k block of a CTA moves 32 KB instead of
  // the 48 KB of a 128 x 256 tile, so a long k loop runs at the MMA rate;
  // the pair's start-up costs about one k block more (measured: pairs win
  // from two rounds of tiles on, single CTAs on one round).
  if (ValidPairShape(256, N, epilogue)) {
    const double units = static_cast<double>(((M + 2 * kBM - 1) / (2 * kBM)) * ((N + 255) / 256));
    const double pairs = ClusterCapacity(2, sms) / 2;
    const double cost = std::ceil(units / pairs) * kblocks * 0.85 + kFill + 3.0;
    if (cost < best_cost - 1e-9) best = {256, 1, false, true};
  }
  return best;
}

namespace {

size_t WorkspaceNeed(int M, int N, const GemmShapeChoice& c) {
  if (c.splits <= 1 || (c.cluster && !c.xchg)) return 0;
  const size_t tiles = static_cast<size_t>(Tiles(M, N, c.bn));
  if (c.cluster) return tiles * static_cast<size_t>(c.splits) * kBM * c.bn * sizeof(float);
  return tiles * sizeof(uint32_t);
}

}  // namespace

size_t GemmWorkspaceBytes(int M, int N, int K, int epilogue, int sms) {
  return WorkspaceNeed(M, N, ChooseGemmShape(M, N, K, epilogue, true, sms));
}

void PlanGemm(GemmPlan* plan, const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t w_rows,
              int b_row_offset, void* y, int64_t ldy, int M, int N, int K, int epilogue,
              const ov_epilogue_args* ea, void* workspace, size_t workspace_bytes, int sms,
              uint32_t* err, bool allow_xchg) {
  OV_REQUIRE(M > 0 && N > 0 && K > 0, "empty GEMM");
  OV_REQUIRE(K % kBK == 0, "GEMM K must be a multiple of 64");
  OV_REQUIRE(ldx % 8 == 0 && ldx >= K, "x row stride must be a multiple of 8 and >= K");
  OV_REQUIRE(epilogue >= OV_EPI_STORE_F32 && epilogue <= OV_EPI_QKNORM_ROPE_F16, "epilogue");
  const bool half_out = epilogue == OV_EPI_SWIGLU_F16 || epilogue == OV_EPI_QKNORM_ROPE_F16;
  OV_REQUIRE(ldy % (half_out ? 8 : 4) == 0, "y row stride must be a multiple of 16 bytes");
  OV_REQUIRE((reinterpret_cast<uintptr_t>(y) & 15u) == 0, "y must be 16-byte aligned");
  // A workspace too small (or, for the partial slices, not 16-byte
  // aligned) for the chosen split-K form: choose again without one.
  const bool ws_ok = workspace != nullptr && workspace_bytes > 0;
  GemmShapeChoice choice = ChooseGemmShape(M, N, K, epilogue, ws_ok, sms, allow_xchg);
  if (workspace_bytes < WorkspaceNeed(M, N, choice) ||
      (choice.xchg && (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0))
    choice = ChooseGemmShape(M, N, K, epilogue, false, sms, allow_xchg);
  int out_cols = N;
  if (epilogue == OV_EPI_SWIGLU_F16) {
    OV_REQUIRE(N % 128 == 0, "SwiGLU output features must be a multiple of 128");
    out_cols = N / 2;
    OV_REQUIRE(ldy >= out_cols, "y row stride");
  } else if (epilogue == OV_EPI_QKNORM_ROPE_F16) {
    OV_REQUIRE(ea != nullptr && ea->head_dim == 128, "QK-norm epilogue needs head_dim 128");
    OV_REQUIRE(N == (ea->heads + 2 * ea->kv_heads) * 128, "QKV width");
    OV_REQUIRE(ea->q_norm && ea->k_norm && ea->positions && ea->rope_cos && ea->rope_sin,
               "QK-norm epilogue operands missing");
    OV_REQUIRE(ldy >= N, "y row stride");
  } else {
    OV_REQUIRE(N % 4 == 0 && ldy >= N, "output features must be a multiple of 4");
  }
  plan->epilogue = epilogue;
  plan->bn = choice.bn;
  plan->pair = choice.pair;
  GemmArgs& a = plan->args;
  a = GemmArgs{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.kblocks = K / kBK;
  a.splits = choice.splits;
  a.b_row_offset = b_row_offset;
  a.num_m = (M + kBM * (choice.pair ? 2 : 1) - 1) / (kBM * (choice.pair ? 2 : 1));
  a.num_n = (N + choice.bn - 1) / choice.bn;
  a.units = a.num_m * a.num_n * a.splits;
  a.out_cols = out_cols;
  a.err = err != nullptr ? err : DeviceErrorWord();
  if (choice.splits > 1 && !choice.cluster) a.counters = static_cast<uint32_t*>(workspace);
  a.cluster = choice.cluster ? 1 : 0;
  if (choice.xchg) a.xchg = static_cast<float*>(workspace);
  plan->cluster_x = choice.cluster ? static_cast<unsigned>(choice.splits) : 1u;
  if (ea != nullptr) {
    a.q_norm = ea->q_norm;
    a.k_norm = ea->k_norm;
    a.positions = ea->positions;
    a.rope_cos = ea->rope_cos;
    a.rope_sin = ea->rope_sin;
    a.max_positions = ea->max_positions;
    a.heads = ea->heads;
    a.kv_heads = ea->kv_heads;
    a.epsilon = ea->epsilon;
  }
  EncodeTensorMap2D(&plan->map_a, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<uint64_t>(K),
                    static_cast<uint64_t>(M), static_cast<uint64_t>(ldx) * 2, kBK, kBM,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  EncodeTensorMap2D(&plan->map_b, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<uint64_t>(K),
                    static_cast<uint64_t>(w_rows), static_cast<uint64_t>(K) * 2, kBK,
                    static_cast<uint32_t>(choice.pair ? choice.bn / 2 : choice.bn),
                    CU_TENSOR_MAP_SWIZZLE_128B);
  // y: 128-byte row pieces (32 floats or 64 halves) x 128 rows per box.
  if (half_out)
    EncodeTensorMap2D(&plan->map_y, y, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      static_cast<uint64_t>(out_cols), static_cast<uint64_t>(M),
                      static_cast<uint64_t>(ldy) * 2, 64, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    EncodeTensorMap2D(&plan->map_y, y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                      static_cast<uint64_t>(out_cols), static_cast<uint64_t>(M),
                      static_cast<uint64_t>(ldy) * 4, 32, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  // With split-K every round of the persistent grid holds whole tiles, so a
  // split only waits for lower-numbered CTAs of its own round.
  // Cluster split-K: one unit per CTA, the splits of a tile in one cluster.
  int grid = std::min(a.units, sms);
  if (a.splits > 1) grid = std::max(a.splits, grid / a.splits * a.splits);
  if (a.cluster) grid = a.units;
  if (choice.pair) {
    // Persistent CTA pairs, one pair per two SMs that a 2-cluster can hold.
    grid = 2 * std::max(1, std::min(a.units, ClusterCapacity(2, sms) / 2));
    plan->cluster_x = 2;
  }
  plan->grid = dim3(static_cast<unsigned>(grid), 1, 1);
  switch (InstanceKey(choice.bn, epilogue, choice.pair)) {
#define OV_SMEM_CASE(BN, EPI, PAIR)   \
  case InstanceKey(BN, EPI, PAIR): \
    plan->smem_bytes = TileConfig<BN, EPI, PAIR>::kSmemBytes; \
    break;
    OV_GEMM_INSTANCES(OV_SMEM_CASE)
#undef OV_SMEM_CASE
    default: throw Error(OV_ERR_UNSUPPORTED, "no GEMM kernel for this epilogue / tile");
  }
}

void ConfigureGemmKernels() {
#define OV_CONFIGURE(BN, EPI, PAIR)                                             \
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<BN, EPI, PAIR>),  \
                    static_cast<int>(TileConfig<BN, EPI, PAIR>::kSmemBytes));
  OV_GEMM_INSTANCES(OV_CONFIGURE)
#undef OV_CONFIGURE
  int dev = 0;
  Check(cudaGetDevice(&dev), "get device");
  if (dev < 0 || dev >= 64 || g_cluster_ctas[dev][0] > 0) return;
  // Resident CTAs in clusters of 1..8 (every instance holds one CTA per SM).
  for (int i = 0; i < 4; ++i) {
    const unsigned size = 1u << i;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(size * 16, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = TileConfig<256, OV_EPI_ACCUM_F32>::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_kernel<256, OV_EPI_ACCUM_F32, false>, &cfg) !=
        cudaSuccess) {
      ClearError();
      clusters = 0;
    }
    g_cluster_ctas[dev][i] = std::max(1, clusters * static_cast<int>(size));
  }
}

void LaunchGemm(const GemmPlan& p, cudaStream_t stream) {
  switch (InstanceKey(p.bn, p.epilogue, p.pair)) {
#define OV_LAUNCH_CASE(BN, EPI, PAIR)                                             \
  case InstanceKey(BN, EPI, PAIR):                                                \
    SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<BN, EPI, PAIR>),  \
                      static_cast<int>(TileConfig<BN, EPI, PAIR>::kSmemBytes));   \
    LaunchTyped<BN, EPI, PAIR>(p, stream);                                        \
    break;
    OV_GEMM_INSTANCES(OV_LAUNCH_CASE)
#undef OV_LAUNCH_CASE
    default: throw Error(OV_ERR_UNSUPPORTED, "no GEMM kernel for this epilogue / tile");
  }
}

}  // namespace ovb

// ------------------------------------------------ allocation-free variant
//
// ov_gemm_f16_noalloc takes its split-K scratch (the per-tile order
// counters) from this file-scope device array instead of a caller-supplied
// workspace.  Every GPU that loads the library holds it until the process
// exits.  In host code the array's name only stands for the symbol, so its
// device address is looked up with cudaGetSymbolAddress once per device
// (with that device current) and that address is what the kernel receives.
constexpr size_t kNoAllocScratchBytes = size_t{64} << 10;  // 64 KiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Bounded waits of this variant report into this word (it allocates nothing,
// so it cannot use the lazily allocated device error word).
static __device__ __align__(256) uint32_t g_noalloc_status[64];

namespace ovb {
namespace {

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mutex;
uint8_t* g_noalloc_scratch_ptr[kNoAllocDevices] = {};
uint32_t* g_noalloc_status_ptr[kNoAllocDevices] = {};

// Once per device, with it current: device addresses of the static arrays,
// cleared split-K counters and status word, the kernels' shared-memory
// limits and the resident-cluster capacities the tile chooser reads (the
// same set-up ov_gemm_f16's callers get, so both entry points choose the
// same tiles).  None of it allocates device memory.
void NoAllocSetup(uint8_t** scratch, uint32_t** status) {
  int device = 0;
  Check(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kNoAllocDevices) throw Error(OV_ERR_INVALID, "device index");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[device] == nullptr) {
    void* sp = nullptr;
    void* tp = nullptr;
    Check(cudaGetSymbolAddress(&sp, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    Check(cudaGetSymbolAddress(&tp, g_noalloc_status), "cudaGetSymbolAddress(status)");
    Check(cudaMemset(sp, 0, kNoAllocScratchBytes), "clear split-K counters");
    Check(cudaMemset(tp, 0, sizeof(uint32_t) * 64), "clear status word");
#define OV_SET_DIRECT(BN, EPI, PAIR)                                                   \
  Check(cudaFuncSetAttribute(gemm_kernel<BN, EPI, PAIR>,                               \
                             cudaFuncAttributeMaxDynamicSharedMemorySize,              \
                             static_cast<int>(TileConfig<BN, EPI, PAIR>::kSmemBytes)), \
        "cudaFuncSetAttribute(max dynamic shared memory)");
    OV_GEMM_INSTANCES(OV_SET_DIRECT)
#undef OV_SET_DIRECT
    ConfigureGemmKernels();
    g_noalloc_status_ptr[device] = static_cast<uint32_t*>(tp);
    g_noalloc_scratch_ptr[device] = static_cast<uint8_t*>(sp);
  }
  *scratch = g_noalloc_scratch_ptr[device];
  *status = g_noalloc_status_ptr[device];
}

}  // namespace

uint32_t* NoAllocStatusWord() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kNoAllocDevices) {
    (void)cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  return g_noalloc_status_ptr[device];
}

}  // namespace ovb

using namespace ovb;

extern "C" {

int ov_gemm_f16(const uint16_t* x, size_t ldx, const uint16_t* w, void* y, size_t ldy,
                size_t rows, size_t in, size_t out, int epilogue,
                const ov_epilogue_args* args, void* workspace, size_t workspace_bytes,
                ov_stream_t stream) {
  return Guard("ov_gemm_f16: ", [&] {
    if (rows == 0) return;
    GemmPlan plan;
    PlanGemm(&plan, x, static_cast<int64_t>(ldx), w, static_cast<int64_t>(out), 0, y,
             static_cast<int64_t>(ldy), static_cast<int>(rows), static_cast<int>(out),
             static_cast<int>(in), epilogue, args, workspace, workspace_bytes, SmCount());
    LaunchGemm(plan, AsStream(stream));
  });
}

size_t ov_gemm_workspace_bytes(size_t rows, size_t in, size_t out, int epilogue) {
  int sms = 148;
  try {
    sms = SmCount();
  } catch (...) {
  }
  return GemmWorkspaceBytes(static_cast<int>(rows), static_cast<int>(out), static_cast<int>(in),
                            epilogue, sms);
}

int ov_interleave_gate_up(const uint16_t* gate_up, size_t width, size_t in, uint16_t* output) {
  return Guard("ov_interleave_gate_up: ", [&] {
    const size_t group = OV_SWIGLU_GROUP;
    OV_REQUIRE(width % group == 0, "width must be a multiple of OV_SWIGLU_GROUP");
    for (size_t j = 0; j < width; ++j) {
      const size_t g = j / group;
      const size_t r = j % group;
      const uint16_t* gate = gate_up + j * in;
      const uint16_t* up = gate_up + (width + j) * in;
      std::copy(gate, gate + in, output + (2 * g * group + r) * in);
      std::copy(up, up + in, output + (2 * g * group + group + r) * in);
    }
  });
}

int ov_gemm_f16_noalloc(const uint16_t* x, size_t ldx, const uint16_t* w, void* y, size_t ldy,
                        size_t rows, size_t in, size_t out, int epilogue,
                        const ov_epilogue_args* args, ov_stream_t stream) {
  return Guard("ov_gemm_f16_noalloc: ", [&] {
    uint8_t* scratch = nullptr;
    uint32_t* status = nullptr;
    NoAllocSetup(&scratch, &status);
    if (rows == 0) return;
    const int sms = SmCount();
    // The static array holds split-K order counters only (one per output
    // tile of the serialised form); the partial-slice exchange, whose
    // workspace grows with the product, is not offered here.
    const size_t need = WorkspaceNeed(
        static_cast<int>(rows), static_cast<int>(out),
        ChooseGemmShape(static_cast<int>(rows), static_cast<int>(out), static_cast<int>(in),
                        epilogue, true, sms, /*allow_xchg=*/false));
    if (need > kNoAllocScratchBytes)
      throw Error(OV_ERR_INVALID, "needs " + std::to_string(need) +
                                      " bytes of split-K scratch, more than the " +
                                      std::to_string(kNoAllocScratchBytes) + "-byte static array");
    GemmPlan plan;
    PlanGemm(&plan, x, static_cast<int64_t>(ldx), w, static_cast<int64_t>(out), 0, y,
             static_cast<int64_t>(ldy), static_cast<int>(rows), static_cast<int>(out),
             static_cast<int>(in), epilogue, args, scratch, kNoAllocScratchBytes, sms, status,
             /*allow_xchg=*/false);
    // The order counters must start at zero.  The last split of each tile
    // resets its counter, but a split whose wait timed out leaves it set,
    // so every call clears the counters it uses, in stream order.
    if (plan.args.counters != nullptr)
      Check(cudaMemsetAsync(plan.args.counters, 0, need, AsStream(stream)),
            "clear split-K counters");
    switch (InstanceKey(plan.bn, plan.epilogue, plan.pair)) {
#define OV_DIRECT_CASE(BN, EPI, PAIR) \
  case InstanceKey(BN, EPI, PAIR): LaunchTyped<BN, EPI, PAIR>(plan, AsStream(stream)); break;
      OV_GEMM_INSTANCES(OV_DIRECT_CASE)
#undef OV_DIRECT_CASE
      default: throw Error(OV_ERR_UNSUPPORTED, "no GEMM kernel for this epilogue / tile");
    }
  });
}

}  // extern "C"

