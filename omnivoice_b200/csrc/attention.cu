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
  if (seq < 0 || seq >= args.num_seqs) {  // uniform over the CTA, before any barrier
    if (threadIdx.x == 0) atomicOr(args.err, kErrBadArgument);
    return;
  }
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

// ------------------------------------------------------------------------
// Query-tile pairs with the output transposed: O^T = V^T P^T.
//
// A tcgen05.mma of kind::f16 (K = 16) occupies the tensor core for about
// the same time whether N is 128 or 256, so the pair's P V product is
// issued as O^T (M = the 128 head dims, N = the pair's 256 queries): 8
// MMAs per key tile instead of 2 x 8 of N = 128, 24 MMAs per key tile in
// all with the two S = Q K^T products.  A = V^T is the V tile read
// MN-major; B = P is [256 queries][128 keys] in shared memory, K-major,
// written by the softmax threads.  Roles (320 threads):
//   softmax     warpgroup g owns query tile g: thread r reads row r of S_g
//               (tensor-memory lane r, columns 128 g ..), frees S_g for the
//               next key tile, keeps the running maximum (raised only when
//               it grows by more than 2^8), writes half P into row
//               128 g + r of the P buffer once the previous O^T product is
//               done, and on a raise rescales the group's O^T columns (all
//               128 threads: thread d owns head-dim lane d of O^T);
//   producer    warp 8: the two Q tiles once, then K and V tiles through a
//               3-slot ring in the order the MMAs consume them
//               (K0 K1 V0 K2 V1 K3 V2 ...);
//   MMA         warp 9, one thread: S_g(t + 1) as soon as the softmax has
//               read S_g(t), then O^T(t) once both P_g(t) are written.
// Tensor memory: S_0 [0, 128), S_1 [128, 256), O^T [256, 512).  The
// probabilities are rounded to half before the division by the row sum,
// as in the other forms.
constexpr int kRing = 3;
constexpr uint32_t kPBox = 256 * 128;  // [256 queries][64 keys] half: 32 KB
// Q0 Q1 | ring | P (2 boxes) | barriers, tensor-memory slot, per-row factors | alignment.
constexpr uint32_t kPairSmemBytes = 2 * kTile + kRing * kTile + 2 * kPBox + 1280 + 1024;
static_assert(kPairSmemBytes <= 232448, "attention_pair_kernel shared memory");

// Position of K(t) / V(t) in the ring's load order K0 K1 V0 K2 V1 ... V(nt-1).
__device__ __forceinline__ int KPos(int t) { return t == 0 ? 0 : 2 * t - 1; }
__device__ __forceinline__ int VPos(int t, int nt) { return t + 1 < nt ? 2 * t + 2 : 2 * t + 1; }

__global__ void __launch_bounds__(320, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap map_qkv,
                          const __grid_constant__ CUtensorMap map_out, const AttnArgs args) {
  pdl_trigger();
  int seq, tile;
  if (args.items != nullptr) {
    seq = args.items[2 * blockIdx.y];
    tile = args.items[2 * blockIdx.y + 1] & 0xFFFFFF;
  } else {
    seq = blockIdx.y;
    tile = 2 * blockIdx.x;
  }
  const int h = args.items != nullptr ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.z);
  if (seq < 0 || seq >= args.num_seqs) {  // uniform over the CTA, before any barrier
    if (threadIdx.x == 0) atomicOr(args.err, kErrBadArgument);
    return;
  }
  const int start = args.cu_seqlens[seq];
  const int len = args.cu_seqlens[seq + 1] - start;
  const int q0 = tile * kQ;
  if (q0 >= len) return;  // uniform over the CTA, before any barrier
  const int groups = q0 + kQ < len ? 2 : 1;
  const int kvh = h / (args.heads / args.kv_heads);
  const int nt = (len + kKeys - 1) / kKeys;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;                     // [2 tiles] x 32 KB
  uint8_t* ring = q_s + 2 * kTile;         // [3 slots] x 32 KB
  uint8_t* p_s = ring + kRing * kTile;     // [2 key halves] x [256][64] half
  uint64_t* bar = reinterpret_cast<uint64_t*>(p_s + 2 * kPBox);
  uint64_t* q_full = bar;        // [1]
  uint64_t* full = bar + 1;      // [3] ring slot landed
  uint64_t* empty = bar + 4;     // [3] ring slot read by its MMAs
  uint64_t* s_full = bar + 7;    // [2] S_g written
  uint64_t* s_free = bar + 9;    // [2] S_g read by the softmax
  uint64_t* p_full = bar + 11;   // [1] P of every group written
  uint64_t* pv_done = bar + 12;  // [1] an O^T product complete
  uint64_t* o_done = bar + 13;   // [1] the last O^T product complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);
  float* factor = reinterpret_cast<float*>(bar + 32);  // [2][128] rescale factors, then 1 / l

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&s_free[g], 128);
    }
    mbar_init(p_full, static_cast<uint32_t>(128 * groups));
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    fence_mbar_init();
    tma_prefetch_map(&map_qkv);
    tma_prefetch_map(&map_out);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, k, v of the previous kernel are complete

  if (warp == 8) {
    // Producer: lane 0 issues every copy in consumption order.
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, groups * kTile);
      for (int g = 0; g < groups; ++g) {
        tma_load_2d(q_s + g * kTile, &map_qkv, q_full, h * kD, start + q0 + g * kQ);
        tma_load_2d(q_s + g * kTile + kHalfTile, &map_qkv, q_full, h * kD + 64,
                    start + q0 + g * kQ);
      }
      int issued = 0;
      for (int i = 0; i < 2 * nt; ++i) {
        const int slot = i % kRing;
        if (i >= kRing &&
            !mbar_wait(&empty[slot], static_cast<uint32_t>(i / kRing - 1) & 1u, args.err))
          break;
        bool value;
        int kt;
        if (i == 0) {
          value = false, kt = 0;
        } else if (i == 2 * nt - 1) {
          value = true, kt = nt - 1;
        } else if (i & 1) {
          value = false, kt = (i + 1) / 2;
        } else {
          value = true, kt = i / 2 - 1;
        }
        const int col = (value ? args.heads + args.kv_heads + kvh : args.heads + kvh) * kD;
        uint8_t* d = ring + slot * kTile;
        mbar_arrive_expect_tx(&full[slot], kTile);
        tma_load_2d(d, &map_qkv, &full[slot], col, start + kt * kKeys);
        tma_load_2d(d + kHalfTile, &map_qkv, &full[slot], col + 64, start + kt * kKeys);
        ++issued;
      }
      // Let the copies land before the CTA can exit.
      (void)mbar_wait(q_full, 0, args.err);
      for (int i = issued > kRing ? issued - kRing : 0; i < issued; ++i)
        (void)mbar_wait(&full[i % kRing], static_cast<uint32_t>(i / kRing) & 1u, args.err);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kQ, kKeys, 0);
      const uint32_t idesc_o = idesc_f16_f32(kD, static_cast<uint32_t>(kQ * groups), 0, 1);
      const uint32_t qa = smem_u32(q_s);
      const uint32_t pa = smem_u32(p_s);
      auto parity = [](int pos) { return static_cast<uint32_t>(pos / kRing) & 1u; };
      auto issue_s = [&](int g, int t) {
        const uint32_t ka = smem_u32(ring + (KPos(t) % kRing) * kTile);
        const uint32_t d = tmem + static_cast<uint32_t>(g * 128);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfTile + (kk & 3) * 32;
          umma_f16_ss(d, smem_desc_sw128(qa + g * kTile + off, 16, 1024),
                      smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      bool ok = mbar_wait(q_full, 0, args.err) && mbar_wait(&full[0], 0, args.err);
      if (ok) {
        tc_fence_after_sync();
        for (int g = 0; g < groups; ++g) issue_s(g, 0);
        umma_commit(&empty[0]);
      }
      for (int t = 0; ok && t < nt; ++t) {
        if (t + 1 < nt) {
          const int kp = KPos(t + 1);
          ok = mbar_wait(&full[kp % kRing], parity(kp), args.err);
          for (int g = 0; ok && g < groups; ++g) {
            ok = mbar_wait(&s_free[g], static_cast<uint32_t>(t) & 1u, args.err);
            if (!ok) break;
            tc_fence_after_sync();
            issue_s(g, t + 1);  // S_g(t) is in the softmax's registers
          }
          if (!ok) break;
          umma_commit(&empty[kp % kRing]);
        }
        const int vp = VPos(t, nt);
        ok = mbar_wait(p_full, static_cast<uint32_t>(t) & 1u, args.err) &&
             mbar_wait(&full[vp % kRing], parity(vp), args.err);
        if (!ok) break;
        tc_fence_after_sync();
        const uint32_t va = smem_u32(ring + (vp % kRing) * kTile);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          umma_f16_ss(tmem + 256, smem_desc_sw128(va + kk * 16 * 128, kHalfTile, 1024),
                      smem_desc_sw128(pa + (kk >> 2) * kPBox + (kk & 3) * 32, 16, 1024), idesc_o,
                      (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&empty[vp % kRing]);
        if (t == nt - 1) umma_commit(o_done);
      }
    }
  } else if (warp < 4 * groups) {
    // Softmax warpgroup g; a timed-out wait does not end the loop, so every
    // thread keeps meeting the group's named barriers.
    const int g = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of S_g; head-dim lane of O^T
    const uint32_t bar_id = 1 + static_cast<uint32_t>(g);
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + static_cast<uint32_t>(g * 128) + lane_off;
    const uint32_t o_addr = tmem + 256 + static_cast<uint32_t>(g * 128) + lane_off;
    const int prow = g * 128 + r;
    float* fac = factor + g * 128;
    float m = -INFINITY, l = 0.0f;
    for (int t = 0; t < nt; ++t) {
      (void)mbar_wait(&s_full[g], static_cast<uint32_t>(t) & 1u, args.err);
      __syncwarp();
      tc_fence_after_sync();
      uint32_t ka[32], kb[32], kc[32], kd[32];
      tmem_ld_32x32b_x32(s_addr, ka);
      tmem_ld_32x32b_x32(s_addr + 32, kb);
      tmem_ld_32x32b_x32(s_addr + 64, kc);
      tmem_ld_32x32b_x32(s_addr + 96, kd);
      tmem_ld_wait();
      tc_fence_before_sync();
      mbar_arrive(&s_free[g]);  // S_g(t + 1) may overwrite the columns
      const int valid = min(kKeys, len - t * kKeys);
      if (valid < kKeys) {
        mask_keys(ka, 0, valid);
        mask_keys(kb, 32, valid);
        mask_keys(kc, 64, valid);
        mask_keys(kd, 96, valid);
      }
      const float mt =
          fmaxf(fmaxf(max32(ka), max32(kb)), fmaxf(max32(kc), max32(kd))) * args.scale_log2;
      bool grow = false;
      float alpha = 1.0f;
      if (t == 0) {
        m = mt;
      } else if (mt > m + kRescaleThreshold) {
        grow = true;
        alpha = ex2_approx(m - mt);
        m = mt;
      }
      // The group rescales O^T together (each thread owns a head-dim lane
      // of every query's column) when any of its rows raised its maximum.
      const bool rescale = t > 0 && named_barrier_or(bar_id, 128, grow);
      // Probabilities first (the exponentials overlap the tensor core's
      // O^T(t - 1) and S(t + 1)), held packed until the P buffer is free.
      const float neg_m = -m;
      uint32_t pa[16], pb[16], pc[16], pd[16];
      float rowsum = probs32(ka, args.scale_log2, neg_m, pa);
      rowsum += probs32(kb, args.scale_log2, neg_m, pb);
      rowsum += probs32(kc, args.scale_log2, neg_m, pc);
      rowsum += probs32(kd, args.scale_log2, neg_m, pd);
      // O^T(t - 1) complete: the P buffer is free and O^T is stable.
      if (t > 0) {
        (void)mbar_wait(pv_done, static_cast<uint32_t>(t - 1) & 1u, args.err);
        __syncwarp();
        tc_fence_after_sync();
      }
      // P row 128 g + r: keys [0, 64) in box 0, [64, 128) in box 1,
      // 128B-swizzled.
      {
        uint8_t* row0 = p_s + prow * 128;
        const int sw = prow & 7;
        auto put = [&](const uint32_t(&part)[16], int c) {
          uint8_t* row = row0 + (c >> 1) * kPBox;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int piece = (c & 1) * 4 + q;
            *reinterpret_cast<uint4*>(row + ((piece ^ sw) << 4)) =
                make_uint4(part[4 * q], part[4 * q + 1], part[4 * q + 2], part[4 * q + 3]);
          }
        };
        put(pa, 0);
        put(pb, 1);
        put(pc, 2);
        put(pd, 3);
      }
      if (rescale) {
        fac[r] = alpha;
        named_barrier(bar_id, 128);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_addr + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            o[j] = __float_as_uint(__uint_as_float(o[j]) * fac[c * 32 + j]);
          tmem_st_32x32b_x16(o_addr + c * 32, *reinterpret_cast<const uint32_t(*)[16]>(&o[0]));
          tmem_st_32x32b_x16(o_addr + c * 32 + 16,
                             *reinterpret_cast<const uint32_t(*)[16]>(&o[16]));
        }
        tmem_st_wait();
      }
      l = l * alpha + rowsum;
      fence_proxy_async_smem();
      tc_fence_before_sync();
      mbar_arrive(p_full);
    }
    // Epilogue: O^T / l through the group's Q buffer (idle since its last
    // S MMA) as 128B-swizzled [128 queries][64] boxes.
    (void)mbar_wait(o_done, 0, args.err);
    __syncwarp();
    tc_fence_after_sync();
    named_barrier(bar_id, 128);  // the last rescale's factors are read
    fac[r] = 1.0f / l;
    named_barrier(bar_id, 128);
    uint8_t* stage = q_s + g * kTile;
    {
      const int d = r;  // this thread's head-dim lane
      uint8_t* col = stage + (d >> 6) * kHalfTile + ((d & 7) << 1);
      const int piece = (d & 63) >> 3;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(o_addr + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int q = c * 32 + j;
          *reinterpret_cast<__half*>(col + q * 128 + ((piece ^ (q & 7)) << 4)) =
              __float2half_rn(__uint_as_float(o[j]) * fac[q]);
        }
      }
    }
    fence_proxy_async_smem();
    named_barrier(bar_id, 128);
    const int tile_row0 = q0 + g * kQ;
    if (tile_row0 + kQ <= len) {
      if (r == 0) {
        tma_store_2d(&map_out, stage, h * kD, start + tile_row0);
        tma_store_2d(&map_out, stage + kHalfTile, h * kD + 64, start + tile_row0);
        bulk_commit_group();
        bulk_wait_group_read<0>();
      }
    } else if (tile_row0 + r < len) {
      // Last, partial tile: rows past the sequence end belong to the next
      // sequence, so plain stores of the valid rows (thread r: row r).
      __half* dst = args.out + static_cast<int64_t>(start + tile_row0 + r) * args.ld_out + h * kD;
#pragma unroll
      for (int piece = 0; piece < 16; ++piece) {
        const uint8_t* src = stage + (piece >> 3) * kHalfTile + r * 128 +
                             (((piece & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst + piece * 8) = *reinterpret_cast<const uint4*>(src);
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// Tile pairs run attention_kernel<2> (O = P V per tile) unless OV_ATTN_PAIR=t
// selects attention_pair_kernel (O^T = V^T P^T), which measured slower on
// the config-4 step (24.1 ms against 19.4 ms per step of 28 launches).
static bool PairsWithOutputTransposed() {
  const char* env = std::getenv("OV_ATTN_PAIR");
  return env != nullptr && std::strcmp(env, "t") == 0;
}

void ConfigureAttentionKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<2>),
                    static_cast<int>(kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel<4>),
                    static_cast<int>(kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_pair_kernel),
                    static_cast<int>(kPairSmemBytes));
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
  a.num_seqs = num_seqs;
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
  } else if (PairsWithOutputTransposed()) {
    SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_pair_kernel),
                      static_cast<int>(kPairSmemBytes));
    Launch(attention_pair_kernel, grid, dim3(320), kPairSmemBytes, stream,
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
extern "C" int ov_attention_varlen_items(const uint16_t* qkv, size_t ld_qkv, size_t rows,
                                         const int32_t* cu_seqlens, size_t num_seqs,
                                         size_t max_seqlen, const int32_t* items, size_t n_items,
                                         int single_tiles, size_t heads, size_t kv_heads,
                                         size_t head_dim, float scale, uint16_t* out,
                                         size_t ld_out, ov_stream_t stream) {
  return Guard("ov_attention_varlen_items: ", [&] {
    OV_REQUIRE(head_dim == 128, "head_dim must be 128");
    OV_REQUIRE(kv_heads > 0 && heads % kv_heads == 0, "heads must be a multiple of kv_heads");
    OV_REQUIRE(ld_qkv % 8 == 0 && ld_qkv >= (heads + 2 * kv_heads) * head_dim, "qkv stride");
    OV_REQUIRE(ld_out % 8 == 0 && ld_out >= heads * head_dim, "out stride");
    if (rows == 0 || num_seqs == 0 || n_items == 0) return;
    OV_REQUIRE(items != nullptr, "items must not be null");
    OV_REQUIRE(n_items <= 65535u, "too many work items");
    OV_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0, "out must be 16-byte aligned");
    CUtensorMap map, map_out;
    EncodeQkvMap(&map, qkv, static_cast<int64_t>(ld_qkv), static_cast<int64_t>(rows),
                 static_cast<int64_t>((heads + 2 * kv_heads) * head_dim));
    EncodeAttnOutMap(&map_out, out, static_cast<int64_t>(ld_out), static_cast<int64_t>(rows),
                     static_cast<int64_t>(heads * head_dim));
    LaunchAttention(map, map_out, cu_seqlens, static_cast<int>(num_seqs),
                    static_cast<int>(max_seqlen), items, static_cast<int>(n_items),
                    static_cast<int>(heads), static_cast<int>(kv_heads), scale,
                    reinterpret_cast<__half*>(out), static_cast<int64_t>(ld_out),
                    AsStream(stream), single_tiles != 0);
  });
}
