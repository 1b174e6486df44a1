// Bidirectional grouped-query attention over packed variable-length
// sequences on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-sequence attention (generator.cpp:122-172:
// a batched Q K^T GEMM into float32 scores [heads][L][L], SoftmaxKernel
// writing half probabilities, a batched P V GEMM and MergeHeadsKernel) with
// one flash-style kernel: scores never leave the SM.
//
// CTA = (two 128-query tiles of one sequence, query head h); kv head =
// h / (heads / kv_heads).  320 threads:
//   warps 0..3  softmax group 0 (query tile 0), warps 4..7 group 1 (tile 1):
//               thread r owns query row r = tensor-memory lane r.  Per key
//               tile it reads its 128 scores S from tensor memory, keeps a
//               running maximum (raised only when it grows by more than 2^8,
//               rescaling O in tensor memory then), writes the half
//               probabilities P back over its S columns and accumulates the
//               row sum;
//   warp 8      TMA producer: both query tiles once, then K and V tiles of
//               128 keys into a 2-deep ring;
//   warp 9      tensor-memory owner and MMA issuer, one thread.  The two
//               groups ping-pong: while group 0 turns S0 into P0 the tensor
//               core runs group 1's S1 = Q1 K^T; then it runs O0 += P0 V
//               (A operand read from tensor memory, V as an MN-major smem
//               operand) and the next S0 while group 1 works, and so on.
// Tensor memory: group g uses columns [256g, 256g+128) for S / P and
// [256g+128, 256g+256) for O.
// Probabilities are rounded to half before the P V product as in the
// reference (generator_kernels.hip:231-246); unlike the reference they are
// rounded before, not after, the division by the row sum.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kQ = 128;        // queries per group
constexpr int kKeys = 128;     // keys per tile
constexpr int kD = 128;        // head dim
// Softmax warpgroups per CTA: 2 (tile pairs, or one tile split in two
// key halves) or 4 (one tile split in four key quarters); plus a producer
// and an MMA warp.
constexpr int ThreadsOf(int wgs) { return 128 * wgs + 64; }
constexpr uint32_t kHalfTile = 128 * 64 * 2;  // one [128][64] half box: 16 KB
constexpr uint32_t kTile = 2 * kHalfTile;     // [128][128] half: 32 KB
// Q0, Q1 | K, V ring of two stages | barriers, row-statistics exchange.
constexpr uint32_t kSmemBytes = 2 * kTile + 2 * 2 * kTile + 1024 + 8192;
constexpr float kRescaleThreshold = 8.0f;     // log2 units: P stays below 2^8

// 2^x by the MUFU instruction (relative error far below the half rounding
// the probabilities get); 2^-inf = +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Scores of keys at or past `valid` (outside the sequence) become -inf.
__device__ __forceinline__ void mask_keys(uint32_t (&r)[32], int first, int valid) {
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (first + j >= valid) r[j] = 0xFF800000u;
}

__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = fmaxf(__uint_as_float(r[j]), __uint_as_float(r[j + 16]));
#pragma unroll
  for (int w = 8; w > 0; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) v[j] = fmaxf(v[j], v[j + w]);
  return v[0];
}

// p = 2^(s * scale - m) for 32 scores, packed as 16 half pairs; returns the
// sum of the unrounded p.
__device__ __forceinline__ float probs32(const uint32_t (&r)[32], float scale, float neg_m,
                                         uint32_t (&packed)[16]) {
  float a = 0.0f, b = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float p0 = ex2_approx(fmaf(__uint_as_float(r[j]), scale, neg_m));
    const float p1 = ex2_approx(fmaf(__uint_as_float(r[j + 1]), scale, neg_m));
    a += p0;
    b += p1;
    packed[j / 2] = pack_half2(p0, p1);
  }
  return a + b;
}


struct AttnArgs {
  const int32_t* cu_seqlens;
  // [n][2] work items (sequence, first 128-query tile | max groups << 24),
  // one per blockIdx.y with the head in blockIdx.x; or null: sequence
  // blockIdx.y, tiles 2 blockIdx.x and 2 blockIdx.x + 1, head blockIdx.z.
  const int32_t* items;
  __half* out;
  int64_t ld_out;
  int heads;
  int kv_heads;
  float scale_log2;  // softmax scale * log2(e)
  uint32_t* err;
  int single;        // items == null: one 128-query tile per CTA (tile blockIdx.x)
};

// The softmax warpgroups' part of attention_kernel (see there); kParts:
// 1 = each warpgroup owns a query tile, 2 or 4 = kParts warpgroups share
// one query tile, each taking 128 / kParts key columns and O columns.
template <int kParts>
__device__ __forceinline__ void SoftmaxRole(const AttnArgs& args, const CUtensorMap* map_out_p,
                                            uint32_t tmem, uint64_t* s_full, uint64_t* p_full,
                                            uint64_t* o_done, uint64_t* pv_done, float* xmax,
                                            float* xsum,
                                            uint8_t* q_s, int warp, int lane, int len, int nt,
                                            int q0, int start, int h) {
  // Softmax warpgroups (warps 0-3: wg 0, warps 4-7: wg 1); a thread owns
  // one query row (tensor-memory lane).  With two query tiles warpgroup g
  // owns tile g (S/P and O regions g).  With one tile both share it
  // ("split"): warpgroup wg takes key columns [64 wg, 64 wg + 64) of every
  // S tile and O columns [64 wg, 64 wg + 64), and the two halves of a row
  // meet in shared memory for the row maximum and the row sum.
  constexpr bool split = kParts > 1;
  constexpr int kCols = 128 / kParts;   // key columns and O columns per warpgroup
  constexpr int kChunks = kCols / 32;   // 32-column chunks of them
  const int wg = warp >> 2;
  const int g = split ? 0 : wg;
  const int row = (warp & 3) * 32 + lane;
  const int col0 = split ? kCols * wg : 0;  // first key column and first O column
  constexpr int halves = split ? 1 : 2;     // 64-column halves of keys, upper one reloaded
  const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t o_addr = tmem + static_cast<uint32_t>(g * 256 + 128) + lane_off;
  float m = -INFINITY, l = 0.0f;
  // A timed-out wait (error word set) does not end the loop: every warp
  // keeps meeting the named barriers of the split tile and of the epilogue.
  for (int t = 0; t < nt; ++t) {
    // Split: S(t) in region t & 1 (two phases per region); else region g.
    const int sb = split ? (t & 1) : g;
    const uint32_t sphase = split ? static_cast<uint32_t>(t >> 1) & 1u : static_cast<uint32_t>(t) & 1u;
    const uint32_t s_addr = tmem + static_cast<uint32_t>(sb * 256) + lane_off;
    (void)mbar_wait(&s_full[sb], sphase, args.err);
    __syncwarp();  // the tensor-memory accesses below are warp-collective
    tc_fence_after_sync();
    const int valid = min(kKeys, len - t * kKeys);
    // Pass 1: row maximum over this warpgroup's key columns, all held in
    // registers (one tensor-memory round trip per tile) for pass 2; keys
    // past the sequence end read as -inf.  P is written over S columns
    // k / 2 (by this warpgroup in a tile pair, by the other warpgroups of a
    // split tile once all passed the exchange barrier), so no S column is
    // read after it.
    float mt = -INFINITY;
    uint32_t ka[32], kb[kChunks >= 2 ? 32 : 1];
    uint32_t kc[halves == 2 ? 32 : 1], kd[halves == 2 ? 32 : 1];
    if constexpr (halves == 2) {
      tmem_ld_32x32b_x32(s_addr + col0, ka);
      tmem_ld_32x32b_x32(s_addr + col0 + 32, kb);
      tmem_ld_32x32b_x32(s_addr + col0 + 64, kc);
      tmem_ld_32x32b_x32(s_addr + col0 + 96, kd);
      tmem_ld_wait();
      if (valid < kKeys) {
        mask_keys(ka, col0, valid);
        mask_keys(kb, col0 + 32, valid);
        mask_keys(kc, col0 + 64, valid);
        mask_keys(kd, col0 + 96, valid);
      }
      mt = fmaxf(fmaxf(max32(ka), max32(kb)), fmaxf(max32(kc), max32(kd)));
    } else if constexpr (kChunks >= 2) {
      tmem_ld_32x32b_x32(s_addr + col0, ka);
      tmem_ld_32x32b_x32(s_addr + col0 + 32, kb);
      tmem_ld_wait();
      if (valid < kKeys) {
        mask_keys(ka, col0, valid);
        mask_keys(kb, col0 + 32, valid);
      }
      mt = fmaxf(mt, fmaxf(max32(ka), max32(kb)));
    } else {
      tmem_ld_32x32b_x32(s_addr + col0, ka);
      tmem_ld_wait();
      if (valid < kKeys) mask_keys(ka, col0, valid);
      mt = max32(ka);
    }
    if (split) {  // the row's parts meet in shared memory
      float* xm = xmax + (t & 1) * (128 * kParts);
      xm[wg * 128 + row] = mt;
      named_barrier(1, 128 * kParts);
      mt = xm[row];
#pragma unroll
      for (int q = 1; q < kParts; ++q) mt = fmaxf(mt, xm[q * 128 + row]);
    }
    mt *= args.scale_log2;
    // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
    // rescales when any of its rows needs it; rows whose maximum did not
    // grow past the threshold keep theirs (alpha = 1).  Both warpgroups of
    // a split tile see the same maxima, so they decide alike and each
    // rescales its own O columns.  The rescale of O runs after this tile's
    // probabilities are written (the scores' registers are free then) and
    // before P V(t) is signalled.
    bool rescale = false;
    float alpha = 1.0f;
    if (t == 0) {
      m = mt;
    } else {
      const bool grow = mt > m + kRescaleThreshold;
      rescale = __any_sync(0xFFFFFFFFu, grow);
      if (rescale) {
        const float m_new = grow ? mt : m;
        alpha = ex2_approx(m - m_new);
        m = m_new;
      }
    }
    // Pass 2: probabilities, written as half pairs over the consumed S
    // columns (key k -> column k / 2).
    float rowsum = 0.0f;
    const float neg_m = -m;
    if constexpr (kChunks >= 2) {
      uint32_t pa[16], pb[16];
      rowsum += probs32(ka, args.scale_log2, neg_m, pa);
      rowsum += probs32(kb, args.scale_log2, neg_m, pb);
      tmem_st_32x32b_x16(s_addr + col0 / 2, pa);
      tmem_st_32x32b_x16(s_addr + col0 / 2 + 16, pb);
    } else {
      uint32_t pa[16];
      rowsum += probs32(ka, args.scale_log2, neg_m, pa);
      tmem_st_32x32b_x16(s_addr + col0 / 2, pa);
    }
    if constexpr (halves == 2) {
      uint32_t pa[16], pb[16];
      rowsum += probs32(kc, args.scale_log2, neg_m, pa);
      rowsum += probs32(kd, args.scale_log2, neg_m, pb);
      tmem_st_32x32b_x16(s_addr + col0 / 2 + 32, pa);
      tmem_st_32x32b_x16(s_addr + col0 / 2 + 48, pb);
    }
    if (rescale) {
      // Two tiles: the previous P V of this tile completed before S_t was
      // written (one thread issues both, in order), so O is stable here.
      // Split: S(t) may have run before P V(t - 1); wait for it.
      if (split) {
        (void)mbar_wait(pv_done, static_cast<uint32_t>(t - 1) & 1u, args.err);
        __syncwarp();
        tc_fence_after_sync();
      }
      l *= alpha;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_addr + col0 + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
        tmem_st_32x32b_x16(o_addr + col0 + c * 32, *reinterpret_cast<const uint32_t(*)[16]>(&r[0]));
        tmem_st_32x32b_x16(o_addr + col0 + c * 32 + 16,
                           *reinterpret_cast<const uint32_t(*)[16]>(&r[16]));
      }
    }
    l += rowsum;
    tmem_st_wait();
    tc_fence_before_sync();
    mbar_arrive(&p_full[sb]);
  }
  if (split) {  // row sum = the sum of the parts, in part order
    xsum[wg * 128 + row] = l;
    named_barrier(1, 128 * kParts);
    l = xsum[row];
#pragma unroll
    for (int q = 1; q < kParts; ++q) l += xsum[q * 128 + row];
  }
  (void)mbar_wait(&o_done[g], 0, args.err);
  __syncwarp();
  {
    tc_fence_after_sync();
    const float inv = 1.0f / l;
    const int tile_row0 = q0 + g * kQ;
    if (tile_row0 + kQ <= len) {
      // Whole tile: O (half) through the tile's Q buffer, idle since its
      // last S MMA, as 128B-swizzled [128][64] boxes, one TMA store each.
      uint8_t* stage = q_s + g * kTile;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int ocol = col0 + c * 32;  // output column of this chunk
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_addr + ocol, r);
        tmem_ld_wait();
        uint8_t* dst = stage + (ocol >> 6) * kHalfTile + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int piece = ((ocol & 63) >> 3) + q;  // 16-byte piece within the 128-byte row
          *reinterpret_cast<uint4*>(dst + ((piece ^ (row & 7)) << 4)) =
              make_uint4(pack_half2(__uint_as_float(r[8 * q]) * inv, __uint_as_float(r[8 * q + 1]) * inv),
                         pack_half2(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv),
                         pack_half2(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv),
                         pack_half2(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv));
        }
      }
      fence_proxy_async_smem();
      // Each 64-column half is stored once the warpgroups writing it
      // (one for a tile pair or a 2-way split, two for a 4-way split) have.
      constexpr int kWgPerHalf = kParts == 4 ? 2 : 1;
      named_barrier(split ? 2 + (col0 >> 6) : 2 + wg, 128 * kWgPerHalf);
      if (wg % kWgPerHalf == 0 && (warp & 3) == 0 && lane == 0) {
        for (int b = col0 >> 6; b < (col0 >> 6) + halves; ++b)
          tma_store_2d(map_out_p, stage + b * kHalfTile, h * kD + b * 64, start + tile_row0);
        bulk_commit_group();
        bulk_wait_group_read<0>();  // staging read; the writes complete with the grid
      }
    } else {
      // Last, partial tile of a sequence: rows past its end belong to the
      // next sequence, so plain stores of the valid rows.
      const bool store = tile_row0 + row < len;
      __half* dst = args.out + static_cast<int64_t>(start + tile_row0 + row) * args.ld_out + h * kD;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int ocol = col0 + c * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_addr + ocol, r);
        tmem_ld_wait();
        if (store) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(r[j + e]) * inv;
            *reinterpret_cast<uint4*>(dst + ocol + j) =
                make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]),
                           pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
          }
        }
      }
    }
  }
}

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
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_s + 2 * kTile);
  // K and V tiles have their own barriers: a K stage frees when its S
  // MMAs are done, well before the P V that frees the V stage, so the
  // next K tiles load ahead.
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2 stages]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2 groups, or 2 S regions of one tile]
  uint64_t* p_full = bars + 11;   // [2]
  uint64_t* o_done = bars + 13;   // [2 groups]
  uint64_t* pv_done = bars + 15;  // one query tile: each P V complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  float* xmax = reinterpret_cast<float*>(bars + 18);  // [2 tiles][kWG warpgroups][128 rows]
  float* xsum = xmax + 2 * kWG * 128;                 // [kWG warpgroups][128 rows]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      // One query tile: every softmax warpgroup arrives on p_full[i].
      mbar_init(&p_full[i], groups == 1 ? 128 * kWG : 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(pv_done, 1);
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
    // Lane 0 loads Q and the K tiles, lane 1 the V tiles, each into a
    // 2-deep ring; stage t & 1 is refilled once the MMAs reading it are done.
    if (lane < 2) {
      const bool keys = lane == 0;
      const int col = keys ? (args.heads + kvh) * kD : (args.heads + args.kv_heads + kvh) * kD;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      uint8_t* ring = keys ? k_s : v_s;
      if (keys) {
        const int qcol = h * kD;
        mbar_arrive_expect_tx(q_full, groups * kTile);
        for (int g = 0; g < groups; ++g) {
          tma_load_2d(q_s + g * kTile, &map_qkv, q_full, qcol, start + q0 + g * kQ);
          tma_load_2d(q_s + g * kTile + kHalfTile, &map_qkv, q_full, qcol + 64,
                      start + q0 + g * kQ);
        }
      }
      int issued = 0;
      for (int t = 0; t < nt; ++t) {
        const int st = t & 1;
        if (t >= 2 && !mbar_wait(&empty[st], static_cast<uint32_t>((t >> 1) - 1) & 1u, args.err))
          break;
        mbar_arrive_expect_tx(&full[st], kTile);
        const int key0 = start + t * kKeys;
        uint8_t* d = ring + st * kTile;
        tma_load_2d(d, &map_qkv, &full[st], col, key0);
        tma_load_2d(d + kHalfTile, &map_qkv, &full[st], col + 64, key0);
        ++issued;
      }
      // Let this lane's copies land before the CTA can exit.
      if (keys) (void)mbar_wait(q_full, 0, args.err);
      for (int t = issued > 2 ? issued - 2 : 0; t < issued; ++t)
        (void)mbar_wait(&full[t & 1], static_cast<uint32_t>(t >> 1) & 1u, args.err);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kQ, kKeys, 0);
      constexpr uint32_t idesc_o = idesc_f16_f32(kQ, kD, 1);
      const uint32_t qa = smem_u32(q_s);
      // S_g = Q_g K_t^T into the S columns of group g.
      auto issue_s = [&](int g, int t) {
        const uint32_t ka = smem_u32(k_s + (t & 1) * kTile);
        const uint32_t d = tmem + static_cast<uint32_t>(g * 256);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfTile + (kk & 3) * 32;
          umma_f16_ss(d, smem_desc_sw128(qa + g * kTile + off, 16, 1024),
                      smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      // O_g += P_g V_t, P_g read from tensor memory (16 keys = 8 columns).
      auto issue_pv = [&](int g, int t) {
        const uint32_t va = smem_u32(v_s + (t & 1) * kTile);
        const uint32_t p = tmem + static_cast<uint32_t>(g * 256);
        const uint32_t o = p + 128;
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          umma_f16_ts(o, p + static_cast<uint32_t>(kk * 8),
                      smem_desc_sw128(va + kk * 16 * 128, kHalfTile, 1024), idesc_o,
                      (t > 0 || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(q_full, 0, args.err) && mbar_wait(&k_full[0], 0, args.err);
      if (ok && groups == 1) {
        // One query tile: S alternates between the two S/P regions, so
        // S(t + 1) runs on the tensor core while the softmax turns S(t)
        // into P(t).  S(j) reuses region j & 1 once P V(j - 2) was issued
        // (in-order MMAs) and needs K(j); P V(j) needs P(j).  Whichever is
        // ready goes first.
        auto issue_s1 = [&](int t) {
          const uint32_t ka = smem_u32(k_s + (t & 1) * kTile);
          const uint32_t d = tmem + static_cast<uint32_t>((t & 1) * 256);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalfTile + (kk & 3) * 32;
            umma_f16_ss(d, smem_desc_sw128(qa + off, 16, 1024),
                        smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[t & 1]);
          umma_commit(&k_empty[t & 1]);  // K(t) consumed
        };
        auto issue_pv1 = [&](int t) {
          const uint32_t va = smem_u32(v_s + (t & 1) * kTile);
          const uint32_t p = tmem + static_cast<uint32_t>((t & 1) * 256);
          const uint32_t o = tmem + 128;
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk)
            umma_f16_ts(o, p + static_cast<uint32_t>(kk * 8),
                        smem_desc_sw128(va + kk * 16 * 128, kHalfTile, 1024), idesc_o,
                        (t > 0 || kk > 0) ? 1u : 0u);
          umma_commit(pv_done);
          if (t == nt - 1) umma_commit(&o_done[0]);
          umma_commit(&v_empty[t & 1]);  // V(t) consumed
        };
        tc_fence_after_sync();
        issue_s1(0);
        int next_s = 1, next_pv = 0;
        uint64_t idle_since = 0;
        while (next_pv < nt) {
          bool progress = false;
          if (next_s < nt && next_s <= next_pv + 1 &&
              mbar_test_wait(&k_full[next_s & 1], static_cast<uint32_t>(next_s >> 1) & 1u)) {
            tc_fence_after_sync();
            issue_s1(next_s++);
            progress = true;
          }
          if (next_pv < next_s &&
              mbar_test_wait(&p_full[next_pv & 1], static_cast<uint32_t>(next_pv >> 1) & 1u) &&
              mbar_test_wait(&v_full[next_pv & 1], static_cast<uint32_t>(next_pv >> 1) & 1u)) {
            tc_fence_after_sync();
            issue_pv1(next_pv++);
            progress = true;
          }
          if (progress) {
            idle_since = 0;
          } else if (idle_since == 0) {
            idle_since = global_timer_ns();
          } else if (global_timer_ns() - idle_since > kWaitLimitNs) {
            atomicOr(args.err, kErrWaitTimeout);
            break;
          }
        }
        ok = false;  // done: skip the two-tile schedule below
      }
      if (ok) {
        tc_fence_after_sync();
        for (int g = 0; g < groups; ++g) issue_s(g, 0);
        umma_commit(&k_empty[0]);
      }
      for (int t = 0; ok && t < nt; ++t) {
        const bool more = t + 1 < nt;
        for (int g = 0; g < groups; ++g) {
          if (!mbar_wait(&p_full[g], static_cast<uint32_t>(t) & 1u, args.err) ||
              (g == 0 && !mbar_wait(&v_full[t & 1], static_cast<uint32_t>(t >> 1) & 1u, args.err))) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_pv(g, t);
          if (!more) {
            umma_commit(&o_done[g]);
            continue;
          }
          if (g == 0 && !mbar_wait(&k_full[(t + 1) & 1], static_cast<uint32_t>((t + 1) >> 1) & 1u,
                                   args.err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_s(g, t + 1);  // runs after this group's P V (in-order MMAs)
        }
        if (!ok) break;
        umma_commit(&v_empty[t & 1]);
        if (more) umma_commit(&k_empty[(t + 1) & 1]);
      }
    }
  } else if constexpr (kWG == 4) {
    SoftmaxRole<4>(args, &map_out, tmem, s_full, p_full, o_done, pv_done, xmax, xsum, q_s, warp,
                   lane, len, nt, q0, start, h);
  } else {
    if (groups == 1)
      SoftmaxRole<2>(args, &map_out, tmem, s_full, p_full, o_done, pv_done, xmax, xsum, q_s,
                     warp, lane, len, nt, q0, start, h);
    else
      SoftmaxRole<1>(args, &map_out, tmem, s_full, p_full, o_done, pv_done, xmax, xsum, q_s,
                     warp, lane, len, nt, q0, start, h);
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
