// Device building blocks of the tcgen05 flash attention (attention.cu).
//
// One work item = (sequence, one or two 128-query tiles, query head h); kv
// head = h / (heads / kv_heads).  Three roles:
//   softmax     two warpgroups (SoftmaxRole): thread r owns query row r =
//               tensor-memory lane r.  Per key tile it reads its 128 scores
//               S from tensor memory, keeps a running maximum (raised only
//               when it grows by more than 2^8, rescaling O in tensor memory
//               then), writes the half probabilities P back over its S
//               columns and accumulates the row sum;
//   producer    one warp (AttnProduce): lane 0 loads the query tiles once,
//               then the K tiles, lane 1 the V tiles, each into a 2-deep
//               ring with its own barriers;
//   MMA         one thread (AttnIssue).  Two query tiles: the two groups
//               ping-pong (while group 0 turns S0 into P0 the tensor core
//               runs group 1's S1 = Q1 K^T, then O0 += P0 V with P read from
//               tensor memory and V as an MN-major smem operand, and the next
//               S0, and so on).  One query tile: both warpgroups share it
//               (each half of the key columns and of O) and S alternates
//               between two tensor-memory regions, so S(t + 1) runs while
//               the softmax turns S(t) into P(t).
// Tensor memory: group g uses columns [256g, 256g+128) for S / P and
// [256g+128, 256g+256) for O.  Probabilities are rounded to half before the
// P V product as in the reference (generator_kernels.hip:231-246); unlike
// the reference they are rounded before, not after, the division by the
// row sum.
//
// Every mbarrier wait takes its phase as (completions of that barrier in
// earlier work items + uses in this item) & 1, so one set of barriers can
// serve consecutive items of a CTA (AttnPhase tracks the first term, each
// role keeping its own copy; a CTA of the kernel in attention.cu runs one
// item, all counts 0).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "internal.hpp"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kQ = 128;        // queries per group
constexpr int kKeys = 128;     // keys per tile
constexpr int kD = 128;        // head dim
constexpr uint32_t kHalfTile = 128 * 64 * 2;  // one [128][64] half box: 16 KB
constexpr uint32_t kTile = 2 * kHalfTile;     // [128][128] half: 32 KB
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
  int num_seqs;  // entries of cu_seqlens - 1; a work item naming another sequence is skipped
  __half* out;
  int64_t ld_out;
  int heads;
  int kv_heads;
  float scale_log2;  // softmax scale * log2(e)
  uint32_t* err;
  int single;        // items == null: one 128-query tile per CTA (tile blockIdx.x)
};

// The barriers of one work item (shared memory).
struct AttnBars {
  uint64_t* q_full;   // [1] query tiles landed
  uint64_t* k_full;   // [2] K stage landed
  uint64_t* k_empty;  // [2] K stage read by its S MMAs
  uint64_t* v_full;   // [2]
  uint64_t* v_empty;  // [2] V stage read by its P V MMAs
  uint64_t* s_full;   // [2] S of group g (two tiles) or of region t & 1 (one tile)
  uint64_t* p_full;   // [2] P written over S
  uint64_t* o_done;   // [2] last P V of group g complete
  uint64_t* pv_done;  // [1] one tile: each P V complete
};

// Parity of the completions each barrier saw in earlier work items.
struct AttnPhase {
  enum : int {
    kQFull = 0, kKFull = 1, kKEmpty = 3, kVFull = 5, kVEmpty = 7, kSFull = 9, kPFull = 11,
    kODone = 13, kPvDone = 15
  };
  uint32_t bits = 0;
  __device__ __forceinline__ uint32_t operator()(int bar) const { return (bits >> bar) & 1u; }
  // After an item of `nt` key tiles and `groups` query tiles.
  __device__ __forceinline__ void Advance(int nt, int groups) {
    auto flip = [&](int bar, int count) { bits ^= static_cast<uint32_t>(count & 1) << bar; };
    const int n0 = (nt + 1) / 2, n1 = nt / 2;  // key tiles in ring stage 0 / 1
    flip(kQFull, 1);
    flip(kKFull, n0);
    flip(kKFull + 1, n1);
    flip(kKEmpty, n0);
    flip(kKEmpty + 1, n1);
    flip(kVFull, n0);
    flip(kVFull + 1, n1);
    flip(kVEmpty, n0);
    flip(kVEmpty + 1, n1);
    if (groups == 2) {
      flip(kSFull, nt);
      flip(kSFull + 1, nt);
      flip(kPFull, nt);
      flip(kPFull + 1, nt);
      flip(kODone, 1);
      flip(kODone + 1, 1);
    } else {
      flip(kSFull, n0);
      flip(kSFull + 1, n1);
      flip(kPFull, n0);
      flip(kPFull + 1, n1);
      flip(kODone, 1);
      flip(kPvDone, nt);
    }
  }
};

// Initial counts of the barriers (one thread, before any use).
__device__ __forceinline__ void InitAttnBars(const AttnBars& b, int softmax_threads_per_p) {
  mbar_init(b.q_full, 1);
  for (int i = 0; i < 2; ++i) {
    mbar_init(&b.k_full[i], 1);
    mbar_init(&b.k_empty[i], 1);
    mbar_init(&b.v_full[i], 1);
    mbar_init(&b.v_empty[i], 1);
    mbar_init(&b.s_full[i], 1);
    mbar_init(&b.p_full[i], static_cast<uint32_t>(softmax_threads_per_p));
    mbar_init(&b.o_done[i], 1);
  }
  mbar_init(b.pv_done, 1);
}

// The softmax warpgroups' part of a work item; kParts: 1 = each warpgroup
// owns a query tile, 2 or 4 = kParts warpgroups share one query tile, each
// taking 128 / kParts key columns and O columns.  wg: this thread's
// warpgroup; quarter: its warp's tensor-memory lane quarter (warp index
// % 4).  bar_base: three consecutive named-barrier ids this role may use.
// Each thread arrives `p_arrive` times on p_full per key tile (p_full's
// count / the threads that share the tile).  The output goes through the
// query tiles' shared memory (idle after the last S MMA) by TMA store.
template <int kParts>
__device__ __forceinline__ void SoftmaxRole(const AttnArgs& args, const CUtensorMap* map_out_p,
                                            uint32_t tmem, const AttnBars& bars,
                                            const AttnPhase& ph, float* xmax, float* xsum,
                                            uint8_t* q_s, int wg, int quarter, int lane, int len,
                                            int nt, int q0, int start, int h, uint32_t bar_base,
                                            uint32_t p_arrive) {
  // With two query tiles warpgroup g owns tile g (S/P and O regions g).
  // With one tile the warpgroups share it ("split"): warpgroup wg takes
  // key columns [kCols wg, kCols (wg + 1)) of every S tile and O columns
  // alike, and the parts of a row meet in shared memory for the row
  // maximum and the row sum.
  constexpr bool split = kParts > 1;
  constexpr int kCols = 128 / kParts;   // key columns and O columns per warpgroup
  constexpr int kChunks = kCols / 32;   // 32-column chunks of them
  const int g = split ? 0 : wg;
  const int row = quarter * 32 + lane;
  const int col0 = split ? kCols * wg : 0;  // first key column and first O column
  constexpr int halves = split ? 1 : 2;     // 64-column halves of keys, upper one reloaded
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t o_addr = tmem + static_cast<uint32_t>(g * 256 + 128) + lane_off;
  float m = -INFINITY, l = 0.0f;
  // A timed-out wait (error word set) does not end the loop: every warp
  // keeps meeting the named barriers of the split tile and of the epilogue.
  for (int t = 0; t < nt; ++t) {
    // Split: S(t) in region t & 1 (two phases per region); else region g.
    const int sb = split ? (t & 1) : g;
    const uint32_t sphase =
        ph(AttnPhase::kSFull + sb) ^ (split ? static_cast<uint32_t>(t >> 1) & 1u
                                            : static_cast<uint32_t>(t) & 1u);
    const uint32_t s_addr = tmem + static_cast<uint32_t>(sb * 256) + lane_off;
    (void)mbar_wait(&bars.s_full[sb], sphase, args.err);
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
      named_barrier(bar_base, 128 * kParts);
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
        (void)mbar_wait(bars.pv_done,
                        ph(AttnPhase::kPvDone) ^ (static_cast<uint32_t>(t - 1) & 1u), args.err);
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
    mbar_arrive_cnt(&bars.p_full[sb], p_arrive);
  }
  if (split) {  // row sum = the sum of the parts, in part order
    xsum[wg * 128 + row] = l;
    named_barrier(bar_base, 128 * kParts);
    l = xsum[row];
#pragma unroll
    for (int q = 1; q < kParts; ++q) l += xsum[q * 128 + row];
  }
  (void)mbar_wait(&bars.o_done[g], ph(AttnPhase::kODone + g), args.err);
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
      named_barrier(split ? bar_base + 1 + (col0 >> 6) : bar_base + 1 + wg, 128 * kWgPerHalf);
      if (wg % kWgPerHalf == 0 && quarter == 0 && lane == 0) {
        for (int b = col0 >> 6; b < (col0 >> 6) + halves; ++b)
          tma_store_2d(map_out_p, stage + b * kHalfTile, h * kD + b * 64, start + tile_row0);
        bulk_commit_group();
        bulk_wait_group_read<0>();  // staging read; the writes complete later
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

// The producer warp's part of a work item: lane 0 loads the query tiles
// and the K tiles, lane 1 the V tiles, each into a 2-deep ring; stage
// t & 1 is refilled once the MMAs reading it are done.  Each lane lets its
// copies land before returning.
__device__ __forceinline__ void AttnProduce(const AttnArgs& args, const CUtensorMap* map_qkv,
                                            const AttnBars& bars, const AttnPhase& ph,
                                            uint8_t* q_s, uint8_t* k_s, uint8_t* v_s, int lane,
                                            int start, int q0, int groups, int nt, int h,
                                            int kvh) {
  if (lane >= 2) return;
  const bool keys = lane == 0;
  const int col = keys ? (args.heads + kvh) * kD : (args.heads + args.kv_heads + kvh) * kD;
  uint64_t* full = keys ? bars.k_full : bars.v_full;
  uint64_t* empty = keys ? bars.k_empty : bars.v_empty;
  const int full_bit = keys ? AttnPhase::kKFull : AttnPhase::kVFull;
  const int empty_bit = keys ? AttnPhase::kKEmpty : AttnPhase::kVEmpty;
  uint8_t* ring = keys ? k_s : v_s;
  if (keys) {
    const int qcol = h * kD;
    mbar_arrive_expect_tx(bars.q_full, groups * kTile);
    for (int g = 0; g < groups; ++g) {
      tma_load_2d(q_s + g * kTile, map_qkv, bars.q_full, qcol, start + q0 + g * kQ);
      tma_load_2d(q_s + g * kTile + kHalfTile, map_qkv, bars.q_full, qcol + 64,
                  start + q0 + g * kQ);
    }
  }
  int issued = 0;
  for (int t = 0; t < nt; ++t) {
    const int st = t & 1;
    if (t >= 2 && !mbar_wait(&empty[st],
                             ph(empty_bit + st) ^ (static_cast<uint32_t>((t >> 1) - 1) & 1u),
                             args.err))
      break;
    mbar_arrive_expect_tx(&full[st], kTile);
    const int key0 = start + t * kKeys;
    uint8_t* d = ring + st * kTile;
    tma_load_2d(d, map_qkv, &full[st], col, key0);
    tma_load_2d(d + kHalfTile, map_qkv, &full[st], col + 64, key0);
    ++issued;
  }
  // Let this lane's copies land before the CTA can exit.
  if (keys) (void)mbar_wait(bars.q_full, ph(AttnPhase::kQFull), args.err);
  for (int t = issued > 2 ? issued - 2 : 0; t < issued; ++t)
    (void)mbar_wait(&full[t & 1], ph(full_bit + (t & 1)) ^ (static_cast<uint32_t>(t >> 1) & 1u),
                    args.err);
}

// The MMA thread's part of a work item (see the file comment for the two
// schedules).  Returns false when a bounded wait gave up.
__device__ __forceinline__ bool AttnIssue(const AttnArgs& args, uint32_t tmem, const AttnBars& bars,
                                          const AttnPhase& ph, uint8_t* q_s, uint8_t* k_s,
                                          uint8_t* v_s, int groups, int nt) {
  constexpr uint32_t idesc_s = idesc_f16_f32(kQ, kKeys, 0);
  constexpr uint32_t idesc_o = idesc_f16_f32(kQ, kD, 1);
  const uint32_t qa = smem_u32(q_s);
  auto kphase = [&](int t) {
    return ph(AttnPhase::kKFull + (t & 1)) ^ (static_cast<uint32_t>(t >> 1) & 1u);
  };
  auto vphase = [&](int t) {
    return ph(AttnPhase::kVFull + (t & 1)) ^ (static_cast<uint32_t>(t >> 1) & 1u);
  };
  bool ok = mbar_wait(bars.q_full, ph(AttnPhase::kQFull), args.err) &&
            mbar_wait(&bars.k_full[0], kphase(0), args.err);
  if (!ok) return false;
  if (groups == 1) {
    // One query tile: S alternates between the two S/P regions, so
    // S(t + 1) runs on the tensor core while the softmax turns S(t) into
    // P(t).  S(j) reuses region j & 1 once P V(j - 2) was issued (in-order
    // MMAs) and needs K(j); P V(j) needs P(j).  Whichever is ready goes
    // first.
    auto issue_s1 = [&](int t) {
      const uint32_t ka = smem_u32(k_s + (t & 1) * kTile);
      const uint32_t d = tmem + static_cast<uint32_t>((t & 1) * 256);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kHalfTile + (kk & 3) * 32;
        umma_f16_ss(d, smem_desc_sw128(qa + off, 16, 1024), smem_desc_sw128(ka + off, 16, 1024),
                    idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(&bars.s_full[t & 1]);
      umma_commit(&bars.k_empty[t & 1]);  // K(t) consumed
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
      umma_commit(bars.pv_done);
      if (t == nt - 1) umma_commit(&bars.o_done[0]);
      umma_commit(&bars.v_empty[t & 1]);  // V(t) consumed
    };
    tc_fence_after_sync();
    issue_s1(0);
    int next_s = 1, next_pv = 0;
    uint64_t idle_since = 0;
    while (next_pv < nt) {
      bool progress = false;
      if (next_s < nt && next_s <= next_pv + 1 &&
          mbar_test_wait(&bars.k_full[next_s & 1], kphase(next_s))) {
        tc_fence_after_sync();
        issue_s1(next_s++);
        progress = true;
      }
      if (next_pv < next_s &&
          mbar_test_wait(&bars.p_full[next_pv & 1],
                         ph(AttnPhase::kPFull + (next_pv & 1)) ^
                             (static_cast<uint32_t>(next_pv >> 1) & 1u)) &&
          mbar_test_wait(&bars.v_full[next_pv & 1], vphase(next_pv))) {
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
        return false;
      }
    }
    return true;
  }
  // Two query tiles.
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
    umma_commit(&bars.s_full[g]);
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
  tc_fence_after_sync();
  for (int g = 0; g < groups; ++g) issue_s(g, 0);
  umma_commit(&bars.k_empty[0]);
  for (int t = 0; t < nt; ++t) {
    const bool more = t + 1 < nt;
    for (int g = 0; g < groups; ++g) {
      if (!mbar_wait(&bars.p_full[g], ph(AttnPhase::kPFull + g) ^ (static_cast<uint32_t>(t) & 1u),
                     args.err) ||
          (g == 0 && !mbar_wait(&bars.v_full[t & 1], vphase(t), args.err)))
        return false;
      tc_fence_after_sync();
      issue_pv(g, t);
      if (!more) {
        umma_commit(&bars.o_done[g]);
        continue;
      }
      if (g == 0 && !mbar_wait(&bars.k_full[(t + 1) & 1], kphase(t + 1), args.err)) return false;
      tc_fence_after_sync();
      issue_s(g, t + 1);  // runs after this group's P V (in-order MMAs)
    }
    umma_commit(&bars.v_empty[t & 1]);
    if (more) umma_commit(&bars.k_empty[(t + 1) & 1]);
  }
  return true;
}

}  // namespace
}  // namespace ovb
