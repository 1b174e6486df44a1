// Device building blocks of the tcgen05 GEMM kernel (gemm.cu): tile
// constants, the output-tile walk, the fused epilogues (float32 store or
// residual reduce-add, SwiGLU, QK RMSNorm + RoPE) and the split-K partial
// exchange through a global workspace.  See gemm.cu for the kernel that
// drives them.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.hpp"
#include "internal.hpp"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 320;  // producer warp, MMA warp, 8 epilogue warps
constexpr int kRingBytes = 196608;
constexpr uint32_t kStageTile = 128 * 128;  // one staging tile: 128 rows x 128 bytes
constexpr int kGroupM = 8;                  // rasterisation group of m tiles

// PAIR: a CTA pair runs 256-row tiles with cta_group::2 MMAs; each CTA
// loads its 128 rows of A and half (BN / 2 rows) of the B tile.
template <int BN, int EPI, bool PAIR = false>
struct TileConfig {
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = (PAIR ? BN / 2 : BN) * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kRingBytes / kStageBytes;
  static constexpr uint32_t kNormFloats = EPI == OV_EPI_QKNORM_ROPE_F16 ? 256 : 0;
  static constexpr size_t kSmemBytes =
      static_cast<size_t>(kStages) * kStageBytes + 2 * kStageTile + kNormFloats * 4 + 1024 + 512;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// silu(g) * u with the hardware exponential and a fast divide: both are
// accurate to a few float32 ulps, far below the half rounding that follows
// (generator_kernels.hip:196-198 computes g / (1 + exp(-g)) * u).  For
// g < -88 the exponential overflows and __fdividef returns 0, the limit.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// Shared-memory 16-byte load kept in program order with the tensor-memory
// loads around it (a volatile asm): the compiler does not hoist a head's
// worth of norm weights into registers ahead of use.
__device__ __forceinline__ float4 lds_in_order(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// Unit u -> (m tile, n tile, split).  Tiles are visited in groups of
// kGroupM m tiles, all n tiles of a group before the next group, so a
// group's activations stay in L2 while the weights stream past.
__device__ __forceinline__ void UnitCoords(const GemmArgs& a, int u, int& m_tile, int& n_tile,
                                           int& split) {
  const int tile = u / a.splits;
  split = u - tile * a.splits;
  const int per_group = kGroupM * a.num_n;
  const int g = tile / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(kGroupM, a.num_m - first_m);
  const int local = tile - g * per_group;
  n_tile = local / gm;
  m_tile = first_m + local % gm;
}

// Epilogue state.  Eight epilogue warps form two groups of four; each
// group has one thread per tile row (tensor-memory lane) and the groups
// split each tile's columns, so every SM sub-partition runs two epilogue
// warps.
struct EpilogueCtx {
  uint8_t* staging;      // 2 x kStageTile, 1024-byte aligned
  uint32_t chunk_iter;   // chunks this group staged (non-ring mode)
  uint32_t joint_iter;   // chunks both groups staged together (non-ring mode)
  int ep;                // 0..255
  int gep;               // 0..127: index within the group; 0 leads the group
  int group;             // 0 or 1
  int row;               // tile row = tensor-memory lane
  // Last unit of this CTA: the operand ring is idle (every load consumed,
  // every MMA complete), so each chunk takes its own kStageTile slot of it
  // and no chunk waits for an earlier store to drain.
  uint8_t* ring;         // nullptr: stage through the two staging tiles
};

constexpr uint32_t kGroupBarrier = 1;  // + group: the 128 threads of a group
constexpr uint32_t kEpiBarrier = 3;    // all 256 epilogue threads

// RoPE cos / sin of one row's position for the 32 rotated pairs this
// group computes (QK-norm epilogue), loaded before the accumulator is
// ready so the loads overlap the tile's MMAs.
struct RopeRow {
  float4 c[8];
  float4 s[8];
};

template <int EPI>
__device__ __forceinline__ void LoadRopeRow(const GemmArgs& a, int m_tile, int row, int group,
                                            RopeRow& r) {
  if constexpr (EPI == OV_EPI_QKNORM_ROPE_F16) {
    const int64_t grow = static_cast<int64_t>(m_tile) * kBM + row;
    int pos = grow < a.M ? __ldg(a.positions + grow) : 0;
    if (pos < 0 || pos >= a.max_positions) {
      atomicOr(a.err, kErrBadArgument);
      pos = 0;
    }
    const float4* cs =
        reinterpret_cast<const float4*>(a.rope_cos + static_cast<int64_t>(pos) * 64) + 8 * group;
    const float4* sn =
        reinterpret_cast<const float4*>(a.rope_sin + static_cast<int64_t>(pos) * 64) + 8 * group;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      r.c[k] = __ldg(cs + k);
      r.s[k] = __ldg(sn + k);
    }
  }
}

__device__ __forceinline__ float F4At(const float4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// One group writes its threads' 128-byte row pieces into a staging tile
// (ring slot `slot`, or the group's staging tile) and the group leader
// stores (or reduce-adds) the tile at column x, row y0.
template <bool kReduce>
__device__ __forceinline__ void EmitGroup(EpilogueCtx& c, const CUtensorMap* map,
                                          const uint32_t (&w)[32], int x, int y0, int slot) {
  uint8_t* buf;
  const uint32_t bar = kGroupBarrier + static_cast<uint32_t>(c.group);
  if (c.ring != nullptr) {
    buf = c.ring + slot * kStageTile;
  } else {
    buf = c.staging + c.group * kStageTile;
    if (c.chunk_iter > 0 && c.gep == 0) bulk_wait_group_read<0>();
    named_barrier(bar, 128);  // the group's staging tile is free again
  }
  uint8_t* dst = buf + c.row * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<uint4*>(dst + ((q ^ (c.row & 7)) << 4)) =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  fence_proxy_async_smem();
  named_barrier(bar, 128);
  if (c.gep == 0) {
    if (kReduce)
      tma_reduce_add_2d(map, buf, x, y0);
    else
      tma_store_2d(map, buf, x, y0);
    bulk_commit_group();
  }
  ++c.chunk_iter;
}

// Both groups fill one staging tile, group g the 64-byte half g of every
// row piece (16 words); thread 0 stores it at column x, row y0.
__device__ __forceinline__ void EmitJoint(EpilogueCtx& c, const CUtensorMap* map,
                                          const uint32_t (&w)[16], int x, int y0, int slot) {
  uint8_t* buf;
  if (c.ring != nullptr) {
    buf = c.ring + slot * kStageTile;
  } else {
    buf = c.staging + (c.joint_iter & 1u) * kStageTile;
    if (c.joint_iter >= 2 && c.ep == 0) bulk_wait_group_read<1>();
    named_barrier(kEpiBarrier, 256);
  }
  uint8_t* dst = buf + c.row * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(dst + (((4 * c.group + q) ^ (c.row & 7)) << 4)) =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  fence_proxy_async_smem();
  named_barrier(kEpiBarrier, 256);
  if (c.ep == 0) {
    tma_store_2d(map, buf, x, y0);
    bulk_commit_group();
  }
  ++c.joint_iter;
}

template <int BN, int EPI>
__device__ __forceinline__ void EpilogueUnit(const GemmArgs& a, const CUtensorMap* map_y,
                                             EpilogueCtx& c, uint32_t tacc, int m_tile,
                                             int n_tile, const float* norm_w,
                                             const RopeRow& rope) {
  const int y0 = m_tile * kBM;
  if constexpr (EPI == OV_EPI_STORE_F32 || EPI == OV_EPI_ACCUM_F32) {
    // 32-column chunks; group g takes the chunks k with k % 2 == g.
    const int chunks = min(BN, a.out_cols - n_tile * BN + 31) / 32;  // >= 1
    if (c.ring != nullptr) {
      // Each chunk into its own ring slot, the tensor-memory load of the
      // group's next chunk in flight while this one is written; one
      // barrier, then the group leader issues the group's stores.
      const uint32_t bar = kGroupBarrier + static_cast<uint32_t>(c.group);
      uint32_t r[2][32];
      int issued = 0;
      if (c.group < chunks) {
        tmem_ld_32x32b_x32(tacc + c.group * 32, r[0]);
        tmem_ld_wait();
      }
#pragma unroll
      for (int i = 0; i < BN / 64; ++i) {
        const int k = 2 * i + c.group;
        if (k >= chunks) break;  // uniform over the group
        const int kn = k + 2;
        if (kn < chunks) tmem_ld_32x32b_x32(tacc + kn * 32, r[(i + 1) & 1]);
        uint8_t* dst = c.ring + k * kStageTile + c.row * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<uint4*>(dst + ((q ^ (c.row & 7)) << 4)) =
              make_uint4(r[i & 1][4 * q], r[i & 1][4 * q + 1], r[i & 1][4 * q + 2],
                         r[i & 1][4 * q + 3]);
        ++issued;
        if (kn < chunks) tmem_ld_wait();
      }
      fence_proxy_async_smem();
      named_barrier(bar, 128);
      if (c.gep == 0 && issued > 0) {
        for (int k = c.group; k < chunks; k += 2) {
          const uint8_t* buf = c.ring + k * kStageTile;
          if (EPI == OV_EPI_ACCUM_F32)
            tma_reduce_add_2d(map_y, buf, n_tile * BN + k * 32, y0);
          else
            tma_store_2d(map_y, buf, n_tile * BN + k * 32, y0);
        }
        bulk_commit_group();
      }
    } else {
#pragma unroll 1
      for (int k = c.group; k < chunks; k += 2) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tacc + k * 32, r);
        tmem_ld_wait();
        EmitGroup<EPI == OV_EPI_ACCUM_F32>(c, map_y, r, n_tile * BN + k * 32, y0, k);
      }
    }
  } else if constexpr (EPI == OV_EPI_SWIGLU_F16) {
    // The tile holds BN / 128 groups of [64 gate | 64 up] columns; each
    // gives 64 half outputs = one 128-byte row piece.  Epilogue group g
    // takes the gate/up groups gi with gi % 2 == g.
    constexpr int G = OV_SWIGLU_GROUP;
#pragma unroll 1
    for (int gi = c.group; gi < BN / (2 * G); gi += 2) {
      uint32_t out[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t g[32], u[32];
        tmem_ld_32x32b_x32(tacc + gi * 2 * G + h * 32, g);
        tmem_ld_32x32b_x32(tacc + gi * 2 * G + G + h * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          out[h * 16 + j / 2] =
              pack_half2(silu_mul(__uint_as_float(g[j]), __uint_as_float(u[j])),
                         silu_mul(__uint_as_float(g[j + 1]), __uint_as_float(u[j + 1])));
      }
      EmitGroup<false>(c, map_y, out, n_tile * (BN / 2) + gi * G, y0, gi);
    }
  } else if constexpr (EPI == OV_EPI_QKNORM_ROPE_F16) {
    // BN / 128 heads per tile.  Group g computes the rotated pairs
    // (i, i + 64) for i in [32 g, 32 g + 32) of every head: the low 64-byte
    // half (g = 0) or the high half (g = 1) of both output row pieces.
    // Each group reads the whole head once for its RMS.
    static_assert(BN % 128 == 0, "whole heads per tile");
    const int i_base = 32 * c.group;
#pragma unroll 1
    for (int hh = 0; hh < BN / 128; ++hh) {
      const int slot = n_tile * (BN / 128) + hh;
      const uint32_t th = tacc + hh * 128;
      if (slot < a.heads + a.kv_heads) {
        const float* w = norm_w + (slot < a.heads ? 0 : 128);
        // RMS of the head: four 16-column loads in flight per wait.
        float ss = 0.0f;
#pragma unroll
        for (int q4 = 0; q4 < 8; q4 += 4) {
          uint32_t r[4][16];
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld_32x32b_x16(th + (q4 + q) * 16, r[q]);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int j = 0; j < 16; ++j)
              ss = fmaf(__uint_as_float(r[q][j]), __uint_as_float(r[q][j]), ss);
        }
        const float scale = 1.0f / sqrtf(ss / 128.0f + a.epsilon);
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int b = 0; b < 2; ++b) {  // pairs i_base + 16 b .. + 15
          const int i0 = i_base + 16 * b;
          uint32_t r1[16], r2[16];
          tmem_ld_32x32b_x16(th + i0, r1);
          tmem_ld_32x32b_x16(th + 64 + i0, r2);
          tmem_ld_wait();
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float4 w14 = lds_in_order(w + i0 + i4 * 4);
            const float4 w24 = lds_in_order(w + 64 + i0 + i4 * 4);
            float l4[4], h4[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int k = 4 * b + i4;  // RopeRow index of pair i0 + 4 i4 + t
              const float cc = F4At(rope.c[k], t);
              const float sn = F4At(rope.s[k], t);
              const float x1 = F4At(w14, t) * (__uint_as_float(r1[i4 * 4 + t]) * scale);
              const float x2 = F4At(w24, t) * (__uint_as_float(r2[i4 * 4 + t]) * scale);
              l4[t] = __fsub_rn(__fmul_rn(x1, cc), __fmul_rn(x2, sn));
              h4[t] = __fadd_rn(__fmul_rn(x2, cc), __fmul_rn(x1, sn));
            }
            const int o = 8 * b + 2 * i4;
            lo[o] = pack_half2(l4[0], l4[1]);
            lo[o + 1] = pack_half2(l4[2], l4[3]);
            hi[o] = pack_half2(h4[0], h4[1]);
            hi[o + 1] = pack_half2(h4[2], h4[3]);
          }
        }
        EmitJoint(c, map_y, lo, slot * 128, y0, 2 * hh);
        EmitJoint(c, map_y, hi, slot * 128 + 64, y0, 2 * hh + 1);
      } else {
        // v heads: plain half conversion of this group's columns.
        uint32_t lo[16], hi[16];
        uint32_t r1[32], r2[32];
        tmem_ld_32x32b_x32(th + i_base, r1);
        tmem_ld_32x32b_x32(th + 64 + i_base, r2);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          lo[j] = pack_half2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1]));
          hi[j] = pack_half2(__uint_as_float(r2[2 * j]), __uint_as_float(r2[2 * j + 1]));
        }
        EmitJoint(c, map_y, lo, slot * 128, y0, 2 * hh);
        EmitJoint(c, map_y, hi, slot * 128 + 64, y0, 2 * hh + 1);
      }
    }
  }
}

// Cluster split-K.  After every CTA of the cluster has finished its MMAs
// (a cluster barrier), the idle operand ring of each CTA holds an inbox of
// S - 1 slots followed by an outbox of S - 1 slots, each [128 rows][BN / S]
// floats with 16-byte pieces XOR-swizzled by row.  Rank r owns column slice
// r of the tile.

// Slot of rank `other` among the S - 1 ranks other than `self`.
__device__ __forceinline__ int PeerSlot(int other, int self) { return other < self ? other : other - 1; }

// Step 1: every other rank's slice of this CTA's partial goes from tensor
// memory into the outbox (the two epilogue groups take alternate 32-column
// chunks); then one thread sends each outbox slot to its rank's inbox with
// a bulk copy that completes on that rank's inbox barrier.
template <int BN>
__device__ __forceinline__ void ClusterSend(uint32_t tacc, uint8_t* ring, const EpilogueCtx& c,
                                            int rank, int splits, uint64_t* inbox_bar) {
  const int cols = BN / splits;
  const uint32_t slot_bytes = static_cast<uint32_t>(kBM * cols * 4);
  uint8_t* outbox = ring + (splits - 1) * slot_bytes;
  int chunk = 0;
#pragma unroll 1
  for (int j = 0; j < splits; ++j) {
    if (j == rank) continue;
    uint8_t* slot = outbox + PeerSlot(j, rank) * slot_bytes;
#pragma unroll 1
    for (int cc = 0; cc < cols; cc += 32, ++chunk) {
      if ((chunk & 1) != c.group) continue;  // uniform over the group
      uint32_t v[32];
      tmem_ld_32x32b_x32(tacc + static_cast<uint32_t>(j * cols + cc), v);
      tmem_ld_wait();
      uint8_t* dst = slot + (c.row * cols + cc) * 4;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(dst + ((q ^ (c.row & 7)) << 4)) =
            make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  fence_proxy_async_smem();
  named_barrier(kEpiBarrier, 256);
  if (c.ep == 0) {
    const uint32_t inbox = smem_u32(ring);
    for (int j = 0; j < splits; ++j) {
      if (j == rank) continue;
      const uint32_t src = smem_u32(outbox + PeerSlot(j, rank) * slot_bytes);
      const uint32_t dst = mapa_shared(inbox + PeerSlot(rank, j) * slot_bytes, j);
      bulk_copy_to_peer(dst, src, slot_bytes, mapa_shared(smem_u32(inbox_bar), j));
    }
  }
}

// Step 2: this rank's slice is the sum of the splits' partials in split
// order (its own from tensor memory, the others from the inbox), stored or
// added into y like an unsplit tile; group g takes the chunks cc / 32 with
// the parity g.
template <int BN, int EPI>
__device__ __forceinline__ void ClusterReduce(const GemmArgs& a, const CUtensorMap* map_y,
                                              EpilogueCtx& c, uint32_t tacc, const uint8_t* ring,
                                              int m_tile, int n_tile, int rank) {
  const int splits = a.splits;
  const int cols = BN / splits;
  const int slot_bytes = kBM * cols * 4;
  const int y0 = m_tile * kBM;
#pragma unroll 1
  for (int cc = 32 * c.group; cc < cols; cc += 64) {
    const int x = n_tile * BN + rank * cols + cc;
    if (x >= a.out_cols) break;  // uniform over the group
    float acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
#pragma unroll 1
    for (int j = 0; j < splits; ++j) {
      if (j == rank) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tacc + static_cast<uint32_t>(rank * cols + cc), v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] += __uint_as_float(v[e]);
      } else {
        const uint8_t* src = ring + PeerSlot(j, rank) * slot_bytes + (c.row * cols + cc) * 4;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 t = *reinterpret_cast<const float4*>(src + ((q ^ (c.row & 7)) << 4));
          acc[4 * q] += t.x;
          acc[4 * q + 1] += t.y;
          acc[4 * q + 2] += t.z;
          acc[4 * q + 3] += t.w;
        }
      }
    }
    uint32_t w[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(acc[e]);
    EmitGroup<EPI == OV_EPI_ACCUM_F32>(c, map_y, w, x, y0, 0);
  }
}


// Cluster split-K through global memory (args.xchg set): each rank writes
// the other ranks' column slices of its partial to the workspace, then
// arrives (release, cluster scope) on each peer's inbox barrier; rank r
// waits for the S - 1 arrivals and sums slice r in split order, its own
// part from tensor memory.  No rank writes into another's shared memory,
// so nothing waits for a peer's ring to be free or for its copies to be
// read.  Workspace slot (tile, sender j, slice r): 128 x BN / S floats as
// [32-column chunk][16-byte piece q][row][4 floats], so a warp's accesses
// to one piece are 512 contiguous bytes.
template <int BN, int S>
__device__ __forceinline__ void XchgSend(const GemmArgs& a, uint32_t tacc, const EpilogueCtx& c,
                                         int tile, int rank) {
  constexpr int kCols = BN / S;
  constexpr int kSlot4 = kBM * kCols / 4;  // float4s per slot
  constexpr int kPer = kCols / 32;         // 32-column chunks per slice
  constexpr int kChunks = (S - 1) * kPer;  // chunks sent; group g sends g, g + 2, ...
  float4* base = reinterpret_cast<float4*>(a.xchg) + (static_cast<size_t>(tile) * S + rank) * S * kSlot4;
  // Chunk ch: slice of peer p = ch / kPer (split j = p, or p + 1 past this
  // rank), columns (ch % kPer) * 32 of the slice.
  auto column = [&](int ch) {
    const int p = ch / kPer;
    return (p < rank ? p : p + 1) * kCols + (ch % kPer) * 32;
  };
  uint32_t v[2][32];
  if (c.group < kChunks) {
    tmem_ld_32x32b_x32(tacc + static_cast<uint32_t>(column(c.group)), v[0]);
    tmem_ld_wait();
  }
#pragma unroll
  for (int i = 0; i < (kChunks + 1) / 2; ++i) {
    const int ch = 2 * i + c.group;
    if (ch >= kChunks) break;  // uniform over the group
    const int next = ch + 2;
    if (next < kChunks) tmem_ld_32x32b_x32(tacc + static_cast<uint32_t>(column(next)), v[(i + 1) & 1]);
    const int col = column(ch);
    float4* dst = base + (col / kCols) * kSlot4 + ((col % kCols) / 32) * 8 * kBM + c.row;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      __stcg(dst + q * kBM,
             make_float4(__uint_as_float(v[i & 1][4 * q]), __uint_as_float(v[i & 1][4 * q + 1]),
                         __uint_as_float(v[i & 1][4 * q + 2]), __uint_as_float(v[i & 1][4 * q + 3])));
    if (next < kChunks) tmem_ld_wait();
  }
}

// Adds this rank's own part (from tensor memory) into acc.
__device__ __forceinline__ void AddOwn(float (&acc)[32], uint32_t taddr) {
  uint32_t own[32];
  tmem_ld_32x32b_x32(taddr, own);
  tmem_ld_wait();
#pragma unroll
  for (int e = 0; e < 32; ++e) acc[e] += __uint_as_float(own[e]);
}

template <int BN, int EPI, int S>
__device__ __forceinline__ void XchgReduce(const GemmArgs& a, const CUtensorMap* map_y,
                                           EpilogueCtx& c, uint32_t tacc, int tile, int m_tile,
                                           int n_tile, int rank) {
  constexpr int kCols = BN / S;
  constexpr int kSlot4 = kBM * kCols / 4;
  constexpr int kPeers = S - 1;
  constexpr int kBatch = kPeers < 2 ? kPeers : 2;  // peers' loads in flight together
  const float4* slots =
      reinterpret_cast<const float4*>(a.xchg) + static_cast<size_t>(tile) * S * S * kSlot4;
  const int y0 = m_tile * kBM;
#pragma unroll 1
  for (int cc = 32 * c.group; cc < kCols; cc += 64) {
    const int x = n_tile * BN + rank * kCols + cc;
    if (x >= a.out_cols) break;  // uniform over the group
    const uint32_t own = tacc + static_cast<uint32_t>(rank * kCols + cc);
    float acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
    // Peer p is split j = p (p < rank) or p + 1; the own part goes between
    // peers rank - 1 and rank, so the sum runs in split order.
#pragma unroll
    for (int p0 = 0; p0 < kPeers; p0 += kBatch) {
      float4 t[kBatch][8];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int p = p0 + b;
        if (p >= kPeers) break;
        const int j = p < rank ? p : p + 1;
        const float4* src = slots + (j * S + rank) * kSlot4 + (cc / 32) * 8 * kBM + c.row;
#pragma unroll
        for (int q = 0; q < 8; ++q) t[b][q] = __ldcg(src + q * kBM);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int p = p0 + b;
        if (p >= kPeers) break;
        if (p == rank) AddOwn(acc, own);  // uniform over the CTA
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          acc[4 * q] += t[b][q].x;
          acc[4 * q + 1] += t[b][q].y;
          acc[4 * q + 2] += t[b][q].z;
          acc[4 * q + 3] += t[b][q].w;
        }
      }
    }
    if (rank == kPeers) AddOwn(acc, own);
    uint32_t w[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(acc[e]);
    EmitGroup<EPI == OV_EPI_ACCUM_F32>(c, map_y, w, x, y0, cc / 32);
  }
}

}  // namespace
}  // namespace ovb
