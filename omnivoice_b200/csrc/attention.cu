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

#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kQ = 128;        // queries per group
constexpr int kKeys = 128;     // keys per tile
constexpr int kD = 128;        // head dim
constexpr int kThreads = 320;  // 2 softmax groups + producer + MMA warp
constexpr uint32_t kHalfTile = 128 * 64 * 2;  // one [128][64] half box: 16 KB
constexpr uint32_t kTile = 2 * kHalfTile;     // [128][128] half: 32 KB
constexpr uint32_t kSmemBytes = 2 * kTile /*Q0,Q1*/ + 2 * 2 * kTile /*K,V ring*/ + 1024 + 256;
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
  // or null: sequence blockIdx.y, tiles 2 blockIdx.x and 2 blockIdx.x + 1.
  const int32_t* items;
  __half* out;
  int64_t ld_out;
  int heads;
  int kv_heads;
  float scale_log2;  // softmax scale * log2(e)
  uint32_t* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_qkv, const AttnArgs args) {
  pdl_wait();
  pdl_trigger();
  int seq, tile, max_groups;
  if (args.items != nullptr) {
    seq = args.items[2 * blockIdx.x];
    const int code = args.items[2 * blockIdx.x + 1];
    tile = code & 0xFFFFFF;
    max_groups = code >> 24;
  } else {
    seq = blockIdx.y;
    tile = 2 * blockIdx.x;
    max_groups = 2;
  }
  const int h = blockIdx.z;
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
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2 groups]
  uint64_t* p_full = bars + 7;    // [2 groups]
  uint64_t* o_done = bars + 9;    // [2 groups]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_map(&map_qkv);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      const int qcol = h * kD;
      const int kcol = (args.heads + kvh) * kD;
      const int vcol = (args.heads + args.kv_heads + kvh) * kD;
      mbar_arrive_expect_tx(q_full, groups * kTile);
      for (int g = 0; g < groups; ++g) {
        tma_load_2d(q_s + g * kTile, &map_qkv, q_full, qcol, start + q0 + g * kQ);
        tma_load_2d(q_s + g * kTile + kHalfTile, &map_qkv, q_full, qcol + 64, start + q0 + g * kQ);
      }
      int issued = 0;
      for (int t = 0; t < nt; ++t) {
        const int st = t & 1;
        if (t >= 2 && !mbar_wait(&kv_empty[st], static_cast<uint32_t>((t >> 1) - 1) & 1u, args.err))
          break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
        const int key0 = start + t * kKeys;
        uint8_t* kd = k_s + st * kTile;
        uint8_t* vd = v_s + st * kTile;
        tma_load_2d(kd, &map_qkv, &kv_full[st], kcol, key0);
        tma_load_2d(kd + kHalfTile, &map_qkv, &kv_full[st], kcol + 64, key0);
        tma_load_2d(vd, &map_qkv, &kv_full[st], vcol, key0);
        tma_load_2d(vd + kHalfTile, &map_qkv, &kv_full[st], vcol + 64, key0);
        ++issued;
      }
      (void)mbar_wait(q_full, 0, args.err);
      for (int t = issued > 2 ? issued - 2 : 0; t < issued; ++t)
        (void)mbar_wait(&kv_full[t & 1], static_cast<uint32_t>(t >> 1) & 1u, args.err);
    }
  } else if (warp == 9) {
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
      bool ok = mbar_wait(q_full, 0, args.err) && mbar_wait(&kv_full[0], 0, args.err);
      if (ok) {
        tc_fence_after_sync();
        for (int g = 0; g < groups; ++g) issue_s(g, 0);
      }
      for (int t = 0; ok && t < nt; ++t) {
        const bool more = t + 1 < nt;
        for (int g = 0; g < groups; ++g) {
          if (!mbar_wait(&p_full[g], static_cast<uint32_t>(t) & 1u, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_pv(g, t);
          if (!more) {
            umma_commit(&o_done[g]);
            continue;
          }
          if (g == 0 && !mbar_wait(&kv_full[(t + 1) & 1], static_cast<uint32_t>((t + 1) >> 1) & 1u,
                                   args.err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_s(g, t + 1);  // runs after this group's P V (in-order MMAs)
        }
        umma_commit(&kv_empty[t & 1]);
      }
    }
  } else {
    // Softmax groups: thread owns query row `row` of group g.
    const int g = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const bool active = g < groups;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + static_cast<uint32_t>(g * 256) + lane_off;
    const uint32_t o_addr = s_addr + 128;
    float m = -INFINITY, l = 0.0f;
    bool ok = active;
    for (int t = 0; ok && t < nt; ++t) {
      // Warp-uniform outcome: the tensor-memory accesses below are
      // warp-collective.
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s_full[g], static_cast<uint32_t>(t) & 1u, args.err))) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const int valid = min(kKeys, len - t * kKeys);
      // Pass 1: row maximum (two 32-column chunks in registers at a time;
      // keys past the sequence end read as -inf).
      float mt = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(s_addr + half * 64, ra);
        tmem_ld_32x32b_x32(s_addr + half * 64 + 32, rb);
        tmem_ld_wait();
        if (valid < kKeys) {
          mask_keys(ra, half * 64, valid);
          mask_keys(rb, half * 64 + 32, valid);
        }
        mt = fmaxf(mt, fmaxf(max32(ra), max32(rb)));
      }
      mt *= args.scale_log2;
      if (t == 0) {
        m = mt;
      } else {
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole
        // warp rescales when any of its rows needs it; rows whose maximum
        // did not grow past the threshold keep theirs (alpha = 1).
        const bool grow = mt > m + kRescaleThreshold;
        if (__any_sync(0xFFFFFFFFu, grow)) {
          // The previous P V of this group completed before S_t was written
          // (one thread issues both, in order), so O is stable here.
          const float m_new = grow ? mt : m;
          const float alpha = ex2_approx(m - m_new);
          l *= alpha;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(o_addr + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
            tmem_st_32x32b_x16(o_addr + c * 32,
                               *reinterpret_cast<const uint32_t(*)[16]>(&r[0]));
            tmem_st_32x32b_x16(o_addr + c * 32 + 16,
                               *reinterpret_cast<const uint32_t(*)[16]>(&r[16]));
          }
          m = m_new;
        }
      }
      // Pass 2: probabilities, written as half pairs over the consumed S
      // columns (keys 32c..32c+31 -> columns 16c..16c+15).
      float rowsum = 0.0f;
      const float neg_m = -m;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(s_addr + half * 64, ra);
        tmem_ld_32x32b_x32(s_addr + half * 64 + 32, rb);
        tmem_ld_wait();
        if (valid < kKeys) {
          mask_keys(ra, half * 64, valid);
          mask_keys(rb, half * 64 + 32, valid);
        }
        uint32_t pa[16], pb[16];
        rowsum += probs32(ra, args.scale_log2, neg_m, pa);
        rowsum += probs32(rb, args.scale_log2, neg_m, pb);
        tmem_st_32x32b_x16(s_addr + half * 32, pa);
        tmem_st_32x32b_x16(s_addr + half * 32 + 16, pb);
      }
      l += rowsum;
      tmem_st_wait();
      tc_fence_before_sync();
      mbar_arrive(&p_full[g]);
    }
    if (__all_sync(0xFFFFFFFFu, ok && mbar_wait(&o_done[g], 0, args.err))) {
      tc_fence_after_sync();
      const float inv = 1.0f / l;
      const bool store = q0 + g * kQ + row < len;
      __half* dst =
          args.out + static_cast<int64_t>(start + q0 + g * kQ + row) * args.ld_out + h * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_addr + c * 32, r);
        tmem_ld_wait();
        if (store) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(r[j + e]) * inv;
            *reinterpret_cast<uint4*>(dst + c * 32 + j) =
                make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]),
                           pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
          }
        }
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

void ConfigureAttentionKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel),
                    static_cast<int>(kSmemBytes));
}

// items: device [n_items][2] (sequence, first 128-query tile | max groups
// << 24); null to cover ceil(max_seqlen / 256) tile pairs of every sequence.
void LaunchAttention(const CUtensorMap& map_qkv, const int32_t* cu_seqlens, int num_seqs,
                     int max_seqlen, const int32_t* items, int n_items, int heads, int kv_heads,
                     float scale, __half* out, int64_t ld_out, cudaStream_t stream) {
  if (num_seqs == 0 || max_seqlen == 0) return;
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel),
                    static_cast<int>(kSmemBytes));
  AttnArgs a;
  a.cu_seqlens = cu_seqlens;
  a.items = items;
  a.out = out;
  a.ld_out = ld_out;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = DeviceErrorWord();
  const dim3 grid = items != nullptr
                        ? dim3(static_cast<unsigned>(n_items), 1, static_cast<unsigned>(heads))
                        : dim3(static_cast<unsigned>((max_seqlen + 2 * kQ - 1) / (2 * kQ)),
                               static_cast<unsigned>(num_seqs), static_cast<unsigned>(heads));
  Launch(attention_kernel, grid, dim3(kThreads), kSmemBytes, stream, "attention kernel launch",
         map_qkv, a);
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
    CUtensorMap map;
    EncodeQkvMap(&map, qkv, static_cast<int64_t>(ld_qkv), static_cast<int64_t>(rows),
                 static_cast<int64_t>((heads + 2 * kv_heads) * head_dim));
    LaunchAttention(map, cu_seqlens, static_cast<int>(num_seqs), static_cast<int>(max_seqlen),
                    nullptr, 0, static_cast<int>(heads), static_cast<int>(kv_heads), scale,
                    reinterpret_cast<__half*>(out), static_cast<int64_t>(ld_out),
                    AsStream(stream));
  });
}
