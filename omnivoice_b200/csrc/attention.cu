// Bidirectional grouped-query attention over packed variable-length
// sequences on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-sequence attention (generator.cpp:122-172:
// a batched Q K^T GEMM into float32 scores [heads][L][L], SoftmaxKernel
// writing half probabilities, a batched P V GEMM and MergeHeadsKernel) with
// one flash-style kernel: scores never leave the SM.
//
// CTA = (128-query tile, sequence, query head h); kv head = h / (heads /
// kv_heads).  Warp roles (192 threads):
//   warps 0..3  softmax: thread r owns query row r (tensor-memory lane r);
//               reads S from tensor memory twice (row max, then
//               probabilities), writes half P into 128B-swizzled shared
//               memory and folds each tile's P V product into float32
//               registers with the running-max correction;
//   warp 4      TMA producer: Q once, then K and V tiles of 128 keys into a
//               2-deep ring;
//   warp 5      tensor-memory owner and MMA issuer: S_t = Q K_t^T into one of
//               two 128-column S buffers (S_{t+1} is issued while S_t is in
//               softmax), then O_t = P_t V_t (V as an MN-major operand) into
//               a 128-column O buffer.
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

constexpr int kQ = 128;       // queries per CTA
constexpr int kKeys = 128;    // keys per tile
constexpr int kD = 128;       // head dim
constexpr int kThreads = 192;
constexpr uint32_t kHalfTile = 128 * 64 * 2;   // one [128][64] half box: 16 KB
constexpr uint32_t kTile = 2 * kHalfTile;      // [128][128] half: 32 KB
constexpr uint32_t kSmemBytes = kTile /*Q*/ + 2 * 2 * kTile /*K,V ring*/ + kTile /*P*/ + 1024 + 256;

struct AttnArgs {
  const int32_t* cu_seqlens;
  __half* out;
  int64_t ld_out;
  int heads;
  int kv_heads;
  float scale_log2;  // softmax scale * log2(e)
  uint32_t* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_qkv, const AttnArgs args) {
  const int seq = blockIdx.y;
  const int h = blockIdx.z;
  const int start = args.cu_seqlens[seq];
  const int len = args.cu_seqlens[seq + 1] - start;
  const int q0 = blockIdx.x * kQ;
  if (q0 >= len) return;  // uniform over the CTA, before any barrier
  const int kvh = h / (args.heads / args.kv_heads);
  const int nt = (len + kKeys - 1) / kKeys;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;
  uint8_t* k_s = q_s + kTile;         // [2 stages] x 32 KB
  uint8_t* v_s = k_s + 2 * kTile;     // [2 stages] x 32 KB
  uint8_t* p_s = v_s + 2 * kTile;     // 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_full = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    fence_mbar_init();
    tma_prefetch_map(&map_qkv);
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s[2] = {tmem, tmem + 128};
  const uint32_t tmem_o = tmem + 256;

  if (warp == 4) {
    if (lane == 0) {
      const int qcol = h * kD;
      const int kcol = (args.heads + kvh) * kD;
      const int vcol = (args.heads + args.kv_heads + kvh) * kD;
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_2d(q_s, &map_qkv, q_full, qcol, start + q0);
      tma_load_2d(q_s + kHalfTile, &map_qkv, q_full, qcol + 64, start + q0);
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
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kQ, kKeys, 0);
      constexpr uint32_t idesc_o = idesc_f16_f32(kQ, kD, 1);
      bool ok = mbar_wait(q_full, 0, args.err);
      const uint32_t qa = smem_u32(q_s);
      auto issue_s = [&](int t) -> bool {
        const int st = t & 1;
        if (!mbar_wait(&kv_full[st], static_cast<uint32_t>(t >> 1) & 1u, args.err)) return false;
        if (t >= 2 && !mbar_wait(&s_free[st], static_cast<uint32_t>((t >> 1) - 1) & 1u, args.err))
          return false;
        tc_fence_after_sync();
        const uint32_t ka = smem_u32(k_s + st * kTile);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfTile + (kk & 3) * 32;
          umma_f16_ss(tmem_s[st], smem_desc_sw128(qa + off, 16, 1024),
                      smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int t = 0; ok && t < nt; ++t) {
        if (t + 1 < nt && !issue_s(t + 1)) break;
        if (!mbar_wait(p_full, static_cast<uint32_t>(t) & 1u, args.err)) break;
        tc_fence_after_sync();
        const uint32_t pa = smem_u32(p_s);
        const uint32_t va = smem_u32(v_s + (t & 1) * kTile);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * kHalfTile + (kk & 3) * 32;
          umma_f16_ss(tmem_o, smem_desc_sw128(pa + poff, 16, 1024),
                      smem_desc_sw128(va + kk * 16 * 128, kHalfTile, 1024), idesc_o,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(o_full);
        umma_commit(&kv_empty[t & 1]);
      }
    }
  } else {
    // Softmax warps: thread owns query row `row` = tensor-memory lane.
    const int row = warp * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float acc[kD];
#pragma unroll
    for (int j = 0; j < kD; ++j) acc[j] = 0.0f;
    float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      const int b = t & 1;
      if (!mbar_wait(&s_full[b], static_cast<uint32_t>(t >> 1) & 1u, args.err)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const int valid = min(kKeys, len - t * kKeys);
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_s[b] + lane_off + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c * 32 + j < valid) mt = fmaxf(mt, __uint_as_float(r[j]) * args.scale_log2);
      }
      const float m_new = fmaxf(m, mt);
      const float alpha = exp2f(m - m_new);
      if (t > 0) {
        // Fold O_{t-1} = P_{t-1} V_{t-1} (relative to m_{t-1}) into acc.
        if (!mbar_wait(o_full, static_cast<uint32_t>(t - 1) & 1u, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_o + lane_off + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[c * 32 + j] = fmaf(acc[c * 32 + j], alpha_prev, __uint_as_float(r[j]));
        }
      }
      float rowsum = 0.0f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_s[b] + lane_off + c * 32, r);
        tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = c * 32 + j < valid
                               ? exp2f(__uint_as_float(r[j]) * args.scale_log2 - m_new) : 0.0f;
          const float p1 = c * 32 + j + 1 < valid
                               ? exp2f(__uint_as_float(r[j + 1]) * args.scale_log2 - m_new) : 0.0f;
          rowsum += p0 + p1;
          packed[j / 2] = pack_half2(p0, p1);
        }
        // keys 32c..32c+31 of row `row`: 128B-swizzled K-major P operand.
        uint8_t* prow = p_s + (c >> 1) * kHalfTile + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 1) * 4 + q) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + chunk * 16) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      l = l * alpha + rowsum;
      m = m_new;
      alpha_prev = alpha;
      tc_fence_before_sync();
      fence_proxy_async_smem();
      mbar_arrive(&s_free[b]);
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_full, static_cast<uint32_t>(nt - 1) & 1u, args.err)) {
      tc_fence_after_sync();
      const float inv = 1.0f / l;
      const bool store = q0 + row < len;
      __half* dst = args.out + static_cast<int64_t>(start + q0 + row) * args.ld_out + h * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_o + lane_off + c * 32, r);
        tmem_ld_wait();
        if (store) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              o[e] = fmaf(acc[c * 32 + j + e], alpha_prev, __uint_as_float(r[j + e])) * inv;
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
  if (warp == 5) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

void ConfigureAttentionKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel),
                    static_cast<int>(kSmemBytes));
}

void LaunchAttention(const CUtensorMap& map_qkv, const int32_t* cu_seqlens, int num_seqs,
                     int max_seqlen, int heads, int kv_heads, float scale, __half* out,
                     int64_t ld_out, cudaStream_t stream) {
  if (num_seqs == 0 || max_seqlen == 0) return;
  SetMaxDynamicSmem(reinterpret_cast<const void*>(attention_kernel),
                    static_cast<int>(kSmemBytes));
  AttnArgs a;
  a.cu_seqlens = cu_seqlens;
  a.out = out;
  a.ld_out = ld_out;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = DeviceErrorWord();
  const dim3 grid(static_cast<unsigned>((max_seqlen + kQ - 1) / kQ),
                  static_cast<unsigned>(num_seqs), static_cast<unsigned>(heads));
  attention_kernel<<<grid, kThreads, kSmemBytes, stream>>>(map_qkv, a);
  Check(cudaGetLastError(), "attention kernel launch");
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
                    static_cast<int>(heads), static_cast<int>(kv_heads), scale,
                    reinterpret_cast<__half*>(out), static_cast<int64_t>(ld_out),
                    AsStream(stream));
  });
}
