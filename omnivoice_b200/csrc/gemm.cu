// y (+)= x * w^T on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the reference's hipBLASLt wrapper (gemm.cpp:80-288, HalfGemm)
// and fuses the element-wise kernels that follow each product in
// generator.cpp:272-300: SwiGLU (generator_kernels.hip:191-200), QK
// RMSNorm + RoPE (:102-159) and the residual add (beta = 1).
//
// One CTA computes one 128 x BN tile of y, optionally over a slice of K:
//   warp 0      TMA producer: 128x64 tiles of x and BNx64 tiles of w,
//               128-byte swizzled, into a STAGES-deep shared-memory ring;
//   warp 1      allocates BN tensor-memory columns and, from one thread,
//               issues tcgen05.mma (M=128, N=BN, K=16) into them, releasing
//               ring slots with tcgen05.commit;
//   warps 2..5  epilogue: each thread owns one accumulator row (tensor
//               memory lane), loads it with tcgen05.ld and applies the
//               fused epilogue.
// Split-K (residual epilogue only) is deterministic: every split writes
// its partial tile to a workspace and the last split to arrive sums the
// partials in split order before adding them to y.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "gemm.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kRingBytes = 196608;
// Split-K workspace: arrival counters first (zero between launches), then
// the partial tiles.
constexpr size_t kCounterBytes = 1024;

template <int BN>
struct TileConfig {
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kRingBytes / kStageBytes;
  static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + 1024 + 256;
};

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int BN, int EPI>
__device__ __forceinline__ void epilogue(const GemmArgs& a, uint32_t tmem, int m_tile, int n_tile,
                                         int split, int* flag) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quarter = warp & 3;  // tensor memory lanes 32*quarter .. +31
  const int row_local = quarter * 32 + lane;
  const int64_t grow = static_cast<int64_t>(m_tile) * kBM + row_local;
  const bool row_ok = grow < a.M;
  const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);

  if constexpr (EPI == OV_EPI_STORE_F32 || EPI == OV_EPI_ACCUM_F32) {
    if (EPI == OV_EPI_ACCUM_F32 && a.splits > 1) {
      const int tile = m_tile * gridDim.x + n_tile;
      float* part_base = a.partials + static_cast<int64_t>(tile) * a.splits * (kBM * BN);
      float* mine = part_base + static_cast<int64_t>(split) * (kBM * BN) + row_local * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(trow + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          __stcg(reinterpret_cast<float4*>(mine + c0 + j),
                 make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                             __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])));
      }
      __threadfence();
      named_barrier(1, 128);
      if (threadIdx.x == 64) {
        const uint32_t prev = atomicAdd(a.counters + tile, 1u);
        *flag = prev == static_cast<uint32_t>(a.splits - 1) ? 1 : 0;
      }
      named_barrier(1, 128);
      if (*flag == 0) return;
      __threadfence();
      if (row_ok) {
        float* y = static_cast<float*>(a.y) + grow * a.ldy + n_tile * BN;
        const float* rowp = part_base + row_local * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 4) {
          if (n_tile * BN + c >= a.N) break;
          float4 acc = __ldcg(reinterpret_cast<const float4*>(rowp + c));
          for (int s = 1; s < a.splits; ++s) {
            const float4 p =
                __ldcg(reinterpret_cast<const float4*>(rowp + static_cast<int64_t>(s) * kBM * BN + c));
            acc.x += p.x;
            acc.y += p.y;
            acc.z += p.z;
            acc.w += p.w;
          }
          float4 old = *reinterpret_cast<const float4*>(y + c);
          old.x += acc.x;
          old.y += acc.y;
          old.z += acc.z;
          old.w += acc.w;
          *reinterpret_cast<float4*>(y + c) = old;
        }
      }
      if (threadIdx.x == 64) a.counters[tile] = 0u;
      return;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(trow + c0, r);
      tmem_ld_wait();
      const int gcol = n_tile * BN + c0;
      if (row_ok) {
        float* y = static_cast<float*>(a.y) + grow * a.ldy + gcol;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          if (gcol + j < a.N) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                   __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            if (EPI == OV_EPI_ACCUM_F32) {
              const float4 old = *reinterpret_cast<const float4*>(y + j);
              v.x = old.x + v.x;
              v.y = old.y + v.y;
              v.z = old.z + v.z;
              v.w = old.w + v.w;
            }
            *reinterpret_cast<float4*>(y + j) = v;
          }
        }
      }
    }
  } else if constexpr (EPI == OV_EPI_SWIGLU_F16) {
    // The tile holds BN / 128 groups of [64 gate | 64 up] columns.
    constexpr int G = OV_SWIGLU_GROUP;
#pragma unroll 1
    for (int gi = 0; gi < BN / (2 * G); ++gi) {
#pragma unroll 1
      for (int c0 = 0; c0 < G; c0 += 32) {
        uint32_t g[32], u[32];
        tmem_ld_32x32b_x32(trow + gi * 2 * G + c0, g);
        tmem_ld_32x32b_x32(trow + gi * 2 * G + G + c0, u);
        tmem_ld_wait();
        if (row_ok) {
          __half* y = static_cast<__half*>(a.y) + grow * a.ldy + n_tile * (BN / 2) + gi * G + c0;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 packed;
            packed.x = pack_half2(silu_mul(__uint_as_float(g[j]), __uint_as_float(u[j])),
                                  silu_mul(__uint_as_float(g[j + 1]), __uint_as_float(u[j + 1])));
            packed.y = pack_half2(silu_mul(__uint_as_float(g[j + 2]), __uint_as_float(u[j + 2])),
                                  silu_mul(__uint_as_float(g[j + 3]), __uint_as_float(u[j + 3])));
            packed.z = pack_half2(silu_mul(__uint_as_float(g[j + 4]), __uint_as_float(u[j + 4])),
                                  silu_mul(__uint_as_float(g[j + 5]), __uint_as_float(u[j + 5])));
            packed.w = pack_half2(silu_mul(__uint_as_float(g[j + 6]), __uint_as_float(u[j + 6])),
                                  silu_mul(__uint_as_float(g[j + 7]), __uint_as_float(u[j + 7])));
            *reinterpret_cast<uint4*>(y + j) = packed;
          }
        }
      }
    }
  } else if constexpr (EPI == OV_EPI_QKNORM_ROPE_F16) {
    static_assert(BN == 128, "one head of 128 per tile");
    float v[128];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(trow + c * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[c * 32 + j] = __uint_as_float(r[j]);
    }
    if (!row_ok) return;
    const int slot = n_tile;
    __half* y = static_cast<__half*>(a.y) + grow * a.ldy + slot * 128;
    if (slot < a.heads + a.kv_heads) {
      const float* w = slot < a.heads ? a.q_norm : a.k_norm;
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < 128; ++j) ss = fmaf(v[j], v[j], ss);
      const float scale = 1.0f / sqrtf(ss / 128.0f + a.epsilon);
      int pos = a.positions[grow];
      if (pos < 0 || pos >= a.max_positions) {
        atomicOr(a.err, kErrBadArgument);
        pos = 0;
      }
      const float* cs = a.rope_cos + static_cast<int64_t>(pos) * 64;
      const float* sn = a.rope_sin + static_cast<int64_t>(pos) * 64;
#pragma unroll
      for (int i0 = 0; i0 < 64; i0 += 8) {
        float lo[8], hi[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int i = i0 + t;
          const float x1 = w[i] * (v[i] * scale);
          const float x2 = w[i + 64] * (v[i + 64] * scale);
          const float c = cs[i];
          const float s = sn[i];
          lo[t] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
          hi[t] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        }
        uint4 p0, p1;
        p0.x = pack_half2(lo[0], lo[1]);
        p0.y = pack_half2(lo[2], lo[3]);
        p0.z = pack_half2(lo[4], lo[5]);
        p0.w = pack_half2(lo[6], lo[7]);
        p1.x = pack_half2(hi[0], hi[1]);
        p1.y = pack_half2(hi[2], hi[3]);
        p1.z = pack_half2(hi[4], hi[5]);
        p1.w = pack_half2(hi[6], hi[7]);
        *reinterpret_cast<uint4*>(y + i0) = p0;
        *reinterpret_cast<uint4*>(y + 64 + i0) = p1;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 128; j += 8) {
        uint4 p;
        p.x = pack_half2(v[j], v[j + 1]);
        p.y = pack_half2(v[j + 2], v[j + 3]);
        p.z = pack_half2(v[j + 4], v[j + 5]);
        p.w = pack_half2(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(y + j) = p;
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const GemmArgs args) {
  using Cfg = TileConfig<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + kStages * Cfg::kBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;
  const int split = blockIdx.z;
  const int kb0 = split * args.kblocks / args.splits;
  const int kb1 = (split + 1) * args.kblocks / args.splits;
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % kStages;
        const uint32_t phase = static_cast<uint32_t>(i / kStages) & 1u;
        if (i >= kStages && !mbar_wait(&empty[s], phase ^ 1u, args.err)) break;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
        tma_load_2d(sa + s * Cfg::kABytes, &map_a, &full[s], (kb0 + i) * kBK, m_tile * kBM);
        tma_load_2d(sb + s * Cfg::kBBytes, &map_b, &full[s], (kb0 + i) * kBK,
                    args.b_row_offset + n_tile * BN);
        ++issued;
      }
      // Let the copies this thread started land before the CTA can exit.
      for (int i = std::max(0, issued - kStages); i < issued; ++i)
        (void)mbar_wait(&full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u, args.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % kStages;
        const uint32_t phase = static_cast<uint32_t>(i / kStages) & 1u;
        if (!mbar_wait(&full[s], phase, args.err)) break;
        tc_fence_after_sync();
        const uint32_t a0 = smem_u32(sa + s * Cfg::kABytes);
        const uint32_t b0 = smem_u32(sb + s * Cfg::kBBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          umma_f16_ss(tmem, smem_desc_sw128(a0 + k * 32, 16, 1024),
                      smem_desc_sw128(b0 + k * 32, 16, 1024), idesc,
                      (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(done);
    }
  } else {
    // Every epilogue thread runs the epilogue even after a timed-out wait
    // (the error word is set) so the 128 threads stay in step for the
    // split-K named barrier.
    (void)mbar_wait(done, 0, args.err);
    tc_fence_after_sync();
    epilogue<BN, EPI>(args, tmem, m_tile, n_tile, split, flag);
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN, int EPI>
void LaunchTyped(const GemmPlan& p, cudaStream_t stream) {
  auto kernel = gemm_kernel<BN, EPI>;
  SetMaxDynamicSmem(reinterpret_cast<const void*>(kernel),
                    static_cast<int>(TileConfig<BN>::kSmemBytes));
  kernel<<<p.grid, kThreads, TileConfig<BN>::kSmemBytes, stream>>>(p.map_a, p.map_b, p.args);
  Check(cudaGetLastError(), "gemm kernel launch");
}

int Tiles(int M, int N, int bn) { return ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn); }

}  // namespace

GemmShapeChoice ChooseGemmShape(int M, int N, int K, int epilogue, bool have_workspace, int sms) {
  GemmShapeChoice c{128, 1};
  if (epilogue == OV_EPI_QKNORM_ROPE_F16) return c;
  // Time of a tile is proportional to its width; a wave is `sms` tiles.
  // A 256-wide tile runs the tensor pipe at full rate; a 128-wide one
  // loses a little to operand reads (weight 1.1 per column).
  auto cost = [&](int bn) {
    const int waves = (Tiles(M, N, bn) + sms - 1) / sms;
    return waves * bn * (bn == 128 ? 1.1 : 1.0);
  };
  const bool can256 = epilogue != OV_EPI_SWIGLU_F16 || N % 256 == 0;
  if (can256 && cost(256) <= cost(128)) c.bn = 256;
  if (epilogue == OV_EPI_ACCUM_F32 && have_workspace) {
    c.bn = 128;
    const int tiles = Tiles(M, N, 128);
    const int kblocks = K / kBK;
    int splits = 1;
    while (splits < 8 && tiles * (splits + 1) <= sms && kblocks / (splits + 1) >= 4) ++splits;
    c.splits = splits;
  }
  return c;
}

size_t GemmWorkspaceBytes(int M, int N, int K, int epilogue, int sms) {
  const GemmShapeChoice c = ChooseGemmShape(M, N, K, epilogue, true, sms);
  if (c.splits <= 1) return 0;
  const size_t tiles = static_cast<size_t>(Tiles(M, N, c.bn));
  return kCounterBytes + tiles * c.splits * kBM * c.bn * sizeof(float);
}

void PlanGemm(GemmPlan* plan, const uint16_t* x, int64_t ldx, const uint16_t* w, int64_t w_rows,
              int b_row_offset, void* y, int64_t ldy, int M, int N, int K, int epilogue,
              const ov_epilogue_args* ea, void* workspace, size_t workspace_bytes, int sms,
              uint32_t* err) {
  OV_REQUIRE(M > 0 && N > 0 && K > 0, "empty GEMM");
  OV_REQUIRE(K % kBK == 0, "GEMM K must be a multiple of 64");
  OV_REQUIRE(ldx % 8 == 0 && ldx >= K, "x row stride must be a multiple of 8 and >= K");
  OV_REQUIRE(epilogue >= OV_EPI_STORE_F32 && epilogue <= OV_EPI_QKNORM_ROPE_F16, "epilogue");
  const bool half_out = epilogue == OV_EPI_SWIGLU_F16 || epilogue == OV_EPI_QKNORM_ROPE_F16;
  OV_REQUIRE(ldy % (half_out ? 8 : 4) == 0, "y row stride must allow 16-byte vector stores");
  OV_REQUIRE((reinterpret_cast<uintptr_t>(y) & 15u) == 0, "y must be 16-byte aligned");
  GemmShapeChoice choice =
      ChooseGemmShape(M, N, K, epilogue, workspace != nullptr && workspace_bytes > 0, sms);
  if (choice.splits > 1) {
    const size_t need = GemmWorkspaceBytes(M, N, K, epilogue, sms);
    if (workspace_bytes < need) choice.splits = 1;
  }
  if (epilogue == OV_EPI_SWIGLU_F16) {
    OV_REQUIRE(N % 128 == 0 && N % choice.bn == 0,
               "SwiGLU output features must be a multiple of 128");
    OV_REQUIRE(ldy >= N / 2, "y row stride");
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
  GemmArgs& a = plan->args;
  a = GemmArgs{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.kblocks = K / kBK;
  a.splits = choice.splits;
  a.b_row_offset = b_row_offset;
  a.ldy = ldy;
  a.y = y;
  a.err = err != nullptr ? err : DeviceErrorWord();
  if (choice.splits > 1) {
    // Counters live at a fixed place, ahead of the partial tiles, so a
    // workspace shared by products of different shapes keeps them zero
    // (every split-K launch leaves its counters at zero).
    OV_REQUIRE(Tiles(M, N, choice.bn) * sizeof(uint32_t) <= kCounterBytes, "split-K tile count");
    a.counters = static_cast<uint32_t*>(workspace);
    a.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  }
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
                    static_cast<uint32_t>(choice.bn), CU_TENSOR_MAP_SWIZZLE_128B);
  plan->grid = dim3(static_cast<unsigned>((N + choice.bn - 1) / choice.bn),
                    static_cast<unsigned>((M + kBM - 1) / kBM),
                    static_cast<unsigned>(choice.splits));
  plan->smem_bytes = choice.bn == 256 ? TileConfig<256>::kSmemBytes : TileConfig<128>::kSmemBytes;
}

void ConfigureGemmKernels() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<128, OV_EPI_STORE_F32>),
                    static_cast<int>(TileConfig<128>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<256, OV_EPI_STORE_F32>),
                    static_cast<int>(TileConfig<256>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<128, OV_EPI_ACCUM_F32>),
                    static_cast<int>(TileConfig<128>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<256, OV_EPI_ACCUM_F32>),
                    static_cast<int>(TileConfig<256>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<128, OV_EPI_SWIGLU_F16>),
                    static_cast<int>(TileConfig<128>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<256, OV_EPI_SWIGLU_F16>),
                    static_cast<int>(TileConfig<256>::kSmemBytes));
  SetMaxDynamicSmem(reinterpret_cast<const void*>(gemm_kernel<128, OV_EPI_QKNORM_ROPE_F16>),
                    static_cast<int>(TileConfig<128>::kSmemBytes));
}

void LaunchGemm(const GemmPlan& p, cudaStream_t stream) {
  switch (p.epilogue * 1000 + p.bn) {
    case OV_EPI_STORE_F32 * 1000 + 128: LaunchTyped<128, OV_EPI_STORE_F32>(p, stream); break;
    case OV_EPI_STORE_F32 * 1000 + 256: LaunchTyped<256, OV_EPI_STORE_F32>(p, stream); break;
    case OV_EPI_ACCUM_F32 * 1000 + 128: LaunchTyped<128, OV_EPI_ACCUM_F32>(p, stream); break;
    case OV_EPI_ACCUM_F32 * 1000 + 256: LaunchTyped<256, OV_EPI_ACCUM_F32>(p, stream); break;
    case OV_EPI_SWIGLU_F16 * 1000 + 128: LaunchTyped<128, OV_EPI_SWIGLU_F16>(p, stream); break;
    case OV_EPI_SWIGLU_F16 * 1000 + 256: LaunchTyped<256, OV_EPI_SWIGLU_F16>(p, stream); break;
    case OV_EPI_QKNORM_ROPE_F16 * 1000 + 128:
      LaunchTyped<128, OV_EPI_QKNORM_ROPE_F16>(p, stream);
      break;
    default: throw Error(OV_ERR_UNSUPPORTED, "no GEMM kernel for this epilogue / tile");
  }
}

}  // namespace ovb

// ------------------------------------------------ allocation-free variant
//
// ov_gemm_f16_noalloc takes its split-K scratch from this file-scope device
// array instead of a caller-supplied workspace.  Every GPU that loads the
// library holds it until the process exits.  In host code the array's name
// only stands for the symbol, so its device address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and that
// address is what the kernel receives.
constexpr size_t kNoAllocScratchBytes = size_t{10} << 20;  // 10 MiB per device
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

template <int BN, int EPI>
void SetSmemDirect() {
  Check(cudaFuncSetAttribute(gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(TileConfig<BN>::kSmemBytes)),
        "cudaFuncSetAttribute(max dynamic shared memory)");
}

// Once per device, with it current: device addresses of the static arrays,
// cleared split-K counters, and the kernels' shared-memory limits.
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
    Check(cudaMemset(sp, 0, kCounterBytes), "clear split-K counters");
    Check(cudaMemset(tp, 0, sizeof(uint32_t) * 64), "clear status word");
    SetSmemDirect<128, OV_EPI_STORE_F32>();
    SetSmemDirect<256, OV_EPI_STORE_F32>();
    SetSmemDirect<128, OV_EPI_ACCUM_F32>();
    SetSmemDirect<256, OV_EPI_ACCUM_F32>();
    SetSmemDirect<128, OV_EPI_SWIGLU_F16>();
    SetSmemDirect<256, OV_EPI_SWIGLU_F16>();
    SetSmemDirect<128, OV_EPI_QKNORM_ROPE_F16>();
    g_noalloc_status_ptr[device] = static_cast<uint32_t*>(tp);
    g_noalloc_scratch_ptr[device] = static_cast<uint8_t*>(sp);
  }
  *scratch = g_noalloc_scratch_ptr[device];
  *status = g_noalloc_status_ptr[device];
}

template <int BN, int EPI>
void LaunchDirect(const GemmPlan& p, cudaStream_t stream) {
  gemm_kernel<BN, EPI><<<p.grid, kThreads, TileConfig<BN>::kSmemBytes, stream>>>(p.map_a, p.map_b,
                                                                                p.args);
  Check(cudaGetLastError(), "gemm kernel launch");
}

}  // namespace
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
    const size_t need = GemmWorkspaceBytes(static_cast<int>(rows), static_cast<int>(out),
                                           static_cast<int>(in), epilogue, sms);
    if (need > kNoAllocScratchBytes)
      throw Error(OV_ERR_INVALID, "needs " + std::to_string(need) +
                                      " bytes of split-K scratch, more than the " +
                                      std::to_string(kNoAllocScratchBytes) + "-byte static array");
    GemmPlan plan;
    PlanGemm(&plan, x, static_cast<int64_t>(ldx), w, static_cast<int64_t>(out), 0, y,
             static_cast<int64_t>(ldy), static_cast<int>(rows), static_cast<int>(out),
             static_cast<int>(in), epilogue, args, scratch, kNoAllocScratchBytes, sms, status);
    const cudaStream_t s = AsStream(stream);
    switch (plan.epilogue * 1000 + plan.bn) {
      case OV_EPI_STORE_F32 * 1000 + 128: LaunchDirect<128, OV_EPI_STORE_F32>(plan, s); break;
      case OV_EPI_STORE_F32 * 1000 + 256: LaunchDirect<256, OV_EPI_STORE_F32>(plan, s); break;
      case OV_EPI_ACCUM_F32 * 1000 + 128: LaunchDirect<128, OV_EPI_ACCUM_F32>(plan, s); break;
      case OV_EPI_ACCUM_F32 * 1000 + 256: LaunchDirect<256, OV_EPI_ACCUM_F32>(plan, s); break;
      case OV_EPI_SWIGLU_F16 * 1000 + 128: LaunchDirect<128, OV_EPI_SWIGLU_F16>(plan, s); break;
      case OV_EPI_SWIGLU_F16 * 1000 + 256: LaunchDirect<256, OV_EPI_SWIGLU_F16>(plan, s); break;
      case OV_EPI_QKNORM_ROPE_F16 * 1000 + 128:
        LaunchDirect<128, OV_EPI_QKNORM_ROPE_F16>(plan, s);
        break;
      default: throw Error(OV_ERR_UNSUPPORTED, "no GEMM kernel for this epilogue / tile");
    }
  });
}

}  // extern "C"
