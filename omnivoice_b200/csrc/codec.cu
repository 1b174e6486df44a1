// Kernels of the audio tokenizer's decoder (RVQ codes -> 24 kHz samples),
// the step after the generator (reference codec.cpp:197-262,
// codec_state.hpp:217-289, kernels/codec_kernels.hip:11-79).
//
// Layout: every signal is time-major [rows][channels] float32 (channels
// contiguous), so a convolution is an implicit GEMM with M = output time
// rows, N = output channels and K = taps x input channels, and the A tile
// of one tap is a TMA box of the input at a shifted row (rows before 0 or
// past the end read as zeros: the convolution's padding).
//
// Precision: the reference decodes in float32 (hipblasSgemm).  The tensor
// cores here run kind::tf32 with the split-operand scheme: every operand x
// is stored as hi = tf32(x) and lo = x - hi, and a product accumulates
// hi*hi + hi*lo + lo*hi in float32 tensor memory, which keeps float32
// accuracy (the dropped lo*lo term is ~2^-22 relative).  Weights are split
// once at load; activations are split by the epilogue that produces them.
//
// Fusions: the snake activation (codec_kernels.hip:11-27) that precedes
// every convolution is applied by the epilogue of the convolution that
// produces its input, together with the bias (AddChannelBias) and the
// residual add (codec_state.hpp:255-262); a ConvTranspose1d runs as `stride`
// two-tap phase convolutions (no columns buffer, no col2im pass); fc2 is
// folded into the RVQ tables at load, so the codebook sum yields the first
// convolution's input directly.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>

#include "codec_kernels.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ptx.cuh"

namespace ovb {
namespace codec {
namespace {

constexpr int kBM = 128;           // output rows per tile (tensor-memory lanes)
constexpr int kKC = 32;            // input channels per k block: 128 bytes of float32
// Threads: warp 0 TMA, warp 1 MMA, then epilogue groups of four warps.
constexpr uint32_t kATile = kBM * kKC * 4;

template <int BN>
struct ConvTile {
  static constexpr uint32_t kBTile = BN * kKC * 4;
  static constexpr uint32_t kStage = 2 * kATile + 2 * kBTile;  // A hi, A lo, B hi, B lo
  static constexpr int kStages = BN == 128 ? 3 : 4;
  // Three accumulators of BN columns per tile and kAccBufs tiles in
  // flight, each with its own epilogue group (the epilogues of earlier
  // tiles under the MMAs of the next), as many as tensor memory holds; with
  // one buffer two groups share each tile.
  static constexpr int kAccBufs = BN == 128 ? 1 : (BN == 64 ? 2 : 4);
  static constexpr int kGroups = kAccBufs < 2 ? 2 : kAccBufs;
  static constexpr int kThreads = 64 + 128 * kGroups;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + 1024 + 256;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(3 * BN * kAccBufs <= static_cast<int>(kTmemCols), "tensor memory budget");
};

// Instruction descriptor of tcgen05.mma kind::tf32: tf32 A and B (format
// 2), float32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(uint32_t m, uint32_t n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// x rounded to the nearest tf32 (ties away from zero), as a float32.
__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// codec_kernels.hip:20-24: x + sin(a x)^2 / (a + 1e-9).
__device__ __forceinline__ float snake(float x, float a) {
  const float s = sinf(a * x);
  return x + (1.0f / (a + 1e-9f)) * (s * s);
}

__device__ __forceinline__ void store_split(float* hi, float* lo, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = tf32_hi(v[4 * q + e]);
      l[e] = v[4 * q + e] - h[e];
    }
    reinterpret_cast<float4*>(hi)[q] = make_float4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<float4*>(lo)[q] = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// Tile t of a launch -> (m tile, n tile, phase), m fastest so consecutive
// CTAs read neighbouring input rows.
struct TileCoord {
  int m0, n0, phase;
};
__device__ __forceinline__ TileCoord DecodeTile(int t, int m_tiles, int n_tiles, int bn) {
  const int per_phase = m_tiles * n_tiles;
  TileCoord c;
  c.phase = t / per_phase;
  const int r = t - c.phase * per_phase;
  c.n0 = (r / m_tiles) * bn;
  c.m0 = (r - (r / m_tiles) * m_tiles) * kBM;
  return c;
}

// Tap geometry of tap `tap` for a tile: input row of the tile's first
// output position, and the weight tap.
__device__ __forceinline__ void TapGeometry(const ConvArgs& a, const TileCoord& c, int tap,
                                            int& in_row, int& w_tap) {
  if (a.stride > 0) {
    const int d = (c.phase + a.pad) / a.stride;
    const int k0 = (c.phase + a.pad) - d * a.stride;
    in_row = c.m0 + d - tap;
    w_tap = k0 + tap * a.stride;
  } else {
    in_row = c.m0 + tap * a.dilation - a.pad;
    w_tap = tap;
  }
}

// One convolution (or the phases of a transposed one) as an implicit GEMM,
// persistent over 128-row tiles.
//   plain:      out[m] = bias + sum_t W[t] in[m + t * dilation - pad]
//   transposed: out[m * stride + r] = bias + W[k0] in[m + d] + W[k0 + stride] in[m + d - 1]
//               for phase r, d = (r + pad) / stride, k0 = (r + pad) % stride
//               (ConvTranspose1d with kernel 2 stride, padding pad = ceil(stride / 2) and
//               output padding stride % 2, codec_state.hpp:265-283 + Col2Im).
// W is [taps][cout][cin] (hi and lo planes), the input [rows][cin] (hi and lo).
// Warp 0 issues the TMA loads, warp 1 the MMAs, the other warps form
// epilogue groups of four: with NB accumulator buffers group g takes the
// tiles t with t % NB == g, with one buffer two groups share each tile
// (alternate 32-column chunks).
template <int BN>
__global__ void __launch_bounds__(ConvTile<BN>::kThreads, 1)
    conv_kernel(const __grid_constant__ CUtensorMap map_a_hi,
                const __grid_constant__ CUtensorMap map_a_lo,
                const __grid_constant__ CUtensorMap map_b_hi,
                const __grid_constant__ CUtensorMap map_b_lo, const ConvArgs a) {
  using Cfg = ConvTile<BN>;
  constexpr int S = Cfg::kStages;
  constexpr int NB = Cfg::kAccBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStage);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;    // [NB]
  uint64_t* tempty = tfull + NB;  // [NB]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + NB);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (a.m_count + kBM - 1) / kBM;
  const int n_tiles = a.cout / BN;
  const int tiles = m_tiles * n_tiles * (a.stride > 0 ? a.stride : 1);
  const int kpt = a.cin / kKC;  // k blocks per tap
  const int kblocks = a.taps * kpt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], NB >= 2 ? 128 : 256);
    }
    fence_mbar_init();
    tma_prefetch_map(&map_a_hi);
    tma_prefetch_map(&map_a_lo);
    tma_prefetch_map(&map_b_hi);
    tma_prefetch_map(&map_b_lo);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the input signal is written by the previous kernel
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const TileCoord c = DecodeTile(t, m_tiles, n_tiles, BN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          if (it >= static_cast<uint32_t>(S) &&
              !mbar_wait(&empty[s], ((it / S) - 1) & 1u, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * Cfg::kStage;
          const int tap = kb / kpt;
          const int x = (kb - tap * kpt) * kKC;
          int in_row, w_tap;
          TapGeometry(a, c, tap, in_row, w_tap);
          mbar_arrive_expect_tx(&full[s], Cfg::kStage);
          tma_load_2d(st, &map_a_hi, &full[s], x, in_row);
          tma_load_2d(st + kATile, &map_a_lo, &full[s], x, in_row);
          tma_load_2d(st + 2 * kATile, &map_b_hi, &full[s], x, w_tap * a.cout + c.n0);
          tma_load_2d(st + 2 * kATile + Cfg::kBTile, &map_b_lo, &full[s], x,
                      w_tap * a.cout + c.n0);
        }
      }
      // The copies in flight land before the CTA may exit.
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t i = first; i < it; ++i) (void)mbar_wait(&full[i % S], (i / S) & 1u, a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Per tile three accumulators of BN columns: hi*hi of the even and of
      // the odd k blocks, and the small cross terms hi*lo + lo*hi.  Every
      // tensor-core accumulation rounds to float32, so fewer accumulations
      // into each sum keep the rounding error of long K (7 taps x 1024
      // channels) down; the epilogue adds the three in float32.
      constexpr uint32_t idesc = idesc_tf32_f32(kBM, BN);
      uint32_t it = 0;
      int acc_iter = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++acc_iter) {
        const int buf = acc_iter % NB;
        const int use = acc_iter / NB;
        if (use >= 1 && !mbar_wait(&tempty[buf], static_cast<uint32_t>(use - 1) & 1u, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * 3 * BN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          if (!mbar_wait(&full[s], (it / S) & 1u, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t base = smem_u32(smem + s * Cfg::kStage);
          const uint32_t d_main = acc + static_cast<uint32_t>((kb & 1) * BN);
          const uint32_t d_cross = acc + static_cast<uint32_t>(2 * BN);
#pragma unroll
          for (int k = 0; k < kKC / 8; ++k) {  // K = 8 per tf32 MMA: 32 bytes along the row
            const uint64_t ah = smem_desc_sw128(base + k * 32, 16, 1024);
            const uint64_t al = smem_desc_sw128(base + kATile + k * 32, 16, 1024);
            const uint64_t bh = smem_desc_sw128(base + 2 * kATile + k * 32, 16, 1024);
            const uint64_t bl =
                smem_desc_sw128(base + 2 * kATile + Cfg::kBTile + k * 32, 16, 1024);
            umma_tf32_ss(d_cross, al, bh, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            umma_tf32_ss(d_cross, ah, bl, idesc, 1u);
            umma_tf32_ss(d_main, ah, bh, idesc, (kb > 1 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[buf]);  // arrives when every MMA of the tile completed
      }
    }
  } else {
    // Epilogue: one thread per output row, 32-column chunks.
    const int group = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    int acc_iter = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++acc_iter) {
      const int buf = acc_iter % NB;
      if (NB >= 2 && buf != group) continue;  // another group's tile
      const TileCoord c = DecodeTile(t, m_tiles, n_tiles, BN);
      const int m = c.m0 + row;
      const bool valid = m < a.m_count;
      const int64_t orow = a.stride > 0 ? static_cast<int64_t>(m) * a.stride + c.phase : m;
      // Every epilogue thread continues after a timed-out wait (the error
      // word is set) so the group stays in step.
      (void)mbar_wait(&tfull[buf], static_cast<uint32_t>(acc_iter / NB) & 1u, a.err);
      __syncwarp();
      tc_fence_after_sync();
      const uint32_t acc = tmem + lanes + static_cast<uint32_t>(buf * 3 * BN);
#pragma unroll 1
      for (int ch = (NB >= 2 ? 0 : group); ch < BN / 32; ch += (NB >= 2 ? 1 : 2)) {
        float v[32];
        {
          uint32_t r0[32], r2[32];
          tmem_ld_32x32b_x32(acc + ch * 32, r0);
          tmem_ld_32x32b_x32(acc + 2 * BN + ch * 32, r2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]) + __uint_as_float(r2[j]);
          if (kblocks > 1) {  // uniform: the odd k blocks' sum exists
            tmem_ld_32x32b_x32(acc + BN + ch * 32, r0);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(r0[j]);
          }
        }
        if (!valid) continue;
        const int co = c.n0 + ch * 32;
        const int64_t off = orow * a.cout + co;
        const float4* b4 = reinterpret_cast<const float4*>(a.bias + co);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b = __ldg(b4 + q);
          v[4 * q] += b.x;
          v[4 * q + 1] += b.y;
          v[4 * q + 2] += b.z;
          v[4 * q + 3] += b.w;
        }
        if (a.resid != nullptr) {
          const float4* x4 = reinterpret_cast<const float4*>(a.resid + off);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 x = x4[q];
            v[4 * q] += x.x;
            v[4 * q + 1] += x.y;
            v[4 * q + 2] += x.z;
            v[4 * q + 3] += x.w;
          }
        }
        if (a.out_x != nullptr) {
          float4* o4 = reinterpret_cast<float4*>(a.out_x + off);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        if (a.alpha != nullptr) {
          const float4* al4 = reinterpret_cast<const float4*>(a.alpha + co);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 al = __ldg(al4 + q);
            v[4 * q] = snake(v[4 * q], al.x);
            v[4 * q + 1] = snake(v[4 * q + 1], al.y);
            v[4 * q + 2] = snake(v[4 * q + 2], al.z);
            v[4 * q + 3] = snake(v[4 * q + 3], al.w);
          }
        }
        store_split(a.out_hi + off, a.out_lo + off, v);
      }
      tc_fence_before_sync();
      mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// RVQ decode + fc2 (codec.cpp:215-233 with the tables of codec.cpp:136-160
// and fc2 folded together at load): latent[t][c] = bias[c] +
// sum_b table[b][codes[b][t]][c], written as the input convolution's
// split planes.  One CTA per frame.
__global__ void __launch_bounds__(256)
    codes_kernel(const float* __restrict__ table, const float* __restrict__ bias,
                 const int32_t* __restrict__ codes, int codebooks, int entries, int frames,
                 int width, float* __restrict__ hi, float* __restrict__ lo, uint32_t* err) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float sum = bias[c];
    for (int b = 0; b < codebooks; ++b) {
      int code = codes[static_cast<int64_t>(b) * frames + t];
      if (code < 0 || code >= entries) {
        if (c == 0) atomicOr(err, kErrBadArgument);
        code = 0;
      }
      sum += table[(static_cast<int64_t>(b) * entries + code) * width + c];
    }
    const float h = tf32_hi(sum);
    hi[static_cast<int64_t>(t) * width + c] = h;
    lo[static_cast<int64_t>(t) * width + c] = sum - h;
  }
}

// The output convolution (channels -> 1, kernel 7, codec.cpp:252-253): one
// thread per sample; the CTA stages its rows plus the 3-row halos of the
// snake'd input (hi + lo = the float32 value) in shared memory, rows padded
// by one word so the threads of a warp (consecutive rows) hit distinct banks.
constexpr int kOutRows = 128;
constexpr int kOutMaxC = 64;
__global__ void __launch_bounds__(kOutRows)
    output_conv_kernel(const float* __restrict__ hi, const float* __restrict__ lo, int rows,
                       int channels, const float* __restrict__ weight /* [7][channels] */,
                       const float* __restrict__ bias, float* __restrict__ out) {
  __shared__ float tile[(kOutRows + 6) * (kOutMaxC + 1)];
  __shared__ float w[7 * kOutMaxC];
  pdl_wait();
  pdl_trigger();
  const int stride = channels + 1;
  const int t0 = blockIdx.x * kOutRows;
  for (int i = threadIdx.x; i < 7 * channels; i += kOutRows) w[i] = weight[i];
  for (int i = threadIdx.x; i < (kOutRows + 6) * channels; i += kOutRows) {
    const int r = i / channels, c = i - r * channels;
    const int t = t0 - 3 + r;
    float v = 0.0f;
    if (t >= 0 && t < rows) {
      const int64_t k = static_cast<int64_t>(t) * channels + c;
      v = hi[k] + lo[k];
    }
    tile[r * stride + c] = v;
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= rows) return;
  float acc = 0.0f;
  for (int k = 0; k < 7; ++k) {
    const float* row = tile + (threadIdx.x + k) * stride;
    const float* wk = w + k * channels;
    for (int c = 0; c < channels; ++c) acc = fmaf(wk[c], row[c], acc);
  }
  out[t] = acc + bias[0];
}

// Load-time products of the RVQ tables: C[m][n] = sum_k A[m][k] B[n][k]
// (+ bias[n]), float32, 16 x 16 tiles.
__global__ void __launch_bounds__(256)
    dense_kernel(const float* __restrict__ A, const float* __restrict__ B,
                 const float* __restrict__ bias, float* __restrict__ C, int M, int N, int K) {
  __shared__ float as[16][17], bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m = blockIdx.y * 16 + ty, n = blockIdx.x * 16 + tx;
  float acc = 0.0f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int ma = blockIdx.y * 16 + ty, nb = blockIdx.x * 16 + ty;
    as[ty][tx] = (ma < M && k0 + tx < K) ? A[static_cast<int64_t>(ma) * K + k0 + tx] : 0.0f;
    bs[ty][tx] = (nb < N && k0 + tx < K) ? B[static_cast<int64_t>(nb) * K + k0 + tx] : 0.0f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(as[ty][k], bs[tx][k], acc);
    __syncthreads();
  }
  if (m < M && n < N) C[static_cast<int64_t>(m) * N + n] = acc + (bias != nullptr ? bias[n] : 0.0f);
}

__global__ void split_kernel(const float* __restrict__ src, float* __restrict__ hi,
                             float* __restrict__ lo, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = src[i];
    const float h = tf32_hi(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

template <int BN>
void LaunchConvTyped(const ConvPlan& p, cudaStream_t stream) {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(conv_kernel<BN>),
                    static_cast<int>(ConvTile<BN>::kSmem));
  Launch(conv_kernel<BN>, p.grid, dim3(ConvTile<BN>::kThreads), ConvTile<BN>::kSmem, stream,
         "codec conv launch", p.map_a_hi, p.map_a_lo, p.map_b_hi, p.map_b_lo, p.args);
}

}  // namespace

void PlanConv(ConvPlan* p, const float* in_hi, const float* in_lo, int rows_in,
              const ConvWeights& w, int m_count, int phases, const ConvArgs& args) {
  OV_REQUIRE(w.cin % kKC == 0, "codec conv: input channels must be a multiple of 32");
  OV_REQUIRE(w.cout % 32 == 0, "codec conv: output channels must be a multiple of 32");
  // Tiles of up to 64 output channels (measured on the default decoder:
  // 2.58 ms per 250 frames against 2.65 ms with 128 and 3.11 ms with 32,
  // the wider tile buying no MMA rate where the operand feed binds);
  // OV_CODEC_BN=<32|64|128> in the environment overrides the cap (tuning aid).
  int cap = 64;
  if (const char* env = std::getenv("OV_CODEC_BN")) {
    const int v = std::atoi(env);
    if (v == 32 || v == 64 || v == 128) cap = v;
  }
  p->bn = std::min(w.cout, cap);
  OV_REQUIRE(p->bn == 32 || p->bn == 64 || p->bn == 128, "codec conv: output channels");
  p->args = args;
  p->args.cin = w.cin;
  p->args.cout = w.cout;
  p->args.m_count = m_count;
  p->args.bias = w.bias.get();
  if (p->args.err == nullptr) p->args.err = DeviceErrorWord();
  EncodeTensorMap2D(&p->map_a_hi, in_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.cin, rows_in,
                    static_cast<uint64_t>(w.cin) * 4, kKC, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  EncodeTensorMap2D(&p->map_a_lo, in_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.cin, rows_in,
                    static_cast<uint64_t>(w.cin) * 4, kKC, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t w_rows = static_cast<uint64_t>(w.taps) * w.cout;
  EncodeTensorMap2D(&p->map_b_hi, w.hi.get(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.cin, w_rows,
                    static_cast<uint64_t>(w.cin) * 4, kKC, static_cast<uint32_t>(p->bn),
                    CU_TENSOR_MAP_SWIZZLE_128B);
  EncodeTensorMap2D(&p->map_b_lo, w.lo.get(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.cin, w_rows,
                    static_cast<uint64_t>(w.cin) * 4, kKC, static_cast<uint32_t>(p->bn),
                    CU_TENSOR_MAP_SWIZZLE_128B);
  const int tiles = (m_count + kBM - 1) / kBM * (w.cout / p->bn) * phases;
  p->grid = dim3(static_cast<unsigned>(std::min(tiles, SmCount())), 1, 1);
}

void LaunchConv(const ConvPlan& p, cudaStream_t stream) {
  switch (p.bn) {
    case 32: LaunchConvTyped<32>(p, stream); break;
    case 64: LaunchConvTyped<64>(p, stream); break;
    default: LaunchConvTyped<128>(p, stream); break;
  }
}

void LaunchCodes(const float* table, const float* bias, const int32_t* codes, int codebooks,
                 int entries, int frames, int width, float* hi, float* lo, cudaStream_t stream) {
  if (frames == 0) return;
  Launch(codes_kernel, dim3(static_cast<unsigned>(frames)), dim3(256), 0, stream,
         "codec codes launch", table, bias, codes, codebooks, entries, frames, width, hi, lo,
         DeviceErrorWord());
}

void LaunchOutputConv(const float* hi, const float* lo, int rows, int channels,
                      const float* weight, const float* bias, float* out, cudaStream_t stream) {
  OV_REQUIRE(channels <= kOutMaxC, "codec output conv: too many channels");
  if (rows == 0) return;
  Launch(output_conv_kernel, dim3(static_cast<unsigned>((rows + kOutRows - 1) / kOutRows)),
         dim3(kOutRows), 0, stream, "codec output conv launch", hi, lo, rows, channels, weight,
         bias, out);
}

void LaunchDense(const float* A, const float* B, const float* bias, float* C, int M, int N, int K,
                 cudaStream_t stream) {
  Launch(dense_kernel, dim3(static_cast<unsigned>((N + 15) / 16), static_cast<unsigned>((M + 15) / 16)),
         dim3(256), 0, stream, "codec table launch", A, B, bias, C, M, N, K);
}

void LaunchSplit(const float* src, float* hi, float* lo, int64_t n, cudaStream_t stream) {
  if (n == 0) return;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
  Launch(split_kernel, dim3(blocks), dim3(256), 0, stream, "codec split launch", src, hi, lo, n);
}

}  // namespace codec
}  // namespace ovb
