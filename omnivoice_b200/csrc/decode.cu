// The decoding tail of one unmasking step on the device:
//   score_kernel  - guided log-softmax scoring, generator_kernels.hip:212-265
//   select_kernel - PositionSelector::Fill (decoding.cpp:70-106) and the
//                   code write-back of generator.cpp:526-535.
// Both read per-utterance descriptors so one launch serves a packed batch.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>

#include "internal.hpp"
#include "launch.hpp"
#include "ov_kernels.h"
#include "pack.hpp"
#include "ptx.cuh"

namespace ovb {
namespace {

constexpr int kScoreWarps = 8;
constexpr int kMaxVocabPerLane = 33;  // vocab <= 1056
constexpr int kSelectThreads = 1024;
constexpr int kMaxSlots = 32768;      // codebooks * frames per utterance

// Maps a float to a key whose unsigned order is the float order (+0 and -0
// must be canonicalised by the caller).
__device__ __forceinline__ uint32_t OrderedKey(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Philox-4x32-10 (Salmon, Moraes, Dror & Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): returns the first output word.
__device__ __forceinline__ uint32_t Philox4x32(uint32_t c0, uint32_t c1, uint32_t c2,
                                               uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0;
    const uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

__device__ __forceinline__ float GumbelFromUniform(float u) {
  return -logf(-logf(u + 1e-10f) + 1e-10f);
}

// One warp per (frame, codebook) item; rows held in registers so logits
// are read from memory once.
__global__ void __launch_bounds__(kScoreWarps * 32)
    score_kernel(const float* __restrict__ logits, int64_t ld, int total_frames, int codebooks,
                 int vocab, uint32_t mask_id, float guidance, const UttDesc* __restrict__ utts,
                 const int32_t* __restrict__ frame_utt, int single_frames,
                 int32_t* __restrict__ prediction, float* __restrict__ confidence) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kScoreWarps + (threadIdx.x >> 5);
  if (item >= static_cast<int64_t>(total_frames) * codebooks) return;
  const int gf = static_cast<int>(item / codebooks);
  const int c = static_cast<int>(item % codebooks);
  int64_t cond_row, uncond_row, out;
  if (utts != nullptr) {
    const UttDesc d = utts[frame_utt[gf]];
    const int f = gf - d.frame_base;
    cond_row = d.logit_row + f;
    uncond_row = cond_row + d.frames;
    out = d.slot_base + static_cast<int64_t>(c) * d.frames + f;
  } else {
    cond_row = gf;
    uncond_row = single_frames + gf;
    out = static_cast<int64_t>(c) * single_frames + gf;
  }
  const float* cr = logits + cond_row * ld + static_cast<int64_t>(c) * vocab;
  const float* ur = logits + uncond_row * ld + static_cast<int64_t>(c) * vocab;
  float x[kMaxVocabPerLane], y[kMaxVocabPerLane];
  float cmax = -FLT_MAX, umax = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxVocabPerLane; ++i) {
    const int j = lane + 32 * i;
    x[i] = j < vocab ? cr[j] : -FLT_MAX;
    y[i] = j < vocab ? ur[j] : -FLT_MAX;
    cmax = fmaxf(cmax, x[i]);
    umax = fmaxf(umax, y[i]);
  }
  cmax = warp_max(cmax);
  umax = warp_max(umax);
  float csum = 0.f, usum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVocabPerLane; ++i) {
    if (lane + 32 * i < vocab) {
      csum += expf(x[i] - cmax);
      usum += expf(y[i] - umax);
    }
  }
  const float clse = cmax + logf(warp_sum(csum));
  const float ulse = umax + logf(warp_sum(usum));
  float gmax = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxVocabPerLane; ++i) {
    // c + guidance * (c - u), rounded step by step like the reference.
    const float cc = __fsub_rn(x[i], clse);
    const float uu = __fsub_rn(y[i], ulse);
    x[i] = __fadd_rn(cc, __fmul_rn(guidance, __fsub_rn(cc, uu)));
    if (lane + 32 * i < vocab) gmax = fmaxf(gmax, x[i]);
  }
  gmax = warp_max(gmax);
  float gsum = 0.f;
  float best = -FLT_MAX;
  int best_index = vocab;
#pragma unroll
  for (int i = 0; i < kMaxVocabPerLane; ++i) {
    const int j = lane + 32 * i;
    if (j < vocab) {
      gsum += expf(x[i] - gmax);
      if (j != static_cast<int>(mask_id) && x[i] > best) {
        best = x[i];
        best_index = j;
      }
    }
  }
  const float glse = gmax + logf(warp_sum(gsum));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, best_index, o);
    if (ov > best || (ov == best && oi < best_index)) {
      best = ov;
      best_index = oi;
    }
  }
  if (lane == 0) {
    prediction[out] = best_index;
    confidence[out] = best - glse;
  }
}

// Block-wide exclusive prefix sum of one value per thread.
__device__ __forceinline__ int BlockExclusiveScan(int value, int* warp_totals, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int inclusive = value;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, inclusive, o);
    if (lane >= o) inclusive += n;
  }
  if (lane == 31) warp_totals[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    const int nwarps = blockDim.x >> 5;
    int t = lane < nwarps ? warp_totals[lane] : 0;
    int inc = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += n;
    }
    if (lane < nwarps) warp_totals[lane] = inc - t;  // exclusive warp offsets
    if (lane == 31) *total = inc;
  }
  __syncthreads();
  return warp_totals[warp] + inclusive - value;
}

// One CTA per utterance.  Keys live in shared memory; a 4-pass 8-bit radix
// select finds the count-th largest key T, then every key > T and the
// lowest-index keys == T are taken, which is exactly the set of the first
// `count` slots under the reference's (score desc, index asc) order.
__global__ void __launch_bounds__(kSelectThreads)
    select_kernel(const int32_t* __restrict__ prediction, const float* __restrict__ confidence,
                  int codebooks, float layer_penalty, float temperature, int noise_mode,
                  uint32_t mask_id, int32_t* __restrict__ codes,
                  int32_t* __restrict__ unmasked_at, int32_t* __restrict__ ids,
                  int64_t ids_rows, UttDesc single, const UttDesc* __restrict__ table,
                  StepControl ctl, int explicit_count, int explicit_step,
                  int single_cond_row, int single_uncond_row, uint32_t* err) {
  extern __shared__ uint32_t keys[];
  __shared__ uint32_t hist[256];
  __shared__ int warp_totals[32];
  __shared__ int s_total;
  __shared__ uint32_t s_digit;
  __shared__ int s_remaining;
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const UttDesc d = table != nullptr ? table[blockIdx.x] : single;
  const int frames = d.frames;
  const int n = codebooks * frames;
  if (n > kMaxSlots) {
    if (tid == 0) atomicOr(err, kErrBadArgument);
    return;
  }
  int step = explicit_step;
  int count = explicit_count;
  int launch = 0;
  if (table != nullptr && d.counts != nullptr) {
    launch = ctl.launch[blockIdx.x];
    step = ctl.step_list[launch];
    count = d.counts[step];
  }
  count = min(count, n);
  const float* gumbel = nullptr;
  if (noise_mode == OV_NOISE_BUFFER && d.gumbel != nullptr)
    gumbel = d.gumbel + (table != nullptr ? static_cast<int64_t>(step) * d.gumbel_stride : 0);
  const int32_t* pred = prediction + d.slot_base;
  const float* conf = confidence + d.slot_base;
  int32_t* code = codes + d.slot_base;
  for (int i = tid; i < n; i += blockDim.x) {
    const int c = i / frames;
    float score = conf[i] - static_cast<float>(c) * layer_penalty;
    if (temperature > 0.0f) {
      float g = 0.0f;
      if (noise_mode == OV_NOISE_BUFFER) {
        g = gumbel != nullptr ? gumbel[i] : 0.0f;
      } else if (noise_mode == OV_NOISE_DEVICE) {
        const uint32_t r = Philox4x32(static_cast<uint32_t>(i), static_cast<uint32_t>(step),
                                      0u, 0u, static_cast<uint32_t>(d.noise_seed),
                                      static_cast<uint32_t>(d.noise_seed >> 32));
        g = GumbelFromUniform(static_cast<float>(r >> 8) * 0x1.0p-24f);
      }
      score = __fadd_rn(__fdiv_rn(score, temperature), g);
    }
    if (code[i] != static_cast<int32_t>(mask_id)) score = -INFINITY;
    if (score == 0.0f) score = 0.0f;  // one key for +0 and -0
    keys[i] = OrderedKey(score);
  }
  __syncthreads();
  if (count > 0) {
    uint32_t prefix = 0, prefix_mask = 0;
    int remaining = count;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += blockDim.x) {
        const uint32_t k = keys[i];
        if ((k & prefix_mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid < 32) {
        // lane l owns bins [8l, 8l+8); find the bin where the running count
        // from the top reaches `remaining`.
        uint32_t local = 0;
#pragma unroll
        for (int b = 0; b < 8; ++b) local += hist[tid * 8 + b];
        uint32_t above = 0;  // sum over lanes > tid
        uint32_t inc = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xFFFFFFFFu, inc, o);
          if (tid + o < 32) inc += v;
        }
        above = inc - local;
        const uint32_t want = static_cast<uint32_t>(remaining);
        if (above < want && want <= above + local) {
          uint32_t cum = above;
          for (int b = 7; b >= 0; --b) {
            const uint32_t h = hist[tid * 8 + b];
            if (cum + h >= want) {
              s_digit = static_cast<uint32_t>(tid * 8 + b);
              s_remaining = static_cast<int>(want - cum);
              break;
            }
            cum += h;
          }
        }
      }
      __syncthreads();
      prefix |= s_digit << shift;
      prefix_mask |= 255u << shift;
      remaining = s_remaining;
      __syncthreads();
    }
    const uint32_t threshold = prefix;
    const int need = remaining;  // keys == threshold to take, lowest index first
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int begin = min(n, tid * per);
    const int end = min(n, begin + per);
    int equal = 0;
    for (int i = begin; i < end; ++i) equal += keys[i] == threshold ? 1 : 0;
    int rank = BlockExclusiveScan(equal, warp_totals, &s_total);
    const int64_t cond_base = table != nullptr ? d.row_base + d.length - frames : single_cond_row;
    const int64_t uncond_base = table != nullptr ? d.row_base + d.length : single_uncond_row;
    for (int i = begin; i < end; ++i) {
      const uint32_t k = keys[i];
      bool take = k > threshold;
      if (k == threshold) {
        take = rank < need;
        ++rank;
      }
      if (!take) continue;
      const int c = i / frames;
      const int f = i % frames;
      const int32_t value = pred[i];
      code[i] = value;
      if (unmasked_at != nullptr) unmasked_at[d.slot_base + i] = step;
      if (ids != nullptr) {
        ids[c * ids_rows + cond_base + f] = value;
        ids[c * ids_rows + uncond_base + f] = value;
      }
    }
  }
  if (table != nullptr && d.counts != nullptr && tid == 0) ctl.launch[blockIdx.x] = launch + 1;
}

}  // namespace

void LaunchScore(const float* logits, int64_t ld, int total_frames, int codebooks, int vocab,
                 uint32_t mask_id, float guidance, const UttDesc* utts, const int32_t* frame_utt,
                 int single_frames, int32_t* prediction, float* confidence,
                 cudaStream_t stream) {
  if (total_frames == 0) return;
  if (vocab > 32 * kMaxVocabPerLane) throw Error(OV_ERR_UNSUPPORTED, "vocab > 1056");
  const int64_t items = static_cast<int64_t>(total_frames) * codebooks;
  Launch(score_kernel, dim3(static_cast<unsigned>((items + kScoreWarps - 1) / kScoreWarps)),
         dim3(kScoreWarps * 32), 0, stream, "score kernel launch", logits, ld, total_frames,
         codebooks, vocab, mask_id, guidance, utts, frame_utt, single_frames, prediction,
         confidence);
}

void ConfigureSelectKernel() {
  SetMaxDynamicSmem(reinterpret_cast<const void*>(select_kernel),
                    kMaxSlots * static_cast<int>(sizeof(uint32_t)));
}

void LaunchSelect(const int32_t* prediction, const float* confidence, int codebooks,
                  float layer_penalty, float temperature, int noise_mode, uint32_t mask_id,
                  int32_t* codes, int32_t* unmasked_at, int32_t* ids, int64_t ids_rows,
                  const UttDesc& single, const UttDesc* table, int utterances,
                  StepControl ctl, int max_slots, int explicit_count, int explicit_step,
                  int single_cond_row, int single_uncond_row, cudaStream_t stream) {
  if (utterances == 0) return;
  if (max_slots > kMaxSlots)
    throw Error(OV_ERR_UNSUPPORTED, "more than 32768 code slots in one utterance");
  const size_t smem = static_cast<size_t>(max_slots > 0 ? max_slots : 1) * sizeof(uint32_t);
  SetMaxDynamicSmem(reinterpret_cast<const void*>(select_kernel),
                    kMaxSlots * static_cast<int>(sizeof(uint32_t)));
  Launch(select_kernel, dim3(utterances), dim3(kSelectThreads), smem, stream,
         "select kernel launch", prediction, confidence, codebooks, layer_penalty, temperature,
         noise_mode, mask_id, codes, unmasked_at, ids, ids_rows, single, table, ctl,
         explicit_count, explicit_step, single_cond_row, single_uncond_row, DeviceErrorWord());
}

}  // namespace ovb

using namespace ovb;

extern "C" {

int ov_score(const float* logits, size_t ld, size_t frames, size_t codebooks, size_t vocab,
             uint32_t mask_id, float guidance, int32_t* prediction, float* confidence,
             ov_stream_t stream) {
  return Guard("ov_score: ", [&] {
    LaunchScore(logits, static_cast<int64_t>(ld), static_cast<int>(frames),
                static_cast<int>(codebooks), static_cast<int>(vocab), mask_id, guidance,
                nullptr, nullptr, static_cast<int>(frames), prediction, confidence,
                AsStream(stream));
  });
}

int ov_select_positions(const int32_t* prediction, const float* confidence, size_t codebooks,
                        size_t frames, size_t count, float layer_penalty, float temperature,
                        int noise_mode, const float* gumbel, uint64_t noise_seed, int32_t step,
                        uint32_t mask_id, int32_t* codes, int32_t* unmasked_at, int32_t* ids,
                        size_t ids_rows, size_t cond_row, size_t uncond_row,
                        ov_stream_t stream) {
  return Guard("ov_select_positions: ", [&] {
    OV_REQUIRE(noise_mode != OV_NOISE_BUFFER || gumbel != nullptr || temperature <= 0.0f,
               "noise buffer missing");
    UttDesc d{};
    d.frames = static_cast<int32_t>(frames);
    d.noise_seed = noise_seed;
    d.gumbel = gumbel;
    d.gumbel_stride = static_cast<int32_t>(codebooks * frames);
    StepControl ctl{nullptr, nullptr};
    LaunchSelect(prediction, confidence, static_cast<int>(codebooks), layer_penalty,
                 temperature, noise_mode, mask_id, codes, unmasked_at, ids,
                 static_cast<int64_t>(ids_rows), d, nullptr, 1, ctl,
                 static_cast<int>(codebooks * frames), static_cast<int>(count), step,
                 static_cast<int>(cond_row), static_cast<int>(uncond_row), AsStream(stream));
  });
}

float ov_gumbel_from_uniform(float uniform) {
  return -std::log(-std::log(uniform + 1e-10f) + 1e-10f);
}

}  // extern "C"
