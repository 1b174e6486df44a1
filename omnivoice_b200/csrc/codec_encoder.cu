// The audio tokenizer's encoder on one GPU (voice cloning): 24 kHz samples
// to residual-vector-quantized codes.  Replaces the reference's
// Codec::Encode (codec_encoder.cpp:249-458) and its weight loading
// (LoadEncoder, codec_encoder.cpp:72-247), behind the C-ABI of ov_codec.h.
//
// Everything runs in float32 on the CUDA cores, time-major ([time][channels],
// so a convolution tap is a row offset and a strided convolution a row
// step):
//   conv_kernel       every convolution and dense layer as one implicit GEMM
//                     (64 x 64 output tiles, 16-deep k chunks through shared
//                     memory, 4 x 4 outputs per thread) with the element-wise
//                     work around it fused: snake or ELU on the input as it is
//                     loaded, bias, GELU and a residual add on the output
//   attention_kernel  HuBERT's multi-head attention, one warp per query with
//                     an online softmax over shared-memory key / value tiles
//   groupnorm / layernorm / gather-scale, and rvq_kernel: the quantizer, one
//                     CTA per frame walking the codebooks in order.
// The encoder runs once per cloned voice and is cached by the caller
// (runner.cpp:148-172), so it is sized for correctness and a few
// milliseconds per second of audio, not for the tensor cores.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include "device_buffer.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ov_codec.h"
#include "ptx.cuh"
#include "safetensors.hpp"
#include "synthetic.hpp"

namespace ovb {
namespace encoder {
namespace {

constexpr int kResidualKernel = 7;        // codec_state.hpp:26
constexpr int kDilations[3] = {1, 3, 9};  // codec_state.hpp:27
constexpr float kGroupNormEps = 1e-5f;    // codec_encoder.cpp:286
constexpr int kHubertPad = 160;           // codec_encoder.cpp:262-263

enum Pre : int { kPreNone = 0, kPreSnake = 1, kPreElu = 2 };
enum Act : int { kActNone = 0, kActGelu = 1 };

__device__ __forceinline__ float gelu(float x) {  // encoder_kernels.hip:41-43
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// ------------------------------------------------------------ convolution

struct ConvArgs {
  const float* x;      // [rows_in][ldx]; group g reads channels g * cin_g ..
  int64_t ldx;
  int rows_in;
  const float* w;      // [groups][taps][cout_g][cin_g]
  const float* bias;   // [groups * cout_g] or null
  const float* alpha;  // snake alphas [cin] (kPreSnake)
  float* y;            // [rows_out][ldy]
  int64_t ldy;
  const float* resid;  // [rows_out][ldr] added after the activation, or null (may be y)
  int64_t ldr;
  int rows_out, cin_g, cout_g, groups, taps, stride, dilation, pad, pre, act;
  // Split-K: splits > 1 CTAs share each output tile, split s taking
  // (tap, 16-channel chunk) steps [s * per_split, (s + 1) * per_split) and
  // writing raw sums to partial[s][rows_out][groups * cout_g]; reduce_kernel
  // adds the splits in order and applies the epilogue.
  float* partial;
  int splits, per_split;
};

constexpr int kTileM = 64, kTileN = 64, kTileK = 16;

// y[m][o] = act(bias[o] + sum_{tap, i} w[g][tap][o][i] pre(x[m s + tap d - pad][g cin_g + i]))
//           + resid[m][o]; rows outside the input read as zero (no pre).
__global__ void __launch_bounds__(256) conv_kernel(const ConvArgs a) {
  __shared__ __align__(16) float xs[kTileK][kTileM + 4];
  __shared__ __align__(16) float ws[kTileK][kTileN + 4];
  const int g = blockIdx.z / a.splits;
  const int split = blockIdx.z % a.splits;
  const int kchunks = (a.cin_g + kTileK - 1) / kTileK;
  const int it0 = split * a.per_split;
  const int it1 = min(it0 + a.per_split, a.taps * kchunks);
  const int m0 = blockIdx.x * kTileM;
  const int n0 = blockIdx.y * kTileN;
  const int tx = threadIdx.x & 15;   // output columns n0 + 4 tx ..
  const int ty = threadIdx.x >> 4;   // output rows m0 + 4 ty ..
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int it = it0; it < it1; ++it) {
    const int tap = it / kchunks;
    const int k0 = (it % kchunks) * kTileK;
    const float* wt = a.w + (static_cast<int64_t>(g) * a.taps + tap) * a.cout_g * a.cin_g;
    {
      for (int i = threadIdx.x; i < kTileM * kTileK; i += 256) {
        const int r = i >> 4, kk = i & 15;
        const int m = m0 + r, ch = k0 + kk;
        float v = 0.0f;
        if (m < a.rows_out && ch < a.cin_g) {
          const int64_t src = static_cast<int64_t>(m) * a.stride + static_cast<int64_t>(tap) * a.dilation - a.pad;
          if (src >= 0 && src < a.rows_in) {
            const int c = g * a.cin_g + ch;
            v = a.x[src * a.ldx + c];
            if (a.pre == kPreSnake) {
              const float al = a.alpha[c];
              const float s = sinf(al * v);
              v = v + s * s / (al + 1e-9f);  // codec_kernels.hip:11-27
            } else if (a.pre == kPreElu) {
              v = v > 0.0f ? v : expm1f(v);
            }
          }
        }
        xs[kk][r] = v;
      }
      for (int i = threadIdx.x; i < kTileN * kTileK; i += 256) {
        const int nn = i >> 4, kk = i & 15;
        const int n = n0 + nn, k = k0 + kk;
        ws[kk][nn] = n < a.cout_g && k < a.cin_g ? wt[static_cast<int64_t>(n) * a.cin_g + k] : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kTileK; ++kk) {
        const float4 xv = *reinterpret_cast<const float4*>(&xs[kk][4 * ty]);
        const float4 wv = *reinterpret_cast<const float4*>(&ws[kk][4 * tx]);
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
        const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + 4 * ty + i;
    if (m >= a.rows_out) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + 4 * tx + j;
      if (n >= a.cout_g) continue;
      const int o = g * a.cout_g + n;
      if (a.splits > 1) {
        a.partial[(static_cast<int64_t>(split) * a.rows_out + m) * (a.groups * a.cout_g) + o] = acc[i][j];
        continue;
      }
      float v = acc[i][j] + (a.bias != nullptr ? a.bias[o] : 0.0f);
      if (a.act == kActGelu) v = gelu(v);
      if (a.resid != nullptr) v += a.resid[static_cast<int64_t>(m) * a.ldr + o];
      a.y[static_cast<int64_t>(m) * a.ldy + o] = v;
    }
  }
}

// The splits of conv_kernel summed in split order, then its epilogue.
__global__ void reduce_kernel(const ConvArgs a) {
  const int cout = a.groups * a.cout_g;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(a.rows_out) * cout) return;
  const int64_t m = i / cout;
  const int o = static_cast<int>(i % cout);
  float v = 0.0f;
  for (int s = 0; s < a.splits; ++s) v += a.partial[s * static_cast<int64_t>(a.rows_out) * cout + i];
  v += a.bias != nullptr ? a.bias[o] : 0.0f;
  if (a.act == kActGelu) v = gelu(v);
  if (a.resid != nullptr) v += a.resid[m * a.ldr + o];
  a.y[m * a.ldy + o] = v;
}

// ------------------------------------------------------------- attention

// HuBERT self-attention (codec_encoder.cpp:330-356): qkv [T][3H] (q | k | v),
// out [T][H]; head h uses columns h d .. h d + d - 1 of each.  One warp per
// query, eight queries of one head per CTA; keys and values pass through
// shared memory 32 at a time; softmax(scale q.k) with a running maximum.
constexpr int kAttnKeys = 32;
constexpr int kAttnMaxD = 128;

__global__ void __launch_bounds__(256) attention_kernel(const float* qkv, int rows, int width,
                                                        int head_dim, float scale, float* out) {
  __shared__ float ks[kAttnKeys][kAttnMaxD + 1];
  __shared__ float vs[kAttnKeys][kAttnMaxD + 1];
  __shared__ float qs[8][kAttnMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int q = blockIdx.x * 8 + warp;
  const int64_t ld = 3 * static_cast<int64_t>(width);
  const int d = head_dim;
  for (int i = lane; i < d; i += 32) qs[warp][i] = q < rows ? qkv[q * ld + h * d + i] : 0.0f;
  float m = -INFINITY, l = 0.0f;
  float o[kAttnMaxD / 32];
#pragma unroll
  for (int t = 0; t < kAttnMaxD / 32; ++t) o[t] = 0.0f;
  for (int k0 = 0; k0 < rows; k0 += kAttnKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kAttnKeys * d; i += 256) {
      const int r = i / d, c = i % d;
      const int key = k0 + r;
      ks[r][c] = key < rows ? qkv[key * ld + width + h * d + c] : 0.0f;
      vs[r][c] = key < rows ? qkv[key * ld + 2 * width + h * d + c] : 0.0f;
    }
    __syncthreads();
    const int key = k0 + lane;
    float s = -INFINITY;
    if (key < rows) {
      float dot = 0.0f;
      for (int c = 0; c < d; ++c) dot = fmaf(qs[warp][c], ks[lane][c], dot);
      s = dot * scale;
    }
    const float m_new = fmaxf(m, warp_max(s));
    const float corr = expf(m - m_new);  // 0 on the first tile (m = -inf)
    const float p = key < rows ? expf(s - m_new) : 0.0f;
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int t = 0; t < kAttnMaxD / 32; ++t) o[t] *= corr;
    for (int j = 0; j < kAttnKeys; ++j) {
      const float pj = __shfl_sync(0xFFFFFFFFu, p, j);
#pragma unroll
      for (int t = 0; t < kAttnMaxD / 32; ++t) {
        const int c = lane + 32 * t;
        if (c < d) o[t] = fmaf(pj, vs[j][c], o[t]);
      }
    }
    m = m_new;
  }
  if (q < rows) {
    const float inv = 1.0f / l;
#pragma unroll
    for (int t = 0; t < kAttnMaxD / 32; ++t) {
      const int c = lane + 32 * t;
      if (c < d) out[q * static_cast<int64_t>(width) + h * d + c] = o[t] * inv;
    }
  }
}

// --------------------------------------------------------- normalisations

// Per-channel group norm over time + GELU, in place on [rows][channels]
// (encoder_kernels.hip GroupNormGeluKernel): 32 channels per CTA, eight
// row lanes.
__global__ void __launch_bounds__(256) groupnorm_gelu_kernel(float* x, int rows, int channels,
                                                             const float* weight,
                                                             const float* bias, float eps) {
  __shared__ float part[8][33];
  __shared__ float stat[32];
  const int cl = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  const bool ok = c < channels;
  float s = 0.0f;
  if (ok)
    for (int r = rl; r < rows; r += 8) s += x[static_cast<int64_t>(r) * channels + c];
  part[rl][cl] = s;
  __syncthreads();
  if (rl == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += part[i][cl];
    stat[cl] = t / static_cast<float>(rows);
  }
  __syncthreads();
  const float mean = stat[cl];
  float q = 0.0f;
  if (ok)
    for (int r = rl; r < rows; r += 8) {
      const float v = x[static_cast<int64_t>(r) * channels + c] - mean;
      q += v * v;
    }
  __syncthreads();
  part[rl][cl] = q;
  __syncthreads();
  if (rl == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += part[i][cl];
    stat[cl] = rsqrtf(t / static_cast<float>(rows) + eps);
  }
  __syncthreads();
  if (!ok) return;
  const float inv = stat[cl], w = weight[c], b = bias[c];
  for (int r = rl; r < rows; r += 8) {
    float* p = x + static_cast<int64_t>(r) * channels + c;
    *p = gelu((*p - mean) * inv * w + b);
  }
}

// Row layer norm (encoder_kernels.hip LayerNormKernel), one warp per row;
// y may be x.
__global__ void __launch_bounds__(256) layernorm_kernel(const float* x, float* y, int rows,
                                                        int width, const float* weight,
                                                        const float* bias, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* in = x + static_cast<int64_t>(row) * width;
  float s = 0.0f;
  for (int j = lane; j < width; j += 32) s += in[j];
  const float mean = warp_sum(s) / static_cast<float>(width);
  float q = 0.0f;
  for (int j = lane; j < width; j += 32) {
    const float v = in[j] - mean;
    q += v * v;
  }
  const float inv = rsqrtf(warp_sum(q) / static_cast<float>(width) + eps);
  float* o = y + static_cast<int64_t>(row) * width;
  for (int j = lane; j < width; j += 32) o[j] = (in[j] - mean) * inv * weight[j] + bias[j];
}

__global__ void add_kernel(float* y, const float* x, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] += x[i];
}

// out[f][:] = total[f * step][:] * scale (the averaged states of every
// step-th HuBERT frame, codec_encoder.cpp:357-378).
__global__ void pick_scale_kernel(const float* total, int width, int step, int frames, float scale,
                                  float* out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(frames) * width) return;
  const int64_t f = i / width, c = i % width;
  out[i] = total[f * step * width + c] * scale;
}

// ------------------------------------------------------------- quantizer

// codec_encoder.cpp:436-456 for one frame per CTA: per codebook, h =
// project_in(r); the entry maximising -((|h|^2 - 2 h.e) + |e|^2), lowest
// index on ties (encoder_kernels.hip NearestEntryKernel); r -= its decoded
// vector.  residual [frames][J] is consumed in place.
__global__ void __launch_bounds__(256) rvq_kernel(float* residual, int frames, int joint,
                                                  int codebooks, int entries, int dim,
                                                  const float* proj_w, const float* proj_b,
                                                  const float* codebook, const float* norms,
                                                  const float* tables, int32_t* codes) {
  extern __shared__ float sm[];
  float* r = sm;              // [joint]
  float* hv = r + joint;      // [dim]
  float* best_v = hv + dim;   // [256]
  int* best_i = reinterpret_cast<int*>(best_v + 256);
  const int f = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* row = residual + static_cast<int64_t>(f) * joint;
  for (int j = threadIdx.x; j < joint; j += 256) r[j] = row[j];
  __syncthreads();
  for (int c = 0; c < codebooks; ++c) {
    const float* W = proj_w + static_cast<int64_t>(c) * dim * joint;
    for (int k = warp; k < dim; k += 8) {
      float s = 0.0f;
      for (int j = lane; j < joint; j += 32) s = fmaf(W[static_cast<int64_t>(k) * joint + j], r[j], s);
      s = warp_sum(s);
      if (lane == 0) hv[k] = s + proj_b[c * dim + k];
    }
    __syncthreads();
    float norm = 0.0f;
    for (int k = 0; k < dim; ++k) norm = fmaf(hv[k], hv[k], norm);
    const float* E = codebook + static_cast<int64_t>(c) * entries * dim;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int e = threadIdx.x; e < entries; e += 256) {
      float dot = 0.0f;
      for (int k = 0; k < dim; ++k) dot = fmaf(hv[k], E[static_cast<int64_t>(e) * dim + k], dot);
      const float dist = -((norm - 2.0f * dot) + norms[c * entries + e]);
      if (dist > bv) {  // ascending e: the first maximum
        bv = dist;
        bi = e;
      }
    }
    best_v[threadIdx.x] = bv;
    best_i[threadIdx.x] = bi;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
      if (threadIdx.x < s) {
        const float ov = best_v[threadIdx.x + s];
        const int oi = best_i[threadIdx.x + s];
        if (ov > best_v[threadIdx.x] || (ov == best_v[threadIdx.x] && oi < best_i[threadIdx.x])) {
          best_v[threadIdx.x] = ov;
          best_i[threadIdx.x] = oi;
        }
      }
      __syncthreads();
    }
    const int idx = min(max(best_i[0], 0), entries - 1);
    if (threadIdx.x == 0) codes[static_cast<int64_t>(c) * frames + f] = idx;
    const float* t = tables + (static_cast<int64_t>(c) * entries + idx) * joint;
    for (int j = threadIdx.x; j < joint; j += 256) r[j] -= t[j];
    __syncthreads();
  }
}

}  // namespace

// ------------------------------------------------------------------ engine

using TensorSource = std::function<const float*(const std::string&, const std::vector<uint64_t>&)>;

struct Conv {
  DeviceBuffer<float> w;     // [groups][taps][cout_g][cin_g]
  DeviceBuffer<float> bias;  // [cout] or empty
  int cin_g = 0, cout_g = 0, groups = 1, taps = 1, stride = 1, dilation = 1, pad = 0;

  int RowsOut(int rows_in) const {
    return (rows_in + 2 * pad - dilation * (taps - 1) - 1) / stride + 1;
  }
};

struct HubertLayer {
  Conv qkv, out, inter, final_;
  DeviceBuffer<float> n1w, n1b, n2w, n2b;
};

struct ResUnit {
  DeviceBuffer<float> alpha1, alpha2;
  Conv conv1, conv2;
};

struct DacBlock {
  ResUnit units[3];
  DeviceBuffer<float> alpha;
  Conv down;
};

class EncoderEngine {
 public:
  EncoderEngine(const ov_codec_encoder_config& cfg, int device) : cfg_(cfg), device_(device) {
    Check(cudaSetDevice(device_), "cudaSetDevice");
    Check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    sms_ = SmCount();
    CheckConfig();
  }
  ~EncoderEngine() {
    if (stream_ != nullptr) {
      (void)cudaSetDevice(device_);
      (void)cudaStreamDestroy(stream_);
    }
  }
  EncoderEngine(const EncoderEngine&) = delete;
  EncoderEngine& operator=(const EncoderEngine&) = delete;

  size_t FrameSamples() const {
    size_t p = 1;
    for (size_t i = 0; i < cfg_.num_downsampling; ++i) p *= cfg_.downsampling_ratios[i];
    return p;
  }
  void Load(const TensorSource& src);
  size_t Encode(const float* samples, size_t count, int32_t* codes, size_t capacity);

 private:
  void CheckConfig() const;
  size_t Joint() const { return cfg_.hidden_size + cfg_.latent_channels; }
  DeviceBuffer<float> Upload(const float* data, size_t n);
  Conv MakeConv(const TensorSource& src, const std::string& prefix, int cin, int cout, int kernel,
                int stride, int dilation, int pad, int groups, bool bias);
  Conv MakeDense(const TensorSource& src, const std::string& prefix, int in, int out);
  DeviceBuffer<float> Vec(const TensorSource& src, const std::string& name,
                          const std::vector<uint64_t>& shape);
  // Runs `c` on x [rows_in][ldx] into y [rows_out][ldy] (rows_out < 0: the
  // convolution's own output length); returns rows_out.
  int Run(const Conv& c, const float* x, int64_t ldx, int rows_in, float* y, int64_t ldy,
          int pre = kPreNone, const float* alpha = nullptr, int act = kActNone,
          const float* resid = nullptr, int64_t ldr = 0, int rows_out = -1);
  void LayerNorm(const float* x, float* y, int rows, int width, const DeviceBuffer<float>& w,
                 const DeviceBuffer<float>& b, float eps);

  ov_codec_encoder_config cfg_;
  int device_;
  cudaStream_t stream_ = nullptr;
  // HuBERT
  std::vector<Conv> features_;
  DeviceBuffer<float> gn_w_, gn_b_, proj_nw_, proj_nb_, enc_nw_, enc_nb_;
  Conv projection_, position_;
  std::vector<HubertLayer> layers_;
  // semantic encoder
  Conv sem_in_;
  Conv sem_unit_[2][2][2];  // [block][unit][conv1, conv2]
  Conv sem_conv_[2];
  // DAC encoder
  Conv dac_in_;
  std::vector<DacBlock> blocks_;
  DeviceBuffer<float> dac_alpha_;
  Conv dac_out_;
  // quantizer
  Conv fc_;
  DeviceBuffer<float> proj_in_w_, proj_in_b_, codebooks_, norms_, tables_;
  // work buffers
  DeviceBuffer<float> buf_[6];
  DeviceBuffer<float> partial_;  // split-K partial sums
  int sms_ = 148;
  DeviceBuffer<int32_t> codes_;
};

void EncoderEngine::CheckConfig() const {
  const ov_codec_encoder_config& c = cfg_;
  auto need = [](bool ok, const char* what) {
    if (!ok) throw Error(OV_ERR_UNSUPPORTED, std::string("unsupported codec encoder: ") + what);
  };
  need(c.sample_rate > 0 && c.semantic_sample_rate > 0, "sample rates");
  need(c.codebooks >= 1 && c.codebook_size >= 1 && c.codebook_dim >= 1, "quantizer shape");
  need(c.hidden_size >= 1 && c.heads >= 1 && c.hidden_size % c.heads == 0, "hidden / heads");
  need(c.hidden_size / c.heads <= kAttnMaxD, "head width above 128");
  need(c.position_groups >= 1 && c.hidden_size % c.position_groups == 0, "positional groups");
  need(c.num_convs >= 1 && c.num_convs <= 8 && c.num_downsampling >= 1 && c.num_downsampling <= 8,
       "stage counts");
  need(c.encoder_channels >= 1 && c.latent_channels >= 1, "acoustic widths");
  size_t sem_frame = 1;
  for (size_t i = 0; i < c.num_convs; ++i) sem_frame *= c.conv_strides[i];
  need(c.semantic_sample_rate % sem_frame == 0, "semantic frame");
  const size_t frame = FrameSamples();
  need(c.sample_rate % frame == 0, "codec frame");
  const size_t sem_rate = c.semantic_sample_rate / sem_frame, rate = c.sample_rate / frame;
  need(sem_rate % rate == 0, "semantic frame rate not a multiple of the codec's");  // config.cpp:260-266
  const size_t joint = Joint();
  need(joint <= 8192 && c.codebook_dim <= 1024, "quantizer widths");
}

DeviceBuffer<float> EncoderEngine::Upload(const float* data, size_t n) {
  DeviceBuffer<float> b(n);
  Check(cudaMemcpyAsync(b.get(), data, n * sizeof(float), cudaMemcpyHostToDevice, stream_),
        "upload encoder weights");
  Check(cudaStreamSynchronize(stream_), "upload encoder weights");
  return b;
}

DeviceBuffer<float> EncoderEngine::Vec(const TensorSource& src, const std::string& name,
                                       const std::vector<uint64_t>& shape) {
  size_t n = 1;
  for (uint64_t d : shape) n *= d;
  return Upload(src(name, shape), n);
}

// [cout][cin / groups][kernel] -> [groups][kernel][cout / groups][cin / groups].
Conv EncoderEngine::MakeConv(const TensorSource& src, const std::string& prefix, int cin,
                             int cout, int kernel, int stride, int dilation, int pad, int groups,
                             bool bias) {
  Conv c;
  c.cin_g = cin / groups;
  c.cout_g = cout / groups;
  c.groups = groups;
  c.taps = kernel;
  c.stride = stride;
  c.dilation = dilation;
  c.pad = pad;
  const float* w = src(prefix + ".weight", {static_cast<uint64_t>(cout), static_cast<uint64_t>(c.cin_g),
                                            static_cast<uint64_t>(kernel)});
  std::vector<float> r(static_cast<size_t>(cout) * c.cin_g * kernel);
  for (int o = 0; o < cout; ++o) {
    const int g = o / c.cout_g, n = o % c.cout_g;
    for (int i = 0; i < c.cin_g; ++i)
      for (int k = 0; k < kernel; ++k)
        r[((static_cast<size_t>(g) * kernel + k) * c.cout_g + n) * c.cin_g + i] =
            w[(static_cast<size_t>(o) * c.cin_g + i) * kernel + k];
  }
  c.w = Upload(r.data(), r.size());
  if (bias) c.bias = Vec(src, prefix + ".bias", {static_cast<uint64_t>(cout)});
  return c;
}

Conv EncoderEngine::MakeDense(const TensorSource& src, const std::string& prefix, int in, int out) {
  Conv c;
  c.cin_g = in;
  c.cout_g = out;
  c.w = Vec(src, prefix + ".weight", {static_cast<uint64_t>(out), static_cast<uint64_t>(in)});
  c.bias = Vec(src, prefix + ".bias", {static_cast<uint64_t>(out)});
  return c;
}

void EncoderEngine::Load(const TensorSource& src) {
  Check(cudaSetDevice(device_), "cudaSetDevice");
  const ov_codec_encoder_config& c = cfg_;
  const int H = static_cast<int>(c.hidden_size);
  const auto u = [](size_t v) { return static_cast<uint64_t>(v); };
  // HuBERT (codec_encoder.cpp:77-171).
  int in = 1;
  for (size_t i = 0; i < c.num_convs; ++i) {
    const int ch = static_cast<int>(c.conv_channels[i]);
    features_.push_back(MakeConv(src, "semantic_model.feature_extractor.conv_layers." +
                                          std::to_string(i) + ".conv",
                                 in, ch, static_cast<int>(c.conv_kernels[i]),
                                 static_cast<int>(c.conv_strides[i]), 1, 0, 1, false));
    in = ch;
  }
  const std::string fe = "semantic_model.feature_extractor.conv_layers.0.layer_norm.";
  gn_w_ = Vec(src, fe + "weight", {u(c.conv_channels[0])});
  gn_b_ = Vec(src, fe + "bias", {u(c.conv_channels[0])});
  proj_nw_ = Vec(src, "semantic_model.feature_projection.layer_norm.weight", {u(in)});
  proj_nb_ = Vec(src, "semantic_model.feature_projection.layer_norm.bias", {u(in)});
  projection_ = MakeDense(src, "semantic_model.feature_projection.projection", in, H);
  {
    // Weight norm folded (dim = 2: one gain per tap over the taps' norms),
    // codec_encoder.cpp:103-137.
    const int K = static_cast<int>(c.position_kernel), G = static_cast<int>(c.position_groups);
    const int gw = H / G;
    const std::string p = "semantic_model.encoder.pos_conv_embed.conv.";
    const float* g0 = src(p + "parametrizations.weight.original0", {1, 1, u(K)});
    const std::vector<float> gain(g0, g0 + K);
    const float* v = src(p + "parametrizations.weight.original1", {u(H), u(gw), u(K)});
    std::vector<double> norms(K, 0.0);
    for (size_t i = 0; i < static_cast<size_t>(H) * gw; ++i)
      for (int k = 0; k < K; ++k) norms[k] += static_cast<double>(v[i * K + k]) * v[i * K + k];
    std::vector<float> folded(static_cast<size_t>(H) * gw * K);
    for (size_t i = 0; i < static_cast<size_t>(H) * gw; ++i)
      for (int k = 0; k < K; ++k)
        folded[i * K + k] = static_cast<float>(gain[k] * v[i * K + k] / std::sqrt(norms[k]));
    position_ = MakeConv(
        [&](const std::string& name, const std::vector<uint64_t>& shape) -> const float* {
          if (name == "pos.weight") return folded.data();
          return src(p + "bias", shape);
        },
        "pos", H, H, K, 1, 1, K / 2, G, false);
    position_.bias = Vec(src, p + "bias", {u(H)});
  }
  enc_nw_ = Vec(src, "semantic_model.encoder.layer_norm.weight", {u(H)});
  enc_nb_ = Vec(src, "semantic_model.encoder.layer_norm.bias", {u(H)});
  const int I = static_cast<int>(c.intermediate_size);
  for (size_t l = 0; l < c.layers; ++l) {
    const std::string p = "semantic_model.encoder.layers." + std::to_string(l) + ".";
    HubertLayer L;
    // q, k, v stacked into one projection (codec_encoder.cpp:35-52).
    std::vector<float> w(static_cast<size_t>(3) * H * H), b(3 * static_cast<size_t>(H));
    const char* names[3] = {"q_proj", "k_proj", "v_proj"};
    for (int j = 0; j < 3; ++j) {
      const float* wd = src(p + "attention." + names[j] + ".weight", {u(H), u(H)});
      std::copy(wd, wd + static_cast<size_t>(H) * H, w.begin() + static_cast<size_t>(j) * H * H);
      const float* bd = src(p + "attention." + names[j] + ".bias", {u(H)});
      std::copy(bd, bd + H, b.begin() + static_cast<size_t>(j) * H);
    }
    L.qkv.cin_g = H;
    L.qkv.cout_g = 3 * H;
    L.qkv.w = Upload(w.data(), w.size());
    L.qkv.bias = Upload(b.data(), b.size());
    L.out = MakeDense(src, p + "attention.out_proj", H, H);
    L.n1w = Vec(src, p + "layer_norm.weight", {u(H)});
    L.n1b = Vec(src, p + "layer_norm.bias", {u(H)});
    L.inter = MakeDense(src, p + "feed_forward.intermediate_dense", H, I);
    L.final_ = MakeDense(src, p + "feed_forward.output_dense", I, H);
    L.n2w = Vec(src, p + "final_layer_norm.weight", {u(H)});
    L.n2b = Vec(src, p + "final_layer_norm.bias", {u(H)});
    layers_.push_back(std::move(L));
  }
  // Semantic encoder (codec_encoder.cpp:172-194).
  sem_in_ = MakeConv(src, "encoder_semantic.conv", H, H, 3, 1, 1, 1, 1, false);
  for (int blk = 0; blk < 2; ++blk) {
    const std::string p = "encoder_semantic.conv_blocks." + std::to_string(blk);
    for (int un = 0; un < 2; ++un) {
      const std::string q = p + ".res_units." + std::to_string(un);
      sem_unit_[blk][un][0] = MakeConv(src, q + ".conv1", H, H, 3, 1, 1, 1, 1, false);
      sem_unit_[blk][un][1] = MakeConv(src, q + ".conv2", H, H, 1, 1, 1, 0, 1, false);
    }
    sem_conv_[blk] = MakeConv(src, p + ".conv", H, H, 3, 1, 1, 1, 1, true);
  }
  // DAC encoder (codec_encoder.cpp:195-226).
  int ch = static_cast<int>(c.encoder_channels);
  dac_in_ = MakeConv(src, "acoustic_encoder.conv1", 1, ch, kResidualKernel, 1, 1, 3, 1, true);
  for (size_t i = 0; i < c.num_downsampling; ++i) {
    const std::string p = "acoustic_encoder.block." + std::to_string(i) + ".";
    const int s = static_cast<int>(c.downsampling_ratios[i]);
    DacBlock B;
    for (int un = 0; un < 3; ++un) {
      const std::string q = p + "res_unit" + std::to_string(un + 1) + ".";
      B.units[un].alpha1 = Vec(src, q + "snake1.alpha", {1, u(ch), 1});
      B.units[un].alpha2 = Vec(src, q + "snake2.alpha", {1, u(ch), 1});
      const int d = kDilations[un];
      B.units[un].conv1 = MakeConv(src, q + "conv1", ch, ch, kResidualKernel, 1, d,
                                   (kResidualKernel - 1) * d / 2, 1, true);
      B.units[un].conv2 = MakeConv(src, q + "conv2", ch, ch, 1, 1, 1, 0, 1, true);
    }
    B.alpha = Vec(src, p + "snake1.alpha", {1, u(ch), 1});
    B.down = MakeConv(src, p + "conv1", ch, 2 * ch, 2 * s, s, 1, (s + 1) / 2, 1, true);
    blocks_.push_back(std::move(B));
    ch *= 2;
  }
  dac_alpha_ = Vec(src, "acoustic_encoder.snake1.alpha", {1, u(ch), 1});
  dac_out_ = MakeConv(src, "acoustic_encoder.conv2", ch, static_cast<int>(c.latent_channels), 3, 1,
                      1, 1, 1, true);
  // fc and the quantizer (codec_encoder.cpp:227-246; decoded entries as
  // codec.cpp:136-160).
  const int J = static_cast<int>(Joint());
  fc_ = MakeDense(src, "fc", J, J);
  const int C = static_cast<int>(c.codebooks), E = static_cast<int>(c.codebook_size),
            D = static_cast<int>(c.codebook_dim);
  std::vector<float> pw(static_cast<size_t>(C) * D * J), pb(static_cast<size_t>(C) * D),
      cb(static_cast<size_t>(C) * E * D), nrm(static_cast<size_t>(C) * E);
  tables_ = DeviceBuffer<float>(static_cast<size_t>(C) * E * J);
  for (int q = 0; q < C; ++q) {
    const std::string p = "quantizer.quantizers." + std::to_string(q) + ".";
    const float* w = src(p + "project_in.weight", {u(D), u(J)});
    std::copy(w, w + static_cast<size_t>(D) * J, pw.begin() + static_cast<size_t>(q) * D * J);
    const float* b = src(p + "project_in.bias", {u(D)});
    std::copy(b, b + D, pb.begin() + static_cast<size_t>(q) * D);
    const float* e0 = src(p + "codebook.embed", {u(E), u(D)});
    std::copy(e0, e0 + static_cast<size_t>(E) * D, cb.begin() + static_cast<size_t>(q) * E * D);
    const float* e = cb.data() + static_cast<size_t>(q) * E * D;
    for (int k = 0; k < E; ++k) {  // encoder_kernels.hip SquaredNormsKernel
      float s = 0.0f;
      for (int d = 0; d < D; ++d) s += e[static_cast<size_t>(k) * D + d] * e[static_cast<size_t>(k) * D + d];
      nrm[static_cast<size_t>(q) * E + k] = s;
    }
    // Decoded entries: project_out(embed) + bias, as a dense layer on the GPU.
    Conv out = MakeDense(src, p + "project_out", D, J);
    DeviceBuffer<float> emb = Upload(e, static_cast<size_t>(E) * D);
    Run(out, emb.get(), D, E, tables_.get() + static_cast<size_t>(q) * E * J, J);
    Check(cudaStreamSynchronize(stream_), "decoded entries");
  }
  proj_in_w_ = Upload(pw.data(), pw.size());
  proj_in_b_ = Upload(pb.data(), pb.size());
  codebooks_ = Upload(cb.data(), cb.size());
  norms_ = Upload(nrm.data(), nrm.size());
}

int EncoderEngine::Run(const Conv& c, const float* x, int64_t ldx, int rows_in, float* y,
                       int64_t ldy, int pre, const float* alpha, int act, const float* resid,
                       int64_t ldr, int rows_out) {
  ConvArgs a{};
  a.x = x;
  a.ldx = ldx;
  a.rows_in = rows_in;
  a.w = c.w.get();
  a.bias = c.bias.size() > 0 ? c.bias.get() : nullptr;
  a.alpha = alpha;
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  a.rows_out = rows_out >= 0 ? rows_out : c.RowsOut(rows_in);
  a.cin_g = c.cin_g;
  a.cout_g = c.cout_g;
  a.groups = c.groups;
  a.taps = c.taps;
  a.stride = c.stride;
  a.dilation = c.dilation;
  a.pad = c.pad;
  a.pre = pre;
  a.act = act;
  if (a.rows_out <= 0) throw Error(OV_ERR_INVALID, "reference audio too short for a convolution");
  // Split-K when the output tiles alone leave SMs idle: about two CTAs per
  // SM, each split at least 8 steps deep.
  const int tiles = ((a.rows_out + kTileM - 1) / kTileM) * ((a.cout_g + kTileN - 1) / kTileN) * c.groups;
  const int steps = c.taps * ((c.cin_g + kTileK - 1) / kTileK);
  int splits = std::min({(2 * sms_ + tiles - 1) / tiles, steps / 8, 16});
  splits = std::max(splits, 1);
  a.per_split = (steps + splits - 1) / splits;
  a.splits = (steps + a.per_split - 1) / a.per_split;
  a.partial = nullptr;
  if (a.splits > 1) {
    const size_t n = static_cast<size_t>(a.splits) * a.rows_out * c.groups * c.cout_g;
    (void)partial_.Reserve(n);
    a.partial = partial_.get();
  }
  const dim3 grid((a.rows_out + kTileM - 1) / kTileM, (a.cout_g + kTileN - 1) / kTileN,
                  c.groups * a.splits);
  Launch(conv_kernel, grid, dim3(256), 0, stream_, "encoder conv launch", a);
  if (a.splits > 1) {
    const int64_t n = static_cast<int64_t>(a.rows_out) * c.groups * c.cout_g;
    Launch(reduce_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream_,
           "encoder split-K reduce launch", a);
  }
  return a.rows_out;
}

void EncoderEngine::LayerNorm(const float* x, float* y, int rows, int width,
                              const DeviceBuffer<float>& w, const DeviceBuffer<float>& b,
                              float eps) {
  Launch(layernorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream_, "layer norm launch", x, y,
         rows, width, static_cast<const float*>(w.get()), static_cast<const float*>(b.get()), eps);
}

// The reference's Resample (audio.cpp:265-321): torchaudio's windowed-sinc
// resampler, kernel in float32 operation by operation, sums in float64.
std::vector<float> Resample(const float* x, size_t n, uint32_t from_rate, uint32_t to_rate) {
  if (from_rate == to_rate || n == 0) return std::vector<float>(x, x + n);
  constexpr int kZero = 6;
  constexpr double kRolloff = 0.99;
  const uint32_t g = std::gcd(from_rate, to_rate);
  const int64_t from = from_rate / g, to = to_rate / g;
  const double base = static_cast<double>(std::min(from, to)) * kRolloff;
  const auto width = static_cast<int64_t>(std::ceil(kZero * static_cast<double>(from) / base));
  const int64_t taps = 2 * width + from;
  std::vector<float> kernel(static_cast<size_t>(to * taps));
  const auto base_f = static_cast<float>(base);
  const auto pi_f = static_cast<float>(3.14159265358979323846);
  const auto scale_f = static_cast<float>(base / static_cast<double>(from));
  for (int64_t phase = 0; phase < to; ++phase)
    for (int64_t tap = 0; tap < taps; ++tap) {
      const float index = static_cast<float>(tap - width) / static_cast<float>(from);
      float t = static_cast<float>(-phase) / static_cast<float>(to) + index;
      t *= base_f;
      t = std::clamp(t, -static_cast<float>(kZero), static_cast<float>(kZero));
      const float cosine = std::cos(t * pi_f / static_cast<float>(kZero) / 2.0f);
      const float window = cosine * cosine;
      t *= pi_f;
      const float sinc = t == 0.0f ? 1.0f : std::sin(t) / t;
      kernel[static_cast<size_t>(phase * taps + tap)] = sinc * (window * scale_f);
    }
  const auto length = static_cast<int64_t>(n);
  const auto out_len = static_cast<int64_t>(
      std::ceil(static_cast<double>(to) * static_cast<double>(length) / static_cast<double>(from)));
  std::vector<float> out(static_cast<size_t>(out_len));
  for (int64_t o = 0; o < out_len; ++o) {
    const int64_t block = o / to, phase = o % to;
    const float* w = &kernel[static_cast<size_t>(phase * taps)];
    const int64_t origin = block * from - width;
    double sum = 0.0;
    const int64_t first = std::max<int64_t>(0, -origin);
    const int64_t last = std::min<int64_t>(taps, length - origin);
    for (int64_t tap = first; tap < last; ++tap)
      sum += static_cast<double>(w[tap]) * x[static_cast<size_t>(origin + tap)];
    out[static_cast<size_t>(o)] = static_cast<float>(sum);
  }
  return out;
}

size_t EncoderEngine::Encode(const float* samples, size_t count, int32_t* codes, size_t capacity) {
  Check(cudaSetDevice(device_), "cudaSetDevice");
  const ov_codec_encoder_config& c = cfg_;
  const size_t frame = FrameSamples();
  if (count == 0 || count % frame != 0)
    throw Error(OV_ERR_INVALID, "reference audio must be a whole number of frames");
  const int frames = static_cast<int>(count / frame);
  if (codes != nullptr && capacity < c.codebooks * static_cast<size_t>(frames))
    throw Error(OV_ERR_INVALID, "code buffer too small");
  const int H = static_cast<int>(c.hidden_size), J = static_cast<int>(Joint());
  cudaStream_t s = stream_;
  // ---- HuBERT input: resampled to 16 kHz with 160 zero samples each side.
  std::vector<float> r16 = Resample(samples, count, c.sample_rate, c.semantic_sample_rate);
  r16.insert(r16.begin(), kHubertPad, 0.0f);
  r16.insert(r16.end(), kHubertPad, 0.0f);
  // Buffer sizes: the largest feature map, the DAC's signals, HuBERT's rows.
  int len = static_cast<int>(r16.size());
  size_t feat = static_cast<size_t>(len);
  for (const Conv& f : features_) {
    len = f.RowsOut(len);
    if (len <= 0) throw Error(OV_ERR_INVALID, "reference audio too short for the feature extractor");
    feat = std::max(feat, static_cast<size_t>(len) * f.cout_g);
  }
  const int steps = len;
  const size_t rows_max = std::max<size_t>(static_cast<size_t>(steps) *
                                               std::max<size_t>(3 * H, c.intermediate_size),
                                           static_cast<size_t>(count) * c.encoder_channels);
  const size_t need = std::max(feat, rows_max);
  for (int i = 0; i < 6; ++i) (void)buf_[i].Reserve(need);
  float* A = buf_[0].get();
  float* B = buf_[1].get();
  Check(cudaMemcpyAsync(A, r16.data(), r16.size() * sizeof(float), cudaMemcpyHostToDevice, s),
        "upload audio");
  // Feature extractor (codec_encoder.cpp:270-289).
  len = static_cast<int>(r16.size());
  int width = 1;
  for (size_t i = 0; i < features_.size(); ++i) {
    const Conv& f = features_[i];
    len = Run(f, A, width, len, B, f.cout_g, kPreNone, nullptr, i == 0 ? kActNone : kActGelu);
    width = f.cout_g;
    if (i == 0)
      Launch(groupnorm_gelu_kernel, dim3((width + 31) / 32), dim3(256), 0, s, "group norm launch", B,
             len, width, static_cast<const float*>(gn_w_.get()),
             static_cast<const float*>(gn_b_.get()), kGroupNormEps);
    std::swap(A, B);
  }
  // Layer norm, projection, positional convolution + GELU added, encoder
  // layer norm (codec_encoder.cpp:290-309).
  const float eps = c.layer_norm_eps;
  LayerNorm(A, A, steps, width, proj_nw_, proj_nb_, eps);
  float* h = buf_[2].get();
  float* h2 = buf_[3].get();
  Run(projection_, A, width, steps, h, H);
  Run(position_, h, H, steps, h2, H, kPreNone, nullptr, kActGelu, h, H, steps);
  LayerNorm(h2, h2, steps, H, enc_nw_, enc_nb_, eps);
  std::swap(h, h2);
  float* total = buf_[4].get();
  Check(cudaMemcpyAsync(total, h, static_cast<size_t>(steps) * H * sizeof(float),
                        cudaMemcpyDeviceToDevice, s),
        "copy hidden states");
  // Layers (codec_encoder.cpp:310-368).
  float* qkv = buf_[0].get();
  float* att = buf_[1].get();
  float* mid = buf_[5].get();
  const int d = H / static_cast<int>(c.heads);
  const int64_t n_h = static_cast<int64_t>(steps) * H;
  for (const HubertLayer& L : layers_) {
    Run(L.qkv, h, H, steps, qkv, 3 * H);
    Launch(attention_kernel, dim3((steps + 7) / 8, static_cast<unsigned>(c.heads)), dim3(256), 0, s,
           "encoder attention launch", static_cast<const float*>(qkv), steps, H, d,
           1.0f / std::sqrt(static_cast<float>(d)), att);
    Run(L.out, att, H, steps, h, H, kPreNone, nullptr, kActNone, h, H);
    LayerNorm(h, h, steps, H, L.n1w, L.n1b, eps);
    Run(L.inter, h, H, steps, mid, static_cast<int64_t>(c.intermediate_size), kPreNone, nullptr,
        kActGelu);
    Run(L.final_, mid, static_cast<int64_t>(c.intermediate_size), steps, h, H, kPreNone, nullptr,
        kActNone, h, H);
    LayerNorm(h, h, steps, H, L.n2w, L.n2b, eps);
    Launch(add_kernel, dim3(static_cast<unsigned>((n_h + 255) / 256)), dim3(256), 0, s,
           "accumulate launch", total, static_cast<const float*>(h), n_h);
  }
  // Every semantic_stride-th averaged frame (codec_encoder.cpp:357-378).
  size_t sem_frame = 1;
  for (size_t i = 0; i < c.num_convs; ++i) sem_frame *= c.conv_strides[i];
  const int stride = static_cast<int>((c.semantic_sample_rate / sem_frame) / (c.sample_rate / frame));
  if (steps < frames * stride)
    throw Error(OV_ERR_INVALID, "reference audio is too short for the semantic encoder");
  float* x = buf_[0].get();
  float* y = buf_[1].get();
  float* z = buf_[2].get();
  const int64_t n_sem = static_cast<int64_t>(frames) * H;
  Launch(pick_scale_kernel, dim3(static_cast<unsigned>((n_sem + 255) / 256)), dim3(256), 0, s,
         "pick launch", static_cast<const float*>(total), H, stride, frames,
         1.0f / static_cast<float>(layers_.size() + 1), x);
  // Semantic encoder (codec_encoder.cpp:379-398) into joint[:, latent ..].
  float* joint = buf_[3].get();
  const int latent = static_cast<int>(c.latent_channels);
  Run(sem_in_, x, H, frames, y, H);                      // y = b
  for (int blk = 0; blk < 2; ++blk) {
    for (int un = 0; un < 2; ++un) {
      Run(sem_unit_[blk][un][0], y, H, frames, z, H, kPreElu);             // c = conv1(elu(b))
      Run(sem_unit_[blk][un][1], z, H, frames, y, H, kPreElu, nullptr, kActNone, y, H);  // b += conv2(elu(c))
    }
    if (blk == 0) {
      Run(sem_conv_[blk], y, H, frames, x, H);
      std::swap(x, y);
    } else {
      Run(sem_conv_[blk], y, H, frames, joint + latent, J);
    }
  }
  // DAC encoder into joint[:, 0 .. latent) (codec_encoder.cpp:399-424).
  float* sig = buf_[4].get();  // HuBERT's total is consumed
  float* sig2 = buf_[0].get();
  float* tmp = buf_[1].get();
  Check(cudaMemcpyAsync(tmp, samples, count * sizeof(float), cudaMemcpyHostToDevice, s), "upload audio");
  int T = Run(dac_in_, tmp, 1, static_cast<int>(count), sig, dac_in_.cout_g);
  int ch = dac_in_.cout_g;
  float* ybuf = buf_[2].get();
  for (const DacBlock& blk : blocks_) {
    for (const ResUnit& un : blk.units) {
      Run(un.conv1, sig, ch, T, ybuf, ch, kPreSnake, un.alpha1.get());
      Run(un.conv2, ybuf, ch, T, sig, ch, kPreSnake, un.alpha2.get(), kActNone, sig, ch);
    }
    T = Run(blk.down, sig, ch, T, sig2, 2 * ch, kPreSnake, blk.alpha.get());
    ch *= 2;
    std::swap(sig, sig2);
  }
  if (T != frames) throw Error(OV_ERR_INVALID, "acoustic and semantic frame counts differ");
  Run(dac_out_, sig, ch, T, joint, J, kPreSnake, dac_alpha_.get());
  // fc and the quantizer (codec_encoder.cpp:425-458).
  float* residual = buf_[5].get();
  Run(fc_, joint, J, frames, residual, J);
  (void)codes_.Reserve(c.codebooks * static_cast<size_t>(frames));
  const int E = static_cast<int>(c.codebook_size), D = static_cast<int>(c.codebook_dim);
  // At most (8192 + 1024 + 256) floats + 256 ints (CheckConfig): under 48 KB.
  const size_t smem = (static_cast<size_t>(J) + D + 256) * sizeof(float) + 256 * sizeof(int);
  Launch(rvq_kernel, dim3(frames), dim3(256), smem, s, "quantizer launch", residual, frames, J,
         static_cast<int>(c.codebooks), E, D, static_cast<const float*>(proj_in_w_.get()),
         static_cast<const float*>(proj_in_b_.get()), static_cast<const float*>(codebooks_.get()),
         static_cast<const float*>(norms_.get()), static_cast<const float*>(tables_.get()),
         codes_.get());
  if (codes != nullptr)
    Check(cudaMemcpyAsync(codes, codes_.get(), c.codebooks * static_cast<size_t>(frames) * sizeof(int32_t),
                          cudaMemcpyDeviceToHost, s),
          "download codes");
  Check(cudaStreamSynchronize(s), "encode");
  return static_cast<size_t>(frames);
}

}  // namespace encoder
}  // namespace ovb

struct ov_codec_encoder {
  std::unique_ptr<ovb::encoder::EncoderEngine> engine;
  std::vector<float> scratch;  // synthetic tensors
};

using ovb::Guard;

extern "C" {

void ov_codec_encoder_default_config(ov_codec_encoder_config* c) {
  std::memset(c, 0, sizeof(*c));
  c->sample_rate = 24000;
  c->codebooks = 8;
  c->codebook_size = 1024;
  c->codebook_dim = 64;
  c->semantic_sample_rate = 16000;
  c->hidden_size = 768;
  c->intermediate_size = 3072;
  c->heads = 12;
  c->layers = 12;
  c->position_kernel = 128;
  c->position_groups = 16;
  c->layer_norm_eps = 1e-5f;
  const size_t kernels[7] = {10, 3, 3, 3, 3, 2, 2}, strides[7] = {5, 2, 2, 2, 2, 2, 2};
  c->num_convs = 7;
  for (int i = 0; i < 7; ++i) {
    c->conv_channels[i] = 512;
    c->conv_kernels[i] = kernels[i];
    c->conv_strides[i] = strides[i];
  }
  c->encoder_channels = 64;
  c->latent_channels = 256;
  const size_t ratios[5] = {8, 5, 4, 2, 3};
  c->num_downsampling = 5;
  for (int i = 0; i < 5; ++i) c->downsampling_ratios[i] = ratios[i];
}

int ov_codec_encoder_load(const ov_codec_encoder_config* config, const char* path, int device,
                          ov_codec_encoder** encoder) {
  *encoder = nullptr;
  return Guard("OmniVoice audio tokenizer: ", [&] {
    OV_REQUIRE(config != nullptr && path != nullptr, "config / path missing");
    auto e = std::make_unique<ov_codec_encoder>();
    e->engine = std::make_unique<ovb::encoder::EncoderEngine>(*config, device);
    ovb::SafetensorsFile file(path);
    e->engine->Load([&](const std::string& name, const std::vector<uint64_t>& shape) {
      return file.ExpectF32(name, shape);
    });
    *encoder = e.release();
  });
}

int ov_codec_encoder_create_synthetic(const ov_codec_encoder_config* config, uint64_t seed,
                                      int device, ov_codec_encoder** encoder) {
  *encoder = nullptr;
  return Guard("OmniVoice audio tokenizer: ", [&] {
    OV_REQUIRE(config != nullptr, "config missing");
    auto e = std::make_unique<ov_codec_encoder>();
    e->engine = std::make_unique<ovb::encoder::EncoderEngine>(*config, device);
    uint64_t tensor = 0;
    std::vector<float>& buf = e->scratch;
    // The scales of the test weights: N(0, 1 / fan_in) projections and
    // convolutions, norm weights near 1, small biases, snake alphas in
    // [0.5, 2), N(0, 1) codebooks and positional directions.
    e->engine->Load([&](const std::string& name, const std::vector<uint64_t>& shape) {
      size_t n = 1;
      for (uint64_t d : shape) n *= d;
      buf.assign(n, 0.0f);
      const uint64_t base = ovb::SyntheticBase(seed, ++tensor);
      const auto ends = [&](const char* suffix) {
        const size_t l = std::strlen(suffix);
        return name.size() >= l && name.compare(name.size() - l, l, suffix) == 0;
      };
      if (ends("alpha") || ends("original0")) {
        for (size_t i = 0; i < n; ++i)
          buf[i] = 0.5f + 1.5f * static_cast<float>(ovb::Mix64(base + i) >> 40) * 0x1p-24f;
        return buf.data();
      }
      float std = 1.0f, mean = 0.0f;
      if (name.find("norm") != std::string::npos && ends("weight")) {
        std = 0.1f;
        mean = 1.0f;
      } else if (ends("bias")) {
        std = 0.05f;
      } else if (!ends("codebook.embed") && !ends("original1")) {
        std = static_cast<float>(1.0 / std::sqrt(static_cast<double>(n / shape[0])));
      }
      const float scale = ovb::SyntheticScale(std);
      for (size_t i = 0; i < n; ++i) buf[i] = mean + ovb::SyntheticValue(base, i, scale);
      return buf.data();
    });
    e->scratch.clear();
    e->scratch.shrink_to_fit();
    *encoder = e.release();
  });
}

void ov_codec_encoder_free(ov_codec_encoder* encoder) { delete encoder; }

size_t ov_codec_encoder_frame_samples(const ov_codec_encoder* encoder) {
  return encoder != nullptr ? encoder->engine->FrameSamples() : 0;
}

int ov_codec_encode(ov_codec_encoder* encoder, const float* samples, size_t count, int32_t* codes,
                    size_t capacity, size_t* frames) {
  if (frames != nullptr) *frames = 0;
  return Guard("OmniVoice encode: ", [&] {
    OV_REQUIRE(encoder != nullptr && samples != nullptr && codes != nullptr && frames != nullptr,
               "encoder / samples / codes / frames missing");
    *frames = encoder->engine->Encode(samples, count, codes, capacity);
  });
}

}  // extern "C"
