// The audio tokenizer's decoder on one GPU: weight loading (reference
// codec.cpp:26-106,114-193 for the decoder tensors), the per-frame-count
// plan of convolutions, and decode (codec.cpp:195-262), behind the C-ABI of
// ov_codec.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "codec_kernels.hpp"
#include "internal.hpp"
#include "launch.hpp"
#include "ov_codec.h"
#include "safetensors.hpp"
#include "synthetic.hpp"

namespace ovb {
namespace codec {
namespace {

constexpr int kResidualKernel = 7;            // codec_state.hpp:26
constexpr int kDilations[3] = {1, 3, 9};      // codec_state.hpp:27

// Host tensor source: (name, shape) -> float32 data valid until the next call.
using TensorSource = std::function<const float*(const std::string&, const std::vector<uint64_t>&)>;

DeviceBuffer<float> Upload(const float* data, size_t count, cudaStream_t s) {
  DeviceBuffer<float> b(count);
  Check(cudaMemcpyAsync(b.get(), data, count * sizeof(float), cudaMemcpyHostToDevice, s),
        "upload codec weights");
  Check(cudaStreamSynchronize(s), "upload codec weights");
  return b;
}

// Host [taps][cout][cin] weights -> device hi / lo planes.
ConvWeights MakeConv(const std::vector<float>& w, const float* bias, int cin, int cout, int taps,
                     cudaStream_t s) {
  ConvWeights c;
  c.cin = cin;
  c.cout = cout;
  c.taps = taps;
  DeviceBuffer<float> raw = Upload(w.data(), w.size(), s);
  c.hi = DeviceBuffer<float>(w.size());
  c.lo = DeviceBuffer<float>(w.size());
  LaunchSplit(raw.get(), c.hi.get(), c.lo.get(), static_cast<int64_t>(w.size()), s);
  c.bias = Upload(bias, static_cast<size_t>(cout), s);
  Check(cudaStreamSynchronize(s), "split codec weights");
  return c;
}

}  // namespace

struct Unit {
  DeviceBuffer<float> alpha1, alpha2;
  ConvWeights conv1, conv2;
};

struct Block {
  int stride = 0;
  DeviceBuffer<float> alpha;
  ConvWeights up;
  Unit units[3];
};

class CodecEngine {
 public:
  CodecEngine(const ov_codec_config& cfg, int device) : cfg_(cfg), device_(device) {
    Activate();
    Check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    (void)DeviceErrorWord();
    CheckConfig();
  }
  ~CodecEngine() {
    if (stream_ != nullptr) {
      (void)cudaSetDevice(device_);
      (void)cudaStreamDestroy(stream_);
    }
  }
  CodecEngine(const CodecEngine&) = delete;
  CodecEngine& operator=(const CodecEngine&) = delete;

  size_t FrameSamples() const {
    size_t p = 1;
    for (size_t i = 0; i < cfg_.num_upsampling; ++i) p *= cfg_.upsampling_ratios[i];
    return p;
  }

  cudaStream_t Stream() const { return stream_; }
  void Load(const TensorSource& src);
  void Decode(const int32_t* codes, size_t frames, float* audio, cudaStream_t s);
  void DecodeHost(const int32_t* codes, size_t frames, float* audio);

 private:
  void Activate() const { Check(cudaSetDevice(device_), "cudaSetDevice"); }
  void CheckConfig() const;
  void Plan(size_t frames);
  size_t Hidden() const { return cfg_.semantic_hidden + cfg_.latent_channels; }

  ov_codec_config cfg_;
  int device_;
  cudaStream_t stream_ = nullptr;
  // Weights.
  DeviceBuffer<float> table_;     // [codebooks][entries][latent]: fc2(project_out(codebook))
  DeviceBuffer<float> lat_bias_;  // [latent]: fc2 bias
  ConvWeights input_;
  std::vector<Block> blocks_;
  DeviceBuffer<float> final_alpha_;
  DeviceBuffer<float> out_w_, out_b_;  // [7][channels], [1]
  // Work buffers and the plan of the last frame count.
  DeviceBuffer<int32_t> codes_;
  DeviceBuffer<float> lat_hi_, lat_lo_, x_, audio_;
  DeviceBuffer<float> plane_hi_[3], plane_lo_[3];
  size_t planned_frames_ = 0;
  std::vector<ConvPlan> plans_;
  const float* final_hi_ = nullptr;
  const float* final_lo_ = nullptr;
  int final_channels_ = 0;
};

// config.cpp:203-222 (ParseAcoustic's checks) plus the widths the kernels take.
void CodecEngine::CheckConfig() const {
  const ov_codec_config& c = cfg_;
  auto need = [](bool ok, const char* what) {
    if (!ok) throw Error(OV_ERR_UNSUPPORTED, std::string("unsupported codec: ") + what);
  };
  need(c.codebooks > 0 && c.codebook_size > 0 && c.codebook_dim > 0, "codebooks");
  need(c.num_upsampling >= 1 && c.num_upsampling <= 8, "upsampling block count");
  need(c.latent_channels % 32 == 0 && c.latent_channels > 0, "latent channels % 32");
  size_t ch = c.decoder_channels;
  need(ch % 32 == 0, "decoder channels % 32");
  for (size_t i = 0; i < c.num_upsampling; ++i) {
    need(c.upsampling_ratios[i] >= 1 && c.upsampling_ratios[i] <= 16, "upsampling ratio");
    need(ch % 2 == 0, "decoder channels can't be halved once per block");
    ch /= 2;
    need(ch % 32 == 0, "every block width must be a multiple of 32");
  }
  need(ch <= 64, "final width must be at most 64");
}

void CodecEngine::Load(const TensorSource& src) {
  Activate();
  cudaStream_t s = stream_;
  using Shape = std::vector<uint64_t>;
  const size_t E = cfg_.codebook_size, D = cfg_.codebook_dim, Hd = Hidden();
  const size_t lat = cfg_.latent_channels;
  auto fetch = [&](const std::string& name, const Shape& shape) {
    size_t n = 1;
    for (uint64_t d : shape) n *= d;
    const float* p = src(name, shape);
    return std::vector<float>(p, p + n);
  };
  // RVQ tables through project_out (codec.cpp:136-160), then fc2 folded in:
  // table[c][e] = W_fc2 (P_c embed_c[e] + b_c); the fc2 bias is added once.
  {
    const std::vector<float> fc2 = fetch("fc2.weight", {lat, Hd});
    DeviceBuffer<float> fc2_d = Upload(fc2.data(), fc2.size(), s);
    lat_bias_ = Upload(fetch("fc2.bias", {lat}).data(), lat, s);
    table_ = DeviceBuffer<float>(cfg_.codebooks * E * lat);
    DeviceBuffer<float> tab(E * Hd);
    for (size_t c = 0; c < cfg_.codebooks; ++c) {
      const std::string p = "quantizer.quantizers." + std::to_string(c) + ".";
      DeviceBuffer<float> embed = Upload(fetch(p + "codebook.embed", {E, D}).data(), E * D, s);
      DeviceBuffer<float> proj = Upload(fetch(p + "project_out.weight", {Hd, D}).data(), Hd * D, s);
      DeviceBuffer<float> bias = Upload(fetch(p + "project_out.bias", {Hd}).data(), Hd, s);
      LaunchDense(embed.get(), proj.get(), bias.get(), tab.get(), static_cast<int>(E),
                  static_cast<int>(Hd), static_cast<int>(D), s);
      LaunchDense(tab.get(), fc2_d.get(), nullptr, table_.get() + c * E * lat, static_cast<int>(E),
                  static_cast<int>(lat), static_cast<int>(Hd), s);
      Check(cudaStreamSynchronize(s), "RVQ table");
    }
  }
  // Conv1d weight [out][in][k] -> [k][out][in] (codec.cpp:46-54).
  auto conv = [&](const std::string& prefix, size_t in, size_t out, size_t k) {
    const std::vector<float> w = fetch(prefix + ".weight", {out, in, k});
    std::vector<float> r(out * in * k);
    for (size_t o = 0; o < out; ++o)
      for (size_t i = 0; i < in; ++i)
        for (size_t t = 0; t < k; ++t) r[(t * out + o) * in + i] = w[(o * in + i) * k + t];
    const std::vector<float> b = fetch(prefix + ".bias", {out});
    return MakeConv(r, b.data(), static_cast<int>(in), static_cast<int>(out), static_cast<int>(k), s);
  };
  auto alpha = [&](const std::string& name, size_t ch) {
    return Upload(fetch(name, {1, ch, 1}).data(), ch, s);
  };
  input_ = conv("acoustic_decoder.conv1", lat, cfg_.decoder_channels, kResidualKernel);
  size_t ch = cfg_.decoder_channels;
  blocks_.clear();
  blocks_.resize(cfg_.num_upsampling);
  for (size_t i = 0; i < cfg_.num_upsampling; ++i) {
    const std::string p = "acoustic_decoder.block." + std::to_string(i) + ".";
    const size_t out = ch / 2, stride = cfg_.upsampling_ratios[i], k = 2 * stride;
    Block& b = blocks_[i];
    b.stride = static_cast<int>(stride);
    b.alpha = alpha(p + "snake1.alpha", ch);
    // ConvTranspose1d weight [in][out][2 s] -> [k][out][in] (codec.cpp:69-86).
    {
      const std::vector<float> w = fetch(p + "conv_t1.weight", {ch, out, k});
      std::vector<float> r(k * out * ch);
      for (size_t in = 0; in < ch; ++in)
        for (size_t o = 0; o < out; ++o)
          for (size_t t = 0; t < k; ++t) r[(t * out + o) * ch + in] = w[(in * out + o) * k + t];
      const std::vector<float> bias = fetch(p + "conv_t1.bias", {out});
      b.up = MakeConv(r, bias.data(), static_cast<int>(ch), static_cast<int>(out),
                      static_cast<int>(k), s);
    }
    for (int u = 0; u < 3; ++u) {
      const std::string q = p + "res_unit" + std::to_string(u + 1) + ".";
      b.units[u].alpha1 = alpha(q + "snake1.alpha", out);
      b.units[u].alpha2 = alpha(q + "snake2.alpha", out);
      b.units[u].conv1 = conv(q + "conv1", out, out, kResidualKernel);
      b.units[u].conv2 = conv(q + "conv2", out, out, 1);
    }
    ch = out;
  }
  final_alpha_ = alpha("acoustic_decoder.snake1.alpha", ch);
  {
    const std::vector<float> w = fetch("acoustic_decoder.conv2.weight", {1, ch, kResidualKernel});
    std::vector<float> r(kResidualKernel * ch);
    for (size_t c = 0; c < ch; ++c)
      for (int t = 0; t < kResidualKernel; ++t) r[t * ch + c] = w[c * kResidualKernel + t];
    out_w_ = Upload(r.data(), r.size(), s);
    out_b_ = Upload(fetch("acoustic_decoder.conv2.bias", {1}).data(), 1, s);
  }
  final_channels_ = static_cast<int>(ch);
  planned_frames_ = 0;
}

// The convolution sequence of Decode (codec.cpp:234-253) for `frames`.
// Plane buffers: the block input's split planes alternate between 0 and 1,
// plane 2 holds a residual unit's inner activation, x_ the residual stream.
void CodecEngine::Plan(size_t frames) {
  if (frames == planned_frames_) return;
  const size_t lat = cfg_.latent_channels;
  size_t rows = frames, ch = cfg_.decoder_channels, biggest = frames * ch;
  for (const Block& b : blocks_) {
    rows *= b.stride;
    ch /= 2;
    biggest = std::max(biggest, rows * ch);
  }
  codes_.Reserve(cfg_.codebooks * frames);
  lat_hi_.Reserve(frames * lat);
  lat_lo_.Reserve(frames * lat);
  x_.Reserve(biggest);
  audio_.Reserve(rows);
  for (int i = 0; i < 3; ++i) {
    plane_hi_[i].Reserve(biggest);
    plane_lo_[i].Reserve(biggest);
  }
  plans_.clear();
  const int F = static_cast<int>(frames);
  int cur = 0;
  auto next_alpha = [&](size_t block, int unit) -> const float* {
    // The snake applied to the output of unit `unit` of block `block`.
    if (unit < 2) return blocks_[block].units[unit + 1].alpha1.get();
    return block + 1 < blocks_.size() ? blocks_[block + 1].alpha.get() : final_alpha_.get();
  };
  {
    ConvPlan p;
    ConvArgs a;
    a.taps = kResidualKernel;
    a.pad = (kResidualKernel - 1) / 2;
    a.alpha = blocks_.empty() ? final_alpha_.get() : blocks_[0].alpha.get();
    a.out_hi = plane_hi_[cur].get();
    a.out_lo = plane_lo_[cur].get();
    PlanConv(&p, lat_hi_.get(), lat_lo_.get(), F, input_, F, 1, a);
    plans_.push_back(p);
  }
  int length = F;
  for (size_t i = 0; i < blocks_.size(); ++i) {
    const Block& b = blocks_[i];
    const int nxt = 1 - cur;
    {
      ConvPlan p;
      ConvArgs a;
      a.taps = 2;
      a.stride = b.stride;
      a.pad = (b.stride + 1) / 2;
      a.out_x = x_.get();
      a.alpha = b.units[0].alpha1.get();
      a.out_hi = plane_hi_[nxt].get();
      a.out_lo = plane_lo_[nxt].get();
      PlanConv(&p, plane_hi_[cur].get(), plane_lo_[cur].get(), length, b.up, length, b.stride, a);
      plans_.push_back(p);
    }
    length *= b.stride;
    for (int u = 0; u < 3; ++u) {
      const int d = kDilations[u];
      ConvPlan p1;
      ConvArgs a1;
      a1.taps = kResidualKernel;
      a1.dilation = d;
      a1.pad = (kResidualKernel - 1) * d / 2;
      a1.alpha = b.units[u].alpha2.get();
      a1.out_hi = plane_hi_[2].get();
      a1.out_lo = plane_lo_[2].get();
      PlanConv(&p1, plane_hi_[nxt].get(), plane_lo_[nxt].get(), length, b.units[u].conv1, length,
               1, a1);
      plans_.push_back(p1);
      ConvPlan p2;
      ConvArgs a2;
      a2.taps = 1;
      a2.resid = x_.get();
      a2.out_x = u < 2 ? x_.get() : nullptr;  // the last unit's sum is only snaked
      a2.alpha = next_alpha(i, u);
      a2.out_hi = plane_hi_[nxt].get();
      a2.out_lo = plane_lo_[nxt].get();
      PlanConv(&p2, plane_hi_[2].get(), plane_lo_[2].get(), length, b.units[u].conv2, length, 1, a2);
      plans_.push_back(p2);
    }
    cur = nxt;
  }
  final_hi_ = plane_hi_[cur].get();
  final_lo_ = plane_lo_[cur].get();
  planned_frames_ = frames;
}

void CodecEngine::Decode(const int32_t* codes, size_t frames, float* audio, cudaStream_t s) {
  Activate();
  if (frames == 0) return;
  OV_REQUIRE(frames <= (size_t{1} << 20), "too many frames");
  Plan(frames);
  const PdlScope pdl(true);
  LaunchCodes(table_.get(), lat_bias_.get(), codes, static_cast<int>(cfg_.codebooks),
              static_cast<int>(cfg_.codebook_size), static_cast<int>(frames),
              static_cast<int>(cfg_.latent_channels), lat_hi_.get(), lat_lo_.get(), s);
  for (const ConvPlan& p : plans_) LaunchConv(p, s);
  LaunchOutputConv(final_hi_, final_lo_, static_cast<int>(frames * FrameSamples()),
                   final_channels_, out_w_.get(), out_b_.get(), audio, s);
}

// codec.cpp:204-214,255-259: host checks, upload, decode, download.
void CodecEngine::DecodeHost(const int32_t* codes, size_t frames, float* audio) {
  Activate();
  const size_t n = cfg_.codebooks * frames;
  for (size_t i = 0; i < n; ++i)
    if (codes[i] < 0 || static_cast<size_t>(codes[i]) >= cfg_.codebook_size)
      throw Error(OV_ERR_INVALID, "code outside the codebook");
  if (frames == 0) return;
  Plan(frames);
  Check(cudaMemcpyAsync(codes_.get(), codes, n * sizeof(int32_t), cudaMemcpyHostToDevice, stream_),
        "upload codes");
  Decode(codes_.get(), frames, audio_.get(), stream_);
  Check(cudaMemcpyAsync(audio, audio_.get(), frames * FrameSamples() * sizeof(float),
                        cudaMemcpyDeviceToHost, stream_),
        "download audio");
  Check(cudaStreamSynchronize(stream_), "decode");
  uint32_t flags = 0;
  CheckStatus(ov_take_device_errors(&flags, stream_));
  if (flags & kErrWaitTimeout) throw Error(OV_ERR_TIMEOUT, "a device-side wait timed out");
  if (flags & kErrBadArgument) throw Error(OV_ERR_INVALID, "a kernel rejected an argument");
}

}  // namespace codec
}  // namespace ovb

struct ov_codec {
  std::unique_ptr<ovb::codec::CodecEngine> engine;
  std::vector<float> scratch;  // synthetic tensors
};

using ovb::Guard;

extern "C" {

void ov_codec_default_config(ov_codec_config* c) {
  std::memset(c, 0, sizeof(*c));
  c->codebooks = 8;
  c->codebook_size = 1024;
  c->codebook_dim = 64;
  c->semantic_hidden = 768;
  c->latent_channels = 256;
  c->decoder_channels = 1024;
  const size_t ratios[5] = {8, 5, 4, 2, 3};
  for (int i = 0; i < 5; ++i) c->upsampling_ratios[i] = ratios[i];
  c->num_upsampling = 5;
  c->sample_rate = 24000;
}

int ov_codec_load(const ov_codec_config* config, const char* path, int device, ov_codec** codec) {
  *codec = nullptr;
  return Guard("OmniVoice audio tokenizer: ", [&] {
    OV_REQUIRE(config != nullptr && path != nullptr, "config / path missing");
    auto c = std::make_unique<ov_codec>();
    c->engine = std::make_unique<ovb::codec::CodecEngine>(*config, device);
    ovb::SafetensorsFile file(path);
    c->engine->Load([&](const std::string& name, const std::vector<uint64_t>& shape) {
      return file.ExpectF32(name, shape);
    });
    *codec = c.release();
  });
}

int ov_codec_create_synthetic(const ov_codec_config* config, uint64_t seed, int device,
                              ov_codec** codec) {
  *codec = nullptr;
  return Guard("OmniVoice audio tokenizer: ", [&] {
    OV_REQUIRE(config != nullptr, "config missing");
    auto c = std::make_unique<ov_codec>();
    c->engine = std::make_unique<ovb::codec::CodecEngine>(*config, device);
    uint64_t tensor = 0;
    std::vector<float>& buf = c->scratch;
    // Same scales as the test weights: N(0, 1 / fan_in) convolutions (x 0.5
    // inside residual units), snake alphas in [0.5, 2), N(0, 1) codebooks.
    c->engine->Load([&](const std::string& name, const std::vector<uint64_t>& shape) {
      size_t n = 1;
      for (uint64_t d : shape) n *= d;
      buf.assign(n, 0.0f);
      const uint64_t base = ovb::SyntheticBase(seed, ++tensor);
      const auto ends = [&](const char* suffix) {
        const size_t l = std::strlen(suffix);
        return name.size() >= l && name.compare(name.size() - l, l, suffix) == 0;
      };
      if (ends("alpha")) {
        for (size_t i = 0; i < n; ++i)
          buf[i] = 0.5f + 1.5f * static_cast<float>(ovb::Mix64(base + i) >> 40) * 0x1p-24f;
        return buf.data();
      }
      float std = 1.0f;
      if (ends("bias")) {
        std = 0.05f;
      } else if (!ends("codebook.embed")) {
        const bool transposed = name.find("conv_t1") != std::string::npos;
        const double fan_in = transposed ? 2.0 * shape[0]
                                         : static_cast<double>(n / shape[0]);
        std = static_cast<float>((name.find("res_unit") != std::string::npos ? 0.5 : 1.0) /
                                 std::sqrt(fan_in));
      }
      const float scale = ovb::SyntheticScale(std);
      for (size_t i = 0; i < n; ++i) buf[i] = ovb::SyntheticValue(base, i, scale);
      return buf.data();
    });
    c->scratch.clear();
    c->scratch.shrink_to_fit();
    *codec = c.release();
  });
}

void ov_codec_free(ov_codec* codec) { delete codec; }

size_t ov_codec_frame_samples(const ov_codec* codec) {
  return codec != nullptr ? codec->engine->FrameSamples() : 0;
}

int ov_codec_decode(ov_codec* codec, const int32_t* codes, size_t frames, float* audio) {
  return Guard("OmniVoice decode: ", [&] {
    OV_REQUIRE(codec != nullptr && (frames == 0 || (codes != nullptr && audio != nullptr)),
               "codec / codes / audio missing");
    codec->engine->DecodeHost(codes, frames, audio);
  });
}

int ov_codec_decode_device(ov_codec* codec, const int32_t* codes, size_t frames, float* audio,
                           ov_stream_t stream) {
  return Guard("OmniVoice decode: ", [&] {
    OV_REQUIRE(codec != nullptr && (frames == 0 || (codes != nullptr && audio != nullptr)),
               "codec / codes / audio missing");
    codec->engine->Decode(codes, frames, audio,
                          stream != nullptr ? ovb::AsStream(stream) : codec->engine->Stream());
  });
}

}  // extern "C"
