// Exercises the C++ drop-in API (generator.hpp, gemm.hpp) on a B200.
//
// usage: dropin_test <model_root> <out_dir> <vocab> <hidden> <intermediate>
//                    <layers> <heads> <kv_heads>
//
// Loads <model_root>/model.safetensors through Generator::Load, writes the
// input it built and the results of Forward, Score, Generate and
// GenerateBatch to <out_dir> (raw little-endian arrays) for the Python test
// to compare with the C-ABI, and checks in place: the error prefixes,
// cancellation, batch == single generation, and HalfGemm::Linear /
// Matmul against a float64 host product.  Prints "ok" and exits 0 when
// every check holds.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <random>
#include <string>
#include <tuple>
#include <vector>

#include "decoding.hpp"
#include "gemm.hpp"
#include "generator.hpp"
#include "ov_runtime.h"

using namespace gufo::models::omnivoice;

namespace {

int failures = 0;

void Expect(bool ok, const std::string& what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what.c_str());
    ++failures;
  }
}

template <typename T>
void Write(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
}

// float -> IEEE half bits, round to nearest even (finite normal range).
std::uint16_t ToHalf(float x) {
  std::uint32_t b;
  std::memcpy(&b, &x, 4);
  const std::uint32_t sign = (b >> 16) & 0x8000u;
  int exp = static_cast<int>((b >> 23) & 0xFF) - 127 + 15;
  std::uint32_t mant = b & 0x7FFFFFu;
  if (exp <= 0) return static_cast<std::uint16_t>(sign);  // tests use no subnormals
  std::uint32_t h = (static_cast<std::uint32_t>(exp) << 10) | (mant >> 13);
  const std::uint32_t rest = mant & 0x1FFFu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
  return static_cast<std::uint16_t>(sign | h);
}

float FromHalf(std::uint16_t h) {
  const int exp = (h >> 10) & 0x1F;
  const float mant = static_cast<float>(h & 0x3FF);
  const float v = exp == 0 ? mant * std::ldexp(1.0f, -24) : (1.0f + mant / 1024.0f) * std::ldexp(1.0f, exp - 15);
  return (h & 0x8000) ? -v : v;
}

struct Device {
  void* p = nullptr;
  explicit Device(std::size_t bytes) { ov_malloc(&p, bytes); }
  ~Device() { ov_free(p); }
};

void CheckGemm(ov_stream_t stream) {
  std::mt19937 rng(5);
  std::uniform_int_distribution<int> pick(-64, 64);
  HalfGemm gemm(nullptr, stream);
  // Linear on the tcgen05 path (K % 64 == 0) and on the general kernel.
  for (const auto& [rows, in, out, acc] : std::vector<std::tuple<int, int, int, bool>>{
           {100, 128, 256, false}, {333, 1024, 1000, true}, {37, 72, 40, true}}) {
    std::vector<std::uint16_t> x(rows * in), w(out * in);
    std::vector<float> xf(x.size()), wf(w.size()), y0(rows * out);
    for (std::size_t i = 0; i < x.size(); ++i) xf[i] = FromHalf(x[i] = ToHalf(pick(rng) / 32.0f));
    for (std::size_t i = 0; i < w.size(); ++i) wf[i] = FromHalf(w[i] = ToHalf(pick(rng) / 256.0f));
    for (auto& v : y0) v = pick(rng) / 8.0f;
    Device dx(x.size() * 2), dw(w.size() * 2), dy(y0.size() * 4);
    ov_memcpy_h2d_async(dx.p, x.data(), x.size() * 2, stream);
    ov_memcpy_h2d_async(dw.p, w.data(), w.size() * 2, stream);
    ov_memcpy_h2d_async(dy.p, y0.data(), y0.size() * 4, stream);
    gemm.Linear(dx.p, dw.p, static_cast<float*>(dy.p), rows, in, out, acc);
    std::vector<float> y(y0.size());
    ov_memcpy_d2h_async(y.data(), dy.p, y.size() * 4, stream);
    ov_stream_sync(stream);
    double worst = 0;
    for (int r = 0; r < rows; ++r)
      for (int o = 0; o < out; ++o) {
        double ref = acc ? y0[r * out + o] : 0.0;
        for (int k = 0; k < in; ++k) ref += static_cast<double>(xf[r * in + k]) * wf[o * in + k];
        worst = std::max(worst, std::fabs(ref - y[r * out + o]));
      }
    Expect(worst < 1e-3, "HalfGemm::Linear " + std::to_string(rows) + "x" + std::to_string(in) +
                             "x" + std::to_string(out) + " max err " + std::to_string(worst));
  }
  // Strided-batched Matmul with every transpose combination.
  for (int ta = 0; ta < 2; ++ta)
    for (int tb = 0; tb < 2; ++tb) {
      MatmulShape s;
      s.transpose_a = ta;
      s.transpose_b = tb;
      s.m = 45;
      s.n = 70;
      s.k = 53;
      s.lda = (ta ? s.k : s.m) + 3;
      s.ldb = (tb ? s.n : s.k) + 1;
      s.ldc = s.m + 2;
      s.batch = 3;
      s.stride_a = static_cast<std::int64_t>(s.lda * (ta ? s.m : s.k));
      s.stride_b = static_cast<std::int64_t>(s.ldb * (tb ? s.k : s.n));
      s.stride_c = static_cast<std::int64_t>(s.ldc * s.n);
      s.accumulate = (ta + tb) % 2 == 1;
      std::vector<std::uint16_t> a(s.stride_a * s.batch), b(s.stride_b * s.batch);
      std::vector<float> c0(s.stride_c * s.batch);
      for (auto& v : a) v = ToHalf(pick(rng) / 32.0f);
      for (auto& v : b) v = ToHalf(pick(rng) / 32.0f);
      for (auto& v : c0) v = pick(rng) / 4.0f;
      Device da(a.size() * 2), db(b.size() * 2), dc(c0.size() * 4);
      ov_memcpy_h2d_async(da.p, a.data(), a.size() * 2, stream);
      ov_memcpy_h2d_async(db.p, b.data(), b.size() * 2, stream);
      ov_memcpy_h2d_async(dc.p, c0.data(), c0.size() * 4, stream);
      gemm.Matmul(s, s, da.p, db.p, static_cast<float*>(dc.p));
      std::vector<float> c(c0.size());
      ov_memcpy_d2h_async(c.data(), dc.p, c.size() * 4, stream);
      ov_stream_sync(stream);
      double worst = 0;
      for (std::size_t bi = 0; bi < s.batch; ++bi)
        for (std::size_t i = 0; i < s.m; ++i)
          for (std::size_t j = 0; j < s.n; ++j) {
            const std::size_t ci = bi * s.stride_c + i + j * s.ldc;
            double ref = s.accumulate ? c0[ci] : 0.0;
            for (std::size_t l = 0; l < s.k; ++l) {
              const float av = FromHalf(a[bi * s.stride_a + (ta ? l + i * s.lda : i + l * s.lda)]);
              const float bv = FromHalf(b[bi * s.stride_b + (tb ? j + l * s.ldb : l + j * s.ldb)]);
              ref += static_cast<double>(av) * bv;
            }
            worst = std::max(worst, std::fabs(ref - c[ci]));
          }
      Expect(worst < 1e-3, "HalfGemm::Matmul ta=" + std::to_string(ta) + " tb=" +
                               std::to_string(tb) + " max err " + std::to_string(worst));
    }
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 9) {
    std::fprintf(stderr, "usage: %s model_root out_dir vocab hidden inter layers heads kv\n",
                 argv[0]);
    return 2;
  }
  const std::string root = argv[1], out = argv[2];
  Config cfg;
  cfg.backbone.vocab_size = std::stoul(argv[3]);
  cfg.backbone.hidden_size = std::stoul(argv[4]);
  cfg.backbone.intermediate_size = std::stoul(argv[5]);
  cfg.backbone.layers = std::stoul(argv[6]);
  cfg.backbone.heads = std::stoul(argv[7]);
  cfg.backbone.kv_heads = std::stoul(argv[8]);
  cfg.backbone.head_dim = 128;
  cfg.backbone.max_positions = 40960;
  cfg.backbone.rms_norm_eps = 1e-6F;
  cfg.backbone.rope_theta = 1e6F;
  cfg.audio_codebooks = 8;
  cfg.audio_vocab_size = 1025;
  cfg.audio_mask_id = 1024;

  std::string error;
  Expect(Generator::Load(cfg, root + "/missing-dir", &error) == nullptr, "load of a missing model");
  Expect(error.rfind("OmniVoice generator: ", 0) == 0, "load error prefix: " + error);

  auto gen = Generator::Load(cfg, root, &error);
  if (gen == nullptr) {
    std::fprintf(stderr, "load failed: %s\n", error.c_str());
    return 1;
  }
  std::vector<std::uint32_t> text;
  for (int i = 0; i < 9; ++i) text.push_back(static_cast<std::uint32_t>((i * 977 + 13) % cfg.backbone.vocab_size));
  std::vector<std::int32_t> ref(8 * 10);
  for (std::size_t i = 0; i < ref.size(); ++i) ref[i] = static_cast<std::int32_t>((i * 131 + 7) % 1024);
  const ConditionalInput in = ConditionalInput::Build(text, ref, 10, 33, 8, 1024);
  const ConditionalInput in2 = ConditionalInput::Build(text, {}, 0, 21, 8, 1024);
  Write(out + "/ids.i32", in.ids);
  Write(out + "/meta.i32", std::vector<std::int32_t>{static_cast<std::int32_t>(in.length),
                                                      static_cast<std::int32_t>(in.audio_start),
                                                      static_cast<std::int32_t>(in.target_frames)});
  std::vector<float> logits;
  Expect(gen->Forward(in, &logits, &error), "Forward: " + error);
  Write(out + "/forward.f32", logits);
  std::vector<std::int32_t> prediction;
  std::vector<float> confidence;
  Expect(gen->Score(in, 2.0F, &prediction, &confidence, &error), "Score: " + error);
  Write(out + "/prediction.i32", prediction);
  Write(out + "/confidence.f32", confidence);

  DecodingConfig decoding;
  GenerationResult result;
  Expect(gen->Generate(in, decoding, 7, {}, &result, &error), "Generate: " + error);
  Write(out + "/codes.i32", result.codes);
  Write(out + "/unmasked.i32", result.unmasked_at);

  std::vector<GenerationResult> batch;
  Expect(gen->GenerateBatch({in, in2}, decoding, {7, 8}, [] { return false; }, &batch, &error),
         "GenerateBatch: " + error);
  GenerationResult single2;
  Expect(gen->Generate(in2, decoding, 8, {}, &single2, &error), "Generate 2: " + error);
  Expect(batch.size() == 2 && batch[0].codes == result.codes &&
             batch[0].unmasked_at == result.unmasked_at && batch[1].codes == single2.codes,
         "GenerateBatch equals single generations");

  int polls = 0;
  error.clear();
  const bool done = gen->Generate(in, decoding, 7, [&] { return ++polls > 3; }, &result, &error);
  Expect(!done && error == "cancelled", "cancellation reports \"cancelled\", got: " + error);

  ConditionalInput broken = in;
  broken.ids.pop_back();
  Expect(!gen->Forward(broken, &logits, &error) && error.rfind("OmniVoice forward: ", 0) == 0,
         "forward error prefix: " + error);

  ov_stream_t stream = nullptr;
  ov_stream_create(&stream);
  CheckGemm(stream);
  ov_stream_destroy(stream);

  if (failures != 0) return 1;
  std::printf("ok\n");
  return 0;
}
