// CPU restatement of the OmniVoice generator hot path.
// TEST INFRASTRUCTURE ONLY (see oracle.h): the checker of the CUDA path and
// the timed CPU baseline, never part of the product.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <limits>
#include <memory>
#include <numeric>
#include <random>
#include <thread>
#include <vector>

namespace {

using Half = _Float16;

int g_threads = std::max(1u, std::thread::hardware_concurrency());

inline float RoundHalf(float x) { return static_cast<float>(static_cast<Half>(x)); }

// Runs body(begin, end) over [0, count) split across the oracle's threads.
void ParallelFor(size_t count, const std::function<void(size_t, size_t)>& body) {
  const size_t workers = std::min<size_t>(static_cast<size_t>(std::max(1, g_threads)), count);
  if (workers <= 1) {
    if (count > 0) body(0, count);
    return;
  }
  std::vector<std::thread> pool;
  const size_t chunk = (count + workers - 1) / workers;
  for (size_t w = 0; w < workers; ++w) {
    const size_t b = w * chunk;
    const size_t e = std::min(count, b + chunk);
    if (b >= e) break;
    pool.emplace_back([&body, b, e] { body(b, e); });
  }
  for (auto& t : pool) t.join();
}

// ---------------------------------------------------------------- weights
// The synthetic checkpoint, restated from its definition: the value of
// element i of tensor t is float(s - 131070) * (std / sqrt((65536^2-1)/3)),
// s the sum of the four 16-bit lanes of splitmix64-mix(base + i) with
// base = mix(seed ^ t * 0x9E3779B97F4A7C15).  Per layer l the tensor id is
// 64 (l + 1) + {q 0, k 1, v 2, o 3, gate 4, up 5, down 6}; the text
// embeddings are tensor 1, audio embeddings 2, audio heads 3.

uint64_t Mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

struct Synthetic {
  uint64_t base;
  float scale;
  Synthetic(uint64_t seed, uint64_t tensor, float std)
      : base(Mix(seed ^ (tensor * 0x9E3779B97F4A7C15ull))),
        scale(static_cast<float>(static_cast<double>(std) /
                                 std::sqrt((65536.0 * 65536.0 - 1.0) / 3.0))) {}
  float operator()(uint64_t i) const {
    const uint64_t h = Mix(base + i);
    const int32_t s = static_cast<int32_t>((h & 0xFFFF) + ((h >> 16) & 0xFFFF) +
                                           ((h >> 32) & 0xFFFF) + ((h >> 48) & 0xFFFF));
    return static_cast<float>(s - 131070) * scale;
  }
};

constexpr float kStd = 0.02f;

// A linear weight [out][in] stored transposed [in][out] as the float
// values of its half rounding (the reference converts weights to half,
// generator.cpp:31-49, 324-352).
struct Linear {
  size_t in = 0, out = 0;
  std::vector<float> wt;  // [in][out]
};

void FillLinearPart(Linear* lin, size_t out_offset, size_t rows, uint64_t seed, uint64_t tensor) {
  const Synthetic gen(seed, tensor, kStd);
  ParallelFor(rows, [&](size_t b, size_t e) {
    for (size_t o = b; o < e; ++o)
      for (size_t k = 0; k < lin->in; ++k)
        lin->wt[k * lin->out + out_offset + o] = RoundHalf(gen(o * lin->in + k));
  });
}

struct Layer {
  Linear qkv, o, gate_up, down;
  std::vector<float> input_norm, post_norm, q_norm, k_norm;
};

struct Model {
  oc_config cfg;
  uint64_t seed;
  Synthetic text;  // rows generated on demand
  std::vector<float> audio_embeddings;  // [C*V][H] float32
  Linear heads;                         // [C*V] outputs
  std::vector<float> final_norm;
  std::vector<Layer> layers;
  std::vector<float> rope_cos, rope_sin;  // [max_positions][head_dim/2]
  Model(const oc_config& c, uint64_t s) : cfg(c), seed(s), text(s, 1, kStd) {}
};

// ------------------------------------------------------------------- GEMM
// y[r][o] (+)= sum_k x[r][k] * w[o][k] with float32 accumulation in k order.
bool g_reversed_sums = false;

void Gemm(const float* x, size_t rows, const Linear& w, float* y, bool accumulate) {
  const size_t in = w.in, out = w.out;
  constexpr size_t kRb = 4, kOb = 256;
  const size_t row_blocks = (rows + kRb - 1) / kRb;
  const size_t out_blocks = (out + kOb - 1) / kOb;
  ParallelFor(row_blocks * out_blocks, [&](size_t b, size_t e) {
    float acc[kRb][kOb];
    for (size_t item = b; item < e; ++item) {
      const size_t r0 = (item / out_blocks) * kRb;
      const size_t o0 = (item % out_blocks) * kOb;
      const size_t nr = std::min(kRb, rows - r0);
      const size_t no = std::min(kOb, out - o0);
      for (size_t i = 0; i < kRb; ++i)
        for (size_t j = 0; j < kOb; ++j) acc[i][j] = 0.0f;
      for (size_t kk = 0; kk < in; ++kk) {
        const size_t k = g_reversed_sums ? in - 1 - kk : kk;
        const float* wr = &w.wt[k * out + o0];
        for (size_t i = 0; i < nr; ++i) {
          const float xv = x[(r0 + i) * in + k];
          float* a = acc[i];
          for (size_t j = 0; j < no; ++j) a[j] = std::fma(xv, wr[j], a[j]);
        }
      }
      for (size_t i = 0; i < nr; ++i) {
        float* yr = y + (r0 + i) * out + o0;
        for (size_t j = 0; j < no; ++j) yr[j] = accumulate ? yr[j] + acc[i][j] : acc[i][j];
      }
    }
  });
}

// generator_kernels.hip:85-97: half(w * (x * rsqrt(mean(x^2) + eps))).
void RmsNormRow(const float* x, const float* w, size_t width, float eps, float* out) {
  float squares = 0.0f;
  for (size_t d = 0; d < width; ++d) squares += x[d] * x[d];
  const float scale = 1.0f / std::sqrt(squares / static_cast<float>(width) + eps);
  for (size_t d = 0; d < width; ++d) out[d] = RoundHalf(w[d] * (x[d] * scale));
}

}  // namespace

extern "C" {

void oc_set_threads(int threads) { g_threads = std::max(1, threads); }
int oc_get_threads(void) { return g_threads; }

void* oc_model_synthetic(const oc_config* config, uint64_t seed) {
  const oc_config& c = *config;
  auto m = std::make_unique<Model>(c, seed);
  const size_t H = c.hidden_size, I = c.intermediate_size, D = c.head_dim;
  const size_t audio_rows = c.audio_codebooks * c.audio_vocab_size;
  m->audio_embeddings.resize(audio_rows * H);
  {
    const Synthetic gen(seed, 2, kStd);
    ParallelFor(audio_rows, [&](size_t b, size_t e) {
      for (size_t i = b * H; i < e * H; ++i) m->audio_embeddings[i] = gen(i);
    });
  }
  m->heads.in = H;
  m->heads.out = audio_rows;
  m->heads.wt.resize(H * audio_rows);
  FillLinearPart(&m->heads, 0, audio_rows, seed, 3);
  m->final_norm.assign(H, 1.0f);
  m->layers.resize(c.layers);
  const size_t q_rows = c.heads * D, kv_rows = c.kv_heads * D;
  for (size_t l = 0; l < c.layers; ++l) {
    Layer& L = m->layers[l];
    const uint64_t t0 = 64 * (l + 1);
    L.qkv.in = H;
    L.qkv.out = q_rows + 2 * kv_rows;
    L.qkv.wt.resize(H * L.qkv.out);
    FillLinearPart(&L.qkv, 0, q_rows, seed, t0 + 0);
    FillLinearPart(&L.qkv, q_rows, kv_rows, seed, t0 + 1);
    FillLinearPart(&L.qkv, q_rows + kv_rows, kv_rows, seed, t0 + 2);
    L.o.in = q_rows;
    L.o.out = H;
    L.o.wt.resize(q_rows * H);
    FillLinearPart(&L.o, 0, H, seed, t0 + 3);
    L.gate_up.in = H;
    L.gate_up.out = 2 * I;
    L.gate_up.wt.resize(H * 2 * I);
    FillLinearPart(&L.gate_up, 0, I, seed, t0 + 4);
    FillLinearPart(&L.gate_up, I, I, seed, t0 + 5);
    L.down.in = I;
    L.down.out = H;
    L.down.wt.resize(I * H);
    FillLinearPart(&L.down, 0, H, seed, t0 + 6);
    L.input_norm.assign(H, 1.0f);
    L.post_norm.assign(H, 1.0f);
    L.q_norm.assign(D, 1.0f);
    L.k_norm.assign(D, 1.0f);
  }
  const size_t half = D / 2;
  m->rope_cos.resize(c.max_positions * half);
  m->rope_sin.resize(c.max_positions * half);
  for (size_t i = 0; i < half; ++i) {
    // generator_kernels.hip:209-214.
    const float inv_freq = 1.0f / std::pow(c.rope_theta, static_cast<float>(2 * i) /
                                                              static_cast<float>(D));
    for (size_t p = 0; p < c.max_positions; ++p) {
      const float angle = static_cast<float>(p) * inv_freq;
      m->rope_cos[p * half + i] = std::cos(angle);
      m->rope_sin[p * half + i] = std::sin(angle);
    }
  }
  return m.release();
}

void oc_model_free(void* model) { delete static_cast<Model*>(model); }

void oc_synthetic_values(uint64_t seed, uint64_t tensor, float std, uint64_t first, size_t count,
                         float* out) {
  const Synthetic gen(seed, tensor, std);
  for (size_t i = 0; i < count; ++i) out[i] = gen(first + i);
}

int oc_forward(void* model, const int32_t* ids, size_t length, size_t audio_start,
               size_t frames, float* logits, int layers_to_run, float* hidden_out) {
  Model& m = *static_cast<Model*>(model);
  const oc_config& c = m.cfg;
  const size_t H = c.hidden_size, D = c.head_dim, C = c.audio_codebooks;
  const size_t V = c.audio_vocab_size;
  const size_t heads = c.heads, kv_heads = c.kv_heads, group = heads / kv_heads;
  const size_t R = length + frames;
  const size_t qkv_w = (heads + 2 * kv_heads) * D;
  if (frames > length || audio_start > length) return 1;
  // generator.cpp:218-258: positions, target rows, the packed ids.
  std::vector<int32_t> positions(R), packed(C * R);
  for (size_t r = 0; r < length; ++r) positions[r] = static_cast<int32_t>(r);
  for (size_t f = 0; f < frames; ++f) positions[length + f] = static_cast<int32_t>(f);
  for (size_t cb = 0; cb < C; ++cb) {
    std::copy(ids + cb * length, ids + (cb + 1) * length, &packed[cb * R]);
    std::copy(ids + cb * length + length - frames, ids + (cb + 1) * length, &packed[cb * R + length]);
  }
  for (size_t t = 0; t < audio_start; ++t)
    if (ids[t] < 0 || static_cast<size_t>(ids[t]) >= c.vocab_size) return 2;
  // Embed (generator_kernels.hip:62-83, text rows from generator.cpp:204-217).
  std::vector<float> hidden(R * H);
  ParallelFor(R, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) {
      float* out = &hidden[r * H];
      if (r < audio_start) {
        const uint64_t id = static_cast<uint64_t>(ids[r]);
        for (size_t d = 0; d < H; ++d) out[d] = m.text(id * H + d);
        continue;
      }
      for (size_t d = 0; d < H; ++d) {
        float sum = 0.0f;
        for (size_t cb = 0; cb < C; ++cb) {
          const size_t entry = cb * V + static_cast<size_t>(packed[cb * R + r]);
          sum += m.audio_embeddings[entry * H + d];
        }
        out[d] = sum;
      }
    }
  });
  const size_t run = layers_to_run < 0 ? c.layers : std::min<size_t>(c.layers, layers_to_run);
  std::vector<float> normed(R * std::max(H, c.intermediate_size));
  std::vector<float> qkv(R * qkv_w), q(R * heads * D), k(R * kv_heads * D), v(R * kv_heads * D);
  std::vector<float> merged(R * heads * D), gate_up(R * 2 * c.intermediate_size);
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));
  for (size_t li = 0; li < run; ++li) {
    const Layer& L = m.layers[li];
    ParallelFor(R, [&](size_t b, size_t e) {
      for (size_t r = b; r < e; ++r)
        RmsNormRow(&hidden[r * H], L.input_norm.data(), H, c.rms_norm_eps, &normed[r * H]);
    });
    Gemm(normed.data(), R, L.qkv, qkv.data(), false);
    // QkNormRope (generator_kernels.hip:102-159).
    ParallelFor(R, [&](size_t b, size_t e) {
      for (size_t r = b; r < e; ++r) {
        const float* in = &qkv[r * qkv_w];
        const size_t pos = static_cast<size_t>(positions[r]);
        for (size_t slot = 0; slot < heads + 2 * kv_heads; ++slot) {
          const float* x = in + slot * D;
          if (slot >= heads + kv_heads) {
            float* out = &v[(r * kv_heads + (slot - heads - kv_heads)) * D];
            for (size_t d = 0; d < D; ++d) out[d] = RoundHalf(x[d]);
            continue;
          }
          const bool is_q = slot < heads;
          const float* w = is_q ? L.q_norm.data() : L.k_norm.data();
          float squares = 0.0f;
          for (size_t d = 0; d < D; ++d) squares += x[d] * x[d];
          const float s = 1.0f / std::sqrt(squares / static_cast<float>(D) + c.rms_norm_eps);
          float* out = is_q ? &q[(r * heads + slot) * D] : &k[(r * kv_heads + slot - heads) * D];
          const size_t half = D / 2;
          for (size_t i = 0; i < half; ++i) {
            const float a = w[i] * (x[i] * s);
            const float bb = w[i + half] * (x[i + half] * s);
            const float cs = m.rope_cos[pos * half + i];
            const float sn = m.rope_sin[pos * half + i];
            out[i] = RoundHalf(a * cs - bb * sn);
            out[i + half] = RoundHalf(bb * cs + a * sn);
          }
        }
      }
    });
    // Attention per sequence (generator.cpp:122-172): scores, half softmax
    // probabilities (generator_kernels.hip:231-246), values, merge to half.
    struct Seq {
      size_t first, len;
    };
    const Seq seqs[2] = {{0, length}, {length, frames}};
    for (const Seq& sq : seqs) {
      ParallelFor(heads * sq.len, [&](size_t b, size_t e) {
        std::vector<float> srow(sq.len), o(D);
        for (size_t item = b; item < e; ++item) {
          const size_t h = item / sq.len, i = item % sq.len;
          const size_t kvh = h / group;
          const float* qi = &q[((sq.first + i) * heads + h) * D];
          float maximum = -std::numeric_limits<float>::max();
          for (size_t j = 0; j < sq.len; ++j) {
            const float* kj = &k[((sq.first + j) * kv_heads + kvh) * D];
            float s = 0.0f;
            for (size_t d = 0; d < D; ++d) s += qi[d] * kj[d];
            srow[j] = s;
            maximum = std::max(maximum, s * scale);
          }
          float sum = 0.0f;
          for (size_t j = 0; j < sq.len; ++j) sum += std::exp(srow[j] * scale - maximum);
          const float inverse = 1.0f / sum;
          std::fill(o.begin(), o.end(), 0.0f);
          for (size_t j = 0; j < sq.len; ++j) {
            const float p = RoundHalf(std::exp(srow[j] * scale - maximum) * inverse);
            const float* vj = &v[((sq.first + j) * kv_heads + kvh) * D];
            for (size_t d = 0; d < D; ++d) o[d] += p * vj[d];
          }
          float* out = &merged[(sq.first + i) * heads * D + h * D];
          for (size_t d = 0; d < D; ++d) out[d] = RoundHalf(o[d]);
        }
      });
    }
    Gemm(merged.data(), R, L.o, hidden.data(), true);
    ParallelFor(R, [&](size_t b, size_t e) {
      for (size_t r = b; r < e; ++r)
        RmsNormRow(&hidden[r * H], L.post_norm.data(), H, c.rms_norm_eps, &normed[r * H]);
    });
    Gemm(normed.data(), R, L.gate_up, gate_up.data(), false);
    const size_t I = c.intermediate_size;
    ParallelFor(R, [&](size_t b, size_t e) {
      for (size_t r = b; r < e; ++r)
        for (size_t i = 0; i < I; ++i) {
          // generator_kernels.hip:191-200.
          const float g = gate_up[r * 2 * I + i];
          const float silu = g / (1.0f + std::exp(-g));
          normed[r * I + i] = RoundHalf(silu * gate_up[r * 2 * I + I + i]);
        }
    });
    Gemm(normed.data(), R, L.down, hidden.data(), true);
  }
  if (hidden_out != nullptr) std::copy(hidden.begin(), hidden.end(), hidden_out);
  if (logits == nullptr) return 0;
  // GatherRows + final RmsNorm + audio heads (generator.cpp:295-300).
  std::vector<float> final_normed(2 * frames * H);
  for (size_t f = 0; f < frames; ++f) {
    RmsNormRow(&hidden[(length - frames + f) * H], m.final_norm.data(), H, c.rms_norm_eps,
               &final_normed[f * H]);
    RmsNormRow(&hidden[(length + f) * H], m.final_norm.data(), H, c.rms_norm_eps,
               &final_normed[(frames + f) * H]);
  }
  Gemm(final_normed.data(), 2 * frames, m.heads, logits, false);
  return 0;
}

// generator_kernels.hip:212-265 (ScoreKernel), sequential sums.
int oc_score(const float* logits, size_t ld, size_t frames, size_t codebooks, size_t vocab,
             uint32_t mask_id, float guidance, int32_t* prediction, float* confidence) {
  ParallelFor(frames * codebooks, [&](size_t b, size_t e) {
    std::vector<float> g(vocab);
    for (size_t item = b; item < e; ++item) {
      const size_t f = item / codebooks, cb = item % codebooks;
      const float* cr = logits + f * ld + cb * vocab;
      const float* ur = logits + (frames + f) * ld + cb * vocab;
      float cmax = -std::numeric_limits<float>::max(), umax = cmax;
      for (size_t j = 0; j < vocab; ++j) {
        cmax = std::max(cmax, cr[j]);
        umax = std::max(umax, ur[j]);
      }
      float csum = 0.0f, usum = 0.0f;
      for (size_t j = 0; j < vocab; ++j) {
        csum += std::exp(cr[j] - cmax);
        usum += std::exp(ur[j] - umax);
      }
      const float clse = cmax + std::log(csum);
      const float ulse = umax + std::log(usum);
      float gmax = -std::numeric_limits<float>::max();
      for (size_t j = 0; j < vocab; ++j) {
        const float cc = cr[j] - clse;
        const float uu = ur[j] - ulse;
        const float diff = cc - uu;
        const float scaled = guidance * diff;
        g[j] = cc + scaled;
        gmax = std::max(gmax, g[j]);
      }
      float gsum = 0.0f;
      float best = -std::numeric_limits<float>::max();
      int best_index = static_cast<int>(vocab);
      for (size_t j = 0; j < vocab; ++j) {
        gsum += std::exp(g[j] - gmax);
        if (j != mask_id && g[j] > best) {
          best = g[j];
          best_index = static_cast<int>(j);
        }
      }
      const float glse = gmax + std::log(gsum);
      prediction[cb * frames + f] = best_index;
      confidence[cb * frames + f] = best - glse;
    }
  });
  return 0;
}

// decoding.cpp:12-40.
void oc_schedule(size_t total, size_t steps, float t_shift, size_t* out) {
  std::vector<float> times(steps + 1);
  const float step = 1.0f / static_cast<float>(steps);
  const size_t halfway = (steps + 1) / 2;
  for (size_t i = 0; i <= steps; ++i) {
    // torch.linspace in float32: up from 0 in the first half, down from 1.
    float t = i < halfway ? step * static_cast<float>(i)
                          : 1.0f - step * static_cast<float>(steps - i);
    t = t_shift * t / (1.0f + (t_shift - 1.0f) * t);
    times[i] = t;
  }
  size_t remaining = total;
  for (size_t i = 0; i < steps; ++i) {
    size_t count = remaining;
    if (i + 1 < steps) {
      const double delta = static_cast<double>(times[i + 1]) - static_cast<double>(times[i]);
      count = std::min(static_cast<size_t>(std::ceil(static_cast<double>(total) * delta)),
                       remaining);
    }
    out[i] = count;
    remaining -= count;
  }
}

// decoding.cpp:42-62.
void oc_build_input(const uint32_t* text_ids, size_t text_count, const int32_t* reference_codes,
                    size_t reference_frames, size_t target_frames, size_t codebooks,
                    uint32_t mask_id, int32_t* ids_out) {
  const size_t length = text_count + reference_frames + target_frames;
  for (size_t cb = 0; cb < codebooks; ++cb) {
    int32_t* row = ids_out + cb * length;
    for (size_t t = 0; t < length; ++t) row[t] = static_cast<int32_t>(mask_id);
    for (size_t t = 0; t < text_count; ++t) row[t] = static_cast<int32_t>(text_ids[t]);
    for (size_t f = 0; f < reference_frames; ++f)
      row[text_count + f] = reference_codes[cb * reference_frames + f];
  }
}

// decoding.cpp:84-85: u = (x >> 40) * 2^-24, gumbel = -log(-log(u + 1e-10) + 1e-10).
void oc_reference_gumbel(uint64_t seed, size_t count, float* out) {
  std::mt19937_64 random(seed);
  for (size_t i = 0; i < count; ++i) {
    const float uniform = static_cast<float>(random() >> 40) * 0x1.0p-24F;
    out[i] = -std::log(-std::log(uniform + 1e-10F) + 1e-10F);
  }
}

// decoding.cpp:70-107.
size_t oc_select(size_t count, size_t codebooks, size_t frames, const int32_t* prediction,
                 const float* confidence, uint32_t mask_id, float layer_penalty,
                 float temperature, const float* gumbel, int32_t* codes, size_t* chosen) {
  const size_t total = codebooks * frames;
  std::vector<float> scores(total);
  for (size_t cb = 0; cb < codebooks; ++cb) {
    const float penalty = static_cast<float>(cb) * layer_penalty;
    for (size_t f = 0; f < frames; ++f) {
      const size_t index = cb * frames + f;
      float score = confidence[index] - penalty;
      if (temperature > 0.0f) score = score / temperature + (gumbel ? gumbel[index] : 0.0f);
      if (codes[index] != static_cast<int32_t>(mask_id))
        score = -std::numeric_limits<float>::infinity();
      scores[index] = score;
    }
  }
  count = std::min(count, total);
  std::vector<size_t> order(total);
  std::iota(order.begin(), order.end(), size_t{0});
  std::partial_sort(order.begin(), order.begin() + static_cast<std::ptrdiff_t>(count),
                    order.end(), [&scores](size_t a, size_t b) {
                      if (scores[a] != scores[b]) return scores[a] > scores[b];
                      return a < b;
                    });
  for (size_t i = 0; i < count; ++i) {
    codes[order[i]] = prediction[order[i]];
    if (chosen != nullptr) chosen[i] = order[i];
  }
  return count;
}

void oc_set_accumulation_order(int reversed) { g_reversed_sums = reversed != 0; }

// generator.cpp:486-543.
int oc_generate(void* model, const int32_t* ids, size_t length, size_t audio_start,
                size_t frames, size_t steps, float guidance, float t_shift,
                float layer_penalty, float temperature, uint64_t seed,
                const float* gumbel_all, int32_t* codes, int32_t* unmasked_at) {
  return oc_generate_traced(model, ids, length, audio_start, frames, steps, guidance, t_shift,
                            layer_penalty, temperature, seed, gumbel_all, codes, unmasked_at,
                            nullptr, nullptr, nullptr);
}

int oc_generate_traced(void* model, const int32_t* ids, size_t length, size_t audio_start,
                       size_t frames, size_t steps, float guidance, float t_shift,
                       float layer_penalty, float temperature, uint64_t seed,
                       const float* gumbel_all, int32_t* codes, int32_t* unmasked_at,
                       int32_t* step_ids, int32_t* step_prediction, float* step_confidence) {
  Model& m = *static_cast<Model*>(model);
  const size_t C = m.cfg.audio_codebooks, V = m.cfg.audio_vocab_size;
  const uint32_t mask = m.cfg.audio_mask_id;
  const size_t count = C * frames;
  std::vector<int32_t> current(ids, ids + C * length);
  std::fill(codes, codes + count, static_cast<int32_t>(mask));
  std::fill(unmasked_at, unmasked_at + count, -1);
  std::vector<size_t> schedule(steps);
  oc_schedule(count, steps, t_shift, schedule.data());
  std::vector<float> logits(2 * frames * C * V);
  std::vector<int32_t> prediction(count);
  std::vector<float> confidence(count), noise(count);
  std::vector<size_t> chosen(count);
  std::mt19937_64 random(seed);
  for (size_t step = 0; step < steps; ++step) {
    if (schedule[step] == 0) continue;
    int status = oc_forward(model, current.data(), length, audio_start, frames, logits.data(),
                            -1, nullptr);
    if (status != 0) return status;
    oc_score(logits.data(), C * V, frames, C, V, mask, guidance, prediction.data(),
             confidence.data());
    if (step_ids != nullptr)
      std::copy(current.begin(), current.end(), step_ids + step * C * length);
    if (step_prediction != nullptr)
      std::copy(prediction.begin(), prediction.end(), step_prediction + step * count);
    if (step_confidence != nullptr)
      std::copy(confidence.begin(), confidence.end(), step_confidence + step * count);
    const float* gumbel = nullptr;
    if (temperature > 0.0f) {
      if (gumbel_all != nullptr) {
        gumbel = gumbel_all + step * count;
      } else {
        for (size_t i = 0; i < count; ++i) {
          const float uniform = static_cast<float>(random() >> 40) * 0x1.0p-24F;
          noise[i] = -std::log(-std::log(uniform + 1e-10F) + 1e-10F);
        }
        gumbel = noise.data();
      }
    }
    const size_t n = oc_select(schedule[step], C, frames, prediction.data(), confidence.data(),
                               mask, layer_penalty, temperature, gumbel, codes, chosen.data());
    for (size_t i = 0; i < n; ++i) unmasked_at[chosen[i]] = static_cast<int32_t>(step);
    for (size_t cb = 0; cb < C; ++cb)
      std::copy(codes + cb * frames, codes + (cb + 1) * frames,
                &current[cb * length + length - frames]);
  }
  return 0;
}

}  // extern "C"
