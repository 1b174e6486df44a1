// Deterministic random-init weights, bit-identical on host and device.
//
// value(i) = float(s - 131070) * scale, where s is the sum of the four
// 16-bit lanes of h = mix64(base + i), base = mix64(seed ^ tensor * phi64),
// mix64 the splitmix64 finaliser (Steele, Lea & Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014).  s follows an Irwin-Hall
// distribution of four discrete uniforms: mean 131070, standard deviation
// sqrt((65536^2 - 1) / 3), so scale = std / that deviation gives an
// approximately N(0, std^2) weight.  Only integer arithmetic, one exact
// int->float conversion and one rounded multiply are involved, so host and
// device produce the same floats.
#pragma once

#include <cmath>
#include <cstdint>

#if defined(__CUDACC__)
#define OVB_HD __host__ __device__ __forceinline__
#else
#define OVB_HD inline
#endif

namespace ovb {

OVB_HD uint64_t Mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

OVB_HD uint64_t SyntheticBase(uint64_t seed, uint64_t tensor) {
  return Mix64(seed ^ (tensor * 0x9E3779B97F4A7C15ull));
}

inline float SyntheticScale(float std) {
  const double deviation = std::sqrt((65536.0 * 65536.0 - 1.0) / 3.0);
  return static_cast<float>(static_cast<double>(std) / deviation);
}

OVB_HD float SyntheticValue(uint64_t base, uint64_t index, float scale) {
  const uint64_t h = Mix64(base + index);
  const int32_t s = static_cast<int32_t>((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) +
                                         ((h >> 32) & 0xFFFFu) + ((h >> 48) & 0xFFFFu));
  return static_cast<float>(s - 131070) * scale;
}

// Tensor numbering of the synthetic checkpoint: per layer l the tensor id is
// 64 * (l + 1) + kind; the global tensors use ids below 64.
enum SyntheticTensor : uint64_t {
  kTextEmbeddings = 1,
  kAudioEmbeddings = 2,
  kAudioHeads = 3,
  kLayerQ = 0,
  kLayerK = 1,
  kLayerV = 2,
  kLayerO = 3,
  kLayerGate = 4,
  kLayerUp = 5,
  kLayerDown = 6,
};

OVB_HD uint64_t LayerTensor(uint64_t layer, uint64_t kind) { return 64 * (layer + 1) + kind; }

}  // namespace ovb
