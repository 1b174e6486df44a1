// Minimal stand-in for the Gufo SDK's extension registry (see tts.hpp in
// this directory): the two calls the OmniVoice provider makes
// (provider.cpp:8-19), recording what they receive.
#ifndef GUFO_EXT_REGISTRY_HPP_
#define GUFO_EXT_REGISTRY_HPP_

#include <string>
#include <vector>

#include <gufo/ext/tts.hpp>

namespace gufo::ext {

/// A provider's identity, as the extension's generated constants give it.
struct ProviderInfo {
  const char* id;
  const char* extension;
};

class Registry {
 public:
  void AddProvider(const ProviderInfo& provider) { providers.push_back(provider); }
  void AddTtsProvider(TtsProvider provider) { tts.push_back(std::move(provider)); }

  std::vector<ProviderInfo> providers;
  std::vector<TtsProvider> tts;
};

}  // namespace gufo::ext

#endif  // GUFO_EXT_REGISTRY_HPP_
