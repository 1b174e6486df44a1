// Minimal stand-in for the constants Gufo generates from the extension's
// manifest (extension.json): the provider identity provider.cpp:10-11
// registers.
#ifndef GUFO_EXT_GENERATED_OMNIVOICE_CONSTANTS_HPP_
#define GUFO_EXT_GENERATED_OMNIVOICE_CONSTANTS_HPP_

#include <gufo/ext/registry.hpp>

namespace gufo::ext::generated::extension_omnivoice {

inline constexpr ProviderInfo kProvider_omnivoice{"omnivoice", "omnivoice"};

}  // namespace gufo::ext::generated::extension_omnivoice

#endif  // GUFO_EXT_GENERATED_OMNIVOICE_CONSTANTS_HPP_
