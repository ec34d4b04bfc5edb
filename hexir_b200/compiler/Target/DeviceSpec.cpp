//===- DeviceSpec.cpp - cpu | cuda | cuda:N | cuda:F-L --------------------===//
//
// Builds without LLVM (standard C++17); compiled and tested in this
// repository by tests/test_compiler_surface.py.
//
//===----------------------------------------------------------------------===//
#include "DeviceSpec.h"

namespace hexir_b200 {
namespace {

// At most four decimal digits (GPU ordinals of one box; the writer's limit).
bool parseOrdinal(std::string_view s, uint32_t *v) {
  if (s.empty() || s.size() > 4)
    return false;
  uint32_t x = 0;
  for (char c : s) {
    if (c < '0' || c > '9')
      return false;
    x = x * 10 + static_cast<uint32_t>(c - '0');
  }
  *v = x;
  return true;
}

bool startsWith(std::string_view s, std::string_view prefix) {
  return s.substr(0, prefix.size()) == prefix;
}

} // namespace

bool parseDeviceSpec(std::string_view text, DeviceSpec *out) {
  DeviceSpec d;
  if (text == "cpu") {
    *out = d;
    return true;
  }
  d.cuda = true;
  if (text == "cuda" || text == "gpu") {
    *out = d;
    return true;
  }
  std::string_view rest;
  if (startsWith(text, "cuda:"))
    rest = text.substr(5);
  else if (startsWith(text, "gpu:"))
    rest = text.substr(4);
  else
    return false;
  d.ordinal = true;
  const size_t dash = rest.find('-');
  if (dash == std::string_view::npos) {
    if (!parseOrdinal(rest, &d.first))
      return false;
    *out = d;
    return true;
  }
  uint32_t last = 0;
  if (!parseOrdinal(rest.substr(0, dash), &d.first) ||
      !parseOrdinal(rest.substr(dash + 1), &last) || last < d.first)
    return false;
  d.count = last - d.first + 1;
  *out = d;
  return true;
}

std::string_view deviceKind(std::string_view text) {
  DeviceSpec d;
  if (!parseDeviceSpec(text, &d))
    return {};
  return d.cuda ? std::string_view("cuda") : std::string_view("cpu");
}

std::string canonicalDeviceSpec(std::string_view text) {
  DeviceSpec d;
  if (!parseDeviceSpec(text, &d))
    return {};
  if (!d.cuda)
    return "cpu";
  if (!d.ordinal)
    return "cuda";
  std::string s = "cuda:" + std::to_string(d.first);
  if (d.count > 1)
    s += "-" + std::to_string(d.first + d.count - 1);
  return s;
}

bool isCudaSpec(std::string_view text) { return deviceKind(text) == "cuda"; }

} // namespace hexir_b200
