// fault.cc -- host-side fault injection (include/hexir_b200/fault.h).

#include "fault.h"

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "hexir_b200/fault.h"

namespace hexir {

namespace {

constexpr int kSites = 3;
const char *const kSiteNames[kSites] = {"alloc", "launch", "nccl"};

struct Rule {
  uint64_t first = 0;
  bool onward = false;
};

struct Rules {
  std::vector<Rule> by_site[kSites];
};

struct State {
  std::atomic<bool> active{false};
  std::atomic<uint64_t> calls[kSites] = {};
  std::mutex mu;
  Rules rules;
};

State &state() {
  static State *s = new State;  // never destroyed: checked during exit too
  return *s;
}

int site_index(const std::string &name) {
  for (int i = 0; i < kSites; ++i)
    if (name == kSiteNames[i])
      return i;
  return -1;
}

// "site:N[+]" entries separated by commas; false on any malformed entry.
bool parse(const char *spec, Rules *out) {
  const std::string all(spec);
  for (size_t pos = 0; pos <= all.size();) {
    size_t comma = all.find(',', pos);
    if (comma == std::string::npos)
      comma = all.size();
    const std::string entry = all.substr(pos, comma - pos);
    pos = comma + 1;
    const size_t colon = entry.find(':');
    if (colon == std::string::npos)
      return false;
    const int site = site_index(entry.substr(0, colon));
    std::string count = entry.substr(colon + 1);
    Rule rule;
    if (!count.empty() && count.back() == '+') {
      rule.onward = true;
      count.pop_back();
    }
    if (site < 0 || count.empty() || count.size() > 18)
      return false;
    for (char c : count)
      if (c < '0' || c > '9')
        return false;
    rule.first = std::strtoull(count.c_str(), nullptr, 10);
    if (rule.first == 0)
      return false;
    out->by_site[site].push_back(rule);
  }
  return true;
}

void install(const Rules &rules) {
  State &s = state();
  std::lock_guard<std::mutex> lock(s.mu);
  s.rules = rules;
  bool any = false;
  for (int i = 0; i < kSites; ++i) {
    s.calls[i].store(0, std::memory_order_relaxed);
    any = any || !rules.by_site[i].empty();
  }
  s.active.store(any, std::memory_order_release);
}

std::once_flag g_env_once;

void load_env() {
  const char *spec = std::getenv("HEXIR_FAULT");
  if (!spec || !*spec)
    return;
  Rules rules;
  if (parse(spec, &rules))
    install(rules);
  else
    std::fprintf(stderr, "hexir: ignoring malformed HEXIR_FAULT '%s'\n", spec);
}

}  // namespace

bool fault_hit(FaultSite site) {
  std::call_once(g_env_once, load_env);
  State &s = state();
  if (!s.active.load(std::memory_order_acquire))
    return false;
  const int i = static_cast<int>(site);
  const uint64_t n = s.calls[i].fetch_add(1, std::memory_order_relaxed) + 1;
  std::lock_guard<std::mutex> lock(s.mu);
  for (const Rule &r : s.rules.by_site[i])
    if (n == r.first || (r.onward && n >= r.first))
      return true;
  return false;
}

}  // namespace hexir

extern "C" hexir_status_t hexir_fault_configure(const char *spec) {
  std::call_once(hexir::g_env_once, hexir::load_env);
  hexir::Rules rules;
  if (spec && *spec && !hexir::parse(spec, &rules))
    return HEXIR_ERROR_INVALID_ARGUMENT;
  hexir::install(rules);
  return HEXIR_OK;
}

extern "C" uint64_t hexir_fault_calls(const char *site) {
  std::call_once(hexir::g_env_once, hexir::load_env);
  const int i = site ? hexir::site_index(site) : -1;
  if (i < 0)
    return 0;
  hexir::State &s = hexir::state();
  if (!s.active.load(std::memory_order_acquire))
    return 0;
  return s.calls[i].load(std::memory_order_relaxed);
}
