#include "config.h"

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <string>

namespace sh {

static const char* lookup(const char* name, std::string* key) {
  *key = std::string("SUFFIX_HYBRID_") + name;
  return std::getenv(key->c_str());
}

size_t env_size(const char* name, size_t def, size_t lo, size_t hi) {
  std::string key;
  const char* raw = lookup(name, &key);
  size_t v = def;
  if (raw != nullptr) {
    // Accept only a plain non-negative decimal integer (like an unsigned
    // parse): leading/trailing garbage or a sign means "use the default".
    const char* p = raw;
    bool ok = *p != '\0';
    unsigned long long acc = 0;
    for (; *p; ++p) {
      if (*p < '0' || *p > '9') {
        ok = false;
        break;
      }
      unsigned long long next = acc * 10ull + static_cast<unsigned long long>(*p - '0');
      if (next / 10ull != acc) {  // overflow
        ok = false;
        break;
      }
      acc = next;
    }
    if (ok) v = static_cast<size_t>(acc);
  }
  return std::clamp(v, lo, hi);
}

double env_double(const char* name, double def) {
  std::string key;
  const char* raw = lookup(name, &key);
  if (raw == nullptr || *raw == '\0') return def;
  char* end = nullptr;
  errno = 0;
  double v = std::strtod(raw, &end);
  if (end == raw || *end != '\0' || errno != 0 || !std::isfinite(v)) return def;
  return v;
}

std::string env_string(const char* name) {
  std::string key;
  const char* raw = lookup(name, &key);
  return raw ? std::string(raw) : std::string();
}

CacheConfig CacheConfig::from_env() {
  CacheConfig c;
  c.n = env_size("INDEX_N", 8, 1, 128);
  c.depth = env_size("MAX_TREE_DEPTH", 64, 1, 4096);
  c.sequences = env_size("MAX_CACHED_REQUESTS", 512, 0, 100000);
  c.tokens = env_size("MAX_CACHED_TOKENS", 1048576, 0, 100000000);
  c.positions = env_size("MAX_POSITIONS_PER_NGRAM", 64, 1, 4096);
  c.candidates = env_size("MAX_CANDIDATES", 32, 1, 4096);
  c.support = env_size("MIN_TOKEN_COUNT", 1, 1, 4096);
  c.factor = std::max(0.0, env_double("MAX_SPEC_FACTOR", 1.0));
  c.offset = env_double("MAX_SPEC_OFFSET", 0.0);
  c.prompts = env_size("INDEX_PROMPTS", 0, 0, 1) == 1;
  return c;
}

}  // namespace sh
