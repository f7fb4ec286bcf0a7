// Environment-driven knobs of the proposer core.
//
// Every knob is read when the owning object is constructed (never cached
// process-wide), so a test or an operator can change SUFFIX_HYBRID_* between
// constructions.  Names, defaults and clamps match the reference's knobs
// (reference: src/lib.rs:85-127, src/engine.rs:210-243, src/mixer.rs:142-147).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace sh {

// Integer knob SUFFIX_HYBRID_<name>: unparsable or missing -> default, then
// clamped to [lo, hi].  Negative text does not parse as unsigned -> default.
size_t env_size(const char* name, size_t def, size_t lo, size_t hi);
// Float knob; non-finite or unparsable -> default.
double env_double(const char* name, double def);
// Raw string knob (empty when unset).
std::string env_string(const char* name);

struct CacheConfig {
  size_t n;           // INDEX_N: n-gram order of the corpus index
  size_t depth;       // MAX_TREE_DEPTH: lookback window for match extension
  size_t sequences;   // MAX_CACHED_REQUESTS
  size_t tokens;      // MAX_CACHED_TOKENS
  size_t positions;   // MAX_POSITIONS_PER_NGRAM
  size_t candidates;  // MAX_CANDIDATES
  size_t support;     // MIN_TOKEN_COUNT
  double factor;      // MAX_SPEC_FACTOR
  double offset;      // MAX_SPEC_OFFSET
  bool prompts;       // INDEX_PROMPTS

  static CacheConfig from_env();
};

}  // namespace sh
