// In-request n-gram lookup ("prompt lookup").
//
// Semantics (reference: src/engine.rs:29-82): for orders n in [lo, hi], find
// the LATEST earlier occurrence of the context's last n tokens (never the
// suffix itself); the longest order that occurs wins and its continuation
// (up to `cap` tokens) is the draft, scored n/(n+1).  `window` > 0 keeps only
// occurrences whose end-aligned distance q = len - n - pos is below `window`.
//
// Two implementations with identical results:
//  * ngram_scan: one backward pass over the context (O(context) per call),
//    used for one-off contexts;
//  * NgramIndex: an incremental per-request index (chain of previous
//    occurrences of every lo-gram) for contexts that grow by a few tokens
//    per decode step.  A query walks only the occurrences of the tail
//    lo-gram, newest first, so steady-state cost no longer scales with the
//    context length.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

namespace sh {

struct NgramResult {
  std::vector<int64_t> tokens;
  double score = 0.0;
};

NgramResult ngram_scan(const int64_t* ctx, size_t len, size_t lo, size_t hi, size_t cap, size_t window);

class NgramIndex {
 public:
  NgramIndex() = default;
  explicit NgramIndex(size_t lo) : lo_(lo) {}
  // Query over ctx[0:len); indexes any positions not yet covered first.  The
  // caller guarantees ctx only grows by appending between calls (or calls
  // reset() when it does not).
  NgramResult query(const int64_t* ctx, size_t len, size_t hi, size_t cap, size_t window);
  void reset() {
    head_.clear();
    prev_.clear();
    indexed_ = 0;
  }
  size_t lo() const { return lo_; }

 private:
  void extend(const int64_t* ctx, size_t len);
  void rehash(const int64_t* ctx, size_t cap);
  size_t lo_ = 4;
  std::vector<int32_t> head_;  // bucket -> latest position (or -1)
  std::vector<int32_t> prev_;  // position -> previous position in chain
  size_t indexed_ = 0;         // lo-grams starting at [0, indexed_) are indexed
};

}  // namespace sh
