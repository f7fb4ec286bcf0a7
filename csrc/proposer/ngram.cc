#include "ngram.h"

#include <algorithm>
#include <limits>

#include "suffix_cache.h"

namespace sh {

namespace {
constexpr size_t kUnset = std::numeric_limits<size_t>::max();

NgramResult pick(const int64_t* ctx, size_t len, size_t lo, size_t hi, size_t cap, const size_t* latest) {
  NgramResult r;
  for (size_t n = hi + 1; n-- > lo;) {
    const size_t pos = latest[n - lo];
    if (pos == kUnset) continue;
    const size_t end = std::min(pos + n + cap, len);
    r.tokens.assign(ctx + pos + n, ctx + end);
    r.score = static_cast<double>(n) / static_cast<double>(n + 1);
    return r;
  }
  return r;
}

// Backward LCP between the context ending at len - q and the context's end,
// capped at hi (and at len - q so the match never runs past the start).
inline size_t lcp_back(const int64_t* ctx, size_t len, size_t q, size_t hi) {
  size_t l = 0;
  while (l < hi && q + l < len && ctx[len - 1 - q - l] == ctx[len - 1 - l]) ++l;
  return l;
}
}  // namespace

NgramResult ngram_scan(const int64_t* ctx, size_t len, size_t lo, size_t hi, size_t cap, size_t window) {
  if (cap == 0) return {};
  if (len == 0) return {};
  hi = std::min(hi, len - 1);
  if (hi < lo) return {};
  const size_t q_max = window == 0 ? len : std::min(window, len);
  size_t latest_buf[129];
  std::vector<size_t> latest_heap;
  size_t* latest = latest_buf;
  if (hi - lo + 1 > 129) {
    latest_heap.resize(hi - lo + 1);
    latest = latest_heap.data();
  }
  std::fill(latest, latest + (hi - lo + 1), kUnset);
  for (size_t q = 1; q < q_max; ++q) {
    const size_t l = lcp_back(ctx, len, q, hi);
    if (l < lo) continue;
    for (size_t n = lo; n <= std::min(l, hi); ++n)
      if (latest[n - lo] == kUnset) latest[n - lo] = len - n - q;
    if (latest[hi - lo] != kUnset) break;
  }
  return pick(ctx, len, lo, hi, cap, latest);
}

void NgramIndex::rehash(const int64_t* ctx, size_t want) {
  size_t cap = 1024;
  while (cap < want * 2) cap <<= 1;
  head_.assign(cap, -1);
  const size_t mask = cap - 1;
  for (size_t p = 0; p < indexed_; ++p) {
    const size_t b = window_hash(ctx + p, lo_) & mask;
    prev_[p] = head_[b];
    head_[b] = static_cast<int32_t>(p);
  }
}

void NgramIndex::extend(const int64_t* ctx, size_t len) {
  if (len < lo_) return;
  const size_t last = len - lo_ + 1;  // lo-grams starting at [0, last)
  if (last <= indexed_) return;
  prev_.resize(last);
  if (head_.size() < last * 2) {
    rehash(ctx, last);
  }
  const size_t mask = head_.size() - 1;
  for (size_t p = indexed_; p < last; ++p) {
    const size_t b = window_hash(ctx + p, lo_) & mask;
    prev_[p] = head_[b];
    head_[b] = static_cast<int32_t>(p);
  }
  indexed_ = last;
}

NgramResult NgramIndex::query(const int64_t* ctx, size_t len, size_t hi, size_t cap, size_t window) {
  const size_t lo = lo_;
  if (cap == 0 || len == 0) return {};
  if (len > static_cast<size_t>(std::numeric_limits<int32_t>::max())) return ngram_scan(ctx, len, lo, hi, cap, window);
  hi = std::min(hi, len - 1);
  if (hi < lo) return {};
  if (len < indexed_ + lo - 1) reset();  // context shrank: start over
  extend(ctx, len);
  const size_t q_max = window == 0 ? len : std::min(window, len);
  size_t latest_buf[129];
  std::vector<size_t> latest_heap;
  size_t* latest = latest_buf;
  if (hi - lo + 1 > 129) {
    latest_heap.resize(hi - lo + 1);
    latest = latest_heap.data();
  }
  std::fill(latest, latest + (hi - lo + 1), kUnset);
  // The tail lo-gram starts at len - lo; an occurrence starting at p sits at
  // end-aligned distance q = len - lo - p.  Walk the chain newest first.
  const size_t tail = len - lo;
  const size_t mask = head_.size() - 1;
  int32_t p = head_[window_hash(ctx + tail, lo) & mask];
  while (p >= 0) {
    const size_t up = static_cast<size_t>(p);
    if (up < tail) {
      const size_t q = tail - up;
      if (q >= q_max) break;  // older occurrences are all out of the window
      const size_t l = lcp_back(ctx, len, q, hi);
      if (l >= lo) {
        for (size_t n = lo; n <= std::min(l, hi); ++n)
          if (latest[n - lo] == kUnset) latest[n - lo] = len - n - q;
        if (latest[hi - lo] != kUnset) break;
      }
    }
    p = prev_[up];
  }
  return pick(ctx, len, lo, hi, cap, latest);
}

}  // namespace sh
