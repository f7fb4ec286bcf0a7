#include "engine.h"

#include <algorithm>

namespace sh {

namespace {
constexpr size_t kFingerprint = 64;  // head/tail identity window
}

Engine::Engine(size_t num_speculative_tokens, size_t max_model_len) {
  if (max_model_len == 0 || max_model_len > 16777216) throw ValueError("max_model_len must be in 1..16777216");
  corpus_ = std::make_shared<SharedCorpus>(CacheConfig::from_env());
  const size_t override_k = env_size("MAX_SPEC_TOKENS", 0, 0, 4096);
  k_ = override_k == 0 ? std::min<size_t>(num_speculative_tokens, 4096) : override_k;
  max_model_len_ = max_model_len;
  max_rows_ = env_size("MAX_ACTIVE_ROWS", 4096, 1, 65536);
  ngram_min_ = env_size("NGRAM_MIN", 4, 1, 128);
  ngram_max_ = env_size("NGRAM_MAX", 16, ngram_min_, 128);
  ngram_window_ = env_size("NGRAM_WINDOW", 0, 0, 16777216);
  use_ngram_ = env_size("USE_NGRAM", 1, 0, 1) == 1;
  log_interval_ = env_size("LOG_INTERVAL", 100, 1, 1000000);
  stats_interval_ = env_size("STATS_INTERVAL", 100, 1, 1000000);
}

std::vector<std::vector<int64_t>> Engine::propose(const std::vector<char>& sampled_nonempty, const IntVector& counts,
                                                  const IntMatrix& tokens) {
  const size_t size = sampled_nonempty.size();
  if (size > max_rows_ || counts.n < size || tokens.rows < size)
    throw ValueError("batch dimensions exceed buffers or MAX_ACTIVE_ROWS");
  for (size_t i = 0; i < size; ++i) {
    const int64_t n = counts.at(i);
    if (n < 0 || static_cast<size_t>(n) > tokens.cols || static_cast<size_t>(n) > max_model_len_)
      throw ValueError("num_tokens_no_spec outside buffer/max_model_len");
  }
  // Validation passed: from here on the call mutates state.
  std::vector<Row> old = std::move(rows_);
  rows_.clear();
  for (Row& r : old) r.taken = false;
  std::vector<Row> current;
  current.reserve(size);
  for (size_t i = 0; i < size; ++i) {
    const size_t n = static_cast<size_t>(counts.at(i));
    const int64_t* fast = tokens.row64(i);
    auto prefix_of_row = [&](const Row& r) -> bool {
      const size_t m = r.ctx.size();
      if (r.taken || m == 0 || m > n) return false;
      const size_t w = std::min(kFingerprint, m);
      if (fast) {
        return std::equal(r.ctx.begin(), r.ctx.begin() + w, fast) &&
               std::equal(r.ctx.end() - w, r.ctx.end(), fast + (m - w));
      }
      for (size_t j = 0; j < w; ++j)
        if (r.ctx[j] != tokens.at(i, j)) return false;
      for (size_t j = m - w; j < m; ++j)
        if (r.ctx[j] != tokens.at(i, j)) return false;
      return true;
    };
    Row* match = nullptr;
    if (i < old.size() && prefix_of_row(old[i])) {
      match = &old[i];
    } else {
      for (Row& r : old)
        if (prefix_of_row(r)) {
          match = &r;
          break;
        }
    }
    Row row;
    if (match) {
      match->taken = true;
      row.ctx = std::move(match->ctx);
      row.index = std::move(match->index);
    } else {
      row.index = NgramIndex(ngram_min_);
    }
    const size_t have = row.ctx.size();
    // geometric growth: a row that grows by a few tokens per call must not be copied whole every call
    if (row.ctx.capacity() < n) row.ctx.reserve(std::max(n, row.ctx.capacity() + row.ctx.capacity() / 2));
    if (fast) {
      row.ctx.insert(row.ctx.end(), fast + have, fast + n);
    } else {
      for (size_t j = have; j < n; ++j) row.ctx.push_back(tokens.at(i, j));
    }
    current.push_back(std::move(row));
  }
  std::vector<std::vector<int64_t>> result(size);
  {
    std::lock_guard<std::mutex> lock(corpus_->mu);
    SuffixCorpus& cache = corpus_->corpus;
    for (Row& r : old)
      if (!r.taken) cache.add(r.ctx);
    const double ng_ratio = static_cast<double>(ngram_max_) / static_cast<double>(ngram_max_ + 1);
    for (size_t i = 0; i < size; ++i) {
      Row& row = current[i];
      const size_t len = row.ctx.size();
      const size_t cap = std::min(k_, max_model_len_ > len ? max_model_len_ - len : 0);
      if (!sampled_nonempty[i] || cap == 0) continue;
      SpecResult suf = cache.speculate(row.ctx.data(), len, cap);
      const double suf_val = suf.score * static_cast<double>(suf.tokens.size());
      NgramResult ng;
      if (use_ngram_ && suf_val < ng_ratio * static_cast<double>(cap))
        ng = row.index.query(row.ctx.data(), len, ngram_max_, cap, ngram_window_);
      if (!suf.tokens.empty() && suf_val >= ng.score * static_cast<double>(ng.tokens.size())) {
        ++suffix_proposals_;
        match_sum_ += suf.match_len;
        result[i] = std::move(suf.tokens);
      } else {
        if (!ng.tokens.empty()) ++ngram_proposals_;
        result[i] = std::move(ng.tokens);
      }
      proposed_ += result[i].size();
    }
  }
  rows_ = std::move(current);
  ++calls_;
  return result;
}

std::pair<bool, bool> Engine::record_total(uint64_t elapsed_ns) {
  total_ns_ += elapsed_ns;
  return {calls_ % log_interval_ == 0, calls_ % stats_interval_ == 0};
}

Engine::Stats Engine::stats() const {
  Stats s{};
  s.calls = calls_;
  s.proposed = proposed_;
  s.suffix_proposals = suffix_proposals_;
  s.ngram_proposals = ngram_proposals_;
  s.avg_match_len = static_cast<double>(match_sum_) / static_cast<double>(std::max<uint64_t>(suffix_proposals_, 1));
  s.active_requests = rows_.size();
  size_t t = 0;
  for (const Row& r : rows_) t += r.ctx.size();
  s.active_context_tokens = t;
  s.native_ns = native_ns_;
  s.total_ns = total_ns_;
  return s;
}

}  // namespace sh
