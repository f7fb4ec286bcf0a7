// Weight-free proposer: cross-request suffix corpus + in-request n-gram.
//
// Contract of the reference's custom_class engine (reference:
// src/engine.rs:85-323): `propose(sampled, num_tokens_no_spec, token_ids)`
// receives authoritative CPU rows that ALREADY contain the sampled tokens.
// Row identity is proven with 64-token head/tail windows, continuing rows
// append only their delta, rows that leave the batch are ingested into the
// corpus, and each row's draft is the better (score x length) of the suffix
// draft and the n-gram draft (the n-gram scan is skipped when it cannot win).
// Continuing rows carry an incremental n-gram index, so the per-step cost is
// independent of context length.
#pragma once
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "ngram.h"
#include "suffix_cache.h"
#include "views.h"

namespace sh {

class Engine {
 public:
  Engine(size_t num_speculative_tokens, size_t max_model_len);

  std::vector<std::vector<int64_t>> propose(const std::vector<char>& sampled_nonempty, const IntVector& counts,
                                            const IntMatrix& tokens);
  std::pair<bool, bool> record_total(uint64_t elapsed_ns);
  void add_native_ns(uint64_t ns) { native_ns_ += ns; }

  std::shared_ptr<SharedCorpus> corpus() const { return corpus_; }
  size_t k() const { return k_; }
  bool use_ngram() const { return use_ngram_; }

  struct Stats {
    uint64_t calls, proposed, suffix_proposals, ngram_proposals;
    double avg_match_len;
    size_t active_requests, active_context_tokens;
    uint64_t native_ns, total_ns;
  };
  Stats stats() const;

 private:
  struct Row {
    std::vector<int64_t> ctx;
    NgramIndex index;
    bool taken = false;
  };
  std::shared_ptr<SharedCorpus> corpus_;
  std::vector<Row> rows_;
  size_t k_, max_model_len_, max_rows_;
  size_t ngram_min_, ngram_max_, ngram_window_;
  bool use_ngram_;
  uint64_t calls_ = 0, proposed_ = 0, suffix_proposals_ = 0, ngram_proposals_ = 0, match_sum_ = 0;
  uint64_t native_ns_ = 0, total_ns_ = 0, log_interval_, stats_interval_;
};

}  // namespace sh
