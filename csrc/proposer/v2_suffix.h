// Drafter-free suffix-only proposer over a zero-copy token buffer.
//
// Per request it mirrors the full token history (fresh rows copy once,
// continuing rows prove continuity with 64-token boundary windows and append
// only the delta), drafts from the shared corpus, ingests departed rows
// (longer than 8 tokens), and publishes ragged widths or a uniform-k pallet
// padded with the row's first (always in-vocabulary) token.  An optional
// acceptance-EWMA width gate narrows the publish toward what the row wins.
// Behaviour follows the reference (reference: src/mixer.rs:912-1376).
#pragma once
#include <memory>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "mixer.h"
#include "suffix_cache.h"
#include "views.h"

namespace sh {

class V2SuffixProposer {
 public:
  V2SuffixProposer(size_t k, size_t max_model_len, size_t min_len, bool uniform_k, bool width_gate);

  // Fills packed [n, k] (row-major, zero padded) and widths [n].
  void propose(const std::vector<std::string_view>& ids, const std::vector<int64_t>& indices, const IntVector& totals,
               const IntMatrix& tokens, std::vector<int64_t>* packed, std::vector<int64_t>* widths);
  void clear_widths();
  void add_elapsed(uint64_t ns) { elapsed_ns_ += ns; }

  std::vector<std::pair<std::string, size_t>> widths_table() const;
  std::vector<std::pair<std::string, std::pair<double, size_t>>> gate_table() const;
  std::shared_ptr<SharedCorpus> corpus() const { return corpus_; }
  size_t k() const { return k_; }

  struct Stats {
    uint64_t steps, hits, hit_tokens, ingested, resets, padded;
    bool uniform_k, width_gate;
    size_t active;
    uint64_t elapsed_ns;
  };
  Stats stats() const;

 private:
  struct GateRow {
    double ewma;
    size_t last_width;
  };
  struct Mirror {
    std::vector<int64_t> tokens;
    uint64_t order;
  };
  std::shared_ptr<SharedCorpus> corpus_;
  std::unordered_map<std::string, Mirror, StrHash, std::equal_to<>> mirror_;
  std::unordered_map<std::string, size_t, StrHash, std::equal_to<>> widths_;
  std::unordered_map<std::string, GateRow, StrHash, std::equal_to<>> gate_;
  size_t k_, max_model_len_, min_len_;
  bool uniform_k_, width_gate_;
  uint64_t steps_ = 0, hits_ = 0, hit_tokens_ = 0, ingested_ = 0, resets_ = 0, padded_ = 0, elapsed_ns_ = 0;
  uint64_t order_ = 0;
};

// Greedy verification oracle: accept run + emit mask per request
// (reference: src/verify_fusion.rs:48-113).
void rejection_greedy_accept(const int64_t* draft, const int64_t* argmax, size_t num_tokens, const int64_t* cu,
                             size_t batch, size_t max_spec_len, int32_t* accept_count, int32_t* emit_mask);

}  // namespace sh
