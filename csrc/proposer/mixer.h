// Hybrid native/suffix draft mixer.
//
// One coherent chain per request: a native-drafter prefix followed by a
// suffix-corpus tail conditioned on that prefix.  Verified accepted lengths
// train a per-request acceptance EWMA (the native budget) and a suffix gate.
// Behaviour follows the reference's mixer (reference: src/mixer.rs:82-888):
//  * legacy split (default): budget = ceil(EWMA) in [1, k]; native prefix
//    floored at cap-1 unless the row is at full budget; the corpus lookup is
//    keyed on context + native[:prefix-1]; the suffix tail replaces the
//    unearned native tail while the gate is open, else only appends;
//  * SUFFIX_HYBRID_SPLIT=diverge: the candidate (corpus, else in-request
//    n-gram) is compared with the native draft; at the first disagreement a
//    per-evidence-bucket Laplace trust decides which source continues, and
//    the next step's verified token grades both sources.
// Rows absent from a call are finalized into the shared corpus.
#pragma once
#include <memory>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "ngram.h"
#include "suffix_cache.h"
#include "views.h"

namespace sh {

struct StrHash {
  using is_transparent = void;
  size_t operator()(std::string_view s) const noexcept { return std::hash<std::string_view>{}(s); }
};

enum class Continuity { Fresh, Continuing, Reset };

class HybridMixer {
 public:
  HybridMixer(size_t num_speculative_tokens, size_t max_model_len);

  // List API: full authoritative contexts, exact prefix continuity.  The
  // returned drafts live in the mixer (reused by the next call).
  const std::vector<std::vector<int64_t>>& mix(const std::vector<std::string_view>& ids,
                                        const std::vector<std::vector<int64_t>>& contexts,
                                        const std::vector<std::vector<int64_t>>& native,
                                        const std::vector<int64_t>* accepted);
  // Buffer API: rows read from a CPU token matrix, continuity proven with
  // 64-token head/tail windows; only the delta is copied.
  const std::vector<std::vector<int64_t>>& mix_matrix(const std::vector<std::string_view>& ids, const IntVector& counts,
                                               const IntMatrix& tokens,
                                               const std::vector<std::vector<int64_t>>& native,
                                               const std::vector<int64_t>* accepted);

  const std::vector<size_t>& last_native_counts() const { return last_native_; }
  size_t cache_tokens() const;
  std::shared_ptr<SharedCorpus> corpus() const { return corpus_; }

  struct Stats {
    uint64_t calls, native_tested, native_accepted, suffix_tested, suffix_accepted, native_proposed,
        suffix_proposed, elapsed_ns;
    double mean_accept_estimate;
    size_t active_tracked;
    bool diverge;
    uint64_t div_observed, div_suffix_published, self_hits;
    std::vector<double> div_trust;
  };
  Stats stats() const;

 private:
  static constexpr size_t kBuckets = 6;
  struct Divergence {
    size_t j;
    int64_t suffix_tok, native_tok;
    size_t bucket;
  };
  struct Previous {
    std::vector<int64_t> context;
    size_t native = 0, length = 0, arm = 0;
    double accept_estimate = 0.0;
    bool has_gate = false;
    double gate = 0.0;  // suffix_estimate
    bool had_suffix = false;
    bool has_div = false;
    Divergence div{};
    NgramIndex self_index;
    uint64_t order = 0;  // first-seen order: deterministic ingestion
    uint64_t stamp = 0;  // last call that saw this row
  };
  using Table = std::unordered_map<std::string, Previous, StrHash, std::equal_to<>>;

  // Looks every id up once (filling found_) and rejects a bad batch before
  // any state changes.
  void validate(const std::vector<std::string_view>& ids, const std::vector<std::vector<int64_t>>& native,
                const std::vector<int64_t>* accepted);
  template <class Decide>
  const std::vector<std::vector<int64_t>>& mix_core(const std::vector<std::string_view>& ids,
                                             const std::vector<std::vector<int64_t>>& native,
                                             const std::vector<int64_t>* accepted, Decide&& decide);
  template <class Decide>
  std::pair<std::vector<int64_t>, size_t> diverge_row(SuffixCorpus& cache, std::string_view id, size_t i,
                                                      const std::vector<int64_t>& native, int64_t accepted,
                                                      Decide&& decide);
  static double trust(const double* w) { return (w[0] + 1.0) / (w[0] + w[1] + 2.0); }

  std::shared_ptr<SharedCorpus> corpus_;
  Table previous_;
  size_t k_, max_model_len_, initial_;
  uint64_t calls_ = 0, decisions_ = 0, order_ = 0;
  std::vector<size_t> last_native_;
  uint64_t native_tested_ = 0, native_accepted_ = 0, suffix_tested_ = 0, suffix_accepted_ = 0;
  uint64_t native_proposed_ = 0, suffix_proposed_ = 0, elapsed_ns_ = 0;
  bool diverge_;
  double div_threshold_;
  size_t self_lo_, self_hi_, self_window_;
  double div_wins_[kBuckets][2] = {};
  uint64_t div_observed_ = 0, div_suffix_published_ = 0, self_hits_ = 0;
  std::vector<int64_t> conditioned_;
  std::vector<Table::iterator> found_;
  // Per-call scratch kept across calls (no allocation once warm).
  std::vector<std::vector<int64_t>> result_;
  std::vector<int64_t> delta_;
  std::vector<std::pair<size_t, size_t>> hashes_;
};

}  // namespace sh
