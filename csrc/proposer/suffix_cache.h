// Bounded cross-request suffix corpus.
//
// A FIFO of finished token sequences (bounded by count and by total tokens)
// plus an index from every length-n token window to the most recent
// positions where it occurs.  `speculate` looks up the context's last
// n-gram, extends each hit backwards against the context, keeps the set of
// longest matches and majority-votes their continuations step by step.
// Behaviour (knobs, tie-breaks, score, draft cap) follows the reference's
// corpus (reference: src/lib.rs:128-271); the data layout is this project's
// own: a linear-probing table keyed by a rolling window hash whose buckets
// hold (sequence id, position) hits, with sequence storage in a FIFO ring so
// an id resolves by subtraction instead of a second hash lookup.
#pragma once
#include <cstdint>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "config.h"

namespace sh {

struct Hit {
  uint64_t id;
  uint64_t pos;
};

struct SpecResult {
  std::vector<int64_t> tokens;
  double score = 0.0;
  size_t match_len = 0;
};

class SuffixCorpus {
 public:
  explicit SuffixCorpus(CacheConfig cfg);

  // Ingest one finished sequence (copied; long sequences keep their tail).
  void add(const int64_t* data, size_t len);
  void add(const std::vector<int64_t>& v) { add(v.data(), v.size()); }
  // Drafts up to `max_tokens` continuation tokens for `context`.
  SpecResult speculate(const int64_t* context, size_t len, size_t max_tokens) const;
  // Change the index order (test seam); the index is rebuilt for the new n.
  void set_n(size_t n);

  std::map<std::string, size_t> stats() const;
  size_t cached_tokens() const { return tokens_; }
  // The held sequences in FIFO order, oldest first (what a snapshot stores).
  const std::deque<std::vector<int64_t>>& sequences() const { return seqs_; }
  const CacheConfig& cfg() const { return cfg_; }
  CacheConfig& mutable_cfg() { return cfg_; }

 private:
  struct Bucket {
    std::vector<Hit> hits;  // ascending id order; oldest first
  };
  struct Slot {
    uint64_t h = 0;  // 0 = empty
    uint32_t bucket = 0;
  };

  const std::vector<int64_t>& seq(uint64_t id) const { return seqs_[id - first_id_]; }
  void evict_oldest();
  void index_sequence(uint64_t id);
  void rebuild_index();
  // Table operations.
  int64_t find_slot(uint64_t h, const int64_t* key) const;
  uint32_t find_or_insert(uint64_t h, const int64_t* key);
  void erase_slot(size_t slot);
  void grow();
  bool key_equals(const Bucket& b, const int64_t* key) const;

  CacheConfig cfg_;
  std::deque<std::vector<int64_t>> seqs_;  // FIFO: front = oldest = first_id_
  uint64_t first_id_ = 0;
  uint64_t next_id_ = 0;
  size_t tokens_ = 0;

  std::vector<Slot> table_;
  size_t used_ = 0;
  std::vector<Bucket> buckets_;
  std::vector<uint32_t> free_buckets_;
  size_t live_buckets_ = 0;
};

// Thread-safe shared handle: the Python SuffixCache object, Engine, mixer and
// suffix-only proposer all hold the same corpus.
struct SharedCorpus {
  explicit SharedCorpus(CacheConfig c) : corpus(c) {}
  std::mutex mu;
  SuffixCorpus corpus;
};

// Window hashing shared with the in-request n-gram index.
uint64_t window_hash(const int64_t* w, size_t n);

// Corpus snapshot, so the corpus survives a restart.  File layout (little-endian):
//   "SHCORP01" | u32 version (1) | u32 window n at save | u64 sequence count |
//   per sequence: u64 length, length x i64 tokens | u64 FNV-1a 64 of every byte after the magic
// save writes `path`.tmp and renames it over `path` (a crash leaves the old snapshot whole) and returns the
// number of sequences written.  load reads and checks the whole file before it touches the corpus, then adds
// the sequences oldest first through the normal ingest path (the corpus bounds and eviction apply) and
// returns how many it added; a missing, truncated or corrupt file leaves the corpus unchanged and reports
// the reason in *err (return -1).
int64_t save_corpus(const SuffixCorpus& c, const std::string& path, std::string* err);
int64_t load_corpus(SuffixCorpus& c, const std::string& path, std::string* err);

}  // namespace sh
