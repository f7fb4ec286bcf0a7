#include "mixer.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <unordered_set>

namespace sh {

namespace {
constexpr size_t kBoundary = 64;

inline size_t sat_sub(size_t a, size_t b) { return a > b ? a - b : 0; }

inline uint64_t now_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}

inline size_t div_bucket(bool self_lookup, size_t matched) {
  const size_t tier = matched < 16 ? 0 : (matched < 32 ? 1 : 2);
  return tier + (self_lookup ? 3 : 0);
}
}  // namespace

HybridMixer::HybridMixer(size_t k, size_t max_model_len) {
  if (k < 1 || k > 64 || max_model_len < 1 || max_model_len > 16777216)
    throw ValueError("hybrid budget must be 1..64 and context 1..16777216");
  corpus_ = std::make_shared<SharedCorpus>(CacheConfig::from_env());
  k_ = k;
  max_model_len_ = max_model_len;
  initial_ = k;
  std::string split = env_string("SPLIT");
  // trim
  const auto b = split.find_first_not_of(" \t\r\n");
  const auto e = split.find_last_not_of(" \t\r\n");
  split = b == std::string::npos ? std::string() : split.substr(b, e - b + 1);
  diverge_ = split == "diverge";
  div_threshold_ = std::clamp(env_double("DIVERGE_THRESHOLD", 0.5), 0.0, 1.0);
  self_lo_ = env_size("SELF_NGRAM_MIN", 4, 1, 128);
  self_hi_ = env_size("SELF_NGRAM_MAX", 16, 1, 128);
  self_window_ = env_size("SELF_NGRAM_WINDOW", 8192, 0, 16777216);
}

size_t HybridMixer::cache_tokens() const {
  std::lock_guard<std::mutex> lock(corpus_->mu);
  return corpus_->corpus.cached_tokens();
}

void HybridMixer::validate(const std::vector<std::string_view>& ids, const std::vector<std::vector<int64_t>>& native,
                           const std::vector<int64_t>* accepted) {
  const size_t n = ids.size();
  bool bad = n > 4096 || native.size() != n || (accepted && accepted->size() != n);
  if (!bad && n > 1) {
    // Duplicate ids: sort 64-bit hashes, compare strings only on equal hash.
    std::vector<std::pair<size_t, size_t>>& hs = hashes_;
    hs.resize(n);
    for (size_t i = 0; i < n; ++i) hs[i] = {StrHash{}(ids[i]), i};
    std::sort(hs.begin(), hs.end());
    for (size_t i = 1; i < n && !bad; ++i)
      for (size_t j = i; j > 0 && hs[j - 1].first == hs[i].first; --j)
        if (ids[hs[j - 1].second] == ids[hs[i].second]) {
          bad = true;
          break;
        }
  }
  if (!bad)
    for (const auto& d : native) {
      if (d.size() > k_) {
        bad = true;
        break;
      }
      for (int64_t t : d)
        if (t < 0) {
          bad = true;
          break;
        }
      if (bad) break;
    }
  if (bad) throw ValueError("invalid hybrid batch dimensions, IDs, token IDs or budget");
  // Reserve before looking up so inserts later in the call never rehash and
  // the cached iterators stay valid.
  previous_.reserve(previous_.size() + n);
  found_.resize(n);
  for (size_t i = 0; i < n; ++i) found_[i] = previous_.find(ids[i]);
  if (accepted) {
    for (size_t i = 0; i < n; ++i) {
      const int64_t a = (*accepted)[i];
      if (a < -1) throw ValueError("accepted length exceeds previous proposal");
      if (found_[i] != previous_.end() && a > static_cast<int64_t>(found_[i]->second.length))
        throw ValueError("accepted length exceeds previous proposal");
    }
  }
}

template <class Decide>
std::pair<std::vector<int64_t>, size_t> HybridMixer::diverge_row(SuffixCorpus& cache, std::string_view id, size_t i,
                                                                 const std::vector<int64_t>& native,
                                                                 int64_t accepted, Decide&& decide) {
  auto it = previous_.find(id);
  std::vector<int64_t> delta;
  const Continuity c = decide(i, it == previous_.end() ? nullptr : &it->second.context, delta);
  Previous* p;
  if (it != previous_.end()) {
    p = &it->second;
    if (c == Continuity::Continuing) {
      if (p->has_div) {
        const Divergence d = p->div;
        p->has_div = false;
        // delta[:a] are the accepted drafts and delta[a] the bonus token, so
        // the verified token at j is known iff j <= a.
        if (accepted >= static_cast<int64_t>(d.j) && delta.size() > d.j) {
          const int64_t truth = delta[d.j];
          double* w = div_wins_[d.bucket];
          w[0] *= 0.999;
          w[1] *= 0.999;
          w[0] += truth == d.suffix_tok ? 1.0 : 0.0;
          w[1] += truth == d.native_tok ? 1.0 : 0.0;
          ++div_observed_;
        }
      }
      p->context.insert(p->context.end(), delta.begin(), delta.end());
    } else {
      cache.add(p->context);
      p->context = std::move(delta);
      p->has_div = false;
      p->self_index.reset();
    }
  } else {
    Previous fresh;
    fresh.context = std::move(delta);
    fresh.accept_estimate = static_cast<double>(initial_);
    fresh.self_index = NgramIndex(self_lo_);
    fresh.order = order_++;
    fresh.stamp = calls_ + 1;
    p = &previous_.emplace(std::string(id), std::move(fresh)).first->second;
  }
  const std::vector<int64_t>& ctx = p->context;
  const size_t cap = std::min({k_, sat_sub(max_model_len_, ctx.size()), native.size()});
  SpecResult sr = cache.speculate(ctx.data(), ctx.size(), cap);
  std::vector<int64_t> cand = std::move(sr.tokens);
  size_t matched = sr.match_len;
  bool self_lookup = false;
  if (cand.size() < cap && self_hi_ >= self_lo_) {
    NgramResult ng = p->self_index.query(ctx.data(), ctx.size(), self_hi_, cap, self_window_);
    const size_t order = ng.score > 0.0 ? static_cast<size_t>(std::llround(ng.score / (1.0 - ng.score))) : 0;
    if (ng.tokens.size() > cand.size() || (!ng.tokens.empty() && order > matched)) {
      cand = std::move(ng.tokens);
      matched = order;
      self_lookup = true;
      ++self_hits_;
    }
  }
  if (cand.size() > cap) cand.resize(cap);
  std::vector<int64_t> draft(native.begin(), native.begin() + cap);
  size_t native_count = cap;
  p->has_div = false;
  for (size_t j = 0; j < cand.size(); ++j) {
    if (cand[j] == native[j]) continue;
    const size_t bucket = div_bucket(self_lookup, matched);
    p->div = Divergence{j, cand[j], native[j], bucket};
    p->has_div = true;
    if (trust(div_wins_[bucket]) > div_threshold_) {
      std::copy(cand.begin(), cand.end(), draft.begin());
      native_count = j;
      ++div_suffix_published_;
      suffix_proposed_ += cand.size() - j;
    }
    break;
  }
  native_proposed_ += native_count;
  p->native = native_count;
  p->length = draft.size();
  p->arm = cap;
  p->had_suffix = native_count < cap;
  return {std::move(draft), native_count};
}

template <class Decide>
const std::vector<std::vector<int64_t>>& HybridMixer::mix_core(const std::vector<std::string_view>& ids,
                                                        const std::vector<std::vector<int64_t>>& native,
                                                        const std::vector<int64_t>* accepted, Decide&& decide) {
  const uint64_t start = now_ns();
  const size_t n = ids.size();
  const uint64_t stamp = calls_ + 1;
  // found_ was filled by validate(): one lookup per row for the whole call.
  for (size_t i = 0; i < n; ++i)
    if (found_[i] != previous_.end()) found_[i]->second.stamp = stamp;
  // 1) Feedback: exactly one rejected position is tested, the rest censored.
  if (accepted) {
    for (size_t i = 0; i < n; ++i) {
      const int64_t a = (*accepted)[i];
      if (a < 0) continue;
      auto it = found_[i];
      if (it == previous_.end()) continue;
      Previous& p = it->second;
      const size_t acc = static_cast<size_t>(a);
      const size_t tested = std::min(acc + 1, p.length);
      native_tested_ += std::min(tested, p.native);
      native_accepted_ += std::min(acc, p.native);
      suffix_tested_ += sat_sub(tested, p.native);
      suffix_accepted_ += sat_sub(acc, p.native);
      if (p.length > 0) {
        // Full acceptance jumps back to the published width; a partial one
        // decays the estimate (censored tails never train it down).
        p.accept_estimate = acc >= p.length ? static_cast<double>(p.length) : 0.7 * p.accept_estimate + 0.3 * acc;
        // The suffix gate trains only on proposals that carried a non-native
        // tail and were rejected inside the native prefix.
        if (p.had_suffix && acc < p.native) {
          const double got = static_cast<double>(sat_sub(acc, p.native));
          p.gate = p.has_gate ? 0.7 * p.gate + 0.3 * got : got;
          p.has_gate = true;
        }
      }
    }
  }
  std::lock_guard<std::mutex> lock(corpus_->mu);
  SuffixCorpus& cache = corpus_->corpus;
  // 2) Rows absent from this batch are finalized into the corpus, in the
  // order they were first seen (deterministic corpus ids).
  if (previous_.size() > n || n == 0) {
    std::vector<std::pair<uint64_t, Table::iterator>> gone;
    for (auto it = previous_.begin(); it != previous_.end(); ++it)
      if (it->second.stamp != stamp) gone.emplace_back(it->second.order, it);
    std::sort(gone.begin(), gone.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    for (auto& g : gone) {
      cache.add(g.second->second.context);
      previous_.erase(g.second);
    }
  }
  last_native_.clear();
  std::vector<std::vector<int64_t>>& result = result_;
  result.resize(n);  // inner vectors keep their capacity from earlier calls
  const size_t depth = cache.cfg().depth;
  std::vector<int64_t>& delta = delta_;
  for (size_t i = 0; i < n; ++i) {
    const std::vector<int64_t>& nat = native[i];
    if (diverge_) {
      const int64_t a = accepted ? (*accepted)[i] : -1;
      auto dr = diverge_row(cache, ids[i], i, nat, a, decide);
      last_native_.push_back(dr.second);
      result[i] = std::move(dr.first);
      ++decisions_;
      continue;
    }
    auto it = found_[i];
    const bool occupied = it != previous_.end();
    delta.clear();
    const Continuity c = decide(i, occupied ? &it->second.context : nullptr, delta);
    if (c == Continuity::Reset && occupied) {
      // A different request reuses the slot: finalize the old history
      // before this row's lookup (the new request may continue it).
      cache.add(it->second.context);
      it->second.context.clear();
    }
    const bool continuing = occupied && c == Continuity::Continuing;
    const bool fresh_row = !occupied || c == Continuity::Reset;
    const size_t context_len = continuing ? it->second.context.size() + delta.size() : delta.size();
    const size_t cap = std::min({k_, sat_sub(max_model_len_, context_len), nat.size()});
    const bool has_est = continuing;
    const double est = has_est ? it->second.accept_estimate : 0.0;
    const bool fed = cache.cached_tokens() > 0;
    size_t budget = cap;
    if (fed) {
      const double v = has_est ? est : static_cast<double>(initial_);
      const double cv = std::ceil(v);
      size_t b = cv <= 0.0 ? 0 : static_cast<size_t>(cv);
      b = std::clamp<size_t>(b, 1, k_);
      budget = std::min(b, cap);
    }
    const size_t floor_ = std::max<size_t>(sat_sub(cap, 1), 1);
    size_t prefix = cap;
    if (occupied && c != Continuity::Reset) {
      const size_t b = std::min(budget, cap);
      prefix = b >= cap ? cap : std::max(b, floor_);
    }
    // Lookup key: the last `depth` tokens of context + native[:prefix-1].
    conditioned_.clear();
    if (continuing) {
      const std::vector<int64_t>& pc = it->second.context;
      const size_t take = std::min(sat_sub(depth, delta.size()), pc.size());
      conditioned_.insert(conditioned_.end(), pc.end() - take, pc.end());
    }
    const size_t dskip = sat_sub(delta.size(), depth);
    conditioned_.insert(conditioned_.end(), delta.begin() + dskip, delta.end());
    conditioned_.insert(conditioned_.end(), nat.begin(), nat.begin() + sat_sub(prefix, 1));
    SpecResult sr = cache.speculate(conditioned_.data(), conditioned_.size(), cap);
    const bool has_gate = occupied && it->second.has_gate;
    const double gate = has_gate ? it->second.gate : 0.0;
    std::vector<int64_t>& draft = result[i];
    size_t native_count;
    bool had_suffix;
    if (sr.tokens.empty() || fresh_row) {
      draft.assign(nat.begin(), nat.begin() + cap);
      native_count = cap;
      had_suffix = false;
    } else {
      const size_t keep_prefix = sat_sub(prefix, 1);
      const std::vector<int64_t>& tail = sr.tokens;
      const size_t dropped = prefix - keep_prefix;
      const bool replaces = prefix > keep_prefix && tail.size() >= dropped && (!has_gate || gate >= 1.0);
      if (replaces) {
        draft.assign(nat.begin(), nat.begin() + keep_prefix);
        draft.insert(draft.end(), tail.begin(), tail.end());
      } else {
        // Gate closed (or short tail): extension only, never overwrite.
        draft.assign(nat.begin(), nat.begin() + prefix);
        const size_t room = sat_sub(cap, draft.size());
        draft.insert(draft.end(), tail.begin(), tail.begin() + std::min(room, tail.size()));
      }
      const size_t keep = std::min(draft.size(), cap);
      draft.resize(keep);
      size_t nc = std::min(keep_prefix, keep);
      while (nc < keep && nc < nat.size() && draft[nc] == nat[nc]) ++nc;
      native_count = nc;
      had_suffix = draft.size() > nc;
    }
    native_proposed_ += native_count;
    suffix_proposed_ += sat_sub(draft.size(), native_count);
    last_native_.push_back(native_count);
    const bool seed = !has_est;
    const double ae = (occupied && !seed) ? it->second.accept_estimate : static_cast<double>(initial_);
    const bool hg = (occupied && !seed) ? it->second.has_gate : false;
    const double g = (occupied && !seed) ? it->second.gate : 0.0;
    if (occupied) {
      Previous& p = it->second;
      if (c == Continuity::Continuing) {
        p.context.insert(p.context.end(), delta.begin(), delta.end());
      } else {
        cache.add(p.context);  // already emptied above on Reset
        p.context.assign(delta.begin(), delta.end());
        p.self_index.reset();
      }
      p.native = native_count;
      p.length = draft.size();
      p.arm = budget;
      p.accept_estimate = ae;
      p.has_gate = hg;
      p.gate = g;
      p.had_suffix = had_suffix;
    } else {
      Previous fresh;
      fresh.context.assign(delta.begin(), delta.end());
      fresh.native = native_count;
      fresh.length = draft.size();
      fresh.arm = budget;
      fresh.accept_estimate = ae;
      fresh.has_gate = hg;
      fresh.gate = g;
      fresh.had_suffix = had_suffix;
      fresh.self_index = NgramIndex(self_lo_);
      fresh.order = order_++;
      fresh.stamp = stamp;
      previous_.emplace(std::string(ids[i]), std::move(fresh));
    }
    ++decisions_;
  }
  ++calls_;
  elapsed_ns_ += now_ns() - start;
  return result;
}

const std::vector<std::vector<int64_t>>& HybridMixer::mix(const std::vector<std::string_view>& ids,
                                                   const std::vector<std::vector<int64_t>>& contexts,
                                                   const std::vector<std::vector<int64_t>>& native,
                                                   const std::vector<int64_t>* accepted) {
  validate(ids, native, accepted);
  if (contexts.size() != ids.size()) throw ValueError("invalid hybrid batch dimensions, IDs, token IDs or budget");
  for (const auto& c : contexts)
    if (c.size() > max_model_len_) throw ValueError("invalid hybrid batch dimensions, IDs, token IDs or budget");
  auto decide = [&](size_t i, const std::vector<int64_t>* tracked, std::vector<int64_t>& delta) -> Continuity {
    const std::vector<int64_t>& ctx = contexts[i];
    if (!tracked) {
      delta.assign(ctx.begin(), ctx.end());
      return Continuity::Fresh;
    }
    if (ctx.size() >= tracked->size() && std::equal(tracked->begin(), tracked->end(), ctx.begin())) {
      delta.assign(ctx.begin() + tracked->size(), ctx.end());
      return Continuity::Continuing;
    }
    delta.assign(ctx.begin(), ctx.end());
    return Continuity::Reset;
  };
  return mix_core(ids, native, accepted, decide);
}

const std::vector<std::vector<int64_t>>& HybridMixer::mix_matrix(const std::vector<std::string_view>& ids,
                                                          const IntVector& counts, const IntMatrix& tokens,
                                                          const std::vector<std::vector<int64_t>>& native,
                                                          const std::vector<int64_t>* accepted) {
  validate(ids, native, accepted);
  const size_t n = ids.size();
  if (counts.n < n) throw ValueError("missing counts");
  if (tokens.rows < n) throw ValueError("invalid row bounds");
  for (size_t i = 0; i < n; ++i) {
    const int64_t c = counts.at(i);
    if (c < 0 || static_cast<size_t>(c) > tokens.cols || static_cast<size_t>(c) > max_model_len_)
      throw ValueError("invalid row bounds");
  }
  auto decide = [&](size_t i, const std::vector<int64_t>* tracked, std::vector<int64_t>& delta) -> Continuity {
    const size_t count = static_cast<size_t>(counts.at(i));
    const int64_t* fast = tokens.row64(i);
    auto copy = [&](size_t from) {
      if (fast) {
        delta.assign(fast + from, fast + count);
      } else {
        delta.clear();
        delta.reserve(count - from);
        for (size_t j = from; j < count; ++j) delta.push_back(tokens.at(i, j));
      }
    };
    if (!tracked) {
      copy(0);
      return Continuity::Fresh;
    }
    const size_t l = tracked->size();
    bool cont = count >= l;
    if (cont) {
      const size_t w = std::min(kBoundary, l);
      if (fast) {
        cont = std::equal(tracked->begin(), tracked->begin() + w, fast) &&
               std::equal(tracked->end() - w, tracked->end(), fast + (l - w));
      } else {
        for (size_t j = 0; j < w && cont; ++j) cont = (*tracked)[j] == tokens.at(i, j);
        for (size_t j = l - w; j < l && cont; ++j) cont = (*tracked)[j] == tokens.at(i, j);
      }
    }
    if (cont) {
      copy(l);
      return Continuity::Continuing;
    }
    copy(0);
    return Continuity::Reset;
  };
  return mix_core(ids, native, accepted, decide);
}

HybridMixer::Stats HybridMixer::stats() const {
  Stats s{};
  s.calls = calls_;
  s.native_tested = native_tested_;
  s.native_accepted = native_accepted_;
  s.suffix_tested = suffix_tested_;
  s.suffix_accepted = suffix_accepted_;
  s.native_proposed = native_proposed_;
  s.suffix_proposed = suffix_proposed_;
  s.elapsed_ns = elapsed_ns_;
  double sum = 0.0;
  for (const auto& kv : previous_) sum += kv.second.accept_estimate;
  s.mean_accept_estimate = previous_.empty() ? 0.0 : sum / static_cast<double>(previous_.size());
  s.active_tracked = previous_.size();
  s.diverge = diverge_;
  s.div_observed = div_observed_;
  s.div_suffix_published = div_suffix_published_;
  s.self_hits = self_hits_;
  for (size_t b = 0; b < kBuckets; ++b) s.div_trust.push_back(trust(div_wins_[b]));
  return s;
}

}  // namespace sh
