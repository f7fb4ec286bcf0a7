#include "v2_suffix.h"

#include <algorithm>
#include <cmath>
#include <unordered_set>

namespace sh {

namespace {
constexpr size_t kBoundary = 64;
}

V2SuffixProposer::V2SuffixProposer(size_t k, size_t max_model_len, size_t min_len, bool uniform_k, bool width_gate) {
  if (k < 1 || k > 64 || max_model_len < 1 || max_model_len > 16777216)
    throw ValueError("suffix-only k must be 1..64 and context 1..16777216");
  corpus_ = std::make_shared<SharedCorpus>(CacheConfig::from_env());
  k_ = k;
  max_model_len_ = max_model_len;
  min_len_ = std::max<size_t>(min_len, 1);
  uniform_k_ = uniform_k;
  width_gate_ = width_gate;
}

void V2SuffixProposer::propose(const std::vector<std::string_view>& ids, const std::vector<int64_t>& indices,
                               const IntVector& totals, const IntMatrix& tokens, std::vector<int64_t>* packed,
                               std::vector<int64_t>* widths) {
  const size_t n = ids.size();
  if (indices.size() < n) throw ValueError("suffix-only batch dimension mismatch");
  if (totals.n < n) throw ValueError("totals shorter than request ids");
  for (size_t i = 0; i < n; ++i) {
    const int64_t t = totals.at(i);
    if (t < 0 || static_cast<size_t>(t) > tokens.cols || static_cast<size_t>(t) > max_model_len_)
      throw ValueError("suffix-only row bounds");
    const size_t r = static_cast<size_t>(std::max<int64_t>(indices[i], 0));
    if (r >= tokens.rows) throw ValueError("suffix-only row index outside the token buffer");
  }
  packed->assign(n * k_, 0);
  widths->assign(n, 0);
  // 1) Departed rows donate their full history (prompt + generation).
  {
    std::unordered_set<std::string_view> live(ids.begin(), ids.end());
    std::vector<std::pair<uint64_t, std::string>> gone;
    for (const auto& kv : mirror_)
      if (!live.count(kv.first)) gone.emplace_back(kv.second.order, kv.first);
    std::sort(gone.begin(), gone.end());
    for (auto& g : gone) {
      auto it = mirror_.find(g.second);
      widths_.erase(g.second);
      gate_.erase(g.second);
      if (it->second.tokens.size() > 8) {
        std::lock_guard<std::mutex> lock(corpus_->mu);
        corpus_->corpus.add(it->second.tokens);
        ++ingested_;
      }
      mirror_.erase(it);
    }
  }
  // 2) Per row: continuity proof, in-place extend, corpus lookup.
  uint64_t padded_now = 0;
  for (size_t i = 0; i < n; ++i) {
    const std::string_view rid = ids[i];
    const size_t total = static_cast<size_t>(totals.at(i));
    const size_t r = static_cast<size_t>(std::max<int64_t>(indices[i], 0));
    const int64_t* fast = tokens.row64(r);
    auto tok_at = [&](size_t j) { return fast ? fast[j] : tokens.at(r, j); };
    auto it = mirror_.find(rid);
    const bool tracked = it != mirror_.end();
    const size_t tracked_len = tracked ? it->second.tokens.size() : 0;
    bool cont = false;
    if (tracked && total >= tracked_len) {
      const std::vector<int64_t>& t = it->second.tokens;
      const size_t l = t.size();
      const size_t w = std::min(kBoundary, l);
      cont = true;
      for (size_t j = 0; j < w && cont; ++j) cont = t[j] == tok_at(j);
      for (size_t j = l - w; j < l && cont; ++j) cont = t[j] == tok_at(j);
    }
    if (cont) {
      std::vector<int64_t>& t = it->second.tokens;
      for (size_t j = t.size(); j < total; ++j) t.push_back(tok_at(j));
    } else {
      if (tracked) ++resets_;
      std::vector<int64_t> fresh;
      fresh.reserve(total);
      for (size_t j = 0; j < total; ++j) fresh.push_back(tok_at(j));
      if (tracked) {
        it->second.tokens = std::move(fresh);
      } else {
        it = mirror_.emplace(std::string(rid), Mirror{std::move(fresh), order_++}).first;
      }
    }
    const std::vector<int64_t>& row = it->second.tokens;
    const int64_t pad = row.empty() ? 0 : row.front();
    SpecResult sr;
    {
      std::lock_guard<std::mutex> lock(corpus_->mu);
      sr = corpus_->corpus.speculate(row.data(), row.size(), k_);
    }
    std::vector<int64_t> out;
    size_t real_w = 0;
    if (!sr.tokens.empty() && sr.tokens.size() >= min_len_) {
      real_w = std::min(sr.tokens.size(), k_);
      out.assign(sr.tokens.begin(), sr.tokens.begin() + real_w);
    }
    if (width_gate_) {
      // Feedback: on a continuing row the total grew by (accepted drafts + 1
      // sampled token) since the last view; retracted publishes (last_width
      // 0) and non-steps are censored.
      size_t gate_w = k_;
      bool have = false;
      double ewma = 0.0;
      auto g = gate_.find(rid);
      if (g != gate_.end()) {
        if (cont && g->second.last_width > 0 && tracked) {
          const size_t delta = total - tracked_len;
          if (delta >= 1) {
            const size_t a = std::min(delta - 1, g->second.last_width);
            g->second.ewma = a >= g->second.last_width ? static_cast<double>(g->second.last_width + 1)
                                                       : 0.7 * g->second.ewma + 0.3 * static_cast<double>(a);
          }
        }
        const double c = std::ceil(g->second.ewma);
        gate_w = std::clamp<size_t>(c <= 0 ? 0 : static_cast<size_t>(c), 1, k_);
        have = true;
        ewma = g->second.ewma;
      }
      if (gate_w < real_w) {
        out.resize(gate_w);
        real_w = gate_w;
      }
      const size_t last_width = uniform_k_ ? k_ : real_w;
      if (g != gate_.end()) {
        g->second.last_width = last_width;
      } else {
        gate_.emplace(std::string(rid), GateRow{have ? ewma : static_cast<double>(k_), last_width});
      }
    }
    size_t width = real_w;
    if (uniform_k_) {
      while (out.size() < k_) out.push_back(pad);
      width = k_;
    }
    if (real_w > 0) {
      ++hits_;
      hit_tokens_ += real_w;
    }
    auto w = widths_.find(rid);
    if (w != widths_.end())
      w->second = width;
    else
      widths_.emplace(std::string(rid), width);
    if (uniform_k_ && real_w < width) ++padded_now;
    (*widths)[i] = static_cast<int64_t>(width);
    for (size_t j = 0; j < out.size() && j < k_; ++j) (*packed)[i * k_ + j] = out[j];
  }
  ++steps_;
  padded_ += padded_now;
}

void V2SuffixProposer::clear_widths() {
  for (auto& kv : widths_) {
    kv.second = 0;
    auto g = gate_.find(kv.first);
    if (g != gate_.end()) g->second.last_width = 0;
  }
}

std::vector<std::pair<std::string, size_t>> V2SuffixProposer::widths_table() const {
  return {widths_.begin(), widths_.end()};
}

std::vector<std::pair<std::string, std::pair<double, size_t>>> V2SuffixProposer::gate_table() const {
  std::vector<std::pair<std::string, std::pair<double, size_t>>> out;
  for (const auto& kv : gate_) out.push_back({kv.first, {kv.second.ewma, kv.second.last_width}});
  return out;
}

V2SuffixProposer::Stats V2SuffixProposer::stats() const {
  return Stats{steps_, hits_, hit_tokens_, ingested_, resets_, padded_, uniform_k_, width_gate_, mirror_.size(),
               elapsed_ns_};
}

void rejection_greedy_accept(const int64_t* draft, const int64_t* argmax, size_t num_tokens, const int64_t* cu,
                             size_t batch, size_t max_spec_len, int32_t* accept_count, int32_t* emit_mask) {
  const size_t width = max_spec_len + 1;
  std::fill(emit_mask, emit_mask + batch * width, 0);
  for (size_t b = 0; b < batch; ++b) {
    const size_t start = b == 0 ? 0 : static_cast<size_t>(std::max<int64_t>(cu[b - 1], 0));
    const size_t end = std::min(static_cast<size_t>(std::max<int64_t>(cu[b], 0)), num_tokens);
    const size_t owned = std::min(end > start ? end - start : 0, max_spec_len);
    size_t count = 0;
    while (count < owned) {
      const size_t idx = start + count;
      // A padded (-1) draft or any mismatch ends the accepted run.
      if (draft[idx] >= 0 && draft[idx] == argmax[idx])
        ++count;
      else
        break;
    }
    accept_count[b] = static_cast<int32_t>(count);
    for (size_t p = 0; p <= std::min(count, max_spec_len); ++p) emit_mask[b * width + p] = 1;
  }
}

}  // namespace sh
