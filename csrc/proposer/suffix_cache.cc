#include "suffix_cache.h"

#include <cstdio>
#include <cstring>

#include <algorithm>
#include <cmath>
#include <stdexcept>

namespace sh {

namespace {
constexpr uint64_t kBase = 0x9E3779B97F4A7C15ull;  // odd multiplier (golden ratio)

inline uint64_t finalize(uint64_t x) {
  // splitmix64 avalanche step, then reserve 0 for "empty slot".
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x ? x : 1;
}

inline uint64_t poly(const int64_t* w, size_t n) {
  uint64_t h = 0;
  for (size_t i = 0; i < n; ++i) h = h * kBase + static_cast<uint64_t>(w[i]);
  return h;
}

inline uint64_t pow_base(size_t e) {
  uint64_t r = 1;
  for (size_t i = 0; i < e; ++i) r *= kBase;
  return r;
}
}  // namespace

uint64_t window_hash(const int64_t* w, size_t n) { return finalize(poly(w, n)); }

SuffixCorpus::SuffixCorpus(CacheConfig cfg) : cfg_(cfg) { table_.resize(1024); }

bool SuffixCorpus::key_equals(const Bucket& b, const int64_t* key) const {
  const Hit& h = b.hits.front();
  const int64_t* s = seq(h.id).data() + h.pos;
  for (size_t i = 0; i < cfg_.n; ++i)
    if (s[i] != key[i]) return false;
  return true;
}

int64_t SuffixCorpus::find_slot(uint64_t h, const int64_t* key) const {
  const size_t mask = table_.size() - 1;
  for (size_t i = h & mask;; i = (i + 1) & mask) {
    const Slot& s = table_[i];
    if (s.h == 0) return -1;
    if (s.h == h && key_equals(buckets_[s.bucket], key)) return static_cast<int64_t>(i);
  }
}

void SuffixCorpus::grow() {
  std::vector<Slot> old;
  old.swap(table_);
  table_.assign(old.size() * 2, Slot{});
  const size_t mask = table_.size() - 1;
  for (const Slot& s : old) {
    if (s.h == 0) continue;
    size_t i = s.h & mask;
    while (table_[i].h != 0) i = (i + 1) & mask;
    table_[i] = s;
  }
}

uint32_t SuffixCorpus::find_or_insert(uint64_t h, const int64_t* key) {
  if ((used_ + 1) * 2 > table_.size()) grow();
  const size_t mask = table_.size() - 1;
  size_t i = h & mask;
  for (;; i = (i + 1) & mask) {
    Slot& s = table_[i];
    if (s.h == 0) break;
    if (s.h == h && key_equals(buckets_[s.bucket], key)) return s.bucket;
  }
  uint32_t b;
  if (!free_buckets_.empty()) {
    b = free_buckets_.back();
    free_buckets_.pop_back();
  } else {
    b = static_cast<uint32_t>(buckets_.size());
    buckets_.emplace_back();
  }
  table_[i].h = h;
  table_[i].bucket = b;
  ++used_;
  ++live_buckets_;
  return b;
}

void SuffixCorpus::erase_slot(size_t i) {
  // Backward-shift deletion keeps every probe chain gap-free.
  const size_t mask = table_.size() - 1;
  size_t j = i;
  for (;;) {
    j = (j + 1) & mask;
    if (table_[j].h == 0) break;
    const size_t home = table_[j].h & mask;
    const bool movable = (j > i) ? (home <= i || home > j) : (home <= i && home > j);
    if (movable) {
      table_[i] = table_[j];
      i = j;
    }
  }
  table_[i] = Slot{};
  --used_;
}

void SuffixCorpus::index_sequence(uint64_t id) {
  const std::vector<int64_t>& s = seq(id);
  const size_t n = cfg_.n;
  if (s.size() < n) return;
  const uint64_t top = pow_base(n - 1);
  uint64_t raw = poly(s.data(), n);
  for (size_t pos = 0; pos + n <= s.size(); ++pos) {
    if (pos > 0) raw = (raw - static_cast<uint64_t>(s[pos - 1]) * top) * kBase + static_cast<uint64_t>(s[pos + n - 1]);
    const uint64_t h = finalize(raw);
    Bucket& b = buckets_[find_or_insert(h, s.data() + pos)];
    b.hits.push_back(Hit{id, pos});
    if (b.hits.size() > cfg_.positions) b.hits.erase(b.hits.begin());
  }
}

void SuffixCorpus::evict_oldest() {
  if (seqs_.empty()) return;
  const uint64_t id = first_id_;
  const std::vector<int64_t>& s = seqs_.front();
  const size_t n = cfg_.n;
  if (s.size() >= n) {
    const uint64_t top = pow_base(n - 1);
    uint64_t raw = poly(s.data(), n);
    for (size_t pos = 0; pos + n <= s.size(); ++pos) {
      if (pos > 0) raw = (raw - static_cast<uint64_t>(s[pos - 1]) * top) * kBase + static_cast<uint64_t>(s[pos + n - 1]);
      const int64_t slot = find_slot(finalize(raw), s.data() + pos);
      if (slot < 0) continue;  // already removed by an earlier window
      Bucket& b = buckets_[table_[slot].bucket];
      // Hits are in ascending id order, so this sequence's hits lead.
      size_t k = 0;
      while (k < b.hits.size() && b.hits[k].id == id) ++k;
      if (k) b.hits.erase(b.hits.begin(), b.hits.begin() + k);
      if (b.hits.empty()) {
        const uint32_t bi = table_[slot].bucket;
        erase_slot(static_cast<size_t>(slot));
        buckets_[bi].hits = std::vector<Hit>();
        free_buckets_.push_back(bi);
        --live_buckets_;
      }
    }
  }
  tokens_ -= s.size();
  seqs_.pop_front();
  ++first_id_;
}

void SuffixCorpus::add(const int64_t* data, size_t len) {
  if (cfg_.sequences == 0 || cfg_.tokens <= cfg_.n) return;
  if (len > cfg_.tokens) {  // keep the most recent tail
    data += len - cfg_.tokens;
    len = cfg_.tokens;
  }
  if (len <= cfg_.n) return;
  while (seqs_.size() >= cfg_.sequences || tokens_ + len > cfg_.tokens) evict_oldest();
  if (seqs_.empty()) first_id_ = next_id_;
  seqs_.emplace_back(data, data + len);  // capacity == length
  const uint64_t id = next_id_++;
  tokens_ += len;
  index_sequence(id);
}

void SuffixCorpus::rebuild_index() {
  table_.assign(1024, Slot{});
  used_ = 0;
  buckets_.clear();
  free_buckets_.clear();
  live_buckets_ = 0;
  for (uint64_t id = first_id_; id < next_id_; ++id) index_sequence(id);
}

void SuffixCorpus::set_n(size_t n) {
  n = std::clamp<size_t>(n, 1, 128);
  if (n == cfg_.n) return;
  cfg_.n = n;
  rebuild_index();
}

SpecResult SuffixCorpus::speculate(const int64_t* context, size_t len, size_t max_tokens) const {
  SpecResult r;
  const size_t n = cfg_.n;
  const size_t wlen = std::min(len, cfg_.depth);
  const int64_t* w = context + (len - wlen);
  if (max_tokens == 0 || wlen < n) return r;
  const int64_t slot = find_slot(window_hash(w + wlen - n, n), w + wlen - n);
  if (slot < 0) return r;
  const std::vector<Hit>& hits = buckets_[table_[slot].bucket].hits;

  // Longest backward extension among the most recent `candidates` hits.
  struct End {
    uint64_t id, pos;
    const int64_t* s;
    size_t slen;
  };
  End ends_buf[64];
  std::vector<End> ends_heap;
  End* ends = ends_buf;
  size_t ne = 0;
  const size_t take = std::min(hits.size(), cfg_.candidates);
  if (take > 64) {
    ends_heap.resize(take);
    ends = ends_heap.data();
  }
  size_t best = 0;
  for (size_t c = 0; c < take; ++c) {
    const Hit& h = hits[hits.size() - 1 - c];
    const std::vector<int64_t>& s = seq(h.id);
    size_t m = n;
    while (m < wlen && m < h.pos + n && s[h.pos + n - m - 1] == w[wlen - m - 1]) ++m;
    if (m > best) {
      best = m;
      ne = 0;
    }
    if (m == best) ends[ne++] = End{h.id, h.pos + n, s.data(), s.size()};
  }
  const double capf = std::max(0.0, cfg_.factor * static_cast<double>(best) + cfg_.offset);
  const size_t cap = std::min(max_tokens, capf >= 1.8e19 ? SIZE_MAX : static_cast<size_t>(capf));

  struct Vote {
    int64_t tok;
    size_t support;
    uint64_t id, pos;
  };
  std::vector<Vote> votes;
  votes.reserve(ne);
  double score = 1.0;
  for (size_t step = 0; step < cap; ++step) {
    votes.clear();
    for (size_t e = 0; e < ne; ++e) {
      const End& en = ends[e];
      if (en.pos + step >= en.slen) continue;
      const int64_t tok = en.s[en.pos + step];
      Vote* v = nullptr;
      for (Vote& x : votes)
        if (x.tok == tok) {
          v = &x;
          break;
        }
      if (!v) {
        votes.push_back(Vote{tok, 0, en.id, en.pos});
        v = &votes.back();
      }
      ++v->support;
      if (std::tie(en.id, en.pos) > std::tie(v->id, v->pos)) {
        v->id = en.id;
        v->pos = en.pos;
      }
    }
    if (votes.empty()) break;
    // Winner: most support, then most recent (id, pos), then larger token.
    const Vote* win = &votes[0];
    for (const Vote& x : votes)
      if (std::tie(x.support, x.id, x.pos, x.tok) > std::tie(win->support, win->id, win->pos, win->tok)) win = &x;
    if (win->support < cfg_.support) break;
    score *= static_cast<double>(win->support) / static_cast<double>(ne);
    const int64_t tok = win->tok;
    r.tokens.push_back(tok);
    size_t keep = 0;
    for (size_t e = 0; e < ne; ++e)
      if (ends[e].pos + step < ends[e].slen && ends[e].s[ends[e].pos + step] == tok) ends[keep++] = ends[e];
    ne = keep;
  }
  r.score = r.tokens.empty() ? 0.0 : score;
  r.match_len = best;
  return r;
}

std::map<std::string, size_t> SuffixCorpus::stats() const {
  size_t positions = 0, capacity = 0;
  for (uint64_t id = first_id_; id < next_id_; ++id) capacity += seq(id).capacity();
  for (const Slot& s : table_)
    if (s.h) positions += buckets_[s.bucket].hits.size();
  return {
      {"num_sequences", seqs_.size()},
      {"num_index_keys", live_buckets_},
      {"index_positions", positions},
      {"cached_tokens", tokens_},
      {"allocated_token_capacity", capacity},
      {"index_n", cfg_.n},
      {"max_cached_requests", cfg_.sequences},
      {"max_cached_tokens", cfg_.tokens},
  };
}

namespace {

constexpr char kSnapMagic[8] = {'S', 'H', 'C', 'O', 'R', 'P', '0', '1'};
constexpr uint32_t kSnapVersion = 1;

// FNV-1a, 64-bit (offset basis 14695981039346656037, prime 1099511628211).
struct Fnv {
  uint64_t h = 14695981039346656037ull;
  void feed(const void* p, size_t n) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
  }
};

}  // namespace

int64_t save_corpus(const SuffixCorpus& c, const std::string& path, std::string* err) {
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) {
    if (err) *err = "cannot open " + tmp + " for writing";
    return -1;
  }
  Fnv fnv;
  bool ok = std::fwrite(kSnapMagic, 1, sizeof(kSnapMagic), f) == sizeof(kSnapMagic);
  auto put = [&](const void* p, size_t n) {
    if (!ok) return;
    ok = std::fwrite(p, 1, n, f) == n;
    fnv.feed(p, n);
  };
  const uint32_t version = kSnapVersion, n = static_cast<uint32_t>(c.cfg().n);
  const uint64_t count = c.sequences().size();
  put(&version, sizeof(version));
  put(&n, sizeof(n));
  put(&count, sizeof(count));
  for (const auto& seq : c.sequences()) {
    const uint64_t len = seq.size();
    put(&len, sizeof(len));
    put(seq.data(), len * sizeof(int64_t));
  }
  if (ok) ok = std::fwrite(&fnv.h, 1, sizeof(fnv.h), f) == sizeof(fnv.h);
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    if (err) *err = "cannot write " + path;
    return -1;
  }
  return static_cast<int64_t>(count);
}

int64_t load_corpus(SuffixCorpus& c, const std::string& path, std::string* err) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    if (err) *err = "cannot open " + path;
    return -1;
  }
  std::vector<unsigned char> buf;
  unsigned char chunk[1 << 16];
  size_t got;
  while ((got = std::fread(chunk, 1, sizeof(chunk), f)) > 0) buf.insert(buf.end(), chunk, chunk + got);
  std::fclose(f);
  auto fail = [&](const char* why) -> int64_t {
    if (err) *err = path + ": " + why;
    return -1;
  };
  const size_t head = sizeof(kSnapMagic) + 4 + 4 + 8;
  if (buf.size() < head + 8 || std::memcmp(buf.data(), kSnapMagic, sizeof(kSnapMagic)) != 0)
    return fail("not a corpus snapshot");
  Fnv fnv;
  fnv.feed(buf.data() + sizeof(kSnapMagic), buf.size() - sizeof(kSnapMagic) - 8);
  uint64_t sum;
  std::memcpy(&sum, buf.data() + buf.size() - 8, 8);
  if (sum != fnv.h) return fail("checksum mismatch");
  uint32_t version;
  uint64_t count;
  std::memcpy(&version, buf.data() + sizeof(kSnapMagic), 4);
  std::memcpy(&count, buf.data() + sizeof(kSnapMagic) + 8, 8);
  if (version != kSnapVersion) return fail("unsupported snapshot version");
  // walk the sequence table once to check every length before anything is added
  std::vector<std::pair<size_t, uint64_t>> spans;  // (byte offset of the tokens, length)
  size_t off = head;
  const size_t end = buf.size() - 8;
  for (uint64_t i = 0; i < count; ++i) {
    if (end - off < 8) return fail("truncated sequence table");
    uint64_t len;
    std::memcpy(&len, buf.data() + off, 8);
    off += 8;
    if (len > (end - off) / sizeof(int64_t)) return fail("truncated sequence");
    spans.emplace_back(off, len);
    off += len * sizeof(int64_t);
  }
  if (off != end) return fail("trailing bytes");
  std::vector<int64_t> toks;
  for (const auto& sp : spans) {
    toks.resize(sp.second);
    std::memcpy(toks.data(), buf.data() + sp.first, sp.second * sizeof(int64_t));
    c.add(toks);
  }
  return static_cast<int64_t>(count);
}

}  // namespace sh
