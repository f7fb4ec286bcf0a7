// Python module `_native`: the proposer core's public surface.
//
// Class and method names, argument order and return shapes match the
// reference's native module so a user of `suffix_hybrid._native` can switch
// without code changes (reference: src/lib.rs:445-551): SuffixCache, Engine,
// HybridMixer, V2SuffixProposer, rejection_greedy_accept, VERSION.
// Integer buffers are read in place through strided views (NumPy arrays or
// CPU tensors exposed as NumPy), never converted to Python lists.  Every
// entry point converts an unexpected C++ failure into RuntimeError so the
// caller's degrade-to-native-draft guard runs (drafts are advisory; the
// target model verifies every token).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <chrono>
#include <string>
#include <string_view>

#include "decider.h"
#include "engine.h"
#include "mixer.h"
#include "suffix_cache.h"
#include "v2_suffix.h"

namespace py = pybind11;
using namespace sh;

static const char* kVersion = "0.3.0-native-cpp-b200";

namespace {

template <class F>
auto guard(const char* what, F&& f) -> decltype(f()) {
  try {
    return f();
  } catch (const ValueError& e) {
    throw py::value_error(e.what());
  } catch (const py::error_already_set&) {
    throw;
  } catch (const py::builtin_exception&) {
    throw;
  } catch (const std::exception& e) {
    throw std::runtime_error(std::string("suffix_hybrid ") + what + " failed (" + e.what() +
                             "); caller must degrade to native drafts");
  }
}

uint64_t now_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}

bool int_dtype(const py::array& a, int* itemsize) {
  const py::dtype dt = a.dtype();
  const char kind = dt.kind();
  if (kind != 'i' && kind != 'u') return false;
  const int sz = static_cast<int>(dt.itemsize());
  if (sz != 4 && sz != 8) return false;
  // Only int32/int64 (unsigned widths would reinterpret high values).
  if (kind == 'u') return false;
  *itemsize = sz;
  return true;
}

bool is_ndarray(const py::handle& h) { return py::isinstance<py::array>(h); }

IntMatrix as_matrix(const py::handle& obj, const char* err) {
  if (!is_ndarray(obj)) throw ValueError(err);
  py::array a = py::reinterpret_borrow<py::array>(obj);
  int itemsize = 0;
  if (a.ndim() != 2 || !int_dtype(a, &itemsize)) throw ValueError(err);
  IntMatrix m;
  m.base = static_cast<const char*>(a.data());
  m.rows = static_cast<size_t>(a.shape(0));
  m.cols = static_cast<size_t>(a.shape(1));
  m.s0 = a.strides(0);
  m.s1 = a.strides(1);
  m.itemsize = itemsize;
  return m;
}

IntVector as_vector(const py::handle& obj, const char* err) {
  if (!is_ndarray(obj)) throw ValueError(err);
  py::array a = py::reinterpret_borrow<py::array>(obj);
  int itemsize = 0;
  if (a.ndim() != 1 || !int_dtype(a, &itemsize)) throw ValueError(err);
  IntVector v;
  v.base = static_cast<const char*>(a.data());
  v.n = static_cast<size_t>(a.shape(0));
  v.s = a.strides(0);
  v.itemsize = itemsize;
  return v;
}

// Python sequence of ints (list, tuple, NumPy 1-D int array) -> vector.
std::vector<int64_t> to_tokens(const py::handle& obj) {
  std::vector<int64_t> out;
  if (is_ndarray(obj)) {
    py::array a = py::reinterpret_borrow<py::array>(obj);
    int itemsize = 0;
    if (a.ndim() == 1 && int_dtype(a, &itemsize)) {
      IntVector v = as_vector(obj, "tokens");
      out.resize(v.n);
      for (size_t i = 0; i < v.n; ++i) out[i] = v.at(i);
      return out;
    }
  }
  PyObject* seq = PySequence_Fast(obj.ptr(), "expected a sequence of token ids");
  if (!seq) throw py::error_already_set();
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  PyObject** items = PySequence_Fast_ITEMS(seq);
  out.resize(static_cast<size_t>(n));
  for (Py_ssize_t i = 0; i < n; ++i) {
    const long long v = PyLong_AsLongLong(items[i]);
    if (v == -1 && PyErr_Occurred()) {
      Py_DECREF(seq);
      throw py::error_already_set();
    }
    out[static_cast<size_t>(i)] = v;
  }
  Py_DECREF(seq);
  return out;
}

std::vector<std::vector<int64_t>> to_token_lists(const py::handle& obj) {
  PyObject* seq = PySequence_Fast(obj.ptr(), "expected a sequence of token lists");
  if (!seq) throw py::error_already_set();
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  PyObject** items = PySequence_Fast_ITEMS(seq);
  std::vector<std::vector<int64_t>> out(static_cast<size_t>(n));
  try {
    for (Py_ssize_t i = 0; i < n; ++i) out[static_cast<size_t>(i)] = to_tokens(items[i]);
  } catch (...) {
    Py_DECREF(seq);
    throw;
  }
  Py_DECREF(seq);
  return out;
}

// Request ids: zero-copy UTF-8 views into the caller's str objects (valid
// for the duration of the call; the caller's list keeps them alive).
// Owns the sequences PySequence_Fast returns while one call uses views into
// them (a few per call; no Python allocation, unlike a list).
struct Keep {
  py::object objs[4];
  int n = 0;
  void append(py::object o) {
    if (n >= 4) throw std::runtime_error("internal: too many kept sequences");
    objs[n++] = std::move(o);
  }
};

void to_ids_into(const py::handle& obj, Keep* keep, std::vector<std::string_view>& ids) {
  PyObject* seq = PySequence_Fast(obj.ptr(), "request ids must be a sequence of str");
  if (!seq) throw py::error_already_set();
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  PyObject** items = PySequence_Fast_ITEMS(seq);
  ids.resize(static_cast<size_t>(n));
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (!PyUnicode_Check(items[i])) {
      Py_DECREF(seq);
      throw ValueError("request ids must be str");
    }
    Py_ssize_t len = 0;
    const char* s = PyUnicode_AsUTF8AndSize(items[i], &len);
    if (!s) {
      Py_DECREF(seq);
      throw py::error_already_set();
    }
    ids[static_cast<size_t>(i)] = std::string_view(s, static_cast<size_t>(len));
  }
  keep->append(py::reinterpret_steal<py::object>(seq));
}

std::vector<std::string_view> to_ids(const py::handle& obj, Keep* keep) {
  std::vector<std::string_view> ids;
  to_ids_into(obj, keep, ids);
  return ids;
}

// Accepted lengths (list / tuple / NumPy of ints) into a reused vector.
void to_tokens_into(const py::handle& obj, std::vector<int64_t>& out) {
  if (PyList_CheckExact(obj.ptr())) {
    const Py_ssize_t n = PyList_GET_SIZE(obj.ptr());
    out.resize(static_cast<size_t>(n));
    for (Py_ssize_t i = 0; i < n; ++i) {
      const long long v = PyLong_AsLongLong(PyList_GET_ITEM(obj.ptr(), i));
      if (v == -1 && PyErr_Occurred()) throw py::error_already_set();
      out[static_cast<size_t>(i)] = v;
    }
    return;
  }
  out = to_tokens(obj);
}

// Drafts in: int64 rows plus the caller's int objects, so published tokens
// equal to a native draft token reuse that object instead of allocating.
struct DraftRows {
  std::vector<std::vector<int64_t>> values;
  std::vector<std::vector<PyObject*>> objs;  // borrowed; caller keeps them alive
};

// Fills `out` in place: its vectors keep their capacity across calls, so a
// warm call allocates nothing for the draft rows.
void to_draft_rows(const py::handle& obj, Keep* keep, DraftRows& out) {
  PyObject* seq = PySequence_Fast(obj.ptr(), "native drafts must be a sequence of token lists");
  if (!seq) throw py::error_already_set();
  keep->append(py::reinterpret_steal<py::object>(seq));
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  PyObject** rows = PySequence_Fast_ITEMS(seq);
  out.values.resize(static_cast<size_t>(n));
  out.objs.resize(static_cast<size_t>(n));
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (PyList_CheckExact(rows[i]) || PyTuple_CheckExact(rows[i])) {
      PyObject* r = rows[i];
      const bool list = PyList_CheckExact(r);
      const Py_ssize_t m = list ? PyList_GET_SIZE(r) : PyTuple_GET_SIZE(r);
      auto& v = out.values[static_cast<size_t>(i)];
      auto& o = out.objs[static_cast<size_t>(i)];
      v.resize(static_cast<size_t>(m));
      o.resize(static_cast<size_t>(m));
      for (Py_ssize_t j = 0; j < m; ++j) {
        PyObject* it = list ? PyList_GET_ITEM(r, j) : PyTuple_GET_ITEM(r, j);
        const long long x = PyLong_AsLongLong(it);
        if (x == -1 && PyErr_Occurred()) throw py::error_already_set();
        v[static_cast<size_t>(j)] = x;
        o[static_cast<size_t>(j)] = PyLong_CheckExact(it) ? it : nullptr;
      }
    } else {
      out.values[static_cast<size_t>(i)] = to_tokens(rows[i]);
      out.objs[static_cast<size_t>(i)].assign(out.values[static_cast<size_t>(i)].size(), nullptr);
    }
  }
}

// Per-thread draft-row scratch of the mixer calls (the borrowed int objects are
// valid for one call: the caller's lists are kept alive by `keep`).
DraftRows& draft_scratch() {
  static thread_local DraftRows rows;
  return rows;
}

py::list to_pylist_reuse(const std::vector<std::vector<int64_t>>& rows, const DraftRows& src) {
  py::list out(rows.size());
  for (size_t i = 0; i < rows.size(); ++i) {
    const auto& r = rows[i];
    PyObject* inner = PyList_New(static_cast<Py_ssize_t>(r.size()));
    if (!inner) throw py::error_already_set();
    const auto& sv = src.values[i];
    const auto& so = src.objs[i];
    for (size_t j = 0; j < r.size(); ++j) {
      PyObject* item;
      if (j < sv.size() && sv[j] == r[j] && so[j] != nullptr) {
        item = so[j];
        Py_INCREF(item);
      } else {
        item = PyLong_FromLongLong(r[j]);
      }
      PyList_SET_ITEM(inner, static_cast<Py_ssize_t>(j), item);
    }
    PyList_SET_ITEM(out.ptr(), static_cast<Py_ssize_t>(i), inner);
  }
  return out;
}

py::list to_pylist(const std::vector<std::vector<int64_t>>& rows) {
  py::list out(rows.size());
  for (size_t i = 0; i < rows.size(); ++i) {
    PyObject* inner = PyList_New(static_cast<Py_ssize_t>(rows[i].size()));
    if (!inner) throw py::error_already_set();
    for (size_t j = 0; j < rows[i].size(); ++j) PyList_SET_ITEM(inner, static_cast<Py_ssize_t>(j), PyLong_FromLongLong(rows[i][j]));
    PyList_SET_ITEM(out.ptr(), static_cast<Py_ssize_t>(i), inner);
  }
  return out;
}

py::dict corpus_stats(const std::shared_ptr<SharedCorpus>& c) {
  std::lock_guard<std::mutex> lock(c->mu);
  py::dict d;
  for (const auto& kv : c->corpus.stats()) d[py::str(kv.first)] = kv.second;
  return d;
}

struct PySuffixCache {
  std::shared_ptr<SharedCorpus> c;
};

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "Native proposer core: suffix corpus, n-gram, hybrid mixer, suffix-only proposer, greedy verify oracle";
  m.attr("VERSION") = kVersion;

  py::class_<PySuffixCache>(m, "SuffixCache")
      .def(py::init([]() { return PySuffixCache{std::make_shared<SharedCorpus>(CacheConfig::from_env())}; }))
      .def("add_sequence",
           [](PySuffixCache& s, py::handle tokens) {
             std::vector<int64_t> t = to_tokens(tokens);
             guard("add_sequence", [&] {
               std::lock_guard<std::mutex> lock(s.c->mu);
               s.c->corpus.add(t);
               return 0;
             });
           })
      .def("add_prompt",
           [](PySuffixCache& s, py::handle tokens) {
             std::vector<int64_t> t = to_tokens(tokens);
             guard("add_prompt", [&] {
               std::lock_guard<std::mutex> lock(s.c->mu);
               if (s.c->corpus.cfg().prompts) s.c->corpus.add(t);
               return 0;
             });
           })
      .def("speculate",
           [](PySuffixCache& s, py::handle context, int64_t max_tokens) {
             std::vector<int64_t> ctx = to_tokens(context);
             SpecResult r = guard("speculate", [&] {
               std::lock_guard<std::mutex> lock(s.c->mu);
               return s.c->corpus.speculate(ctx.data(), ctx.size(), static_cast<size_t>(std::max<int64_t>(max_tokens, 0)));
             });
             return py::make_tuple(py::cast(r.tokens), r.score, r.match_len);
           })
      .def("set_test_n",
           [](PySuffixCache& s, size_t n) {
             std::lock_guard<std::mutex> lock(s.c->mu);
             s.c->corpus.set_n(n);
           })
      .def("save",
           [](PySuffixCache& s, const std::string& path) {
             std::string err;
             int64_t r;
             {
               std::lock_guard<std::mutex> lock(s.c->mu);
               r = save_corpus(s.c->corpus, path, &err);
             }
             if (r < 0) throw std::runtime_error("suffix corpus snapshot: " + err);
             return r;
           },
           "Write the corpus (its sequences, oldest first) to a snapshot file; returns the sequence count.")
      .def("load",
           [](PySuffixCache& s, const std::string& path) {
             std::string err;
             int64_t r;
             {
               std::lock_guard<std::mutex> lock(s.c->mu);
               r = load_corpus(s.c->corpus, path, &err);
             }
             if (r < 0) throw std::runtime_error("suffix corpus restore: " + err);
             return r;
           },
           "Add a snapshot's sequences (checked whole before any is added); returns the sequence count.")
      .def("stats", [](PySuffixCache& s) { return corpus_stats(s.c); });

  py::class_<Engine>(m, "Engine")
      .def(py::init([](size_t k, size_t max_len) { return guard("Engine", [&] { return new Engine(k, max_len); }); }),
           py::arg("num_speculative_tokens") = 8, py::arg("max_model_len") = 32768)
      .def_property_readonly("suffix_cache", [](const Engine& e) { return PySuffixCache{e.corpus()}; })
      .def_property_readonly("num_speculative_tokens", &Engine::k)
      .def_property_readonly("use_ngram", &Engine::use_ngram)
      .def("propose",
           [](Engine& e, py::handle sampled, py::handle counts, py::handle tokens) {
             const uint64_t t0 = now_ns();
             PyObject* seq = PySequence_Fast(sampled.ptr(), "sampled_token_ids must be a sequence");
             if (!seq) throw py::error_already_set();
             const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
             std::vector<char> nonempty(static_cast<size_t>(n));
             for (Py_ssize_t i = 0; i < n; ++i) {
               const Py_ssize_t len = PyObject_Length(PySequence_Fast_GET_ITEM(seq, i));
               if (len < 0) {
                 Py_DECREF(seq);
                 throw py::error_already_set();
               }
               nonempty[static_cast<size_t>(i)] = len > 0;
             }
             Py_DECREF(seq);
             auto drafts = guard("propose", [&] {
               IntVector c = as_vector(counts, "num_tokens_no_spec must be a 1D int32/int64 NumPy array");
               IntMatrix t = as_matrix(tokens, "token_ids_cpu must be a 2D int32/int64 NumPy array");
               return e.propose(nonempty, c, t);
             });
             py::list out = to_pylist(drafts);
             e.add_native_ns(now_ns() - t0);
             return out;
           })
      .def("record_total",
           [](Engine& e, uint64_t ns) {
             auto r = e.record_total(ns);
             return py::make_tuple(r.first, r.second);
           })
      .def("get_stats", [](const Engine& e) {
        Engine::Stats s = e.stats();
        py::dict d;
        d["version"] = kVersion;
        d["calls"] = s.calls;
        d["proposed"] = s.proposed;
        d["accepted"] = py::none();
        d["acceptance_rate"] = py::none();
        d["acceptance_source"] = "engine_metrics_only";
        d["suffix_proposals"] = s.suffix_proposals;
        d["ngram_proposals"] = s.ngram_proposals;
        d["avg_match_len"] = s.avg_match_len;
        d["active_requests"] = s.active_requests;
        d["active_context_tokens"] = s.active_context_tokens;
        d["native_time_ns"] = s.native_ns;
        d["total_proposer_time_ns"] = s.total_ns;
        d["cache"] = corpus_stats(e.corpus());
        return d;
      });

  py::class_<HybridMixer>(m, "HybridMixer")
      .def(py::init([](size_t k, size_t max_len) { return guard("HybridMixer", [&] { return new HybridMixer(k, max_len); }); }),
           py::arg("num_speculative_tokens"), py::arg("max_model_len"))
      .def_property_readonly("suffix_cache", [](const HybridMixer& x) { return PySuffixCache{x.corpus()}; })
      .def(
          "mix",
          [](HybridMixer& x, py::handle request_ids, py::handle contexts, py::handle native_drafts,
             py::object accepted_lengths, py::object step_time_ns) {
            (void)step_time_ns;
            Keep keep;
            DraftRows& nat = draft_scratch();
            const auto& drafts = guard("mix", [&]() -> const std::vector<std::vector<int64_t>>& {
              std::vector<std::string_view> ids = to_ids(request_ids, &keep);
              std::vector<std::vector<int64_t>> ctx = to_token_lists(contexts);
              to_draft_rows(native_drafts, &keep, nat);
              std::vector<int64_t> acc;
              const bool has_acc = !accepted_lengths.is_none();
              if (has_acc) acc = to_tokens(accepted_lengths);
              return x.mix(ids, ctx, nat.values, has_acc ? &acc : nullptr);
            });
            return to_pylist_reuse(drafts, nat);
          },
          py::arg("request_ids"), py::arg("contexts"), py::arg("native_drafts"), py::arg("accepted_lengths") = py::none(),
          py::arg("step_time_ns") = py::none())
      .def(
          "mix_numpy",
          [](HybridMixer& x, py::handle request_ids, py::handle counts, py::handle tokens, py::handle native_drafts,
             py::object accepted_lengths, py::object step_time_ns) {
            (void)step_time_ns;
            Keep keep;
            DraftRows& nat = draft_scratch();
            static thread_local std::vector<std::string_view> ids;
            static thread_local std::vector<int64_t> acc;
            const auto& drafts = guard("mix_numpy", [&]() -> const std::vector<std::vector<int64_t>>& {
              to_ids_into(request_ids, &keep, ids);
              IntVector c = as_vector(counts, "counts must be int32/int64 NumPy");
              IntMatrix t = as_matrix(tokens, "tokens must be int32/int64 NumPy");
              to_draft_rows(native_drafts, &keep, nat);
              const bool has_acc = !accepted_lengths.is_none();
              if (has_acc) to_tokens_into(accepted_lengths, acc);
              return x.mix_matrix(ids, c, t, nat.values, has_acc ? &acc : nullptr);
            });
            return to_pylist_reuse(drafts, nat);
          },
          py::arg("request_ids"), py::arg("num_tokens_no_spec"), py::arg("token_ids_cpu"), py::arg("native_drafts"),
          py::arg("accepted_lengths") = py::none(), py::arg("step_time_ns") = py::none())
      .def("last_native_counts", [](const HybridMixer& x) { return x.last_native_counts(); })
      .def("cache_tokens", &HybridMixer::cache_tokens)
      .def("get_stats", [](const HybridMixer& x) {
        HybridMixer::Stats s = x.stats();
        py::dict d;
        d["calls"] = s.calls;
        d["native_tested"] = s.native_tested;
        d["native_accepted"] = s.native_accepted;
        d["suffix_tested"] = s.suffix_tested;
        d["suffix_accepted"] = s.suffix_accepted;
        d["native_proposed"] = s.native_proposed;
        d["suffix_proposed"] = s.suffix_proposed;
        d["native_mix_time_ns"] = s.elapsed_ns;
        d["mean_accept_estimate"] = s.mean_accept_estimate;
        d["active_tracked"] = s.active_tracked;
        d["split_mode"] = s.diverge ? "diverge" : "legacy";
        d["div_observed"] = s.div_observed;
        d["div_suffix_published"] = s.div_suffix_published;
        d["self_hits"] = s.self_hits;
        d["div_trust"] = s.div_trust;
        d["cache"] = corpus_stats(x.corpus());
        return d;
      });

  py::class_<V2SuffixProposer>(m, "V2SuffixProposer")
      .def(py::init([](size_t k, size_t max_len, size_t min_len, bool uniform_k, bool width_gate) {
             return guard("V2SuffixProposer", [&] { return new V2SuffixProposer(k, max_len, min_len, uniform_k, width_gate); });
           }),
           py::arg("num_speculative_tokens"), py::arg("max_model_len"), py::arg("min_len") = 1,
           py::arg("uniform_k") = false, py::arg("width_gate") = false)
      .def(
          "propose_suffix_only",
          [](V2SuffixProposer& p, py::handle request_ids, py::handle indices, py::handle totals, py::handle tokens) {
            const uint64_t t0 = now_ns();
            Keep keep;
            std::vector<int64_t> packed, widths;
            size_t n = 0;
            guard("propose_suffix_only", [&] {
              std::vector<std::string_view> ids = to_ids(request_ids, &keep);
              n = ids.size();
              IntVector tv = as_vector(totals, "totals must be int64 1D NumPy");
              if (tv.n < n) throw ValueError("totals shorter than request ids");
              std::vector<int64_t> idx;
              try {
                idx = to_tokens(indices);
              } catch (const py::error_already_set&) {
                throw ValueError("indices must be ints");
              }
              if (idx.size() < n) throw ValueError("indices shorter than request ids");
              IntMatrix tm = as_matrix(tokens, "tokens must be int32/int64 2D NumPy");
              p.propose(ids, idx, tv, tm, &packed, &widths);
              return 0;
            });
            const size_t k = p.k();
            py::array_t<int64_t> pk({static_cast<py::ssize_t>(n), static_cast<py::ssize_t>(k)});
            std::copy(packed.begin(), packed.end(), pk.mutable_data());
            py::array_t<int64_t> wd(static_cast<py::ssize_t>(n));
            std::copy(widths.begin(), widths.end(), wd.mutable_data());
            p.add_elapsed(now_ns() - t0);
            return py::make_tuple(pk, wd);
          },
          py::arg("request_ids"), py::arg("indices"), py::arg("totals"), py::arg("tokens"))
      .def_property_readonly("widths_table",
                             [](const V2SuffixProposer& p) {
                               py::dict d;
                               for (const auto& kv : p.widths_table()) d[py::str(kv.first)] = kv.second;
                               return d;
                             })
      .def_property_readonly("suffix_cache", [](const V2SuffixProposer& p) { return PySuffixCache{p.corpus()}; })
      .def("clear_widths", &V2SuffixProposer::clear_widths)
      .def_property_readonly("gate_table",
                             [](const V2SuffixProposer& p) {
                               py::dict d;
                               for (const auto& kv : p.gate_table())
                                 d[py::str(kv.first)] = py::make_tuple(kv.second.first, kv.second.second);
                               return d;
                             })
      .def("get_stats", [](const V2SuffixProposer& p) {
        V2SuffixProposer::Stats s = p.stats();
        py::dict d;
        d["steps"] = s.steps;
        d["hits"] = s.hits;
        d["hit_tokens"] = s.hit_tokens;
        d["ingested"] = s.ingested;
        d["resets"] = s.resets;
        d["padded"] = s.padded;
        d["uniform_k"] = s.uniform_k;
        d["width_gate"] = s.width_gate;
        d["active"] = s.active;
        d["elapsed_ns"] = s.elapsed_ns;
        d["cache"] = corpus_stats(p.corpus());
        return d;
      });

  // Decision-endpoint helpers (reference: src/lib.rs:431-443); malformed requests raise ValueError.
  m.def(
      "decider_prepare",
      [](const std::string& request_json, const std::string& codes_json, const std::string& profile) {
        py::gil_scoped_release nogil;
        return decider_prepare(request_json, codes_json, profile);
      },
      py::arg("request_json"), py::arg("codes_json"), py::arg("profile") = "pplx");
  m.def(
      "decider_answer",
      [](const std::string& request_json, const std::string& logits_json, double temperature,
         const std::string& profile) {
        py::gil_scoped_release nogil;
        return decider_answer(request_json, logits_json, temperature, profile);
      },
      py::arg("request_json"), py::arg("logits_json"), py::arg("temperature"), py::arg("profile") = "pplx");
  m.def(
      "rejection_greedy_accept",
      [](py::handle draft_token_ids, py::handle target_argmax, py::handle cu_num_draft_tokens, size_t max_spec_len) {
        auto as_i64 = [](py::handle h, const char* name) {
          if (!is_ndarray(h)) throw py::value_error(std::string(name) + " must be a contiguous i64 1D array");
          py::array a = py::reinterpret_borrow<py::array>(h);
          if (a.ndim() != 1 || a.dtype().kind() != 'i' || a.dtype().itemsize() != 8)
            throw py::value_error(std::string(name) + " must be a contiguous i64 1D array");
          if (!(a.flags() & py::array::c_style)) throw py::value_error(std::string(name) + " is not contiguous");
          return a;
        };
        py::array d = as_i64(draft_token_ids, "draft_token_ids");
        py::array t = as_i64(target_argmax, "target_argmax");
        py::array c = as_i64(cu_num_draft_tokens, "cu_num_draft_tokens");
        if (d.shape(0) != t.shape(0))
          throw py::value_error("draft_token_ids (" + std::to_string(d.shape(0)) + ") and target_argmax (" +
                                std::to_string(t.shape(0)) + ") length mismatch");
        const size_t batch = static_cast<size_t>(c.shape(0));
        py::array_t<int32_t> count(static_cast<py::ssize_t>(batch));
        py::array_t<int32_t> mask({static_cast<py::ssize_t>(batch), static_cast<py::ssize_t>(max_spec_len + 1)});
        rejection_greedy_accept(static_cast<const int64_t*>(d.data()), static_cast<const int64_t*>(t.data()),
                                static_cast<size_t>(d.shape(0)), static_cast<const int64_t*>(c.data()), batch,
                                max_spec_len, count.mutable_data(), mask.mutable_data());
        return py::make_tuple(count, mask);
      },
      py::arg("draft_token_ids"), py::arg("target_argmax"), py::arg("cu_num_draft_tokens"), py::arg("max_spec_len"));
}
