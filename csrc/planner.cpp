// Native cache-build planner for the TinyGPT-PRA device path.
//
// Given one batch of collator rows (each with its root reference handles and the
// documents they carry), this computes what the batched device encoder needs:
//   * per row, the child-first traversal of the reference graph with the
//     reference's recursion semantics (src/pra_torch/resolution.py:124-236):
//     cycle detection on the ancestry path, missing-URI policy, a shared budget
//     per root traversal, the max-depth / max-children limits, and "visible"
//     entries (every entry already planned in the row, when the entry has a
//     ready child);
//   * tokens of every resolved text (word-id vocabularies natively, any other
//     tokenizer through its Python `encode`);
//   * fixed-window chunking with overlap and the max-chunks overflow policy
//     (src/pra_torch/chunking.py:215-267, 180-212), chunk ids `uri#chunk=i`;
//   * dependency waves (an entry encodes after every entry it may attend to),
//     encode-sequence numbering, and every wave's int32 tables (token ids,
//     padding bytes, lengths, budgets, gist rows, routing namespaces), plus the
//     prompt's routing namespace and the chunk tables, all packed into ONE int32
//     array so the device receives them in a single pinned copy.
//
// The Python planner (DeviceRuntime.plan_row / plan_batch) stays the oracle and
// the fallback: `plan_batch` returns None whenever a row needs something this
// planner does not do (non-fixed chunking, a policy that warns or raises, an
// entry longer than the native limit, a reference token the tokenizer has not
// registered yet), and the caller then plans the batch in Python, which raises
// or warns exactly as before.  Output tables are identical (tested on CPU).
#include <pybind11/numpy.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace py = pybind11;

namespace planner {
namespace {

constexpr const char* kImplicitHeadUri = "pra://implicit/prompt/head";

struct Fallback {};  // thrown to hand the batch to the Python planner

struct BudgetExceeded {
  std::string message;
};

struct Config {
  bool recursive = true;
  int max_depth = 0;
  int max_children = 0;
  int64_t max_refs = 0;
  int64_t max_tokens = 0;
  int cycle_policy = 0;    // 0 skip, 1 error, 2 link_only
  int missing_policy = 0;  // 0 skip, 1 warn, 2 error
  int limit = 0;           // native token limit of one encode
  int budget_limit = 0;    // limit minus the safety reserve
  int cap = -1;            // max materialised memory tokens (-1: none)
  int chunk_size = 0;
  int overlap = 0;
  int max_chunks = -1;  // -1: unlimited
  int overflow = 0;     // 0 truncate, 1 merge_tail, 2 error
  bool kmeans = false;
  bool single_pass = false;  // one encode group over every chunk (layer-synchronous cache build)
};

// A resolved document of one row (shared by every URI that resolves to it).
struct Doc {
  py::object text;                  // the resolved text (kept for lazy records)
  std::vector<std::string> children;  // reference-table values, de-duplicated, in order
  std::vector<int32_t> tokens;
  bool tokenized = false;
};

struct Entry {
  int row = 0;
  std::string uri;
  int doc = -1;
  bool use_memory = false;
  int depth = 0;
  int local = 0;  // index within its row
  int wave = 0;
  int chunk_begin = 0, chunk_end = 0;  // global chunk range (contiguous per entry)
};

struct Chunk {
  int entry = 0;
  int index = 0;  // position within its entry (the `#chunk=i` suffix)
  int start = 0, end = 0;
  int seq = -1;
};

struct Event {
  std::string uri, kind, parent, detail;
  int depth = 0;
  bool has_parent = false, has_detail = false;
};

struct Dependency {
  std::string parent, child, action;
  bool cyclic = false, has_parent = false;
};

// Word-id tokenizer: "t<digits>" -> the number (below the base vocabulary, else 0),
// registered reference tokens -> their ids, anything else -> 0.  Texts with
// non-ASCII bytes, and unregistered "<REF_n>" words (which the Python tokenizer
// would register), go through Python.
struct Tokenizer {
  py::object py_tok;
  bool word_ids = false;
  int64_t base_vocab = 0;
  std::unordered_map<std::string, int32_t> refs;

  static bool is_space(unsigned char c) { return c == ' ' || (c >= 9 && c <= 13) || (c >= 0x1c && c <= 0x1f); }

  static bool is_ref_token(const char* p, size_t n) {
    static const char kPrefix[] = "<REF_";
    if (n < 7 || std::memcmp(p, kPrefix, 5) != 0 || p[n - 1] != '>') return false;
    for (size_t i = 5; i + 1 < n; ++i)
      if (p[i] < '0' || p[i] > '9') return false;
    return true;
  }

  int32_t word(const char* p, size_t n) const {
    if (n >= 2 && p[0] == 't') {
      bool digits = true;
      for (size_t i = 1; i < n && digits; ++i) digits = p[i] >= '0' && p[i] <= '9';
      if (digits) {
        if (n - 1 > 15) return 0;
        int64_t v = 0;
        for (size_t i = 1; i < n; ++i) v = v * 10 + (p[i] - '0');
        return v < base_vocab ? static_cast<int32_t>(v) : 0;
      }
    }
    auto it = refs.find(std::string(p, n));
    if (it != refs.end()) return it->second;
    if (is_ref_token(p, n)) throw Fallback{};  // would be registered by the Python tokenizer
    return 0;
  }

  void encode(const py::object& text, std::vector<int32_t>& out) const {
    out.clear();
    Py_ssize_t size = 0;
    const char* s = PyUnicode_AsUTF8AndSize(text.ptr(), &size);
    if (s == nullptr) throw py::error_already_set();
    bool ascii = true;
    for (Py_ssize_t i = 0; i < size && ascii; ++i) ascii = static_cast<unsigned char>(s[i]) < 0x80;
    if (!word_ids || !ascii) {
      for (auto v : py_tok.attr("encode")(text)) out.push_back(v.cast<int32_t>());
      return;
    }
    Py_ssize_t i = 0;
    while (i < size) {
      while (i < size && is_space(static_cast<unsigned char>(s[i]))) ++i;
      Py_ssize_t j = i;
      while (j < size && !is_space(static_cast<unsigned char>(s[j]))) ++j;
      if (j > i) out.push_back(word(s + i, static_cast<size_t>(j - i)));
      i = j;
    }
  }
};

// dict(value), as the Python planner copies mappings.
py::object dict_(const py::handle& value) {
  PyObject* out = PyObject_CallOneArg(reinterpret_cast<PyObject*>(&PyDict_Type), value.ptr());
  if (out == nullptr) throw py::error_already_set();
  return py::reinterpret_steal<py::object>(out);
}

py::object dict_get(const py::handle& d, const char* key, const py::object& fallback) {
  PyObject* v = PyDict_GetItemString(d.ptr(), key);  // borrowed
  return v ? py::reinterpret_borrow<py::object>(v) : fallback;
}

class RowPlanner {
 public:
  RowPlanner(const Config& cfg, const Tokenizer& tok, int row) : cfg_(cfg), tok_(tok), row_(row) {}

  // Collator metadata of one row -> ordered document sources and roots.  The Python planner
  // merges every source into one dict (later definitions replace earlier ones); looking a URI up
  // from the last source backwards gives the same value without copying the (often large,
  // dataset-wide) document maps every reference carries.
  void collect(const py::handle& item) {
    py::object refs = item.attr("__getitem__")("references");
    for (auto ref : refs) {
      std::string uri = py::str(ref.attr("uri"));
      if (uri == kImplicitHeadUri) throw Fallback{};  // the Python path raises for the reserved URI
      py::object meta_obj = ref.attr("metadata");
      py::object meta = (meta_obj.is_none() || PyDict_Check(meta_obj.ptr())) ? meta_obj : dict_(meta_obj);
      Source root;
      root.uri = uri;
      root.text = meta.is_none() ? py::str("") : py::str(dict_get(meta, "text", py::str("")));
      root.table = meta.is_none() ? py::object(py::none()) : dict_get(meta, "reference_table", py::none());
      sources_.push_back(std::move(root));
      py::object docs = meta.is_none() ? py::object(py::none()) : dict_get(meta, "documents", py::none());
      if (py::bool_(docs)) {
        if (!PyDict_Check(docs.ptr())) docs = dict_(docs);
        if (sources_.size() < 2 || sources_[sources_.size() - 2].map.ptr() != docs.ptr()) {
          PyObject *key, *value;
          Py_ssize_t pos = 0;
          while (PyDict_Next(docs.ptr(), &pos, &key, &value))
            if (!PyUnicode_CheckExact(key)) throw Fallback{};  // str(key) could merge keys
          Source map;
          map.map = docs;
          sources_.push_back(std::move(map));
        } else {
          // the same map object again: keep its position as the latest definition
          Source map;
          map.map = docs;
          sources_.push_back(std::move(map));
        }
      }
      if (root_seen_.insert(uri).second) roots_.push_back(uri);
    }
  }

  void plan() {
    for (const auto& uri : roots_) {
      Budget budget{0, 0};
      std::vector<std::string> ancestry;
      try {
        ensure(uri, 0, ancestry, budget, nullptr);
      } catch (const BudgetExceeded&) {
        throw Fallback{};  // a root over budget raises in the Python planner
      }
    }
  }

  std::vector<Entry> entries;
  std::vector<std::vector<int>> entry_chunks;  // row-local chunk lists (index, start, end) triples
  std::vector<Doc> docs;
  std::vector<Event> events;
  std::vector<Dependency> deps;

 private:
  struct Budget {
    int64_t refs, tokens;
  };

  // The merged documents' value of `key`: 1 and (text, table) for a root definition, 2 and the
  // value for a map entry (None counts as absent, like `documents.get`), 0 when undefined.
  int lookup(const std::string& key, py::object& text, py::object& table, py::object& value) const {
    py::object k;
    for (auto it = sources_.rbegin(); it != sources_.rend(); ++it) {
      if (it->map) {
        if (!k) k = py::str(key);
        PyObject* v = PyDict_GetItemWithError(it->map.ptr(), k.ptr());  // borrowed
        if (v == nullptr) {
          if (PyErr_Occurred()) throw py::error_already_set();
          continue;
        }
        value = py::reinterpret_borrow<py::object>(v);
        return value.is_none() ? 0 : 2;
      }
      if (it->uri == key) {
        text = it->text;
        table = it->table;
        return 1;
      }
    }
    return 0;
  }

  // InMemoryResolver.resolve: exact URI, then its anchor-free base.
  int resolve(const std::string& uri) {
    std::string key = uri;
    py::object text, table, value;
    int kind = lookup(key, text, table, value);
    if (kind == 0) {
      const auto hash = uri.find('#');
      if (hash == std::string::npos) return -1;
      key = uri.substr(0, hash);
      kind = lookup(key, text, table, value);
      if (kind == 0) return -1;
    }
    auto cached = doc_index_.find(key);
    if (cached != doc_index_.end()) return cached->second;
    Doc doc;
    if (kind == 1) {
      doc.text = text;
    } else if (PyDict_Check(value.ptr())) {
      doc.text = py::str(dict_get(value, "text", py::str("")));
      table = dict_get(value, "reference_table", py::none());
    } else {
      doc.text = py::str(value);
    }
    if (table && !table.is_none() && py::bool_(table)) {
      // {str(k): str(v)} keeps first-insertion order and the last value of keys equal as strings
      py::object t = PyDict_Check(table.ptr()) ? table : dict_(table);
      std::unordered_map<std::string, size_t> slot;
      std::vector<std::string> values;
      PyObject *k, *v;
      Py_ssize_t pos = 0;
      while (PyDict_Next(t.ptr(), &pos, &k, &v)) {
        std::string key_s = py::str(k), value_s = py::str(v);
        auto found = slot.find(key_s);
        if (found == slot.end()) {
          slot.emplace(key_s, values.size());
          values.push_back(value_s);
        } else {
          values[found->second] = value_s;
        }
      }
      std::unordered_set<std::string> seen;
      for (auto& child : values)
        if (seen.insert(child).second) doc.children.push_back(child);
    }
    if (static_cast<int>(doc.children.size()) > cfg_.max_children) doc.children.resize(std::max(cfg_.max_children, 0));
    const int index = static_cast<int>(docs.size());
    docs.push_back(std::move(doc));
    doc_index_.emplace(key, index);
    return index;
  }

  void ensure(const std::string& uri, int depth, std::vector<std::string>& ancestry, Budget& budget,
              const std::string* parent) {
    if (std::find(ancestry.begin(), ancestry.end(), uri) != ancestry.end()) {
      static const char* kActions[] = {"skip", "error", "link_only"};
      deps.push_back({parent ? *parent : std::string(), uri, kActions[cfg_.cycle_policy], true, parent != nullptr});
      event(uri, "cycle", depth, parent);
      if (cfg_.cycle_policy == 1) throw Fallback{};
      return;
    }
    const int d = resolve(uri);
    if (d < 0) {
      if (cfg_.missing_policy != 0) throw Fallback{};
      py::object err = py::module_::import("builtins").attr("KeyError")(py::str("Reference URI is not available: " + uri));
      Event e{uri, "missing", std::string(), py::str(err), depth, false, true};
      events.push_back(std::move(e));
      return;
    }
    if (ready_.count(uri)) {
      event(uri, "cache_hit", depth, parent);
      return;
    }
    Doc& doc = docs[d];
    if (!doc.tokenized) {
      tok_.encode(doc.text, doc.tokens);
      doc.tokenized = true;
    }
    const int64_t n = static_cast<int64_t>(doc.tokens.size());
    if (budget.refs + 1 > cfg_.max_refs) throw BudgetExceeded{"max_total_references exhausted"};
    if (budget.tokens + n > cfg_.max_tokens) throw BudgetExceeded{"max_total_tokens exhausted"};
    budget.refs += 1;
    budget.tokens += n;
    event(uri, "building", depth, parent);
    const std::vector<std::string> children = docs[d].children;  // copy: docs may grow below
    if (cfg_.recursive && depth < cfg_.max_depth) {
      ancestry.push_back(uri);
      for (const auto& child : children) {
        deps.push_back({uri, child, "resolve", false, true});
        try {
          ensure(child, depth + 1, ancestry, budget, &uri);
        } catch (const BudgetExceeded& error) {
          Event e{child, "budget_exhausted", uri, error.message, depth + 1, true, true};
          events.push_back(std::move(e));
          break;
        }
      }
      ancestry.pop_back();
    } else if (!children.empty()) {
      const char* reason = cfg_.recursive ? "max_depth" : "recursion_disabled";
      for (const auto& child : children) deps.push_back({uri, child, reason, false, true});
    }
    bool use_memory = false;
    if (cfg_.recursive)
      for (const auto& child : children) use_memory = use_memory || ready_.count(child) > 0;
    if (n > cfg_.limit) throw Fallback{};  // needs bounded encoding
    Entry entry;
    entry.row = row_;
    entry.uri = uri;
    entry.doc = d;
    entry.use_memory = use_memory;
    entry.depth = depth;
    entry.local = static_cast<int>(entries.size());
    entries.push_back(entry);
    entry_chunks.push_back(chunk_spans(static_cast<int>(n)));
    ready_.insert(uri);
    event(uri, "ready", depth, parent);
  }

  // Fixed windows of chunk_size advancing by chunk_size - overlap, then the max-chunks policy.
  std::vector<int> chunk_spans(int n) const {
    std::vector<int> spans;  // (index, start, end) triples
    if (n == 0) return spans;
    const int size = cfg_.chunk_size, stride = cfg_.chunk_size - cfg_.overlap;
    int count = 0;
    for (int start = 0; start < n; start += stride) {
      const int stop = std::min(start + size, n);
      spans.insert(spans.end(), {count++, start, stop});
      if (stop == n) break;
    }
    if (cfg_.max_chunks >= 0 && count > cfg_.max_chunks) {
      if (cfg_.overflow == 2 || cfg_.max_chunks == 0) throw Fallback{};
      spans.resize(3 * static_cast<size_t>(cfg_.max_chunks));
      if (cfg_.overflow == 1) spans.back() = n;  // merge_tail: the last kept chunk runs to the end
    }
    return spans;
  }

  void event(const std::string& uri, const char* kind, int depth, const std::string* parent) {
    Event e;
    e.uri = uri;
    e.kind = kind;
    e.depth = depth;
    if (parent) {
      e.parent = *parent;
      e.has_parent = true;
    }
    events.push_back(std::move(e));
  }

  const Config& cfg_;
  const Tokenizer& tok_;
  int row_;
  struct Source {
    std::string uri;         // a root definition: its URI, text and reference table
    py::object text, table;
    py::object map;          // or a documents map (uri -> value)
  };
  std::vector<Source> sources_;
  std::unordered_map<std::string, int> doc_index_;
  std::vector<std::string> roots_;
  std::unordered_set<std::string> root_seen_;
  std::unordered_set<std::string> ready_;
};

// Growing int32 array with named (offset, words, count) slices.
class Packer {
 public:
  void put(py::dict& t, const char* name, const std::vector<int32_t>& values) {
    const size_t count = values.empty() ? 1 : values.size();
    t[name] = py::make_tuple(data.size(), count, count);
    if (values.empty())
      data.push_back(0);
    else
      data.insert(data.end(), values.begin(), values.end());
  }

  void put_bytes(py::dict& t, const char* name, const std::vector<uint8_t>& bytes) {
    const size_t words = (bytes.size() + 3) / 4;
    t[name] = py::make_tuple(data.size(), words, bytes.size());
    const size_t at = data.size();
    data.resize(at + words, 0);
    if (!bytes.empty()) std::memcpy(data.data() + at, bytes.data(), bytes.size());
  }

  std::vector<int32_t> data;
};

// Routing namespace arrays of `rows` (lists of global entry ids): per row its entries by URI,
// per entry its chunks with their rank in chunk-id (string) order.
void namespace_arrays(const std::vector<std::vector<int>>& rows, const std::vector<Entry>& entries,
                      const std::vector<std::vector<int>>& rank_of_index, std::vector<int32_t> out[6]) {
  auto& row_pos_off = out[0];
  auto& row_ref_off = out[1];
  auto& ref_pos_off = out[2];
  auto& pos_chunk = out[3];
  auto& pos_ref = out[4];
  auto& pos_rank = out[5];
  for (int i = 0; i < 6; ++i) out[i].clear();
  row_pos_off.push_back(0);
  row_ref_off.push_back(0);
  ref_pos_off.push_back(0);
  std::vector<int> by_uri;
  for (const auto& ids : rows) {
    by_uri.assign(ids.begin(), ids.end());
    std::stable_sort(by_uri.begin(), by_uri.end(), [&](int a, int b) { return entries[a].uri < entries[b].uri; });
    for (size_t local = 0; local < by_uri.size(); ++local) {
      const Entry& e = entries[by_uri[local]];
      const int count = e.chunk_end - e.chunk_begin;
      for (int c = e.chunk_begin; c < e.chunk_end; ++c) {
        pos_chunk.push_back(c);
        pos_ref.push_back(static_cast<int32_t>(local));
        pos_rank.push_back(rank_of_index[count][c - e.chunk_begin]);
      }
      ref_pos_off.push_back(static_cast<int32_t>(pos_chunk.size()));
    }
    row_pos_off.push_back(static_cast<int32_t>(pos_chunk.size()));
    row_ref_off.push_back(static_cast<int32_t>(ref_pos_off.size() - 1));
  }
}

// rank_of_index[n][i]: position of chunk i among n chunks of one entry sorted by `uri#chunk=i` (i.e. by
// the decimal string of i).
const std::vector<int>& ranks(std::vector<std::vector<int>>& memo, int n) {
  if (static_cast<int>(memo.size()) <= n) memo.resize(n + 1);
  auto& r = memo[n];
  if (static_cast<int>(r.size()) != n) {
    std::vector<int> order(n);
    for (int i = 0; i < n; ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [](int a, int b) { return std::to_string(a) < std::to_string(b); });
    r.assign(n, 0);
    for (int k = 0; k < n; ++k) r[order[k]] = k;
  }
  return r;
}

template <typename T>
py::array_t<T> to_array(const std::vector<T>& v) {
  py::array_t<T> a(static_cast<py::ssize_t>(v.size()));
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
  return a;
}

py::object plan_batch_impl(const py::list& rows, const py::object& tokenizer, const py::dict& c) {
  Config cfg;
  cfg.recursive = c["recursive"].cast<bool>();
  cfg.max_depth = c["max_depth"].cast<int>();
  cfg.max_children = c["max_children"].cast<int>();
  cfg.max_refs = c["max_refs"].cast<int64_t>();
  cfg.max_tokens = c["max_tokens"].cast<int64_t>();
  cfg.cycle_policy = c["cycle_policy"].cast<int>();
  cfg.missing_policy = c["missing_policy"].cast<int>();
  cfg.limit = c["limit"].cast<int>();
  cfg.budget_limit = c["budget_limit"].cast<int>();
  cfg.cap = c["cap"].cast<int>();
  cfg.chunk_size = c["chunk_size"].cast<int>();
  cfg.overlap = c["overlap"].cast<int>();
  cfg.max_chunks = c["max_chunks"].cast<int>();
  cfg.overflow = c["overflow"].cast<int>();
  cfg.kmeans = c["kmeans"].cast<bool>();
  cfg.single_pass = c.contains("single_pass") && c["single_pass"].cast<bool>();
  if (cfg.chunk_size <= 0 || cfg.chunk_size - cfg.overlap <= 0 || cfg.max_children < 0) return py::none();

  Tokenizer tok;
  tok.py_tok = tokenizer;
  if (py::hasattr(tokenizer, "native_word_ids")) {
    py::object spec = tokenizer.attr("native_word_ids")();
    if (!spec.is_none()) {
      auto pair = spec.cast<py::tuple>();
      tok.word_ids = true;
      tok.base_vocab = pair[0].cast<int64_t>();
      for (auto kv : pair[1].cast<py::dict>()) tok.refs.emplace(py::str(kv.first), kv.second.cast<int32_t>());
    }
  }

  // 1. per-row traversal, tokenisation and chunking
  std::vector<RowPlanner> planners;
  planners.reserve(rows.size());
  try {
    for (size_t r = 0; r < rows.size(); ++r) {
      planners.emplace_back(cfg, tok, static_cast<int>(r));
      planners.back().collect(rows[r]);
      planners.back().plan();
    }
  } catch (const Fallback&) {
    return py::none();
  }

  // 2. batch numbering: entries and chunks of every row, in row order
  std::vector<Entry> entries;
  std::vector<Chunk> chunks;
  std::vector<std::vector<int>> row_entries(rows.size());
  std::vector<int> entry_visible_begin, visible;  // CSR of visible global entries
  std::vector<int32_t> chunk_token_off{0}, tokens;
  std::vector<int> entry_doc_row;  // (row, doc) to find a chunk's tokens
  for (size_t r = 0; r < planners.size(); ++r) {
    auto& p = planners[r];
    const int e0 = static_cast<int>(entries.size());
    for (size_t i = 0; i < p.entries.size(); ++i) {
      Entry e = p.entries[i];
      e.chunk_begin = static_cast<int>(chunks.size());
      const auto& spans = p.entry_chunks[i];
      const auto& toks = p.docs[e.doc].tokens;
      for (size_t k = 0; k < spans.size(); k += 3) {
        Chunk ch;
        ch.entry = e0 + static_cast<int>(i);
        ch.index = spans[k];
        ch.start = spans[k + 1];
        ch.end = spans[k + 2];
        chunks.push_back(ch);
        tokens.insert(tokens.end(), toks.begin() + ch.start, toks.begin() + ch.end);
        chunk_token_off.push_back(static_cast<int32_t>(tokens.size()));
      }
      e.chunk_end = static_cast<int>(chunks.size());
      // every entry planned earlier in the row is visible to an entry with a ready child
      int wave = 0;
      if (e.use_memory) {
        int deepest = -1;
        for (int v = e0; v < e0 + static_cast<int>(i); ++v) deepest = std::max(deepest, entries[v].wave);
        wave = deepest + 1;
      }
      e.wave = wave;
      row_entries[r].push_back(static_cast<int>(entries.size()));
      entries.push_back(e);
    }
  }
  int seq_len = 1;
  bool any_chunk = false;
  for (const auto& ch : chunks) {
    seq_len = any_chunk ? std::max(seq_len, ch.end - ch.start) : ch.end - ch.start;
    any_chunk = true;
  }
  if (!any_chunk) seq_len = 1;
  int n_waves = 0;
  for (const auto& e : entries) n_waves = std::max(n_waves, e.wave + 1);
  std::vector<std::vector<int>> waves(n_waves);
  int seq = 0;
  for (int w = 0; w < n_waves; ++w)
    for (const auto& e : entries)
      if (e.wave == w)
        for (int ch = e.chunk_begin; ch < e.chunk_end; ++ch) {
          chunks[ch].seq = seq++;
          waves[w].push_back(ch);
        }

  if (cfg.single_pass && n_waves > 1) {  // every chunk in one group, in encode-sequence order
    std::vector<int> all;
    for (const auto& w : waves) all.insert(all.end(), w.begin(), w.end());
    waves.assign(1, all);
  }

  // 3. packed tables
  std::vector<std::vector<int>> rank_memo;
  for (const auto& e : entries) ranks(rank_memo, e.chunk_end - e.chunk_begin);
  Packer pk;
  py::list wave_tables;
  const int L = seq_len;
  std::vector<int32_t> ns[6];
  for (const auto& members : waves) {
    py::dict t;
    const int n = static_cast<int>(members.size());
    std::vector<int32_t> ids(static_cast<size_t>(n) * L, 0), lens(n), last(n), budget(n), gist_rows(n), dest(n);
    std::vector<uint8_t> valid(static_cast<size_t>(n) * L, 0);
    int max_len = 1;
    for (int i = 0; i < n; ++i) {
      const Chunk& ch = chunks[members[i]];
      const int k = ch.end - ch.start;
      std::copy(tokens.begin() + chunk_token_off[members[i]], tokens.begin() + chunk_token_off[members[i] + 1],
                ids.begin() + static_cast<size_t>(i) * L);
      std::fill(valid.begin() + static_cast<size_t>(i) * L, valid.begin() + static_cast<size_t>(i) * L + k, 1);
      lens[i] = k;
      last[i] = k - 1;
      const int room = cfg.budget_limit - k;
      budget[i] = std::max(0, cfg.cap >= 0 ? std::min(room, cfg.cap) : room);
      gist_rows[i] = ch.seq * L;
      dest[i] = members[i];
      max_len = i == 0 ? k : std::max(max_len, k);
    }
    pk.put(t, "ids", ids);
    pk.put_bytes(t, "valid", valid);
    pk.put(t, "lens", lens);
    pk.put(t, "last", last);
    pk.put(t, "budget", budget);
    pk.put(t, "gist_rows", gist_rows);
    pk.put(t, "dest", dest);
    if (cfg.kmeans) {  // filled by the caller from its k-means initialisation tables
      pk.put(t, "km_first", std::vector<int32_t>(n, 0));
      pk.put(t, "km_off", std::vector<int32_t>(n, 0));
    }
    bool has_ns = false;
    for (int c : members) has_ns = has_ns || entries[chunks[c].entry].use_memory;
    if (has_ns) {
      std::vector<std::vector<int>> visible_rows;
      visible_rows.reserve(n);
      for (int c : members) {
        const Entry& e = entries[chunks[c].entry];
        std::vector<int> vis;
        if (e.use_memory) {
          const auto& row = row_entries[e.row];
          vis.assign(row.begin(), row.begin() + e.local);
        }
        visible_rows.push_back(std::move(vis));
      }
      namespace_arrays(visible_rows, entries, rank_memo, ns);
      static const char* kNames[] = {"ns0", "ns1", "ns2", "ns3", "ns4", "ns5"};
      for (int i = 0; i < 6; ++i) pk.put(t, kNames[i], ns[i]);
      t["ns_empty"] = py::bool_(ns[3].empty());
    }
    t["has_ns"] = py::bool_(has_ns);
    t["n"] = n;
    t["max_len"] = n ? max_len : 1;
    wave_tables.append(t);
  }
  // the prompt's namespace (every row sees all of its entries) and the chunk tables
  py::dict prompt;
  namespace_arrays(row_entries, entries, rank_memo, ns);
  static const char* kNames[] = {"ns0", "ns1", "ns2", "ns3", "ns4", "ns5"};
  for (int i = 0; i < 6; ++i) pk.put(prompt, kNames[i], ns[i]);
  prompt["ns_empty"] = py::bool_(ns[3].empty());
  std::vector<int32_t> c_start, c_len, c_row;
  for (const auto& ch : chunks) {
    c_start.push_back(ch.start);
    c_len.push_back(ch.end - ch.start);
    c_row.push_back(ch.seq * L);
  }
  pk.put(prompt, "chunk_start", c_start);
  pk.put(prompt, "chunk_len", c_len);
  pk.put(prompt, "chunk_pool_row", c_row);

  // 4. record arrays for lazily built Python records
  const size_t ne = entries.size(), nc = chunks.size();
  std::vector<int32_t> e_row(ne), e_wave(ne), e_use(ne), e_depth(ne), e_local(ne), e_cb(ne), e_ce(ne);
  py::list e_uri(ne), e_text(ne);
  for (size_t i = 0; i < ne; ++i) {
    const Entry& e = entries[i];
    e_row[i] = e.row;
    e_wave[i] = e.wave;
    e_use[i] = e.use_memory;
    e_depth[i] = e.depth;
    e_local[i] = e.local;
    e_cb[i] = e.chunk_begin;
    e_ce[i] = e.chunk_end;
    e_uri[i] = py::str(e.uri);
    e_text[i] = planners[e.row].docs[e.doc].text;
  }
  std::vector<int32_t> ch_entry(nc), ch_index(nc), ch_start(nc), ch_end(nc), ch_seq(nc);
  for (size_t i = 0; i < nc; ++i) {
    ch_entry[i] = chunks[i].entry;
    ch_index[i] = chunks[i].index;
    ch_start[i] = chunks[i].start;
    ch_end[i] = chunks[i].end;
    ch_seq[i] = chunks[i].seq;
  }
  py::list row_entries_py, audit;
  for (size_t r = 0; r < planners.size(); ++r) {
    py::list ids;
    for (int e : row_entries[r]) ids.append(e);
    row_entries_py.append(ids);
    py::list ev, dp;
    for (const auto& e : planners[r].events)
      ev.append(py::make_tuple(e.uri, e.kind, e.depth, e.has_parent ? py::object(py::str(e.parent)) : py::none(),
                               e.has_detail ? py::object(py::str(e.detail)) : py::none()));
    for (const auto& d : planners[r].deps)
      dp.append(py::make_tuple(d.has_parent ? py::object(py::str(d.parent)) : py::none(), d.child, d.cyclic,
                               d.action));
    audit.append(py::make_tuple(ev, dp));
  }
  py::list waves_py;
  for (const auto& w : waves) {
    py::list members;
    for (int ch : w) members.append(ch);
    waves_py.append(members);
  }

  py::dict out;
  out["packed"] = to_array(pk.data);
  out["wave_tables"] = wave_tables;
  out["prompt"] = prompt;
  out["waves"] = waves_py;
  out["seq_len"] = seq_len;
  out["rows"] = row_entries_py;
  out["audit"] = audit;
  out["entry_row"] = to_array(e_row);
  out["entry_wave"] = to_array(e_wave);
  out["entry_use_memory"] = to_array(e_use);
  out["entry_depth"] = to_array(e_depth);
  out["entry_local"] = to_array(e_local);
  out["entry_chunk_begin"] = to_array(e_cb);
  out["entry_chunk_end"] = to_array(e_ce);
  out["entry_uri"] = e_uri;
  out["entry_text"] = e_text;
  out["chunk_entry"] = to_array(ch_entry);
  out["chunk_index"] = to_array(ch_index);
  out["chunk_start"] = to_array(ch_start);
  out["chunk_end"] = to_array(ch_end);
  out["chunk_seq"] = to_array(ch_seq);
  out["chunk_token_off"] = to_array(chunk_token_off);
  out["tokens"] = to_array(tokens);
  return out;
}

}  // namespace
}  // namespace planner

// Exposed through the extension module (bindings.cpp).
py::object pra_plan_batch(const py::list& rows, const py::object& tokenizer, const py::dict& cfg) {
  return planner::plan_batch_impl(rows, tokenizer, cfg);
}
