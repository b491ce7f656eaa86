// Byte-level BPE (fit and encode) and the best-fit row packer of the nanochat
// data stream, in C++ (``priml/baselines/nanochat/data.py:452-741`` packs in
// Python; ``scripts/prepare_data.py`` fits with the Rust rustbpe package and
// encodes with tiktoken).
//
// * BpeTrainer: counts the pre-split chunks it is fed (the split regex runs in
//   Python), then learns `num_merges` merges. Pair counts are maintained
//   incrementally: only the words that contain the merged pair are rewritten,
//   and a max-heap with lazy invalidation yields the next pair (highest count,
//   ties to the smallest (left, right) ids). Merge i creates id 256 + i.
// * BpeEncoder: applies the merges by rank (the lowest-ranked adjacent pair is
//   merged everywhere in the chunk, repeatedly), caching chunk -> ids; batches
//   are encoded on worker threads with the GIL released.
// * Packer: rows of `row_len` tokens filled from a document buffer exactly as
//   the reference stream does: before every placement the caller refills the
//   buffer up to `buffer_size` documents; the largest document that fits the
//   remaining space is placed (first in buffer order on ties); when none fits,
//   the shortest is cropped to fill the row. No padding, every position real.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace py = pybind11;

namespace {

inline uint64_t key(int32_t a, int32_t b) { return (static_cast<uint64_t>(static_cast<uint32_t>(a)) << 32) | static_cast<uint32_t>(b); }
inline int32_t left(uint64_t k) { return static_cast<int32_t>(k >> 32); }
inline int32_t right(uint64_t k) { return static_cast<int32_t>(k & 0xFFFFFFFFu); }

class BpeTrainer {
 public:
  void add_chunks(const std::vector<std::string>& chunks) {
    for (const auto& c : chunks)
      if (!c.empty()) ++counts_[c];
  }
  int64_t unique_chunks() const { return static_cast<int64_t>(counts_.size()); }

  std::vector<std::pair<int32_t, int32_t>> fit(int num_merges) {
    py::gil_scoped_release release;
    std::vector<std::vector<int32_t>> words;
    std::vector<int64_t> weight;
    words.reserve(counts_.size());
    for (const auto& kv : counts_) {
      std::vector<int32_t> w(kv.first.size());
      for (size_t i = 0; i < kv.first.size(); ++i) w[i] = static_cast<uint8_t>(kv.first[i]);
      words.push_back(std::move(w));
      weight.push_back(kv.second);
    }
    std::unordered_map<uint64_t, int64_t> pc;
    std::unordered_map<uint64_t, std::unordered_set<int32_t>> where;
    for (int32_t wi = 0; wi < static_cast<int32_t>(words.size()); ++wi) {
      const auto& w = words[wi];
      for (size_t i = 0; i + 1 < w.size(); ++i) {
        const uint64_t k = key(w[i], w[i + 1]);
        pc[k] += weight[wi];
        where[k].insert(wi);
      }
    }
    // (count, -left, -right): the largest count first, then the smallest pair
    using Entry = std::tuple<int64_t, int64_t, int64_t>;
    std::priority_queue<Entry> heap;
    for (const auto& kv : pc) heap.emplace(kv.second, -static_cast<int64_t>(left(kv.first)), -static_cast<int64_t>(right(kv.first)));
    std::vector<std::pair<int32_t, int32_t>> merges;
    merges.reserve(num_merges);
    while (static_cast<int>(merges.size()) < num_merges && !heap.empty()) {
      auto [cnt, na, nb] = heap.top();
      heap.pop();
      const int32_t a = static_cast<int32_t>(-na), b = static_cast<int32_t>(-nb);
      const uint64_t k = key(a, b);
      auto it = pc.find(k);
      const int64_t cur = it == pc.end() ? 0 : it->second;
      if (cur <= 0) continue;
      if (cur != cnt) {  // stale entry: requeue at the current count
        heap.emplace(cur, na, nb);
        continue;
      }
      const int32_t id = 256 + static_cast<int32_t>(merges.size());
      merges.emplace_back(a, b);
      std::vector<int32_t> affected(where[k].begin(), where[k].end());
      std::sort(affected.begin(), affected.end());
      std::unordered_map<uint64_t, int64_t> delta;
      for (int32_t wi : affected) {
        auto& w = words[wi];
        bool has = false;
        for (size_t i = 0; i + 1 < w.size(); ++i)
          if (w[i] == a && w[i + 1] == b) {
            has = true;
            break;
          }
        if (!has) continue;
        const int64_t c = weight[wi];
        for (size_t i = 0; i + 1 < w.size(); ++i) delta[key(w[i], w[i + 1])] -= c;
        std::vector<int32_t> out;
        out.reserve(w.size());
        for (size_t i = 0; i < w.size();) {
          if (i + 1 < w.size() && w[i] == a && w[i + 1] == b) {
            out.push_back(id);
            i += 2;
          } else {
            out.push_back(w[i]);
            i += 1;
          }
        }
        w.swap(out);
        for (size_t i = 0; i + 1 < w.size(); ++i) {
          const uint64_t nk = key(w[i], w[i + 1]);
          delta[nk] += c;
          where[nk].insert(wi);
        }
      }
      for (const auto& d : delta) {
        if (d.second == 0) continue;
        int64_t& v = pc[d.first];
        v += d.second;
        if (d.second > 0 && v > 0) heap.emplace(v, -static_cast<int64_t>(left(d.first)), -static_cast<int64_t>(right(d.first)));
      }
      pc.erase(k);
      where.erase(k);
    }
    return merges;
  }

 private:
  std::unordered_map<std::string, int64_t> counts_;
};

class BpeEncoder {
 public:
  explicit BpeEncoder(const std::vector<std::pair<int32_t, int32_t>>& merges) : n_merges_(static_cast<int32_t>(merges.size())) {
    for (int32_t r = 0; r < n_merges_; ++r) rank_[key(merges[r].first, merges[r].second)] = r;
    bytes_.resize(256 + n_merges_);
    for (int i = 0; i < 256; ++i) bytes_[i] = std::string(1, static_cast<char>(i));
    for (int32_t r = 0; r < n_merges_; ++r) bytes_[256 + r] = bytes_[merges[r].first] + bytes_[merges[r].second];
  }

  int32_t vocab_size() const { return 256 + n_merges_; }

  std::vector<int32_t> encode_chunk(const std::string& chunk) {
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto it = cache_.find(chunk);
      if (it != cache_.end()) return it->second;
    }
    std::vector<int32_t> ids(chunk.size());
    for (size_t i = 0; i < chunk.size(); ++i) ids[i] = static_cast<uint8_t>(chunk[i]);
    while (ids.size() > 1) {
      int32_t best = INT32_MAX;
      for (size_t i = 0; i + 1 < ids.size(); ++i) {
        auto it = rank_.find(key(ids[i], ids[i + 1]));
        if (it != rank_.end() && it->second < best) best = it->second;
      }
      if (best == INT32_MAX) break;
      const int32_t a = merges_left(best), b = merges_right(best), id = 256 + best;
      std::vector<int32_t> out;
      out.reserve(ids.size());
      for (size_t i = 0; i < ids.size();) {
        if (i + 1 < ids.size() && ids[i] == a && ids[i + 1] == b) {
          out.push_back(id);
          i += 2;
        } else {
          out.push_back(ids[i]);
          i += 1;
        }
      }
      ids.swap(out);
    }
    std::lock_guard<std::mutex> lock(mu_);
    if (cache_.size() < kCacheLimit) cache_.emplace(chunk, ids);
    return ids;
  }

  // documents: each a list of pre-split chunks; returns token ids per document (prefix optional)
  std::vector<std::vector<int32_t>> encode_batch(const std::vector<std::vector<std::string>>& docs, int prefix,
                                                 int num_threads) {
    std::vector<std::vector<int32_t>> out(docs.size());
    {
      py::gil_scoped_release release;
      auto work = [&](size_t begin, size_t step) {
        for (size_t d = begin; d < docs.size(); d += step) {
          auto& ids = out[d];
          if (prefix >= 0) ids.push_back(prefix);
          for (const auto& c : docs[d]) {
            const auto t = encode_chunk(c);
            ids.insert(ids.end(), t.begin(), t.end());
          }
        }
      };
      const int n = std::max(1, std::min<int>(num_threads, static_cast<int>(docs.size())));
      std::vector<std::thread> pool;
      for (int t = 1; t < n; ++t) pool.emplace_back(work, static_cast<size_t>(t), static_cast<size_t>(n));
      work(0, static_cast<size_t>(n));
      for (auto& th : pool) th.join();
    }
    return out;
  }

  py::bytes token_bytes(int32_t id) const {
    if (id < 0 || id >= vocab_size()) throw std::out_of_range("token id outside the byte-pair vocabulary");
    return py::bytes(bytes_[id]);
  }

  py::bytes decode(const std::vector<int32_t>& ids) const {
    std::string s;
    for (int32_t id : ids) {
      if (id < 0 || id >= vocab_size()) throw std::out_of_range("token id outside the byte-pair vocabulary");
      s += bytes_[id];
    }
    return py::bytes(s);
  }

 private:
  int32_t merges_left(int32_t r) const { return first_of(r, true); }
  int32_t merges_right(int32_t r) const { return first_of(r, false); }
  int32_t first_of(int32_t r, bool l) const {
    // merge r's parts, recovered from the rank table once and memoized
    if (parts_.empty()) {
      parts_.resize(n_merges_);
      for (const auto& kv : rank_) parts_[kv.second] = {left(kv.first), right(kv.first)};
    }
    return l ? parts_[r].first : parts_[r].second;
  }

  static constexpr size_t kCacheLimit = 1 << 20;
  int32_t n_merges_;
  std::unordered_map<uint64_t, int32_t> rank_;
  std::vector<std::string> bytes_;
  mutable std::vector<std::pair<int32_t, int32_t>> parts_;
  std::unordered_map<std::string, std::vector<int32_t>> cache_;
  std::mutex mu_;
};

class Packer {
 public:
  Packer(int64_t buffer_size, int64_t row_len) : buffer_size_(buffer_size), row_len_(row_len) {
    if (buffer_size <= 0 || row_len <= 0) throw std::invalid_argument("buffer_size and row_len must be positive");
  }
  void add(const std::vector<std::vector<int32_t>>& docs) {
    for (const auto& d : docs) buf_.emplace_back(d.begin(), d.end());
  }
  int64_t size() const { return static_cast<int64_t>(buf_.size()); }
  bool needs_refill() const { return static_cast<int64_t>(buf_.size()) < buffer_size_; }

  // Fill rows of out [rows, row_len] from where the last call stopped. Returns true once every row is
  // complete (the next call starts a new batch); false when the buffer must be refilled first.
  bool pack(py::array_t<int64_t, py::array::c_style> out) {
    auto a = out.mutable_unchecked<2>();
    if (a.shape(1) != row_len_) throw std::invalid_argument("out must be [rows, row_len]");
    const int64_t rows = a.shape(0);
    for (; row_ < rows; ++row_) {
      while (pos_ < row_len_) {
        if (needs_refill()) return false;
        const int64_t remaining = row_len_ - pos_;
        int64_t best = -1, best_len = 0;
        for (int64_t i = 0; i < static_cast<int64_t>(buf_.size()); ++i) {
          const int64_t n = static_cast<int64_t>(buf_[i].size());
          if (best_len < n && n <= remaining) {
            best = i;
            best_len = n;
          }
        }
        int64_t take;
        if (best >= 0) {
          take = best_len;
        } else {  // nothing fits: crop the shortest document to the remaining space
          best = 0;
          for (int64_t i = 1; i < static_cast<int64_t>(buf_.size()); ++i)
            if (buf_[i].size() < buf_[best].size()) best = i;
          take = remaining;
        }
        const auto& d = buf_[best];
        for (int64_t j = 0; j < take; ++j) a(row_, pos_ + j) = d[j];
        pos_ += take;
        buf_.erase(buf_.begin() + best);
      }
      pos_ = 0;
    }
    row_ = 0;
    return true;
  }

 private:
  int64_t buffer_size_, row_len_;
  std::vector<std::vector<int64_t>> buf_;
  int64_t row_ = 0, pos_ = 0;
};

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "Byte-level BPE and the best-fit row packer (C++)";
  py::class_<BpeTrainer>(m, "BpeTrainer")
      .def(py::init<>())
      .def("add_chunks", &BpeTrainer::add_chunks)
      .def("unique_chunks", &BpeTrainer::unique_chunks)
      .def("fit", &BpeTrainer::fit, py::arg("num_merges"));
  py::class_<BpeEncoder>(m, "BpeEncoder")
      .def(py::init<const std::vector<std::pair<int32_t, int32_t>>&>(), py::arg("merges"))
      .def("vocab_size", &BpeEncoder::vocab_size)
      .def("encode_chunk", &BpeEncoder::encode_chunk)
      .def("encode_batch", &BpeEncoder::encode_batch, py::arg("docs"), py::arg("prefix") = -1, py::arg("num_threads") = 8)
      .def("token_bytes", &BpeEncoder::token_bytes)
      .def("decode", &BpeEncoder::decode);
  py::class_<Packer>(m, "Packer")
      .def(py::init<int64_t, int64_t>(), py::arg("buffer_size"), py::arg("row_len"))
      .def("add", &Packer::add)
      .def("size", &Packer::size)
      .def("needs_refill", &Packer::needs_refill)
      .def("pack", &Packer::pack);
}
