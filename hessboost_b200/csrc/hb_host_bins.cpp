// Host-side binning of the product library: the cut table
// (HistCuts::from_dmatrix, src/data/quantile.rs:65) and the one-byte
// feature-local bins plus missing bitmap (GHistIndex::from_dmatrix,
// src/data/ghist.rs:213) of a dense row-major f32 matrix, NaN missing.
//
// The cut values come from XGBoost's weighted quantile sketch as the
// reference restates it (src/data/sketch.rs): values stream in row order
// into a queue of 2 * budget entries; each full queue is sorted, folded into
// a summary and carried up a ladder of levels by merge + prune; the final
// merged summary is queried at evenly spaced ranks. Features are sketched
// independently, one per worker thread; every result is a function of the
// feature's values alone.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/hb_backend.h"

namespace {

struct SEntry {
  float rmin, rmax, wmin, value;
  float next_rmin() const { return rmin + wmin; }   // sketch.rs:46 rmin_next
  float prev_rmax() const { return rmax - wmin; }   // sketch.rs:52 rmax_prev
};
using Summary = std::vector<SEntry>;

uint32_t order_key(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  return (b >> 31) ? ~b : (b | 0x80000000u);
}

// SketchSummaryBudget (sketch.rs:58-85): smallest per-level size over a
// ladder of levels holding n values at rank resolution 1 / min(max_bin, n),
// oversampled twice.
size_t level_budget(size_t max_bin, size_t n) {
  const double eps = 1.0 / (double)std::min(max_bin, std::max<size_t>(n, 1));
  if (n == 0) return 1;
  for (uint32_t levels = 1;; ++levels) {
    size_t size = std::min((size_t)std::ceil((double)levels / (eps / 2.0)) + 1, n);
    if ((size_t(1) << levels) * size >= n) return size;
  }
}

// Fold sorted (value, weight) pairs: equal values into one entry.
void fold_sorted(const std::vector<std::pair<float, float>>& in, Summary& out) {
  out.clear();
  float acc = 0.0f;
  for (size_t i = 0; i < in.size();) {
    const float v = in[i].first;
    float w = in[i].second;
    size_t j = i + 1;
    for (; j < in.size() && in[j].first == v; ++j) w += in[j].second;
    out.push_back(SEntry{acc, acc + w, w, v});
    acc += w;
    i = j;
  }
}

// Shrink to at most `cap` entries by answering evenly spaced rank queries
// (WQSummary::SetPrune, sketch.rs:128).
void shrink(Summary& s, size_t cap) {
  if (cap == 0) {
    s.clear();
    return;
  }
  const size_t n = s.size();
  if (n <= cap) return;
  if (cap == 1) {
    s.resize(1);
    return;
  }
  const float lo = s[0].rmax;
  const float span = s[n - 1].rmin - s[0].rmax;
  const size_t steps = cap - 1;
  const SEntry last = s[n - 1];
  SEntry a = s[1], b = s[2];
  size_t kept = 1, cursor = 1, prev = 0;
  for (size_t k = 1; k < steps; ++k) {
    const float target = 2.0f * (((float)k * span) / (float)steps + lo);
    while (cursor < n - 1 && target >= b.rmax + b.rmin) {
      ++cursor;
      a = b;
      if (cursor < n - 1) b = s[cursor + 1];
    }
    if (cursor == n - 1) break;
    if (target < a.next_rmin() + b.prev_rmax()) {
      if (cursor != prev) {
        s[kept++] = a;
        prev = cursor;
      }
    } else if (cursor + 1 != prev) {
      s[kept++] = b;
      prev = cursor + 1;
    }
  }
  if (prev != n - 1) s[kept++] = last;
  s.resize(kept);
}

// WQSummary::SetCombine (sketch.rs:217) as one sequential merge, then
// FixError (:180).
void merge_into(Summary& self, const Summary& other, Summary& tmp) {
  if (other.empty()) return;
  if (self.empty()) {
    self = other;
    return;
  }
  tmp.clear();
  size_t i = 0, j = 0;
  float a_next = 0.0f, b_next = 0.0f;
  while (i < self.size() && j < other.size()) {
    const SEntry& x = self[i];
    const SEntry& y = other[j];
    if (x.value == y.value) {
      tmp.push_back(SEntry{x.rmin + y.rmin, x.rmax + y.rmax, x.wmin + y.wmin, x.value});
      a_next = x.next_rmin();
      b_next = y.next_rmin();
      ++i;
      ++j;
    } else if (x.value < y.value) {
      tmp.push_back(SEntry{x.rmin + b_next, x.rmax + y.prev_rmax(), x.wmin, x.value});
      a_next = x.next_rmin();
      ++i;
    } else {
      tmp.push_back(SEntry{y.rmin + a_next, y.rmax + x.prev_rmax(), y.wmin, y.value});
      b_next = y.next_rmin();
      ++j;
    }
  }
  for (const float tail = other.back().rmax; i < self.size(); ++i) {
    const SEntry& x = self[i];
    tmp.push_back(SEntry{x.rmin + b_next, x.rmax + tail, x.wmin, x.value});
  }
  for (const float tail = self.back().rmax; j < other.size(); ++j) {
    const SEntry& y = other[j];
    tmp.push_back(SEntry{y.rmin + a_next, y.rmax + tail, y.wmin, y.value});
  }
  float pmin = 0.0f, pmax = 0.0f;
  for (SEntry& e : tmp) {
    if (e.rmin < pmin) e.rmin = pmin; else pmin = e.rmin;
    if (e.rmax < pmax) e.rmax = pmax;
    if (e.rmax < e.next_rmin()) e.rmax = e.next_rmin();
    pmax = e.rmax;
  }
  std::swap(self, tmp);
}

// Cut values of a summary (WQSummary::QueryCutValues, sketch.rs:427).
void query(const Summary& s, size_t max_bin, std::vector<float>& out) {
  if (s.empty()) {
    out.push_back(1e-5f);
    return;
  }
  const size_t n = s.size();
  auto skip_le = [&](size_t at, float v) {
    while (at < n && s[at].value <= v) ++at;
    return at;
  };
  float last = s[0].value;
  size_t nv = skip_le(1, last);
  if (n <= max_bin) {
    for (; nv < n; nv = skip_le(nv + 1, last)) {
      last = s[nv].value;
      out.push_back(last);
    }
  } else {
    const double total = (double)s[n - 1].rmax;
    size_t q = 0;
    for (size_t i = 1; i < max_bin; ++i) {
      const double r2 = 2.0 * ((double)i * total / (double)max_bin);
      while (q < n - 2 && r2 >= (double)(s[q + 1].rmin + s[q + 1].rmax)) ++q;
      float v = r2 < (double)(s[q].next_rmin() + s[q + 1].prev_rmax()) ? s[q].value : s[q + 1].value;
      if (v <= last) {
        nv = skip_le(nv, last);
        if (nv == n) break;
        v = s[nv].value;
      } else if (nv < n && s[nv].value <= v) {
        nv = skip_le(nv + 1, v);
      }
      out.push_back(v);
      last = v;
    }
  }
  const float top = s[n - 1].value;
  out.push_back(top + (std::fabs(top) + 1e-5f));
}

// One feature's streaming sketch (WQuantileSketch with unit weights).
class FeatureSketch {
 public:
  FeatureSketch(size_t present, size_t max_bin)
      : max_bin_(max_bin), budget_(level_budget(max_bin, present)) {}

  void add(float v) {
    ++count_;
    if (!queue_.empty() && queue_.back().first == v) {
      queue_.back().second += 1.0f;
      return;
    }
    if (queue_.size() == 2 * budget_) flush();
    queue_.emplace_back(v, 1.0f);
  }

  void cuts(std::vector<float>& out) {
    const size_t final_budget = level_budget(max_bin_, count_);
    flush();
    const size_t cap = std::max(final_budget, budget_);
    Summary all, tmp;
    for (const Summary& lv : ladder_) {
      merge_into(all, lv, tmp);
      shrink(all, cap);
    }
    shrink(all, final_budget);
    query(all, std::min(all.size(), max_bin_), out);
  }

 private:
  void flush() {
    std::stable_sort(queue_.begin(), queue_.end(), [](const auto& a, const auto& b) {
      return order_key(a.first) < order_key(b.first);
    });
    fold_sorted(queue_, carry_);
    queue_.clear();
    size_t l = 0;
    for (;; ++l) {
      if (ladder_.size() <= l) ladder_.emplace_back();
      shrink(carry_, budget_);
      merge_into(carry_, ladder_[l], tmp_);
      ladder_[l].clear();
      if (carry_.size() <= budget_) break;
    }
    std::swap(ladder_[l], carry_);
  }

  size_t max_bin_, budget_;
  size_t count_ = 0;
  std::vector<std::pair<float, float>> queue_;
  std::vector<Summary> ladder_;
  Summary carry_, tmp_;
};

template <class F>
void parallel_for(uint32_t n, F&& fn) {
  unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  unsigned workers = std::min<unsigned>(hw, n);
  std::atomic<uint32_t> next{0};
  std::vector<std::thread> pool;
  for (unsigned w = 0; w + 1 < workers; ++w)
    pool.emplace_back([&] {
      for (uint32_t i; (i = next.fetch_add(1)) < n;) fn(i);
    });
  for (uint32_t i; (i = next.fetch_add(1)) < n;) fn(i);
  for (auto& t : pool) t.join();
}

}  // namespace

extern "C" {

hb_status hb_cuts_dense(const float* x, uint64_t n_rows, uint32_t n_cols, uint32_t max_bin,
                        uint32_t* feature_offset, float* cut_values, uint64_t cap,
                        uint64_t* total) {
  if (!x || !feature_offset || !cut_values || !total || n_cols == 0 || max_bin == 0)
    return HB_INVALID_ARGUMENT;
  std::vector<std::vector<float>> per(n_cols);
  parallel_for(n_cols, [&](uint32_t f) {
    size_t present = 0;
    for (uint64_t r = 0; r < n_rows; ++r) present += !std::isnan(x[r * n_cols + f]);
    FeatureSketch sk(present, max_bin);
    for (uint64_t r = 0; r < n_rows; ++r) {
      const float v = x[r * n_cols + f];
      if (!std::isnan(v)) sk.add(v);
    }
    sk.cuts(per[f]);
  });
  uint64_t at = 0;
  feature_offset[0] = 0;
  for (uint32_t f = 0; f < n_cols; ++f) {
    if (at + per[f].size() > cap) return HB_REFUSED;
    std::copy(per[f].begin(), per[f].end(), cut_values + at);
    at += per[f].size();
    feature_offset[f + 1] = (uint32_t)at;
  }
  *total = at;
  return HB_OK;
}

hb_status hb_bin_dense(const float* x, uint64_t n_rows, uint32_t n_cols,
                       const uint32_t* feature_offset, const float* cut_values, uint8_t* columns,
                       uint64_t* missing, int32_t* dense) {
  if (!x || !feature_offset || !cut_values || !columns || !dense) return HB_INVALID_ARGUMENT;
  for (uint32_t f = 0; f < n_cols; ++f)
    if (feature_offset[f + 1] - feature_offset[f] > 256) return HB_REFUSED;
  const uint64_t words = (n_rows + 63) / 64;
  std::atomic<int> any_missing{0};
  parallel_for(n_cols, [&](uint32_t f) {
    const float* c = cut_values + feature_offset[f];
    const uint32_t nb = feature_offset[f + 1] - feature_offset[f];
    uint64_t* mw = missing ? missing + (uint64_t)f * words : nullptr;
    if (mw) std::fill(mw, mw + words, 0ull);
    bool seen = false;
    for (uint64_t r = 0; r < n_rows; ++r) {
      const float v = x[r * n_cols + f];
      if (std::isnan(v)) {
        columns[(uint64_t)f * n_rows + r] = 0;
        if (mw) mw[r >> 6] |= 1ull << (r & 63);
        seen = true;
        continue;
      }
      // bin = #{cuts <= v}, clamped to the last bin (quantile.rs:285)
      const uint32_t k = (uint32_t)(std::upper_bound(c, c + nb, v) - c);
      columns[(uint64_t)f * n_rows + r] = (uint8_t)std::min(k, nb - 1);
    }
    if (seen) any_missing.store(1);
  });
  *dense = any_missing.load() ? 0 : 1;
  return HB_OK;
}

// DMatrix::from_csr's checks (src/data/dmatrix.rs:459): offsets start at 0
// and ascend to nnz, columns in range, values finite, no column twice in a
// row. `seen` is scratch of n_cols words.
static bool csr_row_ok(const uint64_t* indptr, const uint32_t* indices, const float* values,
                       uint64_t r, uint32_t n_cols, std::vector<uint64_t>& seen, uint64_t stamp) {
  for (uint64_t j = indptr[r]; j < indptr[r + 1]; ++j) {
    const uint32_t c = indices[j];
    if (c >= n_cols || !std::isfinite(values[j]) || seen[c] == stamp) return false;
    seen[c] = stamp;
  }
  return true;
}

static hb_status check_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                           uint64_t n_rows, uint32_t n_cols) {
  if (!indptr || n_rows == 0 || n_cols == 0 || indptr[0] != 0) return HB_INVALID_ARGUMENT;
  for (uint64_t r = 0; r < n_rows; ++r)
    if (indptr[r + 1] < indptr[r]) return HB_INVALID_ARGUMENT;
  if (indptr[n_rows] && (!indices || !values)) return HB_INVALID_ARGUMENT;
  std::atomic<int> bad{0};
  const uint32_t blocks = (uint32_t)std::min<uint64_t>((n_rows + 65535) / 65536, 1u << 30);
  parallel_for(blocks, [&](uint32_t b) {
    std::vector<uint64_t> seen(n_cols, 0);
    const uint64_t r0 = (uint64_t)b * 65536, r1 = std::min<uint64_t>(n_rows, r0 + 65536);
    for (uint64_t r = r0; r < r1 && !bad.load(std::memory_order_relaxed); ++r)
      if (!csr_row_ok(indptr, indices, values, r, n_cols, seen, r + 1)) bad.store(1);
  });
  return bad.load() ? HB_INVALID_ARGUMENT : HB_OK;
}

// HistCuts::from_dmatrix of a CSR matrix (quantile.rs:199, the sparse
// branch): each feature's stored entries in row order through its sketch.
hb_status hb_cuts_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                      uint64_t n_rows, uint32_t n_cols, uint32_t max_bin, uint32_t* feature_offset,
                      float* cut_values, uint64_t cap, uint64_t* total) {
  if (!feature_offset || !cut_values || !total || max_bin == 0) return HB_INVALID_ARGUMENT;
  hb_status st = check_csr(indptr, indices, values, n_rows, n_cols);
  if (st != HB_OK) return st;
  // the CSC view: every column's values in row order (a counting sort)
  const uint64_t nnz = indptr[n_rows];
  std::vector<uint64_t> start(n_cols + 1, 0);
  for (uint64_t j = 0; j < nnz; ++j) ++start[indices[j] + 1];
  for (uint32_t c = 0; c < n_cols; ++c) start[c + 1] += start[c];
  std::vector<float> csc(nnz);
  {
    std::vector<uint64_t> at(start.begin(), start.end() - 1);
    for (uint64_t r = 0; r < n_rows; ++r)
      for (uint64_t j = indptr[r]; j < indptr[r + 1]; ++j) csc[at[indices[j]]++] = values[j];
  }
  std::vector<std::vector<float>> per(n_cols);
  parallel_for(n_cols, [&](uint32_t f) {
    FeatureSketch sk(start[f + 1] - start[f], max_bin);
    for (uint64_t j = start[f]; j < start[f + 1]; ++j) sk.add(csc[j]);
    sk.cuts(per[f]);
  });
  uint64_t at = 0;
  feature_offset[0] = 0;
  for (uint32_t f = 0; f < n_cols; ++f) {
    if (at + per[f].size() > cap) return HB_REFUSED;
    std::copy(per[f].begin(), per[f].end(), cut_values + at);
    at += per[f].size();
    feature_offset[f + 1] = (uint32_t)at;
  }
  *total = at;
  return HB_OK;
}

// GHistIndex::from_dmatrix for CSR (ghist.rs:213): every stored entry's
// global bin, a row's bins ascending (feature order), row_ptr as indptr.
// `dense` = every row holds every feature.
hb_status hb_bin_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                     uint64_t n_rows, uint32_t n_cols, const uint32_t* feature_offset,
                     const float* cut_values, uint64_t* row_ptr, uint32_t* row_bins,
                     int32_t* dense) {
  if (!feature_offset || !cut_values || !row_ptr || !dense) return HB_INVALID_ARGUMENT;
  hb_status st = check_csr(indptr, indices, values, n_rows, n_cols);
  if (st != HB_OK) return st;
  const uint64_t nnz = indptr[n_rows];
  if (nnz && !row_bins) return HB_INVALID_ARGUMENT;
  for (uint32_t f = 0; f < n_cols; ++f)
    if (feature_offset[f + 1] <= feature_offset[f] || feature_offset[f + 1] - feature_offset[f] > 65535)
      return HB_REFUSED;
  std::copy(indptr, indptr + n_rows + 1, row_ptr);
  std::atomic<int> short_row{0};
  const uint32_t blocks = (uint32_t)((n_rows + 65535) / 65536);
  parallel_for(blocks, [&](uint32_t b) {
    const uint64_t r0 = (uint64_t)b * 65536, r1 = std::min<uint64_t>(n_rows, r0 + 65536);
    bool any_short = false;
    for (uint64_t r = r0; r < r1; ++r) {
      const uint64_t a = indptr[r], e = indptr[r + 1];
      any_short |= (e - a) != n_cols;
      for (uint64_t j = a; j < e; ++j) {
        const uint32_t f = indices[j];
        const float* c = cut_values + feature_offset[f];
        const uint32_t nb = feature_offset[f + 1] - feature_offset[f];
        const uint32_t k = (uint32_t)(std::upper_bound(c, c + nb, values[j]) - c);
        row_bins[j] = feature_offset[f] + std::min(k, nb - 1);
      }
      std::sort(row_bins + a, row_bins + e);
    }
    if (any_short) short_row.store(1);
  });
  *dense = short_row.load() ? 0 : 1;
  return HB_OK;
}

}  // extern "C"
