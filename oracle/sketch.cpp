// TEST INFRASTRUCTURE ONLY (see oracle_internal.h).
//
// Restatement of hessboost's weighted quantile sketch, src/data/sketch.rs
// (itself XGBoost's WQuantileSketch), and of the cut construction in
// src/data/quantile.rs. Serial and written for clarity, not speed.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "oracle_internal.h"

namespace orc {

namespace {

using Entry = WQSketch::Entry;

inline float rmin_next(const Entry& e) { return e.rmin + e.wmin; }   // sketch.rs:46
inline float rmax_prev(const Entry& e) { return e.rmax - e.wmin; }   // sketch.rs:52

// Monotone u32 key of an f32 (src/data/sort.rs:14 `sort_key`).
inline uint32_t sort_key(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// sketch.rs:58 `sketch_epsilon`
double sketch_epsilon(size_t max_bin, size_t n_samples) {
  size_t n = std::max<size_t>(n_samples, 1);
  return 1.0 / (double)std::min(max_bin, n);
}

// sketch.rs:65 `limit_size_level`
size_t limit_size_level(size_t maxn, double eps) {
  if (maxn == 0) return 1;
  double internal_eps = eps / 2.0;
  for (uint32_t nlevel = 1;; ++nlevel) {
    double c = std::ceil((double)nlevel / internal_eps);
    size_t limit = std::min((size_t)c + 1, maxn);
    if ((size_t(1) << nlevel) * limit >= maxn) return limit;
  }
}

// sketch.rs:88 `set_from_sorted`
void set_from_sorted(const std::vector<std::pair<float, float>>& q, std::vector<Entry>& out) {
  out.clear();
  float wsum = 0.0f;
  size_t i = 0;
  while (i < q.size()) {
    float value = q[i].first;
    float w = q[i].second;
    size_t j = i + 1;
    while (j < q.size() && q[j].first == value) {
      w += q[j].second;
      ++j;
    }
    out.push_back(Entry{wsum, wsum + w, w, value});
    wsum += w;
    i = j;
  }
}

// sketch.rs:128 `set_prune`
void set_prune(std::vector<Entry>& data, size_t maxsize) {
  if (maxsize == 0) {
    data.clear();
    return;
  }
  size_t src_size = data.size();
  if (src_size <= maxsize) return;
  if (maxsize == 1) {
    data.resize(1);
    return;
  }
  Entry* d = data.data();
  float begin = d[0].rmax;
  float range = d[src_size - 1].rmin - d[0].rmax;
  size_t n = maxsize - 1;
  Entry tail = d[src_size - 1];
  Entry left = d[1];
  Entry right = d[2];
  size_t len = 1;
  size_t i = 1, lastidx = 0;
  for (size_t k = 1; k < n; ++k) {
    float dx2 = 2.0f * (((float)k * range) / (float)n + begin);
    while (i < src_size - 1 && dx2 >= right.rmax + right.rmin) {
      ++i;
      left = right;
      if (i < src_size - 1) right = d[i + 1];
    }
    if (i == src_size - 1) break;
    if (dx2 < rmin_next(left) + rmax_prev(right)) {
      if (i != lastidx) {
        d[len++] = left;
        lastidx = i;
      }
    } else if (i + 1 != lastidx) {
      d[len++] = right;
      lastidx = i + 1;
    }
  }
  if (lastidx != src_size - 1) d[len++] = tail;
  data.resize(len);
}

// sketch.rs:180 `fix_error`
void fix_error(std::vector<Entry>& data) {
  float prev_rmin = 0.0f, prev_rmax = 0.0f;
  for (Entry& e : data) {
    if (e.rmin < prev_rmin) {
      e.rmin = prev_rmin;
    } else {
      prev_rmin = e.rmin;
    }
    if (e.rmax < prev_rmax) e.rmax = prev_rmax;
    float rn = rmin_next(e);
    if (e.rmax < rn) e.rmax = rn;
    prev_rmax = e.rmax;
  }
}

// sketch.rs:217 `set_combine`, in the one-pass form its own test pins it to
// (sketch.rs:785 `set_combine_one_pass`).
void set_combine(std::vector<Entry>& self, const std::vector<Entry>& other,
                 std::vector<Entry>& workspace) {
  if (other.empty()) return;
  if (self.empty()) {
    self = other;
    return;
  }
  workspace.clear();
  const std::vector<Entry>& a = self;
  const std::vector<Entry>& b = other;
  size_t ia = 0, ib = 0;
  float aprev = 0.0f, bprev = 0.0f;
  while (ia < a.size() && ib < b.size()) {
    const Entry& ea = a[ia];
    const Entry& eb = b[ib];
    if (ea.value == eb.value) {
      workspace.push_back(Entry{ea.rmin + eb.rmin, ea.rmax + eb.rmax, ea.wmin + eb.wmin, ea.value});
      aprev = rmin_next(ea);
      bprev = rmin_next(eb);
      ++ia;
      ++ib;
    } else if (ea.value < eb.value) {
      workspace.push_back(Entry{ea.rmin + bprev, ea.rmax + rmax_prev(eb), ea.wmin, ea.value});
      aprev = rmin_next(ea);
      ++ia;
    } else {
      workspace.push_back(Entry{eb.rmin + aprev, eb.rmax + rmax_prev(ea), eb.wmin, eb.value});
      bprev = rmin_next(eb);
      ++ib;
    }
  }
  if (ia < a.size()) {
    float brmax = b.back().rmax;
    for (; ia < a.size(); ++ia) {
      const Entry& ea = a[ia];
      workspace.push_back(Entry{ea.rmin + bprev, ea.rmax + brmax, ea.wmin, ea.value});
    }
  }
  if (ib < b.size()) {
    float armax = a.back().rmax;
    for (; ib < b.size(); ++ib) {
      const Entry& eb = b[ib];
      workspace.push_back(Entry{eb.rmin + aprev, eb.rmax + armax, eb.wmin, eb.value});
    }
  }
  fix_error(workspace);
  std::swap(self, workspace);
}

// sketch.rs:427 `query_cut_values`
void query_cut_values(const std::vector<Entry>& data, size_t max_bin, std::vector<float>& out) {
  if (data.empty()) {
    out.push_back(1e-5f);
    return;
  }
  size_t n = data.size();
  auto advance = [&](size_t cursor, float value) {
    while (cursor < n && data[cursor].value <= value) ++cursor;
    return cursor;
  };
  float last_cut = data[0].value;
  size_t next_value = advance(1, last_cut);
  if (n <= max_bin) {
    while (next_value < n) {
      float cpt = data[next_value].value;
      out.push_back(cpt);
      last_cut = cpt;
      next_value = advance(next_value + 1, last_cut);
    }
  } else {
    double total = (double)data[n - 1].rmax;
    size_t q = 0;
    for (size_t i = 1; i < max_bin; ++i) {
      double rank2 = 2.0 * ((double)i * total / (double)max_bin);
      while (q < n - 2 && rank2 >= (double)(data[q + 1].rmin + data[q + 1].rmax)) ++q;
      const Entry& queried =
          rank2 < (double)(rmin_next(data[q]) + rmax_prev(data[q + 1])) ? data[q] : data[q + 1];
      float cpt = queried.value;
      if (cpt <= last_cut) {
        next_value = advance(next_value, last_cut);
        if (next_value == n) break;
        cpt = data[next_value].value;
      } else if (next_value < n && data[next_value].value <= cpt) {
        next_value = advance(next_value + 1, cpt);
      }
      out.push_back(cpt);
      last_cut = cpt;
    }
  }
  float cpt = data[n - 1].value;
  out.push_back(cpt + (std::fabs(cpt) + 1e-5f));
}

}  // namespace

// sketch.rs:83 `summary_budget`
size_t summary_budget(size_t max_bin, size_t n) {
  return limit_size_level(n, sketch_epsilon(max_bin, n));
}

WQSketch::WQSketch(size_t n_values, size_t max_bin, bool unit_weights)
    : max_bin_(max_bin), limit_size_(summary_budget(max_bin, n_values)), unit_weights_(unit_weights) {}

// sketch.rs:477 `push`
void WQSketch::push(float value, float weight) {
  if (weight == 0.0f) return;
  ++num_elements_;
  if (!queue_push(value, weight)) {
    flush_queue();
    queue_push(value, weight);
  }
}

// sketch.rs:520 `queue_push`
bool WQSketch::queue_push(float value, float weight) {
  if (!queue_.empty() && queue_.back().first == value) {
    queue_.back().second += weight;
    return true;
  }
  if (queue_.size() == 2 * limit_size_) return false;
  queue_.emplace_back(value, weight);
  return true;
}

// sketch.rs:542 `flush_queue`. Both the reference's radix sort (unit
// weights) and its comparison sort order by the f32 total order; equal
// values then fold in `set_from_sorted`. A stable sort is used here: for
// unit weights the folded sums are whole numbers and any order gives the
// same bits.
void WQSketch::flush_queue() {
  std::stable_sort(queue_.begin(), queue_.end(),
                   [](const std::pair<float, float>& a, const std::pair<float, float>& b) {
                     return sort_key(a.first) < sort_key(b.first);
                   });
  set_from_sorted(queue_, temp_);
  queue_.clear();
  push_summary();
}

// sketch.rs:575 `push_summary`
void WQSketch::push_summary() {
  size_t l = 0;
  for (;;) {
    if (levels_.size() <= l) levels_.emplace_back();
    set_prune(temp_, limit_size_);
    set_combine(temp_, levels_[l], workspace_);
    levels_[l].clear();
    if (temp_.size() <= limit_size_) break;
    ++l;
  }
  std::swap(levels_[l], temp_);
}

// sketch.rs:607 `summary`
std::vector<WQSketch::Entry> WQSketch::summary(size_t max_size) {
  flush_queue();
  size_t prune_size = std::max(max_size, limit_size_);
  std::vector<Entry> out;
  for (const auto& level : levels_) {
    set_combine(out, level, workspace_);
    set_prune(out, prune_size);
  }
  set_prune(out, max_size);
  return out;
}

// sketch.rs:633 `cut_values`
void WQSketch::cut_values(std::vector<float>& out) {
  size_t budget = summary_budget(max_bin_, num_elements_);
  std::vector<Entry> s = summary(budget);
  query_cut_values(s, std::min(s.size(), max_bin_), out);
}

static inline bool is_missing(float v, float missing) {
  return std::isnan(missing) ? std::isnan(v) : v == missing;  // src/data/dmatrix.rs:30
}

// quantile.rs:115 `HistCuts::build`, dense input, streaming ingest
// (`Ingest { sorted: false }`): every feature's present values in row order.
Cuts cuts_from_dense(const float* x, size_t n_rows, size_t n_cols, const float* weights,
                     size_t max_bin, float missing) {
  Cuts cuts;
  cuts.feature_offset.push_back(0);
  std::vector<std::vector<float>> per(n_cols);
  // Features are independent sketches (quantile.rs:188 runs them in parallel too).
#pragma omp parallel for schedule(dynamic, 1)
  for (long long f = 0; f < (long long)n_cols; ++f) {
    size_t present = 0;
    for (size_t r = 0; r < n_rows; ++r) present += !is_missing(x[r * n_cols + f], missing);
    WQSketch sketch(present, max_bin, weights == nullptr);
    for (size_t r = 0; r < n_rows; ++r) {
      float v = x[r * n_cols + f];
      if (is_missing(v, missing)) continue;
      sketch.push(v, weights ? weights[r] : 1.0f);
    }
    sketch.cut_values(per[f]);
  }
  for (size_t f = 0; f < n_cols; ++f) {
    cuts.values.insert(cuts.values.end(), per[f].begin(), per[f].end());
    cuts.feature_offset.push_back((uint32_t)cuts.values.size());
  }
  return cuts;
}

Cuts cuts_from_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                   size_t n_rows, size_t n_cols, size_t max_bin) {
  // DMatrix::to_csc: every column's values in row order
  std::vector<size_t> start(n_cols + 1, 0);
  const size_t nnz = indptr[n_rows];
  for (size_t j = 0; j < nnz; ++j) ++start[indices[j] + 1];
  for (size_t c = 0; c < n_cols; ++c) start[c + 1] += start[c];
  std::vector<float> csc(nnz);
  {
    std::vector<size_t> at(start.begin(), start.end() - 1);
    for (size_t r = 0; r < n_rows; ++r)
      for (uint64_t j = indptr[r]; j < indptr[r + 1]; ++j) csc[at[indices[j]]++] = values[j];
  }
  Cuts cuts;
  cuts.feature_offset.push_back(0);
  std::vector<std::vector<float>> per(n_cols);
#pragma omp parallel for schedule(dynamic, 1)
  for (long long f = 0; f < (long long)n_cols; ++f) {
    WQSketch sketch(start[f + 1] - start[f], max_bin, true);
    for (size_t j = start[f]; j < start[f + 1]; ++j) sketch.push(csc[j], 1.0f);
    sketch.cut_values(per[f]);
  }
  for (size_t f = 0; f < n_cols; ++f) {
    cuts.values.insert(cuts.values.end(), per[f].begin(), per[f].end());
    cuts.feature_offset.push_back((uint32_t)cuts.values.size());
  }
  return cuts;
}

// quantile.rs:285 `bin_of` (numeric), made feature-local.
uint32_t local_bin_of(const Cuts& cuts, size_t f, float v) {
  const float* begin = cuts.values.data() + cuts.feature_offset[f];
  size_t n = cuts.num_bins(f);
  size_t count = (size_t)(std::upper_bound(begin, begin + n, v,
                                           [](float value, float c) { return value < c; }) -
                          begin);
  return (uint32_t)std::min(count, n ? n - 1 : 0);
}

}  // namespace orc
