// TEST INFRASTRUCTURE ONLY. This directory is the CPU oracle that the tests,
// `__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py` use as
// the checker for the CUDA path. Nothing in `hessboost_b200/` may include,
// link or call it.
//
// It restates, in plain C++, the CPU `tree_method = hist` path of hessboost
// 0.4.9 (a Rust crate that cannot be compiled in this environment). Every
// function cites the reference file:line it follows.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace orc {

// One weighted quantile sketch per numeric feature
// (src/data/sketch.rs:444-639, `WQSketch`).
class WQSketch {
 public:
  WQSketch(size_t n_values, size_t max_bin, bool unit_weights);
  void push(float value, float weight);       // sketch.rs:477 `push`
  void cut_values(std::vector<float>& out);   // sketch.rs:633 `cut_values`

  struct Entry {
    float rmin, rmax, wmin, value;
  };

 private:
  bool queue_push(float value, float weight);
  void flush_queue();
  void push_summary();
  std::vector<Entry> summary(size_t max_size);

  size_t max_bin_;
  size_t limit_size_;
  std::vector<std::pair<float, float>> queue_;
  std::vector<std::vector<Entry>> levels_;
  std::vector<Entry> temp_;
  std::vector<Entry> workspace_;
  size_t num_elements_ = 0;
  bool unit_weights_;
};

size_t summary_budget(size_t max_bin, size_t n);

// Per-feature cut table (src/data/quantile.rs:28 `HistCuts`).
struct Cuts {
  std::vector<uint32_t> feature_offset;  // n_features + 1
  std::vector<float> values;
  size_t n_features() const { return feature_offset.size() - 1; }
  uint32_t num_bins(size_t f) const { return feature_offset[f + 1] - feature_offset[f]; }
};

// `HistCuts::from_dmatrix` for dense row-major input (quantile.rs:65,115).
Cuts cuts_from_dense(const float* x, size_t n_rows, size_t n_cols, const float* weights,
                     size_t max_bin, float missing);

// `HistCuts::bin_of` for a numeric feature: the feature-local bin
// (quantile.rs:285-302): count of cuts <= v, clamped to the last bin.
uint32_t local_bin_of(const Cuts& cuts, size_t f, float v);

// `HistCuts::from_dmatrix` for CSR input (quantile.rs:199, the sparse
// branch): each feature's stored entries, in row order, through its sketch
// (unit weights; every stored value is present).
Cuts cuts_from_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                   size_t n_rows, size_t n_cols, size_t max_bin);

}  // namespace orc
