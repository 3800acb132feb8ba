// TEST INFRASTRUCTURE ONLY (see oracle_internal.h).
//
// CPU restatement of hessboost 0.4.9's `tree_method = hist` training and
// prediction, for the known-answer tests and as the checker of the CUDA
// path. Two summation modes:
//   * f64 (fixed_point = 0): the reference's f64 histogram sums in the order
//     CpuBackend::build forms them (src/tree/hist/mod.rs:420-607), so the
//     trees match the reference's bit for bit (pinned by the saved-model
//     fixtures under tests/golden/).
//   * fixed point (fixed_point = 1): every gradient rounded once to an
//     int64 multiple of a power of two and summed exactly; this is the
//     arithmetic the CUDA path uses, so the two must agree bit for bit.
#include <algorithm>
#include <cassert>
#include <functional>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <numeric>
#include <type_traits>
#include <vector>

#include "oracle.h"
#include "oracle_internal.h"

#ifdef _OPENMP
#include <omp.h>
#endif

namespace orc {
namespace {

constexpr double K_RT_EPS = 1e-6;         // src/lib.rs:366
constexpr float K_RT_EPS_F32 = 1e-6f;     // src/lib.rs:369
constexpr float MIN_HESS = 1e-16f;        // src/objective/mod.rs:150
constexpr size_t ROWS_PER_TASK = 4096;    // src/tree/hist/mod.rs:387
constexpr size_t PARALLEL_THRESHOLD = 2 * ROWS_PER_TASK;  // :389
constexpr size_t GATHER_MAX_ROWS = size_t(1) << 18;       // :394
constexpr float BELOW_ALL_VALUES = -3.40282347e+38f;      // builder/mod.rs:308 (f32::MIN)

inline bool is_missing(float v) { return std::isnan(v); }

// ---------------------------------------------------------------------------
// Binned index (src/data/ghist.rs:195 `GHistIndex`): feature-local bins per
// cell, the missing flag, and the index-level `dense` flag (every row holds
// every feature, ghist.rs:205-208).
// A CSR index (ghist.rs:6-21 `rows`: global bins row by row, no columns)
// keeps only the stored cells: row_bins ascending within a row.
// A dense index keeps each cell's local bin twice, row-major for the
// histograms (one row's cells together) and feature-major for the partition
// (one feature's cells together); a missing cell holds kMissingBin.
constexpr uint16_t kMissingBin = 0xFFFF;

struct Index {
  size_t n_rows = 0, n_cols = 0;
  Cuts cuts;
  std::vector<uint16_t> local;  // [row][feature] local bin or kMissingBin
  std::vector<uint16_t> cols;   // [feature][row], the same bins
  bool dense = true;
  bool csr = false;
  std::vector<uint64_t> row_ptr;   // CSR: n_rows + 1
  std::vector<uint32_t> row_bins;  // CSR: global bins
  // The cell's local bin, or false when it is missing.
  bool cell(size_t r, size_t f, uint32_t& bin) const {
    if (!csr) {
      const uint16_t b = cols[f * n_rows + r];
      if (b == kMissingBin) return false;
      bin = b;
      return true;
    }
    const uint32_t lo = cuts.feature_offset[f], hi = cuts.feature_offset[f + 1];
    const uint32_t* b = row_bins.data() + row_ptr[r];
    const uint32_t* e = row_bins.data() + row_ptr[r + 1];
    const uint32_t* it = std::lower_bound(b, e, lo);
    if (it == e || *it >= hi) return false;
    bin = *it - lo;
    return true;
  }
};

// GHistIndex::from_dmatrix of CSR input: each stored value's global bin.
Index make_index_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                     size_t n, size_t nc, Cuts cuts) {
  Index ix;
  ix.n_rows = n;
  ix.n_cols = nc;
  ix.cuts = std::move(cuts);
  ix.csr = true;
  ix.row_ptr.assign(indptr, indptr + n + 1);
  ix.row_bins.assign(indptr[n], 0);
  bool full = true;
  for (size_t r = 0; r < n; ++r) {
    full = full && indptr[r + 1] - indptr[r] == nc;
    for (uint64_t j = indptr[r]; j < indptr[r + 1]; ++j)
      ix.row_bins[j] = ix.cuts.feature_offset[indices[j]] + local_bin_of(ix.cuts, indices[j], values[j]);
    std::sort(ix.row_bins.begin() + indptr[r], ix.row_bins.begin() + indptr[r + 1]);
  }
  ix.dense = full;
  return ix;
}

Index make_index(const float* x, size_t n, size_t nc, Cuts cuts) {
  Index ix;
  ix.n_rows = n;
  ix.n_cols = nc;
  ix.cuts = std::move(cuts);
  for (size_t f = 0; f < nc; ++f) assert(ix.cuts.num_bins(f) < kMissingBin);  // u16 local bins
  ix.local.assign(n * nc, 0);
  ix.cols.assign(n * nc, 0);
  bool any_missing = false;
#pragma omp parallel for schedule(static) reduction(|| : any_missing)
  for (long long r = 0; r < (long long)n; ++r) {
    for (size_t f = 0; f < nc; ++f) {
      float v = x[r * nc + f];
      uint16_t b = kMissingBin;
      if (is_missing(v)) {
        any_missing = true;
      } else {
        b = (uint16_t)local_bin_of(ix.cuts, f, v);
      }
      ix.local[r * nc + f] = b;
      ix.cols[f * n + r] = b;
    }
  }
  ix.dense = !any_missing;
  return ix;
}

// ---------------------------------------------------------------------------
// Gradient statistics in the two summation modes.
struct GS {  // src/tree/gain.rs:21 `GradStats`
  double grad = 0.0, hess = 0.0;
};
struct IS {  // fixed-point sums
  int64_t grad = 0, hess = 0;
};

struct GradPair {
  float grad, hess;
};

inline double pow2(int e) { return std::ldexp(1.0, e); }

struct Params {
  int objective, n_outputs, max_depth, max_leaves, grow_policy, max_bin;
  float eta;
  double lambda, alpha, gamma, mcw, mds;  // RegParams: every value rounded to f32 (gain.rs:83)
  float spw;
  bool fixed;
  std::vector<int8_t> mono;  // constraints.rs:12 `MonotoneConstraints` (+1, -1, 0)
  int8_t dir(size_t f) const { return f < mono.size() ? mono[f] : 0; }  // constraints.rs:37
};

// constraints.rs:44 `Bounds`: a node's leaf-weight interval.
struct Bounds {
  double lower = -INFINITY, upper = INFINITY;
  double clamp(double w) const { return std::min(std::max(w, lower), upper); }  // f64::clamp
};

// f64::midpoint (Rust core): (a + b) / 2 without intermediate overflow.
inline double midpoint(double a, double b) {
  const double lo = DBL_MIN * 2.0, hi = DBL_MAX / 2.0;
  const double aa = std::fabs(a), ab = std::fabs(b);
  if (aa <= hi && ab <= hi) return (a + b) / 2.0;
  if (aa < lo) return a + b / 2.0;
  if (ab < lo) return a / 2.0 + b;
  return a / 2.0 + b / 2.0;
}

// constraints.rs:82 `child_bounds`
inline std::pair<Bounds, Bounds> child_bounds(Bounds parent, int dir, double wl, double wr) {
  if (dir == 0) return {parent, parent};
  const double mid = midpoint(wl, wr);
  if (dir > 0) return {Bounds{parent.lower, mid}, Bounds{mid, parent.upper}};
  return {Bounds{mid, parent.upper}, Bounds{parent.lower, mid}};
}

// constraints.rs:117 `satisfies`
inline bool satisfies(int dir, double wl, double wr) {
  if (dir > 0) return wl <= wr;
  if (dir < 0) return wl >= wr;
  return true;
}

// ---------------------------------------------------------------------------
// Split scoring (src/tree/builder/shared.rs:82-141, split.rs:37-58).
inline double threshold_l1(double g, double alpha) {  // gain.rs:96
  if (g > alpha) return g - alpha;
  if (g < -alpha) return g + alpha;
  return 0.0;
}

inline double xgb_calc_weight(double g, double h, const Params& p) {  // shared.rs:87
  if (h <= 0.0) return 0.0;
  double w = -threshold_l1(g, p.alpha) / (h + p.lambda);
  if (p.mds != 0.0 && std::fabs(w) > p.mds) w = std::copysign(p.mds, w);
  return w;
}

// shared.rs:113 `xgb_weight`: rounded to f32, then clamped to the node's
// bounds (shared.rs:100 `apply_bounds`, the bounds rounded to f32).
inline float xgb_weight(double g, double h, const Params& p, Bounds b = Bounds{}) {
  float w = (float)xgb_calc_weight(g, h, p);
  const float lower = (float)b.lower, upper = (float)b.upper;
  if (w < lower) return lower;
  if (w > upper) return upper;
  return w;
}

inline double gain_given_weight(double g, double h, const Params& p, float w) {  // shared.rs:122
  float ww = w * w;
  return -(2.0 * g * (double)w + (h + p.lambda) * (double)ww + 2.0 * p.alpha * (double)std::fabs(w));
}

inline float xgb_node_gain(double g, double h, const Params& p, Bounds b = Bounds{}) {  // shared.rs:136
  if (h <= 0.0) return 0.0f;
  return (float)gain_given_weight(g, h, p, xgb_weight(g, h, p, b));
}

inline bool children_valid(double lh, double rh, double mcw) {  // builder/mod.rs:182
  return lh > 0.0 && rh > 0.0 && lh >= mcw && rh >= mcw;
}

// gain.rs:107 `calc_weight` (leaf values; min_child_weight applies).
inline double calc_weight(double g, double h, const Params& p) {
  if (h < p.mcw || h <= 0.0) return 0.0;
  double w = -threshold_l1(g, p.alpha) / (h + p.lambda);
  if (p.mds > 0.0) w = std::min(std::max(w, -p.mds), p.mds);
  return w;
}

// builder/mod.rs:313 `need_replace`
inline bool need_replace(float incumbent, uint32_t incumbent_feature, float loss, uint32_t feature) {
  if (std::isinf(loss)) return false;
  if (incumbent_feature <= feature) return loss > incumbent;
  return !(incumbent > loss);
}

template <class S>
struct Best {  // builder/mod.rs:64 `BestSplit`
  double loss_chg = 0.0;
  uint32_t feature = 0;
  int32_t bin = -1;  // SplitPos::Bin(global) or -1 = BelowBins
  bool default_left = true;
  S left{}, right{};
  double w_left = 0.0, w_right = 0.0;
};

// ---------------------------------------------------------------------------
// Summation-mode policies.
struct F64Mode {
  using Stat = GS;
  static Stat add(Stat a, Stat b) { return {a.grad + b.grad, a.hess + b.hess}; }
  static Stat sub(Stat a, Stat b) { return {a.grad - b.grad, a.hess - b.hess}; }
  static bool eq(Stat a, Stat b) { return a.grad == b.grad && a.hess == b.hess; }
  double g(Stat s) const { return s.grad; }
  double h(Stat s) const { return s.hess; }
};

struct FixMode {
  using Stat = IS;
  int sg = 0, sh = 0;
  static Stat add(Stat a, Stat b) { return {a.grad + b.grad, a.hess + b.hess}; }
  static Stat sub(Stat a, Stat b) { return {a.grad - b.grad, a.hess - b.hess}; }
  static bool eq(Stat a, Stat b) { return a.grad == b.grad && a.hess == b.hess; }
  double g(Stat s) const { return (double)s.grad * pow2(-sg); }
  double h(Stat s) const { return (double)s.hess * pow2(-sh); }
};

// sum_order (src/tree/hist/mod.rs:420)
bool chain_order(bool dense, size_t index_rows, size_t len, bool contiguous) {
  return len < PARALLEL_THRESHOLD || (dense && (contiguous || index_rows <= GATHER_MAX_ROWS));
}

bool is_contiguous(const std::vector<uint32_t>& rows) {  // walk.rs `contiguous_range`
  return rows.empty() || (size_t)(rows.back() - rows.front()) + 1 == rows.size();
}

// Add rows[b..e) of a dense index into `out`, features [f0, f1) of each
// row, rows in order: each bin sees its rows' values in row order, which is
// all the sum orders below rely on. `Val` is GradPair (f64 sums) or IS
// (fixed point).
template <class Val, class Stat>
void accumulate_dense(const Index& ix, const std::vector<uint32_t>& rows, size_t b, size_t e,
                      size_t f0, size_t f1, const Val* v, Stat* out) {
  const size_t nc = ix.n_cols;
  const uint32_t* off = ix.cuts.feature_offset.data();
  for (size_t i = b; i < e; ++i) {
    const uint32_t r = rows[i];
    const uint16_t* cell = ix.local.data() + (size_t)r * nc;
    const auto g = v[r].grad, h = v[r].hess;
    for (size_t f = f0; f < f1; ++f) {
      if (cell[f] == kMissingBin) continue;
      Stat& o = out[off[f] + cell[f]];
      o.grad += g;
      o.hess += h;
    }
  }
}

// All rows of a dense index into `out`, the features split into one
// contiguous range per thread, each thread walking every row in order over
// its own range: every bin is one chain in row order.
template <class Val, class Stat>
void accumulate_dense_by_features(const Index& ix, const std::vector<uint32_t>& rows, const Val* v,
                                  Stat* out) {
  const size_t nc = ix.n_cols;
  const long long parts = std::max(1, std::min(omp_get_max_threads(), (int)nc));
#pragma omp parallel for schedule(static, 1)
  for (long long t = 0; t < parts; ++t) {
    const size_t f0 = nc * t / parts, f1 = nc * (t + 1) / parts;
    accumulate_dense(ix, rows, 0, rows.size(), f0, f1, v, out);
  }
}

// Accumulate `rows[b..e)` into `out` (walk.rs:46 `accumulate`: one f64
// chain per bin in ascending row order).
void accumulate_f64(const Index& ix, const std::vector<uint32_t>& rows, size_t b, size_t e,
                    const GradPair* gp, GS* out) {
  if (ix.csr) {  // the row's stored cells, rows in order
    for (size_t i = b; i < e; ++i) {
      uint32_t r = rows[i];
      double g = (double)gp[r].grad, h = (double)gp[r].hess;
      for (uint64_t j = ix.row_ptr[r]; j < ix.row_ptr[r + 1]; ++j) {
        GS& o = out[ix.row_bins[j]];
        o.grad += g;
        o.hess += h;
      }
    }
    return;
  }
  accumulate_dense(ix, rows, b, e, 0, ix.n_cols, gp, out);
}

// CpuBackend::build (src/tree/hist/mod.rs:510): the reference's f64 sums.
std::vector<GS> build_hist(const Index& ix, const std::vector<uint32_t>& rows, const GradPair* gp,
                           const F64Mode&) {
  size_t nb = ix.cuts.values.size();
  std::vector<GS> out(nb);
  bool contiguous = ix.dense && is_contiguous(rows);
  if (chain_order(ix.dense, ix.n_rows, rows.size(), contiguous) && ix.csr) {
    // one chain per bin in row order: one pass over the rows' cells
    accumulate_f64(ix, rows, 0, rows.size(), gp, out.data());
    return out;
  }
  if (chain_order(ix.dense, ix.n_rows, rows.size(), contiguous)) {
    // One chain per bin; features are independent, so split them over threads.
    accumulate_dense_by_features(ix, rows, gp, out.data());
    return out;
  }
  // SumOrder::Blocked: chunks of `grain` rows, each summed from zero, then
  // reduced in chunk order (mod.rs:554 `accumulate_blocks`).
  size_t blocks = rows.size() / ROWS_PER_TASK;
  size_t grain = (rows.size() + blocks - 1) / blocks;
  size_t n_chunks = (rows.size() + grain - 1) / grain;
  std::vector<std::vector<GS>> partial(n_chunks);
#pragma omp parallel for schedule(dynamic, 1)
  for (long long c = 0; c < (long long)n_chunks; ++c) {
    partial[c].assign(nb, GS{});
    size_t b = c * grain, e = std::min(rows.size(), b + grain);
    accumulate_f64(ix, rows, b, e, gp, partial[c].data());
  }
  out = partial[0];
#pragma omp parallel for schedule(static)
  for (long long bin = 0; bin < (long long)nb; ++bin) {
    for (size_t c = 1; c < n_chunks; ++c) {
      out[bin].grad += partial[c][bin].grad;
      out[bin].hess += partial[c][bin].hess;
    }
  }
  return out;
}

// The fixed-point histogram: exact int64 sums (order-free).
std::vector<IS> build_hist(const Index& ix, const std::vector<uint32_t>& rows, const IS* q,
                           const FixMode&) {
  size_t nb = ix.cuts.values.size();
  std::vector<IS> out(nb);
  if (ix.csr) {
    // stored cells only; exact sums, so any order: row blocks in parallel
    // into private histograms, then added up
    auto add_rows = [&](size_t b, size_t e, IS* h) {
      for (size_t i = b; i < e; ++i) {
        const uint32_t r = rows[i];
        for (uint64_t j = ix.row_ptr[r]; j < ix.row_ptr[r + 1]; ++j) {
          h[ix.row_bins[j]].grad += q[r].grad;
          h[ix.row_bins[j]].hess += q[r].hess;
        }
      }
    };
    const size_t grain = 16384;
    if (rows.size() <= 2 * grain) {
      add_rows(0, rows.size(), out.data());
      return out;
    }
    const size_t n_chunks = (rows.size() + grain - 1) / grain;
#pragma omp parallel
    {
      std::vector<IS> mine(nb);
#pragma omp for schedule(dynamic, 1) nowait
      for (long long c = 0; c < (long long)n_chunks; ++c)
        add_rows(c * grain, std::min(rows.size(), (size_t)(c + 1) * grain), mine.data());
#pragma omp critical
      for (size_t b = 0; b < nb; ++b) {
        out[b].grad += mine[b].grad;
        out[b].hess += mine[b].hess;
      }
    }
    return out;
  }
  accumulate_dense_by_features(ix, rows, q, out.data());
  return out;
}

// ---------------------------------------------------------------------------
// The tree being grown (src/tree/regtree.rs).
struct Tree {
  std::vector<orc_node> nodes;
  explicit Tree(float root_hess) {
    nodes.push_back(leaf(0.0f, root_hess));
  }
  static orc_node leaf(float value, float sum_hess) {  // regtree.rs:77 `Node::leaf`
    orc_node n{};
    n.left = n.right = -1;
    n.split_feature = 0;
    n.split_cond = 0.0f;
    n.default_left = 1;
    n.leaf_value = value;
    n.sum_hess = sum_hess;
    n.split_gain = 0.0f;
    n.split_bin = -1;
    return n;
  }
  // regtree.rs:549 `expand`
  std::pair<int, int> expand(int nid, uint32_t feature, float cond, int32_t bin, bool default_left,
                             float wl, float hl, float wr, float hr) {
    int left = (int)nodes.size();
    orc_node& n = nodes[nid];
    n.split_cond = cond;
    n.split_feature = feature;
    n.default_left = default_left ? 1 : 0;
    n.left = left;
    n.right = left + 1;
    n.split_bin = bin;
    nodes.push_back(leaf(wl, hl));
    nodes.push_back(leaf(wr, hr));
    return {left, left + 1};
  }
};

// One feature's candidates in for_each_numeric_split order (split.rs:391),
// offered to `best` with need_replace: the forward pass over the bins
// (missing right), then, when the node has missing values of the feature,
// the backward pass (missing left). A candidate is scored by
// SplitScorer::loss_chg (split.rs:37): both children valid, the bounded
// child weights in the feature's monotone direction, the two f32 child
// gains added in f32 minus the node's root gain. True when a candidate
// replaced `best`.
template <class Mode>
bool scan_feature(const Mode& mode, const Params& p, const typename Mode::Stat* hist,
                  typename Mode::Stat total, float root_gain, Bounds bounds, int dir, uint32_t f,
                  uint32_t fs, uint32_t fe, bool dense, Best<typename Mode::Stat>& best) {
  using S = typename Mode::Stat;
  bool found = false;
  auto offer = [&](int32_t bin, bool default_left, S left, S right) {
    double lg = mode.g(left), lh = mode.h(left), rg = mode.g(right), rh = mode.h(right);
    if (!children_valid(lh, rh, p.mcw)) return;
    float wl = xgb_weight(lg, lh, p, bounds);
    float wr = xgb_weight(rg, rh, p, bounds);
    if (!satisfies(dir, (double)wl, (double)wr)) return;
    float gain = (float)gain_given_weight(lg, lh, p, wl) + (float)gain_given_weight(rg, rh, p, wr);
    float loss = gain - root_gain;
    if (need_replace((float)best.loss_chg, best.feature, loss, f)) {
      found = true;
      best.loss_chg = (double)loss;
      best.feature = f;
      best.bin = bin;
      best.default_left = default_left;
      best.left = left;
      best.right = right;
      best.w_left = (double)wl;
      best.w_right = (double)wr;
    }
  };
  if (fe <= fs + 1) return false;  // search.rs:214 degenerate feature
  S acc{};
  for (uint32_t b = fs; b < fe; ++b) {
    acc = Mode::add(acc, hist[b]);
    offer((int32_t)b, false, acc, Mode::sub(total, acc));
  }
  if (dense || Mode::eq(acc, total)) return found;
  S suffix{};
  for (uint32_t off = fe - fs; off-- > 0;) {
    suffix = Mode::add(suffix, hist[fs + off]);
    // SplitPos::backward (builder/mod.rs:263)
    int32_t bin = off == 0 ? -1 : (int32_t)(fs + off - 1);
    offer(bin, true, Mode::sub(total, suffix), suffix);
  }
  return found;
}

// ---------------------------------------------------------------------------
// HistTreeBuilder (src/tree/builder/hist/mod.rs) for one tree, parameterised
// by the summation mode.
template <class Mode>
class Builder {
 public:
  using S = typename Mode::Stat;
  Builder(const Index& ix, const Params& p, const Mode& mode) : ix_(ix), p_(p), mode_(mode) {}

  struct Entry {
    int nid;
    int depth;
    std::vector<uint32_t> rows;
    std::vector<S> hist;
    Best<S> best;
  };

  // Grows the tree; `leaf_rows` receives (node, rows) for every leaf.
  template <class Values>
  Tree grow(const Values* values, std::vector<std::pair<int, std::vector<uint32_t>>>& leaf_rows) {
    values_ = values;
    std::vector<uint32_t> all(ix_.n_rows);
    std::iota(all.begin(), all.end(), 0u);
    S root_stats = root_sum(all);
    Tree tree((float)mode_.h(root_stats));
    stats_.assign(1, root_stats);
    bounds_.assign(1, Bounds{});
    Entry root{0, 0, std::move(all), {}, {}};
    root.hist = build_hist(ix_, root.rows, values_, mode_);
    root.best = evaluate(root.hist, root_stats, bounds_[0]);
    if (p_.grow_policy == 0) {
      grow_depthwise(tree, std::move(root), leaf_rows);
    } else {
      grow_lossguide(tree, std::move(root), leaf_rows);
    }
    // finalize_leaf_values (shared.rs:174): calc_weight_bounded
    // (constraints.rs:70), the weight clamped to the leaf's bounds in f64
    for (size_t id = 0; id < tree.nodes.size(); ++id) {
      if (tree.nodes[id].left == -1) {
        double w = bounds_[id].clamp(calc_weight(mode_.g(stats_[id]), mode_.h(stats_[id]), p_));
        tree.nodes[id].leaf_value = (float)w;
      }
    }
    return tree;
  }

 private:
  S root_sum(const std::vector<uint32_t>& rows) const;

  bool valid(const Best<S>& b) const {  // builder/mod.rs:167 `BestSplit::valid`
    return b.loss_chg > K_RT_EPS && b.loss_chg >= p_.gamma &&
           children_valid(mode_.h(b.left), mode_.h(b.right), p_.mcw);
  }

  // HistTreeBuilder::evaluate (search.rs:37) over every feature, with the
  // sequential candidate order of for_each_numeric_split (split.rs:391)
  // and xgb_update's tie rule (builder/mod.rs:334). The node's root gain
  // and child weights use its monotone bounds (search.rs:130 `node_scorer`),
  // each feature its direction (`scorer`).
  //
  // The features are scored in parallel, each from the empty split, and
  // their winners merged in feature order: the incumbent's feature never
  // exceeds the candidate's, so need_replace is a strict `>` throughout,
  // and the merge keeps the first maximum of the sequential scan.
  Best<S> evaluate(const std::vector<S>& hist, S total, Bounds bounds) const {
    const float root_gain = xgb_node_gain(mode_.g(total), mode_.h(total), p_, bounds);
    const long long nc = (long long)ix_.n_cols;
    std::vector<Best<S>> per(nc);
    std::vector<uint8_t> found(nc, 0);
#pragma omp parallel for schedule(dynamic, 4) if (nc >= 16)
    for (long long f = 0; f < nc; ++f)
      found[f] = scan_feature(mode_, p_, hist.data(), total, root_gain, bounds, p_.dir((size_t)f),
                              (uint32_t)f, ix_.cuts.feature_offset[f], ix_.cuts.feature_offset[f + 1],
                              ix_.dense, per[f]);
    Best<S> best;
    for (long long f = 0; f < nc; ++f)
      if (found[f] && need_replace((float)best.loss_chg, best.feature, (float)per[f].loss_chg, (uint32_t)f))
        best = per[f];
    return best;
  }

  // prepare_split (hist/mod.rs:639): expand the node, record child stats.
  std::pair<int, int> expand(Tree& tree, const Entry& e) {
    const Best<S>& b = e.best;
    float cond = b.bin < 0 ? BELOW_ALL_VALUES : ix_.cuts.values[b.bin];
    auto ids = tree.expand(e.nid, b.feature, cond, b.bin, b.default_left, (float)b.w_left,
                           (float)mode_.h(b.left), (float)b.w_right, (float)mode_.h(b.right));
    tree.nodes[e.nid].split_gain = (float)b.loss_chg;
    stats_.push_back(b.left);
    stats_.push_back(b.right);
    // hist/mod.rs:648: monotone child bounds from the bounded child weights
    auto cb = child_bounds(bounds_[e.nid], p_.dir(b.feature), b.w_left, b.w_right);
    bounds_.push_back(cb.first);
    bounds_.push_back(cb.second);
    return ids;
  }

  // partition_rows (partition.rs:106, route_column :206).
  void partition(const Entry& e, std::vector<uint32_t>& left, std::vector<uint32_t>& right) const {
    const Best<S>& b = e.best;
    uint32_t fs = ix_.cuts.feature_offset[b.feature];
    uint32_t limit = b.bin < 0 ? 0 : (uint32_t)(b.bin + 1 - (int32_t)fs);
    // each row's side (in parallel: a gather of one feature's cells), then
    // the stable split in row order
    const long long n = (long long)e.rows.size();
    std::vector<uint8_t> go(n);
#pragma omp parallel for schedule(static) if (n >= 65536)
    for (long long i = 0; i < n; ++i) {
      uint32_t bin = 0;
      go[i] = ix_.cell(e.rows[i], b.feature, bin) ? bin < limit : b.default_left;
    }
    // stable split: per-chunk left counts, their prefix, then each chunk
    // writes its rows at its offsets, in row order
    const long long chunk = 1 << 16, n_chunks = (n + chunk - 1) / chunk;
    std::vector<size_t> lefts(n_chunks + 1, 0);
#pragma omp parallel for schedule(static) if (n_chunks > 1)
    for (long long c = 0; c < n_chunks; ++c) {
      size_t cnt = 0;
      for (long long i = c * chunk; i < std::min(n, (c + 1) * chunk); ++i) cnt += go[i];
      lefts[c + 1] = cnt;
    }
    for (long long c = 0; c < n_chunks; ++c) lefts[c + 1] += lefts[c];
    const size_t l0 = left.size(), r0 = right.size();
    left.resize(l0 + lefts[n_chunks]);
    right.resize(r0 + (size_t)n - lefts[n_chunks]);
#pragma omp parallel for schedule(static) if (n_chunks > 1)
    for (long long c = 0; c < n_chunks; ++c) {
      size_t li = l0 + lefts[c], ri = r0 + (size_t)(c * chunk) - lefts[c];
      for (long long i = c * chunk; i < std::min(n, (c + 1) * chunk); ++i) {
        if (go[i]) left[li++] = e.rows[i];
        else right[ri++] = e.rows[i];
      }
    }
  }

  // build_children (hist/mod.rs:692) + finish_children.
  void children(const Entry& e, int lid, int rid, bool terminal, Entry& l, Entry& r) {
    l.nid = lid;
    r.nid = rid;
    l.depth = r.depth = e.depth + 1;
    partition(e, l.rows, r.rows);
    if (terminal) return;
    // child_histograms (partition.rs:259): the smaller child is built and
    // its sibling is the parent minus it.
    bool left_smaller = l.rows.size() <= r.rows.size();
    std::vector<S> small = build_hist(ix_, left_smaller ? l.rows : r.rows, values_, mode_);
    std::vector<S> sib(e.hist.size());
    for (size_t i = 0; i < sib.size(); ++i) sib[i] = Mode::sub(e.hist[i], small[i]);
    if (left_smaller) {
      l.hist = std::move(small);
      r.hist = std::move(sib);
    } else {
      l.hist = std::move(sib);
      r.hist = std::move(small);
    }
    l.best = evaluate(l.hist, e.best.left, bounds_[lid]);
    r.best = evaluate(r.hist, e.best.right, bounds_[rid]);
  }

  void grow_depthwise(Tree& tree, Entry root,
                      std::vector<std::pair<int, std::vector<uint32_t>>>& leaf_rows) {
    std::vector<Entry> frontier;
    frontier.push_back(std::move(root));
    int depth = 0;
    const int limit = p_.max_depth > 0 ? p_.max_depth : (1 << 30);  // limit_or_unbounded
    while (depth < limit && !frontier.empty()) {
      std::vector<Entry> next;
      std::vector<std::pair<Entry*, std::pair<int, int>>> pending;
      for (Entry& e : frontier) {
        if (valid(e.best)) {
          pending.push_back({&e, expand(tree, e)});
        } else {
          leaf_rows.emplace_back(e.nid, std::move(e.rows));
        }
      }
      bool terminal = depth + 1 >= limit;
      for (auto& pd : pending) {
        Entry l, r;
        children(*pd.first, pd.second.first, pd.second.second, terminal, l, r);
        next.push_back(std::move(l));
        next.push_back(std::move(r));
      }
      frontier = std::move(next);
      ++depth;
    }
    for (Entry& e : frontier) leaf_rows.emplace_back(e.nid, std::move(e.rows));
  }

  // grow_lossguide (hist/mod.rs:505) with Rust's BinaryHeap pop/push order
  // (max-heap on loss_chg by total order).
  void grow_lossguide(Tree& tree, Entry root,
                      std::vector<std::pair<int, std::vector<uint32_t>>>& leaf_rows) {
    size_t limit = p_.max_depth > 0 ? (size_t)p_.max_depth : SIZE_MAX;
    size_t max_leaves = p_.max_leaves > 0 ? (size_t)p_.max_leaves : SIZE_MAX;
    std::vector<Entry> heap;
    auto key_le = [](const Entry& a, const Entry& b) {  // a <= b under total_cmp
      return total_key(a.best.loss_chg) <= total_key(b.best.loss_chg);
    };
    auto sift_up = [&](size_t start, size_t pos) {
      Entry hole = std::move(heap[pos]);
      while (pos > start) {
        size_t parent = (pos - 1) / 2;
        if (key_le(hole, heap[parent])) break;
        heap[pos] = std::move(heap[parent]);
        pos = parent;
      }
      heap[pos] = std::move(hole);
    };
    auto push = [&](Entry e) {
      heap.push_back(std::move(e));
      sift_up(0, heap.size() - 1);
    };
    auto pop = [&]() {
      Entry item = std::move(heap.back());
      heap.pop_back();
      if (!heap.empty()) {
        std::swap(item, heap[0]);
        // sift_down_to_bottom(0)
        size_t end = heap.size();
        size_t pos = 0;
        Entry hole = std::move(heap[0]);
        size_t child = 1;
        while (end >= 2 && child <= end - 2) {
          if (key_le(heap[child], heap[child + 1])) child += 1;
          heap[pos] = std::move(heap[child]);
          pos = child;
          child = 2 * pos + 1;
        }
        if (child == end - 1) {
          heap[pos] = std::move(heap[child]);
          pos = child;
        }
        heap[pos] = std::move(hole);
        sift_up(0, pos);
      }
      return item;
    };
    auto expandable = [&](const Entry& e) { return (size_t)e.depth < limit && valid(e.best); };
    push(std::move(root));
    size_t n_leaves = 1;
    while (!heap.empty()) {
      Entry e = pop();
      if (n_leaves >= max_leaves) {
        leaf_rows.emplace_back(e.nid, std::move(e.rows));
        break;
      }
      if (!expandable(e)) {
        leaf_rows.emplace_back(e.nid, std::move(e.rows));
        continue;
      }
      auto ids = expand(tree, e);
      Entry l, r;
      children(e, ids.first, ids.second, false, l, r);
      ++n_leaves;
      push(std::move(l));
      push(std::move(r));
    }
    for (Entry& e : heap) leaf_rows.emplace_back(e.nid, std::move(e.rows));
  }

  static int64_t total_key(double v) {  // f64::total_cmp order as a signed key
    int64_t b;
    std::memcpy(&b, &v, 8);
    return b ^ (int64_t)((uint64_t)(b >> 63) >> 1);
  }

  const Index& ix_;
  const Params& p_;
  Mode mode_;
  const typename std::conditional<std::is_same<Mode, F64Mode>::value, GradPair, IS>::type* values_ =
      nullptr;
  std::vector<S> stats_;
  std::vector<Bounds> bounds_;  // hist/mod.rs:916 `NodeStore` bounds, by node id
};

// shared.rs:164 `sum_rows`: an f64 chain in row order.
template <>
GS Builder<F64Mode>::root_sum(const std::vector<uint32_t>& rows) const {
  GS t;
  for (uint32_t r : rows) {
    t.grad += (double)values_[r].grad;
    t.hess += (double)values_[r].hess;
  }
  return t;
}
template <>
IS Builder<FixMode>::root_sum(const std::vector<uint32_t>& rows) const {
  IS t;
  for (uint32_t r : rows) {
    t.grad += values_[r].grad;
    t.hess += values_[r].hess;
  }
  return t;
}

// ---------------------------------------------------------------------------
// Objectives.

// The reference's x86-64 vector exponential (src/simd/x86_64.rs:20-46),
// operation for operation (fma = one rounding).
float exp_vector(float value) {
  const float log2e = 1.44269504088896340736f;
  float t = value * log2e;
  int32_t exponent = (int32_t)std::nearbyint(t);  // cvtps_epi32, round-to-nearest-even
  float ef = (float)exponent;
  float reduced = std::fmaf(-ef, 0.6933594f, value);
  reduced = std::fmaf(ef, 2.1219444e-4f, reduced);
  float squared = reduced * reduced;
  float fourth = squared * squared;
  float pair0 = 1.0f + reduced;
  float pair1 = std::fmaf(1.0f / 6.0f, reduced, 0.5f);
  float pair2 = std::fmaf(1.0f / 120.0f, reduced, 1.0f / 24.0f);
  float pair3 = std::fmaf(1.0f / 5040.0f, reduced, 1.0f / 720.0f);
  float low = std::fmaf(pair1, squared, pair0);
  float high = std::fmaf(pair3, squared, pair2);
  float poly = std::fmaf(high, fourth, low);
  uint32_t bits = (uint32_t)(exponent + 127) << 23;
  float scale;
  std::memcpy(&scale, &bits, 4);
  return poly * scale;
}

// x86_64.rs:63 `sigmoid_f32`
float sigmoid_vector(float v) {
  float e = exp_vector(0.0f - std::fabs(v));
  float den = 1.0f + e;
  float pos = 1.0f / den;
  float neg = e / den;
  return v >= 0.0f ? pos : neg;
}

// simd/mod.rs:421 `sigmoid_scalar`
float sigmoid_scalar(float x) {
  return 1.0f / (std::exp(std::fmin(-x, 88.7f)) + 1.0f);
}

void logistic_pair(float p, float label, float spw, float& g, float& h) {
  float w = 1.0f;
  if (label == 1.0f) w *= spw;
  g = (p - label) * w;
  float ph = p * (1.0f - p);
  h = (ph > MIN_HESS ? ph : MIN_HESS) * w;  // max_ps(a, b) returns b unless a > b
}

}  // namespace

// simd/x86_64.rs:106 `logistic_gradient` + scalar.rs:8, with the whole-batch
// vector/scalar split of objective/mod.rs:195 `rowwise_cells`: 8-row vectors
// over the first n - n % 8 rows (n >= 16), a vector holding a margin above
// 80 in magnitude (or non-finite) on the scalar path, the rest scalar.
void logistic_gradient(const float* m, const float* y, size_t n, float spw, GradPair* out) {
  size_t vrows = n >= 16 ? n - n % 8 : 0;
#pragma omp parallel for schedule(static)
  for (long long v = 0; v < (long long)(vrows / 8); ++v) {
    size_t b = (size_t)v * 8;
    bool regular = true;
    for (int k = 0; k < 8; ++k) regular = regular && (std::fabs(m[b + k]) <= 80.0f);
    for (int k = 0; k < 8; ++k) {
      float p = regular ? sigmoid_vector(m[b + k]) : sigmoid_scalar(m[b + k]);
      logistic_pair(p, y[b + k], spw, out[b + k].grad, out[b + k].hess);
    }
  }
  for (size_t i = vrows; i < n; ++i) {
    logistic_pair(sigmoid_scalar(m[i]), y[i], spw, out[i].grad, out[i].hess);
  }
}

// objective/regression.rs:50 (squared error, unit weights)
void squared_error_gradient(const float* m, const float* y, size_t n, float spw, GradPair* out) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    float w = 1.0f;
    if (y[i] == 1.0f) w *= spw;
    out[i].grad = (m[i] - y[i]) * w;
    out[i].hess = w;
  }
}

// `_mm256_max_ps` / `_mm256_min_ps`: the second operand unless the first is
// strictly greater (smaller), so a NaN in either gives the second.
static inline float maxps(float a, float b) { return a > b ? a : b; }
static inline float minps(float a, float b) { return a < b ? a : b; }

// One row of k = 2 or 4 margins through x86_64.rs:191 `short_softmax_batch`:
// the row's maximum and minimum by `row_reduce` (x86_64.rs:167: lane j takes
// op(v[j], v[j ^ 1]), then for k = 4 op(r[j], r[j ^ 2])), shift =
// maxps(MIN_POSITIVE, max); false when max - min <= 80 fails in a lane (a
// non-finite or wide row: its batch takes the scalar path); otherwise
// p[j] = exp_f32(v[j] - shift) * (1 / sum), the sum reduced the same way.
static bool softmax_short_row(const float* v, int k, float* p) {
  float mx[4], mn[4], t[4], u[4];
  for (int j = 0; j < k; ++j) {
    mx[j] = maxps(v[j], v[j ^ 1]);
    mn[j] = minps(v[j], v[j ^ 1]);
  }
  if (k == 4) {
    for (int j = 0; j < 4; ++j) {
      t[j] = maxps(mx[j], mx[j ^ 2]);
      u[j] = minps(mn[j], mn[j ^ 2]);
    }
    for (int j = 0; j < 4; ++j) {
      mx[j] = t[j];
      mn[j] = u[j];
    }
  }
  float shift[4], e[4], sum[4];
  for (int j = 0; j < k; ++j) {
    shift[j] = maxps(FLT_MIN, mx[j]);
    if (!(shift[j] - mn[j] <= 80.0f)) return false;
  }
  for (int j = 0; j < k; ++j) e[j] = exp_vector(v[j] - shift[j]);
  for (int j = 0; j < k; ++j) sum[j] = e[j] + e[j ^ 1];
  if (k == 4) {
    for (int j = 0; j < 4; ++j) t[j] = sum[j] + sum[j ^ 2];
    for (int j = 0; j < 4; ++j) sum[j] = t[j];
  }
  for (int j = 0; j < k; ++j) p[j] = e[j] * (1.0f / sum[j]);
  return true;
}

// simd/mod.rs:580 `softmax_gradient_row_scalar` for row i: the shift is
// max(f32::MIN_POSITIVE, margins...), the exponentials are summed in f64 and
// the sum rounded to f32, then p = expf(m - shift) / sum,
// g = (p - [class == label]) w, h = max(((2 p)(1 - p)) w, MIN_HESS).
static void softmax_row_scalar(const float* row, float y, int k, GradPair* out) {
  float wmax = FLT_MIN;
  for (int j = 0; j < k; ++j) wmax = std::fmax(row[j], wmax);
  double wsum = 0.0;
  for (int j = 0; j < k; ++j) wsum += (double)expf(row[j] - wmax);
  const float ws = (float)wsum;
  const size_t label = (size_t)y;
  const float w = 1.0f;
  for (int j = 0; j < k; ++j) {
    const float p = expf(row[j] - wmax) / ws;
    const float h = std::fmax(((2.0f * p) * (1.0f - p)) * w, MIN_HESS);
    const float g = ((size_t)j == label ? p - 1.0f : p) * w;
    out[j].grad = g;
    out[j].hess = h;
  }
}

// multi:softmax gradients (objective/multiclass.rs:43 through
// simd/mod.rs:502). x86_64 runs the scalar row kernel for every class count
// but 2 and 4. For those it runs x86_64.rs:273 `short_softmax_gradient`
// (simd/mod.rs:156) when the margins hold at least 16 values
// (MIN_SIMD_LEN, simd/mod.rs:28): vectors of 8 / k whole rows over the first
// n - n % (8 / k) rows, a vector with an irregular row on the scalar path,
// the remaining rows scalar. The vector rows' pairs: g = (p - [class ==
// label]) w, h = maxps(((p 2)(1 - p)) w, MIN_HESS). The chunking of
// objective/mod.rs:195 `rowwise_cells` keeps this whole-batch split. Margins
// row-major, k per row; out in the same layout.
void softmax_gradient(const float* m, const float* y, size_t n, int k, GradPair* out) {
  const size_t rpb = (k == 2 || k == 4) ? (size_t)(8 / k) : 0;
  const size_t vrows = (rpb && n * (size_t)k >= 16) ? n - n % rpb : 0;
#pragma omp parallel for schedule(static)
  for (long long b = 0; b < (long long)(vrows / (rpb ? rpb : 1)); ++b) {
    float p[8];
    bool regular = true;
    for (size_t r = 0; r < rpb; ++r)
      regular = softmax_short_row(m + ((size_t)b * rpb + r) * k, k, p + r * k) && regular;
    for (size_t r = 0; r < rpb; ++r) {
      const size_t i = (size_t)b * rpb + r;
      if (!regular) {
        softmax_row_scalar(m + i * k, y[i], k, out + i * k);
        continue;
      }
      const size_t label = (size_t)y[i];
      const float w = 1.0f;
      for (int j = 0; j < k; ++j) {
        const float q = p[r * k + j];
        out[i * k + j].grad = (q - ((size_t)j == label ? 1.0f : 0.0f)) * w;
        out[i * k + j].hess = maxps(((q * 2.0f) * (1.0f - q)) * w, MIN_HESS);
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (long long i = (long long)vrows; i < (long long)n; ++i)
    softmax_row_scalar(m + (size_t)i * k, y[i], k, out + (size_t)i * k);
}

// multiclass.rs:68 `base_margins_info` (unweighted): class counts in f32,
// divided by the f64 row count (n rounded to f32 first), ln(p + 1e-6) in
// f32, centred by the f32 mean of m / k.
void softmax_intercepts(const float* y, size_t n, int k, float* out) {
  for (int j = 0; j < k; ++j) out[j] = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    const float v = y[i];
    if (v >= 0.0f && (size_t)v < (size_t)k) out[(size_t)v] += 1.0f;
  }
  const double sum_w = (double)(float)n;
  const double inv = 1.0 / sum_w;
  for (int j = 0; j < k; ++j) out[j] = logf((float)((double)out[j] * inv) + 1e-6f);
  const float kk = (float)k;
  float mean = 0.0f;
  for (int j = 0; j < k; ++j) mean += out[j] / kk;
  for (int j = 0; j < k; ++j) out[j] -= mean;
}

// objective/mod.rs:645 `weighted_label_mean` (unweighted)
float label_mean(const float* y, size_t n, size_t stride, size_t col) {
  if (n == 0) return 0.0f;
  double nn = (double)n, s = 0.0;
  for (size_t i = 0; i < n; ++i) s += (double)y[i * stride + col] / nn;
  return (float)s;
}

float logistic_link(float p) {  // classification.rs:69 `link`
  p = std::min(std::max(p, K_RT_EPS_F32), 1.0f - K_RT_EPS_F32);
  return -std::log(1.0f / p - 1.0f);
}

int32_t fixed_scale(float max_abs, uint64_t n) {
  if (!(max_abs > 0.0f) || !std::isfinite(max_abs)) return 0;
  int e;
  std::frexp(max_abs, &e);  // max_abs < 2^e
  int c = 0;
  while (c < 64 && (uint64_t(1) << c) < n) ++c;
  return 53 - c - e;  // every sum of n values within 2^53: exact in an f64
}

}  // namespace orc

using namespace orc;

extern "C" {

int64_t orc_cuts_dense(const float* x, uint64_t n_rows, uint64_t n_cols, const float* weights,
                       uint32_t max_bin, uint32_t* feature_offset, float* cut_values,
                       uint64_t cap) {
  Cuts c = cuts_from_dense(x, n_rows, n_cols, weights, max_bin, NAN);
  if (c.values.size() > cap) return -1;
  std::copy(c.feature_offset.begin(), c.feature_offset.end(), feature_offset);
  std::copy(c.values.begin(), c.values.end(), cut_values);
  return (int64_t)c.values.size();
}

static Cuts cuts_from(const uint32_t* off, const float* vals, uint64_t n_cols) {
  Cuts c;
  c.feature_offset.assign(off, off + n_cols + 1);
  c.values.assign(vals, vals + off[n_cols]);
  return c;
}

int32_t orc_bin_dense(const float* x, uint64_t n, uint64_t nc, const uint32_t* feature_offset,
                      const float* cut_values, uint16_t* bins, uint64_t* missing) {
  Cuts c = cuts_from(feature_offset, cut_values, nc);
  size_t words = (n + 63) / 64;
  std::fill(missing, missing + words * nc, 0ull);
  int32_t dense = 1;
  for (size_t f = 0; f < nc; ++f) {
    for (size_t r = 0; r < n; ++r) {
      float v = x[r * nc + f];
      if (std::isnan(v)) {
        bins[f * n + r] = 0;
        missing[f * words + r / 64] |= 1ull << (r % 64);
        dense = 0;
      } else {
        bins[f * n + r] = (uint16_t)local_bin_of(c, f, v);
      }
    }
  }
  return dense;
}

void orc_gradients(int32_t objective, const float* margins, const float* labels, uint64_t n,
                   float spw, float* gpair) {
  GradPair* out = reinterpret_cast<GradPair*>(gpair);
  if (objective == 1)
    logistic_gradient(margins, labels, n, spw, out);
  else
    squared_error_gradient(margins, labels, n, spw, out);
}

void orc_softmax_gradients(const float* margins, const float* labels, uint64_t n, int32_t k,
                           float* gpair) {
  softmax_gradient(margins, labels, n, k, reinterpret_cast<GradPair*>(gpair));
}

void orc_intercepts(int32_t objective, const float* labels, uint64_t n, int32_t n_outputs,
                    float* out) {
  if (objective == 2) {
    softmax_intercepts(labels, n, n_outputs, out);
    return;
  }
  for (int t = 0; t < n_outputs; ++t) {
    float mean = label_mean(labels, n, (size_t)n_outputs, (size_t)t);
    out[t] = objective == 1 ? logistic_link(mean) : mean;
  }
}

int32_t orc_fixed_scale(float max_abs, uint64_t n) { return fixed_scale(max_abs, n); }


}  // extern "C"

struct orc_trainer {
  orc::Params p;
  orc::Index ix;
  std::vector<float> base, margins, labels;
  size_t n = 0;
  int k = 1;
  // per-round scratch, kept across orc_trainer_rounds calls (every element
  // is written before it is read in a round)
  std::vector<orc::GradPair> gp, gp_all;
  std::vector<float> mk, yk;
  std::vector<orc::IS> q;
};

namespace {

orc::Params params_from(const orc_params* pp) {
  orc::Params p;
  p.objective = pp->objective;
  p.n_outputs = pp->objective == 1 ? 1 : std::max(1, pp->n_outputs);
  p.max_depth = pp->max_depth;
  p.max_leaves = pp->max_leaves;
  p.grow_policy = pp->grow_policy;
  p.max_bin = pp->max_bin;
  p.eta = pp->eta;
  p.lambda = (double)pp->lambda;
  p.alpha = (double)pp->alpha;
  p.gamma = (double)pp->gamma;
  p.mcw = (double)pp->min_child_weight;
  p.mds = (double)pp->max_delta_step;
  p.spw = pp->scale_pos_weight;
  p.fixed = pp->fixed_point != 0;
  if (pp->monotone && pp->n_monotone > 0) p.mono.assign(pp->monotone, pp->monotone + pp->n_monotone);
  return p;
}

// `rounds` rounds of train_trees (src/training/train.rs:222) from the
// trainer's margins.
int64_t run_rounds(orc_trainer* tr, int rounds, orc_node* nodes, uint64_t nodes_cap,
                   uint64_t* tree_ptr) {
  using namespace orc;
  const Params& p = tr->p;
  const size_t n = tr->n;
  const int k = tr->k;
  tr->gp.resize(n);
  tr->gp_all.resize(n * k);
  tr->mk.resize(n);
  tr->yk.resize(n);
  if (p.fixed) tr->q.resize(n);
  std::vector<GradPair>& gp = tr->gp;
  std::vector<GradPair>& gp_all = tr->gp_all;
  std::vector<float>& mk = tr->mk;
  std::vector<float>& yk = tr->yk;
  std::vector<IS>& q = tr->q;
  const long long nn = (long long)n;
  uint64_t used = 0;
  int64_t n_trees = 0;
  tree_ptr[0] = 0;
  for (int round = 0; round < rounds; ++round) {
    // 1. Gradients of every output from this round's margins (round.rs:253).
    if (p.objective == 2) softmax_gradient(tr->margins.data(), tr->labels.data(), n, k, gp_all.data());
    for (int t = 0; t < k && p.objective != 2; ++t) {
#pragma omp parallel for schedule(static)
      for (long long r = 0; r < nn; ++r) {
        mk[r] = tr->margins[r * k + t];
        yk[r] = tr->labels[r * k + t];
      }
      if (p.objective == 1)
        logistic_gradient(mk.data(), yk.data(), n, p.spw, gp.data());
      else
        squared_error_gradient(mk.data(), yk.data(), n, p.spw, gp.data());
#pragma omp parallel for schedule(static)
      for (long long r = 0; r < nn; ++r) gp_all[r * k + t] = gp[r];
    }
    // 2. One tree per output, output-major (round.rs:318).
    for (int t = 0; t < k; ++t) {
#pragma omp parallel for schedule(static)
      for (long long r = 0; r < nn; ++r) gp[r] = gp_all[r * k + t];
      std::vector<std::pair<int, std::vector<uint32_t>>> leaves;
      Tree tree(0.0f);
      if (p.fixed) {
        float mg = 0.0f, mh = 0.0f;
        for (size_t r = 0; r < n; ++r) {
          if (!std::isfinite(gp[r].grad) || !std::isfinite(gp[r].hess)) return -3;
          mg = std::max(mg, std::fabs(gp[r].grad));
          mh = std::max(mh, std::fabs(gp[r].hess));
        }
        FixMode mode;
        mode.sg = fixed_scale(mg, n);
        mode.sh = fixed_scale(mh, n);
        double fg = pow2(mode.sg), fh = pow2(mode.sh);
#pragma omp parallel for schedule(static)
        for (long long r = 0; r < nn; ++r) {
          q[r].grad = std::llrint((double)gp[r].grad * fg);
          q[r].hess = std::llrint((double)gp[r].hess * fh);
        }
        Builder<FixMode> b(tr->ix, p, mode);
        tree = b.grow(q.data(), leaves);
      } else {
        Builder<F64Mode> b(tr->ix, p, F64Mode{});
        tree = b.grow(gp.data(), leaves);
      }
      // round.rs:143 `scale_leaves(eta)` (leaves only, regtree.rs:599).
      float eta = p.eta;
      for (auto& nd : tree.nodes)
        if (nd.left == -1) nd.leaf_value = nd.leaf_value * eta;
      // each row is in one leaf: the leaves update disjoint margins
#pragma omp parallel for schedule(dynamic, 1)
      for (long long li = 0; li < (long long)leaves.size(); ++li) {
        const float v = tree.nodes[leaves[li].first].leaf_value;
        for (uint32_t r : leaves[li].second) tr->margins[(size_t)r * k + t] += v;
      }
      if (used + tree.nodes.size() > nodes_cap) return -1;
      std::copy(tree.nodes.begin(), tree.nodes.end(), nodes + used);
      used += tree.nodes.size();
      ++n_trees;
      tree_ptr[n_trees] = used;
    }
  }
  return n_trees;
}

}  // namespace

extern "C" {

static orc_trainer* trainer_new(const orc_params* pp, uint64_t n, const float* labels,
                                const std::function<orc::Index(const orc::Params&)>& index);

orc_trainer* orc_trainer_new(const orc_params* pp, const float* x, uint64_t n, uint64_t nc,
                             const float* labels) {
  using namespace orc;
  if (!pp || !x || !labels || n == 0 || nc == 0) return nullptr;
  return trainer_new(pp, n, labels, [&](const Params& p) {
    return make_index(x, n, nc, cuts_from_dense(x, n, nc, nullptr, (size_t)p.max_bin, NAN));
  });
}

orc_trainer* orc_trainer_new_csr(const orc_params* pp, const uint64_t* indptr, const uint32_t* indices,
                                 const float* values, uint64_t n, uint64_t nc, const float* labels) {
  using namespace orc;
  if (!pp || !indptr || !labels || n == 0 || nc == 0 || (indptr[n] && (!indices || !values)))
    return nullptr;
  return trainer_new(pp, n, labels, [&](const Params& p) {
    return make_index_csr(indptr, indices, values, n, nc,
                          cuts_from_csr(indptr, indices, values, n, nc, (size_t)p.max_bin));
  });
}

static orc_trainer* trainer_new(const orc_params* pp, uint64_t n, const float* labels,
                                const std::function<orc::Index(const orc::Params&)>& index) {
  using namespace orc;
#ifdef _OPENMP
  if (pp->n_threads > 0) omp_set_num_threads(pp->n_threads);
#endif
  orc_trainer* tr = new orc_trainer();
  tr->p = params_from(pp);
  tr->n = n;
  tr->k = tr->p.n_outputs;
  const int k = tr->k;
  tr->ix = index(tr->p);
  tr->labels.assign(labels, labels + n * (tr->p.objective == 2 ? 1 : k));  // softmax: class ids
  tr->base.assign(k, 0.0f);
  if (std::isnan(pp->base_score)) {
    orc_intercepts(tr->p.objective, labels, n, k, tr->base.data());
  } else {
    for (int t = 0; t < k; ++t)
      tr->base[t] = tr->p.objective == 1 ? logistic_link(pp->base_score) : pp->base_score;
  }
  tr->margins.resize(n * k);
  for (size_t r = 0; r < n; ++r)
    for (int t = 0; t < k; ++t) tr->margins[r * k + t] = tr->base[t];
  return tr;
}

int64_t orc_trainer_rounds(orc_trainer* tr, int32_t rounds, orc_node* nodes, uint64_t nodes_cap,
                           uint64_t* tree_ptr) {
  if (!tr || rounds < 0 || !tree_ptr) return -2;
  return run_rounds(tr, rounds, nodes, nodes_cap, tree_ptr);
}

void orc_trainer_free(orc_trainer* tr) { delete tr; }

uint64_t orc_trainer_margins(const orc_trainer* tr, float* out, uint64_t cap) {
  if (!tr) return 0;
  const uint64_t n = tr->margins.size();
  if (out && cap >= n) std::copy(tr->margins.begin(), tr->margins.end(), out);
  return n;
}

int32_t orc_trainer_set_margins(orc_trainer* tr, const float* m, uint64_t n) {
  if (!tr || !m || n != tr->margins.size()) return -2;
  std::copy(m, m + n, tr->margins.begin());
  return 0;
}

int32_t orc_scan_node(const orc_params* pp, const uint32_t* feature_offset, uint32_t n_cols, int32_t dense,
                      const int64_t* hist, int64_t total_g, int64_t total_h, int32_t sg, int32_t sh,
                      float lower, float upper, const uint32_t* features, const int8_t* directions,
                      uint32_t n_features, orc_scan* out) {
  if (!pp || !feature_offset || !hist || !out || (n_features && !features)) return -2;
  using namespace orc;
  Params p = params_from(pp);
  FixMode mode;
  mode.sg = sg;
  mode.sh = sh;
  const IS* h = reinterpret_cast<const IS*>(hist);
  const IS total{total_g, total_h};
  Bounds b{(double)lower, (double)upper};
  const float root_gain = xgb_node_gain(mode.g(total), mode.h(total), p, b);
  // features in the request's order, each scanned from the empty split,
  // merged with need_replace (search.rs:164 `merge`)
  Best<IS> best;
  bool any = false;
  for (uint32_t j = 0; j < n_features; ++j) {
    const uint32_t f = features[j];
    if (f >= n_cols) return -2;
    Best<IS> one;
    const int dir = directions ? directions[j] : 0;
    if (scan_feature(mode, p, h, total, root_gain, b, dir, f, feature_offset[f], feature_offset[f + 1],
                     dense != 0, one) &&
        need_replace((float)best.loss_chg, best.feature, (float)one.loss_chg, f)) {
      best = one;
      any = true;
    }
  }
  std::memset(out, 0, sizeof(*out));
  out->found = any ? 1 : 0;
  out->feature = best.feature;
  out->bin = best.bin;
  out->default_left = best.default_left ? 1 : 0;
  out->loss_chg = (float)best.loss_chg;
  out->root_gain = root_gain;
  out->left_g = best.left.grad;
  out->left_h = best.left.hess;
  out->w_left = (float)best.w_left;
  out->w_right = (float)best.w_right;
  return 0;
}

int64_t orc_train(const orc_params* pp, const float* x, uint64_t n, uint64_t nc,
                  const float* labels, int32_t rounds, orc_node* nodes, uint64_t nodes_cap,
                  uint64_t* tree_ptr, float* base_out, float* margins_out) {
  if (!pp || !x || !labels || n == 0 || nc == 0 || rounds < 0) return -2;
  orc_trainer* tr = orc_trainer_new(pp, x, n, nc, labels);
  if (!tr) return -2;
  int64_t got = run_rounds(tr, rounds, nodes, nodes_cap, tree_ptr);
  std::copy(tr->base.begin(), tr->base.end(), base_out);
  if (margins_out && got >= 0) std::copy(tr->margins.begin(), tr->margins.end(), margins_out);
  orc_trainer_free(tr);
  return got;
}

int64_t orc_train_csr(const orc_params* pp, const uint64_t* indptr, const uint32_t* indices,
                      const float* values, uint64_t n, uint64_t nc, const float* labels, int32_t rounds,
                      orc_node* nodes, uint64_t nodes_cap, uint64_t* tree_ptr, float* base_out,
                      float* margins_out) {
  if (!pp || !labels || n == 0 || nc == 0 || rounds < 0) return -2;
  orc_trainer* tr = orc_trainer_new_csr(pp, indptr, indices, values, n, nc, labels);
  if (!tr) return -2;
  int64_t got = run_rounds(tr, rounds, nodes, nodes_cap, tree_ptr);
  std::copy(tr->base.begin(), tr->base.end(), base_out);
  if (margins_out && got >= 0) std::copy(tr->margins.begin(), tr->margins.end(), margins_out);
  orc_trainer_free(tr);
  return got;
}

int64_t orc_cuts_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                     uint64_t n_rows, uint64_t n_cols, int32_t max_bin, uint32_t* feature_offset,
                     float* cut_values, uint64_t cap) {
  using namespace orc;
  Cuts c = cuts_from_csr(indptr, indices, values, n_rows, n_cols, (size_t)max_bin);
  if (c.values.size() > cap) return -1;
  std::copy(c.feature_offset.begin(), c.feature_offset.end(), feature_offset);
  std::copy(c.values.begin(), c.values.end(), cut_values);
  return (int64_t)c.values.size();
}

void orc_predict(const orc_node* nodes, const uint64_t* tree_ptr, uint64_t n_trees,
                 int32_t n_outputs, const uint32_t* tree_output, const float* tree_weight,
                 const float* base, const float* x, uint64_t n, uint64_t nc, float* out) {
  // BoostedModel::margin_from_trees (src/model/predict.rs:60): base, then
  // every tree in order adds weight * leaf (f32) to its output.
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)n; ++r) {
    for (int t = 0; t < n_outputs; ++t) out[r * n_outputs + t] = base[t];
    for (uint64_t ti = 0; ti < n_trees; ++ti) {
      const orc_node* tn = nodes + tree_ptr[ti];
      int id = 0;
      while (tn[id].left != -1) {
        // regtree.rs:39 / tree/mod.rs:52: x < split_cond goes left, missing follows default_left
        float v = x[r * nc + tn[id].split_feature];
        bool left = std::isnan(v) ? tn[id].default_left != 0 : v < tn[id].split_cond;
        id = left ? tn[id].left : tn[id].right;
      }
      uint32_t o = tree_output ? tree_output[ti] : (uint32_t)(ti % (uint64_t)n_outputs);
      float w = tree_weight ? tree_weight[ti] : 1.0f;
      float contrib = w * tn[id].leaf_value;
      out[r * n_outputs + o] += contrib;
    }
  }
}

void orc_hist(const float* x, uint64_t n_rows, uint64_t nc, const uint32_t* feature_offset,
              const float* cut_values, const uint32_t* rows, uint64_t n_node_rows,
              const float* gpair, int32_t fixed_point, int32_t sg, int32_t sh, double* out_f64,
              int64_t* out_i64) {
  Index ix = make_index(x, n_rows, nc, cuts_from(feature_offset, cut_values, nc));
  std::vector<uint32_t> rv(rows, rows + n_node_rows);
  const GradPair* gp = reinterpret_cast<const GradPair*>(gpair);
  size_t nb = ix.cuts.values.size();
  if (fixed_point) {
    std::vector<IS> q(n_rows);
    for (size_t r = 0; r < n_rows; ++r) {
      q[r].grad = std::llrint((double)gp[r].grad * pow2(sg));
      q[r].hess = std::llrint((double)gp[r].hess * pow2(sh));
    }
    FixMode mode;
    mode.sg = sg;
    mode.sh = sh;
    std::vector<IS> h = build_hist(ix, rv, q.data(), mode);
    for (size_t b = 0; b < nb; ++b) {
      out_i64[2 * b] = h[b].grad;
      out_i64[2 * b + 1] = h[b].hess;
    }
  } else {
    std::vector<GS> h = build_hist(ix, rv, gp, F64Mode{});
    for (size_t b = 0; b < nb; ++b) {
      out_f64[2 * b] = h[b].grad;
      out_f64[2 * b + 1] = h[b].hess;
    }
  }
}

}  // extern "C"
