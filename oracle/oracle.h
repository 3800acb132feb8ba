/* TEST INFRASTRUCTURE ONLY: the C API of the CPU oracle (see
 * oracle_internal.h). Loaded by the tests, smoke() and bench.py's
 * cpu_baseline leg through ctypes; never by the product library. */
#ifndef HB_ORACLE_H
#define HB_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One tree node, field for field the reference's `Node`
 * (src/tree/regtree.rs:37) plus the split's global bin. 40 bytes. */
typedef struct orc_node {
  int32_t left;            /* -1 for a leaf */
  int32_t right;
  uint32_t split_feature;
  float split_cond;        /* x < split_cond goes left */
  uint32_t default_left;   /* 0/1 */
  float leaf_value;
  float sum_hess;
  float split_gain;
  int32_t split_bin;       /* last global bin routed left; -1 = below every bin */
  uint32_t reserved;
} orc_node;

typedef struct orc_params {
  int32_t objective;       /* 0 reg:squarederror, 1 binary:logistic, 2 multi:softmax */
  int32_t n_outputs;       /* label columns (squared error), classes (softmax) */
  int32_t max_depth;
  int32_t max_leaves;      /* 0 = unlimited */
  int32_t grow_policy;     /* 0 depthwise, 1 lossguide */
  int32_t max_bin;
  float eta;
  float lambda;
  float alpha;
  float gamma;
  float min_child_weight;
  float max_delta_step;
  float scale_pos_weight;
  float base_score;        /* NaN: estimate from the labels */
  int32_t fixed_point;     /* 0: the reference's f64 sums; 1: int64 fixed-point sums */
  int32_t n_threads;       /* 0: all */
  const int8_t* monotone;  /* per feature +1 / -1 / 0 (monotone_constraints); NULL: none */
  int32_t n_monotone;
  int32_t reserved;
} orc_params;

/* HistCuts::from_dmatrix of a dense row-major matrix (NaN = missing).
 * Returns the total bin count, or -1 when `cap` is too small. */
int64_t orc_cuts_dense(const float* x, uint64_t n_rows, uint64_t n_cols, const float* weights,
                       uint32_t max_bin, uint32_t* feature_offset, float* cut_values, uint64_t cap);

/* Feature-local bins, feature-major (bins[f * n + r]; 0 for a missing cell)
 * and the missing bitmap (words[f * ceil(n/64) + r/64] bit r%64). Returns 1
 * when no cell is missing. */
int32_t orc_bin_dense(const float* x, uint64_t n_rows, uint64_t n_cols,
                      const uint32_t* feature_offset, const float* cut_values,
                      uint16_t* bins, uint64_t* missing);

/* Gradient pairs (g, h interleaved) of `objective` at `margins`. */
void orc_gradients(int32_t objective, const float* margins, const float* labels, uint64_t n,
                   float scale_pos_weight, float* gpair);

/* multi:softmax gradient pairs of `k` classes at row-major margins
 * (n x k), labels the class ids, pairs row-major like the margins. */
void orc_softmax_gradients(const float* margins, const float* labels, uint64_t n, int32_t k,
                           float* gpair);

/* Base margin for each of `n_outputs` label columns (labels row-major); for
 * multi:softmax (objective 2) the n_outputs class intercepts of the class
 * ids in `labels`. */
void orc_intercepts(int32_t objective, const float* labels, uint64_t n, int32_t n_outputs,
                    float* out);

/* Train `rounds` rounds. Writes the trees' nodes back to back, tree t at
 * nodes[tree_ptr[t] .. tree_ptr[t+1]), the base margins and the final
 * training margins (row-major, n_outputs per row). Returns the tree count,
 * or -1 when `nodes_cap` is too small, -2 on a bad argument, -3 when the
 * fixed-point mode meets a non-finite gradient. */
int64_t orc_train(const orc_params* p, const float* x, uint64_t n, uint64_t n_cols,
                  const float* labels, int32_t rounds, orc_node* nodes, uint64_t nodes_cap,
                  uint64_t* tree_ptr, float* base_out, float* margins_out);

/* A training session: cuts, binning and intercepts once (orc_trainer_new),
 * then rounds from the session's margins (orc_trainer_rounds), so the rounds
 * can be timed alone. */
typedef struct orc_trainer orc_trainer;
orc_trainer* orc_trainer_new(const orc_params* p, const float* x, uint64_t n, uint64_t n_cols,
                             const float* labels);
int64_t orc_trainer_rounds(orc_trainer* t, int32_t rounds, orc_node* nodes, uint64_t nodes_cap,
                           uint64_t* tree_ptr);
void orc_trainer_free(orc_trainer* t);
/* The session's training margins (n * n_outputs, row-major): copied to `out`
 * when `cap` holds them; returns their count. */
uint64_t orc_trainer_margins(const orc_trainer* t, float* out, uint64_t cap);
/* Replace the session's training margins (the next round's gradients are
 * taken there); -2 when `n` is not the session's margin count. */
int32_t orc_trainer_set_margins(orc_trainer* t, const float* m, uint64_t n);

/* The same on a CSR matrix (DMatrix::from_csr: absent cells missing),
 * binned into a CSR index of global bins (only stored cells are read). */
orc_trainer* orc_trainer_new_csr(const orc_params* p, const uint64_t* indptr, const uint32_t* indices,
                                 const float* values, uint64_t n, uint64_t n_cols, const float* labels);
int64_t orc_train_csr(const orc_params* p, const uint64_t* indptr, const uint32_t* indices,
                      const float* values, uint64_t n, uint64_t n_cols, const float* labels, int32_t rounds,
                      orc_node* nodes, uint64_t nodes_cap, uint64_t* tree_ptr, float* base_out,
                      float* margins_out);
int64_t orc_cuts_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                     uint64_t n_rows, uint64_t n_cols, int32_t max_bin, uint32_t* feature_offset,
                     float* cut_values, uint64_t cap);

/* Raw margins: base + sum over trees in order of weight * leaf, tree t
 * adding to output tree_output[t] (NULL: t % n_outputs) with weight
 * tree_weight[t] (NULL: 1). */
void orc_predict(const orc_node* nodes, const uint64_t* tree_ptr, uint64_t n_trees,
                 int32_t n_outputs, const uint32_t* tree_output, const float* tree_weight,
                 const float* base, const float* x, uint64_t n, uint64_t n_cols, float* out);

/* One node's histogram over `rows` (ascending) of a binned dense matrix:
 * the reference's f64 sums in CpuBackend's order (out_f64: 2 per bin) or
 * the int64 fixed-point sums (out_i64: 2 per bin) with scales 2^sg, 2^sh. */
void orc_hist(const float* x, uint64_t n_rows, uint64_t n_cols, const uint32_t* feature_offset,
              const float* cut_values, const uint32_t* rows, uint64_t n_node_rows,
              const float* gpair, int32_t fixed_point, int32_t sg, int32_t sh, double* out_f64,
              int64_t* out_i64);

/* One node's split search in fixed point (the RowEngine scan seam): the
 * node's int64 histogram (2 per bin) and totals with scales 2^sg, 2^sh, its
 * monotone bounds, and the features to scan in order with their directions
 * (NULL: none); the winner of HistTreeBuilder::evaluate over them. */
typedef struct orc_scan {
  int32_t found;          /* 0: no candidate beats the empty split */
  uint32_t feature;
  int32_t bin;            /* last global bin going left, -1 = below every bin */
  uint32_t default_left;
  float loss_chg;
  float root_gain;
  int64_t left_g, left_h; /* left child statistics (fixed point) */
  float w_left, w_right;  /* bounded child weights */
} orc_scan;
int32_t orc_scan_node(const orc_params* p, const uint32_t* feature_offset, uint32_t n_cols, int32_t dense,
                      const int64_t* hist, int64_t total_g, int64_t total_h, int32_t sg, int32_t sh,
                      float lower, float upper, const uint32_t* features, const int8_t* directions,
                      uint32_t n_features, orc_scan* out);

/* The fixed-point scale exponent for values of largest magnitude `max_abs`
 * summed over `n` rows: every |rint(v * 2^s)| * n stays within 2^53, so
 * every sum is an integer an f64 holds exactly. */
int32_t orc_fixed_scale(float max_abs, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif
