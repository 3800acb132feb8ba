/*
 * hb_backend.h -- C ABI of the B200 hist backend (libhb_cuda.so).
 *
 * One function per method of hessboost's histogram backend seam, with the
 * same meaning, so the Rust side (`CudaHistBackend` in hessboost 0.4.9)
 * could bind it with `extern "C"` unchanged:
 *
 *   trait HistogramBackend   src/tree/hist/mod.rs:73-105
 *   trait RowEngine          src/tree/hist/mod.rs:213-295
 *   CudaHistBackend          src/backend/cuda/mod.rs:1445 (new :1626, upload :1687)
 *   BoostedModel::to_cuda    src/backend/cuda/predict.rs:501
 *   GpuModel::predict_margin src/backend/cuda/predict.rs:401
 *
 * plus entry points the reference does not have: whole-tree growth on the
 * device (`hb_grow_tree`, `hb_train`), the row-sharded communicator
 * (`hb_comm_*`), the host binning helpers (`hb_cuts_dense`,
 * `hb_bin_dense`, `hb_cuts_csr`, `hb_bin_csr`) and the model-file checksum
 * (`hb_xxh64`).
 *
 * Conventions (the reference's, src/tree/hist/mod.rs:107-212):
 *   - every call returns an hb_status; HB_REFUSED means "did not run"
 *     (the trait's `None`): the caller keeps its host path;
 *     HB_DEVICE_FAILED is sticky: after a CUDA or NCCL error every later
 *     call on the engine is refused;
 *   - the caller owns every host buffer and passes pointers and lengths; the
 *     engine copies what it keeps;
 *   - segments carry their tree's stamp; a segment from an earlier tree is
 *     refused;
 *   - calls on one engine must not overlap (one calling thread at a time);
 *     different engines are independent.
 *
 * Histograms are summed in int64 fixed point: each tree's gradients are
 * rounded once to multiples of 2^-s (s per component, chosen from the
 * largest magnitude and the row count so no sum can overflow 2^62) and every
 * sum is then exact, so a histogram does not depend on row order, block
 * order or GPU count. The f64 values returned are those exact sums rounded
 * once to f64.
 */
#ifndef HB_BACKEND_H
#define HB_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t hb_status;
#define HB_OK 0
#define HB_REFUSED 1
#define HB_DEVICE_FAILED 2
#define HB_INVALID_ARGUMENT 3

typedef struct hb_engine hb_engine;
typedef struct hb_predictor hb_predictor;

/* GradStats (src/tree/gain.rs:21). */
typedef struct hb_grad_stats {
  double grad;
  double hess;
} hb_grad_stats;

/* GradPair (src/objective/mod.rs). */
typedef struct hb_grad_pair {
  float grad;
  float hess;
} hb_grad_pair;

/* Segment (src/tree/hist/mod.rs:115): `len` ascending row ids at `offset`
 * of the engine's row buffer. */
typedef struct hb_segment {
  uint64_t offset;
  uint64_t len;
  uint32_t contiguous;
  uint32_t reserved;
  uint64_t tree;
} hb_segment;

/* RowSplit (src/tree/hist/mod.rs:183) with RowRule::Below(limit): present
 * feature-local bins below `limit` go left, missing values follow
 * `default_left`. */
typedef struct hb_row_split {
  hb_segment seg;
  uint32_t feature;
  uint32_t limit;
  uint32_t default_left;
  uint32_t reserved;
} hb_row_split;

/* Partitioned (src/tree/hist/mod.rs:196). */
typedef struct hb_partitioned {
  hb_segment left;
  hb_segment right;
} hb_partitioned;

/* RegParams (src/tree/gain.rs:62), every value already rounded to f32. */
typedef struct hb_reg_params {
  double lambda;
  double alpha;
  double max_delta_step;
  double min_child_weight;
} hb_reg_params;

/* ScanRequest (src/tree/hist/mod.rs:303): the node's histogram slot, its
 * statistics, root_gain and monotone bounds as the scorer uses them (f32),
 * and the features to scan, `features[i]` with monotone direction
 * `directions[i]` (+1, -1, 0; NULL: all 0), merged in that order. */
typedef struct hb_scan_request {
  uint32_t slot;
  uint32_t n_features;
  const uint32_t* features;
  const int8_t* directions;
  hb_grad_stats total;
  float root_gain;
  float lower;
  float upper;
  uint32_t reserved;
} hb_scan_request;

#define HB_SCAN_EMPTY 0
#define HB_SCAN_REPLAY 1
#define HB_SCAN_NUMERIC 2
/* NodeScan (src/tree/hist/mod.rs:327): the winning numeric split of a node
 * after the feature-order merge; `acc` is the pass's accumulated statistics
 * (the left child for a forward pass, the right child for a backward one). */
typedef struct hb_node_scan {
  uint32_t kind;
  uint32_t feature;
  float loss_chg;
  uint32_t backward;
  uint32_t offset;
  uint32_t reserved;
  hb_grad_stats acc;
} hb_node_scan;

#define HB_LOSS_SQUARED_ERROR 0
#define HB_LOSS_LOGISTIC 1
#define HB_LOSS_SOFTMAX 2 /* multi:softmax (objective/multiclass.rs), device growth only */
/* DeviceLoss (src/tree/hist/mod.rs:352). */
typedef struct hb_device_loss {
  int32_t kind;
  float scale_pos_weight;
  float min_hess;
  int32_t reserved;
} hb_device_loss;

/* The binned matrix the backend uploads (GHistIndex, src/data/ghist.rs:195),
 * in one of two layouts (features of at most 256 bins either way):
 *   columns: every feature's local bins, feature-major, one byte each, and
 *            the missing bitmap of an index with missing entries (at most
 *            224 features);
 *   CSR:     `columns` NULL; the stored entries' global bins row by row
 *            (ghist.rs:6-21 `rows`), ascending within a row, offsets in
 *            `row_ptr`; an absent feature is missing. */
/* GHistIndex (src/data/ghist.rs:195). A dense index (columns set) keeps
 * one-byte local bins, so each feature has at most 256 bins; one of more
 * than 224 features is converted to the CSR form on upload. A CSR index
 * (columns NULL) allows up to 65,535 bins a feature. */
typedef struct hb_ghist {
  uint64_t n_rows;
  uint32_t n_cols;
  uint32_t dense;                 /* every row holds every feature */
  const uint32_t* feature_offset; /* n_cols + 1 */
  const float* cut_values;        /* feature_offset[n_cols] */
  const uint8_t* columns;         /* bins[f * n_rows + r], or NULL for CSR */
  const uint64_t* missing;        /* NULL, or bit r%64 of word f*ceil(n_rows/64) + r/64 */
  const uint64_t* row_ptr;        /* CSR: n_rows + 1 offsets from 0 */
  const uint32_t* row_bins;       /* CSR: row_ptr[n_rows] global bins */
} hb_ghist;

/* One tree node: the reference's Node (src/tree/regtree.rs:37) plus the
 * split's global bin (-1: below every bin). 40 bytes. */
typedef struct hb_tree_node {
  int32_t left;
  int32_t right;
  uint32_t split_feature;
  float split_cond;
  uint32_t default_left;
  float leaf_value;
  float sum_hess;
  float split_gain;
  int32_t split_bin;
  uint32_t reserved;
} hb_tree_node;

#define HB_GROW_DEPTHWISE 0
#define HB_GROW_LOSSGUIDE 1
/* The TrainingParams fields the hist path reads (src/config/params.rs:653). */
typedef struct hb_train_params {
  int32_t objective;        /* HB_LOSS_* */
  int32_t max_depth;        /* 0: unlimited */
  int32_t max_leaves;       /* 0: unlimited */
  int32_t grow_policy;      /* HB_GROW_* */
  float eta;
  float lambda;
  float alpha;
  float gamma;
  float min_child_weight;
  float max_delta_step;
  float scale_pos_weight;
  float base_score;         /* NaN: estimate from the labels */
  int32_t num_class;        /* HB_LOSS_SOFTMAX: classes (2..64); else 0 or 1 */
  /* monotone_constraints (src/config/params.rs, Monotone): one direction
   * per feature, +1 increasing, -1 decreasing, 0 none; features past
   * n_monotone are unconstrained. NULL / 0: none. */
  int32_t n_monotone;
  const int8_t* monotone;
} hb_train_params;

/* ---- engine (CudaHistBackend::new + upload) ------------------------- */
hb_status hb_engine_create(int32_t device_ordinal, hb_engine** out);
hb_status hb_engine_destroy(hb_engine* e);
/* CudaHistBackend::upload (src/backend/cuda/mod.rs:1687). */
hb_status hb_engine_upload(hb_engine* e, const hb_ghist* ghist);
/* Human-readable text of the engine's last error (static storage). */
const char* hb_engine_last_error(const hb_engine* e);

/* ---- HistogramBackend (src/tree/hist/mod.rs:73) -------------------- */
/* `prepare`: stage this tree's gradients (one pair per row). */
hb_status hb_prepare(hb_engine* e, const hb_grad_pair* gpair, uint64_t n_rows);
/* `build`: the histogram of `rows` (ascending) into out[total_bins]. */
hb_status hb_build(hb_engine* e, const uint32_t* rows, uint64_t n, hb_grad_stats* out);
/* `build_features`: every bin is built; the feature list only says which
 * bins the caller reads. */
hb_status hb_build_features(hb_engine* e, const uint32_t* rows, uint64_t n,
                            const uint32_t* features, uint32_t n_features, hb_grad_stats* out);

/* hb_build for callers that may not allocate device memory while they run
 * (a host framework that owns all of HBM through its own pool, say). No
 * counterpart in the reference. `rows_dev` (n ascending row ids, u32) and
 * `out_dev` (total_bins (grad, hess) pairs, f64) are device memory of the
 * engine's GPU; the histogram is written to out_dev and the call returns
 * after its kernels finish. Its working memory is one static device array
 * of 512 KiB per device, which limits the index to 32,768 bins (refused
 * above that). It allocates nothing: the first call on a device only looks
 * up that array's address, and should come before any stream capture.
 * Calls on one device share the array; the library serialises them, since
 * overlapping calls would race on it. Bad row ids (not ascending, or past
 * the index) are refused with out_dev zeroed; no row is read. The kernels
 * run on the engine's stream, so rows_dev must be complete when the call
 * starts (synchronise the stream that wrote it first). HB_INVALID_ARGUMENT,
 * with the reason in hb_engine_last_error, for a NULL buffer, more row ids
 * than the index has rows, or out_dev not 8-byte / rows_dev not 4-byte
 * aligned. */
hb_status hb_build_noalloc(hb_engine* e, const uint32_t* rows_dev, uint64_t n,
                           hb_grad_stats* out_dev);

/* ---- RowEngine (src/tree/hist/mod.rs:213) -------------------------- */
hb_status hb_begin_tree(hb_engine* e, const uint32_t* rows, uint64_t n, hb_segment* root);
hb_status hb_root_total(hb_engine* e, const hb_segment* seg, hb_grad_stats* out);
hb_status hb_partition(hb_engine* e, const hb_row_split* splits, uint32_t n,
                       hb_partitioned* out);
/* `histograms`: out[k * total_bins + bin] for the k-th segment. */
hb_status hb_histograms(hb_engine* e, const hb_segment* segs, uint32_t n, hb_grad_stats* out);
/* `rows`: the row ids of each segment, back to back. */
hb_status hb_rows(hb_engine* e, const hb_segment* segs, uint32_t n, uint32_t* out);
hb_status hb_load_margins(hb_engine* e, const float* margins, uint64_t n);
/* `gradients`: the loss's pairs at the device margins; *all_finite as the
 * trait's bool. */
hb_status hb_gradients(hb_engine* e, const hb_device_loss* loss, const float* labels,
                       const float* weights, uint64_t n, int32_t* all_finite);
hb_status hb_add_leaf_values(hb_engine* e, const hb_segment* segs, const float* values,
                             uint32_t n);
/* n = rows, or rows * classes after hb_train_begin_classes (class-major:
 * out[k * rows + r]). */
hb_status hb_read_margins(hb_engine* e, float* out, uint64_t n);
hb_status hb_reserve_hists(hb_engine* e, uint32_t slots, int32_t* reserved);
/* `build_resident`: build nodes[k] into slots[k], then for each pair
 * (siblings[2j] = parent, siblings[2j+1] = built) turn the parent slot into
 * parent - built. */
hb_status hb_build_resident(hb_engine* e, const hb_segment* segs, const uint32_t* slots,
                            uint32_t n, const uint32_t* siblings, uint32_t n_siblings);
hb_status hb_scan_resident(hb_engine* e, const hb_reg_params* reg,
                           const hb_scan_request* requests, uint32_t n, hb_node_scan* out);
hb_status hb_read_hist(hb_engine* e, uint32_t slot, hb_grad_stats* out);
/* Diagnostics (src/backend/cuda/diagnostics.rs): the staged gradient pairs
 * and the fixed-point exponents (sg, sh) of the current tree. */
hb_status hb_read_gradients(hb_engine* e, hb_grad_pair* out, uint64_t n, int32_t* sg, int32_t* sh);

/* ---- whole-tree growth on the device (no reference counterpart) ---- */
/* Grow one tree from the device gradients (hb_gradients or hb_prepare)
 * with every row, the host builder's semantics (HistTreeBuilder,
 * src/tree/builder/hist/mod.rs:261), add its eta-scaled leaves to the
 * device margins, and return its nodes. */
hb_status hb_grow_tree(hb_engine* e, const hb_train_params* p, hb_tree_node* nodes,
                       uint32_t nodes_cap, uint32_t* n_nodes);
/* `rounds` boosting rounds (train_trees, src/training/train.rs:222) of a
 * single-output objective from `base_margin`: hb_train_begin then
 * hb_train_rounds. */
hb_status hb_train(hb_engine* e, const hb_train_params* p, const float* labels, uint64_t n,
                   float base_margin, int32_t rounds, hb_tree_node* nodes, uint64_t nodes_cap,
                   uint64_t* tree_ptr);
/* Start a training run: stage the labels and set every device margin to
 * `base_margin`. */
hb_status hb_train_begin(hb_engine* e, const float* labels, uint64_t n, float base_margin);
/* Start a multi:softmax run of `n_classes` outputs (train_trees with
 * Softmax, src/objective/multiclass.rs): `labels` holds each row's class id
 * (an integer in [0, n_classes)), `base_margins` one margin per class. Each
 * hb_train_rounds round then computes the softmax gradients of every class
 * on the device and grows one tree per class in class order, so the round's
 * trees are nodes[tree_ptr[r * n_classes + k] ...]; size tree_ptr for
 * rounds * n_classes + 1. */
hb_status hb_train_begin_classes(hb_engine* e, const float* labels, uint64_t n,
                                 const float* base_margins, int32_t n_classes);
/* Continue the run by `rounds` rounds (gradients at the device margins, one
 * tree grown on the device, its leaves added to the margins), writing the
 * rounds' trees back to back: tree t at nodes[tree_ptr[t] .. tree_ptr[t+1]). */
hb_status hb_train_rounds(hb_engine* e, const hb_train_params* p, int32_t rounds,
                          hb_tree_node* nodes, uint64_t nodes_cap, uint64_t* tree_ptr);

/* Counters of the engine since the last hb_engine_reset_stats: device time
 * per kernel family (CUDA events on the engine's stream, recorded only when
 * `timing` was switched on), kernel launches, and rows the histogram kernel
 * built with and without a row list. */
#define HB_TIMERS 8 /* gradients, root hist, scan, apply, partition, hist, subtract, other */
typedef struct hb_engine_stats {
  double ms[HB_TIMERS];
  uint64_t timed_launches[HB_TIMERS];
  uint64_t kernel_launches;
  uint64_t rows_built_contiguous;
  uint64_t rows_built_gathered;
  uint64_t rounds;
  /* device time of the last hb_train_rounds call's rounds: CUDA events on
   * the engine's stream right before the first round's work and after the
   * last (graph capture and the trees' read-back excluded) */
  double last_rounds_ms;
} hb_engine_stats;
/* timing: 0 none, 1 events around the histogram kernel only (the light
 * setting for a timed run), 2 events around every kernel family. */
hb_status hb_engine_reset_stats(hb_engine* e, int32_t timing);
hb_status hb_engine_get_stats(hb_engine* e, hb_engine_stats* out);
/* The engine's CUDA stream (a cudaStream_t), for callers that order their
 * own work or events against it. */
hb_status hb_engine_stream(hb_engine* e, void** stream);

/* ---- row sharding over several GPUs (no reference counterpart) ------ */
/* The engine holds rows [row_begin, row_begin + n_rows) of a matrix of
 * `global_rows`; histograms, totals and scales are summed (max-reduced)
 * over every rank with NCCL, so each rank grows the same tree. */
/* Declare this engine's shard before hb_engine_upload: its first row's
 * global index (a multiple of 8, so the logistic gradient's 8-row vectors
 * line up with the whole matrix's) and the matrix's total row count. */
hb_status hb_engine_set_shard(hb_engine* e, uint64_t row_begin, uint64_t global_rows);
hb_status hb_comm_unique_id(uint8_t id[128]);
hb_status hb_comm_init(hb_engine* e, int32_t nranks, int32_t rank, const uint8_t id[128],
                       uint64_t global_rows);

/* ---- prediction (BoostedModel::to_cuda / GpuModel) ----------------- */
hb_status hb_predictor_create(int32_t device_ordinal, const hb_tree_node* nodes,
                              const uint64_t* tree_ptr, uint64_t n_trees,
                              const uint32_t* tree_output, const float* tree_weight,
                              int32_t n_outputs, const float* base, uint32_t n_features,
                              hb_predictor** out);
hb_status hb_predictor_destroy(hb_predictor* p);
/* Host rows in, host margins out (row-major, n_outputs per row). */
hb_status hb_predict_margin(hb_predictor* p, const float* rows, uint64_t n_rows, float* out);
/* Device rows in, device margins out, on `stream` (a cudaStream_t; NULL =
 * the predictor's stream). */
hb_status hb_predict_margin_device(hb_predictor* p, const float* d_rows, uint64_t n_rows,
                                   float* d_out, void* stream);

/* ---- host binning (HistCuts::from_dmatrix, GHistIndex::from_dmatrix) */
/* Cuts of a dense row-major f32 matrix (NaN missing); *total = bin count.
 * HB_REFUSED when `cap` is too small. */
hb_status hb_cuts_dense(const float* x, uint64_t n_rows, uint32_t n_cols, uint32_t max_bin,
                        uint32_t* feature_offset, float* cut_values, uint64_t cap,
                        uint64_t* total);
/* Feature-local one-byte bins (feature-major) and the missing bitmap;
 * *dense = 1 when no cell is missing. HB_REFUSED when a feature has more
 * than 256 bins. */
hb_status hb_bin_dense(const float* x, uint64_t n_rows, uint32_t n_cols,
                       const uint32_t* feature_offset, const float* cut_values,
                       uint8_t* columns, uint64_t* missing, int32_t* dense);

/* Cuts of a CSR matrix (DMatrix::from_csr, src/data/dmatrix.rs:459: absent
 * entries missing; stored values finite, columns in range, none twice in a
 * row, else HB_INVALID_ARGUMENT), each feature's entries in row order
 * (quantile.rs:199). */
hb_status hb_cuts_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                      uint64_t n_rows, uint32_t n_cols, uint32_t max_bin, uint32_t* feature_offset,
                      float* cut_values, uint64_t cap, uint64_t* total);
/* The CSR index: row_ptr (n_rows + 1, = indptr) and every entry's global
 * bin, ascending within its row. HB_REFUSED when a feature has more than
 * 65,535 bins. */
hb_status hb_bin_csr(const uint64_t* indptr, const uint32_t* indices, const float* values,
                     uint64_t n_rows, uint32_t n_cols, const uint32_t* feature_offset,
                     const float* cut_values, uint64_t* row_ptr, uint32_t* row_bins,
                     int32_t* dense);

/* ---- device sketch and binning (HistCuts::from_dmatrix,
 * GHistIndex::from_dmatrix on the GPU) ----------------------------------
 * The same cut values, bit for bit, as hb_cuts_dense / hb_cuts_csr (the
 * reference's WQSketch, src/data/sketch.rs:477-667, fed as
 * src/data/quantile.rs:115 `build` feeds it with unit weights), computed
 * on `device`. HB_REFUSED (reason in hb_sketch_last_error) where the device
 * sketch does not apply and the host functions must be used: a feature with
 * 2^24 or more present values, max_bin above 256, a CSR row whose column
 * indices do not strictly ascend. */
/* Cuts of a dense row-major f32 matrix (NaN missing), and, when `columns`
 * is not NULL, the hb_bin_dense outputs (`missing` may be NULL). */
hb_status hb_sketch_dense(int32_t device, const float* x, uint64_t n_rows, uint32_t n_cols,
                          uint32_t max_bin, uint32_t* feature_offset, float* cut_values,
                          uint64_t cap, uint64_t* total, uint8_t* columns, uint64_t* missing,
                          int32_t* dense);
/* Cuts of a CSR matrix (hb_cuts_csr's checks) and, when `row_bins` is not
 * NULL, the hb_bin_csr bins (row_ptr is `indptr` itself). */
hb_status hb_sketch_csr(int32_t device, const uint64_t* indptr, const uint32_t* indices,
                        const float* values, uint64_t n_rows, uint32_t n_cols, uint32_t max_bin,
                        uint32_t* feature_offset, float* cut_values, uint64_t cap, uint64_t* total,
                        uint32_t* row_bins, int32_t* dense);
/* The reason for the calling thread's last hb_sketch_* failure ("" after a
 * success); valid until that thread's next hb_sketch_* call. */
const char* hb_sketch_last_error(void);
/* CudaHistBackend::new(index) for a raw host matrix: the engine copies it
 * to its device, sketches and bins it there into its resident index, and
 * returns the cuts (the caller keeps them for the model's split values).
 * Equivalent to hb_cuts_dense + hb_bin_dense + hb_engine_upload. */
hb_status hb_engine_upload_dense(hb_engine* e, const float* x, uint64_t n_rows, uint32_t n_cols,
                                 uint32_t max_bin, uint32_t* feature_offset, float* cut_values,
                                 uint64_t cap, uint64_t* total);
/* The CSR twin: hb_cuts_csr + hb_bin_csr + hb_engine_upload. */
hb_status hb_engine_upload_csr(hb_engine* e, const uint64_t* indptr, const uint32_t* indices,
                               const float* values, uint64_t n_rows, uint32_t n_cols,
                               uint32_t max_bin, uint32_t* feature_offset, float* cut_values,
                               uint64_t cap, uint64_t* total);

/* ---- native binary model files (BoostedModel::encode/decode,
 * src/model/native.rs, src/model/container.rs) ---------------------------
 * XXH64 (seed 0) of `len` bytes: the checksum that closes a native model
 * container (container.rs:245 `xxh64`). The section table itself is laid
 * out by the Python host (model_io.to_native_binary). */
hb_status hb_xxh64(const void* data, uint64_t len, uint64_t* out);

/* ---- failure testing (no counterpart in the reference) -------------- */
/* Arm a host-side fault: the engine's `after_calls`-th checked CUDA call
 * from now on (0: the next one), counting only calls made outside stream
 * capture, fails before it reaches CUDA, exactly as a device error would:
 * that call returns HB_DEVICE_FAILED and the engine refuses every later
 * call (the sticky state of src/backend/cuda/driver.rs:26-44), while the
 * GPU and other engines are untouched. -1 disarms. For tests of the
 * caller's fallback (src/tree/hist/mod.rs:209-212). */
hb_status hb_engine_inject_fault(hb_engine* e, int32_t after_calls);

/* ---- measurement (no counterpart in the reference) ------------------ */
/* The shared-memory throughput a histogram update pattern reaches on GPU
 * `device`: one CTA of `threads` threads per SM issues `iters` iterations
 * of pattern `kind` (0 conflict-free red.u32, 1 red.u64, 2 atom.u32 with
 * its result used, 3 ld+st, 4 four red.u32 at random rows, 5 two red.u64
 * at random rows, 6 one word per warp); *lane_ops_per_clk receives lane
 * operations per SM clock cycle (clock64), the slowest SM's. */
hb_status hb_probe_smem(int32_t device, int32_t kind, int32_t threads, int32_t iters,
                        double* lane_ops_per_clk);

/* The bounded wait of the peer-memory histogram exchange, on one GPU: one
 * CTA waits for a peer flag that nothing raises, limited to timeout_ms of
 * the GPU's global timer. *status receives the barrier block's status word
 * afterwards (1: the wait gave up), *waited_ms the kernel's event time.
 * The multi-GPU exchange fails an engine the same way when a rank does not
 * arrive (hb_train_rounds then returns HB_DEVICE_FAILED). */
hb_status hb_peer_wait_probe(int32_t device, int32_t timeout_ms, uint64_t* status, double* waited_ms);

#ifdef __cplusplus
}
#endif
#endif /* HB_BACKEND_H */
