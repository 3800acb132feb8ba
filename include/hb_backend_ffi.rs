// FFI declarations of libhb_cuda.so for hessboost (Rust), the module a
// maintainer adds as src/backend/b200/ffi.rs. One `extern "C"` item per entry
// point of include/hb_backend.h, with the same struct layouts (#[repr(C)]).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_void};

pub type hb_status = i32;
pub const HB_OK: hb_status = 0;
pub const HB_REFUSED: hb_status = 1;          // the trait's `None`
pub const HB_DEVICE_FAILED: hb_status = 2;    // sticky: the engine refuses from now on
pub const HB_INVALID_ARGUMENT: hb_status = 3;
pub const HB_SCAN_EMPTY: u32 = 0;             // NodeScan kinds
pub const HB_SCAN_REPLAY: u32 = 1;
pub const HB_SCAN_NUMERIC: u32 = 2;

#[repr(C)] pub struct hb_engine { _p: [u8; 0] }
#[repr(C)] pub struct hb_predictor { _p: [u8; 0] }

#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct hb_grad_stats { pub grad: f64, pub hess: f64 }            // GradStats
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct hb_grad_pair { pub grad: f32, pub hess: f32 }             // GradPair
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct hb_segment { pub offset: u64, pub len: u64, pub contiguous: u32,
                        pub reserved: u32, pub tree: u64 }          // Segment
#[repr(C)] pub struct hb_row_split { pub seg: hb_segment, pub feature: u32, pub limit: u32,
                                     pub default_left: u32, pub reserved: u32 }
#[repr(C)] #[derive(Default)]
pub struct hb_partitioned { pub left: hb_segment, pub right: hb_segment }
#[repr(C)] pub struct hb_reg_params { pub lambda: f64, pub alpha: f64,
                                      pub max_delta_step: f64, pub min_child_weight: f64 }
#[repr(C)] pub struct hb_scan_request { pub slot: u32, pub n_features: u32,
                                        pub features: *const u32, pub directions: *const i8,
                                        pub total: hb_grad_stats,
                                        pub root_gain: f32, pub lower: f32, pub upper: f32,
                                        pub reserved: u32 }   // ScanRequest: features[i], directions[i]
#[repr(C)] #[derive(Default)]
pub struct hb_node_scan { pub kind: u32, pub feature: u32, pub loss_chg: f32, pub backward: u32,
                          pub offset: u32, pub reserved: u32, pub acc: hb_grad_stats }
#[repr(C)] pub struct hb_device_loss { pub kind: i32, pub scale_pos_weight: f32,
                                       pub min_hess: f32, pub reserved: i32 }
#[repr(C)] pub struct hb_ghist { pub n_rows: u64, pub n_cols: u32, pub dense: u32,
                                 pub feature_offset: *const u32, pub cut_values: *const f32,
                                 pub columns: *const u8, pub missing: *const u64,
                                 // CSR index (columns null): GHistIndex's row CSR of global bins
                                 pub row_ptr: *const u64, pub row_bins: *const u32 }
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct hb_tree_node { pub left: i32, pub right: i32, pub split_feature: u32,
                          pub split_cond: f32, pub default_left: u32, pub leaf_value: f32,
                          pub sum_hess: f32, pub split_gain: f32, pub split_bin: i32,
                          pub reserved: u32 }                      // RegTree's Node
#[repr(C)] pub struct hb_train_params { pub objective: i32, pub max_depth: i32,
                                        pub max_leaves: i32, pub grow_policy: i32, pub eta: f32,
                                        pub lambda: f32, pub alpha: f32, pub gamma: f32,
                                        pub min_child_weight: f32, pub max_delta_step: f32,
                                        pub scale_pos_weight: f32, pub base_score: f32,
                                        pub num_class: i32, pub n_monotone: i32,
                                        pub monotone: *const i8 }  // TrainingParams (hist fields)
pub const HB_TIMERS: usize = 8;
#[repr(C)] #[derive(Default)]
pub struct hb_engine_stats { pub ms: [f64; HB_TIMERS], pub timed_launches: [u64; HB_TIMERS],
                             pub kernel_launches: u64, pub rows_built_contiguous: u64,
                             pub rows_built_gathered: u64, pub rounds: u64,
                             pub last_rounds_ms: f64 }

#[link(name = "hb_cuda")]
extern "C" {
    pub fn hb_engine_create(device_ordinal: i32, out: *mut *mut hb_engine) -> hb_status;
    pub fn hb_engine_destroy(e: *mut hb_engine) -> hb_status;
    pub fn hb_engine_upload(e: *mut hb_engine, g: *const hb_ghist) -> hb_status;
    pub fn hb_engine_last_error(e: *const hb_engine) -> *const c_char;
    pub fn hb_prepare(e: *mut hb_engine, gpair: *const hb_grad_pair, n: u64) -> hb_status;
    pub fn hb_build(e: *mut hb_engine, rows: *const u32, n: u64, out: *mut hb_grad_stats) -> hb_status;
    pub fn hb_build_features(e: *mut hb_engine, rows: *const u32, n: u64, features: *const u32,
                             n_features: u32, out: *mut hb_grad_stats) -> hb_status;
    pub fn hb_begin_tree(e: *mut hb_engine, rows: *const u32, n: u64, root: *mut hb_segment) -> hb_status;
    pub fn hb_root_total(e: *mut hb_engine, seg: *const hb_segment, out: *mut hb_grad_stats) -> hb_status;
    pub fn hb_partition(e: *mut hb_engine, splits: *const hb_row_split, n: u32,
                        out: *mut hb_partitioned) -> hb_status;
    pub fn hb_histograms(e: *mut hb_engine, segs: *const hb_segment, n: u32,
                         out: *mut hb_grad_stats) -> hb_status;
    pub fn hb_rows(e: *mut hb_engine, segs: *const hb_segment, n: u32, out: *mut u32) -> hb_status;
    pub fn hb_load_margins(e: *mut hb_engine, m: *const f32, n: u64) -> hb_status;
    pub fn hb_gradients(e: *mut hb_engine, loss: *const hb_device_loss, labels: *const f32,
                        weights: *const f32, n: u64, all_finite: *mut i32) -> hb_status;
    pub fn hb_add_leaf_values(e: *mut hb_engine, segs: *const hb_segment, values: *const f32,
                              n: u32) -> hb_status;
    pub fn hb_read_margins(e: *mut hb_engine, out: *mut f32, n: u64) -> hb_status;
    pub fn hb_reserve_hists(e: *mut hb_engine, slots: u32, reserved: *mut i32) -> hb_status;
    pub fn hb_build_resident(e: *mut hb_engine, segs: *const hb_segment, slots: *const u32, n: u32,
                             siblings: *const u32, n_siblings: u32) -> hb_status;
    pub fn hb_scan_resident(e: *mut hb_engine, reg: *const hb_reg_params,
                            req: *const hb_scan_request, n: u32, out: *mut hb_node_scan) -> hb_status;
    pub fn hb_read_hist(e: *mut hb_engine, slot: u32, out: *mut hb_grad_stats) -> hb_status;
    pub fn hb_engine_stream(e: *mut hb_engine, stream: *mut *mut c_void) -> hb_status;
    // HistCuts::from_dmatrix + GHistIndex::from_dmatrix (+ upload) on the GPU
    pub fn hb_sketch_dense(device: i32, x: *const f32, n_rows: u64, n_cols: u32, max_bin: u32,
                           feature_offset: *mut u32, cut_values: *mut f32, cap: u64, total: *mut u64,
                           columns: *mut u8, missing: *mut u64, dense: *mut i32) -> hb_status;
    pub fn hb_sketch_csr(device: i32, indptr: *const u64, indices: *const u32, values: *const f32,
                         n_rows: u64, n_cols: u32, max_bin: u32, feature_offset: *mut u32,
                         cut_values: *mut f32, cap: u64, total: *mut u64, row_bins: *mut u32,
                         dense: *mut i32) -> hb_status;
    pub fn hb_sketch_last_error() -> *const c_char;
    pub fn hb_engine_upload_dense(e: *mut hb_engine, x: *const f32, n_rows: u64, n_cols: u32,
                                  max_bin: u32, feature_offset: *mut u32, cut_values: *mut f32,
                                  cap: u64, total: *mut u64) -> hb_status;
    pub fn hb_engine_upload_csr(e: *mut hb_engine, indptr: *const u64, indices: *const u32,
                                values: *const f32, n_rows: u64, n_cols: u32, max_bin: u32,
                                feature_offset: *mut u32, cut_values: *mut f32, cap: u64,
                                total: *mut u64) -> hb_status;
    // the native model container's checksum (src/model/container.rs:245)
    pub fn hb_xxh64(data: *const c_void, len: u64, out: *mut u64) -> hb_status;
    // HistCuts / GHistIndex on the host (C++)
    pub fn hb_cuts_dense(x: *const f32, n_rows: u64, n_cols: u32, max_bin: u32,
                         feature_offset: *mut u32, cut_values: *mut f32, cap: u64,
                         total: *mut u64) -> hb_status;
    pub fn hb_bin_dense(x: *const f32, n_rows: u64, n_cols: u32, feature_offset: *const u32,
                        cut_values: *const f32, columns: *mut u8, missing: *mut u64,
                        dense: *mut i32) -> hb_status;
    pub fn hb_cuts_csr(indptr: *const u64, indices: *const u32, values: *const f32, n_rows: u64,
                       n_cols: u32, max_bin: u32, feature_offset: *mut u32, cut_values: *mut f32,
                       cap: u64, total: *mut u64) -> hb_status;
    pub fn hb_bin_csr(indptr: *const u64, indices: *const u32, values: *const f32, n_rows: u64,
                      n_cols: u32, feature_offset: *const u32, cut_values: *const f32,
                      row_ptr: *mut u64, row_bins: *mut u32, dense: *mut i32) -> hb_status;
    // whole rounds on the device (train_trees / device_round)
    pub fn hb_train(e: *mut hb_engine, p: *const hb_train_params, labels: *const f32, n: u64,
                    base_margin: f32, rounds: i32, nodes: *mut hb_tree_node, nodes_cap: u64,
                    tree_ptr: *mut u64) -> hb_status;
    pub fn hb_train_begin(e: *mut hb_engine, labels: *const f32, n: u64, base_margin: f32) -> hb_status;
    pub fn hb_train_begin_classes(e: *mut hb_engine, labels: *const f32, n: u64,
                                  base_margins: *const f32, n_classes: i32) -> hb_status;
    pub fn hb_train_rounds(e: *mut hb_engine, p: *const hb_train_params, rounds: i32,
                           nodes: *mut hb_tree_node, nodes_cap: u64, tree_ptr: *mut u64) -> hb_status;
    pub fn hb_grow_tree(e: *mut hb_engine, p: *const hb_train_params, nodes: *mut hb_tree_node,
                        nodes_cap: u32, n_nodes: *mut u32) -> hb_status;
    pub fn hb_read_gradients(e: *mut hb_engine, out: *mut hb_grad_pair, n: u64, sg: *mut i32,
                             sh: *mut i32) -> hb_status;
    pub fn hb_build_noalloc(e: *mut hb_engine, rows_dev: *const u32, n: u64,
                            out_dev: *mut hb_grad_stats) -> hb_status;
    pub fn hb_engine_reset_stats(e: *mut hb_engine, timing: i32) -> hb_status;
    pub fn hb_engine_get_stats(e: *mut hb_engine, out: *mut hb_engine_stats) -> hb_status;
    // row sharding over the GPUs of a node
    pub fn hb_engine_set_shard(e: *mut hb_engine, row_begin: u64, global_rows: u64) -> hb_status;
    pub fn hb_comm_unique_id(id: *mut u8) -> hb_status;                 // 128 bytes
    pub fn hb_comm_init(e: *mut hb_engine, nranks: i32, rank: i32, id: *const u8,
                        global_rows: u64) -> hb_status;
    // BoostedModel::to_cuda / GpuModel::predict_margin
    pub fn hb_predictor_create(device_ordinal: i32, nodes: *const hb_tree_node, tree_ptr: *const u64,
                               n_trees: u64, tree_output: *const u32, tree_weight: *const f32,
                               n_outputs: i32, base: *const f32, n_features: u32,
                               out: *mut *mut hb_predictor) -> hb_status;
    pub fn hb_predictor_destroy(p: *mut hb_predictor) -> hb_status;
    pub fn hb_predict_margin(p: *mut hb_predictor, rows: *const f32, n_rows: u64, out: *mut f32) -> hb_status;
    pub fn hb_predict_margin_device(p: *mut hb_predictor, d_rows: *const f32, n_rows: u64,
                                    d_out: *mut f32, stream: *mut c_void) -> hb_status;
    pub fn hb_probe_smem(device: i32, kind: i32, threads: i32, iters: i32,
                         lane_ops_per_clk: *mut f64) -> hb_status;
    pub fn hb_engine_inject_fault(e: *mut hb_engine, after_calls: i32) -> hb_status;
    pub fn hb_peer_wait_probe(device: i32, timeout_ms: i32, status: *mut u64, waited_ms: *mut f64) -> hb_status;
}
