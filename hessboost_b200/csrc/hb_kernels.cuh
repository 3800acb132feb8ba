// Kernel launchers of the hist path (definitions in hb_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "hb_internal.h"

namespace hb {

// Kernels of the round are launched with programmatic stream serialization
// (launch_pdl): a kernel may be scheduled while the one before it on the
// stream finishes, so each begins with pdl_wait(), which waits for that
// kernel's completion and memory (griddepcontrol.wait, a no-op after a
// plain launch) and lets the next kernel be scheduled in turn. This hides
// the launch latency between the round's dependent kernels.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
}

extern bool g_pdl;  // false (HB_NO_PDL=1): plain launches

template <typename... P, typename... A>
inline void launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = g_pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

// Objective gradients at `margin` (the host's bits, see hb_kernels.cu) plus
// the largest |g|, |h| and a non-finite flag, folded into `scale`.
// With `wtree` and *pending set, each row first adds its leaf of that tree
// to its margin (walk_depth > 0: a depthwise tree of that depth, which the
// row-block kernel walks as a complete tree). With blk_pair != 0 each pair
// is also written into the row's block (blk rows a 128-byte line of `rec`).
void launch_gradients(int kind, float* margin, const float* label, const float* weight, float spw,
                      float min_hess, uint64_t n, uint64_t vrows, float2* gpair, Scale* scale,
                      const WNode* wtree, const LevelState* ls_last, int max_nodes, int walk_depth,
                      uint8_t* rec, uint32_t stride, uint32_t mask_off, uint32_t blk, uint32_t blk_pair,
                      const int* pending, int n_sm, cudaStream_t s);
// When *pending is set, add each row's leaf of `wtree` to its margin.
void launch_walk(const WNode* wtree, const LevelState* ls_last, int max_nodes, const uint8_t* rec,
                 uint32_t stride, uint32_t mask_off, uint32_t blk, uint64_t n, float* margin,
                 const int* pending, int n_sm, cudaStream_t s);
// multi:softmax gradients of K classes (class-major margins and pairs,
// K <= 64), first adding each class's pending tree when *pending is set;
// per-class maxima into scale[0..K).
// (K = 2 and 4: the first vrows rows in 8-lane vectors of whole rows.)
void launch_softmax_gradients(int K, float* margin, const float* label, uint64_t n, uint64_t vrows,
                              float min_hess, float2* gpair, Scale* scale, const WNode* wtree,
                              uint32_t wstride, const uint8_t* rec, uint32_t stride, uint32_t mask_off,
                              uint32_t blk, const int* pending, int n_sm, cudaStream_t s);
// When *pending is set, add each class's tree leaves to its margins.
// The pending trees' leaves added to the margins of a CSR index's rows.
void launch_walk_csr(const DevConst& c, int K, const WNode* wtree, uint32_t wstride, float* margin,
                     const int* pending, int n_sm, cudaStream_t s);
// The feature-major copy of the CSR index c (col zeroed, colmiss all ones,
// or NULL when every cell is present).
void launch_csr_columns(const DevConst& c, uint8_t* col, uint64_t* colmiss, int n_sm, cudaStream_t s);
void launch_walk_classes(int K, const WNode* wtree, uint32_t wstride, const uint8_t* rec,
                         uint32_t stride, uint32_t mask_off, uint32_t blk, uint64_t n, float* margin,
                         const int* pending, int n_sm, cudaStream_t s);
// |g|, |h| maxima of staged pairs (HistogramBackend::prepare).
void launch_pair_maxima(const float2* gpair, uint64_t n, Scale* scale, int n_sm, cudaStream_t s);
// Fixed-point exponents from the (reduced) maxima and the global row count.
// ... and clear the pending-tree flag (`pending` may be null).
void launch_scale(Scale* scale, uint64_t global_rows, int* pending, cudaStream_t s);
// Grant the histogram kernels their shared memory (once per device, before
// any stream capture).
void hist_configure();
// Feature-major bins (+ bitmap) -> row-major records.
void launch_encode(const uint8_t* col, const uint64_t* colmiss, uint64_t n_rows, uint32_t n_cols,
                   uint32_t stride, uint32_t mask_off, uint32_t blk, uint8_t* rec, cudaStream_t s);
// Histograms of `entries` (level state `ls`) into `hist`; with `totals`
// non-null also the fixed-point (g, h) totals of the rows. A null `gpair`
// reads each row's pair from its row block (c.blk != 0).
void launch_hist(const DevConst& c, const uint32_t* fo, const uint8_t* rec, const float2* gpair,
                 const Scale* scale, const uint32_t* rows, const HEntry* entries,
                 const LevelState* ls, longlong2* hist, long long* totals,
                 unsigned long long* row_stats, int grid_x, size_t smem, cudaStream_t s);
size_t hist_smem_bytes(const DevConst& c);
int hist_grid(int n_sm);
void launch_subtract(const Triple* pairs, const LevelState* ls, int max_pairs, uint32_t total_bins,
                     longlong2* hist, cudaStream_t s);
// Split scan of every frontier node; a node whose slot is >= sib_base (with
// `pairs`) first gets its sibling histogram parent - built. `dirs`
// ([max_front][n_cols] monotone directions) overrides the run's per-feature
// constraints (c.mono) when set. With best_key, each node's winning feature
// also goes to best_key[node] (a 64-bit maximum, zero beforehand), which the
// level's apply or the lossguide step reads and clears.
void launch_scan(const DevConst& c, const uint32_t* fo, longlong2* hist, const Front* front,
                 const LevelState* ls, const Triple* pairs, int sib_base, const Scale* scale,
                 int max_front, Cand* cand, cudaStream_t s, const int8_t* dirs = nullptr,
                 unsigned long long* best_key = nullptr);
void launch_apply(const DevConst& c, const uint32_t* fo, const float* cuts, const Cand* cand,
                  const Front* front, Front* next, Decision* dec, PItem* items, LevelState* ls,
                  LevelState* ls_next, hb_tree_node* tree, WNode* wtree, const Scale* scale,
                  int depth, int leaf_only, unsigned long long* best_key, cudaStream_t s);
void launch_part_count(const DevConst& c, const uint8_t* col, const uint64_t* colmiss,
                       const uint8_t* rec, int use_record, const uint32_t* rows_in, int identity,
                       const Front* front, const Decision* dec, const PItem* items,
                       const LevelState* ls, int max_items, uint32_t* dirbits, uint32_t* item_left,
                       cudaStream_t s, uint32_t* rows_copy = nullptr);
// One-pass partition: each tile's left rows to a chunk at its node's
// segment start, right rows to one at the end, reserved on fill[2 pair],
// fill[2 pair + 1] (zero before the pass); a child's row order is not the
// stable one. Then launch_part_plan: the children's segments, the fill
// counts cleared, the next level's histogram plan. half = 0: the children
// keep the parent's positions in rows_out (depthwise growth); half = n: the
// positions n away in the other half of one 2n buffer (lossguide growth,
// rows_in == rows_out).
void launch_part_onepass(const DevConst& c, const uint8_t* col, const uint64_t* colmiss,
                         const uint32_t* rows_in, int identity, const Front* front, const Decision* dec,
                         const LevelState* ls, int max_items, uint32_t* fill, uint32_t* rows_out,
                         uint32_t half, cudaStream_t s);
void launch_part_plan(const Front* front, const Decision* dec, const LevelState* ls, uint32_t* fill,
                      Front* next, HEntry* entries, Triple* pairs, LevelState* ls_next, int max_front,
                      uint32_t half, cudaStream_t s);
// Per-node scan of the tiles' left counts and the children's segments; with
// `entries` (device growth) the last CTA also plans the next level's
// histograms (built child = smaller Hessian; entries, sibling pairs, ls_next).
// `ls->done_ctas` must be zero.
void launch_part_scan(const Front* front, const Decision* dec, LevelState* ls, int max_front,
                      const uint32_t* item_left, uint32_t* item_left_off, Front* next,
                      HEntry* entries, Triple* pairs, LevelState* ls_next, cudaStream_t s);
void launch_part_scatter(const Front* front, const Decision* dec, const PItem* items,
                         const LevelState* ls, int max_items, const uint32_t* dirbits,
                         const uint32_t* item_left_off, const Front* next,
                         const uint32_t* rows_in, int identity, uint32_t* rows_out,
                         cudaStream_t s);
// Lossguide growth: one step (merge + push the pending nodes, pop until one
// expands), a new tree's state, and the copy-back of a partitioned segment.
void launch_lg_step(const DevConst& c, const uint32_t* fo, const float* cuts, const Cand* cand,
                    const Front* pend, Front* front, Front* next, Decision* dec, LevelState* ls,
                    LevelState* ls_next, hb_tree_node* tree, WNode* wtree, const Scale* scale,
                    LgKey* heap, LgNode* pool, int heap_cap, LgState* st, int32_t* ndepth,
                    int max_leaves, int depth_limit, int final_step, unsigned long long* best_key,
                    cudaStream_t s);
void launch_lg_setup(LgState* st, int32_t* ndepth, hb_tree_node* tree, const Front* root,
                     const Scale* scale, LevelState* ls_next, cudaStream_t s);
void launch_root_setup(uint64_t n_rows, Front* front, HEntry* entries, LevelState* ls,
                       cudaStream_t s);
void launch_root_stats(Front* front, const long long* totals, cudaStream_t s);
void launch_finish_tree(const hb_tree_node* tree, const LevelState* ls_last, hb_tree_node* forest,
                        uint32_t* counts, int32_t* tree_counter, uint32_t max_nodes,
                        cudaStream_t s);
void launch_dequantize(const longlong2* hist, uint32_t n, const Scale* scale, double* out,
                       cudaStream_t s);
// RowEngine helpers: an iota row list; leaf values added to every segment
// at once; a partition's copy-back with the children's end rows; the
// fixed-point totals of a segment.
// p[0, n) = v.
void launch_fill(float* p, float v, uint64_t n, int n_sm, cudaStream_t s);
void launch_iota(uint32_t* rows, uint32_t first, uint64_t n, int n_sm, cudaStream_t s);
// Each tile (first row position, length <= kAddTile, leaf value bits) adds
// its value to the margins of its rows, a CTA per tile.
constexpr uint32_t kAddTile = 8192;
void launch_add_segments(const uint32_t* rows, const uint4* tiles, uint32_t n_tiles, float* margin,
                         cudaStream_t s);
void launch_finish_partition(const PItem* items, int n_items, const Front* parents, const Front* kids,
                             const uint32_t* rows_out, uint32_t* rows_in, uint32_t* ends, cudaStream_t s);
void launch_seg_total(const uint32_t* rows, uint64_t begin, uint64_t len, const float2* gpair,
                      const Scale* scale, long long* totals, int n_sm, cudaStream_t s);
void launch_add_segment(const uint32_t* rows, uint32_t begin, uint32_t len, float value,
                        float* margin, cudaStream_t s);

// Sum of the histogram words [first, first + count) (longlong2 units) over
// the ranks of `ps`, left in every rank's buffer (hb_peer.cu).
void launch_peer_allreduce(const PeerSet& ps, uint64_t first, uint64_t count, int n_sm, cudaStream_t s);
// One CTA waiting, bounded by ps.timeout_ns, on a flag nothing raises.
void launch_peer_wait_probe(const PeerSet& ps, cudaStream_t s);

}  // namespace hb
