// The engine behind the C ABI: one GPU, one shard of rows, the binned
// matrix resident in HBM, and the per-round pipeline of kernels that grows a
// tree without returning to the host between levels.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "hb_engine_view.h"
#include "hb_internal.h"
#include "hb_kernels.cuh"
#include "hb_sketch.h"

using namespace hb;

// The C ABI's struct layouts (the Python bindings check the same sizes).
static_assert(sizeof(hb_ghist) == 64, "hb_ghist layout");
static_assert(sizeof(hb_tree_node) == 40, "hb_tree_node layout");

namespace {

template <class T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  cudaError_t alloc(size_t count) {
    if (count <= n && p) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    if (count == 0) return cudaSuccess;
    cudaError_t e = cudaMalloc(&p, count * sizeof(T));
    if (e == cudaSuccess) n = count;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
};

constexpr int kTimers = 8;  // gradients, root hist, scan, apply, partition, hist, subtract, other
enum Timer { T_GRAD, T_ROOT, T_SCAN, T_APPLY, T_PART, T_HIST, T_SUB, T_OTHER };

}  // namespace

struct hb_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  int n_sm = 148;
  bool failed = false;
  std::string err;

  // the binned matrix
  bool uploaded = false;
  DevConst c{};
  std::vector<uint32_t> h_fo;
  std::vector<float> h_cuts;
  DevBuf<uint8_t> rec, col;
  DevBuf<uint64_t> colmiss;
  DevBuf<uint64_t> csr_ptr;  // CSR index: row offsets and global bins
  DevBuf<uint32_t> csr_bins;
  bool has_missing = false;
  DevBuf<uint32_t> fo;
  DevBuf<float> cuts;

  // rows
  DevBuf<float2> gpair;

  DevBuf<float> margin, label, weight;
  const float* label_key = nullptr;
  const float* weight_key = nullptr;
  bool margins_loaded = false;
  // Row ids: one allocation of 2n, rows[0] its first half and rows[1] its
  // second (depthwise growth ping-pongs between them; lossguide's one-pass
  // partition moves a node's rows to the other half, its positions read
  // from rows[0] over the whole 2n)
  DevBuf<uint32_t> rows_all;
  uint32_t* rows[2] = {nullptr, nullptr};
  DevBuf<Scale> scale;
  bool staged = false;

  // tree growth
  int alloc_depth = -1;
  DevBuf<longlong2> hist_all;  // [1 totals][slots][total_bins]
  DevBuf<Front> front[2];
  DevBuf<Cand> cand;
  DevBuf<Decision> dec;
  DevBuf<PItem> items;
  DevBuf<uint32_t> dirbits, item_left, item_off;
  // depthwise one-pass partition: per split, the rows placed so far in its
  // left and right child (zero between levels)
  DevBuf<uint32_t> fill;
  // each frontier node's best feature from the scan (a 64-bit maximum),
  // read and cleared by the apply / lossguide step: zero between uses
  DevBuf<unsigned long long> best_key;
  // HB_STABLE_PARTITION=1: the three-pass stable partition in depthwise
  // growth too (children keep ascending row order)
  bool stable_partition = false;
  DevBuf<HEntry> entries;
  DevBuf<Triple> pairs;
  DevBuf<LevelState> ls;
  DevBuf<hb_tree_node> tree;
  DevBuf<WNode> wtree;
  // lossguide growth: the heap of waiting nodes, its state, node depths
  DevBuf<LgKey> lg_heap;
  DevBuf<LgNode> lg_pool;  // lossguide: each heap node's data at its node id
  DevBuf<LgState> lg_state;
  DevBuf<int32_t> lg_depth;
  bool pending_tree = false;  // host mirror of flags[0]: a grown tree's leaves await the margins
  int walk_ls = 1;            // the pending tree: e->ls index holding its node count
  int walk_nodes = 2;         // and the capacity of its WNode array
  int walk_depth = 0;         // and its depth bound (depthwise growth; 0: none)
  DevBuf<int> flags;          // [0]: pending tree (read by the next gradient or walk kernel)
  // the captured round (CUDA graph) and what it was captured for
  cudaGraphExec_t round_exec = nullptr;
  std::vector<unsigned char> round_key;
  uint64_t round_launches = 0;
  bool use_graphs = true;
  cudaEvent_t run_ev[2] = {nullptr, nullptr};  // around the last train_rounds' rounds
  double last_rounds_ms = 0.0;
  int max_items = 0;
  DevBuf<hb_tree_node> forest;
  DevBuf<uint32_t> counts;
  DevBuf<int32_t> tree_counter;

  // RowEngine per-call state
  uint64_t tree_stamp = 0;
  DevBuf<uint32_t> call_rows;
  DevBuf<longlong2> call_hist;
  DevBuf<double> call_out;
  DevBuf<longlong2> resident;
  uint32_t resident_slots = 0;
  DevBuf<long long> seg_total;

  // sharding
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0;
  // HB_PEER_ALLREDUCE=1: level histograms summed over peer memory
  // (hb_peer.cu) instead of by NCCL's allreduce, every rank's hist_all and
  // barrier block mapped here by CUDA IPC. NCCL is the default: at 2 GPUs it
  // measured 861-865 rounds/s against 823-829 for the peer kernel.
  bool peer_mode = false;
  bool peer_ready = false;
  const void* peer_for = nullptr;     // the hist_all the mapping was made for
  DevBuf<unsigned long long> pbar;    // this rank's barrier block
  std::vector<void*> peer_opened;     // IPC mappings to close
  PeerSet ps{};
  uint64_t row_begin = 0;
  uint64_t shard_global = 0;  // rows of the whole matrix when this engine holds a shard (0: not sharded)

  // timing and counters (hb_engine_get_stats)
  bool timing = false;
  uint32_t timing_mask = 0;  // kernel families bracketed by events
  bool mark_open = false;
  std::vector<cudaEvent_t> ev;
  std::vector<int> ev_kind;
  size_t ev_used = 0;
  double timer_ms[kTimers] = {0};
  uint64_t timer_launches[kTimers] = {0};
  uint64_t kernel_launches = 0;
  uint64_t rounds_done = 0;
  DevBuf<unsigned long long> row_stats;  // [contiguous rows built, gathered rows built]
  bool train_begun = false;
  // multi:softmax runs: classes, and the class whose tree is being grown
  // (its slices of gpair, scale and wtree are the ones the level kernels use)
  int n_out = 1;
  int cls = 0;
  size_t wstride = 0;      // WNodes per class in wtree
  int lg_alloc = 0;     // leaves the lossguide buffers hold (0: none)
  int alloc_classes = 0;
  // monotone constraints of the training run (one direction per feature)
  // and the per-(node, feature) directions of a RowEngine scan
  DevBuf<int8_t> mono, scan_dirs;
  std::vector<int8_t> h_mono;
  // RowEngine call buffers: leaf segments and values, partition end rows
  DevBuf<uint4> seg_tiles;  // hb_add_leaf_values' row tiles
  DevBuf<uint32_t> part_ends;
  // fault injection (hb_engine_inject_fault): checked calls left before the
  // one that fails (-1: none armed); no injection while a graph is captured
  int64_t fault_after = -1;
  bool capturing = false;
  // the row blocks hold this tree's pairs (the last gradient pass wrote
  // them): the histogram launches of the growth paths read them there
  bool blk_pairs = false;
};

namespace {
inline float2* cur_gpair(hb_engine* e) { return e->gpair.p + (size_t)e->cls * e->c.n_rows; }
// The pairs the growth paths' histogram launches read: null = the row blocks.
inline const float2* hist_gpair(hb_engine* e) { return e->blk_pairs ? nullptr : cur_gpair(e); }

inline Scale* cur_scale(hb_engine* e) { return e->scale.p + e->cls; }
inline WNode* cur_wtree(hb_engine* e) { return e->wtree.p + (size_t)e->cls * e->wstride; }
}  // namespace

namespace {

thread_local std::string g_last_error;

hb_status fail(hb_engine* e, const char* what, cudaError_t code) {
  e->failed = true;
  e->err = std::string(what) + ": " + cudaGetErrorString(code);
  g_last_error = e->err;
  return HB_DEVICE_FAILED;
}

hb_status refuse(hb_engine* e, const std::string& why) {
  e->err = why;
  g_last_error = why;
  return HB_REFUSED;
}

// A checked CUDA call. With a fault armed (hb_engine_inject_fault) the
// engine's n-th checked call outside stream capture fails before it runs,
// as a device error: the call itself never reaches CUDA.
#define HB_CK(e, call)                                                          \
  do {                                                                          \
    if ((e)->fault_after >= 0 && !(e)->capturing && (e)->fault_after-- == 0)    \
      return fail(e, "injected fault before " #call, cudaErrorMemoryAllocation); \
    cudaError_t _c = (call);                                                    \
    if (_c != cudaSuccess) return fail(e, #call, _c);                           \
  } while (0)

#define HB_NCCL(e, call)                                              \
  do {                                                                \
    ncclResult_t _r = (call);                                         \
    if (_r != ncclSuccess) {                                          \
      (e)->failed = true;                                             \
      (e)->err = std::string(#call) + ": " + ncclGetErrorString(_r);  \
      g_last_error = (e)->err;                                        \
      return HB_DEVICE_FAILED;                                        \
    }                                                                 \
  } while (0)

#define HB_ENTER(e)                                                   \
  do {                                                                \
    if (!(e)) return HB_INVALID_ARGUMENT;                             \
    if ((e)->failed) return HB_REFUSED;                               \
    cudaError_t _d = cudaSetDevice((e)->device);                      \
    if (_d != cudaSuccess) return fail((e), "cudaSetDevice", _d);     \
  } while (0)

// Timing marks (CUDA events on the engine's stream), enabled per train call.
// Under stream capture a mark must become an event-record node of the graph
// (cudaEventRecordExternal); a plain record would only order the capture.
void record_mark(hb_engine* e, cudaEvent_t ev) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(e->stream, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, e->stream, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, e->stream);
}

void mark_begin(hb_engine* e, int kind) {
  e->mark_open = false;
  if (!e->timing || !(e->timing_mask & (1u << kind))) return;
  e->mark_open = true;
  if (e->ev_used + 2 > e->ev.size()) {
    for (int i = 0; i < 256; ++i) {
      cudaEvent_t x;
      cudaEventCreate(&x);
      e->ev.push_back(x);
      e->ev_kind.push_back(0);
    }
  }
  e->ev_kind[e->ev_used] = kind;
  record_mark(e, e->ev[e->ev_used++]);
}
void mark_end(hb_engine* e) {
  if (!e->timing || !e->mark_open) return;
  e->mark_open = false;
  e->ev_kind[e->ev_used] = -1;
  record_mark(e, e->ev[e->ev_used++]);
}
void collect_timers(hb_engine* e) {
  if (!e->timing || e->ev_used == 0) return;
  cudaStreamSynchronize(e->stream);
  for (size_t i = 0; i + 1 < e->ev_used; i += 2) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, e->ev[i], e->ev[i + 1]) == cudaSuccess) {
      e->timer_ms[e->ev_kind[i]] += ms;
      e->timer_launches[e->ev_kind[i]] += 1;
    }
  }
  e->ev_used = 0;
}

hb_status ensure_growth_buffers(hb_engine* e, int max_depth) {
  if (e->alloc_depth >= max_depth && e->alloc_classes >= e->n_out) return HB_OK;
  const DevConst& c = e->c;
  const int max_front = 1 << max_depth;
  const size_t slots = (size_t(1) << max_depth) - 1;
  HB_CK(e, e->hist_all.alloc(1 + slots * c.total_bins));
  HB_CK(e, e->front[0].alloc(max_front));
  HB_CK(e, e->front[1].alloc(max_front));
  HB_CK(e, e->cand.alloc((size_t)max_front * c.n_cols));
  HB_CK(e, e->dec.alloc(max_front));
  e->max_items = (int)((c.n_rows + kTile - 1) / kTile) + max_front + 1;
  HB_CK(e, e->items.alloc(e->max_items));
  HB_CK(e, e->dirbits.alloc((size_t)e->max_items * kTileWords));
  HB_CK(e, e->item_left.alloc(e->max_items));
  HB_CK(e, e->item_off.alloc(e->max_items));
  HB_CK(e, e->fill.alloc((size_t)2 * max_front));
  HB_CK(e, cudaMemset(e->fill.p, 0, sizeof(uint32_t) * 2 * max_front));
  HB_CK(e, e->best_key.alloc(max_front));
  HB_CK(e, cudaMemset(e->best_key.p, 0, sizeof(unsigned long long) * max_front));
  HB_CK(e, e->entries.alloc(max_front));
  HB_CK(e, e->pairs.alloc(max_front));
  HB_CK(e, e->ls.alloc(kMaxDepth + 2));
  HB_CK(e, e->tree.alloc((size_t)2 * max_front));
  e->wstride = (size_t)2 * max_front;
  HB_CK(e, e->wtree.alloc(e->wstride * std::max(e->n_out, 1)));
  e->alloc_depth = max_depth;
  e->alloc_classes = e->n_out;
  e->lg_alloc = 0;
  return HB_OK;
}

void close_peers(hb_engine* e) {
  for (void* p : e->peer_opened) cudaIpcCloseMemHandle(p);
  e->peer_opened.clear();
  e->peer_ready = false;
  e->peer_for = nullptr;
}

// Map every rank's hist_all and barrier block for the peer allreduce (a
// collective: every rank of the communicator calls it at the same point,
// before any round is captured). Re-mapped when this engine's hist_all has
// moved; a failure to map leaves the NCCL allreduce in use.
hb_status ensure_peers(hb_engine* e) {
  if (!e->comm || !e->peer_mode || e->nranks < 2 || e->nranks > kPeerMax) return HB_OK;
  // every rank remaps when any rank's buffer moved (one max-allreduce)
  DevBuf<int> flag;
  HB_CK(e, flag.alloc(1));
  const int moved = (!e->peer_ready || e->peer_for != (const void*)e->hist_all.p) ? 1 : 0;
  HB_CK(e, cudaMemcpyAsync(flag.p, &moved, 4, cudaMemcpyHostToDevice, e->stream));
  HB_NCCL(e, ncclAllReduce(flag.p, flag.p, 1, ncclInt32, ncclMax, e->comm, e->stream));
  int any = 0;
  HB_CK(e, cudaMemcpyAsync(&any, flag.p, 4, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  if (!any) return HB_OK;
  close_peers(e);
  if (e->round_exec) cudaGraphExecDestroy(e->round_exec);  // captured with the old peers
  e->round_exec = nullptr;
  HB_CK(e, e->pbar.alloc(kPeerWords));
  HB_CK(e, cudaMemset(e->pbar.p, 0, sizeof(unsigned long long) * kPeerWords));
  // this rank's two IPC handles, gathered from every rank
  const int n = e->nranks;
  std::vector<unsigned char> mine(2 * sizeof(cudaIpcMemHandle_t)), all(n * mine.size());
  cudaIpcMemHandle_t h0, h1;
  cudaError_t ie = cudaIpcGetMemHandle(&h0, e->hist_all.p);
  if (ie == cudaSuccess) ie = cudaIpcGetMemHandle(&h1, e->pbar.p);
  int ok = ie == cudaSuccess ? 1 : 0;
  if (!ok) cudaGetLastError();
  std::memcpy(mine.data(), &h0, sizeof(h0));
  std::memcpy(mine.data() + sizeof(h0), &h1, sizeof(h1));
  DevBuf<unsigned char> xb;
  HB_CK(e, xb.alloc(all.size()));
  HB_CK(e, cudaMemcpyAsync(xb.p + (size_t)e->rank * mine.size(), mine.data(), mine.size(),
                           cudaMemcpyHostToDevice, e->stream));
  HB_NCCL(e, ncclAllGather(xb.p + (size_t)e->rank * mine.size(), xb.p, mine.size(), ncclUint8, e->comm,
                           e->stream));
  HB_CK(e, cudaMemcpyAsync(all.data(), xb.p, all.size(), cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  PeerSet ps{};
  ps.n = n;
  ps.rank = e->rank;
  const char* to = std::getenv("HB_PEER_TIMEOUT_MS");
  ps.timeout_ns = (uint64_t)(to ? std::max(1, std::atoi(to)) : 5000) * 1000000ull;
  for (int j = 0; j < n && ok; ++j) {
    if (j == e->rank) {
      ps.hist[j] = e->hist_all.p;
      ps.bar[j] = e->pbar.p;
      continue;
    }
    cudaIpcMemHandle_t a, b;
    std::memcpy(&a, all.data() + (size_t)j * mine.size(), sizeof(a));
    std::memcpy(&b, all.data() + (size_t)j * mine.size() + sizeof(a), sizeof(b));
    void* pa = nullptr;
    void* pb = nullptr;
    if (cudaIpcOpenMemHandle(&pa, a, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
        cudaIpcOpenMemHandle(&pb, b, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      if (pa) cudaIpcCloseMemHandle(pa);
      ok = 0;
      break;
    }
    e->peer_opened.push_back(pa);
    e->peer_opened.push_back(pb);
    ps.hist[j] = reinterpret_cast<longlong2*>(pa);
    ps.bar[j] = reinterpret_cast<unsigned long long*>(pb);
  }
  // every rank takes the peer path only if every rank mapped every peer
  HB_CK(e, cudaMemcpyAsync(flag.p, &ok, 4, cudaMemcpyHostToDevice, e->stream));
  HB_NCCL(e, ncclAllReduce(flag.p, flag.p, 1, ncclInt32, ncclMin, e->comm, e->stream));
  int all_ok = 0;
  HB_CK(e, cudaMemcpyAsync(&all_ok, flag.p, 4, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  if (!all_ok) {
    close_peers(e);
    e->peer_mode = false;  // NCCL from now on
    return HB_OK;
  }
  e->ps = ps;
  e->peer_ready = true;
  e->peer_for = e->hist_all.p;
  return HB_OK;
}

// The sum over ranks of hist_all's longlong2 words [first, first + count).
hb_status allreduce_hist(hb_engine* e, uint64_t first, uint64_t count) {
  if (e->peer_ready && e->peer_for == (const void*)e->hist_all.p) {
    launch_peer_allreduce(e->ps, first, count, e->n_sm, e->stream);
    e->kernel_launches += 1;
    HB_CK(e, cudaGetLastError());
    return HB_OK;
  }
  HB_NCCL(e, ncclAllReduce(e->hist_all.p + first, e->hist_all.p + first, 2 * count, ncclInt64, ncclSum, e->comm,
                           e->stream));
  return HB_OK;
}

// A peer wait that timed out fails the engine (read after a synchronize).
hb_status check_peers(hb_engine* e) {
  if (!e->peer_ready) return HB_OK;
  unsigned long long st = 0;
  HB_CK(e, cudaMemcpy(&st, e->pbar.p + kPeerStatus, sizeof(st), cudaMemcpyDeviceToHost));
  if (st) return fail(e, "peer histogram exchange: a rank did not arrive in time", cudaErrorTimeout);
  return HB_OK;
}

// Stage this tree's scale: reduce the maxima over ranks, then the exponents.
hb_status finish_scale(hb_engine* e) {
  if (e->comm) {
    HB_NCCL(e, ncclAllReduce(&cur_scale(e)->maxg_bits, &cur_scale(e)->maxg_bits, 3, ncclUint32,
                             ncclMax, e->comm, e->stream));
  }
  launch_scale(cur_scale(e), e->c.global_rows, e->flags.p, e->stream);
  HB_CK(e, cudaGetLastError());
  return HB_OK;
}

uint64_t vector_rows(hb_engine* e) {
  const uint64_t g = e->c.global_rows;
  const uint64_t vg = g >= 16 ? g - g % 8 : 0;
  if (vg <= e->row_begin) return 0;
  return std::min<uint64_t>(vg - e->row_begin, e->c.n_rows);
}

// This shard's rows that x86_64's short-row softmax kernel (2 or 4 classes)
// takes in vectors of 8 / k whole rows: the matrix's first g - g % (8 / k)
// rows when it holds at least 16 margins (simd/mod.rs:28, :156).
static uint64_t softmax_vector_rows(hb_engine* e, int k) {
  if (k != 2 && k != 4) return 0;
  const uint64_t g = e->c.global_rows, rows = 8 / (uint64_t)k;
  const uint64_t vg = g * (uint64_t)k >= 16 ? g - g % rows : 0;
  if (vg <= e->row_begin) return 0;
  return std::min<uint64_t>(vg - e->row_begin, e->c.n_rows);
}

// Add the last grown tree's leaves to the margins now (the next round's
// gradient kernel does it otherwise).
hb_status flush_pending(hb_engine* e) {
  if (!e->pending_tree) return HB_OK;
  mark_begin(e, T_OTHER);
  if (e->c.csr)
    launch_walk_csr(e->c, e->n_out, e->wtree.p, (uint32_t)e->wstride, e->margin.p, e->flags.p, e->n_sm,
                    e->stream);
  else if (e->n_out > 1)
    launch_walk_classes(e->n_out, e->wtree.p, (uint32_t)e->wstride, e->rec.p, e->c.stride,
                        e->c.mask_off, e->c.blk, e->c.n_rows, e->margin.p, e->flags.p, e->n_sm, e->stream);
  else
    launch_walk(e->wtree.p, e->ls.p + e->walk_ls, e->walk_nodes, e->rec.p, e->c.stride,
                e->c.mask_off, e->c.blk, e->c.n_rows, e->margin.p, e->flags.p, e->n_sm, e->stream);
  mark_end(e);
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0, sizeof(int), e->stream));
  e->kernel_launches += 1;
  e->pending_tree = false;
  HB_CK(e, cudaGetLastError());
  return HB_OK;
}

// Gradients at the margins, first adding a pending tree's leaves when the
// device flag says one waits (so a captured round serves every round).
hb_status run_gradients(hb_engine* e, int kind, float spw, float min_hess, int walk_ls,
                        int walk_nodes, int walk_depth) {
  HB_CK(e, cudaMemsetAsync(e->scale.p, 0, sizeof(Scale), e->stream));
  mark_begin(e, T_GRAD);
  if (walk_ls < 0) {
    walk_ls = e->walk_ls;
    walk_nodes = e->walk_nodes;
    walk_depth = e->walk_depth;
  }
  const bool csr = e->c.csr != 0;
  if (csr) {  // the pending tree's walk over CSR rows first
    launch_walk_csr(e->c, 1, e->wtree.p, (uint32_t)e->wstride, e->margin.p, e->flags.p, e->n_sm,
                    e->stream);
    e->kernel_launches += 1;
  }
  // single-output dense growth reads its pairs from the row blocks
  const uint32_t blk_pair = (!csr && e->n_out == 1 && e->c.blk) ? e->c.blk_pair : 0u;
  launch_gradients(kind, e->margin.p, e->label.p, e->weight_key ? e->weight.p : nullptr, spw,
                   min_hess, e->c.n_rows, vector_rows(e), e->gpair.p, e->scale.p,
                   csr ? nullptr : e->wtree.p, e->ls.p + walk_ls, walk_nodes, walk_depth, e->rec.p, e->c.stride,
                   e->c.mask_off, e->c.blk, blk_pair, e->flags.p, e->n_sm, e->stream);
  e->blk_pairs = blk_pair != 0;
  mark_end(e);
  e->pending_tree = false;
  e->kernel_launches += 2;  // gradients (+ last tree's leaves) + scale
  HB_CK(e, cudaGetLastError());
  hb_status st = finish_scale(e);
  if (st != HB_OK) return st;
  e->staged = true;
  return HB_OK;
}

// Leaves a lossguide tree may reach: max_leaves, else 2^max_depth.
int lg_leaves(const hb_train_params* p) {
  return p->max_leaves > 0 ? p->max_leaves : (1 << std::min(p->max_depth, 20));
}

// Where a grown tree's node count lives (an e->ls index) and how many nodes
// its WNode array can hold: what the next pass's tree walk needs.
void walk_shape(const hb_train_params* p, int& ls_index, int& nodes, int& depth) {
  if (p->grow_policy == HB_GROW_LOSSGUIDE) {
    ls_index = 2;
    nodes = 2 * lg_leaves(p);
    depth = 0;
  } else {
    ls_index = p->max_depth + 1;
    nodes = 2 << p->max_depth;
    depth = p->max_depth;
  }
}

// Node capacity of one tree in the forest buffer.
uint32_t tree_slots(const hb_train_params* p) {
  return p->grow_policy == HB_GROW_LOSSGUIDE ? 2u * (uint32_t)lg_leaves(p) : 2u << p->max_depth;
}

// Grow one tree on the device from the staged gradients (depthwise). Writes
// the tree to e->tree and appends it to the forest buffer when `forest`.
hb_status grow_device(hb_engine* e, const hb_train_params* p, bool to_forest) {
  DevConst& c = e->c;
  const int D = p->max_depth;
  hb_status st = ensure_growth_buffers(e, D);
  if (st != HB_OK) return st;
  c.lambda = (double)p->lambda;
  c.alpha = (double)p->alpha;
  c.gamma = (double)p->gamma;
  c.mcw = (double)p->min_child_weight;
  c.mds = (double)p->max_delta_step;
  c.eta = p->eta;
  c.max_depth = D;
  cudaStream_t s = e->stream;
  const size_t slots = (size_t(1) << D) - 1;
  longlong2* hist = e->hist_all.p + 1;
  long long* totals = reinterpret_cast<long long*>(e->hist_all.p);

  HB_CK(e, cudaMemsetAsync(e->ls.p, 0, sizeof(LevelState) * (kMaxDepth + 2), s));
  HB_CK(e, cudaMemsetAsync(e->hist_all.p, 0, sizeof(longlong2) * (1 + slots * c.total_bins), s));
  HB_CK(e, cudaMemsetAsync(e->fill.p, 0, sizeof(uint32_t) * 2 * ((size_t)1 << D), s));
  launch_root_setup(c.n_rows, e->front[0].p, e->entries.p, e->ls.p, s);
  const size_t smem = hist_smem_bytes(c);
  const int hgrid = hist_grid(e->n_sm);
  mark_begin(e, T_ROOT);
  launch_hist(c, e->fo.p, e->rec.p, hist_gpair(e), cur_scale(e), nullptr, e->entries.p, e->ls.p, hist,
              totals, e->row_stats.p, hgrid, smem, s);
  mark_end(e);
  HB_CK(e, cudaGetLastError());
  if (e->comm) {
    hb_status ast = allreduce_hist(e, 0, 1 + (uint64_t)c.total_bins);
    if (ast != HB_OK) return ast;
  }
  launch_root_stats(e->front[0].p, totals, s);

  int cur = 0;
  uint32_t* rows_in = e->rows[0];
  uint32_t* rows_out = e->rows[1];
  uint64_t launches = 3;
  for (int d = 0; d <= D; ++d) {
    const bool leaf_only = d == D;
    const int max_front = 1 << d;
    LevelState* lsd = e->ls.p + d;
    LevelState* lsn = e->ls.p + d + 1;
    Front* fr = e->front[cur].p;
    Front* nx = e->front[cur ^ 1].p;
    if (!leaf_only) {
      mark_begin(e, T_SCAN);
      // level d's sibling slots start at base + half; their histograms are
      // parent - built, made by the scan itself
      const int sib_base = d == 0 ? INT_MAX : (1 << d) - 1 + (1 << (d - 1));
      launch_scan(c, e->fo.p, hist, fr, lsd, d == 0 ? nullptr : e->pairs.p, sib_base, cur_scale(e),
                  max_front, e->cand.p, s, nullptr, e->best_key.p);
      mark_end(e);
      ++launches;
    }
    mark_begin(e, T_APPLY);
    launch_apply(c, e->fo.p, e->cuts.p, e->cand.p, fr, nx, e->dec.p, e->items.p, lsd, lsn,
                 e->tree.p, cur_wtree(e), cur_scale(e), d, leaf_only ? 1 : 0, e->best_key.p, s);
    mark_end(e);
    ++launches;
    HB_CK(e, cudaGetLastError());
    // Children at the depth limit need no rows: their leaves reach the
    // margins through the tree walk of the next gradient pass.
    if (d + 2 > D) {
      cur ^= 1;
      continue;
    }
    const int max_items = std::min(e->max_items, (int)((c.n_rows + kTile - 1) / kTile) + max_front);
    mark_begin(e, T_PART);
    // feature columns, not row records: a level's gathers of one feature's
    // column and bitmap stay in L2, records do not
    if (e->stable_partition) {
      launch_part_count(c, e->col.p, e->colmiss.p, e->rec.p, 0,
                        rows_in, d == 0, fr, e->dec.p, e->items.p, lsd, max_items, e->dirbits.p,
                        e->item_left.p, s);
      launch_part_scan(fr, e->dec.p, lsd, max_front, e->item_left.p, e->item_off.p, nx,
                       e->entries.p, e->pairs.p, lsn, s);
      launch_part_scatter(fr, e->dec.p, e->items.p, lsd, max_items, e->dirbits.p, e->item_off.p,
                          nx, rows_in, d == 0, rows_out, s);
      ++launches;
    } else {
      launch_part_onepass(c, e->col.p, e->colmiss.p, rows_in, d == 0, fr,
                          e->dec.p, lsd, max_items, e->fill.p, rows_out, 0u, s);
      launch_part_plan(fr, e->dec.p, lsd, e->fill.p, nx, e->entries.p, e->pairs.p, lsn, max_front, 0u, s);
    }
    mark_end(e);
    mark_begin(e, T_HIST);
    launch_hist(c, e->fo.p, e->rec.p, hist_gpair(e), cur_scale(e), rows_out, e->entries.p, lsn, hist,
                nullptr, e->row_stats.p, hgrid, smem, s);
    mark_end(e);
    if (e->comm) {
      const uint64_t base = (uint64_t(1) << (d + 1)) - 1, half = uint64_t(1) << d;
      hb_status ast = allreduce_hist(e, 1 + base * c.total_bins, half * c.total_bins);
      if (ast != HB_OK) return ast;
    }
    launches += 3;  // partition (+ 1 for the stable one) and histogram
    HB_CK(e, cudaGetLastError());
    std::swap(rows_in, rows_out);
    cur ^= 1;
  }
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0x01, sizeof(int), s));
  e->pending_tree = true;
  e->walk_ls = D + 1;
  e->walk_nodes = 2 << D;
  e->walk_depth = D;
  if (to_forest) {
    launch_finish_tree(e->tree.p, e->ls.p + D + 1, e->forest.p, e->counts.p, e->tree_counter.p,
                       (uint32_t)(2u << D), s);
    HB_CK(e, cudaGetLastError());
  }
  // root setup + root hist + root stats, per level scan + apply (+ 3
  // partition passes, the last also planning, and hist above the last two
  // levels), the forest copy
  e->kernel_launches += launches + (to_forest ? 1 : 0);
  e->rounds_done += 1;
  return HB_OK;
}

// Buffers of lossguide growth with at most L leaves (2L nodes, one
// histogram slot per node, a frontier of one node and its two children).
hb_status ensure_lossguide_buffers(hb_engine* e, int L) {
  if (e->lg_alloc >= L && e->alloc_depth < 0) return HB_OK;
  const DevConst& c = e->c;
  const int n_nodes = 2 * L;
  HB_CK(e, e->hist_all.alloc(1 + (size_t)n_nodes * c.total_bins));
  HB_CK(e, e->front[0].alloc(2));
  HB_CK(e, e->front[1].alloc(2));
  HB_CK(e, e->cand.alloc((size_t)2 * c.n_cols));
  HB_CK(e, e->dec.alloc(2));
  e->max_items = std::max(e->max_items, (int)((c.n_rows + kTile - 1) / kTile) + 2);
  HB_CK(e, e->items.alloc(e->max_items));
  HB_CK(e, e->dirbits.alloc((size_t)e->max_items * kTileWords));
  HB_CK(e, e->item_left.alloc(e->max_items));
  HB_CK(e, e->item_off.alloc(e->max_items));
  HB_CK(e, e->entries.alloc(2));
  HB_CK(e, e->pairs.alloc(2));
  HB_CK(e, e->ls.alloc(kMaxDepth + 2));
  HB_CK(e, e->tree.alloc(n_nodes));
  HB_CK(e, e->wtree.alloc(n_nodes));
  HB_CK(e, e->lg_heap.alloc((size_t)L + 2));
  HB_CK(e, e->lg_pool.alloc((size_t)n_nodes));
  HB_CK(e, e->lg_state.alloc(1));
  HB_CK(e, e->lg_depth.alloc(n_nodes));
  HB_CK(e, e->fill.alloc(2));
  HB_CK(e, e->best_key.alloc(2));
  HB_CK(e, cudaMemset(e->best_key.p, 0, 2 * sizeof(unsigned long long)));
  e->wstride = (size_t)n_nodes;
  e->alloc_depth = -1;  // the depthwise sizes no longer hold
  e->lg_alloc = L;
  return HB_OK;
}

// The growth buffers the parameters need, allocated before any capture.
hb_status ensure_buffers(hb_engine* e, const hb_train_params* p) {
  return p->grow_policy == HB_GROW_LOSSGUIDE ? ensure_lossguide_buffers(e, lg_leaves(p))
                                             : ensure_growth_buffers(e, p->max_depth);
}

// Grow one tree with lossguide growth (hist/mod.rs:505) entirely on the
// device: the root's histogram and scan, then max_leaves - 1 steps, each a
// heap step (k_lg_step) and, when it expanded a node, that node's partition,
// the smaller-Hessian child's histogram and both children's scans (the
// sibling made as parent - built by the scan). Histogram slot = node id, so
// no slot is reused within a tree. A node's rows sit in either half of the
// 2n row buffer: the one-pass partition moves its children to the other
// half (the stable one, HB_STABLE_PARTITION=1, scatters into rows[1] and
// copies the segment back, so every node stays in rows[0]).
hb_status grow_lossguide(hb_engine* e, const hb_train_params* p, bool to_forest) {
  DevConst& c = e->c;
  const int L = lg_leaves(p);
  const int n_nodes = 2 * L;
  c.lambda = (double)p->lambda;
  c.alpha = (double)p->alpha;
  c.gamma = (double)p->gamma;
  c.mcw = (double)p->min_child_weight;
  c.mds = (double)p->max_delta_step;
  c.eta = p->eta;
  c.max_depth = p->max_depth;
  hb_status st = ensure_lossguide_buffers(e, L);
  if (st != HB_OK) return st;
  cudaStream_t s = e->stream;
  longlong2* hist = e->hist_all.p + 1;
  long long* totals = reinterpret_cast<long long*>(e->hist_all.p);
  LevelState* ls0 = e->ls.p;      // the root
  LevelState* ls1 = e->ls.p + 1;  // the step's expanded node
  LevelState* ls2 = e->ls.p + 2;  // its children; the tree's node count
  HB_CK(e, cudaMemsetAsync(e->ls.p, 0, sizeof(LevelState) * 3, s));
  HB_CK(e, cudaMemsetAsync(e->hist_all.p, 0, sizeof(longlong2) * (1 + (size_t)n_nodes * c.total_bins), s));
  Front* fr = e->front[0].p;
  Front* nx = e->front[1].p;
  launch_root_setup(c.n_rows, fr, e->entries.p, ls0, s);
  const size_t smem = hist_smem_bytes(c);
  const int hgrid = hist_grid(e->n_sm);
  mark_begin(e, T_ROOT);
  launch_hist(c, e->fo.p, e->rec.p, hist_gpair(e), cur_scale(e), nullptr, e->entries.p, ls0, hist, totals,
              e->row_stats.p, hgrid, smem, s);
  mark_end(e);
  launch_root_stats(fr, totals, s);
  launch_lg_setup(e->lg_state.p, e->lg_depth.p, e->tree.p, fr, cur_scale(e), ls2, s);
  mark_begin(e, T_SCAN);
  launch_scan(c, e->fo.p, hist, fr, ls0, nullptr, 0, cur_scale(e), 1, e->cand.p, s, nullptr, e->best_key.p);
  mark_end(e);
  HB_CK(e, cudaGetLastError());
  uint64_t launches = 5;
  const int max_leaves = p->max_leaves > 0 ? p->max_leaves : INT_MAX;
  const int depth_limit = p->max_depth > 0 ? p->max_depth : INT_MAX;
  uint32_t* rows0 = e->rows[0];
  uint32_t* rows1 = e->rows[1];
  // one-pass partition unless the stable one is asked for (or positions in
  // the 2n buffer would not fit 32 bits); fill zero before the first pass
  const bool onepass = !e->stable_partition && 2 * c.n_rows < (1ull << 32);
  const uint32_t half = (uint32_t)c.n_rows;
  if (onepass) HB_CK(e, cudaMemsetAsync(e->fill.p, 0, 2 * sizeof(uint32_t), s));
  for (int k = 0; k < L; ++k) {
    const bool final_step = k == L - 1;
    mark_begin(e, T_APPLY);
    launch_lg_step(c, e->fo.p, e->cuts.p, e->cand.p, k == 0 ? fr : nx, fr, nx, e->dec.p, ls1, ls2,
                   e->tree.p, e->wtree.p, cur_scale(e), e->lg_heap.p, e->lg_pool.p, L + 2, e->lg_state.p,
                   e->lg_depth.p,
                   max_leaves, depth_limit, final_step ? 1 : 0, e->best_key.p, s);
    mark_end(e);
    ++launches;
    if (final_step) break;
    mark_begin(e, T_PART);
    if (onepass) {
      // the node's rows move to the other half of the 2n row buffer
      launch_part_onepass(c, e->col.p, e->colmiss.p, rows0, k == 0, fr, e->dec.p, ls1, e->max_items,
                          e->fill.p, rows0, half, s);
      launch_part_plan(fr, e->dec.p, ls1, e->fill.p, nx, e->entries.p, e->pairs.p, ls2, 1, half, s);
      launches -= 1;
    } else {
      // the count pass leaves a copy of the node's row ids in rows1, and the
      // scatter writes the children from it back into rows0, where every
      // pending node's rows stay
      launch_part_count(c, e->col.p, e->colmiss.p, e->rec.p, 0, rows0, k == 0,
                        fr, e->dec.p, e->items.p, ls1, e->max_items, e->dirbits.p, e->item_left.p, s,
                        rows1);
      launch_part_scan(fr, e->dec.p, ls1, 1, e->item_left.p, e->item_off.p, nx, e->entries.p,
                       e->pairs.p, ls2, s);
      launch_part_scatter(fr, e->dec.p, e->items.p, ls1, e->max_items, e->dirbits.p, e->item_off.p, nx,
                          rows1, 0, rows0, s);
    }
    mark_end(e);
    mark_begin(e, T_HIST);
    launch_hist(c, e->fo.p, e->rec.p, hist_gpair(e), cur_scale(e), rows0, e->entries.p, ls2, hist, nullptr,
                e->row_stats.p, hgrid, smem, s);
    mark_end(e);
    mark_begin(e, T_SCAN);
    launch_scan(c, e->fo.p, hist, nx, ls2, e->pairs.p, -1, cur_scale(e), 2, e->cand.p, s, nullptr,
                e->best_key.p);
    mark_end(e);
    launches += 5;
    HB_CK(e, cudaGetLastError());
  }
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0x01, sizeof(int), s));
  e->pending_tree = true;
  walk_shape(p, e->walk_ls, e->walk_nodes, e->walk_depth);
  if (to_forest) {
    launch_finish_tree(e->tree.p, ls2, e->forest.p, e->counts.p, e->tree_counter.p,
                       (uint32_t)n_nodes, s);
    HB_CK(e, cudaGetLastError());
  }
  e->kernel_launches += launches + (to_forest ? 1 : 0);
  e->rounds_done += 1;
  return HB_OK;
}

hb_status grow_tree_device(hb_engine* e, const hb_train_params* p, bool to_forest) {
  return p->grow_policy == HB_GROW_LOSSGUIDE ? grow_lossguide(e, p, to_forest)
                                             : grow_device(e, p, to_forest);
}

hb_status stage_monotone(hb_engine* e, const hb_train_params* p);

// The parameters device growth takes (refused otherwise), and the run's
// monotone constraints staged on the device.
hb_status check_params(hb_engine* e, const hb_train_params* p) {
  if (!p) return HB_INVALID_ARGUMENT;
  if (p->grow_policy == HB_GROW_LOSSGUIDE) {
    if (e->comm) return refuse(e, "lossguide growth runs on one GPU");
    if (p->max_leaves < 0 || p->max_depth < 0 || (p->max_leaves == 0 && p->max_depth == 0))
      return refuse(e, "lossguide growth needs max_leaves or max_depth");
    if (lg_leaves(p) < 1 || lg_leaves(p) > 1024)
      return refuse(e, "lossguide growth supports at most 1024 leaves");
    if (p->objective == HB_LOSS_SOFTMAX) return refuse(e, "lossguide growth is single-output");
  } else if (p->grow_policy != HB_GROW_DEPTHWISE) {
    return HB_INVALID_ARGUMENT;
  } else if (p->max_depth < 1 || p->max_depth > kMaxDepth) {
    return refuse(e, "depthwise device growth supports 1 <= max_depth <= 10");
  }
  if (p->objective != HB_LOSS_SQUARED_ERROR && p->objective != HB_LOSS_LOGISTIC &&
      p->objective != HB_LOSS_SOFTMAX)
    return HB_INVALID_ARGUMENT;
  if (p->objective == HB_LOSS_SOFTMAX) {
    if (p->num_class < 2 || p->num_class > 64)
      return refuse(e, "multi:softmax supports num_class 2..64");
    if (e->n_out != p->num_class) return refuse(e, "start the run with hb_train_begin_classes");
  } else if (e->n_out != 1) {
    return refuse(e, "a multi:softmax run is loaded (hb_train_begin resets it)");
  }
  if (!e->uploaded) return refuse(e, "no index uploaded");
  return stage_monotone(e, p);
}

// The run's monotone constraints on the device (before any capture): one
// direction per feature, or none (c.mono = NULL) when every one is 0.
hb_status stage_monotone(hb_engine* e, const hb_train_params* p) {
  std::vector<int8_t> d(e->c.n_cols, 0);
  bool any = false;
  if (p->n_monotone < 0 || (p->n_monotone > 0 && !p->monotone)) return HB_INVALID_ARGUMENT;
  if ((uint32_t)p->n_monotone > e->c.n_cols)
    return refuse(e, "more monotone constraints than features");
  for (int32_t f = 0; f < p->n_monotone; ++f) {
    const int8_t v = p->monotone[f];
    if (v < -1 || v > 1) return refuse(e, "a monotone constraint must be -1, 0 or 1");
    d[f] = v;
    any = any || v != 0;
  }
  if (!any) {
    e->c.mono = nullptr;
    return HB_OK;
  }
  if (d != e->h_mono || !e->mono.p) {
    HB_CK(e, e->mono.alloc(d.size()));
    HB_CK(e, cudaMemcpyAsync(e->mono.p, d.data(), d.size(), cudaMemcpyHostToDevice, e->stream));
    HB_CK(e, cudaStreamSynchronize(e->stream));
    e->h_mono = d;
  }
  e->c.mono = e->mono.p;
  return HB_OK;
}

}  // namespace

// ===========================================================================
// C ABI
extern "C" {

hb_status hb_engine_create(int32_t device_ordinal, hb_engine** out) {
  if (!out) return HB_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  cudaError_t ce = cudaGetDeviceCount(&n);
  if (ce != cudaSuccess || device_ordinal < 0 || device_ordinal >= n) {
    g_last_error = "no such CUDA device";
    return HB_REFUSED;
  }
  hb_engine* e = new hb_engine();
  e->device = device_ordinal;
  if (cudaSetDevice(device_ordinal) != cudaSuccess ||
      cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete e;
    g_last_error = "cannot open the CUDA device";
    return HB_DEVICE_FAILED;
  }
  cudaDeviceGetAttribute(&e->n_sm, cudaDevAttrMultiProcessorCount, device_ordinal);
  hist_configure();
  cudaEventCreate(&e->run_ev[0]);
  cudaEventCreate(&e->run_ev[1]);
  const char* ng = std::getenv("HB_NO_GRAPHS");
  e->use_graphs = !(ng && ng[0] == '1');
  const char* sp = std::getenv("HB_STABLE_PARTITION");
  e->stable_partition = sp && sp[0] == '1';
  const char* pa = std::getenv("HB_PEER_ALLREDUCE");
  e->peer_mode = pa && pa[0] == '1';

  if (e->scale.alloc(1) != cudaSuccess || e->tree_counter.alloc(1) != cudaSuccess ||
      e->seg_total.alloc(2) != cudaSuccess || e->row_stats.alloc(2) != cudaSuccess ||
      cudaMemset(e->row_stats.p, 0, 16) != cudaSuccess || e->flags.alloc(4) != cudaSuccess ||
      cudaMemset(e->flags.p, 0, 16) != cudaSuccess) {
    delete e;
    return HB_DEVICE_FAILED;
  }
  *out = e;
  return HB_OK;
}

hb_status hb_engine_destroy(hb_engine* e) {
  if (!e) return HB_INVALID_ARGUMENT;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  // the round graph holds the level allreduces: release it before the communicator
  if (e->round_exec) cudaGraphExecDestroy(e->round_exec);
  e->round_exec = nullptr;
  close_peers(e);
  e->pbar.release();
  if (e->comm) ncclCommDestroy(e->comm);
  for (auto x : e->ev) cudaEventDestroy(x);
  for (auto x : e->run_ev)
    if (x) cudaEventDestroy(x);
  e->rec.release();
  e->col.release();
  e->colmiss.release();
  e->csr_ptr.release();
  e->csr_bins.release();
  e->fo.release();
  e->cuts.release();
  e->gpair.release();
  e->margin.release();
  e->label.release();
  e->weight.release();
  e->rows_all.release();
  e->rows[0] = e->rows[1] = nullptr;
  e->scale.release();
  e->hist_all.release();
  e->front[0].release();
  e->front[1].release();
  e->cand.release();
  e->dec.release();
  e->items.release();
  e->lg_heap.release();
  e->lg_pool.release();
  e->lg_state.release();
  e->lg_depth.release();
  e->dirbits.release();
  e->item_left.release();
  e->item_off.release();
  e->fill.release();
  e->best_key.release();
  e->entries.release();
  e->pairs.release();
  e->ls.release();
  e->tree.release();
  e->wtree.release();
  e->forest.release();
  e->counts.release();
  e->tree_counter.release();
  e->call_rows.release();
  e->call_hist.release();
  e->call_out.release();
  e->resident.release();
  e->seg_total.release();
  e->row_stats.release();
  e->flags.release();
  e->mono.release();
  e->scan_dirs.release();
  e->seg_tiles.release();
  e->part_ends.release();
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return HB_OK;
}

const char* hb_engine_last_error(const hb_engine* e) {
  return e ? e->err.c_str() : g_last_error.c_str();
}

// The two halves of the row-id buffer for an index of n rows.
static cudaError_t alloc_rows(hb_engine* e, uint64_t n) {
  cudaError_t ce = e->rows_all.alloc(std::max<uint64_t>(2 * n, 2));
  e->rows[0] = e->rows_all.p;
  e->rows[1] = e->rows_all.p ? e->rows_all.p + n : nullptr;
  return ce;
}

// Engine state after a new index: nothing staged, no cached round graph.
static hb_status finish_upload(hb_engine* e) {
  e->uploaded = true;
  e->alloc_depth = -1;
  e->lg_alloc = 0;
  if (e->round_exec) cudaGraphExecDestroy(e->round_exec);
  e->round_exec = nullptr;
  e->label_key = e->weight_key = nullptr;
  e->margins_loaded = false;
  e->staged = false;
  return HB_OK;
}

// A raw matrix already on the device that the upload bins itself (the
// device sketch, hb_sketch.cu), in place of the caller's binned index.
struct RawSource {
  const float* x = nullptr;      // dense row-major, NaN missing
  const uint64_t* ip = nullptr;  // CSR offsets, columns, values
  const uint32_t* ix = nullptr;
  const float* v = nullptr;
  uint64_t nnz = 0;
};

// The CSR half of the upload (ghist.rs:6-21 `rows`): offsets and global
// bins as they are; no record or column copy.
static hb_status upload_csr(hb_engine* e, const hb_ghist* g, const RawSource* raw) {
  DevConst& c = e->c;
  const uint64_t n = c.n_rows;
  cudaStream_t s = e->stream;
  if (raw) {
    HB_CK(e, e->csr_ptr.alloc(n + 1));
    HB_CK(e, e->csr_bins.alloc(std::max<uint64_t>(raw->nnz, 1)));
    DevBuf<int> flag;
    HB_CK(e, flag.alloc(1));
    HB_CK(e, cudaMemcpyAsync(e->csr_ptr.p, raw->ip, 8 * (n + 1), cudaMemcpyDeviceToDevice, s));
    HB_CK(e, bin_csr_device(raw->ip, raw->ix, raw->v, n, c.n_cols, raw->nnz, e->fo.p, e->cuts.p,
                            e->csr_bins.p, flag.p, s));
    int hf = 0;
    HB_CK(e, cudaMemcpyAsync(&hf, flag.p, 4, cudaMemcpyDeviceToHost, s));
    HB_CK(e, cudaStreamSynchronize(s));
    flag.release();
    e->has_missing = (hf & 4) != 0;
    c.dense = e->has_missing ? 0 : 1;
  } else {
    if (g->row_ptr[0] != 0) return HB_INVALID_ARGUMENT;
    const uint64_t nnz = g->row_ptr[n];
    if (nnz && !g->row_bins) return HB_INVALID_ARGUMENT;
    for (uint64_t r = 0; r < n; ++r)
      if (g->row_ptr[r + 1] < g->row_ptr[r]) return HB_INVALID_ARGUMENT;
    for (uint64_t j = 0; j < nnz; ++j)
      if (g->row_bins[j] >= c.total_bins) return refuse(e, "row_bins: a bin beyond the cuts");
    HB_CK(e, e->csr_ptr.alloc(n + 1));
    HB_CK(e, e->csr_bins.alloc(std::max<uint64_t>(nnz, 1)));
    HB_CK(e, cudaMemcpyAsync(e->csr_ptr.p, g->row_ptr, 8 * (n + 1), cudaMemcpyHostToDevice, s));
    if (nnz) HB_CK(e, cudaMemcpyAsync(e->csr_bins.p, g->row_bins, 4 * nnz, cudaMemcpyHostToDevice, s));
    e->has_missing = !g->dense;
  }
  c.csr = 1;
  c.csr_ptr = e->csr_ptr.p;
  c.csr_bins = e->csr_bins.p;
  e->col.release();
  e->rec.release();
  e->colmiss.release();
  c.csr_col = nullptr;
  c.csr_colmiss = nullptr;
  // The index also held feature-major when local bins fit a byte and the
  // copy takes at most half the free memory (HB_CSR_COLUMNS=0: never): the
  // partition and the walks read a row's split cell as one byte and one bit
  // instead of binary-searching the row's bins.
  const char* cc = std::getenv("HB_CSR_COLUMNS");
  const uint64_t words = (n + 63) / 64;
  // the bitmap unless every row stores every feature (an absent cell reads
  // as missing, as the binary search finds it)
  const uint64_t nnz = raw ? raw->nnz : g->row_ptr[n];
  const bool bitmap = e->has_missing || nnz != n * (uint64_t)c.n_cols;
  const uint64_t bytes = (uint64_t)c.n_cols * n + (bitmap ? 8ull * c.n_cols * words : 0ull);
  size_t free_b = 0, total_b = 0;
  if (!(cc && cc[0] == '0') && c.max_bins <= 256 && n && c.n_cols &&
      cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && bytes <= free_b / 2) {
    HB_CK(e, e->col.alloc((size_t)c.n_cols * n));
    HB_CK(e, cudaMemsetAsync(e->col.p, 0, (size_t)c.n_cols * n, s));
    if (bitmap) {
      HB_CK(e, e->colmiss.alloc((size_t)c.n_cols * words));
      HB_CK(e, cudaMemsetAsync(e->colmiss.p, 0xFF, 8 * (size_t)c.n_cols * words, s));
    }
    launch_csr_columns(c, e->col.p, bitmap ? e->colmiss.p : nullptr, e->n_sm, s);
    HB_CK(e, cudaGetLastError());
    c.csr_col = e->col.p;
    c.csr_colmiss = bitmap ? e->colmiss.p : nullptr;
  }
  return HB_OK;
}

// CudaHistBackend::new + upload (src/backend/cuda/mod.rs:1626,1687) of the
// index `g`; with `raw`, the bins (and the dense flag) come from binning the
// raw device matrix against g's cuts instead of from g.
// The CSR form (ghist.rs:6-21 `rows`: each present cell's global bin, in
// feature order within its row) of a dense index given as feature-major
// local bins and a missing bitmap: the layout an index wider than the row
// records hold (kMaxRecordFeatures features) trains on. Absent cells are the
// missing ones, the reference's own equivalence of the two layouts.
static void dense_to_csr(const hb_ghist* g, std::vector<uint64_t>& ptr, std::vector<uint32_t>& bins) {
  const uint64_t n = g->n_rows, words = (n + 63) / 64;
  ptr.assign(n + 1, 0);
  auto present = [&](uint64_t r, uint32_t f) {
    return !g->missing || !((g->missing[(uint64_t)f * words + r / 64] >> (r % 64)) & 1ull);
  };
  for (uint64_t r = 0; r < n; ++r) {
    uint64_t k = 0;
    for (uint32_t f = 0; f < g->n_cols; ++f) k += present(r, f);
    ptr[r + 1] = ptr[r] + k;
  }
  bins.resize(ptr[n]);
  for (uint64_t r = 0; r < n; ++r) {
    uint64_t at = ptr[r];
    for (uint32_t f = 0; f < g->n_cols; ++f)
      if (present(r, f)) bins[at++] = g->feature_offset[f] + g->columns[(uint64_t)f * n + r];
  }
}

static hb_status upload_index(hb_engine* e, const hb_ghist* g, const RawSource* raw) {
  bool csr = raw ? raw->ip != nullptr : (g && !g->columns && g->row_ptr);
  if (!g || !g->feature_offset || !g->cut_values || (!raw && !g->columns && !csr) ||
      (raw && !raw->x && !raw->ip) || g->n_rows == 0 || g->n_cols == 0)
    return HB_INVALID_ARGUMENT;
  if (g->n_rows >= (1ull << 32)) return refuse(e, "at most 2^32 - 1 rows per device");
  std::vector<uint64_t> wide_ptr;
  std::vector<uint32_t> wide_bins;
  hb_ghist wide_g;
  if (!csr && g->n_cols > kMaxRecordFeatures) {
    if (raw) return refuse(e, "a raw dense matrix of more than 224 features: upload its CSR form");
    dense_to_csr(g, wide_ptr, wide_bins);
    wide_g = *g;
    wide_g.columns = nullptr;
    wide_g.missing = nullptr;
    wide_g.row_ptr = wide_ptr.data();
    wide_g.row_bins = wide_bins.empty() ? nullptr : wide_bins.data();
    g = &wide_g;
    csr = true;
  }
  DevConst& c = e->c;
  const uint64_t shard_rows = e->shard_global;
  c = DevConst{};
  e->blk_pairs = false;
  c.n_rows = g->n_rows;
  c.global_rows = shard_rows > g->n_rows ? shard_rows : g->n_rows;
  c.n_cols = g->n_cols;
  e->h_fo.assign(g->feature_offset, g->feature_offset + g->n_cols + 1);
  c.total_bins = e->h_fo.back();
  uint32_t widest = 0;
  for (uint32_t f = 0; f < g->n_cols; ++f) widest = std::max(widest, e->h_fo[f + 1] - e->h_fo[f]);
  if (!csr && widest > 256) return refuse(e, "features of more than 256 bins need the CSR index");
  if (widest > 65535) return refuse(e, "at most 65,535 bins per feature");
  c.max_bins = widest;
  c.mask_off = (g->n_cols + 3) / 4 * 4;
  c.stride = (c.mask_off + 4 * ((g->n_cols + 31) / 32) + 15) / 16 * 16;
  c.dense = g->dense ? 1 : 0;
  c.n_groups = (g->n_cols + kGroupFeatures - 1) / kGroupFeatures;
  // Both histogram kernels give the same exact sums; HB_HIST_KERNEL=64
  // selects the 64-bit-atomic one for every size (comparison runs).
  const char* hk = std::getenv("HB_HIST_KERNEL");
  c.hist64 = (hk && std::strcmp(hk, "64") == 0) ? 1u : 0u;
  // HB_SCAN_KERNEL=cta keeps the CTA-per-feature scan for every width.
  const char* sk = std::getenv("HB_SCAN_KERNEL");
  c.scan_cta = (sk && std::strcmp(sk, "cta") == 0) ? 1u : 0u;
  e->h_cuts.assign(g->cut_values, g->cut_values + c.total_bins);
  // a raw dense matrix may have missing cells: the bitmap is kept until the
  // binning says otherwise
  e->has_missing = raw ? true : g->missing != nullptr;

  const uint64_t n = c.n_rows, words = (n + 63) / 64;
  HB_CK(e, e->fo.alloc(c.n_cols + 1));
  HB_CK(e, e->cuts.alloc(c.total_bins));
  c.fo = e->fo.p;
  if (csr) {
    HB_CK(e, e->gpair.alloc(n));
    HB_CK(e, e->margin.alloc(n));
    HB_CK(e, e->label.alloc(n));
    HB_CK(e, alloc_rows(e, n));
    cudaStream_t s = e->stream;
    HB_CK(e, cudaMemcpyAsync(e->fo.p, e->h_fo.data(), 4 * (c.n_cols + 1), cudaMemcpyHostToDevice, s));
    HB_CK(e, cudaMemcpyAsync(e->cuts.p, e->h_cuts.data(), 4 * c.total_bins, cudaMemcpyHostToDevice, s));
    hb_status st = upload_csr(e, g, raw);
    if (st != HB_OK) return st;
    HB_CK(e, cudaStreamSynchronize(s));
    return finish_upload(e);
  }
  HB_CK(e, e->col.alloc((size_t)c.n_cols * n));
  // HB_ROW_BLOCKS=0 keeps records `stride` apart and the pairs apart
  const char* rb = std::getenv("HB_ROW_BLOCKS");
  c.blk = (rb && rb[0] == '0') ? 0u : block_rows(c.stride);
  c.blk_pair = c.blk * c.stride;
  HB_CK(e, e->rec.alloc(rec_bytes(n, c.stride, c.blk)));
  // the partition reads the bitmap whenever one is held
  if (e->has_missing) HB_CK(e, e->colmiss.alloc((size_t)c.n_cols * words));
  else e->colmiss.release();
  HB_CK(e, e->gpair.alloc(n));
  HB_CK(e, e->margin.alloc(n));
  HB_CK(e, e->label.alloc(n));
  HB_CK(e, alloc_rows(e, n));
  cudaStream_t s = e->stream;
  HB_CK(e, cudaMemcpyAsync(e->fo.p, e->h_fo.data(), 4 * (c.n_cols + 1), cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaMemcpyAsync(e->cuts.p, e->h_cuts.data(), 4 * c.total_bins, cudaMemcpyHostToDevice, s));
  if (raw) {
    DevBuf<int> any;
    HB_CK(e, any.alloc(1));
    HB_CK(e, bin_dense_device(raw->x, n, c.n_cols, e->fo.p, e->cuts.p, e->col.p, e->colmiss.p, any.p, s));
    int h_any = 0;
    HB_CK(e, cudaMemcpyAsync(&h_any, any.p, 4, cudaMemcpyDeviceToHost, s));
    HB_CK(e, cudaStreamSynchronize(s));
    any.release();
    if (!h_any) {
      e->has_missing = false;
      e->colmiss.release();
    }
    c.dense = h_any ? 0 : 1;
  } else {
    HB_CK(e, cudaMemcpyAsync(e->col.p, g->columns, (size_t)c.n_cols * n, cudaMemcpyHostToDevice, s));
    if (e->has_missing)
      HB_CK(e, cudaMemcpyAsync(e->colmiss.p, g->missing, 8 * (size_t)c.n_cols * words,
                               cudaMemcpyHostToDevice, s));
  }
  HB_CK(e, cudaMemsetAsync(e->rec.p, 0, rec_bytes(n, c.stride, c.blk), s));
  launch_encode(e->col.p, e->has_missing ? e->colmiss.p : nullptr, n, c.n_cols, c.stride,
                c.mask_off, c.blk, e->rec.p, s);
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaStreamSynchronize(s));
  e->csr_ptr.release();
  e->csr_bins.release();
  return finish_upload(e);
}

hb_status hb_engine_upload(hb_engine* e, const hb_ghist* g) {
  HB_ENTER(e);
  return upload_index(e, g, nullptr);
}

// The sketch's outcome as the engine's: a refusal leaves the engine usable,
// a device error is sticky.
static hb_status sketch_status(hb_engine* e, hb_status st, const std::string& why) {
  if (st == HB_OK) return HB_OK;
  if (st == HB_REFUSED) return refuse(e, why);
  if (st == HB_DEVICE_FAILED) {
    e->failed = true;
    e->err = why;
    g_last_error = why;
  }
  return st;
}

static hb_status copy_cuts(hb_engine* e, const std::vector<uint32_t>& fo, const std::vector<float>& cuts,
                           uint32_t n_cols, uint32_t* feature_offset, float* cut_values, uint64_t cap,
                           uint64_t* total) {
  if (cuts.size() > cap) return refuse(e, "cut_values capacity below the cut count");
  std::memcpy(feature_offset, fo.data(), 4 * (size_t)(n_cols + 1));
  std::memcpy(cut_values, cuts.data(), 4 * cuts.size());
  *total = cuts.size();
  return HB_OK;
}

hb_status hb_engine_upload_dense(hb_engine* e, const float* x, uint64_t n_rows, uint32_t n_cols,
                                 uint32_t max_bin, uint32_t* feature_offset, float* cut_values,
                                 uint64_t cap, uint64_t* total) {
  HB_ENTER(e);
  if (!x || !feature_offset || !cut_values || !total || n_rows == 0 || n_cols == 0 || max_bin == 0)
    return HB_INVALID_ARGUMENT;
  if (e->comm || e->shard_global > n_rows)
    return refuse(e, "a row shard needs the whole matrix's cuts: hb_sketch_dense of the whole "
                     "matrix, then hb_bin_dense of the shard and hb_engine_upload");
  if (n_rows >= (1ull << 32)) return refuse(e, "at most 2^32 - 1 rows per device");
  if (n_cols > kMaxRecordFeatures) return refuse(e, "at most 224 features per raw dense upload");
  cudaStream_t s = e->stream;
  DevBuf<float> dx;
  HB_CK(e, dx.alloc((size_t)n_rows * n_cols));
  HB_CK(e, cudaMemcpyAsync(dx.p, x, 4 * (size_t)n_rows * n_cols, cudaMemcpyHostToDevice, s));
  std::vector<uint32_t> fo;
  std::vector<float> cuts;
  std::string why;
  hb_status st = sketch_status(e, sketch_dense_cuts(e->device, dx.p, n_rows, n_cols, max_bin, s, fo, cuts, why), why);
  if (st != HB_OK) return st;
  st = copy_cuts(e, fo, cuts, n_cols, feature_offset, cut_values, cap, total);
  if (st != HB_OK) return st;
  hb_ghist g{};
  g.n_rows = n_rows;
  g.n_cols = n_cols;
  g.feature_offset = fo.data();
  g.cut_values = cuts.data();
  RawSource raw;
  raw.x = dx.p;
  st = upload_index(e, &g, &raw);
  dx.release();
  return st;
}

hb_status hb_engine_upload_csr(hb_engine* e, const uint64_t* indptr, const uint32_t* indices,
                               const float* values, uint64_t n_rows, uint32_t n_cols, uint32_t max_bin,
                               uint32_t* feature_offset, float* cut_values, uint64_t cap,
                               uint64_t* total) {
  HB_ENTER(e);
  if (!indptr || !feature_offset || !cut_values || !total || n_rows == 0 || n_cols == 0 ||
      max_bin == 0 || indptr[0] != 0)
    return HB_INVALID_ARGUMENT;
  if (e->comm || e->shard_global > n_rows)
    return refuse(e, "a row shard needs the whole matrix's cuts: hb_sketch_csr of the whole "
                     "matrix, then hb_bin_csr of the shard and hb_engine_upload");
  if (n_rows >= (1ull << 32)) return refuse(e, "at most 2^32 - 1 rows per device");
  const uint64_t nnz = indptr[n_rows];
  if (nnz && (!indices || !values)) return HB_INVALID_ARGUMENT;
  cudaStream_t s = e->stream;
  DevBuf<uint64_t> dip;
  DevBuf<uint32_t> dix;
  DevBuf<float> dv;
  HB_CK(e, dip.alloc(n_rows + 1));
  HB_CK(e, dix.alloc(std::max<uint64_t>(nnz, 1)));
  HB_CK(e, dv.alloc(std::max<uint64_t>(nnz, 1)));
  HB_CK(e, cudaMemcpyAsync(dip.p, indptr, 8 * (n_rows + 1), cudaMemcpyHostToDevice, s));
  if (nnz) {
    HB_CK(e, cudaMemcpyAsync(dix.p, indices, 4 * nnz, cudaMemcpyHostToDevice, s));
    HB_CK(e, cudaMemcpyAsync(dv.p, values, 4 * nnz, cudaMemcpyHostToDevice, s));
  }
  std::vector<uint32_t> fo;
  std::vector<float> cuts;
  std::string why;
  hb_status st = sketch_status(
      e, sketch_csr_cuts(e->device, dip.p, dix.p, dv.p, n_rows, n_cols, nnz, max_bin, s, fo, cuts, why), why);
  if (st != HB_OK) return st;
  st = copy_cuts(e, fo, cuts, n_cols, feature_offset, cut_values, cap, total);
  if (st != HB_OK) return st;
  hb_ghist g{};
  g.n_rows = n_rows;
  g.n_cols = n_cols;
  g.feature_offset = fo.data();
  g.cut_values = cuts.data();
  RawSource raw;
  raw.ip = dip.p;
  raw.ix = dix.p;
  raw.v = dv.p;
  raw.nnz = nnz;
  return upload_index(e, &g, &raw);
}

// ---- HistogramBackend ------------------------------------------------------
hb_status hb_prepare(hb_engine* e, const hb_grad_pair* gpair, uint64_t n) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if (!gpair || n != e->c.n_rows) return HB_INVALID_ARGUMENT;
  cudaStream_t s = e->stream;
  HB_CK(e, cudaMemcpyAsync(e->gpair.p, gpair, 8 * n, cudaMemcpyHostToDevice, s));
  e->blk_pairs = false;
  HB_CK(e, cudaMemsetAsync(e->scale.p, 0, sizeof(Scale), s));
  launch_pair_maxima(e->gpair.p, n, e->scale.p, e->n_sm, s);
  HB_CK(e, cudaGetLastError());
  hb_status st = finish_scale(e);
  if (st != HB_OK) return st;
  Scale h;
  HB_CK(e, cudaMemcpyAsync(&h, e->scale.p, sizeof(Scale), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  if (h.nonfinite) {
    e->staged = false;
    return refuse(e, "non-finite gradients");
  }
  e->staged = true;
  return HB_OK;
}

// Histograms of `n` row lists already on the device (call_rows, entries
// back to back) into call_hist slots 0..n-1, dequantised into `out`.
static hb_status build_entries(hb_engine* e, const std::vector<HEntry>& en, longlong2* dst,
                               uint32_t n_slots_to_zero, const uint32_t* rows_dev) {
  DevConst& c = e->c;
  cudaStream_t s = e->stream;
  HB_CK(e, e->entries.alloc(std::max<size_t>(en.size(), 1)));
  HB_CK(e, e->ls.alloc(kMaxDepth + 2));
  LevelState lsh{};
  lsh.n_hentries = (int32_t)en.size();
  uint64_t total = 0;
  for (const auto& x : en) total += x.len;
  lsh.hist_rows = total;
  HB_CK(e, cudaMemcpyAsync(e->entries.p, en.data(), sizeof(HEntry) * en.size(), cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaMemcpyAsync(e->ls.p, &lsh, sizeof(LevelState), cudaMemcpyHostToDevice, s));
  if (n_slots_to_zero)
    HB_CK(e, cudaMemsetAsync(dst, 0, sizeof(longlong2) * (size_t)n_slots_to_zero * c.total_bins, s));
  launch_hist(c, e->fo.p, e->rec.p, e->gpair.p, e->scale.p, rows_dev, e->entries.p, e->ls.p, dst,
              nullptr, nullptr, hist_grid(e->n_sm), hist_smem_bytes(c), s);
  HB_CK(e, cudaGetLastError());
  return HB_OK;
}

static hb_status download_hist(hb_engine* e, const longlong2* src, uint32_t n_hists,
                               hb_grad_stats* out) {
  const size_t bins = (size_t)n_hists * e->c.total_bins;
  HB_CK(e, e->call_out.alloc(2 * bins));
  launch_dequantize(src, (uint32_t)bins, e->scale.p, e->call_out.p, e->stream);
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaMemcpyAsync(out, e->call_out.p, 16 * bins, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

hb_status hb_build(hb_engine* e, const uint32_t* rows, uint64_t n, hb_grad_stats* out) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  if ((!rows && n) || !out) return HB_INVALID_ARGUMENT;
  for (uint64_t i = 0; i < n; ++i)
    if (rows[i] >= e->c.n_rows || (i && rows[i] <= rows[i - 1])) return refuse(e, "rows must ascend within the index");
  HB_CK(e, e->call_rows.alloc(std::max<uint64_t>(n, 1)));
  HB_CK(e, e->call_hist.alloc(e->c.total_bins));
  if (n) HB_CK(e, cudaMemcpyAsync(e->call_rows.p, rows, 4 * n, cudaMemcpyHostToDevice, e->stream));
  std::vector<HEntry> en(1);
  en[0].slot = 0;
  en[0].identity = 0;
  en[0].begin = 0;
  en[0].len = (uint32_t)n;
  en[0].prefix = 0;
  hb_status st = build_entries(e, en, e->call_hist.p, 1, e->call_rows.p);
  if (st != HB_OK) return st;
  return download_hist(e, e->call_hist.p, 1, out);
}

hb_status hb_build_features(hb_engine* e, const uint32_t* rows, uint64_t n,
                            const uint32_t* features, uint32_t n_features, hb_grad_stats* out) {
  (void)features;
  (void)n_features;
  return hb_build(e, rows, n, out);
}

// ---- RowEngine ----------------------------------------------------------
static bool seg_ok(const hb_engine* e, const hb_segment* s) {
  return s && s->tree == e->tree_stamp && s->offset + s->len <= e->c.n_rows;
}

// check_rows (src/backend/cuda/mod.rs:817): every row inside the index,
// strictly ascending, and whether the list is one contiguous run; chunks of
// the list checked by the host's threads.
static void check_rows(const uint32_t* rows, uint64_t n, uint64_t n_rows, bool& inside, bool& ascending,
                       bool& run) {
  inside = ascending = run = true;
  if (!n) return;
  const uint64_t chunk = 1 << 20;
  const uint64_t n_chunks = (n + chunk - 1) / chunk;
  std::vector<unsigned char> ok(3 * n_chunks, 1);
  auto work = [&](uint64_t c0, uint64_t c1) {
    for (uint64_t c = c0; c < c1; ++c) {
      const uint64_t a = c * chunk, b = std::min(n, a + chunk);
      bool in = true, asc = a == 0 || rows[a - 1] < rows[a], rn = true;
      const uint32_t first = rows[0];
      for (uint64_t i = a; i < b; ++i) {
        in &= rows[i] < n_rows;
        rn &= (uint64_t)rows[i] == (uint64_t)first + i;
        if (i > a) asc &= rows[i - 1] < rows[i];
      }
      ok[3 * c] = in;
      ok[3 * c + 1] = asc;
      ok[3 * c + 2] = rn;
    }
  };
  const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  const uint64_t per = (n_chunks + hw - 1) / hw;
  std::vector<std::thread> pool;
  for (uint64_t c0 = per; c0 < n_chunks; c0 += per) pool.emplace_back(work, c0, std::min(n_chunks, c0 + per));
  work(0, std::min(n_chunks, per));
  for (auto& t : pool) t.join();
  for (uint64_t c = 0; c < n_chunks; ++c) {
    inside &= ok[3 * c] != 0;
    ascending &= ok[3 * c + 1] != 0;
    run &= ok[3 * c + 2] != 0;
  }
}

hb_status hb_begin_tree(hb_engine* e, const uint32_t* rows, uint64_t n, hb_segment* root) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if ((!rows && n) || !root || n > e->c.n_rows) return HB_INVALID_ARGUMENT;
  bool inside, ascending, run;
  check_rows(rows, n, e->c.n_rows, inside, ascending, run);
  if (!inside || !ascending) return refuse(e, "rows must be ascending and distinct");
  // a contiguous run is written on the device (place_rows, cuda/mod.rs:1830)
  if (n && run)
    launch_iota(e->rows[0], rows[0], n, e->n_sm, e->stream);
  else if (n)
    HB_CK(e, cudaMemcpyAsync(e->rows[0], rows, 4 * n, cudaMemcpyHostToDevice, e->stream));
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaStreamSynchronize(e->stream));
  ++e->tree_stamp;
  root->offset = 0;
  root->len = n;
  root->contiguous = (n == 0 || run) ? 1 : 0;
  root->reserved = 0;
  root->tree = e->tree_stamp;
  return HB_OK;
}

hb_status hb_histograms(hb_engine* e, const hb_segment* segs, uint32_t n, hb_grad_stats* out) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  if ((!segs && n) || (!out && n)) return HB_INVALID_ARGUMENT;
  std::vector<HEntry> en;
  uint64_t prefix = 0;
  for (uint32_t k = 0; k < n; ++k) {
    if (!seg_ok(e, &segs[k])) return refuse(e, "stale or foreign segment");
    HEntry x{};
    x.slot = (int32_t)k;
    x.identity = 0;
    x.begin = (uint32_t)segs[k].offset;
    x.len = (uint32_t)segs[k].len;
    x.prefix = prefix;
    prefix += x.len;
    en.push_back(x);
  }
  if (!n) return HB_OK;
  HB_CK(e, e->call_hist.alloc((size_t)n * e->c.total_bins));
  hb_status st = build_entries(e, en, e->call_hist.p, n, e->rows[0]);
  if (st != HB_OK) return st;
  return download_hist(e, e->call_hist.p, n, out);
}

hb_status hb_root_total(hb_engine* e, const hb_segment* seg, hb_grad_stats* out) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  if (!seg_ok(e, seg) || !out) return HB_INVALID_ARGUMENT;
  // The exact int64 sum of the segment's fixed-point pairs (the same
  // integers the histograms sum, so any order).
  cudaStream_t s = e->stream;
  HB_CK(e, cudaMemsetAsync(e->seg_total.p, 0, 16, s));
  launch_seg_total(e->rows[0], seg->offset, seg->len, e->gpair.p, e->scale.p, e->seg_total.p, e->n_sm, s);
  HB_CK(e, cudaGetLastError());
  long long t[2];
  Scale h;
  HB_CK(e, cudaMemcpyAsync(t, e->seg_total.p, 16, cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaMemcpyAsync(&h, e->scale.p, sizeof(Scale), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  out->grad = (double)t[0] * std::ldexp(1.0, -h.sg);
  out->hess = (double)t[1] * std::ldexp(1.0, -h.sh);
  return HB_OK;
}

hb_status hb_partition(hb_engine* e, const hb_row_split* splits, uint32_t n, hb_partitioned* out) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if ((!splits || !out) && n) return HB_INVALID_ARGUMENT;
  if (!n) return HB_OK;
  hb_status st = ensure_growth_buffers(e, 1);
  if (st != HB_OK) return st;
  DevConst& c = e->c;
  std::vector<Front> fr(n);
  std::vector<Decision> dc(n);
  std::vector<PItem> it;
  for (uint32_t k = 0; k < n; ++k) {
    const hb_row_split& sp = splits[k];
    if (!seg_ok(e, &sp.seg)) return refuse(e, "stale or foreign segment");
    if (sp.feature >= c.n_cols) return HB_INVALID_ARGUMENT;
    for (uint32_t j = 0; j < k; ++j) {
      const hb_segment& o = splits[j].seg;
      if (sp.seg.offset < o.offset + o.len && o.offset < sp.seg.offset + sp.seg.len)
        return refuse(e, "overlapping segments");
    }
    fr[k].begin = (uint32_t)sp.seg.offset;
    fr[k].len = (uint32_t)sp.seg.len;
    dc[k].split = 1;
    dc[k].pair = (int32_t)k;
    dc[k].feature = sp.feature;
    dc[k].limit = sp.limit;
    dc[k].default_left = sp.default_left ? 1 : 0;
    dc[k].item_begin = (int32_t)it.size();
    uint32_t tiles = (fr[k].len + kTile - 1) / kTile;
    dc[k].item_count = (int32_t)tiles;
    for (uint32_t t = 0; t < tiles; ++t) {
      PItem p{};
      p.k = (int32_t)k;
      p.kind = 1;
      p.off = t * kTile;
      p.len = std::min<uint32_t>(kTile, fr[k].len - t * kTile);
      it.push_back(p);
    }
  }
  const int n_items = (int)it.size();
  HB_CK(e, e->front[0].alloc(n));
  HB_CK(e, e->front[1].alloc(2 * (size_t)n));
  HB_CK(e, e->dec.alloc(n));
  HB_CK(e, e->items.alloc(std::max(n_items, 1)));
  HB_CK(e, e->dirbits.alloc((size_t)std::max(n_items, 1) * kTileWords));
  HB_CK(e, e->item_left.alloc(std::max(n_items, 1)));
  HB_CK(e, e->item_off.alloc(std::max(n_items, 1)));
  e->alloc_depth = -1;  // the growth buffers were resized for this call
  LevelState lsh{};
  lsh.n_front = (int32_t)n;
  lsh.n_items = n_items;
  cudaStream_t s = e->stream;
  HB_CK(e, cudaMemcpyAsync(e->front[0].p, fr.data(), sizeof(Front) * n, cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaMemcpyAsync(e->dec.p, dc.data(), sizeof(Decision) * n, cudaMemcpyHostToDevice, s));
  if (n_items)
    HB_CK(e, cudaMemcpyAsync(e->items.p, it.data(), sizeof(PItem) * n_items, cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaMemcpyAsync(e->ls.p, &lsh, sizeof(LevelState), cudaMemcpyHostToDevice, s));
  if (n_items) {
    launch_part_count(c, e->col.p, e->colmiss.p, e->rec.p, 0,
                      e->rows[0], 0, e->front[0].p, e->dec.p, e->items.p, e->ls.p, n_items,
                      e->dirbits.p, e->item_left.p, s);
  }
  launch_part_scan(e->front[0].p, e->dec.p, e->ls.p, (int)n, e->item_left.p, e->item_off.p,
                   e->front[1].p, nullptr, nullptr, nullptr, s);
  if (n_items) {
    launch_part_scatter(e->front[0].p, e->dec.p, e->items.p, e->ls.p, n_items, e->dirbits.p,
                        e->item_off.p, e->front[1].p, e->rows[0], 0, e->rows[1], s);
  }
  HB_CK(e, cudaGetLastError());
  // the children back in rows[0] and their end rows, one launch
  HB_CK(e, e->part_ends.alloc(4 * (size_t)n));
  HB_CK(e, cudaMemsetAsync(e->part_ends.p, 0, 16 * (size_t)n, s));
  launch_finish_partition(e->items.p, n_items, e->front[0].p, e->front[1].p, e->rows[1], e->rows[0],
                          e->part_ends.p, s);
  HB_CK(e, cudaGetLastError());
  std::vector<Front> nx(2 * (size_t)n);
  std::vector<uint32_t> ends(4 * (size_t)n);
  HB_CK(e, cudaMemcpyAsync(nx.data(), e->front[1].p, sizeof(Front) * 2 * n, cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaMemcpyAsync(ends.data(), e->part_ends.p, 4 * ends.size(), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  for (uint32_t k = 0; k < n; ++k) {
    for (int side = 0; side < 2; ++side) {
      const Front& f = nx[2 * k + side];
      hb_segment& sg = side ? out[k].right : out[k].left;
      sg.offset = f.begin;
      sg.len = f.len;
      sg.tree = e->tree_stamp;
      sg.reserved = 0;
      const uint32_t lo = ends[4 * k + 2 * side], hi = ends[4 * k + 2 * side + 1];
      sg.contiguous = f.len == 0 || (uint64_t)(hi - lo) + 1 == f.len ? 1 : 0;
    }
  }
  return HB_OK;
}

hb_status hb_rows(hb_engine* e, const hb_segment* segs, uint32_t n, uint32_t* out) {
  HB_ENTER(e);
  uint64_t at = 0;
  for (uint32_t k = 0; k < n; ++k) {
    if (!seg_ok(e, &segs[k])) return refuse(e, "stale or foreign segment");
    if (segs[k].len)
      HB_CK(e, cudaMemcpyAsync(out + at, e->rows[0] + segs[k].offset, 4 * segs[k].len,
                               cudaMemcpyDeviceToHost, e->stream));
    at += segs[k].len;
  }
  HB_CK(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

hb_status hb_load_margins(hb_engine* e, const float* margins, uint64_t n) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if (!margins || n != e->c.n_rows) return HB_INVALID_ARGUMENT;
  HB_CK(e, cudaMemcpyAsync(e->margin.p, margins, 4 * n, cudaMemcpyHostToDevice, e->stream));
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0, sizeof(int), e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  e->margins_loaded = true;
  e->pending_tree = false;
  e->label_key = e->weight_key = nullptr;
  return HB_OK;
}

hb_status hb_read_margins(hb_engine* e, float* out, uint64_t n) {
  HB_ENTER(e);
  if (!e->margins_loaded) return refuse(e, "no margin run");
  if (!out || (n != e->c.n_rows && n != e->c.n_rows * (uint64_t)e->n_out)) return HB_INVALID_ARGUMENT;
  HB_CK(e, cudaMemcpyAsync(out, e->margin.p, 4 * n, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

static hb_status stage_labels(hb_engine* e, const float* labels, const float* weights, uint64_t n) {
  cudaStream_t s = e->stream;
  if (e->label_key != labels) {
    HB_CK(e, cudaMemcpyAsync(e->label.p, labels, 4 * n, cudaMemcpyHostToDevice, s));
    e->label_key = labels;
  }
  if (weights && e->weight_key != weights) {
    HB_CK(e, e->weight.alloc(n));
    HB_CK(e, cudaMemcpyAsync(e->weight.p, weights, 4 * n, cudaMemcpyHostToDevice, s));
  }
  e->weight_key = weights;
  return HB_OK;
}

hb_status hb_gradients(hb_engine* e, const hb_device_loss* loss, const float* labels,
                       const float* weights, uint64_t n, int32_t* all_finite) {
  HB_ENTER(e);
  if (!e->uploaded || !e->margins_loaded) return refuse(e, "no margin run");
  if (!loss || !labels || n != e->c.n_rows || !all_finite) return HB_INVALID_ARGUMENT;
  if (loss->kind != HB_LOSS_SQUARED_ERROR && loss->kind != HB_LOSS_LOGISTIC) return HB_INVALID_ARGUMENT;
  if (e->row_begin % 8) return refuse(e, "shards must start on a multiple of 8 rows");
  hb_status st = stage_labels(e, labels, weights, n);
  if (st != HB_OK) return st;
  st = run_gradients(e, loss->kind, loss->scale_pos_weight, loss->min_hess, -1, 0, 0);
  if (st != HB_OK) return st;
  Scale h;
  HB_CK(e, cudaMemcpyAsync(&h, e->scale.p, sizeof(Scale), cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  *all_finite = h.nonfinite ? 0 : 1;
  if (h.nonfinite) e->staged = false;
  return HB_OK;
}

hb_status hb_add_leaf_values(hb_engine* e, const hb_segment* segs, const float* values, uint32_t n) {
  HB_ENTER(e);
  if (!e->margins_loaded) return refuse(e, "no margin run");
  for (uint32_t k = 0; k < n; ++k)
    if (!seg_ok(e, &segs[k])) return refuse(e, "stale or foreign segment");
  if (!n) return HB_OK;
  if (!values) return HB_INVALID_ARGUMENT;
  // segments cut into tiles of kAddTile rows, so a large leaf spreads over
  // many CTAs
  std::vector<uint4> tiles;
  for (uint32_t k = 0; k < n; ++k) {
    uint32_t bits;
    std::memcpy(&bits, values + k, 4);
    for (uint64_t o = 0; o < segs[k].len; o += kAddTile)
      tiles.push_back(make_uint4((uint32_t)(segs[k].offset + o),
                                 (uint32_t)std::min<uint64_t>(kAddTile, segs[k].len - o), bits, 0u));
  }
  if (tiles.empty()) return HB_OK;
  cudaStream_t s = e->stream;
  HB_CK(e, e->seg_tiles.alloc(tiles.size()));
  HB_CK(e, cudaMemcpyAsync(e->seg_tiles.p, tiles.data(), sizeof(uint4) * tiles.size(), cudaMemcpyHostToDevice, s));
  launch_add_segments(e->rows[0], e->seg_tiles.p, (uint32_t)tiles.size(), e->margin.p, s);
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaStreamSynchronize(s));
  return HB_OK;
}

hb_status hb_reserve_hists(hb_engine* e, uint32_t slots, int32_t* reserved) {
  HB_ENTER(e);
  if (!e->uploaded || !reserved) return HB_INVALID_ARGUMENT;
  const size_t need = (size_t)slots * e->c.total_bins * sizeof(longlong2);
  if ((size_t)slots * e->c.total_bins > e->resident.n) {  // only a buffer that must grow asks the driver
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    if (need > free_b / 2) {
      *reserved = 0;
      return HB_OK;
    }
  }
  HB_CK(e, e->resident.alloc(std::max<size_t>((size_t)slots * e->c.total_bins, 1)));
  e->resident_slots = slots;
  *reserved = 1;
  return HB_OK;
}

hb_status hb_build_resident(hb_engine* e, const hb_segment* segs, const uint32_t* slots, uint32_t n,
                            const uint32_t* siblings, uint32_t n_siblings) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  std::vector<HEntry> en;
  uint64_t prefix = 0;
  for (uint32_t k = 0; k < n; ++k) {
    if (!seg_ok(e, &segs[k])) return refuse(e, "stale or foreign segment");
    if (slots[k] >= e->resident_slots) return refuse(e, "slot not reserved");
    HEntry x{};
    x.slot = (int32_t)slots[k];
    x.begin = (uint32_t)segs[k].offset;
    x.len = (uint32_t)segs[k].len;
    x.prefix = prefix;
    prefix += x.len;
    en.push_back(x);
  }
  cudaStream_t s = e->stream;
  const uint32_t tb = e->c.total_bins;
  for (uint32_t k = 0; k < n; ++k)
    HB_CK(e, cudaMemsetAsync(e->resident.p + (size_t)slots[k] * tb, 0, sizeof(longlong2) * tb, s));
  if (n) {
    hb_status st = build_entries(e, en, e->resident.p, 0, e->rows[0]);
    if (st != HB_OK) return st;
  }
  if (n_siblings) {
    std::vector<Triple> tr(n_siblings);
    for (uint32_t j = 0; j < n_siblings; ++j) {
      uint32_t parent = siblings[2 * j], built = siblings[2 * j + 1];
      if (parent >= e->resident_slots || built >= e->resident_slots) return refuse(e, "slot not reserved");
      tr[j].parent = (int32_t)parent;
      tr[j].built = (int32_t)built;
      tr[j].sibling = (int32_t)parent;
    }
    HB_CK(e, e->pairs.alloc(n_siblings));
    e->alloc_depth = std::min(e->alloc_depth, 0);
    LevelState lsh{};
    lsh.n_pairs = (int32_t)n_siblings;
    HB_CK(e, cudaMemcpyAsync(e->pairs.p, tr.data(), sizeof(Triple) * n_siblings, cudaMemcpyHostToDevice, s));
    HB_CK(e, cudaMemcpyAsync(e->ls.p, &lsh, sizeof(LevelState), cudaMemcpyHostToDevice, s));
    launch_subtract(e->pairs.p, e->ls.p, (int)n_siblings, tb, e->resident.p, s);
  }
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaStreamSynchronize(s));
  return HB_OK;
}

hb_status hb_scan_resident(hb_engine* e, const hb_reg_params* reg, const hb_scan_request* req,
                           uint32_t n, hb_node_scan* out) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  if (!reg || ((!req || !out) && n)) return HB_INVALID_ARGUMENT;
  if (!n) return HB_OK;
  DevConst c = e->c;
  c.lambda = reg->lambda;
  c.alpha = reg->alpha;
  c.mds = reg->max_delta_step;
  c.mcw = reg->min_child_weight;
  c.mono = nullptr;  // the requests' own directions apply
  cudaStream_t s = e->stream;
  Scale h;
  HB_CK(e, cudaMemcpyAsync(&h, e->scale.p, sizeof(Scale), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  // every request is checked before any launch
  std::vector<Front> fr(n);
  std::vector<int8_t> dirs((size_t)n * c.n_cols, 0);
  for (uint32_t k = 0; k < n; ++k) {
    const hb_scan_request& q = req[k];
    if (q.slot >= e->resident_slots) return refuse(e, "slot not reserved");
    if (q.n_features && !q.features) return HB_INVALID_ARGUMENT;
    for (uint32_t j = 0; j < q.n_features; ++j) {
      const uint32_t f = q.features[j];
      if (f >= c.n_cols) return HB_INVALID_ARGUMENT;
      const int8_t d = q.directions ? q.directions[j] : 0;
      if (d < -1 || d > 1) return refuse(e, "a monotone direction must be -1, 0 or 1");
      dirs[(size_t)k * c.n_cols + f] = d;
    }
    fr[k].slot = (int32_t)q.slot;
    fr[k].g = std::llrint(std::ldexp(q.total.grad, h.sg));
    fr[k].h = std::llrint(std::ldexp(q.total.hess, h.sh));
    fr[k].lower = (double)q.lower;
    fr[k].upper = (double)q.upper;
    fr[k].root_gain = q.root_gain;
    fr[k].root_gain_given = 1;
  }
  HB_CK(e, e->front[0].alloc(n));
  HB_CK(e, e->cand.alloc((size_t)n * c.n_cols));
  HB_CK(e, e->scan_dirs.alloc(dirs.size()));
  e->alloc_depth = -1;
  LevelState lsh{};
  HB_CK(e, cudaMemcpyAsync(e->front[0].p, fr.data(), sizeof(Front) * n, cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaMemcpyAsync(e->scan_dirs.p, dirs.data(), dirs.size(), cudaMemcpyHostToDevice, s));
  for (uint32_t k0 = 0; k0 < n; k0 += 65535) {  // grid.y holds at most 65,535 nodes
    const uint32_t m = std::min<uint32_t>(65535u, n - k0);
    lsh.n_front = (int32_t)m;
    HB_CK(e, cudaMemcpyAsync(e->ls.p, &lsh, sizeof(LevelState), cudaMemcpyHostToDevice, s));
    launch_scan(c, e->fo.p, e->resident.p, e->front[0].p + k0, e->ls.p, nullptr, 0, e->scale.p,
                (int)m, e->cand.p + (size_t)k0 * c.n_cols, s, e->scan_dirs.p + (size_t)k0 * c.n_cols);
    // the level state is read by the launch before the next chunk's copy
    HB_CK(e, cudaStreamSynchronize(s));
  }
  HB_CK(e, cudaGetLastError());
  std::vector<Cand> cd((size_t)n * c.n_cols);
  HB_CK(e, cudaMemcpyAsync(cd.data(), e->cand.p, sizeof(Cand) * cd.size(), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  const double ig = std::ldexp(1.0, -h.sg), ih = std::ldexp(1.0, -h.sh);
  for (uint32_t k = 0; k < n; ++k) {
    // the features' winners merged in the request's order from the empty
    // split (merge_scans, cuda-kernels/src/categorical.rs:637): a finite
    // loss replaces the incumbent when larger, or, from a lower feature,
    // when not smaller (need_replace, src/tree/builder/mod.rs:313)
    float best = 0.0f;
    uint32_t best_feature = 0;
    int chosen = -1;
    for (uint32_t j = 0; j < req[k].n_features; ++j) {
      const uint32_t f = req[k].features[j];
      const float loss = cd[(size_t)k * c.n_cols + f].loss;
      if (std::isinf(loss) || std::isnan(loss)) continue;
      const bool replace = best_feature <= f ? loss > best : !(best > loss);
      if (replace) {
        best = loss;
        best_feature = f;
        chosen = (int)f;
      }
    }
    hb_node_scan& o = out[k];
    std::memset(&o, 0, sizeof(o));
    if (chosen < 0) {
      o.kind = HB_SCAN_EMPTY;
      continue;
    }
    const Cand& x = cd[(size_t)k * c.n_cols + chosen];
    const uint32_t fs = e->h_fo[chosen];
    o.kind = HB_SCAN_NUMERIC;
    o.feature = (uint32_t)chosen;
    o.loss_chg = x.loss;
    o.backward = x.default_left ? 1 : 0;
    if (!x.default_left) {
      o.offset = (uint32_t)(x.bin - (int)fs);
      o.acc.grad = (double)x.lg * ig;
      o.acc.hess = (double)x.lh * ih;
    } else {
      o.offset = x.bin < 0 ? 0 : (uint32_t)(x.bin - (int)fs + 1);
      o.acc.grad = (double)(fr[k].g - x.lg) * ig;
      o.acc.hess = (double)(fr[k].h - x.lh) * ih;
    }
  }
  return HB_OK;
}

hb_status hb_read_hist(hb_engine* e, uint32_t slot, hb_grad_stats* out) {
  HB_ENTER(e);
  if (slot >= e->resident_slots || !out) return HB_INVALID_ARGUMENT;
  return download_hist(e, e->resident.p + (size_t)slot * e->c.total_bins, 1, out);
}

hb_status hb_read_gradients(hb_engine* e, hb_grad_pair* out, uint64_t n, int32_t* sg, int32_t* sh) {
  HB_ENTER(e);
  if (!e->uploaded || !e->staged) return refuse(e, "no staged gradients");
  if (!out || n != e->c.n_rows || !sg || !sh) return HB_INVALID_ARGUMENT;
  Scale h;
  HB_CK(e, cudaMemcpyAsync(out, e->gpair.p, 8 * n, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaMemcpyAsync(&h, e->scale.p, sizeof(Scale), cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  *sg = h.sg;
  *sh = h.sh;
  return HB_OK;
}

// ---- whole-tree growth -------------------------------------------------------
hb_status hb_grow_tree(hb_engine* e, const hb_train_params* p, hb_tree_node* nodes,
                       uint32_t nodes_cap, uint32_t* n_nodes) {
  HB_ENTER(e);
  hb_status st = check_params(e, p);
  if (st != HB_OK) return st;
  if (!e->uploaded || !e->staged || !e->margins_loaded) return refuse(e, "no staged gradients or margins");
  if (!nodes || !n_nodes) return HB_INVALID_ARGUMENT;
  st = grow_tree_device(e, p, false);
  if (st != HB_OK) return st;
  const int walk_ls = e->walk_ls;
  st = flush_pending(e);
  if (st != HB_OK) return st;
  LevelState last;
  HB_CK(e, cudaMemcpyAsync(&last, e->ls.p + walk_ls, sizeof(LevelState), cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  if ((uint32_t)last.n_nodes > nodes_cap) return refuse(e, "nodes_cap too small");
  HB_CK(e, cudaMemcpyAsync(nodes, e->tree.p, sizeof(hb_tree_node) * last.n_nodes, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  *n_nodes = (uint32_t)last.n_nodes;
  e->staged = false;
  return HB_OK;
}

// One boosting round (gradients, with the previous tree's leaves, and a
// tree) as stream work.
static hb_status round_work(hb_engine* e, const hb_train_params* p) {
  if (p->objective == HB_LOSS_SOFTMAX) {
    // every class's gradients from the round's margins (round.rs:253), then
    // one tree per class in class order (round.rs:318)
    cudaStream_t s = e->stream;
    HB_CK(e, cudaMemsetAsync(e->scale.p, 0, sizeof(Scale) * e->n_out, s));
    mark_begin(e, T_GRAD);
    if (e->c.csr) {  // the pending trees' walks over CSR rows first
      launch_walk_csr(e->c, e->n_out, e->wtree.p, (uint32_t)e->wstride, e->margin.p, e->flags.p, e->n_sm, s);
      e->kernel_launches += 1;
    }
    launch_softmax_gradients(e->n_out, e->margin.p, e->label.p, e->c.n_rows,
                             softmax_vector_rows(e, e->n_out), 1e-16f, e->gpair.p,
                             e->scale.p, e->wtree.p, (uint32_t)e->wstride, e->rec.p, e->c.stride,
                             e->c.mask_off, e->c.blk, e->c.csr ? nullptr : e->flags.p, e->n_sm, s);
    e->blk_pairs = false;
    mark_end(e);
    HB_CK(e, cudaGetLastError());
    e->pending_tree = false;
    e->kernel_launches += 1;
    for (int k = 0; k < e->n_out; ++k) {
      e->cls = k;
      hb_status st = finish_scale(e);
      if (st == HB_OK) st = grow_tree_device(e, p, true);
      if (st != HB_OK) {
        e->cls = 0;
        return st;
      }
      e->kernel_launches += 1;  // scale
    }
    e->cls = 0;
    e->staged = true;
    return HB_OK;
  }
  int wl = 0, wn = 0, wd = 0;
  walk_shape(p, wl, wn, wd);
  hb_status st = run_gradients(e, p->objective, p->scale_pos_weight, 1e-16f, wl, wn, wd);
  if (st != HB_OK) return st;
  return grow_tree_device(e, p, true);
}

// Rounds as CUDA graphs: the kernels of a round are captured once and the
// graph replayed, so no launch gaps separate them. With timing on, all the
// rounds are captured into one graph, each kernel family bracketed by event
// nodes, so the per-kernel times come from the same run.
static hb_status graph_rounds(hb_engine* e, const hb_train_params* p, int rounds) {
  cudaStream_t s = e->stream;
  auto capture = [&](int n, cudaGraphExec_t* exec) -> hb_status {
    HB_CK(e, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    e->capturing = true;
    hb_status st = HB_OK;
    for (int r = 0; r < n && st == HB_OK; ++r) st = round_work(e, p);
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamEndCapture(s, &g);
    e->capturing = false;
    if (st != HB_OK) {
      if (g) cudaGraphDestroy(g);
      return st;
    }
    if (ce != cudaSuccess) return fail(e, "cudaStreamEndCapture", ce);
    ce = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(e, "cudaGraphInstantiate", ce);
    return HB_OK;
  };
  if (e->timing) {
    // enough events for every mark of every round, created before capture
    // (two events a mark; a lossguide tree marks four families a step)
    const size_t per_tree = p->grow_policy == HB_GROW_LOSSGUIDE ? 8 * (size_t)lg_leaves(p) + 32 : 64;
    const size_t need = e->ev_used + (size_t)rounds * per_tree * std::max(e->n_out, 1) + 64;
    while (e->ev.size() < need) {
      cudaEvent_t x;
      HB_CK(e, cudaEventCreate(&x));
      e->ev.push_back(x);
      e->ev_kind.push_back(0);
    }
    cudaGraphExec_t exec = nullptr;
    hb_status st = capture(rounds, &exec);
    if (st != HB_OK) return st;
    HB_CK(e, cudaEventRecord(e->run_ev[0], s));
    cudaError_t ce = cudaGraphLaunch(exec, s);
    if (ce == cudaSuccess) ce = cudaEventRecord(e->run_ev[1], s);
    cudaError_t ce2 = cudaStreamSynchronize(s);
    cudaGraphExecDestroy(exec);
    if (ce != cudaSuccess) return fail(e, "cudaGraphLaunch", ce);
    if (ce2 != cudaSuccess) return fail(e, "cudaStreamSynchronize", ce2);
    return HB_OK;
  }
  // the round graph depends on the parameters, the communicator and every
  // buffer it touches (a buffer that grew has moved)
  const void* ptrs[] = {e->comm, e->rec.p, e->col.p, e->colmiss.p, e->fo.p, e->cuts.p,
                        e->gpair.p, e->margin.p, e->label.p, e->weight.p, e->rows[0],
                        e->rows[1], e->scale.p, e->hist_all.p, e->front[0].p, e->front[1].p,
                        e->cand.p, e->dec.p, e->items.p, e->dirbits.p, e->item_left.p,
                        e->item_off.p, e->entries.p, e->pairs.p, e->ls.p, e->tree.p,
                        e->wtree.p, e->forest.p, e->counts.p, e->tree_counter.p,
                        e->row_stats.p, e->flags.p, e->lg_heap.p, e->lg_pool.p, e->lg_state.p,
                        e->lg_depth.p, e->csr_ptr.p, e->csr_bins.p, e->fill.p, e->best_key.p};
  const int weighted = e->weight_key ? 1 : 0;
  std::vector<unsigned char> key(sizeof(hb_train_params) + sizeof(ptrs) + sizeof(int) * 2);
  std::memcpy(key.data(), p, sizeof(hb_train_params));
  std::memcpy(key.data() + sizeof(hb_train_params), ptrs, sizeof(ptrs));
  std::memcpy(key.data() + sizeof(hb_train_params) + sizeof(ptrs), &weighted, sizeof(int));
  std::memcpy(key.data() + sizeof(hb_train_params) + sizeof(ptrs) + sizeof(int), &e->max_items,
              sizeof(int));
  key.push_back((unsigned char)e->n_out);
  if (!e->round_exec || key != e->round_key) {
    if (e->round_exec) cudaGraphExecDestroy(e->round_exec);
    e->round_exec = nullptr;
    const uint64_t l0 = e->kernel_launches, r0 = e->rounds_done;
    hb_status st = capture(1, &e->round_exec);
    if (st != HB_OK) return st;
    e->round_launches = e->kernel_launches - l0;
    e->kernel_launches = l0;
    e->rounds_done = r0;
    e->round_key = key;
  }
  HB_CK(e, cudaEventRecord(e->run_ev[0], s));
  for (int r = 0; r < rounds; ++r) {
    HB_CK(e, cudaGraphLaunch(e->round_exec, s));
    e->kernel_launches += e->round_launches;
    e->rounds_done += 1;
  }
  HB_CK(e, cudaEventRecord(e->run_ev[1], s));
  e->pending_tree = true;
  walk_shape(p, e->walk_ls, e->walk_nodes, e->walk_depth);
  return HB_OK;
}

hb_status hb_train_begin(hb_engine* e, const float* labels, uint64_t n, float base_margin) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if (!labels || n != e->c.n_rows) return HB_INVALID_ARGUMENT;
  if (e->row_begin % 8) return refuse(e, "shards must start on a multiple of 8 rows");
  cudaStream_t s = e->stream;
  e->n_out = 1;
  launch_fill(e->margin.p, base_margin, n, e->n_sm, s);  // every margin starts at the base
  HB_CK(e, cudaGetLastError());
  e->margins_loaded = true;
  e->pending_tree = false;
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0, sizeof(int), s));
  e->label_key = nullptr;
  hb_status st = stage_labels(e, labels, nullptr, n);
  if (st != HB_OK) return st;
  HB_CK(e, cudaStreamSynchronize(s));
  e->train_begun = true;
  return HB_OK;
}

hb_status hb_train_begin_classes(hb_engine* e, const float* labels, uint64_t n,
                                 const float* base_margins, int32_t n_classes) {
  HB_ENTER(e);
  if (!e->uploaded) return refuse(e, "no index uploaded");
  if (!labels || !base_margins || n != e->c.n_rows || n_classes < 1 || n_classes > 64)
    return HB_INVALID_ARGUMENT;
  if (e->row_begin % 8) return refuse(e, "shards must start on a multiple of 8 rows");
  for (uint64_t i = 0; i < n; ++i) {
    const float y = labels[i];
    if (!(y >= 0.0f) || y >= (float)n_classes || y != std::floor(y))
      return refuse(e, "labels must be class ids in [0, n_classes)");
  }
  cudaStream_t s = e->stream;
  const size_t kn = (size_t)n_classes * n;
  HB_CK(e, e->margin.alloc(kn));
  HB_CK(e, e->gpair.alloc(kn));
  HB_CK(e, e->scale.alloc(n_classes));
  for (int k = 0; k < n_classes; ++k) launch_fill(e->margin.p + (size_t)k * n, base_margins[k], n, e->n_sm, s);
  HB_CK(e, cudaGetLastError());
  HB_CK(e, cudaMemcpyAsync(e->label.p, labels, 4 * n, cudaMemcpyHostToDevice, s));
  HB_CK(e, cudaStreamSynchronize(s));
  e->label_key = nullptr;
  e->weight_key = nullptr;
  e->n_out = n_classes;
  e->margins_loaded = true;
  e->pending_tree = false;
  HB_CK(e, cudaMemsetAsync(e->flags.p, 0, sizeof(int), s));
  HB_CK(e, cudaStreamSynchronize(s));
  e->train_begun = true;
  return HB_OK;
}

hb_status hb_train_rounds(hb_engine* e, const hb_train_params* p, int32_t rounds,
                          hb_tree_node* nodes, uint64_t nodes_cap, uint64_t* tree_ptr) {
  HB_ENTER(e);
  hb_status st = check_params(e, p);
  if (st != HB_OK) return st;
  if (!e->train_begun || !e->margins_loaded) return refuse(e, "no training run (hb_train_begin)");
  if (rounds < 0 || !tree_ptr || (!nodes && rounds)) return HB_INVALID_ARGUMENT;
  cudaStream_t s = e->stream;
  const uint32_t max_nodes = tree_slots(p);
  const int trees = rounds * e->n_out;  // one tree per class and round
  HB_CK(e, e->forest.alloc(std::max<size_t>((size_t)trees * max_nodes, 1)));
  HB_CK(e, e->counts.alloc(std::max(trees, 1)));
  HB_CK(e, cudaMemsetAsync(e->tree_counter.p, 0, 4, s));
  if (e->use_graphs && rounds > 0) {
    st = ensure_buffers(e, p);
    if (st == HB_OK) st = ensure_peers(e);
    if (st != HB_OK) return st;
    st = graph_rounds(e, p, rounds);
    if (st != HB_OK) return st;
  } else {
    st = ensure_buffers(e, p);
    if (st == HB_OK && rounds > 0) st = ensure_peers(e);
    if (st != HB_OK) return st;
    HB_CK(e, cudaEventRecord(e->run_ev[0], s));
    for (int r = 0; r < rounds; ++r) {
      st = round_work(e, p);
      if (st != HB_OK) return st;
      if (e->timing && e->ev_used + 128 > e->ev.size()) collect_timers(e);
    }
    HB_CK(e, cudaEventRecord(e->run_ev[1], s));
  }
  st = flush_pending(e);
  if (st != HB_OK) return st;
  std::vector<uint32_t> cnt(std::max(trees, 1));
  HB_CK(e, cudaMemcpyAsync(cnt.data(), e->counts.p, 4 * (size_t)std::max(trees, 1), cudaMemcpyDeviceToHost, s));
  HB_CK(e, cudaStreamSynchronize(s));
  st = check_peers(e);
  if (st != HB_OK) return st;
  collect_timers(e);
  {
    float ms = 0.0f;
    e->last_rounds_ms = (rounds > 0 && cudaEventElapsedTime(&ms, e->run_ev[0], e->run_ev[1]) == cudaSuccess) ? ms : 0.0;
  }
  uint64_t used = 0;
  tree_ptr[0] = 0;
  for (int r = 0; r < trees; ++r) {
    used += cnt[r];
    tree_ptr[r + 1] = used;
  }
  if (used > nodes_cap) return refuse(e, "nodes_cap too small");
  for (int r = 0; r < trees; ++r) {
    HB_CK(e, cudaMemcpyAsync(nodes + tree_ptr[r], e->forest.p + (size_t)r * max_nodes,
                             sizeof(hb_tree_node) * cnt[r], cudaMemcpyDeviceToHost, s));
  }
  HB_CK(e, cudaStreamSynchronize(s));
  e->staged = false;
  return HB_OK;
}

hb_status hb_train(hb_engine* e, const hb_train_params* p, const float* labels, uint64_t n,
                   float base_margin, int32_t rounds, hb_tree_node* nodes, uint64_t nodes_cap,
                   uint64_t* tree_ptr) {
  HB_ENTER(e);
  hb_status st = check_params(e, p);
  if (st != HB_OK) return st;
  st = hb_train_begin(e, labels, n, base_margin);
  if (st != HB_OK) return st;
  return hb_train_rounds(e, p, rounds, nodes, nodes_cap, tree_ptr);
}

hb_status hb_engine_inject_fault(hb_engine* e, int32_t after_calls) {
  if (!e) return HB_INVALID_ARGUMENT;
  if (after_calls < -1) return HB_INVALID_ARGUMENT;
  e->fault_after = after_calls;
  return HB_OK;
}

hb_status hb_engine_reset_stats(hb_engine* e, int32_t timing) {
  HB_ENTER(e);
  for (int k = 0; k < kTimers; ++k) {
    e->timer_ms[k] = 0.0;
    e->timer_launches[k] = 0;
  }
  e->ev_used = 0;
  e->kernel_launches = 0;
  e->rounds_done = 0;
  // 1: events around the histogram launches only; 2: around every family
  e->timing = timing != 0;
  e->timing_mask = timing >= 2 ? 0xffu : ((1u << T_ROOT) | (1u << T_HIST));
  HB_CK(e, cudaMemsetAsync(e->row_stats.p, 0, 16, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  return HB_OK;
}

hb_status hb_engine_get_stats(hb_engine* e, hb_engine_stats* out) {
  HB_ENTER(e);
  if (!out) return HB_INVALID_ARGUMENT;
  collect_timers(e);
  unsigned long long rs[2];
  HB_CK(e, cudaMemcpyAsync(rs, e->row_stats.p, 16, cudaMemcpyDeviceToHost, e->stream));
  HB_CK(e, cudaStreamSynchronize(e->stream));
  for (int k = 0; k < kTimers; ++k) {
    out->ms[k] = e->timer_ms[k];
    out->timed_launches[k] = e->timer_launches[k];
  }
  out->kernel_launches = e->kernel_launches;
  out->rows_built_contiguous = rs[0];
  out->rows_built_gathered = rs[1];
  out->rounds = e->rounds_done;
  out->last_rounds_ms = e->last_rounds_ms;
  return HB_OK;
}

hb_status hb_engine_stream(hb_engine* e, void** stream) {
  HB_ENTER(e);
  if (!stream) return HB_INVALID_ARGUMENT;
  *stream = (void*)e->stream;
  return HB_OK;
}

// ---- sharding -------------------------------------------------------------
hb_status hb_comm_unique_id(uint8_t id[128]) {
  if (!id) return HB_INVALID_ARGUMENT;
  ncclUniqueId u;
  if (ncclGetUniqueId(&u) != ncclSuccess) return HB_DEVICE_FAILED;
  std::memcpy(id, u.internal, 128);
  return HB_OK;
}

hb_status hb_comm_init(hb_engine* e, int32_t nranks, int32_t rank, const uint8_t id[128],
                       uint64_t global_rows) {
  HB_ENTER(e);
  if (!id || nranks < 1 || rank < 0 || rank >= nranks) return HB_INVALID_ARGUMENT;
  ncclUniqueId u;
  std::memcpy(u.internal, id, 128);
  if (e->comm) {
    HB_CK(e, cudaStreamSynchronize(e->stream));
    if (e->round_exec) cudaGraphExecDestroy(e->round_exec);  // captured with the old communicator
    e->round_exec = nullptr;
    close_peers(e);
    ncclCommDestroy(e->comm);
    e->comm = nullptr;
  }
  HB_NCCL(e, ncclCommInitRank(&e->comm, nranks, u, rank));
  e->nranks = nranks;
  e->rank = rank;
  e->shard_global = global_rows;
  e->c.global_rows = global_rows;
  return HB_OK;
}

}  // extern "C"

extern "C" hb_status hb_engine_set_shard(hb_engine* e, uint64_t row_begin, uint64_t global_rows) {
  HB_ENTER(e);
  if (row_begin % 8) return refuse(e, "shards must start on a multiple of 8 rows");
  e->row_begin = row_begin;
  e->shard_global = global_rows;
  e->c.global_rows = global_rows;
  return HB_OK;
}

// ---- engine view for entry points in other files --------------------------
namespace hb {

void engine_view(const hb_engine* e, EngineView* v) {
  v->device = e->device;
  v->stream = e->stream;
  v->n_sm = e->n_sm;
  v->failed = e->failed;
  v->uploaded = e->uploaded;
  v->staged = e->staged;
  v->c = &e->c;
  v->fo = e->fo.p;
  v->rec = e->rec.p;
  v->gpair = e->gpair.p;
  v->scale = e->scale.p;
}

hb_status engine_fail(hb_engine* e, const char* what, cudaError_t code) { return fail(e, what, code); }

hb_status engine_refuse(hb_engine* e, const char* why) { return refuse(e, why); }

hb_status engine_invalid(hb_engine* e, const char* why) {
  refuse(e, why);
  return HB_INVALID_ARGUMENT;
}

}  // namespace hb
