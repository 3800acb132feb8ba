// Internal declarations shared by the engine (host) and the kernels.
//
// Data layout in HBM (one engine = one GPU = one shard of rows):
//   rec      row-major records: the feature-local bins (one byte per
//            feature) followed by the missing mask (one bit per feature, u32
//            words at mask_off), `stride` bytes a row; what the histogram
//            kernels gather by row. Records of at most 48 bytes sit in row
//            blocks: 128-byte lines of blk records and then those rows'
//            (g, h) pairs (rec_offset, pair_offset)
//   col      [n_cols][n_rows] u8   feature-major bins: what the partition
//                                  reads for the split feature
//   colmiss  [n_cols][words] u64   missing bitmap, feature-major
//   gpair    [n_rows] float2       this tree's (g, h)
//   margin   [n_rows] f32, label [n_rows] f32
//   rows[2]  [n_rows] u32          row ids, one segment per node: the two
//                                  halves of one 2n buffer (depthwise levels
//                                  ping-pong; lossguide moves a node's
//                                  children to the other half)
//   hist     [slots][total_bins] longlong2 (fixed-point g, h), level-major
//            slot layout: level L owns slots [2^L - 1, 2^(L+1) - 1); within
//            a level the built children come first, their siblings second
#pragma once

#include <cstddef>
#include <cstdint>

#include "../../include/hb_backend.h"

namespace hb {

constexpr int kMaxDepth = 10;            // device growth supports depth <= 10
constexpr int kMaxFront = 1 << kMaxDepth;
constexpr int kTile = 2048;              // partition tile (rows per CTA)
constexpr int kTileWords = kTile / 32;
constexpr int kHistThreads = 1024;
constexpr int kGroupFeatures = 32;       // features per histogram CTA group
constexpr uint32_t kMaxRecordFeatures = 224;  // widest dense index kept as row records

// Fixed-point range: every |q| * rows <= 2^kFixedTop, so each sum is an
// integer below 2^53, exact in an f64.
constexpr int kFixedTop = 53;

// Per-tree scale of the fixed-point gradients: q = rint(v * 2^s).
struct Scale {
  int32_t sg, sh;
  double fg, fh;      // 2^sg, 2^sh
  double ig, ih;      // 2^-sg, 2^-sh
  uint32_t maxg_bits, maxh_bits;  // largest |g|, |h| (f32 bits)
  uint32_t nonfinite;
  uint32_t pad;
};

// Constants of the binned matrix and of the training run.
struct DevConst {
  uint64_t n_rows;        // rows on this device
  uint64_t global_rows;   // rows over every rank (fixed-point scale)
  uint32_t n_cols;
  uint32_t total_bins;
  uint32_t max_bins;      // largest per-feature bin count
  uint32_t stride;        // record bytes
  uint32_t mask_off;      // byte offset of the mask words in a record
  // Row blocks (blk = 2, 3 or 5): each 128-byte line of the record array
  // holds blk records and then those rows' (g, h) pairs, so a gathered row
  // costs one line; blk = 0: records `stride` bytes apart, pairs elsewhere.
  uint32_t blk;
  uint32_t blk_pair;      // byte offset of a line's pairs (blk * stride)
  uint32_t dense;         // index-level: no missing cell anywhere
  uint32_t n_groups;      // feature groups of kGroupFeatures
  uint32_t hist64;        // 1: always the 64-bit-atomic histogram kernel
  uint32_t scan_cta;      // 1: always the CTA-per-feature split scan
  // CSR index (csr = 1): each row's global bins ascending, absent = missing;
  // fo = the device copy of feature_offset (both layouts)
  uint32_t csr;
  const uint64_t* csr_ptr;
  const uint32_t* csr_bins;
  // CSR index also held feature-major (NULL when not built): each cell's
  // local bin (u8) at [f * n_rows + r] and the missing bitmap (absent cells
  // set, NULL when every cell is present) at [f * words + r / 64]
  const uint8_t* csr_col;
  const uint64_t* csr_colmiss;
  const uint32_t* fo;
  // training parameters (RegParams rounded to f32 then widened)
  double lambda, alpha, gamma, mcw, mds;
  float eta;
  int32_t max_depth;
  // monotone direction per feature (+1, -1, 0; constraints.rs:12), device
  // memory, or NULL when no feature is constrained
  const int8_t* mono;
};

constexpr uint32_t kBlockBytes = 128;


// Rows per 128-byte block for a record width: records and their 8-byte pairs
// must fit one line, at least two rows to it.
inline uint32_t block_rows(uint32_t stride) {
  return stride == 16 ? 5u : stride == 32 ? 3u : stride == 48 ? 2u : 0u;
}

// Byte offset of row r's record, and of its (g, h) pair inside the row
// blocks (blk != 0).
__host__ __device__ __forceinline__ uint32_t block_of(uint32_t r, uint32_t blk) {
  return blk == 3u ? r / 3u : blk == 2u ? r >> 1 : r / 5u;
}
__host__ __device__ __forceinline__ uint64_t rec_offset(uint32_t r, uint32_t stride, uint32_t blk) {
  if (!blk) return (uint64_t)r * stride;
  const uint32_t q = block_of(r, blk);
  return (uint64_t)q * kBlockBytes + (r - q * blk) * stride;
}
__host__ __device__ __forceinline__ uint64_t pair_offset(uint32_t r, uint32_t blk, uint32_t blk_pair) {
  const uint32_t q = block_of(r, blk);
  return (uint64_t)q * kBlockBytes + blk_pair + (r - q * blk) * 8u;
}
// Bytes of the record array for n rows (64 spare bytes for vector reads).
inline uint64_t rec_bytes(uint64_t n, uint32_t stride, uint32_t blk) {
  return (blk ? (n + blk - 1) / blk * kBlockBytes : n * stride) + 64;
}

// Peer-memory histogram exchange (hb_peer.cu): every rank's histogram
// buffer and barrier block, mapped into this rank's address space. A
// barrier block holds the arrive flags [kPeerMax], the depart flags
// [kPeerMax] (one per rank, raised to the launch's epoch by that rank),
// then the epoch of the last completed launch, a count of finished CTAs
// and a sticky status word (nonzero: a wait timed out).
constexpr int kPeerMax = 8;
constexpr int kPeerThreads = 256;
constexpr int kPeerArrive = 0, kPeerDepart = 1;
constexpr int kPeerEpoch = 2 * kPeerMax, kPeerCount = kPeerEpoch + 1, kPeerStatus = kPeerEpoch + 2;
constexpr int kPeerWords = kPeerEpoch + 8;
struct PeerSet {
  longlong2* hist[kPeerMax];
  unsigned long long* bar[kPeerMax];
  int n, rank;
  uint64_t timeout_ns;
};

// One frontier entry of the level being grown. The first 32 bytes are read
// as two int4 by the histogram plan (load_front_cg), so every entry of a
// Front array starts on a 16-byte boundary: 16-byte alignment, a size that is
// a multiple of 16.
struct alignas(16) Front {
  int32_t node;       // tree node id
  int32_t slot;       // histogram slot (or -1)
  uint32_t begin;     // segment in the current row buffer
  uint32_t len;
  long long g, h;     // node statistics (fixed point)
  // the node's monotone weight bounds (constraints.rs:44 `Bounds`)
  double lower = -__builtin_huge_val(), upper = __builtin_huge_val();
  float root_gain = 0.0f;       // the caller's root gain (RowEngine scans) ...
  int32_t root_gain_given = 0;  // ... used when set, else computed
};
static_assert(sizeof(Front) % 16 == 0 && alignof(Front) == 16, "Front entries must be 16-byte aligned");

// The best candidate of one (node, feature) pair.
struct Cand {
  float loss;         // -inf: none
  int32_t bin;        // last global bin going left, -1 = below every bin
  int32_t default_left;
  int32_t pad;
  long long lg, lh;   // left child statistics
};

// Decision for one frontier node of the level.
struct Decision {
  int32_t split;      // 1: splits, 0: becomes a leaf
  int32_t pair;       // index among the level's splits
  uint32_t feature;
  uint32_t limit;     // local bins below it go left
  int32_t default_left;
  float leaf_value;   // eta-scaled leaf value when it becomes a leaf
  int32_t item_begin; // first partition work item
  int32_t item_count;
  long long lg, lh;   // left child stats
};

// A partition work item: a tile of one frontier node's segment.
struct PItem {
  int32_t k;          // frontier index
  int32_t kind;       // 1 split, 2 leaf margin add
  uint32_t off;       // tile offset within the segment
  uint32_t len;
};

// One histogram build entry: rows [begin, begin + len) of the row buffer
// into slot `slot`; `prefix` = rows of the entries before it.
struct HEntry {
  int32_t slot;
  int32_t identity;   // rows are the positions themselves
  uint32_t begin;
  uint32_t len;
  uint64_t prefix;
};

// Level bookkeeping written by the device, read by the next kernels.
struct LevelState {
  int32_t n_front;        // frontier entries at this level
  int32_t n_items;        // partition work items
  int32_t n_split;        // splitting nodes
  int32_t n_nodes;        // tree nodes so far
  int32_t n_hentries;     // histogram entries
  int32_t n_pairs;        // sibling subtractions
  uint64_t hist_rows;     // rows to build this level
  int32_t tree_index;     // slot in the forest buffer
  uint32_t done_ctas;     // CTAs of the level's tile scan that have finished
};

// The grown tree as the margin update walks it: a row at a node goes left
// when its feature-local bin is below `limit`, or, missing, when bit 31 of
// `feature` (default_left) is set; the same rule as the partition.
struct WNode {
  int32_t left;       // first child (right = left + 1); -1 for a leaf
  uint32_t feature;   // split feature | default_left << 31
  uint32_t limit;
  float leaf;         // eta-scaled leaf value of a leaf
};

struct Triple {
  int32_t parent, built, sibling, pad;
};

// Lossguide growth (src/tree/builder/hist/mod.rs:505): a node waiting in
// the max-heap with its best split, keyed by the f64::total_cmp order of
// that split's loss change.
struct LgNode {
  long long key;      // total-order key of (double)loss
  int32_t nid, depth;
  uint32_t begin, len;  // its rows in the row buffer
  long long g, h;     // its statistics (fixed point)
  float loss;         // best split: loss change (0: none found)
  int32_t feature;    // -1: none
  int32_t bin;        // last global bin going left, -1 = below every bin
  int32_t default_left;
  long long lg, lh;   // that split's left child statistics
  double lower, upper;  // the node's monotone weight bounds
};

// A lossguide heap entry: the node's key and its id (the node's LgNode is
// kept at that id in a per-tree pool). The heap moves these 16 bytes, its
// comparisons are of the key alone, so it pops in the same order as a heap
// of whole nodes.
struct LgKey {
  long long key;
  int32_t nid;
  int32_t pad;
};

struct LgState {
  int32_t heap_n;     // nodes in the heap
  int32_t n_nodes;    // tree nodes so far
  int32_t n_leaves;   // leaves of the growing tree (a node counts until expanded)
  int32_t done;       // growth finished: every later step does nothing
  int32_t n_pending;  // children (in `next`) whose scan awaits merging
  int32_t pad[3];
};

}  // namespace hb
