// Quantile sketch and binning on the device: the reference's
// HistCuts::from_dmatrix (src/data/quantile.rs:65, the streaming ingest of
// quantile.rs:115 `build` with unit weights) and GHistIndex::from_dmatrix
// (src/data/ghist.rs:213), producing the same cut values bit for bit.
//
// The reference streams each feature's present values, in row order, into
// XGBoost's WQSketch (src/data/sketch.rs:477 `push`): consecutive equal
// values fold into one queue entry; a full queue (2 * limit entries) is
// sorted, summarised (`set_from_sorted` :88) and pushed into a ladder of
// levels (`push_summary` :575: prune to `limit`, combine with the level,
// carry upward while the result exceeds `limit`); the final summary combines
// the levels (`summary` :607) and is queried for the cuts (`query_cut_values`
// :427). Every step but the ladder is independent of the others once the
// queue boundaries are known, and those depend only on the stream:
//
//   1. extract   each feature's present values in row order into one stream
//                (dense: a per-tile compaction; CSR: a stable radix sort of
//                the stored cells by column);
//   2. entries   mark where a value differs from its predecessor: the queue
//                entries, whose weights are run lengths; queue flush k of a
//                feature holds its entries [k * 2 * limit, (k + 1) * 2 * limit);
//   3. chunks    one CTA per flush: radix sort, fold equal values, prune to
//                `limit` (the first step of `push_summary`), all in shared
//                memory, for every flush of every feature at once;
//   4. ladder    one CTA per feature replays `push_summary` over its pruned
//                flushes in order and the final `summary` + query, with
//                block-parallel merges (merge path by binary search, FixError
//                as two prefix maxima) and prunes (each rank query answered
//                by binary search, the sequential cursor recovered as a
//                prefix maximum);
//   5. bin       bin = #{cuts <= v}, clamped to the last bin.
//
// Exactness: with unit weights every weight and rank below 2^24 is a whole
// number, exact in f32, so the sums of step 3 may be formed in any order;
// every other f32/f64 operation is the reference's own, one for one, on the
// same operands (the library is built without FMA contraction). Features
// with 2^24 or more present values are refused (the reference changes sort
// there) and so are sample weights: the host path (hb_cuts_dense) takes them.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "hb_sketch.h"

namespace hb {
namespace {

// WQSummary::Entry (sketch.rs:27).
struct SEntry {
  float rmin, rmax, wmin, value;
};

constexpr int kTileRows = 256;      // rows per extraction / binning CTA
constexpr int kChunkThreads = 512;  // flush CTAs
constexpr int kLadderThreads = 1024;
constexpr uint32_t kMaxLevels = 40;

// Monotone u32 key of an f32 (src/data/sort.rs `sort_key`).
__device__ __forceinline__ uint32_t sort_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unsort_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <class V>
struct MaxOp {
  __device__ __forceinline__ V operator()(const V& a, const V& b) const { return a < b ? b : a; }
};
struct SumU32 {
  __device__ __forceinline__ uint32_t operator()(uint32_t a, uint32_t b) const { return a + b; }
};

// Block-wide scan of an array of `len` items: each thread takes a contiguous
// run, the runs' aggregates are scanned, then put(i, exclusive, value) is
// called for every item in order. get(i) must be pure. Ends with a barrier.
template <int T, class V, class Op, class Get, class Put>
__device__ V block_scan(uint32_t len, V identity, Op op, Get get, Put put,
                        typename cub::BlockScan<V, T>::TempStorage& tmp) {
  const uint32_t per = (len + T - 1) / T;
  const uint32_t a = min(len, threadIdx.x * per), b = min(len, a + per);
  V agg = identity;
  for (uint32_t i = a; i < b; ++i) agg = op(agg, get(i));
  V pre, total;
  cub::BlockScan<V, T>(tmp).ExclusiveScan(agg, pre, identity, op, total);
  for (uint32_t i = a; i < b; ++i) {
    const V v = get(i);
    put(i, pre, v);
    pre = op(pre, v);
  }
  __syncthreads();
  return total;
}

// WQSummary::SetPrune (sketch.rs:128) of the summary d(0..src) into at most
// `maxsize` entries, written through put(j, entry); returns the new length.
// The reference walks rank queries k = 1..n-1 with a cursor i that only
// advances while dx2 >= rmax[i+1] + rmin[i+1]. Ranks never decrease along a
// summary, so the first i that stops the cursor for query k alone is a
// binary search, and the cursor itself is the running maximum of those.
// Query k keeps entry c_k (i or i + 1); an entry is appended when c_k
// differs from c_{k-1} (after a step the last kept index always equals c_k),
// and the walk stops at the first query whose cursor reaches src - 1.
// `ik` is scratch of maxsize words; callers sync before reading the output.
template <int T, class Get, class Put>
__device__ uint32_t prune_block(uint32_t src, uint32_t maxsize, Get d, Put put, uint32_t* ik,
                                typename cub::BlockScan<uint32_t, T>::TempStorage& tmp) {
  if (maxsize == 0) return 0;
  if (src <= maxsize) {
    for (uint32_t i = threadIdx.x; i < src; i += T) put(i, d(i));
    return src;
  }
  if (maxsize == 1) {
    if (threadIdx.x == 0) put(0, d(0));
    return 1;
  }
  const SEntry d0 = d(0), dl = d(src - 1);
  const float begin = d0.rmax;
  const float range = __fsub_rn(dl.rmin, d0.rmax);
  const uint32_t n = maxsize - 1;
  const uint32_t K = n - 1;  // queries k = 1..n-1
  const float fn = (float)n;
  auto dx2_of = [&](uint32_t k) {
    return __fmul_rn(2.0f, __fadd_rn(__fdiv_rn(__fmul_rn((float)k, range), fn), begin));
  };
  // the first i in [1, src-1] where the cursor stops for query k
  for (uint32_t k = 1 + threadIdx.x; k <= K; k += T) {
    const float dx2 = dx2_of(k);
    uint32_t lo = 1, hi = src - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      const SEntry r = d(mid + 1);
      if (dx2 < __fadd_rn(r.rmax, r.rmin)) hi = mid; else lo = mid + 1;
    }
    ik[k - 1] = lo;
  }
  __syncthreads();
  block_scan<T, uint32_t>(
      K, 0u, MaxOp<uint32_t>(), [&](uint32_t i) { return ik[i]; },
      [&](uint32_t i, uint32_t pre, uint32_t v) { ik[i] = pre < v ? v : pre; }, tmp);
  // queries before the first cursor at src - 1 (a prefix: the cursor ascends)
  uint32_t kv;
  {
    uint32_t lo = 0, hi = K;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (ik[mid] < src - 1) lo = mid + 1; else hi = mid;
    }
    kv = lo;
  }
  __syncthreads();
  for (uint32_t k = 1 + threadIdx.x; k <= kv; k += T) {
    const uint32_t i = ik[k - 1];
    const SEntry l = d(i), r = d(i + 1);
    const float lim = __fadd_rn(__fadd_rn(l.rmin, l.wmin), __fsub_rn(r.rmax, r.wmin));
    ik[k - 1] = dx2_of(k) < lim ? i : i + 1;
  }
  __syncthreads();
  const uint32_t np = block_scan<T, uint32_t>(
      kv, 0u, SumU32(),
      [&](uint32_t j) { return ik[j] != (j == 0 ? 0u : ik[j - 1]) ? 1u : 0u; },
      [&](uint32_t j, uint32_t pos, uint32_t v) {
        if (v) put(1 + pos, d(ik[j]));
      },
      tmp);
  const uint32_t last = kv > 0 ? ik[kv - 1] : 0u;
  if (threadIdx.x == 0) {
    put(0, d0);
    if (last != src - 1) put(1 + np, dl);
  }
  return 1 + np + (last != src - 1 ? 1u : 0u);
}

// ---- 1. extraction ---------------------------------------------------------
// Present (non-NaN) cells per (feature, tile of kTileRows rows).
__global__ void __launch_bounds__(kTileRows) k_sk_count(const float* __restrict__ x, uint64_t n,
                                                        uint32_t F, uint64_t n_tiles,
                                                        unsigned long long* __restrict__ counts) {
  const uint64_t r = (uint64_t)blockIdx.x * kTileRows + threadIdx.x;
  const bool in = r < n;
  for (uint32_t f = 0; f < F; ++f) {
    const bool p = in && !isnan(x[r * F + f]);
    const int c = __syncthreads_count(p);
    if (threadIdx.x == 0) counts[(uint64_t)f * n_tiles + blockIdx.x] = (unsigned long long)c;
  }
}

// Each feature's present values in row order: feature f's stream starts at
// offs[f * n_tiles] (the exclusive scan of the counts, feature-major).
__global__ void __launch_bounds__(kTileRows) k_sk_scatter(const float* __restrict__ x, uint64_t n,
                                                          uint32_t F, uint64_t n_tiles,
                                                          const unsigned long long* __restrict__ offs,
                                                          float* __restrict__ vals) {
  using BS = cub::BlockScan<int, kTileRows>;
  __shared__ typename BS::TempStorage tmp;
  const uint64_t r = (uint64_t)blockIdx.x * kTileRows + threadIdx.x;
  const bool in = r < n;
  for (uint32_t f = 0; f < F; ++f) {
    const float v = in ? x[r * F + f] : 0.0f;
    const bool p = in && !isnan(v);
    int rank;
    BS(tmp).ExclusiveSum(p ? 1 : 0, rank);
    __syncthreads();
    if (p) vals[offs[(uint64_t)f * n_tiles + blockIdx.x] + (uint64_t)rank] = v;
  }
}

__global__ void k_sk_stream_starts(const unsigned long long* __restrict__ offs,
                                   const unsigned long long* __restrict__ counts, uint32_t F,
                                   uint64_t n_tiles, unsigned long long* __restrict__ S) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f < F) S[f] = offs[(uint64_t)f * n_tiles];
  if (f == F) {
    const uint64_t last = (uint64_t)F * n_tiles - 1;
    S[F] = offs[last] + counts[last];
  }
}

// CSR checks (DMatrix::from_csr, src/data/dmatrix.rs:459), a warp per row:
// bit 0 of *flags = invalid (descending offsets, column out of range,
// non-finite value), bit 1 = columns not strictly ascending in a row, bit 2 =
// some row lacks a feature.
__global__ void k_sk_csr_check(const uint64_t* __restrict__ ip, const uint32_t* __restrict__ ix,
                               const float* __restrict__ v, uint64_t n, uint32_t F, uint64_t nnz,
                               int* __restrict__ flags) {
  const uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const uint64_t a = ip[row], b = ip[row + 1];
  int bad = 0;
  if (b < a || b > nnz) {  // offsets outside [0, nnz]: read no cell
    bad = 1;
  } else {
    for (uint64_t j = a + lane; j < b; j += 32) {
      const uint32_t c = ix[j];
      if (c >= F || !isfinite(v[j])) bad |= 1;
      if (j > a && ix[j - 1] >= c) bad |= 2;
    }
    if (lane == 0 && b - a != F) bad |= 4;
  }
  bad = __reduce_or_sync(0xffffffffu, (unsigned)bad);
  if (lane == 0 && bad) atomicOr(flags, bad);
}

// Stream starts of a column-sorted cell list: S[f] = first cell of column >= f.
__global__ void k_sk_csr_starts(const uint32_t* __restrict__ col_sorted, uint64_t nnz, uint32_t F,
                                unsigned long long* __restrict__ S) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f > F) return;
  uint64_t lo = 0, hi = nnz;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (col_sorted[mid] < f) lo = mid + 1; else hi = mid;
  }
  S[f] = lo;
}

// ---- 2. queue entries ------------------------------------------------------
// flag[i] = 1 where a queue entry starts: the first value of a feature, or
// a value unequal (f32 !=) to its predecessor (sketch.rs:520 `queue_push`).
__global__ void k_sk_flags(const float* __restrict__ vals, uint64_t P, uint32_t* __restrict__ flag) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < P) flag[i] = (i == 0 || vals[i] != vals[i - 1]) ? 1u : 0u;
}
__global__ void k_sk_feature_flags(const unsigned long long* __restrict__ S, uint32_t F,
                                   uint32_t* __restrict__ flag) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f < F && S[f] < S[f + 1]) flag[S[f]] = 1u;
}
__global__ void k_sk_entry_starts(const uint32_t* __restrict__ flag, const uint32_t* __restrict__ eid,
                                  uint64_t P, uint32_t* __restrict__ es) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < P && flag[i]) es[eid[i]] = (uint32_t)i;
  if (i == P - 1) es[eid[i] + flag[i]] = (uint32_t)P;  // es[E] = P
}
__global__ void k_sk_entry_offsets(const unsigned long long* __restrict__ S,
                                   const uint32_t* __restrict__ flag, const uint32_t* __restrict__ eid,
                                   uint64_t P, uint32_t F, uint32_t* __restrict__ EO) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f > F) return;
  const uint32_t E = eid[P - 1] + flag[P - 1];
  EO[f] = S[f] < P ? eid[S[f]] : E;
}

// ---- 3. one CTA per queue flush -------------------------------------------
struct Chunk {
  uint32_t cnt;    // queue entries in this flush
  uint32_t eb;     // first entry (global entry index)
  uint32_t limit;  // the feature's summary budget
  uint32_t pad;
  uint64_t out;    // SEntry offset of its pruned summary
};

template <int IPT>
struct ChunkSmem {
  static constexpr int kCap = kChunkThreads * IPT;
  struct Pair {
    uint32_t w, c;
  };
  union Front {
    typename cub::BlockRadixSort<uint32_t, kChunkThreads, IPT, uint32_t>::TempStorage sort;
    uint32_t ik[kCap];
  };
  static constexpr size_t up16(size_t b) { return (b + 15) / 16 * 16; }
  // byte offsets of the regions: front | pair scan | u32 scan | gpre | gval | lastk
  static constexpr size_t kPScan = up16(sizeof(Front));
  static constexpr size_t kUScan = kPScan + up16(sizeof(typename cub::BlockScan<Pair, kChunkThreads>::TempStorage));
  static constexpr size_t kGpre = kUScan + up16(sizeof(typename cub::BlockScan<uint32_t, kChunkThreads>::TempStorage));
  static constexpr size_t kGval = kGpre + up16((size_t)(kCap + 1) * 4);
  static constexpr size_t kLast = kGval + up16((size_t)kCap * 4);
  static constexpr size_t bytes() { return kLast + (size_t)kChunkThreads * 4; }
};

struct PairSum {
  template <class P>
  __device__ __forceinline__ P operator()(const P& a, const P& b) const {
    return P{a.w + b.w, a.c + b.c};
  }
};

// Queue::PopSummary + the first prune of push_summary: sort the flush's
// entries by value, fold equal values (set_from_sorted, sketch.rs:88: a
// group's rmin is the weight before it, rmax = rmin + its weight), then
// SetPrune to the feature's budget.
template <int IPT>
__global__ void __launch_bounds__(kChunkThreads, 1)
    k_sk_chunk(const float* __restrict__ vals, const uint32_t* __restrict__ es,
               const Chunk* __restrict__ chunks, SEntry* __restrict__ temps,
               uint32_t* __restrict__ temp_len) {
  using SM = ChunkSmem<IPT>;
  using Pair = typename SM::Pair;
  using Sort = cub::BlockRadixSort<uint32_t, kChunkThreads, IPT, uint32_t>;
  using PScan = cub::BlockScan<Pair, kChunkThreads>;
  using UScan = cub::BlockScan<uint32_t, kChunkThreads>;
  extern __shared__ __align__(16) unsigned char smem[];
  auto& front = *reinterpret_cast<typename SM::Front*>(smem);
  auto& pscan = *reinterpret_cast<typename PScan::TempStorage*>(smem + SM::kPScan);
  auto& uscan = *reinterpret_cast<typename UScan::TempStorage*>(smem + SM::kUScan);
  uint32_t* gpre = reinterpret_cast<uint32_t*>(smem + SM::kGpre);
  float* gval = reinterpret_cast<float*>(smem + SM::kGval);
  uint32_t* lastk = reinterpret_cast<uint32_t*>(smem + SM::kLast);

  const Chunk ch = chunks[blockIdx.x];
  const int t = threadIdx.x;
  uint32_t key[IPT], w[IPT];
  // the sort does not care where an item starts: load striped (coalesced)
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t idx = (uint32_t)j * kChunkThreads + t;
    if (idx < ch.cnt) {
      const uint32_t e = ch.eb + idx;
      const uint32_t a = es[e], b = es[e + 1];
      key[j] = sort_key(vals[a]);
      w[j] = b - a;
    } else {
      key[j] = 0xffffffffu;  // above every finite or infinite value's key
      w[j] = 0u;
    }
  }
  Sort(front.sort).Sort(key, w);  // blocked: thread t holds positions t*IPT + j
  __syncthreads();
  lastk[t] = key[IPT - 1];
  __syncthreads();
  bool start[IPT];
  Pair mine{0u, 0u};
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t pos = (uint32_t)t * IPT + j;
    const bool valid = pos < ch.cnt;
    const float v = unsort_key(key[j]);
    bool s = valid && pos == 0;
    if (valid && pos > 0) {
      const float pv = unsort_key(j > 0 ? key[j - 1] : lastk[t - 1]);
      s = v != pv;  // -0 and +0 fold (f32 ==), as set_from_sorted does
    }
    start[j] = s;
    mine.w += valid ? w[j] : 0u;
    mine.c += s ? 1u : 0u;
  }
  Pair pre, agg;
  PScan(pscan).ExclusiveScan(mine, pre, Pair{0u, 0u}, PairSum(), agg);
  {
    uint32_t wp = pre.w, gi = pre.c;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      if (start[j]) {
        gpre[gi] = wp;
        gval[gi] = unsort_key(key[j]);
        ++gi;
      }
      wp += ((uint32_t)t * IPT + j < ch.cnt) ? w[j] : 0u;
    }
  }
  const uint32_t G = agg.c;
  if (t == 0) gpre[G] = agg.w;
  __syncthreads();
  auto entry = [&](uint32_t g) {
    const uint32_t a = gpre[g], b = gpre[g + 1];
    return SEntry{(float)a, (float)b, (float)(b - a), gval[g]};
  };
  SEntry* out = temps + ch.out;
  const uint32_t len = prune_block<kChunkThreads>(
      G, ch.limit, entry, [&](uint32_t j, const SEntry& e) { out[j] = e; }, front.ik, uscan);
  if (t == 0) temp_len[blockIdx.x] = len;
}

// ---- 4. the ladder, one CTA per feature -----------------------------------
struct FeatPlan {
  uint32_t chunk_begin;  // first flush (index into the chunk arrays)
  uint32_t n_chunks;
  uint32_t limit;
  uint32_t n_levels;     // level buffers in the pool
  uint64_t pool;         // SEntry offset: n_levels + 2 buffers of 2 * limit
  uint32_t fin_begin;    // the merge tree's level summaries the final summary
  uint32_t fin_count;    //   combines (FinItem), lowest level first
};

// One summary of the merge tree: its SEntry offset and the index of its
// length.
struct FinItem {
  uint64_t off;
  uint32_t len;
  uint32_t pad;
};

// One merge of the tree: V = P(C(A, B)) with A the newer block (2j + 1), B
// the older (2j), into `out`; `w` is scratch of 2 * limit entries.
struct MergeTask {
  uint32_t f, limit;
  uint32_t la, lb, lo, pad;  // indices of the lengths of A, B, out
  uint64_t a, b, out, w;
};



// WQSummary::SetCombine (sketch.rs:217) of A and B into O, then FixError
// (:180). Values within a summary are strictly ascending, so entry a of A
// lands after the |B < a| entries of B and the merged pairs before it; an
// unmerged entry takes its rank bounds from its neighbours in the other
// summary exactly as the sequential merge would. Returns |O|.
template <int T>
__device__ uint32_t combine_block(const SEntry* A, uint32_t na, const SEntry* B, uint32_t nb,
                                  SEntry* O, uint32_t* cnt, uint32_t* eq,
                                  typename cub::BlockScan<uint32_t, T>::TempStorage& us,
                                  typename cub::BlockScan<float, T>::TempStorage& fs) {
  if (nb == 0 || na == 0) {
    const SEntry* src = nb == 0 ? A : B;
    const uint32_t n = nb == 0 ? na : nb;
    for (uint32_t i = threadIdx.x; i < n; i += T) O[i] = src[i];
    __syncthreads();
    return n;
  }
  for (uint32_t i = threadIdx.x; i < na; i += T) {
    const float a = A[i].value;
    uint32_t lo = 0, hi = nb;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (B[mid].value < a) lo = mid + 1; else hi = mid;
    }
    cnt[i] = lo;
    eq[i] = (lo < nb && B[lo].value == a) ? 1u : 0u;
  }
  __syncthreads();
  const uint32_t M = block_scan<T, uint32_t>(
      na, 0u, SumU32(), [&](uint32_t i) { return eq[i]; },
      [&](uint32_t i, uint32_t pre, uint32_t v) { eq[i] = (pre << 1) | v; }, us);
  // eq[i] now holds (merged pairs before i) << 1 | (i merged)
  for (uint32_t i = threadIdx.x; i < na; i += T) {
    const SEntry a = A[i];
    const uint32_t cb = cnt[i];
    const uint32_t before = eq[i] >> 1;
    const uint32_t pos = i + cb - before;
    if (eq[i] & 1u) {
      const SEntry b = B[cb];
      O[pos] = SEntry{__fadd_rn(a.rmin, b.rmin), __fadd_rn(a.rmax, b.rmax), __fadd_rn(a.wmin, b.wmin),
                      a.value};
    } else {
      const float bprev = cb > 0 ? __fadd_rn(B[cb - 1].rmin, B[cb - 1].wmin) : 0.0f;
      const float up = cb < nb ? __fsub_rn(B[cb].rmax, B[cb].wmin) : B[nb - 1].rmax;
      O[pos] = SEntry{__fadd_rn(a.rmin, bprev), __fadd_rn(a.rmax, up), a.wmin, a.value};
    }
  }
  for (uint32_t j = threadIdx.x; j < nb; j += T) {
    const SEntry b = B[j];
    uint32_t lo = 0, hi = na;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (A[mid].value < b.value) lo = mid + 1; else hi = mid;
    }
    if (lo < na && A[lo].value == b.value) continue;  // written with its pair
    const uint32_t before = lo < na ? (eq[lo] >> 1) : M;
    const uint32_t pos = j + lo - before;
    const float aprev = lo > 0 ? __fadd_rn(A[lo - 1].rmin, A[lo - 1].wmin) : 0.0f;
    const float up = lo < na ? __fsub_rn(A[lo].rmax, A[lo].wmin) : A[na - 1].rmax;
    O[pos] = SEntry{__fadd_rn(b.rmin, aprev), __fadd_rn(b.rmax, up), b.wmin, b.value};
  }
  __syncthreads();
  const uint32_t no = na + nb - M;
  // FixError: rmin = running max (from 0); rmax = running max of
  // max(rmax, rmin + wmin)
  block_scan<T, float>(
      no, 0.0f, MaxOp<float>(), [&](uint32_t i) { return O[i].rmin; },
      [&](uint32_t i, float pre, float v) { O[i].rmin = pre < v ? v : pre; }, fs);
  block_scan<T, float>(
      no, 0.0f, MaxOp<float>(),
      [&](uint32_t i) {
        const SEntry e = O[i];
        const float rn = __fadd_rn(e.rmin, e.wmin);
        return e.rmax < rn ? rn : e.rmax;
      },
      [&](uint32_t i, float pre, float v) { O[i].rmax = pre < v ? v : pre; }, fs);
  return no;
}

template <int T>
__device__ uint32_t prune_global(const SEntry* src, uint32_t n, uint32_t maxsize, SEntry* dst,
                                 uint32_t* ik, typename cub::BlockScan<uint32_t, T>::TempStorage& us) {
  const uint32_t len = prune_block<T>(
      n, maxsize, [&](uint32_t i) { return src[i]; },
      [&](uint32_t j, const SEntry& e) { dst[j] = e; }, ik, us);
  __syncthreads();
  return len;
}

constexpr int kMergeThreads = 512;

// The ladder as a merge tree (one launch per level, every feature's merges
// at once). While every merge the reference's push_summary performs holds
// more than `limit` entries, each one carries, and level l of the ladder
// then holds exactly V_l(j) = prune(combine(V_{l-1}(2j+1), V_{l-1}(2j)))
// for the block of 2^l flushes its set bit stands for. A merge of `limit`
// or fewer entries would not have carried: it flags its feature, whose
// ladder k_sk_ladder then replays in order instead.
__global__ void __launch_bounds__(kMergeThreads)
    k_sk_merge(const MergeTask* __restrict__ tasks, SEntry* __restrict__ store,
               uint32_t* __restrict__ lens, int* __restrict__ bad) {
  using UScan = cub::BlockScan<uint32_t, kMergeThreads>;
  using FScan = cub::BlockScan<float, kMergeThreads>;
  __shared__ typename UScan::TempStorage us;
  __shared__ typename FScan::TempStorage fs;
  extern __shared__ __align__(16) uint32_t dyn[];
  const MergeTask t = tasks[blockIdx.x];
  uint32_t* cnt = dyn;
  uint32_t* eq = dyn + (t.limit + 1);
  uint32_t* ik = dyn + 2 * (t.limit + 1);
  const uint32_t na = lens[t.la], nb = lens[t.lb];
  SEntry* w = store + t.w;
  const uint32_t m = combine_block<kMergeThreads>(store + t.a, na, store + t.b, nb, w, cnt, eq, us, fs);
  if (m <= t.limit) {
    if (threadIdx.x == 0) atomicOr(&bad[t.f], 1);
  }
  const uint32_t len = prune_global<kMergeThreads>(w, m, t.limit, store + t.out, ik, us);
  if (threadIdx.x == 0) lens[t.lo] = len;
}

// WQSummary::QueryCutValues (sketch.rs:427), sequential.
__device__ uint32_t query_cuts(const SEntry* data, uint32_t n, uint32_t max_bin, float* out) {
  uint32_t m = 0;
  if (n == 0) {
    out[m++] = 1e-5f;
    return m;
  }
  auto advance = [&](uint32_t cur, float v) {
    while (cur < n && data[cur].value <= v) ++cur;
    return cur;
  };
  float last_cut = data[0].value;
  uint32_t next_value = advance(1, last_cut);
  if (n <= max_bin) {
    while (next_value < n) {
      const float cpt = data[next_value].value;
      out[m++] = cpt;
      last_cut = cpt;
      next_value = advance(next_value + 1, last_cut);
    }
  } else {
    const double total = (double)data[n - 1].rmax;
    uint32_t q = 0;
    for (uint32_t i = 1; i < max_bin; ++i) {
      const double rank2 = __dmul_rn(2.0, __ddiv_rn(__dmul_rn((double)i, total), (double)max_bin));
      while (q < n - 2 && rank2 >= (double)__fadd_rn(data[q + 1].rmin, data[q + 1].rmax)) ++q;
      const float lim = __fadd_rn(__fadd_rn(data[q].rmin, data[q].wmin),
                                  __fsub_rn(data[q + 1].rmax, data[q + 1].wmin));
      float cpt = rank2 < (double)lim ? data[q].value : data[q + 1].value;
      if (cpt <= last_cut) {
        next_value = advance(next_value, last_cut);
        if (next_value == n) break;
        cpt = data[next_value].value;
      } else if (next_value < n && data[next_value].value <= cpt) {
        next_value = advance(next_value + 1, cpt);
      }
      out[m++] = cpt;
      last_cut = cpt;
    }
  }
  const float cpt = data[n - 1].value;
  out[m++] = __fadd_rn(cpt, __fadd_rn(fabsf(cpt), 1e-5f));
  return m;
}

// push_summary (sketch.rs:575) over the feature's pruned flushes in order,
// then summary (:607) and the cut query. Levels live in a global pool, one
// buffer each; W0 takes combine results, W1 prune results.
__global__ void __launch_bounds__(kLadderThreads, 1)
    k_sk_ladder(const FeatPlan* __restrict__ plans, const Chunk* __restrict__ chunks,
                const SEntry* __restrict__ temps, const uint32_t* __restrict__ temp_len,
                SEntry* __restrict__ pool, uint32_t max_bin, float* __restrict__ cuts,
                uint32_t* __restrict__ n_cuts, int* __restrict__ err, const int* __restrict__ bad,
                const FinItem* __restrict__ fin) {
  using UScan = cub::BlockScan<uint32_t, kLadderThreads>;
  using FScan = cub::BlockScan<float, kLadderThreads>;
  __shared__ typename UScan::TempStorage us;
  __shared__ typename FScan::TempStorage fs;
  __shared__ uint32_t lvl_len[kMaxLevels];
  extern __shared__ __align__(16) uint32_t dyn[];
  const FeatPlan p = plans[blockIdx.x];
  const uint32_t L = p.limit;
  const uint64_t cap = 2ull * L;
  uint32_t* cnt = dyn;
  uint32_t* eq = dyn + (L + 1);
  uint32_t* ik = dyn + 2 * (L + 1);
  SEntry* base = pool + p.pool;
  auto level = [&](uint32_t l) { return base + l * cap; };
  SEntry* W0 = base + (uint64_t)p.n_levels * cap;
  SEntry* W1 = W0 + cap;
  if (!bad[blockIdx.x]) {
    // every merge carried: the ladder's levels are the merge tree's
    // summaries of the flush count's set bits; summary() combines them from
    // the lowest level up
    uint32_t outlen = 0;
    for (uint32_t k = 0; k < p.fin_count; ++k) {
      const FinItem it = fin[p.fin_begin + k];
      const uint32_t ll = temp_len[it.len];
      if (ll == 0) continue;
      if (outlen == 0) {
        for (uint32_t i = threadIdx.x; i < ll; i += blockDim.x) W1[i] = temps[it.off + i];
        __syncthreads();
        outlen = ll;
        continue;
      }
      const uint32_t m = combine_block<kLadderThreads>(W1, outlen, temps + it.off, ll, W0, cnt, eq, us, fs);
      outlen = prune_global<kLadderThreads>(W0, m, L, W1, ik, us);
    }
    if (threadIdx.x == 0) {
      const uint32_t mb = min(outlen, max_bin);
      n_cuts[blockIdx.x] = query_cuts(W1, outlen, mb, cuts + (uint64_t)blockIdx.x * max_bin);
    }
    return;
  }
  for (uint32_t l = threadIdx.x; l < kMaxLevels; l += blockDim.x) lvl_len[l] = 0;
  __syncthreads();
  uint32_t used = 0;  // levels ever touched
  for (uint32_t c = 0; c < p.n_chunks; ++c) {
    const uint32_t ci = p.chunk_begin + c;
    const SEntry* cur = temps + chunks[ci].out;
    uint32_t curlen = temp_len[ci];
    for (uint32_t l = 0;; ++l) {
      if (l >= p.n_levels) {
        if (threadIdx.x == 0) atomicOr(err, 1);
        return;
      }
      used = max(used, l + 1);
      if (l > 0) {
        curlen = prune_global<kLadderThreads>(cur, curlen, L, W1, ik, us);
        cur = W1;
      }
      const uint32_t ll = lvl_len[l];
      __syncthreads();
      if (ll == 0) {
        for (uint32_t i = threadIdx.x; i < curlen; i += blockDim.x) level(l)[i] = cur[i];
        if (threadIdx.x == 0) lvl_len[l] = curlen;
        __syncthreads();
        break;
      }
      curlen = combine_block<kLadderThreads>(cur, curlen, level(l), ll, W0, cnt, eq, us, fs);
      cur = W0;
      if (curlen <= L) {
        for (uint32_t i = threadIdx.x; i < curlen; i += blockDim.x) level(l)[i] = cur[i];
        if (threadIdx.x == 0) lvl_len[l] = curlen;
        __syncthreads();
        break;
      }
      if (threadIdx.x == 0) lvl_len[l] = 0;
      __syncthreads();
    }
  }
  // summary(budget): combine the levels in order, pruning to the budget
  // (the summary budget of the values seen equals the level budget L)
  uint32_t outlen = 0;
  for (uint32_t l = 0; l < used; ++l) {
    const uint32_t ll = lvl_len[l];
    if (ll == 0) continue;
    if (outlen == 0) {
      for (uint32_t i = threadIdx.x; i < ll; i += blockDim.x) W1[i] = level(l)[i];
      __syncthreads();
      outlen = ll;
      continue;
    }
    const uint32_t m = combine_block<kLadderThreads>(W1, outlen, level(l), ll, W0, cnt, eq, us, fs);
    outlen = prune_global<kLadderThreads>(W0, m, L, W1, ik, us);
  }
  if (threadIdx.x == 0) {
    const uint32_t mb = min(outlen, max_bin);
    n_cuts[blockIdx.x] = query_cuts(W1, outlen, mb, cuts + (uint64_t)blockIdx.x * max_bin);
  }
}

// ---- 5. binning ------------------------------------------------------------
__device__ __forceinline__ uint32_t local_bin(const float* __restrict__ c, uint32_t nb, float v) {
  uint32_t lo = 0, hi = nb;  // upper_bound: the first cut above v
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (v < __ldg(c + mid)) hi = mid; else lo = mid + 1;
  }
  return lo < nb - 1 ? lo : nb - 1;
}

__global__ void __launch_bounds__(kTileRows)
    k_sk_bin_dense(const float* __restrict__ x, uint64_t n, uint32_t F, const uint32_t* __restrict__ fo,
                   const float* __restrict__ cuts, uint8_t* __restrict__ cols,
                   uint64_t* __restrict__ miss, int* __restrict__ any_missing) {
  const uint64_t r = (uint64_t)blockIdx.x * kTileRows + threadIdx.x;
  const bool in = r < n;
  const uint64_t words = (n + 63) / 64;
  const uint64_t warp_row = r - (threadIdx.x & 31);
  bool seen = false;
  for (uint32_t f = 0; f < F; ++f) {
    const float v = in ? x[r * F + f] : 0.0f;
    const bool m = in && isnan(v);
    if (in) {
      const uint32_t s = __ldg(fo + f), nb = __ldg(fo + f + 1) - s;
      cols[(uint64_t)f * n + r] = m ? 0 : (uint8_t)local_bin(cuts + s, nb, v);
    }
    const uint32_t bits = __ballot_sync(0xffffffffu, m);
    if (miss && (threadIdx.x & 31) == 0 && warp_row < n)
      reinterpret_cast<uint32_t*>(miss + (uint64_t)f * words)[warp_row >> 5] = bits;
    seen |= m;
  }
  if (__syncthreads_or(seen) && threadIdx.x == 0) atomicOr(any_missing, 1);
}

__global__ void k_sk_bin_csr(const uint32_t* __restrict__ ix, const float* __restrict__ v,
                             uint64_t nnz, const uint32_t* __restrict__ fo,
                             const float* __restrict__ cuts, uint32_t* __restrict__ bins) {
  const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nnz) return;
  const uint32_t f = ix[j];
  const uint32_t s = __ldg(fo + f), nb = __ldg(fo + f + 1) - s;
  bins[j] = s + local_bin(cuts + s, nb, v[j]);
}

// ---- host side -------------------------------------------------------------
// sketch.rs:58 / :65 / :83 (`sketch_epsilon`, `limit_size_level`,
// `summary_budget`)
size_t limit_size_level(size_t maxn, double eps) {
  if (maxn == 0) return 1;
  const double internal = eps / 2.0;
  for (uint32_t nlevel = 1;; ++nlevel) {
    const size_t limit = std::min((size_t)std::ceil((double)nlevel / internal) + 1, maxn);
    if ((size_t(1) << nlevel) * limit >= maxn) return limit;
  }
}
size_t summary_budget(size_t max_bin, size_t n) {
  const size_t m = std::max<size_t>(n, 1);
  return limit_size_level(n, 1.0 / (double)std::min(max_bin, m));
}

// Device scratch freed on scope exit.
struct Scratch {
  std::vector<void*> ptrs;
  ~Scratch() {
    for (void* p : ptrs) cudaFree(p);
  }
  template <class T>
  cudaError_t get(T** out, size_t count) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return e;
    ptrs.push_back(p);
    *out = static_cast<T*>(p);
    return cudaSuccess;
  }
};

#define SK_CK(call)                                  \
  do {                                               \
    cudaError_t _e = (call);                         \
    if (_e != cudaSuccess) {                         \
      why = std::string(#call) + ": " + cudaGetErrorString(_e); \
      return HB_DEVICE_FAILED;                       \
    }                                                \
  } while (0)

template <int IPT>
cudaError_t launch_chunks(uint32_t n, const float* vals, const uint32_t* es, const Chunk* chunks,
                          SEntry* temps, uint32_t* temp_len, cudaStream_t s) {
  const size_t smem = ChunkSmem<IPT>::bytes();
  cudaError_t e = cudaFuncSetAttribute(k_sk_chunk<IPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k_sk_chunk<IPT><<<n, kChunkThreads, smem, s>>>(vals, es, chunks, temps, temp_len);
  return cudaGetLastError();
}

// Steps 2-4 on feature streams already on the device: vals[S[f]..S[f+1]).
hb_status sketch_streams(const float* d_vals, const std::vector<uint64_t>& S, uint32_t F,
                         uint32_t max_bin, cudaStream_t s, Scratch& sc, std::vector<uint32_t>& fo,
                         std::vector<float>& cuts, std::string& why) {
  const uint64_t P = S[F];
  fo.assign(1, 0u);
  cuts.clear();
  for (uint32_t f = 0; f < F; ++f)
    if (S[f + 1] - S[f] >= (1ull << 24)) {
      why = "a feature with 2^24 or more present values (the host sketch takes it)";
      return HB_REFUSED;
    }
  if (P == 0) {  // every feature empty: one cut each (query_cut_values of an empty summary)
    for (uint32_t f = 0; f < F; ++f) {
      cuts.push_back(1e-5f);
      fo.push_back((uint32_t)cuts.size());
    }
    return HB_OK;
  }
  if (P >= 0xffffffffull) {
    why = "2^32 - 1 or more present cells (the host sketch takes them)";
    return HB_REFUSED;
  }
  const int tpb = 256;
  const unsigned gP = (unsigned)((P + tpb - 1) / tpb);
  uint32_t *flag, *eid, *es, *EO;
  unsigned long long* dS;
  SK_CK(sc.get(&flag, P));
  SK_CK(sc.get(&eid, P));
  SK_CK(sc.get(&dS, F + 1));
  SK_CK(sc.get(&EO, F + 1));
  SK_CK(cudaMemcpyAsync(dS, S.data(), 8 * (F + 1), cudaMemcpyHostToDevice, s));
  k_sk_flags<<<gP, tpb, 0, s>>>(d_vals, P, flag);
  k_sk_feature_flags<<<(F + 255) / 256, 256, 0, s>>>(dS, F, flag);
  SK_CK(cudaGetLastError());
  size_t tb = 0;
  SK_CK(cub::DeviceScan::ExclusiveSum(nullptr, tb, flag, eid, (int64_t)P, s));
  unsigned char* tmp;
  SK_CK(sc.get(&tmp, tb));
  SK_CK(cub::DeviceScan::ExclusiveSum(tmp, tb, flag, eid, (int64_t)P, s));
  uint32_t tail[2];
  SK_CK(cudaMemcpyAsync(&tail[0], eid + P - 1, 4, cudaMemcpyDeviceToHost, s));
  SK_CK(cudaMemcpyAsync(&tail[1], flag + P - 1, 4, cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));
  const uint64_t E = (uint64_t)tail[0] + tail[1];
  SK_CK(sc.get(&es, E + 1));
  k_sk_entry_starts<<<gP, tpb, 0, s>>>(flag, eid, P, es);
  k_sk_entry_offsets<<<(F + 256) / 256, 256, 0, s>>>(dS, flag, eid, P, F, EO);
  SK_CK(cudaGetLastError());
  std::vector<uint32_t> hEO(F + 1);
  SK_CK(cudaMemcpyAsync(hEO.data(), EO, 4 * (F + 1), cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));

  // the flushes of every feature and each feature's ladder
  std::vector<Chunk> hch;
  std::vector<FeatPlan> plans(F);
  uint64_t temp_total = 0, pool_total = 0;
  uint32_t full_max = 0, limit_max = 1;
  for (uint32_t f = 0; f < F; ++f) {
    const uint64_t present = S[f + 1] - S[f];
    const uint32_t L = (uint32_t)summary_budget(max_bin, present);
    const uint32_t full = 2 * L;
    const uint32_t Ef = hEO[f + 1] - hEO[f];
    const uint32_t nch = (Ef + full - 1) / full;
    FeatPlan& p = plans[f];
    p.chunk_begin = (uint32_t)hch.size();
    p.n_chunks = nch;
    p.limit = L;
    uint32_t lv = 1;
    while ((1ull << lv) <= nch) ++lv;
    p.n_levels = std::min<uint32_t>(lv + 1, kMaxLevels);
    p.pool = pool_total;
    pool_total += (uint64_t)(p.n_levels + 2) * 2 * L;
    for (uint32_t c = 0; c < nch; ++c) {
      Chunk ch{};
      ch.eb = hEO[f] + c * full;
      ch.cnt = std::min(full, Ef - c * full);
      ch.limit = L;
      ch.out = temp_total;
      temp_total += L;
      hch.push_back(ch);
    }
    full_max = std::max(full_max, nch ? full : 0u);
    limit_max = std::max(limit_max, L);
  }
  const uint32_t n_chunks = (uint32_t)hch.size();
  if (full_max > (uint32_t)kChunkThreads * 25) {
    why = "a queue larger than one CTA sorts (max_bin above 256)";
    return HB_REFUSED;
  }
  // The merge tree: V_l(j) (l >= 1) of every complete block of 2^l flushes,
  // stored after the flushes' summaries (`store`), lengths after theirs
  // (`lens`); per level the merges of every feature, each with its own
  // scratch; per feature the summaries of its flush count's set bits.
  std::vector<std::vector<MergeTask>> levels;
  std::vector<FinItem> fin;
  uint64_t vstore = 0;
  uint32_t n_lens = n_chunks;
  uint64_t wmax = 0;
  {
    std::vector<uint64_t> wlevel;
    for (uint32_t f = 0; f < F; ++f) {
      FeatPlan& p = plans[f];
      const uint32_t C = p.n_chunks, L = p.limit;
      // offsets and length indices of V_l(j), l >= 1, of this feature
      std::vector<uint64_t> off_l(1, 0);
      std::vector<uint32_t> len_l(1, 0);
      uint64_t at = temp_total + vstore;
      uint32_t li = n_lens;
      for (uint32_t l = 1; (C >> l) > 0; ++l) {
        off_l.push_back(at);
        len_l.push_back(li);
        at += (uint64_t)(C >> l) * L;
        li += C >> l;
      }
      auto v_off = [&](uint32_t l, uint32_t j) -> uint64_t {
        return l == 0 ? hch[p.chunk_begin + j].out : off_l[l] + (uint64_t)j * L;
      };
      auto v_len = [&](uint32_t l, uint32_t j) -> uint32_t {
        return l == 0 ? p.chunk_begin + j : len_l[l] + j;
      };
      for (uint32_t l = 1; (C >> l) > 0; ++l) {
        if (levels.size() < l) levels.emplace_back(), wlevel.push_back(0);
        for (uint32_t j = 0; j < (C >> l); ++j) {
          MergeTask t{};
          t.f = f;
          t.limit = L;
          t.a = v_off(l - 1, 2 * j + 1);
          t.la = v_len(l - 1, 2 * j + 1);
          t.b = v_off(l - 1, 2 * j);
          t.lb = v_len(l - 1, 2 * j);
          t.out = v_off(l, j);
          t.lo = v_len(l, j);
          t.w = wlevel[l - 1];  // relative; the scratch base is added below
          wlevel[l - 1] += 2ull * L;
          levels[l - 1].push_back(t);
        }
      }
      p.fin_begin = (uint32_t)fin.size();
      for (uint32_t l = 0; (C >> l) > 0; ++l)
        if ((C >> l) & 1u) {
          const uint32_t j = (C >> (l + 1)) << 1;
          fin.push_back(FinItem{v_off(l, j), v_len(l, j), 0u});
        }
      p.fin_count = (uint32_t)fin.size() - p.fin_begin;
      vstore = at - temp_total;
      n_lens = li;
    }
    for (uint64_t w : wlevel) wmax = std::max(wmax, w);
  }
  const uint64_t wbase = temp_total + vstore;
  for (auto& lv : levels)
    for (auto& t : lv) t.w += wbase;
  Chunk* dch;
  FeatPlan* dplans;
  SEntry *temps, *pool;
  uint32_t *temp_len, *ncuts;
  float* dcuts;
  int* err;
  SK_CK(sc.get(&dch, n_chunks));
  SK_CK(sc.get(&dplans, F));
  SK_CK(sc.get(&temps, temp_total + vstore + wmax));
  SK_CK(sc.get(&temp_len, n_lens));
  int* bad;
  FinItem* dfin;
  SK_CK(sc.get(&bad, F));
  SK_CK(sc.get(&dfin, std::max<size_t>(fin.size(), 1)));
  SK_CK(cudaMemsetAsync(bad, 0, 4 * (size_t)F, s));
  if (!fin.empty())
    SK_CK(cudaMemcpyAsync(dfin, fin.data(), sizeof(FinItem) * fin.size(), cudaMemcpyHostToDevice, s));
  SK_CK(sc.get(&pool, pool_total));
  SK_CK(sc.get(&dcuts, (uint64_t)F * max_bin));
  SK_CK(sc.get(&ncuts, F));
  SK_CK(sc.get(&err, 1));
  SK_CK(cudaMemsetAsync(err, 0, 4, s));
  if (n_chunks)
    SK_CK(cudaMemcpyAsync(dch, hch.data(), sizeof(Chunk) * n_chunks, cudaMemcpyHostToDevice, s));
  SK_CK(cudaMemcpyAsync(dplans, plans.data(), sizeof(FeatPlan) * F, cudaMemcpyHostToDevice, s));
  if (n_chunks) {
    cudaError_t e;
    if (full_max <= kChunkThreads * 4) e = launch_chunks<4>(n_chunks, d_vals, es, dch, temps, temp_len, s);
    else if (full_max <= kChunkThreads * 8) e = launch_chunks<8>(n_chunks, d_vals, es, dch, temps, temp_len, s);
    else if (full_max <= kChunkThreads * 16) e = launch_chunks<16>(n_chunks, d_vals, es, dch, temps, temp_len, s);
    else e = launch_chunks<25>(n_chunks, d_vals, es, dch, temps, temp_len, s);
    SK_CK(e);
  }
  const size_t dsm = (size_t)3 * (limit_max + 1) * 4;
  if (!levels.empty()) {
    size_t n_tasks = 0;
    for (const auto& lv : levels) n_tasks += lv.size();
    std::vector<MergeTask> flat;
    flat.reserve(n_tasks);
    for (const auto& lv : levels) flat.insert(flat.end(), lv.begin(), lv.end());
    MergeTask* dtasks;
    SK_CK(sc.get(&dtasks, n_tasks));
    SK_CK(cudaMemcpyAsync(dtasks, flat.data(), sizeof(MergeTask) * n_tasks, cudaMemcpyHostToDevice, s));
    SK_CK(cudaFuncSetAttribute(k_sk_merge, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm));
    size_t at = 0;
    for (const auto& lv : levels) {  // one launch per tree level, in order
      k_sk_merge<<<(unsigned)lv.size(), kMergeThreads, dsm, s>>>(dtasks + at, temps, temp_len, bad);
      SK_CK(cudaGetLastError());
      at += lv.size();
    }
  }
  SK_CK(cudaFuncSetAttribute(k_sk_ladder, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm));
  k_sk_ladder<<<F, kLadderThreads, dsm, s>>>(dplans, dch, temps, temp_len, pool, max_bin, dcuts, ncuts, err,
                                             bad, dfin);
  SK_CK(cudaGetLastError());
  std::vector<float> hc((size_t)F * max_bin);
  std::vector<uint32_t> hn(F);
  int herr = 0;
  SK_CK(cudaMemcpyAsync(hc.data(), dcuts, 4 * hc.size(), cudaMemcpyDeviceToHost, s));
  SK_CK(cudaMemcpyAsync(hn.data(), ncuts, 4 * F, cudaMemcpyDeviceToHost, s));
  SK_CK(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));
  if (herr) {
    why = "sketch ladder deeper than planned";
    return HB_DEVICE_FAILED;
  }
  for (uint32_t f = 0; f < F; ++f) {
    if (hn[f] == 0 || hn[f] > max_bin) {
      why = "sketch produced an invalid cut count";
      return HB_DEVICE_FAILED;
    }
    cuts.insert(cuts.end(), hc.begin() + (size_t)f * max_bin, hc.begin() + (size_t)f * max_bin + hn[f]);
    fo.push_back((uint32_t)cuts.size());
  }
  return HB_OK;
}

}  // namespace

hb_status sketch_dense_cuts(int device, const float* d_x, uint64_t n, uint32_t F, uint32_t max_bin,
                            cudaStream_t s, std::vector<uint32_t>& fo, std::vector<float>& cuts,
                            std::string& why) {
  (void)device;
  if (max_bin == 0 || max_bin > 256 || F == 0) {
    why = "max_bin must be 1..256";
    return HB_REFUSED;
  }
  Scratch sc;
  const uint64_t n_tiles = (n + kTileRows - 1) / kTileRows;
  if (n_tiles == 0 || n_tiles >= (1ull << 31)) {
    why = "row count out of range";
    return HB_REFUSED;
  }
  unsigned long long *counts, *offs, *dS;
  SK_CK(sc.get(&counts, (uint64_t)F * n_tiles));
  SK_CK(sc.get(&offs, (uint64_t)F * n_tiles));
  SK_CK(sc.get(&dS, F + 1));
  k_sk_count<<<(unsigned)n_tiles, kTileRows, 0, s>>>(d_x, n, F, n_tiles, counts);
  SK_CK(cudaGetLastError());
  size_t tb = 0;
  const int64_t nc = (int64_t)F * (int64_t)n_tiles;
  SK_CK(cub::DeviceScan::ExclusiveSum(nullptr, tb, counts, offs, nc, s));
  unsigned char* tmp;
  SK_CK(sc.get(&tmp, tb));
  SK_CK(cub::DeviceScan::ExclusiveSum(tmp, tb, counts, offs, nc, s));
  k_sk_stream_starts<<<(F + 256) / 256, 256, 0, s>>>(offs, counts, F, n_tiles, dS);
  SK_CK(cudaGetLastError());
  std::vector<uint64_t> S(F + 1);
  SK_CK(cudaMemcpyAsync(S.data(), dS, 8 * (F + 1), cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));
  float* vals;
  SK_CK(sc.get(&vals, S[F]));
  k_sk_scatter<<<(unsigned)n_tiles, kTileRows, 0, s>>>(d_x, n, F, n_tiles, offs, vals);
  SK_CK(cudaGetLastError());
  return sketch_streams(vals, S, F, max_bin, s, sc, fo, cuts, why);
}

cudaError_t bin_dense_device(const float* d_x, uint64_t n, uint32_t F, const uint32_t* d_fo,
                             const float* d_cuts, uint8_t* d_columns, uint64_t* d_missing,
                             int* d_any_missing, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(d_any_missing, 0, 4, s);
  if (e != cudaSuccess) return e;
  if (d_missing) {
    e = cudaMemsetAsync(d_missing, 0, 8 * (size_t)F * ((n + 63) / 64), s);
    if (e != cudaSuccess) return e;
  }
  const uint64_t tiles = (n + kTileRows - 1) / kTileRows;
  k_sk_bin_dense<<<(unsigned)tiles, kTileRows, 0, s>>>(d_x, n, F, d_fo, d_cuts, d_columns, d_missing,
                                                       d_any_missing);
  return cudaGetLastError();
}

hb_status sketch_csr_cuts(int device, const uint64_t* d_ip, const uint32_t* d_ix, const float* d_v,
                          uint64_t n, uint32_t F, uint64_t nnz, uint32_t max_bin, cudaStream_t s,
                          std::vector<uint32_t>& fo, std::vector<float>& cuts, std::string& why) {
  (void)device;
  if (max_bin == 0 || max_bin > 256 || F == 0 || n == 0) {
    why = "max_bin must be 1..256";
    return HB_REFUSED;
  }
  if (nnz >= (1ull << 31)) {
    why = "2^31 or more stored cells (the host sketch takes them)";
    return HB_REFUSED;
  }
  Scratch sc;
  int* flags;
  SK_CK(sc.get(&flags, 1));
  SK_CK(cudaMemsetAsync(flags, 0, 4, s));
  const uint64_t threads = n * 32;
  k_sk_csr_check<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(d_ip, d_ix, d_v, n, F, nnz, flags);
  SK_CK(cudaGetLastError());
  int hf = 0;
  SK_CK(cudaMemcpyAsync(&hf, flags, 4, cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));
  if (hf & 1) {
    why = "invalid CSR (offsets, column range or a non-finite value)";
    return HB_INVALID_ARGUMENT;
  }
  if (hf & 2) {
    why = "a row's column indices are not strictly ascending (the host path sorts them)";
    return HB_REFUSED;
  }
  uint32_t* col_sorted;
  float* vals;
  unsigned long long* dS;
  SK_CK(sc.get(&col_sorted, nnz));
  SK_CK(sc.get(&vals, nnz));
  SK_CK(sc.get(&dS, F + 1));
  int bits = 1;
  while (bits < 32 && (1ull << bits) < (uint64_t)F) ++bits;
  size_t tb = 0;
  // LSD radix sort is stable: each column keeps its cells in row order
  SK_CK(cub::DeviceRadixSort::SortPairs(nullptr, tb, d_ix, col_sorted, d_v, vals, (int64_t)nnz, 0, bits, s));
  unsigned char* tmp;
  SK_CK(sc.get(&tmp, tb));
  SK_CK(cub::DeviceRadixSort::SortPairs(tmp, tb, d_ix, col_sorted, d_v, vals, (int64_t)nnz, 0, bits, s));
  k_sk_csr_starts<<<(F + 256) / 256, 256, 0, s>>>(col_sorted, nnz, F, dS);
  SK_CK(cudaGetLastError());
  std::vector<uint64_t> S(F + 1);
  SK_CK(cudaMemcpyAsync(S.data(), dS, 8 * (F + 1), cudaMemcpyDeviceToHost, s));
  SK_CK(cudaStreamSynchronize(s));
  return sketch_streams(vals, S, F, max_bin, s, sc, fo, cuts, why);
}

cudaError_t bin_csr_device(const uint64_t* d_ip, const uint32_t* d_ix, const float* d_v, uint64_t n,
                           uint32_t F, uint64_t nnz, const uint32_t* d_fo, const float* d_cuts,
                           uint32_t* d_row_bins, int* d_any_short, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(d_any_short, 0, 4, s);
  if (e != cudaSuccess) return e;
  const uint64_t threads = n * 32;
  // bit 2 of the check's flags: a row without every feature
  k_sk_csr_check<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(d_ip, d_ix, d_v, n, F, nnz, d_any_short);
  if (nnz)
    k_sk_bin_csr<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(d_ix, d_v, nnz, d_fo, d_cuts, d_row_bins);
  return cudaGetLastError();
}

}  // namespace hb

// ---- C ABI: standalone sketches, host buffers in and out --------------------
using hb::SEntry;

namespace {

struct DevicePick {
  int prev = -1;
  explicit DevicePick(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~DevicePick() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// the calling thread's last sketch failure, as hb_engine_last_error(NULL) keeps its own
thread_local std::string g_sketch_error;

hb_status copy_cuts_out(const std::vector<uint32_t>& fo, const std::vector<float>& cuts, uint32_t F,
                        uint32_t* feature_offset, float* cut_values, uint64_t cap, uint64_t* total) {
  if (cuts.size() > cap) return HB_REFUSED;
  std::memcpy(feature_offset, fo.data(), 4 * (size_t)(F + 1));
  if (!cuts.empty()) std::memcpy(cut_values, cuts.data(), 4 * cuts.size());
  *total = cuts.size();
  return HB_OK;
}

}  // namespace

extern "C" {

const char* hb_sketch_last_error(void) { return g_sketch_error.c_str(); }

hb_status hb_sketch_dense(int32_t device, const float* x, uint64_t n_rows, uint32_t n_cols,
                          uint32_t max_bin, uint32_t* feature_offset, float* cut_values, uint64_t cap,
                          uint64_t* total, uint8_t* columns, uint64_t* missing, int32_t* dense) {
  if (!x || !feature_offset || !cut_values || !total || n_rows == 0 || n_cols == 0 || max_bin == 0 ||
      ((columns || missing) && !dense))
    return HB_INVALID_ARGUMENT;
  DevicePick pick(device);
  std::string why;
  cudaStream_t s = nullptr;
  float* d_x = nullptr;
  uint8_t* d_col = nullptr;
  uint64_t* d_miss = nullptr;
  uint32_t* d_fo = nullptr;
  float* d_cuts = nullptr;
  int* d_any = nullptr;
  hb_status st = HB_OK;
  std::vector<uint32_t> fo;
  std::vector<float> cuts;
  const size_t cells = (size_t)n_rows * n_cols;
  const uint64_t words = (n_rows + 63) / 64;
  auto fail = [&](cudaError_t e, const char* what) {
    why = std::string(what) + ": " + cudaGetErrorString(e);
    return HB_DEVICE_FAILED;
  };
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d_x, 4 * cells);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_x, x, 4 * cells, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) st = fail(e, "upload");
  if (st == HB_OK) st = hb::sketch_dense_cuts(device, d_x, n_rows, n_cols, max_bin, s, fo, cuts, why);
  if (st == HB_OK && columns) {
    e = cudaMalloc(&d_col, cells);
    if (e == cudaSuccess && missing) e = cudaMalloc(&d_miss, 8 * (size_t)n_cols * words);
    if (e == cudaSuccess) e = cudaMalloc(&d_fo, 4 * fo.size());
    if (e == cudaSuccess) e = cudaMalloc(&d_cuts, 4 * std::max<size_t>(cuts.size(), 1));
    if (e == cudaSuccess) e = cudaMalloc(&d_any, 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_fo, fo.data(), 4 * fo.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_cuts, cuts.data(), 4 * cuts.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = hb::bin_dense_device(d_x, n_rows, n_cols, d_fo, d_cuts, d_col, d_miss, d_any, s);
    int any = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(columns, d_col, cells, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && missing)
      e = cudaMemcpyAsync(missing, d_miss, 8 * (size_t)n_cols * words, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&any, d_any, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = fail(e, "binning");
    else *dense = any ? 0 : 1;
  }
  if (s) cudaStreamSynchronize(s);
  cudaFree(d_x);
  cudaFree(d_col);
  cudaFree(d_miss);
  cudaFree(d_fo);
  cudaFree(d_cuts);
  cudaFree(d_any);
  if (s) cudaStreamDestroy(s);
  if (st == HB_OK) st = copy_cuts_out(fo, cuts, n_cols, feature_offset, cut_values, cap, total);
  g_sketch_error = why;
  return st;
}

hb_status hb_sketch_csr(int32_t device, const uint64_t* indptr, const uint32_t* indices,
                        const float* values, uint64_t n_rows, uint32_t n_cols, uint32_t max_bin,
                        uint32_t* feature_offset, float* cut_values, uint64_t cap, uint64_t* total,
                        uint32_t* row_bins, int32_t* dense) {
  if (!indptr || !feature_offset || !cut_values || !total || n_rows == 0 || n_cols == 0 ||
      max_bin == 0 || indptr[0] != 0 || (row_bins && !dense))
    return HB_INVALID_ARGUMENT;
  const uint64_t nnz = indptr[n_rows];
  if (nnz && (!indices || !values)) return HB_INVALID_ARGUMENT;
  DevicePick pick(device);
  std::string why;
  cudaStream_t s = nullptr;
  uint64_t* d_ip = nullptr;
  uint32_t* d_ix = nullptr;
  float* d_v = nullptr;
  uint32_t* d_bins = nullptr;
  uint32_t* d_fo = nullptr;
  float* d_cuts = nullptr;
  int* d_flags = nullptr;
  hb_status st = HB_OK;
  std::vector<uint32_t> fo;
  std::vector<float> cuts;
  auto fail = [&](cudaError_t e, const char* what) {
    why = std::string(what) + ": " + cudaGetErrorString(e);
    return HB_DEVICE_FAILED;
  };
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d_ip, 8 * (n_rows + 1));
  if (e == cudaSuccess) e = cudaMalloc(&d_ix, 4 * std::max<uint64_t>(nnz, 1));
  if (e == cudaSuccess) e = cudaMalloc(&d_v, 4 * std::max<uint64_t>(nnz, 1));
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_ip, indptr, 8 * (n_rows + 1), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && nnz) e = cudaMemcpyAsync(d_ix, indices, 4 * nnz, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && nnz) e = cudaMemcpyAsync(d_v, values, 4 * nnz, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) st = fail(e, "upload");
  if (st == HB_OK)
    st = hb::sketch_csr_cuts(device, d_ip, d_ix, d_v, n_rows, n_cols, nnz, max_bin, s, fo, cuts, why);
  if (st == HB_OK && row_bins) {
    e = cudaMalloc(&d_bins, 4 * std::max<uint64_t>(nnz, 1));
    if (e == cudaSuccess) e = cudaMalloc(&d_fo, 4 * fo.size());
    if (e == cudaSuccess) e = cudaMalloc(&d_cuts, 4 * std::max<size_t>(cuts.size(), 1));
    if (e == cudaSuccess) e = cudaMalloc(&d_flags, 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_fo, fo.data(), 4 * fo.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_cuts, cuts.data(), 4 * cuts.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
      e = hb::bin_csr_device(d_ip, d_ix, d_v, n_rows, n_cols, nnz, d_fo, d_cuts, d_bins, d_flags, s);
    int hf = 0;
    if (e == cudaSuccess && nnz) e = cudaMemcpyAsync(row_bins, d_bins, 4 * nnz, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&hf, d_flags, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = fail(e, "binning");
    else *dense = (hf & 4) ? 0 : 1;
  }
  if (s) cudaStreamSynchronize(s);
  cudaFree(d_ip);
  cudaFree(d_ix);
  cudaFree(d_v);
  cudaFree(d_bins);
  cudaFree(d_fo);
  cudaFree(d_cuts);
  cudaFree(d_flags);
  if (s) cudaStreamDestroy(s);
  if (st == HB_OK) st = copy_cuts_out(fo, cuts, n_cols, feature_offset, cut_values, cap, total);
  g_sketch_error = why;
  return st;
}

}  // extern "C"
