// CUDA kernels of the hist path for sm_100a.
//
// Built with -fmad=false: every f32/f64 expression below is evaluated with
// one IEEE rounding per operation, as the reference's Rust does, and the
// only fused multiply-adds are the explicit __fmaf_rn of the reference's
// own vector exponential.
#include <cub/block/block_scan.cuh>
#include <cuda_pipeline.h>
#include <cub/block/block_reduce.cuh>

#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <climits>
#include <cmath>
#include <utility>
#include <vector>

#include "hb_kernels.cuh"

namespace hb {

bool g_pdl = true;

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr float kBelowAll = -FLT_MAX;         // src/tree/builder/mod.rs:308
constexpr double kRtEps = 1e-6;               // src/lib.rs:366

__device__ __forceinline__ double ll2d(long long v) { return __ll2double_rn(v); }

// Word k (0..7) of a 32-byte record held as two uint4.
__device__ __forceinline__ uint32_t pick_word(const uint4& a, const uint4& b, int k) {
  uint32_t w = a.x;
  w = k == 1 ? a.y : w;
  w = k == 2 ? a.z : w;
  w = k == 3 ? a.w : w;
  w = k == 4 ? b.x : w;
  w = k == 5 ? b.y : w;
  w = k == 6 ? b.z : w;
  w = k == 7 ? b.w : w;
  return w;
}


// L2 eviction priority of the (g, h) pairs: every histogram launch of a
// round gathers them again, so they are written, and may be prefetched,
// evict-last.
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void st_hint8(float2* ptr, float2 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(ptr), "f"(v.x), "f"(v.y), "l"(pol)
               : "memory");
}

// ---------------------------------------------------------------------------
// Objectives.

// src/simd/x86_64.rs:20 `exp_f32`: range reduction to [-ln2/2, ln2/2] and a
// seventh-order polynomial in Estrin pairs, operation for operation.
__device__ __forceinline__ float exp_vector(float v) {
  const float log2e = 1.44269504088896340736f;
  float t = __fmul_rn(v, log2e);
  int e = __float2int_rn(t);
  float ef = __int2float_rn(e);
  float r = __fmaf_rn(-ef, 0.6933594f, v);
  r = __fmaf_rn(ef, 2.1219444e-4f, r);
  float sq = __fmul_rn(r, r);
  float fo = __fmul_rn(sq, sq);
  float p0 = __fadd_rn(1.0f, r);
  float p1 = __fmaf_rn(1.0f / 6.0f, r, 0.5f);
  float p2 = __fmaf_rn(1.0f / 120.0f, r, 1.0f / 24.0f);
  float p3 = __fmaf_rn(1.0f / 5040.0f, r, 1.0f / 720.0f);
  float lo = __fmaf_rn(p1, sq, p0);
  float hi = __fmaf_rn(p3, sq, p2);
  float poly = __fmaf_rn(hi, fo, lo);
  float scale = __int_as_float((e + 127) << 23);
  return __fmul_rn(poly, scale);
}

// src/simd/x86_64.rs:63 `sigmoid_f32`
__device__ __forceinline__ float sigmoid_vector(float v) {
  float e = exp_vector(__fsub_rn(0.0f, fabsf(v)));
  float den = __fadd_rn(1.0f, e);
  // 1 / den for v >= 0, e / den otherwise: one correctly rounded division of
  // the selected numerator (the same result as dividing both and selecting)
  return __fdiv_rn(v >= 0.0f ? 1.0f : e, den);
}

// src/simd/mod.rs:421 `sigmoid_scalar`, 1 / (expf(min(-x, 88.7)) + 1). The
// exponential is CUDA's double exp rounded once to f32 (the correctly
// rounded expf except where the double result lies within one double ulp
// of an f32 rounding boundary).
__device__ __forceinline__ float sigmoid_scalar(float x) {
  float t = fminf(-x, 88.7f);
  float e = __double2float_rn(exp((double)t));
  return __fdiv_rn(1.0f, __fadd_rn(e, 1.0f));
}

__device__ __forceinline__ void fold_max(float g, float h, float& mg, float& mh, bool& nonfinite) {
  if (!isfinite(g) || !isfinite(h)) nonfinite = true;
  mg = fmaxf(mg, fabsf(g));
  mh = fmaxf(mh, fabsf(h));
}

__device__ __forceinline__ void reduce_scale(float mg, float mh, bool nonfinite, Scale* scale) {
  for (int o = 16; o > 0; o >>= 1) {
    mg = fmaxf(mg, __shfl_xor_sync(kFull, mg, o));
    mh = fmaxf(mh, __shfl_xor_sync(kFull, mh, o));
  }
  unsigned nf = __ballot_sync(kFull, nonfinite);
  if ((threadIdx.x & 31) == 0) {
    if (mg > 0.0f) atomicMax(&scale->maxg_bits, __float_as_uint(mg));
    if (mh > 0.0f) atomicMax(&scale->maxh_bits, __float_as_uint(mh));
    if (nf) atomicOr(&scale->nonfinite, 1u);
  }
}

// Gradients (one thread per row, grid-stride in whole warps):
//  * reg:squarederror (src/objective/regression.rs:50): g = (p - y) w, h = w,
//    w scaled by scale_pos_weight when y == 1;
//  * binary:logistic (src/simd/x86_64.rs:106 + scalar.rs:8): over the first
//    `vrows` rows (n - n % 8 for n >= 16, objective/mod.rs:195) every aligned
//    group of 8 margins whose magnitudes are all <= 80 takes the vector
//    sigmoid, any other group and the tail the scalar one.
// The leaf of a 32-byte record held in registers (at most 28 features: one
// mask word, word `mask_word` of the record).
__device__ __forceinline__ float walk_leaf_rec32(const WNode* __restrict__ t, const uint4& a, const uint4& b,
                                                 uint32_t mask_word) {
  const uint32_t m = pick_word(a, b, (int)mask_word);
  WNode nd = t[0];
  while (nd.left >= 0) {
    const uint32_t f = nd.feature & 0x7fffffffu;
    const bool miss = (m >> f) & 1u;
    const uint32_t bin = (pick_word(a, b, (int)(f >> 2)) >> ((f & 3) * 8)) & 0xffu;
    const bool left = miss ? (nd.feature >> 31) != 0u : bin < nd.limit;
    nd = t[nd.left + (left ? 0 : 1)];
  }
  return nd.leaf;
}

// The leaf of row r in the walked tree (WNode, staged in shared memory).
__device__ __forceinline__ float walk_leaf(const WNode* __restrict__ t, const uint8_t* __restrict__ rp,
                                           uint32_t stride, uint32_t mask_off) {
  if (stride == 32 && mask_off <= 28)
    return walk_leaf_rec32(t, *reinterpret_cast<const uint4*>(rp), *reinterpret_cast<const uint4*>(rp + 16),
                           mask_off >> 2);
  WNode nd = t[0];
  while (nd.left >= 0) {
    const uint32_t f = nd.feature & 0x7fffffffu;
    const uint32_t m = *reinterpret_cast<const uint32_t*>(rp + mask_off + 4 * (f >> 5));
    const bool miss = (m >> (f & 31)) & 1u;
    const bool left = miss ? (nd.feature >> 31) != 0u : (uint32_t)rp[f] < nd.limit;
    nd = t[nd.left + (left ? 0 : 1)];
  }
  return nd.leaf;
}

__device__ __forceinline__ void stage_tree(const WNode* __restrict__ wtree, const LevelState* ls_last,
                                           WNode* s_tree) {
  const int n = ls_last->n_nodes;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_tree[i] = wtree[i];
  __syncthreads();
}

// The local bin of feature [lo, hi) (global bins) in a CSR row, whose bins
// ascend: the first entry >= lo, present when it is below hi.
__device__ __forceinline__ bool csr_find(const uint32_t* __restrict__ bins, uint64_t a, uint64_t b,
                                         uint32_t lo, uint32_t hi, uint32_t& local) {
  uint64_t e = b;
  while (a < e) {
    const uint64_t m = (a + e) >> 1;
    if (__ldg(bins + m) < lo) a = m + 1; else e = m;
  }
  if (a < b) {
    const uint32_t v = __ldg(bins + a);
    if (v < hi) {
      local = v - lo;
      return true;
    }
  }
  return false;
}

// The leaf a CSR row reaches in one tree (the partition's routing rule:
// local bin < limit goes left, missing follows default_left).
__device__ __forceinline__ float walk_leaf_csr(const WNode* __restrict__ t, const DevConst& c,
                                               uint64_t a, uint64_t b) {
  WNode nd = t[0];
  while (nd.left >= 0) {
    const uint32_t f = nd.feature & 0x7fffffffu;
    uint32_t bin = 0;
    const bool present = csr_find(c.csr_bins, a, b, __ldg(c.fo + f), __ldg(c.fo + f + 1), bin);
    const bool left = present ? bin < nd.limit : (nd.feature >> 31) != 0u;
    nd = t[nd.left + (left ? 0 : 1)];
  }
  return nd.leaf;
}

// The same leaf read from the feature-major copy of the index: one byte and
// one bitmap bit per split instead of a binary search.
__device__ __forceinline__ float walk_leaf_cols(const WNode* __restrict__ t, const DevConst& c,
                                                uint64_t r, uint64_t words) {
  WNode nd = t[0];
  while (nd.left >= 0) {
    const uint64_t f = nd.feature & 0x7fffffffu;
    const bool miss = c.csr_colmiss && ((__ldg(c.csr_colmiss + f * words + (r >> 6)) >> (r & 63)) & 1ull);
    const bool left = miss ? (nd.feature >> 31) != 0u : __ldg(c.csr_col + f * c.n_rows + r) < nd.limit;
    nd = t[nd.left + (left ? 0 : 1)];
  }
  return nd.leaf;
}

// The pending trees' leaves (K outputs, trees wstride nodes apart, margins
// class-major) added to the margins of CSR rows, when the flag says a tree
// waits.
template <bool COLS>
__global__ void k_walk_csr(DevConst c, int K, const WNode* __restrict__ wtree, uint32_t wstride,
                           float* __restrict__ margin, const int* __restrict__ pending) {
  pdl_wait();
  if (!*pending) return;
  const uint64_t n = c.n_rows, words = (n + 63) / 64;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t a = 0, b = 0;
    if (!COLS) {
      a = c.csr_ptr[i];
      b = c.csr_ptr[i + 1];
    }
    for (int k = 0; k < K; ++k) {
      float* m = margin + (uint64_t)k * n + i;
      const WNode* t = wtree + (uint64_t)k * wstride;
      *m = __fadd_rn(*m, COLS ? walk_leaf_cols(t, c, i, words) : walk_leaf_csr(t, c, a, b));
    }
  }
}

// The feature-major copy of a CSR index: thread per row, each stored cell's
// feature found by a binary search of the feature offsets (the row's bins
// ascend, so the search starts at the last cell's feature). Only a
// feature's first cell is written, the one csr_find returns. `col` zeroed
// and `colmiss` all ones beforehand; the bitmap's words are shared by 64
// rows, hence the atomics.
__global__ void k_csr_columns(DevConst c, uint8_t* __restrict__ col,
                              unsigned long long* __restrict__ colmiss) {
  const uint64_t n = c.n_rows, words = (n + 63) / 64;
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t a = c.csr_ptr[r], b = c.csr_ptr[r + 1];
    uint32_t f = 0;
    int prev = -1;
    for (uint64_t j = a; j < b; ++j) {
      const uint32_t gb = __ldg(c.csr_bins + j);
      uint32_t lo = f, hi = c.n_cols - 1;  // the last feature whose first bin is <= gb
      while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) >> 1;
        if (__ldg(c.fo + mid) <= gb) lo = mid; else hi = mid - 1;
      }
      f = lo;
      if ((int)f == prev) continue;
      prev = (int)f;
      col[(uint64_t)f * n + r] = (uint8_t)(gb - __ldg(c.fo + f));
      if (colmiss) atomicAnd(colmiss + (uint64_t)f * words + (r >> 6), ~(1ull << (r & 63)));
    }
  }
}

// Add the previous tree's leaves to the margins: each row walks the tree
// over its binned record (the partition's routing rule), in row order.
__global__ void k_walk(const WNode* __restrict__ wtree, const LevelState* __restrict__ ls_last,
                       const uint8_t* __restrict__ rec, uint32_t stride, uint32_t mask_off, uint32_t blk,
                       uint64_t n, float* __restrict__ margin, const int* __restrict__ pending) {
  extern __shared__ WNode s_tree[];
  if (!*pending) return;
  stage_tree(wtree, ls_last, s_tree);
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    margin[i] = __fadd_rn(margin[i], walk_leaf(s_tree, rec + rec_offset((uint32_t)i, stride, blk), stride,
                                               mask_off));
  }
}

__global__ void k_gradients(int kind, float* __restrict__ margin,
                            const float* __restrict__ label, const float* __restrict__ weight,
                            float spw, float min_hess, uint64_t n, uint64_t vrows,
                            float2* __restrict__ gpair, Scale* scale, const WNode* __restrict__ wtree,
                            const LevelState* __restrict__ ls_last, uint8_t* rec,
                            uint32_t stride, uint32_t mask_off, uint32_t blk, uint32_t blk_pair,
                            const int* __restrict__ pending) {
  pdl_wait();
  extern __shared__ WNode s_tree[];
  if (wtree && !(pending && *pending)) wtree = nullptr;  // no tree waiting for the margins
  if (wtree) stage_tree(wtree, ls_last, s_tree);
  // the round's histogram launches re-read the pairs: from the row blocks
  // when there are any (blk_pair != 0), else from gpair, kept in L2
  const uint64_t pol_keep = l2_evict_last();
  float mg = 0.0f, mh = 0.0f;
  bool nonfinite = false;
  const unsigned lane = threadIdx.x & 31;
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x; base < n; base += step) {
    uint64_t i = base + threadIdx.x;
    bool in = i < n;
    float m = in ? margin[i] : 0.0f;
    if (wtree && in) {
      m = __fadd_rn(m, walk_leaf(s_tree, rec + rec_offset((uint32_t)i, stride, blk), stride, mask_off));
      margin[i] = m;
    }
    float y = in ? label[i] : 0.0f;
    float w = (in && weight) ? weight[i] : 1.0f;
    float g = 0.0f, h = 0.0f;
    if (kind == HB_LOSS_LOGISTIC) {
      bool regular = fabsf(m) <= 80.0f;
      unsigned bal = __ballot_sync(kFull, regular || !in);
      bool group_regular = ((bal >> (lane & ~7u)) & 0xffu) == 0xffu;
      float p = (i < vrows && group_regular) ? sigmoid_vector(m) : sigmoid_scalar(m);
      if (y == 1.0f) w = __fmul_rn(w, spw);
      g = __fmul_rn(__fsub_rn(p, y), w);
      float ph = __fmul_rn(p, __fsub_rn(1.0f, p));
      h = __fmul_rn(ph > min_hess ? ph : min_hess, w);
    } else {
      if (y == 1.0f) w = __fmul_rn(w, spw);
      g = __fmul_rn(__fsub_rn(m, y), w);
      h = w;
    }
    if (in) {
      if (blk_pair) {
        // the pair into its row block; the block's last row also writes the
        // zero tail of the line, so every sector of the pairs is written whole
        gpair[i] = make_float2(g, h);
        const uint32_t q = block_of((uint32_t)i, blk), j = (uint32_t)i - q * blk;
        uint8_t* line = rec + (uint64_t)q * kBlockBytes;
        *reinterpret_cast<float2*>(line + blk_pair + 8u * j) = make_float2(g, h);
        if (j == blk - 1u)
          for (uint32_t o = blk_pair + 8u * blk; o < kBlockBytes; o += 8u)
            *reinterpret_cast<uint2*>(line + o) = make_uint2(0u, 0u);
      } else {
        st_hint8(gpair + i, make_float2(g, h), pol_keep);
      }
      fold_max(g, h, mg, mh, nonfinite);
    }
  }
  reduce_scale(mg, mh, nonfinite, scale);
}

// The same gradients over row blocks of three 32-byte records (13 to 28
// features, one output), one thread per 128-byte block. Each thread issues
// its three rows' loads (the whole line of records, three margins, three
// labels) before using any. A tree of depth D <= kCtMaxDepth (ct_depth) is
// walked as a complete tree, re-laid per CTA in shared memory: position p's
// children are 2p + 1 and 2p + 2, a leaf above depth D passes every row on
// to children that carry its value, so a walk is D steps of one node load
// and one byte load (the record copied to shared memory) with no branch;
// deeper trees (ct_depth = 0) walk the nodes from registers. The leaf is
// the one the pointer walk reaches, bit for bit. A warp covers 96
// consecutive rows, so every aligned group of 8 rows (the logistic vector
// groups) lies within it; a row's group flag gathers the regular-margin
// flags of the (at most four) lanes holding the group's rows.
constexpr int kCtMaxDepth = 10;
constexpr int kGradThreads = 256;
constexpr int kRecPitch = 100;  // bytes of a thread's three staged records (25 words: no bank repeats)

size_t gradients_b3_smem(int max_nodes, int ct_depth) {
  size_t b = sizeof(WNode) * (size_t)max_nodes;
  if (ct_depth > 0) {
    const size_t inner = (size_t(1) << ct_depth) - 1;
    b += 4 * inner + 4 * (inner + 1) + 2 * (2 * inner + 1) + (size_t)kGradThreads * kRecPitch;
    b = (b + 15) / 16 * 16;
  }
  return b;
}

__global__ void __launch_bounds__(kGradThreads, 4)
    k_gradients_b3(int kind, float* __restrict__ margin, const float* __restrict__ label,
                   const float* __restrict__ weight, float spw, float min_hess, uint64_t n, uint64_t vrows,
                   float2* __restrict__ gpair, Scale* scale, const WNode* __restrict__ wtree,
                   const LevelState* __restrict__ ls_last, int max_nodes, int ct_depth,
                   uint8_t* __restrict__ rec, uint32_t mask_word, const int* __restrict__ pending) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char s_dyn[];
  WNode* s_tree = reinterpret_cast<WNode*>(s_dyn);
  if (wtree && !(pending && *pending)) wtree = nullptr;  // no tree waiting for the margins
  const int D = ct_depth;
  const uint32_t inner = D > 0 ? (1u << D) - 1u : 0u;
  // [inner]: feature | min(limit, 256) << 8 | dl << 31 (the records hold at
  // most 28 features of 8-bit bins, so one word a node: one shared wavefront
  // a step)
  uint32_t* s_ct = reinterpret_cast<uint32_t*>(s_tree + max_nodes);
  float* s_leaf = reinterpret_cast<float*>(s_ct + inner);           // [inner + 1]
  int16_t* s_pos = reinterpret_cast<int16_t*>(s_leaf + inner + 1);  // [2 inner + 1]: node of a position
  uint8_t* s_rec = reinterpret_cast<uint8_t*>(s_pos + 2 * inner + 1) + 0;
  s_rec = reinterpret_cast<uint8_t*>(((uintptr_t)s_rec + 15) & ~(uintptr_t)15);
  if (wtree) {
    stage_tree(wtree, ls_last, s_tree);
    if (D > 0) {
      if (threadIdx.x == 0) s_pos[0] = 0;
      __syncthreads();
      for (int d = 0; d < D; ++d) {
        for (uint32_t p = (1u << d) - 1 + threadIdx.x; p < (2u << d) - 1; p += blockDim.x) {
          const int k = s_pos[p];
          const WNode nd = s_tree[k];
          if (nd.left >= 0) {
            s_ct[p] = (nd.feature & 0x800000ffu) | (min(nd.limit, 256u) << 8);
            s_pos[2 * p + 1] = (int16_t)nd.left;
            s_pos[2 * p + 2] = (int16_t)(nd.left + 1);
          } else {  // a leaf: both children carry it
            s_ct[p] = 0u;
            s_pos[2 * p + 1] = (int16_t)k;
            s_pos[2 * p + 2] = (int16_t)k;
          }
        }
        __syncthreads();
      }
      for (uint32_t p = threadIdx.x; p <= inner; p += blockDim.x) s_leaf[p] = s_tree[s_pos[inner + p]].leaf;
      __syncthreads();
    }
  }
  float mg = 0.0f, mh = 0.0f;
  bool nonfinite = false;
  const unsigned lane = threadIdx.x & 31;
  uint8_t* my_rec = s_rec + threadIdx.x * kRecPitch;
  // row indices in 32 bits (an engine holds fewer than 2^32 rows)
  const uint32_t n32 = (uint32_t)n, v32 = (uint32_t)vrows;
  const uint32_t nblk = (n32 + 2u) / 3u;
  const uint32_t step = gridDim.x * blockDim.x;
  // this lane's rows' logistic vector groups: for row j, the first of the
  // (at most four) lanes holding its group, and the group's offset in them
  uint32_t g_lane[3], g_off[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint32_t gs = (3u * lane + j) & ~7u;  // the group's first row within the warp's 96
    g_lane[j] = gs / 3u;
    g_off[j] = gs - 3u * g_lane[j];
  }
  // the loop bound is per warp (its first block), so shuffles see every lane
  for (uint32_t w0 = blockIdx.x * blockDim.x + (threadIdx.x & ~31u); w0 < nblk; w0 += step) {
    const uint32_t q = w0 + lane;
    const uint32_t r0 = 3u * q;
    uint8_t* line = rec + (uint64_t)q * kBlockBytes;
    uint4 L[6];
    float m[3], y[3], w[3];
    if (wtree && D > 0) {
      // The warp's 32 row blocks, 96 record bytes each, loaded in block
      // order: chunk c = lane + 32 k is 16-byte part c % 6 of block c / 6,
      // so a load reads about six blocks instead of 32 (one a lane). Each
      // chunk then goes to its block's staging row.
      const uint32_t nl = min(32u, nblk - w0);
      const uint4* gsrc = reinterpret_cast<const uint4*>(rec + (uint64_t)w0 * kBlockBytes);
      uint8_t* wrec = s_rec + (threadIdx.x & ~31u) * kRecPitch;
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const uint32_t cq = lane + 32u * k, li = cq / 6u;
        if (li < nl) L[k] = gsrc[li * (kBlockBytes / 16u) + (cq - 6u * li)];
      }
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const uint32_t cq = lane + 32u * k, li = cq / 6u;
        if (li < nl) {
          uint32_t* d = reinterpret_cast<uint32_t*>(wrec + li * kRecPitch + 16u * (cq - 6u * li));
          d[0] = L[k].x;
          d[1] = L[k].y;
          d[2] = L[k].z;
          d[3] = L[k].w;
        }
      }
    } else if (wtree && q < nblk) {
#pragma unroll
      for (int k = 0; k < 6; ++k) L[k] = reinterpret_cast<const uint4*>(line)[k];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const bool in = r0 + j < n32;
      m[j] = in ? margin[r0 + j] : 0.0f;
      y[j] = in ? label[r0 + j] : 0.0f;
      w[j] = (in && weight) ? weight[r0 + j] : 1.0f;
    }
    if (wtree && D > 0) {
      __syncwarp();
      // the three walks step together (independent chains of shared loads)
      uint32_t msk[3], idx[3] = {0u, 0u, 0u};
#pragma unroll
      for (int j = 0; j < 3; ++j) msk[j] = reinterpret_cast<const uint32_t*>(my_rec + 32 * j)[mask_word];
      for (int d = 0; d < D; ++d) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const uint32_t cn = s_ct[idx[j]];
          const uint32_t f = cn & 0xffu;
          const bool miss = (msk[j] >> f) & 1u;
          const bool left = miss ? (cn >> 31) != 0u : (uint32_t)my_rec[32 * j + f] < ((cn >> 8) & 0x1ffu);
          idx[j] = 2 * idx[j] + (left ? 1u : 2u);
        }
      }
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        if (r0 + j < n32) {
          m[j] = __fadd_rn(m[j], s_leaf[idx[j] - inner]);
          margin[r0 + j] = m[j];
        }
      }
      __syncwarp();
    } else if (wtree) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        if (r0 + j < n32) {
          m[j] = __fadd_rn(m[j], walk_leaf_rec32(s_tree, L[2 * j], L[2 * j + 1], mask_word));
          margin[r0 + j] = m[j];
        }
      }
    }
    float g[3], h[3];
    if (kind == HB_LOSS_LOGISTIC) {
      uint32_t f = 0;
#pragma unroll
      for (int j = 0; j < 3; ++j) f |= (fabsf(m[j]) <= 80.0f || r0 + j >= n32) ? (1u << j) : 0u;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        uint32_t cat = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) cat |= __shfl_sync(kFull, f, min(g_lane[j] + k, 31u)) << (3 * k);
        const bool group_regular = ((cat >> g_off[j]) & 0xffu) == 0xffu;
        const float p = (r0 + j < v32 && group_regular) ? sigmoid_vector(m[j]) : sigmoid_scalar(m[j]);
        float wj = w[j];
        if (y[j] == 1.0f) wj = __fmul_rn(wj, spw);
        g[j] = __fmul_rn(__fsub_rn(p, y[j]), wj);
        const float ph = __fmul_rn(p, __fsub_rn(1.0f, p));
        h[j] = __fmul_rn(ph > min_hess ? ph : min_hess, wj);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        float wj = w[j];
        if (y[j] == 1.0f) wj = __fmul_rn(wj, spw);
        g[j] = __fmul_rn(__fsub_rn(m[j], y[j]), wj);
        h[j] = wj;
      }
    }
    if (q < nblk) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        if (r0 + j < n32) {
          gpair[r0 + j] = make_float2(g[j], h[j]);
          fold_max(g[j], h[j], mg, mh, nonfinite);
        } else {
          g[j] = h[j] = 0.0f;
        }
      }
      uint4* ps = reinterpret_cast<uint4*>(line + 96);
      ps[0] = make_uint4(__float_as_uint(g[0]), __float_as_uint(h[0]), __float_as_uint(g[1]), __float_as_uint(h[1]));
      ps[1] = make_uint4(__float_as_uint(g[2]), __float_as_uint(h[2]), 0u, 0u);
    }
  }
  reduce_scale(mg, mh, nonfinite, scale);
}

// multi:softmax gradients (objective/multiclass.rs:43), the reference's
// per-row scalar kernel (simd/mod.rs:580), which x86_64 runs for every class
// count but 2 and 4: shift = max(f32::MIN_POSITIVE, margins...), the
// exponentials summed in f64 and the sum rounded to f32, p = exp(m - shift)
// / sum, g = p - [class == label], h = max((2 p)(1 - p), min_hess). exp is
// CUDA's double exp rounded once to f32 (as in sigmoid_scalar). Margins and
// pairs are class-major ([class][row]); with *pending set each row first
// adds its leaf of each class's tree (wtree + class * wstride, read from
// global memory) to that class's margin. Per-class |g|, |h| maxima and a
// non-finite flag go to scale[class].
constexpr int kMaxClasses = 64;

__device__ __forceinline__ float exp_rounded(float t) { return __double2float_rn(exp((double)t)); }

__global__ void k_softmax_gradients(int K, float* __restrict__ margin, const float* __restrict__ label,
                                    uint64_t n, float min_hess, float2* __restrict__ gpair,
                                    Scale* scale, const WNode* __restrict__ wtree, uint32_t wstride,
                                    const uint8_t* __restrict__ rec, uint32_t stride,
                                    uint32_t mask_off, uint32_t blk, const int* __restrict__ pending) {
  pdl_wait();
  __shared__ unsigned s_mg[kMaxClasses], s_mh[kMaxClasses], s_nf[kMaxClasses];
  for (int j = threadIdx.x; j < K; j += blockDim.x) s_mg[j] = s_mh[j] = s_nf[j] = 0u;
  __syncthreads();
  const bool walk = pending != nullptr && *pending != 0;
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const uint8_t* rp = rec + rec_offset((uint32_t)i, stride, blk);
    float wmax = FLT_MIN;
    for (int j = 0; j < K; ++j) {
      float v = margin[(uint64_t)j * n + i];
      if (walk) {
        v = __fadd_rn(v, walk_leaf(wtree + (uint64_t)j * wstride, rp, stride, mask_off));
        margin[(uint64_t)j * n + i] = v;
      }
      wmax = fmaxf(v, wmax);
    }
    double wsum = 0.0;
    for (int j = 0; j < K; ++j) wsum += (double)exp_rounded(__fsub_rn(margin[(uint64_t)j * n + i], wmax));
    const float ws = __double2float_rn(wsum);
    const float y = label[i];
    for (int j = 0; j < K; ++j) {
      const float p = __fdiv_rn(exp_rounded(__fsub_rn(margin[(uint64_t)j * n + i], wmax)), ws);
      const float h = fmaxf(__fmul_rn(__fmul_rn(2.0f, p), __fsub_rn(1.0f, p)), min_hess);
      const float g = (float)j == y ? __fsub_rn(p, 1.0f) : p;
      gpair[(uint64_t)j * n + i] = make_float2(g, h);
      if (!isfinite(g) || !isfinite(h)) atomicOr(&s_nf[j], 1u);
      atomicMax(&s_mg[j], __float_as_uint(fabsf(g)));
      atomicMax(&s_mh[j], __float_as_uint(fabsf(h)));
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < K; j += blockDim.x) {
    if (s_mg[j]) atomicMax(&scale[j].maxg_bits, s_mg[j]);
    if (s_mh[j]) atomicMax(&scale[j].maxh_bits, s_mh[j]);
    if (s_nf[j]) atomicOr(&scale[j].nonfinite, 1u);
  }
}

// `_mm256_max_ps` / `_mm256_min_ps`: the second operand unless the first is
// strictly greater (smaller), so a NaN in either gives the second.
__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ float minps(float a, float b) { return a < b ? a : b; }

// One row of K = 2 or 4 margins through x86_64.rs:191 `short_softmax_batch`:
// row maximum and minimum by `row_reduce` (x86_64.rs:167: lane j takes
// op(v[j], v[j ^ 1]), then for K = 4 op(r[j], r[j ^ 2])), shift =
// maxps(MIN_POSITIVE, max); false when max - min <= 80 fails in a lane
// (non-finite or wide: the row's vector takes the scalar path), otherwise
// p[j] = exp_f32(v[j] - shift) * (1 / sum), the sum reduced the same way.
template <int K>
__device__ __forceinline__ bool softmax_short_row(const float (&v)[K], float (&p)[K]) {
  float mx[K], mn[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    mx[j] = maxps(v[j], v[j ^ 1]);
    mn[j] = minps(v[j], v[j ^ 1]);
  }
  if (K == 4) {
    float t[K], u[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      t[j] = maxps(mx[j], mx[j ^ (K == 4 ? 2 : 0)]);
      u[j] = minps(mn[j], mn[j ^ (K == 4 ? 2 : 0)]);
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      mx[j] = t[j];
      mn[j] = u[j];
    }
  }
  bool regular = true;
  float e[K], sum[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const float shift = maxps(FLT_MIN, mx[j]);
    regular = regular && __fsub_rn(shift, mn[j]) <= 80.0f;
    e[j] = exp_vector(__fsub_rn(v[j], shift));
  }
#pragma unroll
  for (int j = 0; j < K; ++j) sum[j] = __fadd_rn(e[j], e[j ^ 1]);
  if (K == 4) {
    float t[K];
#pragma unroll
    for (int j = 0; j < K; ++j) t[j] = __fadd_rn(sum[j], sum[j ^ (K == 4 ? 2 : 0)]);
#pragma unroll
    for (int j = 0; j < K; ++j) sum[j] = t[j];
  }
#pragma unroll
  for (int j = 0; j < K; ++j) p[j] = __fmul_rn(e[j], __fdiv_rn(1.0f, sum[j]));
  return regular;
}

// multi:softmax gradients for 2 and 4 classes, which x86_64 computes with
// x86_64.rs:273 `short_softmax_gradient` (simd/mod.rs:156): 8-lane vectors
// of 8 / K whole rows over the first `vrows` rows (n - n % (8 / K) of the
// whole matrix when it holds at least 16 margins, MIN_SIMD_LEN,
// simd/mod.rs:28), a vector holding an irregular row on the scalar path
// (the flags of its rows' lanes gathered with a ballot), every other row
// scalar (k_softmax_gradients' rule). Vector rows: g = p - [class ==
// label], h = maxps((p 2)(1 - p), min_hess). Layout, leaf walk and maxima
// as in k_softmax_gradients.
template <int K>
__global__ void k_softmax_short(float* __restrict__ margin, const float* __restrict__ label, uint64_t n,
                                uint64_t vrows, float min_hess, float2* __restrict__ gpair, Scale* scale,
                                const WNode* __restrict__ wtree, uint32_t wstride,
                                const uint8_t* __restrict__ rec, uint32_t stride, uint32_t mask_off,
                                uint32_t blk, const int* __restrict__ pending) {
  pdl_wait();
  constexpr unsigned kRows = 8 / K;  // rows of one vector
  constexpr unsigned kMask = (1u << kRows) - 1u;
  __shared__ unsigned s_mg[K], s_mh[K], s_nf[K];
  if (threadIdx.x < K) s_mg[threadIdx.x] = s_mh[threadIdx.x] = s_nf[threadIdx.x] = 0u;
  __syncthreads();
  const bool walk = pending != nullptr && *pending != 0;
  const unsigned lane = threadIdx.x & 31;
  float mg[K], mh[K];
  bool nf[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    mg[j] = mh[j] = 0.0f;
    nf[j] = false;
  }
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x; base < n; base += step) {
    const uint64_t i = base + threadIdx.x;
    const bool in = i < n;
    float v[K];
#pragma unroll
    for (int j = 0; j < K; ++j) v[j] = in ? margin[(uint64_t)j * n + i] : 0.0f;
    if (in && walk) {
      const uint8_t* rp = rec + rec_offset((uint32_t)i, stride, blk);
#pragma unroll
      for (int j = 0; j < K; ++j) {
        v[j] = __fadd_rn(v[j], walk_leaf(wtree + (uint64_t)j * wstride, rp, stride, mask_off));
        margin[(uint64_t)j * n + i] = v[j];
      }
    }
    float p[K];
    const bool regular = softmax_short_row<K>(v, p);
    const unsigned bal = __ballot_sync(kFull, regular || !in);
    const bool vec = i < vrows && ((bal >> (lane & ~(kRows - 1u))) & kMask) == kMask;
    if (!in) continue;
    const float y = label[i];
    float g[K], h[K];
    if (vec) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        g[j] = __fsub_rn(p[j], (float)j == y ? 1.0f : 0.0f);
        h[j] = maxps(__fmul_rn(__fmul_rn(p[j], 2.0f), __fsub_rn(1.0f, p[j])), min_hess);
      }
    } else {
      float wmax = FLT_MIN;
#pragma unroll
      for (int j = 0; j < K; ++j) wmax = fmaxf(v[j], wmax);
      double wsum = 0.0;
#pragma unroll
      for (int j = 0; j < K; ++j) wsum += (double)exp_rounded(__fsub_rn(v[j], wmax));
      const float ws = __double2float_rn(wsum);
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const float q = __fdiv_rn(exp_rounded(__fsub_rn(v[j], wmax)), ws);
        h[j] = fmaxf(__fmul_rn(__fmul_rn(2.0f, q), __fsub_rn(1.0f, q)), min_hess);
        g[j] = (float)j == y ? __fsub_rn(q, 1.0f) : q;
      }
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      gpair[(uint64_t)j * n + i] = make_float2(g[j], h[j]);
      fold_max(g[j], h[j], mg[j], mh[j], nf[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (nf[j]) atomicOr(&s_nf[j], 1u);
    atomicMax(&s_mg[j], __float_as_uint(mg[j]));
    atomicMax(&s_mh[j], __float_as_uint(mh[j]));
  }
  __syncthreads();
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    if (s_mg[j]) atomicMax(&scale[j].maxg_bits, s_mg[j]);
    if (s_mh[j]) atomicMax(&scale[j].maxh_bits, s_mh[j]);
    if (s_nf[j]) atomicOr(&scale[j].nonfinite, 1u);
  }
}

// Add each class's tree leaves to the class-major margins (the last round's
// trees, when *pending is set).
__global__ void k_walk_classes(int K, const WNode* __restrict__ wtree, uint32_t wstride,
                               const uint8_t* __restrict__ rec, uint32_t stride, uint32_t mask_off,
                               uint32_t blk, uint64_t n, float* __restrict__ margin,
                               const int* __restrict__ pending) {
  if (!*pending) return;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint8_t* rp = rec + rec_offset((uint32_t)i, stride, blk);
    for (int j = 0; j < K; ++j)
      margin[(uint64_t)j * n + i] = __fadd_rn(margin[(uint64_t)j * n + i],
                                             walk_leaf(wtree + (uint64_t)j * wstride, rp, stride, mask_off));
  }
}

__global__ void k_pair_maxima(const float2* __restrict__ gpair, uint64_t n, Scale* scale) {
  float mg = 0.0f, mh = 0.0f;
  bool nonfinite = false;
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x; base < n; base += step) {
    uint64_t i = base + threadIdx.x;
    if (i < n) {
      float2 p = gpair[i];
      fold_max(p.x, p.y, mg, mh, nonfinite);
    }
  }
  reduce_scale(mg, mh, nonfinite, scale);
}

// The exponent s with |rint(v * 2^s)| * n <= 2^53 for every |v| <= max:
// every sum of n such values, and so every histogram bin, total and sibling
// difference, is an integer an f64 holds exactly (the f64 ABI then carries
// the fixed-point sums without loss).
__device__ int fixed_scale(float max_abs, uint64_t n) {
  if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 0;
  int e;
  frexpf(max_abs, &e);  // max_abs < 2^e
  int c = 0;
  while (c < 64 && (1ull << c) < n) ++c;
  return kFixedTop - c - e;
}

__device__ __forceinline__ double pow2d(int e) {
  return __longlong_as_double((long long)(1023 + e) << 52);  // e in [-1022, 1023]
}

__global__ void k_scale(Scale* scale, uint64_t global_rows, int* pending) {
  pdl_wait();
  if (pending) *pending = 0;  // the gradient pass before has added the pending tree
  Scale s = *scale;
  s.sg = fixed_scale(__uint_as_float(s.maxg_bits), global_rows);
  s.sh = fixed_scale(__uint_as_float(s.maxh_bits), global_rows);
  s.fg = pow2d(s.sg);
  s.fh = pow2d(s.sh);
  s.ig = pow2d(-s.sg);
  s.ih = pow2d(-s.sh);
  *scale = s;
}

// ---------------------------------------------------------------------------
// Upload: feature-major bins -> row-major records (GHistIndex columns ->
// the layout the histogram gathers).
__global__ void k_encode(const uint8_t* __restrict__ col, const uint64_t* __restrict__ colmiss,
                         uint64_t n_rows, uint32_t n_cols, uint32_t stride, uint32_t mask_off,
                         uint32_t blk, uint8_t* __restrict__ rec) {
  const uint64_t words = (n_rows + 63) / 64;
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t* out = reinterpret_cast<uint32_t*>(rec + rec_offset((uint32_t)r, stride, blk));
    uint32_t word = 0;
    for (uint32_t f = 0; f < n_cols; ++f) {
      word |= (uint32_t)col[(uint64_t)f * n_rows + r] << ((f & 3) * 8);
      if ((f & 3) == 3 || f + 1 == n_cols) {
        out[f >> 2] = word;
        word = 0;
      }
    }
    for (uint32_t b = ((n_cols + 3) / 4) * 4; b < mask_off; b += 4) out[b >> 2] = 0;
    uint32_t n_mask = (n_cols + 31) / 32;
    for (uint32_t w = 0; w < n_mask; ++w) {
      uint32_t m = 0;
      if (colmiss) {
        for (uint32_t f = w * 32; f < min(n_cols, w * 32 + 32); ++f) {
          uint64_t bit = (colmiss[(uint64_t)f * words + (r >> 6)] >> (r & 63)) & 1ull;
          m |= (uint32_t)bit << (f - w * 32);
        }
      }
      out[(mask_off >> 2) + w] = m;
    }
    for (uint32_t b = mask_off + 4 * n_mask; b < stride; b += 4) out[b >> 2] = 0;
  }
}

// ---------------------------------------------------------------------------
// CSR histogram (hist_sparse, src/backend/cuda/train.rs:1029): one warp per
// row, its lanes over the row's entries, each adding the row's fixed-point
// (g, h) to the node's histogram in global memory (L2-resident: total_bins
// x 16 B) with 64-bit reductions. Rows are split over the CTAs as the dense
// kernel splits them (contiguous shares of the entries' concatenation).
constexpr int kCsrThreads = 512;

__global__ void __launch_bounds__(kCsrThreads)
    k_hist_csr(DevConst c, const float2* __restrict__ gpair, const Scale* __restrict__ scale,
               const uint32_t* __restrict__ rows, const HEntry* __restrict__ entries,
               const LevelState* __restrict__ ls, longlong2* __restrict__ hist,
               long long* __restrict__ totals, unsigned long long* __restrict__ row_stats) {
  pdl_wait();
  const int n_entries = ls->n_hentries;
  const uint64_t total = ls->hist_rows;
  if (n_entries <= 0 || total == 0) return;
  if (row_stats && blockIdx.x == 0 && threadIdx.x == 0)
    atomicAdd(&row_stats[entries[0].identity ? 0 : 1], (unsigned long long)total);
  const uint64_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t a = (uint64_t)blockIdx.x * per;
  const uint64_t b = min(total, a + per);
  const double fg = scale->fg, fh = scale->fh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kWarps = kCsrThreads / 32;
  long long tg = 0, th = 0;
  if (a < b) {
    int e = 0;
    {
      int hi = n_entries - 1;
      while (e < hi) {
        const int mid = (e + hi + 1) >> 1;
        if (entries[mid].prefix <= a) e = mid; else hi = mid - 1;
      }
    }
    uint64_t pos = a;
    while (pos < b && e < n_entries) {
      const HEntry en = entries[e];
      const uint64_t end_e = min(b, en.prefix + en.len);
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(hist + (uint64_t)en.slot * c.total_bins);
      for (uint64_t i = pos + warp; i < end_e; i += kWarps) {
        const uint32_t at = en.begin + (uint32_t)(i - en.prefix);
        const uint32_t row = en.identity ? at : __ldg(rows + at);
        const uint64_t r0 = __ldg(c.csr_ptr + row), r1 = __ldg(c.csr_ptr + row + 1);
        const float2 p = __ldg(gpair + row);
        const long long qg = __double2ll_rn((double)p.x * fg);
        const long long qh = __double2ll_rn((double)p.y * fh);
        if (lane == 0) {
          tg += qg;
          th += qh;
        }
        for (uint64_t j = r0 + lane; j < r1; j += 32) {
          const uint32_t bin = __ldg(c.csr_bins + j);
          atomicAdd(dst + 2 * (uint64_t)bin, (unsigned long long)qg);
          atomicAdd(dst + 2 * (uint64_t)bin + 1, (unsigned long long)qh);
        }
      }
      pos = end_e;
      ++e;
    }
  }
  if (totals != nullptr) {
    using BR = cub::BlockReduce<long long, kCsrThreads>;
    __shared__ typename BR::TempStorage tmp;
    const long long sgt = BR(tmp).Sum(tg);
    __syncthreads();
    const long long sht = BR(tmp).Sum(th);
    if (threadIdx.x == 0 && (sgt || sht)) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[0]), (unsigned long long)sgt);
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[1]), (unsigned long long)sht);
    }
  }
}

// ---------------------------------------------------------------------------
// Histogram. One CTA per SM (1024 threads) per feature group of up to 32
// features; the CTA's share of the level's rows is contiguous in the
// concatenation of the entries, so it flushes its shared histogram once per
// entry it touches. Shared layout: g[bin][32] then h[bin][32] as int64, a
// feature's bins in one bank pair; lane l starts at feature l % nf and walks
// the features cyclically, so a warp's 32 atomics hit distinct features.

__global__ void __launch_bounds__(kHistThreads, 1)
    k_hist(DevConst c, const uint32_t* __restrict__ fo, const uint8_t* __restrict__ rec,
           const float2* __restrict__ gpair, const Scale* __restrict__ scale,
           const uint32_t* __restrict__ rows, const HEntry* __restrict__ entries,
           const LevelState* __restrict__ ls, longlong2* __restrict__ hist,
           long long* __restrict__ totals, unsigned long long* __restrict__ row_stats) {
  pdl_wait();
  extern __shared__ unsigned long long smem[];
  const int n_entries = ls->n_hentries;
  const uint64_t total = ls->hist_rows;
  if (n_entries <= 0 || total == 0) return;
  if (row_stats && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    atomicAdd(&row_stats[entries[0].identity ? 0 : 1], (unsigned long long)total);
  const uint64_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t a = (uint64_t)blockIdx.x * per;
  const uint64_t b = min(total, a + per);
  if (a >= b) return;

  const int g = blockIdx.y;
  const int f0 = g * kGroupFeatures;
  const int nf = min(kGroupFeatures, (int)c.n_cols - f0);
  const int nslots = (int)c.max_bins * 32;
  unsigned long long* sg = smem;
  unsigned long long* sh = smem + nslots;
  for (int i = threadIdx.x; i < 2 * nslots; i += blockDim.x) smem[i] = 0ull;
  __syncthreads();

  const double fg = scale->fg, fh = scale->fh;
  const int lane = threadIdx.x & 31;
  const int start_f = lane % nf;
  const bool wide = c.stride >= (uint32_t)(32 * g + 32);
  const bool want_totals = totals != nullptr && g == 0;
  long long tg = 0, th = 0;

  // the entry holding row position a: the last one whose prefix is <= a
  // (binary search; prefixes ascend)
  int e = 0;
  {
    int hi = n_entries - 1;
    while (e < hi) {
      const int mid = (e + hi + 1) >> 1;
      if (entries[mid].prefix <= a) e = mid; else hi = mid - 1;
    }
  }
  uint64_t pos = a;
  while (pos < b && e < n_entries) {
    const HEntry en = entries[e];
    const uint64_t end_e = min(b, en.prefix + en.len);
    for (uint64_t i = pos + threadIdx.x; i < end_e; i += blockDim.x) {
      const uint32_t at = en.begin + (uint32_t)(i - en.prefix);
      const uint32_t row = en.identity ? at : rows[at];
      const uint8_t* rp = rec + rec_offset(row, c.stride, c.blk);
      const uint4 v0 = *reinterpret_cast<const uint4*>(rp + 32 * g);
      const uint4 v1 = wide ? *reinterpret_cast<const uint4*>(rp + 32 * g + 16) : make_uint4(0, 0, 0, 0);
      const uint32_t mask = *reinterpret_cast<const uint32_t*>(rp + c.mask_off + 4 * g);
      const float2 p = gpair ? gpair[row]
                             : *reinterpret_cast<const float2*>(rec + pair_offset(row, c.blk, c.blk_pair));
      const long long qg = __double2ll_rn((double)p.x * fg);
      const long long qh = __double2ll_rn((double)p.y * fh);
      if (want_totals) {
        tg += qg;
        th += qh;
      }
      int f = start_f;
      for (int s = 0; s < nf; ++s) {
        if (!((mask >> f) & 1u)) {
          const uint32_t w = pick_word(v0, v1, f >> 2);
          const uint32_t bin = (w >> ((f & 3) * 8)) & 0xffu;
          atomicAdd(&sg[bin * 32 + f], (unsigned long long)qg);
          atomicAdd(&sh[bin * 32 + f], (unsigned long long)qh);
        }
        f = (f + 1 == nf) ? 0 : f + 1;
      }
    }
    __syncthreads();
    longlong2* dst = hist + (uint64_t)en.slot * c.total_bins;
    for (int i = threadIdx.x; i < nslots; i += blockDim.x) {
      const int bin = i >> 5, fl = i & 31;
      if (fl < nf) {
        const uint32_t fs = fo[f0 + fl];
        const uint32_t nb = fo[f0 + fl + 1] - fs;
        if ((uint32_t)bin < nb) {
          const unsigned long long vg = sg[i], vh = sh[i];
          if (vg) atomicAdd(reinterpret_cast<unsigned long long*>(&dst[fs + bin].x), vg);
          if (vh) atomicAdd(reinterpret_cast<unsigned long long*>(&dst[fs + bin].y), vh);
        }
      }
      sg[i] = 0ull;
      sh[i] = 0ull;
    }
    __syncthreads();
    pos = end_e;
    ++e;
  }
  if (want_totals) {
    using BR = cub::BlockReduce<long long, kHistThreads>;
    __shared__ typename BR::TempStorage tmp;
    long long sgt = BR(tmp).Sum(tg);
    __syncthreads();
    long long sht = BR(tmp).Sum(th);
    if (threadIdx.x == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[0]), (unsigned long long)sgt);
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[1]), (unsigned long long)sht);
    }
  }
}

// The same histograms with 32-bit shared atomics, which B200 shared memory
// executes several times faster than 64-bit ones. Each fixed-point value q
// (|q| <= 2^(62-c), c = ceil(log2 rows)) is split as q = hi * 2^K + lo with
// 0 <= lo < 2^K; a bin keeps four 32-bit sums (lo and hi of g and of h) in
// shared memory. Both stay exact for R = 2^r rows, K = ceil((64-c)/2),
// r = min(32-K, c+K-32): R * (2^K - 1) < 2^32 and R * 2^(62-c-K) <= 2^30.
// Every R rows the CTA folds them into int64 sums held in registers (each
// thread owns kSlotsPerThread slots), and at the end of an entry adds those
// to the global int64 histogram. Lane l starts at feature l, and the
// record is rotated by l bytes once per row, so step s reads byte s.
constexpr int kH32Threads = 512;
constexpr int kSlotsPerThread = 16;  // 256 bins x 32 feature slots / 512 threads
constexpr int kNSlots = kSlotsPerThread * kH32Threads;  // shared accumulator slots per array
// Bin 256 of every array is a trash row: a missing cell (or a padding
// feature of the group) adds there instead of branching around its update,
// and the row is never folded.
constexpr int kTrashBin = 256;
constexpr int kSlotStride = kNSlots + 32;  // words per array, trash row included

// Staging of one pass of rows (one row per thread): the group's 32 record
// bytes, the (g, h) pair and the group's missing-mask word.
struct StageRow {
  uint4 a, b;
};

// Groups of 32 features a CTA covers: G = 2 when every feature has at most
// 128 bins (two groups' accumulators then share the 8192 slots, slot row
// (group << 7) | bin), else 1. A row's pair is staged once for all of them.
template <int G>
struct H32 {
  // rows staged ahead with cp.async: two stages leave the SM's L1 about 80 KB
  // (three: about 57 KB, four: about 34 KB), which the gathered levels use
  static constexpr int kStages = 2;
  static constexpr int kBinShift = G == 1 ? 8 : 7;  // log2(slot rows per group)
  static constexpr size_t smem() {
    return (size_t)kSlotStride * 16 +
           (size_t)kStages * kH32Threads * (G * sizeof(StageRow) + sizeof(float2) + G * sizeof(uint32_t));
  }
};

// BLK: the record layout (c.blk: 0, or 2, 3, 5 rows a 128-byte block, whose
// record widths are then 48, 32, 16 bytes), a compile-time constant so that
// the row addressing folds; PIB: each row's pair comes from its row block
// instead of `gpair`.
template <int G, int BLK, bool PIB>
__global__ void __launch_bounds__(kH32Threads, 1)
    k_hist32(DevConst c, const uint32_t* __restrict__ fo, const uint8_t* __restrict__ rec,
             const float2* __restrict__ gpair, const Scale* __restrict__ scale,
             const uint32_t* __restrict__ rows, const HEntry* __restrict__ entries,
             const LevelState* __restrict__ ls, longlong2* __restrict__ hist,
             long long* __restrict__ totals, unsigned long long* __restrict__ row_stats, int lo_bits,
             int flush_rows) {
  pdl_wait();
  constexpr int kSt = H32<G>::kStages;
  constexpr int kBS = H32<G>::kBinShift;
  constexpr uint32_t kRecW = BLK == 5 ? 16u : BLK == 3 ? 32u : BLK == 2 ? 48u : 0u;
  static_assert(!PIB || BLK != 0, "pairs in row blocks need the block layout");
  extern __shared__ __align__(16) uint32_t s32[];
  const int n_entries = ls->n_hentries;
  const uint64_t total = ls->hist_rows;
  if (n_entries <= 0 || total == 0) return;
  if (row_stats && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    atomicAdd(&row_stats[entries[0].identity ? 0 : 1], (unsigned long long)total);
  const uint64_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t a = (uint64_t)blockIdx.x * per;
  const uint64_t b = min(total, a + per);
  if (a >= b) return;

  const int g0 = blockIdx.y * G;                          // first group of this CTA
  const int ng = min(G, (int)c.n_groups - g0);            // its groups
  uint32_t* lo_g = s32;
  uint32_t* hi_g = s32 + kSlotStride;
  uint32_t* lo_h = s32 + 2 * kSlotStride;
  uint32_t* hi_h = s32 + 3 * kSlotStride;
  StageRow* srec = reinterpret_cast<StageRow*>(s32 + 4 * kSlotStride);       // [kSt][G][threads]
  float2* sgp = reinterpret_cast<float2*>(srec + kSt * G * kH32Threads);     // [kSt][threads]
  uint32_t* smask = reinterpret_cast<uint32_t*>(sgp + kSt * kH32Threads);    // [kSt][G][threads]
  for (int i = threadIdx.x; i < 4 * kSlotStride; i += blockDim.x) s32[i] = 0u;

  long long acc_g[kSlotsPerThread], acc_h[kSlotsPerThread];
#pragma unroll
  for (int j = 0; j < kSlotsPerThread; ++j) acc_g[j] = acc_h[j] = 0;
  __syncthreads();

  const double fg = scale->fg, fh = scale->fh;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const uint32_t lane4 = (uint32_t)lane << 2;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(s32);
  // per group of the CTA: record width, mask placement, padding features
  bool wide[G], mask_in_block[G];
  uint32_t mask_at[G], dummy[G];
#pragma unroll
  for (int lg = 0; lg < G; ++lg) {
    const int g = g0 + lg;
    const int nfg = lg < ng ? min(kGroupFeatures, (int)c.n_cols - g * kGroupFeatures) : 0;
    wide[lg] = c.stride >= (uint32_t)(32 * g + 32);
    mask_at[lg] = c.mask_off + 4 * g;
    mask_in_block[lg] = mask_at[lg] >= (uint32_t)(32 * g) &&
                        mask_at[lg] + 4 <= (uint32_t)(32 * g + (wide[lg] ? 32 : 16));
    dummy[lg] = nfg >= 32 ? 0u : (0xffffffffu << nfg);  // padded features: trash row
  }
  const bool want_totals = totals != nullptr && g0 == 0;
  const uint32_t lo_mask = (uint32_t)((1ull << lo_bits) - 1ull);
  long long tg = 0, th = 0;

  // Each thread owns kSlotsPerThread / 4 runs of four consecutive slots
  // (slot_of below), moved with 128-bit shared loads and stores.
  auto fold = [&]() {
#pragma unroll
    for (int j = 0; j < kSlotsPerThread / 4; ++j) {
      const int base = 4 * (tid + j * kH32Threads);
      const uint4 a = *reinterpret_cast<const uint4*>(&lo_g[base]);
      const uint4 b = *reinterpret_cast<const uint4*>(&hi_g[base]);
      const uint4 p = *reinterpret_cast<const uint4*>(&lo_h[base]);
      const uint4 q = *reinterpret_cast<const uint4*>(&hi_h[base]);
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(&lo_g[base]) = zero;
      *reinterpret_cast<uint4*>(&hi_g[base]) = zero;
      *reinterpret_cast<uint4*>(&lo_h[base]) = zero;
      *reinterpret_cast<uint4*>(&hi_h[base]) = zero;
      acc_g[4 * j + 0] += ((long long)(int)b.x << lo_bits) + (long long)a.x;
      acc_g[4 * j + 1] += ((long long)(int)b.y << lo_bits) + (long long)a.y;
      acc_g[4 * j + 2] += ((long long)(int)b.z << lo_bits) + (long long)a.z;
      acc_g[4 * j + 3] += ((long long)(int)b.w << lo_bits) + (long long)a.w;
      acc_h[4 * j + 0] += ((long long)(int)q.x << lo_bits) + (long long)p.x;
      acc_h[4 * j + 1] += ((long long)(int)q.y << lo_bits) + (long long)p.y;
      acc_h[4 * j + 2] += ((long long)(int)q.z << lo_bits) + (long long)p.z;
      acc_h[4 * j + 3] += ((long long)(int)q.w << lo_bits) + (long long)p.w;
    }
  };
  auto slot_of = [&](int j) { return 4 * (tid + (j >> 2) * kH32Threads) + (j & 3); };

  // the entry holding row position a: the last one whose prefix is <= a
  // (binary search; prefixes ascend)
  int e = 0;
  {
    int hi = n_entries - 1;
    while (e < hi) {
      const int mid = (e + hi + 1) >> 1;
      if (entries[mid].prefix <= a) e = mid; else hi = mid - 1;
    }
  }
  uint64_t pos = a;
  int since_fold = 0;
  while (pos < b && e < n_entries) {
    const HEntry en = entries[e];
    const uint64_t end_e = min(b, en.prefix + en.len);
    const int n_it = (int)((end_e - pos + kH32Threads - 1) / kH32Threads);
    auto row_at = [&](uint64_t i) -> uint32_t {
      const uint32_t at = en.begin + (uint32_t)(i - en.prefix);
      return en.identity ? at : rows[at];
    };
    // Every thread copies its own future rows into its own staging slots
    // and later reads only those, so the pipeline needs no CTA barrier.
    auto issue = [&](int it, uint32_t row, bool valid) {
      const int st = it % kSt;
      if (valid) {
        const uint8_t* rr = rec + (BLK ? rec_offset(row, kRecW, BLK) : (uint64_t)row * c.stride);
#pragma unroll
        for (int lg = 0; lg < G; ++lg) {
          if (lg < ng) {
            const uint8_t* rp = rr + 32 * (g0 + lg);
            StageRow* d = &srec[(st * G + lg) * kH32Threads + tid];
            __pipeline_memcpy_async(&d->a, rp, 16);
            if (wide[lg]) __pipeline_memcpy_async(&d->b, rp + 16, 16);
            if (!mask_in_block[lg])
              __pipeline_memcpy_async(&smask[(st * G + lg) * kH32Threads + tid], rr + mask_at[lg], 4);
          }
        }
        if (PIB)
          __pipeline_memcpy_async(&sgp[st * kH32Threads + tid], rec + pair_offset(row, BLK, BLK * kRecW), 8);
        else
          __pipeline_memcpy_async(&sgp[st * kH32Threads + tid], &gpair[row], 8);
      }
      __pipeline_commit();
    };
    for (int p = 0; p < kSt - 1; ++p) {
      const uint64_t i = pos + (uint64_t)p * kH32Threads + tid;
      const bool v = i < end_e;
      issue(p, v ? row_at(i) : 0u, v);
    }
    uint64_t ip = pos + (uint64_t)(kSt - 1) * kH32Threads + tid;
    bool pend_valid = ip < end_e;
    uint32_t pend_row = pend_valid ? row_at(ip) : 0u;
    for (int it = 0; it < n_it; ++it) {
      issue(it + kSt - 1, pend_row, pend_valid);
      ip = pos + (uint64_t)(it + kSt) * kH32Threads + tid;
      pend_valid = ip < end_e;
      pend_row = pend_valid ? row_at(ip) : 0u;
      __pipeline_wait_prior(kSt - 1);
      const uint64_t i = pos + (uint64_t)it * kH32Threads + tid;
      if (i < end_e) {
        const int st = it % kSt;
        const float2 pr = sgp[st * kH32Threads + tid];
        const long long qg = __double2ll_rn((double)pr.x * fg);
        const long long qh = __double2ll_rn((double)pr.y * fh);
        if (want_totals) {
          tg += qg;
          th += qh;
        }
        const uint32_t lg_ = (uint32_t)qg & lo_mask, lh = (uint32_t)qh & lo_mask;
        const uint32_t hg = (uint32_t)(qg >> lo_bits), hh = (uint32_t)(qh >> lo_bits);
#pragma unroll
        for (int lg = 0; lg < G; ++lg) {
          if (lg >= ng) break;
          const StageRow sr = srec[(st * G + lg) * kH32Threads + tid];
          const uint4 v1 = wide[lg] ? sr.b : make_uint4(0, 0, 0, 0);
          uint32_t mask;
          if (mask_in_block[lg]) {
            const int mw = (int)(mask_at[lg] - 32 * (g0 + lg)) >> 2;
            mask = pick_word(sr.a, v1, mw);
          } else {
            mask = smask[(st * G + lg) * kH32Threads + tid];
          }
          mask |= dummy[lg];
          // rotate the 32 record bytes right by `lane` bytes: word rotation by
          // lane / 4 (three select stages), then a byte funnel shift
          uint32_t w[8] = {sr.a.x, sr.a.y, sr.a.z, sr.a.w, v1.x, v1.y, v1.z, v1.w};
          const int q = lane >> 2;
          uint32_t t[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) t[j] = (q & 4) ? w[(j + 4) & 7] : w[j];
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = (q & 2) ? t[(j + 2) & 7] : t[j];
#pragma unroll
          for (int j = 0; j < 8; ++j) t[j] = (q & 1) ? w[(j + 1) & 7] : w[j];
          const int sh = (lane & 3) * 8;
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = __funnelshift_r(t[j], t[(j + 1) & 7], sh);
          const uint32_t mrot = __funnelshift_r(mask, mask, lane);
          const uint32_t grow = (uint32_t)lg << (kBS + 7);  // this group's slot rows
          // slot byte offset = row * 128 + 4 * ((lane + s) & 31), row =
          // (group << kBS) | bin; the four arrays sit kSlotStride words apart,
          // one address for all four reds
#pragma unroll
          for (int s = 0; s < 32; ++s) {
            const uint32_t word = w[s >> 2];
            const int k = s & 3;
            const uint32_t binx = (k == 0 ? (word << 7) : (word >> (8 * k - 7))) &
                                  (((1u << kBS) - 1u) << 7);
            const uint32_t rowx = ((mrot >> s) & 1u) ? (uint32_t)(kTrashBin << 7) : (binx | grow);
            const uint32_t ad = sbase + (rowx | ((lane4 + 4u * (uint32_t)s) & 124u));
            asm volatile(
                "red.shared.add.u32 [%0], %1;\n\t"
                "red.shared.add.u32 [%0+%5], %2;\n\t"
                "red.shared.add.u32 [%0+%6], %3;\n\t"
                "red.shared.add.u32 [%0+%7], %4;" ::"r"(ad),
                "r"(lg_), "r"(hg), "r"(lh), "r"(hh), "n"(kSlotStride * 4), "n"(kSlotStride * 8),
                "n"(kSlotStride * 12)
                : "memory");
          }
        }
      }
      since_fold += kH32Threads;
      if (since_fold + kH32Threads > flush_rows) {
        __syncthreads();
        fold();
        __syncthreads();
        since_fold = 0;
      }
    }
    __pipeline_wait_prior(0);
    __syncthreads();
    fold();
    __syncthreads();
    since_fold = 0;
    // Flush: stage the entry's sums feature-major in the (now zero)
    // accumulator arrays, row = group-local feature, bins XOR-swizzled by
    // row / 4 against bank conflicts; then each warp adds one feature's
    // (g, h) words to the node histogram, 32 consecutive 8-byte words (256
    // contiguous bytes) per 64-bit red instruction.
    {
      constexpr int kNB = 1 << kBS;  // bins per feature row
      long long* stg = reinterpret_cast<long long*>(s32);
#pragma unroll
      for (int j = 0; j < kSlotsPerThread; ++j) {
        const int slot = slot_of(j);
        const int row = ((slot >> (kBS + 5)) << 5) | (slot & 31);
        const int bin = (slot >> 5) & (kNB - 1);
        const int at = 2 * (row * kNB + (bin ^ ((row >> 2) & 7)));
        stg[at] = acc_g[j];
        stg[at + 1] = acc_h[j];
        acc_g[j] = acc_h[j] = 0;
      }
      __syncthreads();
      unsigned long long* dstw = reinterpret_cast<unsigned long long*>(hist + (uint64_t)en.slot * c.total_bins);
      const int warp = tid >> 5;
      for (int row = warp; row < G * 32; row += kH32Threads / 32) {
        const int lgs = row >> 5;
        const int f = (g0 + lgs) * kGroupFeatures + (row & 31);
        if (lgs >= ng || f >= (int)c.n_cols) continue;
        const uint32_t fs = fo[f];
        const uint32_t nw = 2 * (fo[f + 1] - fs);
        for (uint32_t w = lane; w < nw; w += 32) {
          const int bin = (int)(w >> 1);
          const long long v = stg[2 * (row * kNB + (bin ^ ((row >> 2) & 7))) + (w & 1)];
          if (v) atomicAdd(dstw + 2 * (uint64_t)fs + w, (unsigned long long)v);
        }
      }
      __syncthreads();
      // the accumulators start the next entry at zero
      uint4* z = reinterpret_cast<uint4*>(s32);
      for (int i = tid; i < kSlotStride; i += kH32Threads) z[i] = make_uint4(0u, 0u, 0u, 0u);
      __syncthreads();
    }
    pos = end_e;
    ++e;
  }
  if (want_totals) {
    using BR = cub::BlockReduce<long long, kH32Threads>;
    __shared__ typename BR::TempStorage tmp;
    long long sgt = BR(tmp).Sum(tg);
    __syncthreads();
    long long sht = BR(tmp).Sum(th);
    if (tid == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[0]), (unsigned long long)sgt);
      atomicAdd(reinterpret_cast<unsigned long long*>(&totals[1]), (unsigned long long)sht);
    }
  }
}

// The k_hist32 instantiation for G groups a CTA, record layout blk and the
// pairs' source (pib: the row blocks). Two groups a CTA need 33 or more
// features, so 48-byte records (blk 2) or wider (blk 0).
using H32Fn = void (*)(DevConst, const uint32_t*, const uint8_t*, const float2*, const Scale*,
                       const uint32_t*, const HEntry*, const LevelState*, longlong2*, long long*,
                       unsigned long long*, int, int);

static H32Fn h32_fn(int G, uint32_t blk, bool pib) {
  if (G == 2) {
    if (blk == 2) return pib ? k_hist32<2, 2, true> : k_hist32<2, 2, false>;
    return blk == 0 ? k_hist32<2, 0, false> : nullptr;
  }
  switch (blk) {
    case 2: return pib ? k_hist32<1, 2, true> : k_hist32<1, 2, false>;
    case 3: return pib ? k_hist32<1, 3, true> : k_hist32<1, 3, false>;
    case 5: return pib ? k_hist32<1, 5, true> : k_hist32<1, 5, false>;
    default: return k_hist32<1, 0, false>;
  }
}

static std::vector<const void*> h32_kernels() {
  std::vector<const void*> v;
  for (int G = 1; G <= 2; ++G)
    for (uint32_t blk : {0u, 2u, 3u, 5u})
      for (bool pib : {false, true})
        if (H32Fn f = (pib && blk == 0) ? nullptr : h32_fn(G, blk, pib)) v.push_back((const void*)f);
  return v;
}

// sibling = parent - built (int64, exact; src/tree/hist/mod.rs:32).
__global__ void k_subtract(const Triple* __restrict__ pairs, const LevelState* __restrict__ ls,
                           uint32_t total_bins, longlong2* __restrict__ hist) {
  const int n_pairs = ls->n_pairs;
  const uint64_t work = (uint64_t)n_pairs * total_bins;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < work;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const Triple t = pairs[i / total_bins];
    const uint32_t bin = (uint32_t)(i % total_bins);
    const longlong2 p = hist[(uint64_t)t.parent * total_bins + bin];
    const longlong2 q = hist[(uint64_t)t.built * total_bins + bin];
    hist[(uint64_t)t.sibling * total_bins + bin] = make_longlong2(p.x - q.x, p.y - q.y);
  }
}

// ---------------------------------------------------------------------------
// Split scoring, XGBoost's f32 arithmetic as the reference states it
// (src/tree/builder/shared.rs:87-141, split.rs:37-58).
__device__ __forceinline__ double threshold_l1(double g, double alpha) {
  if (g > alpha) return g - alpha;
  if (g < -alpha) return g + alpha;
  return 0.0;
}

__device__ __forceinline__ double xgb_calc_weight(double g, double h, const DevConst& c) {
  if (h <= 0.0) return 0.0;
  double w = -threshold_l1(g, c.alpha) / (h + c.lambda);
  if (c.mds != 0.0 && fabs(w) > c.mds) w = copysign(c.mds, w);
  return w;
}

// shared.rs:113 `xgb_weight`: rounded to f32, then clamped to the node's
// monotone bounds as f32 (shared.rs:100 `apply_bounds`).
__device__ __forceinline__ float xgb_weight(double g, double h, const DevConst& c,
                                            float lo = -INFINITY, float up = INFINITY) {
  const float w = __double2float_rn(xgb_calc_weight(g, h, c));
  return w < lo ? lo : (w > up ? up : w);
}

// f64::midpoint: (a + b) / 2 without intermediate overflow.
__device__ __forceinline__ double midpoint(double a, double b) {
  const double lo = DBL_MIN * 2.0, hi = DBL_MAX / 2.0;
  const double aa = fabs(a), ab = fabs(b);
  if (aa <= hi && ab <= hi) return (a + b) / 2.0;
  if (aa < lo) return a + b / 2.0;
  if (ab < lo) return a / 2.0 + b;
  return a / 2.0 + b / 2.0;
}

// f64::clamp (a NaN passes through)
__device__ __forceinline__ double clamp_bounds(double w, double lower, double upper) {
  return w < lower ? lower : (w > upper ? upper : w);
}

// constraints.rs:82 `child_bounds`: the children's bounds after a split on
// a feature of direction `dir` with bounded child weights wl, wr.
__device__ __forceinline__ void child_bounds(double lower, double upper, int dir, float wl, float wr,
                                             double* l_lo, double* l_up, double* r_lo, double* r_up) {
  *l_lo = *r_lo = lower;
  *l_up = *r_up = upper;
  if (dir == 0) return;
  const double mid = midpoint((double)wl, (double)wr);
  if (dir > 0) {
    *l_up = mid;
    *r_lo = mid;
  } else {
    *l_lo = mid;
    *r_up = mid;
  }
}

__device__ __forceinline__ double gain_given_weight(double g, double h, const DevConst& c, float w) {
  const float ww = __fmul_rn(w, w);
  return -(2.0 * g * (double)w + (h + c.lambda) * (double)ww + 2.0 * c.alpha * (double)fabsf(w));
}

__device__ __forceinline__ float node_gain(double g, double h, const DevConst& c,
                                           float lo = -INFINITY, float up = INFINITY) {
  if (h <= 0.0) return 0.0f;
  return __double2float_rn(gain_given_weight(g, h, c, xgb_weight(g, h, c, lo, up)));
}

// SplitScorer::loss_chg (split.rs:37): -inf for invalid children or child
// weights against the feature's monotone direction (constraints.rs:117).
__device__ __forceinline__ float cand_loss(double lg, double lh, double rg, double rh,
                                           float root_gain, const DevConst& c, float lo = -INFINITY,
                                           float up = INFINITY, int dir = 0) {
  if (!(lh > 0.0 && rh > 0.0 && lh >= c.mcw && rh >= c.mcw)) return -INFINITY;
  const float wl = xgb_weight(lg, lh, c, lo, up);
  const float wr = xgb_weight(rg, rh, c, lo, up);
  if (dir > 0 ? !(wl <= wr) : (dir < 0 ? !(wl >= wr) : false)) return -INFINITY;
  const float gain = __fadd_rn(__double2float_rn(gain_given_weight(lg, lh, c, wl)),
                               __double2float_rn(gain_given_weight(rg, rh, c, wr)));
  return __fsub_rn(gain, root_gain);
}

// gain.rs:107 `calc_weight` (leaf values).
__device__ __forceinline__ double calc_weight(double g, double h, const DevConst& c) {
  if (h < c.mcw || h <= 0.0) return 0.0;
  double w = -threshold_l1(g, c.alpha) / (h + c.lambda);
  if (c.mds > 0.0) w = fmin(fmax(w, -c.mds), c.mds);
  return w;
}

// One CTA per (frontier node, feature), one bin per thread: the feature's
// first best candidate in for_each_numeric_split order (split.rs:391): the
// forward pass over the bins (candidate sequence number = bin offset), then,
// when the node has missing values of the feature, the backward pass
// (sequence nb + (nb - 1 - offset)). Prefix sums are exact integers; the
// backward pass's suffix at offset o is (feature total - exclusive prefix
// at o). A node whose slot is a sibling (slot >= sib_base, with `pairs`)
// first gets its histogram as parent - built (src/tree/hist/mod.rs:32),
// stored for the next level, in the same pass.
constexpr int kSplitThreads = 256;  // features of <= 256 bins

__device__ __forceinline__ bool cand_better(float l, int seq, float bl, int bseq) {
  return l > bl || (l == bl && seq < bseq);
}

// A node's best split over its features, kept as one 64-bit maximum: the
// merge rule of builder/mod.rs:313 (`need_replace` over ascending features:
// the largest loss change above 0, the lowest feature among equals) is the
// maximum of (loss bits, ~feature) over the features whose loss is above 0,
// since the bits of positive floats order as the floats do. Each scan's
// winner adds its feature with one atomicMax; the level's apply (or the
// lossguide step) reads the node's key and clears it. 0: no candidate.
__device__ __forceinline__ unsigned long long cand_key(float loss, uint32_t f) {
  return ((unsigned long long)__float_as_uint(loss) << 32) | (unsigned long long)(0xffffffffu - f);
}
__device__ __forceinline__ int key_feature(unsigned long long key) {
  return key ? (int)(0xffffffffu - (uint32_t)key) : -1;
}

__global__ void __launch_bounds__(kSplitThreads)
    k_scan(DevConst c, const uint32_t* __restrict__ fo, longlong2* __restrict__ hist,
           const Front* __restrict__ front, const LevelState* __restrict__ ls,
           const Triple* __restrict__ pairs, int sib_base, const Scale* __restrict__ scale,
           Cand* __restrict__ cand, const int8_t* __restrict__ dirs,
             unsigned long long* __restrict__ best_key) {
  pdl_wait();
  const int f = blockIdx.x;
  const int k = blockIdx.y;
  if (k >= ls->n_front) return;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const Front fr = front[k];
  const uint32_t fs = fo[f];
  const int nb = (int)(fo[f + 1] - fs);
  Cand* out = cand + (uint64_t)k * c.n_cols + f;
  longlong2 v = make_longlong2(0, 0);
  if (fr.slot >= 0 && t < nb) {
    // depthwise: sibling slots start at sib_base; lossguide (sib_base < 0):
    // the one pair of the step, pairs[0]
    const bool sib = pairs != nullptr && (sib_base >= 0 ? fr.slot >= sib_base : fr.slot == pairs[0].sibling);
    if (sib) {
      const Triple tr = pairs[sib_base >= 0 ? fr.slot - sib_base : 0];
      const longlong2 pv = hist[(uint64_t)tr.parent * c.total_bins + fs + t];
      const longlong2 bv = hist[(uint64_t)tr.built * c.total_bins + fs + t];
      v = make_longlong2(pv.x - bv.x, pv.y - bv.y);
      hist[(uint64_t)fr.slot * c.total_bins + fs + t] = v;
    } else {
      v = hist[(uint64_t)fr.slot * c.total_bins + fs + t];
    }
  }
  if (nb <= 1 || fr.slot < 0) {
    if (t == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
    return;
  }
  // block inclusive scan of the exact (g, h) sums
  __shared__ long long s_wg[kSplitThreads / 32], s_wh[kSplitThreads / 32];
  __shared__ float s_bl[kSplitThreads / 32];
  __shared__ int s_bs[kSplitThreads / 32];
  long long ig_ = v.x, ih_ = v.y;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const long long tg = __shfl_up_sync(kFull, ig_, d);
    const long long th = __shfl_up_sync(kFull, ih_, d);
    if (lane >= d) {
      ig_ += tg;
      ih_ += th;
    }
  }
  if (lane == 31) {
    s_wg[warp] = ig_;
    s_wh[warp] = ih_;
  }
  __syncthreads();
  long long off_g = 0, off_h = 0, tot_g = 0, tot_h = 0;
#pragma unroll
  for (int w = 0; w < kSplitThreads / 32; ++w) {
    const long long a = s_wg[w], b = s_wh[w];
    if (w < warp) {
      off_g += a;
      off_h += b;
    }
    tot_g += a;
    tot_h += b;
  }
  const long long incl_g = ig_ + off_g, incl_h = ih_ + off_h;
  const long long excl_g = incl_g - v.x, excl_h = incl_h - v.y;
  const bool has_missing = !c.dense && !(tot_g == fr.g && tot_h == fr.h);

  const double ig = scale->ig, ih = scale->ih;
  // the node's bounds and the feature's direction (search.rs:130-144):
  // per (node, feature) from `dirs` (RowEngine scans), else the training
  // run's per-feature constraints
  const float lo = (float)fr.lower, up = (float)fr.upper;
  const int dir = dirs ? (int)dirs[(uint64_t)k * c.n_cols + f] : (c.mono ? (int)c.mono[f] : 0);
  const float root_gain =
      fr.root_gain_given ? fr.root_gain : node_gain(ll2d(fr.g) * ig, ll2d(fr.h) * ih, c, lo, up);
  float best = -INFINITY;
  int best_seq = INT_MAX;
  long long blg = 0, blh = 0;
  int bbin = -1, bdl = 0;
  // An empty bin's candidates repeat a neighbour's statistics, and that
  // neighbour comes first in its pass (forward: offset t - 1; backward:
  // t + 1), so it keeps any tie: an empty bin is never the first maximum.
  if (t < nb && (v.x != 0 || v.y != 0)) {
    const float l = cand_loss(ll2d(incl_g) * ig, ll2d(incl_h) * ih, ll2d(fr.g - incl_g) * ig,
                              ll2d(fr.h - incl_h) * ih, root_gain, c, lo, up, dir);
    if (isfinite(l)) {
      best = l;
      best_seq = t;
      blg = incl_g;
      blh = incl_h;
      bbin = (int)fs + t;
      bdl = 0;
    }
    if (has_missing) {
      const long long rg = tot_g - excl_g, rh = tot_h - excl_h;
      const long long lg2 = fr.g - rg, lh2 = fr.h - rh;
      const float lb = cand_loss(ll2d(lg2) * ig, ll2d(lh2) * ih, ll2d(rg) * ig, ll2d(rh) * ih,
                                 root_gain, c, lo, up, dir);
      const int seq = nb + (nb - 1 - t);
      if (isfinite(lb) && cand_better(lb, seq, best, best_seq)) {
        best = lb;
        best_seq = seq;
        blg = lg2;
        blh = lh2;
        bbin = t == 0 ? -1 : (int)fs + t - 1;
        bdl = 1;
      }
    }
  }
  // first maximum over the block: larger loss, then earlier candidate
  float wb = best;
  int ws = best_seq;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ob = __shfl_xor_sync(kFull, wb, d);
    const int os = __shfl_xor_sync(kFull, ws, d);
    if (cand_better(ob, os, wb, ws)) {
      wb = ob;
      ws = os;
    }
  }
  if (lane == 0) {
    s_bl[warp] = wb;
    s_bs[warp] = ws;
  }
  __syncthreads();
  float gb = s_bl[0];
  int gs = s_bs[0];
#pragma unroll
  for (int w = 1; w < kSplitThreads / 32; ++w)
    if (cand_better(s_bl[w], s_bs[w], gb, gs)) {
      gb = s_bl[w];
      gs = s_bs[w];
    }
  if (gs == INT_MAX) {  // no finite candidate in this feature
    if (t == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
  } else if (best_seq == gs) {
    Cand e;
    e.loss = best;
    e.bin = bbin;
    e.default_left = bdl;
    e.pad = 0;
    e.lg = blg;
    e.lh = blh;
    *out = e;
    if (best_key && best > 0.0f) atomicMax(best_key + k, cand_key(best, (uint32_t)f));
  }
}

// The split scan for features of more than kSplitThreads bins (CSR indexes
// with max_bin above 256): the same candidates, sequence numbers and
// first-maximum rule as k_scan, the feature's bins taken kSplitThreads at a
// time with the prefix carried between chunks. A first pass forms the
// feature's total (and writes a sibling's histogram as parent - built), the
// second scans and scores.
__global__ void __launch_bounds__(kSplitThreads)
    k_scan_wide(DevConst c, const uint32_t* __restrict__ fo, longlong2* __restrict__ hist,
                const Front* __restrict__ front, const LevelState* __restrict__ ls,
                const Triple* __restrict__ pairs, int sib_base, const Scale* __restrict__ scale,
                Cand* __restrict__ cand, const int8_t* __restrict__ dirs,
             unsigned long long* __restrict__ best_key) {
  pdl_wait();
  const int f = blockIdx.x;
  const int k = blockIdx.y;
  if (k >= ls->n_front) return;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const Front fr = front[k];
  const uint32_t fs = fo[f];
  const int nb = (int)(fo[f + 1] - fs);
  Cand* out = cand + (uint64_t)k * c.n_cols + f;
  if (nb <= 1 || fr.slot < 0) {
    if (t == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
    return;
  }
  const bool sib = pairs != nullptr && (sib_base >= 0 ? fr.slot >= sib_base : fr.slot == pairs[0].sibling);
  Triple tr{};
  if (sib) tr = pairs[sib_base >= 0 ? fr.slot - sib_base : 0];
  __shared__ long long s_wg[kSplitThreads / 32], s_wh[kSplitThreads / 32];
  __shared__ float s_bl[kSplitThreads / 32];
  __shared__ int s_bs[kSplitThreads / 32];
  // pass 1: the feature's total (sibling histograms written as they go)
  long long sum_g = 0, sum_h = 0;
  for (int c0 = 0; c0 < nb; c0 += kSplitThreads) {
    const int b = c0 + t;
    if (b < nb) {
      longlong2 v;
      if (sib) {
        const longlong2 pv = hist[(uint64_t)tr.parent * c.total_bins + fs + b];
        const longlong2 bv = hist[(uint64_t)tr.built * c.total_bins + fs + b];
        v = make_longlong2(pv.x - bv.x, pv.y - bv.y);
        hist[(uint64_t)fr.slot * c.total_bins + fs + b] = v;
      } else {
        v = hist[(uint64_t)fr.slot * c.total_bins + fs + b];
      }
      sum_g += v.x;
      sum_h += v.y;
    }
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    sum_g += __shfl_xor_sync(kFull, sum_g, d);
    sum_h += __shfl_xor_sync(kFull, sum_h, d);
  }
  if (lane == 0) {
    s_wg[warp] = sum_g;
    s_wh[warp] = sum_h;
  }
  __syncthreads();
  long long tot_g = 0, tot_h = 0;
#pragma unroll
  for (int w = 0; w < kSplitThreads / 32; ++w) {
    tot_g += s_wg[w];
    tot_h += s_wh[w];
  }
  __syncthreads();
  const bool has_missing = !c.dense && !(tot_g == fr.g && tot_h == fr.h);
  const double ig = scale->ig, ih = scale->ih;
  const float lo = (float)fr.lower, up = (float)fr.upper;
  const int dir = dirs ? (int)dirs[(uint64_t)k * c.n_cols + f] : (c.mono ? (int)c.mono[f] : 0);
  const float root_gain =
      fr.root_gain_given ? fr.root_gain : node_gain(ll2d(fr.g) * ig, ll2d(fr.h) * ih, c, lo, up);
  float best = -INFINITY;
  int best_seq = INT_MAX;
  long long blg = 0, blh = 0;
  int bbin = -1, bdl = 0;
  // pass 2: chunk by chunk, the block scan plus the carried prefix
  long long carry_g = 0, carry_h = 0;
  for (int c0 = 0; c0 < nb; c0 += kSplitThreads) {
    const int b = c0 + t;
    longlong2 v = make_longlong2(0, 0);
    if (b < nb) v = hist[(uint64_t)fr.slot * c.total_bins + fs + b];
    long long ig_ = v.x, ih_ = v.y;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const long long tg = __shfl_up_sync(kFull, ig_, d);
      const long long th = __shfl_up_sync(kFull, ih_, d);
      if (lane >= d) {
        ig_ += tg;
        ih_ += th;
      }
    }
    if (lane == 31) {
      s_wg[warp] = ig_;
      s_wh[warp] = ih_;
    }
    __syncthreads();
    long long off_g = carry_g, off_h = carry_h, chunk_g = 0, chunk_h = 0;
#pragma unroll
    for (int w = 0; w < kSplitThreads / 32; ++w) {
      if (w < warp) {
        off_g += s_wg[w];
        off_h += s_wh[w];
      }
      chunk_g += s_wg[w];
      chunk_h += s_wh[w];
    }
    __syncthreads();
    const long long incl_g = ig_ + off_g, incl_h = ih_ + off_h;
    const long long excl_g = incl_g - v.x, excl_h = incl_h - v.y;
    if (b < nb && (v.x != 0 || v.y != 0)) {
      const float l = cand_loss(ll2d(incl_g) * ig, ll2d(incl_h) * ih, ll2d(fr.g - incl_g) * ig,
                                ll2d(fr.h - incl_h) * ih, root_gain, c, lo, up, dir);
      if (isfinite(l) && cand_better(l, b, best, best_seq)) {
        best = l;
        best_seq = b;
        blg = incl_g;
        blh = incl_h;
        bbin = (int)fs + b;
        bdl = 0;
      }
      if (has_missing) {
        const long long rg = tot_g - excl_g, rh = tot_h - excl_h;
        const long long lg2 = fr.g - rg, lh2 = fr.h - rh;
        const float lb = cand_loss(ll2d(lg2) * ig, ll2d(lh2) * ih, ll2d(rg) * ig, ll2d(rh) * ih,
                                   root_gain, c, lo, up, dir);
        const int seq = nb + (nb - 1 - b);
        if (isfinite(lb) && cand_better(lb, seq, best, best_seq)) {
          best = lb;
          best_seq = seq;
          blg = lg2;
          blh = lh2;
          bbin = b == 0 ? -1 : (int)fs + b - 1;
          bdl = 1;
        }
      }
    }
    carry_g += chunk_g;
    carry_h += chunk_h;
  }
  float wb = best;
  int ws = best_seq;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ob = __shfl_xor_sync(kFull, wb, d);
    const int os = __shfl_xor_sync(kFull, ws, d);
    if (cand_better(ob, os, wb, ws)) {
      wb = ob;
      ws = os;
    }
  }
  if (lane == 0) {
    s_bl[warp] = wb;
    s_bs[warp] = ws;
  }
  __syncthreads();
  float gb = s_bl[0];
  int gs = s_bs[0];
#pragma unroll
  for (int w = 1; w < kSplitThreads / 32; ++w)
    if (cand_better(s_bl[w], s_bs[w], gb, gs)) {
      gb = s_bl[w];
      gs = s_bs[w];
    }
  if (gs == INT_MAX) {
    if (t == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
  } else if (best_seq == gs) {
    Cand e;
    e.loss = best;
    e.bin = bbin;
    e.default_left = bdl;
    e.pad = 0;
    e.lg = blg;
    e.lh = blh;
    *out = e;
    if (best_key && best > 0.0f) atomicMax(best_key + k, cand_key(best, (uint32_t)f));
  }
}

// The same scan with one warp per (node, feature), for features of at most
// 32 * P bins: lane l holds bins l*P .. l*P+P-1 (its P sums, then a warp
// scan of the lanes' totals). The candidates, their sequence numbers and
// the first-maximum rule are k_scan's, so the winner is the same bit for
// bit; a CTA of kScanWarps warps covers kScanWarps features of one node.
constexpr int kScanWarps = 8;

template <int P>
__global__ void __launch_bounds__(kScanWarps * 32)
    k_scan_w(DevConst c, const uint32_t* __restrict__ fo, longlong2* __restrict__ hist,
             const Front* __restrict__ front, const LevelState* __restrict__ ls,
             const Triple* __restrict__ pairs, int sib_base, const Scale* __restrict__ scale,
             Cand* __restrict__ cand, const int8_t* __restrict__ dirs,
             unsigned long long* __restrict__ best_key) {
  pdl_wait();
  const int k = blockIdx.y;
  if (k >= ls->n_front) return;
  const int lane = threadIdx.x & 31;
  const int f = blockIdx.x * kScanWarps + (threadIdx.x >> 5);
  if (f >= (int)c.n_cols) return;
  const Front fr = front[k];
  const uint32_t fs = fo[f];
  const int nb = (int)(fo[f + 1] - fs);
  Cand* out = cand + (uint64_t)k * c.n_cols + f;
  if (nb <= 1 || fr.slot < 0) {
    if (lane == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
    return;
  }
  bool sib = false;
  Triple tr{};
  if (pairs != nullptr) {
    sib = sib_base >= 0 ? fr.slot >= sib_base : fr.slot == pairs[0].sibling;
    if (sib) tr = pairs[sib_base >= 0 ? fr.slot - sib_base : 0];
  }
  long long vg[P], vh[P];
  long long lg_ = 0, lh_ = 0;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int t = lane * P + i;
    longlong2 v = make_longlong2(0, 0);
    if (t < nb) {
      if (sib) {
        const longlong2 pv = hist[(uint64_t)tr.parent * c.total_bins + fs + t];
        const longlong2 bv = hist[(uint64_t)tr.built * c.total_bins + fs + t];
        v = make_longlong2(pv.x - bv.x, pv.y - bv.y);
        hist[(uint64_t)fr.slot * c.total_bins + fs + t] = v;
      } else {
        v = hist[(uint64_t)fr.slot * c.total_bins + fs + t];
      }
    }
    vg[i] = v.x;
    vh[i] = v.y;
    lg_ += v.x;
    lh_ += v.y;
  }
  // exclusive prefix of the lanes' totals, and the feature's total
  long long eg = lg_, eh = lh_;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const long long tg = __shfl_up_sync(kFull, eg, d);
    const long long th = __shfl_up_sync(kFull, eh, d);
    if (lane >= d) {
      eg += tg;
      eh += th;
    }
  }
  const long long tot_g = __shfl_sync(kFull, eg, 31), tot_h = __shfl_sync(kFull, eh, 31);
  eg -= lg_;
  eh -= lh_;
  const bool has_missing = !c.dense && !(tot_g == fr.g && tot_h == fr.h);
  const double ig = scale->ig, ih = scale->ih;
  // the node's bounds and the feature's direction (search.rs:130-144):
  // per (node, feature) from `dirs` (RowEngine scans), else the training
  // run's per-feature constraints
  const float lo = (float)fr.lower, up = (float)fr.upper;
  const int dir = dirs ? (int)dirs[(uint64_t)k * c.n_cols + f] : (c.mono ? (int)c.mono[f] : 0);
  const float root_gain =
      fr.root_gain_given ? fr.root_gain : node_gain(ll2d(fr.g) * ig, ll2d(fr.h) * ih, c, lo, up);
  float best = -INFINITY;
  int best_seq = INT_MAX;
  long long blg = 0, blh = 0;
  int bbin = -1, bdl = 0;
  long long run_g = eg, run_h = eh;  // exclusive prefix of bin t
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int t = lane * P + i;
    const long long excl_g = run_g, excl_h = run_h;
    run_g += vg[i];
    run_h += vh[i];
    if (t < nb && (vg[i] != 0 || vh[i] != 0)) {
      const float l = cand_loss(ll2d(run_g) * ig, ll2d(run_h) * ih, ll2d(fr.g - run_g) * ig,
                                ll2d(fr.h - run_h) * ih, root_gain, c, lo, up, dir);
      if (isfinite(l) && cand_better(l, t, best, best_seq)) {
        best = l;
        best_seq = t;
        blg = run_g;
        blh = run_h;
        bbin = (int)fs + t;
        bdl = 0;
      }
      if (has_missing) {
        const long long rg = tot_g - excl_g, rh = tot_h - excl_h;
        const long long lg2 = fr.g - rg, lh2 = fr.h - rh;
        const float lb = cand_loss(ll2d(lg2) * ig, ll2d(lh2) * ih, ll2d(rg) * ig, ll2d(rh) * ih,
                                   root_gain, c, lo, up, dir);
        const int seq = nb + (nb - 1 - t);
        if (isfinite(lb) && cand_better(lb, seq, best, best_seq)) {
          best = lb;
          best_seq = seq;
          blg = lg2;
          blh = lh2;
          bbin = t == 0 ? -1 : (int)fs + t - 1;
          bdl = 1;
        }
      }
    }
  }
  float wb = best;
  int ws = best_seq;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ob = __shfl_xor_sync(kFull, wb, d);
    const int os = __shfl_xor_sync(kFull, ws, d);
    if (cand_better(ob, os, wb, ws)) {
      wb = ob;
      ws = os;
    }
  }
  if (ws == INT_MAX) {
    if (lane == 0) {
      Cand e;
      e.loss = -INFINITY;
      e.bin = -1;
      e.default_left = 0;
      e.pad = 0;
      e.lg = e.lh = 0;
      *out = e;
    }
  } else if (best_seq == ws) {
    Cand e;
    e.loss = best;
    e.bin = bbin;
    e.default_left = bdl;
    e.pad = 0;
    e.lg = blg;
    e.lh = blh;
    *out = e;
    if (best_key && best > 0.0f) atomicMax(best_key + k, cand_key(best, (uint32_t)f));
  }
}

// ---------------------------------------------------------------------------
// One CTA decides the whole level: each frontier node's split (features
// merged in order with need_replace, builder/mod.rs:313), validity
// (BestSplit::valid, :167), child ids in frontier order (RegTree::expand,
// regtree.rs:549), child statistics, which child's histogram is built, and
// the partition work items.
__device__ __forceinline__ hb_tree_node make_leaf(float value, float sum_hess) {
  hb_tree_node n;
  n.left = -1;
  n.right = -1;
  n.split_feature = 0;
  n.split_cond = 0.0f;
  n.default_left = 1;
  n.leaf_value = value;
  n.sum_hess = sum_hess;
  n.split_gain = 0.0f;
  n.split_bin = -1;
  n.reserved = 0;
  return n;
}

constexpr int kApplyThreads = 1024;

// T threads, one per frontier node: 256 while the frontier fits, whose block
// scans and barriers are shorter than 1024 threads'
template <int T>
__global__ void __launch_bounds__(T)
    k_apply(DevConst c, const uint32_t* __restrict__ fo, const float* __restrict__ cuts,
            const Cand* __restrict__ cand, const Front* __restrict__ front, Front* __restrict__ next,
            Decision* __restrict__ dec, PItem* __restrict__ items, LevelState* ls,
            LevelState* ls_next, hb_tree_node* __restrict__ tree, WNode* __restrict__ wtree,
            const Scale* __restrict__ scale, int depth, int leaf_only,
            unsigned long long* __restrict__ best_key) {
  pdl_wait();
  using Scan = cub::BlockScan<int, T>;
  __shared__ typename Scan::TempStorage tmp;
  const int n_front = ls->n_front;
  const int n_nodes = ls->n_nodes;
  const int k = threadIdx.x;
  const double ig = scale->ig, ih = scale->ih;
  if (depth == 0 && k == 0 && n_front > 0) tree[0] = make_leaf(0.0f, (float)(ll2d(front[0].h) * ih));

  // each node's best feature: its key from the scan (cand_key), cleared for
  // the next level
  int bf_k = -1;
  if (!leaf_only && k < n_front) {
    bf_k = key_feature(best_key[k]);
    best_key[k] = 0ull;
  }
  Front fr{};
  Cand best{};
  uint32_t best_f = 0;
  int valid = 0;
  if (k < n_front) {
    fr = front[k];
    if (!leaf_only) {
      best.loss = 0.0f;
      best.bin = -1;
      best.default_left = 1;
      const int bf = bf_k;
      if (bf >= 0) {
        best = cand[(uint64_t)k * c.n_cols + bf];
        best_f = (uint32_t)bf;
      }
      const double lh = ll2d(best.lh) * ih;
      const double rh = ll2d(fr.h - best.lh) * ih;
      valid = (double)best.loss > kRtEps && (double)best.loss >= c.gamma && lh > 0.0 &&
              rh > 0.0 && lh >= c.mcw && rh >= c.mcw;
    }
  }
  int pos = 0, n_split = 0;
  Scan(tmp).ExclusiveSum(valid, pos, n_split);
  __syncthreads();

  int n_items_k = 0;
  if (k < n_front) {
    Decision d{};
    d.split = valid;
    d.pair = pos;
    if (valid) {
      const long long lg = best.lg, lh = best.lh;
      const long long rg = fr.g - lg, rh = fr.h - lh;
      const double dlg = ll2d(lg) * ig, dlh = ll2d(lh) * ih;
      const double drg = ll2d(rg) * ig, drh = ll2d(rh) * ih;
      const int left_id = n_nodes + 2 * pos;
      hb_tree_node nd = tree[fr.node];
      nd.split_feature = best_f;
      nd.split_cond = best.bin < 0 ? kBelowAll : cuts[best.bin];
      nd.default_left = best.default_left ? 1u : 0u;
      nd.left = left_id;
      nd.right = left_id + 1;
      nd.split_bin = best.bin;
      nd.split_gain = best.loss;
      tree[fr.node] = nd;
      // the children's bounded weights (RegTree::expand), and their
      // monotone bounds from them (hist/mod.rs:648)
      const float wl = xgb_weight(dlg, dlh, c, (float)fr.lower, (float)fr.upper);
      const float wr = xgb_weight(drg, drh, c, (float)fr.lower, (float)fr.upper);
      tree[left_id] = make_leaf(wl, (float)dlh);
      tree[left_id + 1] = make_leaf(wr, (float)drh);
      const bool terminal = c.max_depth > 0 && depth + 1 >= c.max_depth;
      int lslot = -1, rslot = -1;
      if (!terminal) {
        const int base = (1 << (depth + 1)) - 1, half = 1 << depth;
        const bool left_built = lh <= rh;  // the child with the smaller Hessian sum
        lslot = left_built ? base + pos : base + half + pos;
        rslot = left_built ? base + half + pos : base + pos;
      }
      Front l{}, r{};
      l.node = left_id;
      l.slot = lslot;
      l.g = lg;
      l.h = lh;
      r.node = left_id + 1;
      r.slot = rslot;
      r.g = rg;
      r.h = rh;
      child_bounds(fr.lower, fr.upper, c.mono ? (int)c.mono[best_f] : 0, wl, wr, &l.lower, &l.upper,
                   &r.lower, &r.upper);
      next[2 * pos] = l;
      next[2 * pos + 1] = r;
      d.feature = best_f;
      const uint32_t fs = fo[best_f];
      d.limit = best.bin < 0 ? 0u : (uint32_t)(best.bin + 1) - fs;
      d.default_left = best.default_left;
      d.lg = lg;
      d.lh = lh;
      WNode wn;
      wn.left = left_id;
      wn.feature = best_f | (best.default_left ? 0x80000000u : 0u);
      wn.limit = d.limit;
      wn.leaf = 0.0f;
      wtree[fr.node] = wn;
      n_items_k = (int)((fr.len + kTile - 1) / kTile);
    } else {
      // finalize_leaf_values (shared.rs:174; calc_weight_bounded,
      // constraints.rs:70) then scale_leaves(eta).
      const float w = __double2float_rn(
          clamp_bounds(calc_weight(ll2d(fr.g) * ig, ll2d(fr.h) * ih, c), fr.lower, fr.upper));
      const float v = __fmul_rn(w, c.eta);
      tree[fr.node].leaf_value = v;
      d.leaf_value = v;
      WNode wn;
      wn.left = -1;
      wn.feature = 0u;
      wn.limit = 0u;
      wn.leaf = v;
      wtree[fr.node] = wn;
    }
    dec[k] = d;
  }
  int item0 = 0, n_items = 0;
  Scan(tmp).ExclusiveSum(n_items_k, item0, n_items);
  if (k < n_front) {
    dec[k].item_begin = item0;
    dec[k].item_count = n_items_k;
  }
  if (k == 0) {
    ls->n_items = n_items;
    ls->n_split = n_split;
    ls_next->n_front = 2 * n_split;
    ls_next->n_nodes = n_nodes + 2 * n_split;
    ls_next->tree_index = ls->tree_index;
  }
}

// ---------------------------------------------------------------------------
// Lossguide growth on the device (grow_lossguide, src/tree/builder/hist/
// mod.rs:505). A step merges the pending nodes' scans into their best splits
// and pushes them in order, then pops until a node expands or growth ends.
// A popped node becomes a leaf when the tree already has max_leaves leaves
// (growth then stops and the nodes left in the heap are leaves too), or when
// it is too deep or has no valid split. An expanded node is set up as a
// one-node level for the partition, histogram and scan kernels. The heap is
// Rust's BinaryHeap as the host builder uses it (push: sift_up; pop: swap
// the last into the root, sift_down_to_bottom, sift_up), keyed by the
// f64::total_cmp order of the best loss change.
constexpr int kLgThreads = 256;  // the heap's copies in and out

__device__ __forceinline__ long long total_key(double v) {
  const long long b = __double_as_longlong(v);
  return b ^ (long long)((unsigned long long)(b >> 63) >> 1);
}

__device__ void lg_sift_up(LgKey* heap, int start, int pos) {
  const LgKey hole = heap[pos];
  while (pos > start) {
    const int parent = (pos - 1) / 2;
    if (hole.key <= heap[parent].key) break;
    heap[pos] = heap[parent];
    pos = parent;
  }
  heap[pos] = hole;
}

__device__ LgKey lg_pop(LgKey* heap, int& n) {
  LgKey item = heap[n - 1];
  --n;
  if (n > 0) {
    const LgKey root = heap[0];
    heap[0] = item;
    item = root;
    const int end = n;
    int pos = 0;
    const LgKey hole = heap[0];
    int child = 1;
    while (end >= 2 && child <= end - 2) {
      if (heap[child].key <= heap[child + 1].key) child += 1;
      heap[pos] = heap[child];
      pos = child;
      child = 2 * pos + 1;
    }
    if (child == end - 1) {
      heap[pos] = heap[child];
      pos = child;
    }
    heap[pos] = hole;
    lg_sift_up(heap, 0, pos);
  }
  return item;
}

// finalize_leaf_values (shared.rs:174) then scale_leaves(eta), as k_apply
__device__ void lg_leaf(const LgNode& e, const DevConst& c, double ig, double ih,
                        hb_tree_node* tree, WNode* wtree) {
  const float w =
      __double2float_rn(clamp_bounds(calc_weight(ll2d(e.g) * ig, ll2d(e.h) * ih, c), e.lower, e.upper));
  const float v = __fmul_rn(w, c.eta);
  tree[e.nid].leaf_value = v;
  WNode wn;
  wn.left = -1;
  wn.feature = 0u;
  wn.limit = 0u;
  wn.leaf = v;
  wtree[e.nid] = wn;
}

__device__ void lg_step_serial(const DevConst& c, const uint32_t* __restrict__ fo,
                               const float* __restrict__ cuts, Front* front, Front* next,
                               Decision* dec, LevelState* ls, LevelState* ls_next,
                               hb_tree_node* __restrict__ tree, WNode* __restrict__ wtree, double ig,
                               double ih, LgKey* heap, const LgNode* pool, LgState* st,
                               const LgState S0, const LgKey* s_new, int32_t* __restrict__ ndepth,
                               int max_leaves, int depth_limit, int final_step, int& n_out,
                               int& n_rest);

__global__ void __launch_bounds__(kLgThreads)
    k_lg_step(DevConst c, const uint32_t* __restrict__ fo, const float* __restrict__ cuts,
              const Cand* __restrict__ cand, const Front* __restrict__ pend, Front* front,
              Front* next, Decision* dec, LevelState* ls, LevelState* ls_next,
              hb_tree_node* __restrict__ tree, WNode* __restrict__ wtree,
              const Scale* __restrict__ scale, LgKey* __restrict__ heap, LgNode* __restrict__ pool,
              LgState* st, int32_t* __restrict__ ndepth, int max_leaves, int depth_limit,
              int final_step, unsigned long long* __restrict__ best_key) {
  pdl_wait();
  __shared__ LgKey s_new[2];
  __shared__ int s_n, s_rest;
  extern __shared__ __align__(16) unsigned char lg_dyn[];
  LgKey* sheap = reinterpret_cast<LgKey*>(lg_dyn);  // the heap, worked in shared memory
  const LgState S0 = *st;
  if (S0.done) return;
  const double ig = scale->ig, ih = scale->ih;
  const int np = S0.n_pending;
  for (int i = threadIdx.x; i < S0.heap_n; i += kLgThreads) sheap[i] = heap[i];  // the heap in
  // each pending node's best split over its features (need_replace,
  // builder/mod.rs:313): its key from the scan (cand_key), cleared for the
  // next step; the node into the pool at its id
  if (threadIdx.x < np) {
    const int node = threadIdx.x;
    const int bf = key_feature(best_key[node]);
    best_key[node] = 0ull;
    const Front fr = pend[node];
    LgNode x;
    x.nid = fr.node;
    x.depth = ndepth[fr.node];
    x.begin = fr.begin;
    x.len = fr.len;
    x.g = fr.g;
    x.h = fr.h;
    x.lower = fr.lower;
    x.upper = fr.upper;
    if (bf >= 0) {
      const Cand cd = cand[(uint64_t)node * c.n_cols + bf];
      x.loss = cd.loss;
      x.feature = bf;
      x.bin = cd.bin;
      x.default_left = cd.default_left;
      x.lg = cd.lg;
      x.lh = cd.lh;
    } else {
      x.loss = 0.0f;
      x.feature = -1;
      x.bin = -1;
      x.default_left = 1;
      x.lg = x.lh = 0;
    }
    x.key = total_key((double)x.loss);
    pool[x.nid] = x;
    LgKey k;
    k.key = x.key;
    k.nid = x.nid;
    k.pad = 0;
    s_new[node] = k;
  }
  __syncthreads();
  if (threadIdx.x == 0) lg_step_serial(c, fo, cuts, front, next, dec, ls, ls_next, tree, wtree, ig, ih,
                                       sheap, pool, st, S0, s_new, ndepth, max_leaves, depth_limit,
                                       final_step, s_n, s_rest);
  __syncthreads();
  // when growth ended, the nodes left in the heap become leaves
  for (int i = threadIdx.x; i < s_rest; i += kLgThreads) lg_leaf(pool[sheap[i].nid], c, ig, ih, tree, wtree);
  for (int i = threadIdx.x; i < s_n; i += kLgThreads) heap[i] = sheap[i];  // the heap out
}

// The heap work of a lossguide step, one thread, on the shared copy of the
// heap: the new children pushed, then pops in BinaryHeap order until one
// node expands (its split, children, partition decision) or growth ends.
__device__ void lg_step_serial(const DevConst& c, const uint32_t* __restrict__ fo,
                               const float* __restrict__ cuts, Front* front, Front* next,
                               Decision* dec, LevelState* ls, LevelState* ls_next,
                               hb_tree_node* __restrict__ tree, WNode* __restrict__ wtree, double ig,
                               double ih, LgKey* heap, const LgNode* pool, LgState* st,
                               const LgState S0, const LgKey* s_new, int32_t* __restrict__ ndepth,
                               int max_leaves, int depth_limit, int final_step, int& n_out,
                               int& n_rest) {
  const int np = S0.n_pending;
  LgState S = S0;
  int n = S.heap_n;
  for (int k = 0; k < np; ++k) {
    heap[n] = s_new[k];
    ++n;
    lg_sift_up(heap, 0, n - 1);
  }
  LevelState idle{};
  *ls = idle;  // nothing to partition unless a node expands (also resets done_ctas)
  ls_next->n_front = 0;
  bool expanded = false;
  while (n > 0) {
    const LgNode e = pool[lg_pop(heap, n).nid];
    if (S.n_leaves >= max_leaves) {
      lg_leaf(e, c, ig, ih, tree, wtree);
      S.done = 1;
      break;
    }
    const double lh = ll2d(e.lh) * ih, rh = ll2d(e.h - e.lh) * ih;
    const bool valid = e.feature >= 0 && (double)e.loss > kRtEps && (double)e.loss >= c.gamma &&
                       lh > 0.0 && rh > 0.0 && lh >= c.mcw && rh >= c.mcw;
    if (!(e.depth < depth_limit && valid) || final_step) {
      lg_leaf(e, c, ig, ih, tree, wtree);
      continue;
    }
    // expand (prepare_split, hist/mod.rs:639): children ids in order
    const int left_id = S.n_nodes;
    S.n_nodes += 2;
    const long long rg_q = e.g - e.lg, rh_q = e.h - e.lh;
    const double dlg = ll2d(e.lg) * ig, dlh = ll2d(e.lh) * ih;
    const double drg = ll2d(rg_q) * ig, drh = ll2d(rh_q) * ih;
    hb_tree_node nd = tree[e.nid];
    nd.split_feature = (uint32_t)e.feature;
    nd.split_cond = e.bin < 0 ? kBelowAll : cuts[e.bin];
    nd.default_left = e.default_left ? 1u : 0u;
    nd.left = left_id;
    nd.right = left_id + 1;
    nd.split_bin = e.bin;
    nd.split_gain = e.loss;
    tree[e.nid] = nd;
    const float wl = xgb_weight(dlg, dlh, c, (float)e.lower, (float)e.upper);
    const float wr = xgb_weight(drg, drh, c, (float)e.lower, (float)e.upper);
    tree[left_id] = make_leaf(wl, (float)dlh);
    tree[left_id + 1] = make_leaf(wr, (float)drh);
    ndepth[left_id] = ndepth[left_id + 1] = e.depth + 1;
    const uint32_t fs = fo[e.feature];
    const uint32_t limit = e.bin < 0 ? 0u : (uint32_t)(e.bin + 1) - fs;
    WNode wn;
    wn.left = left_id;
    wn.feature = (uint32_t)e.feature | (e.default_left ? 0x80000000u : 0u);
    wn.limit = limit;
    wn.leaf = 0.0f;
    wtree[e.nid] = wn;
    Front f0{};
    f0.node = e.nid;
    f0.slot = e.nid;  // histogram slot = node id
    f0.begin = e.begin;
    f0.len = e.len;
    f0.g = e.g;
    f0.h = e.h;
    f0.lower = e.lower;
    f0.upper = e.upper;
    front[0] = f0;
    Decision d{};
    d.split = 1;
    d.pair = 0;
    d.feature = (uint32_t)e.feature;
    d.limit = limit;
    d.default_left = e.default_left;
    d.item_begin = 0;
    d.item_count = (int)((e.len + kTile - 1) / kTile);
    d.lg = e.lg;
    d.lh = e.lh;
    dec[0] = d;
    Front l{}, r{};
    l.node = left_id;
    l.slot = left_id;
    l.g = e.lg;
    l.h = e.lh;
    r.node = left_id + 1;
    r.slot = left_id + 1;
    r.g = rg_q;
    r.h = rh_q;
    child_bounds(e.lower, e.upper, c.mono ? (int)c.mono[e.feature] : 0, wl, wr, &l.lower, &l.upper,
                 &r.lower, &r.upper);
    next[0] = l;
    next[1] = r;
    LevelState lv{};
    lv.n_front = 1;
    lv.n_items = d.item_count;
    lv.n_split = 1;
    lv.n_nodes = S.n_nodes;
    *ls = lv;
    ls_next->n_front = 2;
    S.n_leaves += 1;
    expanded = true;
    break;
  }
  if (!expanded) S.done = 1;
  n_rest = 0;
  if (S.done) {  // the nodes left in the heap are leaves (the whole CTA writes them)
    n_rest = n;
    n = 0;
  }
  S.heap_n = n;
  S.n_pending = expanded ? 2 : 0;
  *st = S;
  ls_next->n_nodes = S.n_nodes;
  n_out = n;
}

// Lossguide state of a new tree: the root pending, one node, one leaf.
__global__ void k_lg_setup(LgState* st, int32_t* ndepth, hb_tree_node* tree, const Front* root,
                           const Scale* scale, LevelState* ls_next) {
  pdl_wait();
  LgState S{};
  S.heap_n = 0;
  S.n_nodes = 1;
  S.n_leaves = 1;
  S.done = 0;
  S.n_pending = 1;
  *st = S;
  ndepth[0] = 0;
  tree[0] = make_leaf(0.0f, (float)(ll2d(root->h) * scale->ih));
  ls_next->n_nodes = 1;
}


// ---------------------------------------------------------------------------
// Stable partition (partition.rs:106, route_column :206): present local bin
// < limit goes left, missing follows default_left; the left child keeps the
// segment's first rows, both in ascending order. Three passes over tiles:
// direction bits + counts, per-node exclusive scan, scatter. Leaf items add
// the node's eta-scaled leaf value to the margins of its rows instead.
constexpr int kPartThreads = 256;

// The frontier node owning work item `it` (items are laid out node after
// node, dec[k].item_begin ascending) and the item's tile.
__device__ __forceinline__ PItem locate_item(const Decision* __restrict__ dec, int n_front, int it,
                                             const Front* __restrict__ front) {
  int lo = 0, hi = n_front - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (dec[mid].item_begin <= it) lo = mid; else hi = mid - 1;
  }
  PItem p;
  p.k = lo;
  p.kind = dec[lo].split ? 1 : 2;
  p.off = (uint32_t)(it - dec[lo].item_begin) * kTile;
  p.len = min((uint32_t)kTile, front[lo].len - p.off);
  return p;
}

// Positions of a tile: warp w owns 256 consecutive ones, lane l of pass j
// position w * 256 + j * 32 + l, so a warp's directions are 8 ballot words
// in position order and its prefix needs no other warp until the end.
constexpr int kPerThread = kTile / kPartThreads;  // 8

template <bool CSR>
__global__ void __launch_bounds__(kPartThreads)
    k_part_count(DevConst c, const uint8_t* __restrict__ col, const uint64_t* __restrict__ colmiss,
                 const uint8_t* __restrict__ rec, int use_record,
                 const uint32_t* __restrict__ rows_in, int identity, const Front* __restrict__ front,
                 const Decision* __restrict__ dec, const PItem* __restrict__ items,
                 const LevelState* __restrict__ ls, uint32_t* __restrict__ dirbits,
                 uint32_t* __restrict__ item_left, uint32_t* __restrict__ rows_copy) {
  pdl_wait();
  const int it = blockIdx.x;
  if (it >= ls->n_items) return;
  const PItem pi = locate_item(dec, ls->n_front, it, front);
  if (pi.kind != 1) return;
  const Front fr = front[pi.k];
  const Decision d = dec[pi.k];
  const uint8_t* colf = col + (uint64_t)d.feature * c.n_rows;
  const uint64_t words = (c.n_rows + 63) / 64;
  const uint64_t* missf = colmiss ? colmiss + (uint64_t)d.feature * words : nullptr;
  const uint32_t mword = c.mask_off + 4 * (d.feature >> 5);
  const uint32_t mbit = d.feature & 31;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t base = fr.begin + pi.off;
  uint32_t row[kPerThread];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t i = warp * 256 + j * 32 + lane;
    const uint32_t at = base + min(i, pi.len - 1);
    row[j] = identity ? at : rows_in[at];
  }
  if (rows_copy) {  // the tile's row ids, for a scatter that writes back in place
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const uint32_t i = warp * 256 + j * 32 + lane;
      if (i < pi.len) rows_copy[base + i] = row[j];
    }
  }
  uint32_t bin[kPerThread];
  bool miss[kPerThread];
  const uint32_t csr_lo = c.csr ? __ldg(c.fo + d.feature) : 0u;
  const uint32_t csr_hi = c.csr ? __ldg(c.fo + d.feature + 1) : 0u;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t r = row[j];
    if (CSR) {
      uint32_t lb = 0;
      miss[j] = !csr_find(c.csr_bins, __ldg(c.csr_ptr + r), __ldg(c.csr_ptr + r + 1), csr_lo, csr_hi, lb);
      bin[j] = lb;
    } else if (use_record) {
      const uint8_t* rp = rec + rec_offset(r, c.stride, c.blk);
      bin[j] = rp[d.feature];
      miss[j] = (*reinterpret_cast<const uint32_t*>(rp + mword) >> mbit) & 1u;
    } else {
      bin[j] = colf[r];
      miss[j] = missf && ((missf[r >> 6] >> (r & 63)) & 1ull);
    }
  }
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t i = warp * 256 + j * 32 + lane;
    const bool left = i < pi.len && (miss[j] ? (d.default_left != 0) : (bin[j] < d.limit));
    const unsigned bal = __ballot_sync(kFull, left);
    if (lane == j) dirbits[(uint64_t)it * kTileWords + warp * kPerThread + j] = bal;
    cnt += __popc(bal);
  }
  __shared__ int s_cnt[kPartThreads / 32];
  if (lane == 0) s_cnt[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) t += s_cnt[w];
    item_left[it] = (uint32_t)t;
  }
}

// One-pass partition of depthwise growth: one CTA per tile of a splitting
// node (2048 rows), which routes its rows (the split feature's column and
// missing bitmap, the partition's rule) and moves them at once: its left
// rows to a chunk at the start of the node's segment, its right rows to a
// chunk at the end, each chunk reserved with one atomic on the node's fill
// counts (fill[2 pair], fill[2 pair + 1]; zero before the pass). Rows stay
// ascending within a chunk, but the chunks of a child follow in the order
// the CTAs reserved them, so a child's row order is not the stable one.
// Nothing computed from a segment depends on its order: histograms are
// exact integer sums and the leaf adds go by row. Saves the stable scheme's
// second pass over the rows (the scatter) and its per-node tile scan.
// half = 0: the children take the parent's positions in rows_out (another
// buffer); half = n (lossguide, rows_in == rows_out spanning 2n): they take
// the positions half away in the other half of the buffer (seg_flip).
__device__ __forceinline__ uint32_t seg_flip(uint32_t begin, uint32_t half) {
  return half == 0u ? begin : begin >= half ? begin - half : begin + half;
}

template <bool CSR>
__global__ void __launch_bounds__(kPartThreads, 6)
    k_part_onepass(DevConst c, const uint8_t* __restrict__ col, const uint64_t* __restrict__ colmiss,
                   const uint32_t* rows_in, int identity, const Front* __restrict__ front,
                   const Decision* __restrict__ dec, const LevelState* __restrict__ ls,
                   uint32_t* __restrict__ fill, uint32_t* rows_out, uint32_t half) {
  pdl_wait();
  const int it = blockIdx.x;
  if (it >= ls->n_items) return;
  const PItem pi = locate_item(dec, ls->n_front, it, front);
  if (pi.kind != 1) return;
  const Front fr = front[pi.k];
  const Decision d = dec[pi.k];
  const uint8_t* colf = col + (uint64_t)d.feature * c.n_rows;
  const uint64_t words = (c.n_rows + 63) / 64;
  // the bitmap read as 32-bit words (bit r & 31 of word r >> 5)
  const uint32_t* missw = colmiss ? reinterpret_cast<const uint32_t*>(colmiss + (uint64_t)d.feature * words)
                                  : nullptr;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t base = fr.begin + pi.off;
  const uint32_t t0 = warp * 256 + lane;  // position of row j: t0 + 32 j
  const uint32_t* rin = rows_in + base + t0;
  uint32_t row[kPerThread];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {  // past the tile's end: row 0, read but not moved
    const bool in = t0 + j * 32 < pi.len;
    row[j] = !in ? 0u : identity ? base + t0 + j * 32 : rin[j * 32];
  }
  const uint32_t csr_lo = CSR ? __ldg(c.fo + d.feature) : 0u;
  const uint32_t csr_hi = CSR ? __ldg(c.fo + d.feature + 1) : 0u;
  uint32_t bal[kPerThread];
  uint32_t wl = 0;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t r = row[j];
    bool miss;
    uint32_t bin;
    if (CSR) {
      uint32_t lb = 0;
      miss = !csr_find(c.csr_bins, __ldg(c.csr_ptr + r), __ldg(c.csr_ptr + r + 1), csr_lo, csr_hi, lb);
      bin = lb;
    } else {
      bin = colf[r];
      miss = missw && ((missw[r >> 5] >> (r & 31)) & 1u);
    }
    const bool left = t0 + j * 32 < pi.len && (miss ? (d.default_left != 0) : (bin < d.limit));
    bal[j] = __ballot_sync(kFull, left);
    wl += __popc(bal[j]);
  }
  // the warps' left counts, the tile's totals and the chunk reservations
  __shared__ uint32_t s_wl[kPartThreads / 32];
  __shared__ uint32_t s_base_l, s_base_r;
  if (lane == 0) s_wl[warp] = wl;
  __syncthreads();
  uint32_t before = 0, tile_l = 0;
#pragma unroll
  for (int w = 0; w < kPartThreads / 32; ++w) {
    const uint32_t v = s_wl[w];
    before += w < warp ? v : 0u;
    tile_l += v;
  }
  const uint32_t tile_r = pi.len - tile_l;
  if (threadIdx.x == 0) {
    s_base_l = tile_l ? atomicAdd(&fill[2 * d.pair], tile_l) : 0u;
    s_base_r = tile_r ? atomicAdd(&fill[2 * d.pair + 1], tile_r) : 0u;
  }
  __syncthreads();
  const uint32_t out0 = seg_flip(fr.begin, half);
  // row at position i of the tile, lrank left rows before it: left to
  // left0 + lrank, right to right0 + (i - lrank)
  const uint32_t left0 = out0 + s_base_l;
  const uint32_t right0 = out0 + fr.len - s_base_r - tile_r;
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t i = t0 + j * 32;
    const uint32_t lrank = before + __popc(bal[j] & lt);
    const uint32_t dst = ((bal[j] >> lane) & 1u) ? left0 + lrank : right0 + (i - lrank);
    if (i < pi.len) rows_out[dst] = row[j];
    before += __popc(bal[j]);
  }
}

// After k_part_onepass: the children's segments from the fill counts (the
// left child first), the counts cleared for the next level, then the next
// level's histogram plan. One CTA of T threads, one per frontier node.
template <int T>
__device__ void hist_plan_body(const Front* __restrict__ front, const Decision* __restrict__ dec,
                               const LevelState* __restrict__ ls, const Front* next,
                               HEntry* __restrict__ entries, Triple* __restrict__ pairs,
                               LevelState* __restrict__ ls_next, int terminal);
template <int T>
__global__ void __launch_bounds__(T)
    k_part_plan(const Front* __restrict__ front, const Decision* __restrict__ dec, const LevelState* ls,
                uint32_t* __restrict__ fill, Front* next, HEntry* __restrict__ entries,
                Triple* __restrict__ pairs, LevelState* __restrict__ ls_next, uint32_t half) {
  pdl_wait();
  const int k = threadIdx.x;
  if (k < ls->n_front) {
    const Decision d = dec[k];
    if (d.split) {
      const Front fr = front[k];
      const uint32_t L = fill[2 * d.pair];
      const uint32_t b = seg_flip(fr.begin, half);
      next[2 * d.pair].begin = b;
      next[2 * d.pair].len = L;
      next[2 * d.pair + 1].begin = b + L;
      next[2 * d.pair + 1].len = fr.len - L;
      fill[2 * d.pair] = 0u;
      fill[2 * d.pair + 1] = 0u;
    }
  }
  __syncthreads();
  hist_plan_body<T>(front, dec, ls, next, entries, pairs, ls_next, 0);
}

// One CTA per splitting frontier node: exclusive scan of its tiles' left
// counts (each thread sums kScanPer consecutive tiles, then one block scan
// covers kScanThreads * kScanPer tiles); the children's segments. With
// `entries`, the last CTA to finish then plans the next level's histograms
// (hist_plan_body), which needs every node's segments.
template <int T>
__device__ void hist_plan_body(const Front* __restrict__ front, const Decision* __restrict__ dec,
                               const LevelState* __restrict__ ls, const Front* next,
                               HEntry* __restrict__ entries, Triple* __restrict__ pairs,
                               LevelState* __restrict__ ls_next, int terminal);
constexpr int kScanThreads = 1024;
constexpr int kScanPer = 8;
static_assert(kScanThreads == kApplyThreads, "the plan runs on one tile-scan CTA");
__global__ void __launch_bounds__(kScanThreads)
    k_part_scan(const Front* __restrict__ front, const Decision* __restrict__ dec,
                LevelState* ls, const uint32_t* __restrict__ item_left,
                uint32_t* __restrict__ item_left_off, Front* next, HEntry* __restrict__ entries,
                Triple* __restrict__ pairs, LevelState* __restrict__ ls_next) {
  pdl_wait();
  using Scan = cub::BlockScan<uint32_t, kScanThreads>;
  __shared__ typename Scan::TempStorage tmp;
  const int k = blockIdx.x;
  const Decision d = k < ls->n_front ? dec[k] : Decision{};
  if (k < ls->n_front && d.split) {
    uint32_t run = 0;
    for (int base = 0; base < d.item_count; base += kScanThreads * kScanPer) {
      const int t0 = base + (int)threadIdx.x * kScanPer;
      uint32_t v[kScanPer];
      uint32_t sum = 0;
#pragma unroll
      for (int i = 0; i < kScanPer; ++i) {
        v[i] = t0 + i < d.item_count ? item_left[d.item_begin + t0 + i] : 0u;
        sum += v[i];
      }
      uint32_t ex = 0, agg = 0;
      Scan(tmp).ExclusiveSum(sum, ex, agg);
      __syncthreads();
      uint32_t at = run + ex;
#pragma unroll
      for (int i = 0; i < kScanPer; ++i) {
        if (t0 + i < d.item_count) item_left_off[d.item_begin + t0 + i] = at;
        at += v[i];
      }
      run += agg;
    }
    if (threadIdx.x == 0) {
      const Front fr = front[k];
      next[2 * d.pair].begin = fr.begin;
      next[2 * d.pair].len = run;
      next[2 * d.pair + 1].begin = fr.begin + run;
      next[2 * d.pair + 1].len = fr.len - run;
    }
  }
  if (entries == nullptr) return;
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    __threadfence();  // this CTA's segments before its count
    s_last = atomicAdd(&ls->done_ctas, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  hist_plan_body<kScanThreads>(front, dec, ls, next, entries, pairs, ls_next, 0);
}

__global__ void __launch_bounds__(kPartThreads)
    k_part_scatter(const Front* __restrict__ front, const Decision* __restrict__ dec,
                   const PItem* __restrict__ items, const LevelState* __restrict__ ls,
                   const uint32_t* __restrict__ dirbits, const uint32_t* __restrict__ item_left_off,
                   const Front* __restrict__ next, const uint32_t* __restrict__ rows_in,
                   int identity, uint32_t* __restrict__ rows_out) {
  pdl_wait();
  const int it = blockIdx.x;
  if (it >= ls->n_items) return;
  const PItem pi = locate_item(dec, ls->n_front, it, front);
  if (pi.kind != 1) return;
  const Front fr = front[pi.k];
  const Decision d = dec[pi.k];
  const uint32_t L = next[2 * d.pair].len;
  const uint32_t loff = item_left_off[it];
  const uint32_t base_left = fr.begin + loff;
  const uint32_t base_right = fr.begin + L + (pi.off - loff);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t base = fr.begin + pi.off;
  uint32_t row[kPerThread];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t i = warp * 256 + j * 32 + lane;
    const uint32_t at = base + min(i, pi.len - 1);
    row[j] = identity ? at : rows_in[at];
  }
  const uint32_t mine = lane < kPerThread ? dirbits[(uint64_t)it * kTileWords + warp * kPerThread + lane] : 0u;
  uint32_t bal[kPerThread];
  uint32_t wcount = 0;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    bal[j] = __shfl_sync(kFull, mine, j);
    wcount += __popc(bal[j]);
  }
  __shared__ uint32_t s_cnt[kPartThreads / 32];
  if (lane == 0) s_cnt[warp] = wcount;
  __syncthreads();
  uint32_t before = 0;  // left positions of the tile before this warp's
  for (int w = 0; w < warp; ++w) before += s_cnt[w];
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const uint32_t i = warp * 256 + j * 32 + lane;
    const uint32_t lrank = before + __popc(bal[j] & lt);
    if (i < pi.len) {
      if ((bal[j] >> lane) & 1u) {
        rows_out[base_left + lrank] = row[j];
      } else {
        rows_out[base_right + (i - lrank)] = row[j];
      }
    }
    before += __popc(bal[j]);
  }
}

// Histogram plan of the next level: for every split (not at the depth
// limit) the child with the smaller Hessian sum is built, its sibling is
// parent - built. Entries are in pair order with running row prefixes. Run
// by one CTA of kApplyThreads; the children's segments are read past L1
// (other CTAs wrote them).
__device__ __forceinline__ Front load_front_cg(const Front* p) {
  const int4* q = reinterpret_cast<const int4*>(p);
  const int4 x = __ldcg(q), y = __ldcg(q + 1);
  Front f;
  f.node = x.x;
  f.slot = x.y;
  f.begin = (uint32_t)x.z;
  f.len = (uint32_t)x.w;
  f.g = ((long long)(uint32_t)y.y << 32) | (uint32_t)y.x;
  f.h = ((long long)(uint32_t)y.w << 32) | (uint32_t)y.z;
  return f;
}

template <int T>
__device__ void hist_plan_body(const Front* __restrict__ front, const Decision* __restrict__ dec,
                               const LevelState* __restrict__ ls, const Front* next,
                               HEntry* __restrict__ entries, Triple* __restrict__ pairs,
                               LevelState* __restrict__ ls_next, int terminal) {
  using Scan = cub::BlockScan<unsigned long long, T>;
  __shared__ typename Scan::TempStorage tmp;
  const int k = threadIdx.x;
  const int n_front = ls->n_front;
  unsigned long long rows = 0;
  HEntry en{};
  Triple tr{};
  bool active = false;
  if (!terminal && k < n_front) {
    const Decision d = dec[k];
    if (d.split) {
      active = true;
      const Front l = load_front_cg(&next[2 * d.pair]), r = load_front_cg(&next[2 * d.pair + 1]);
      const bool left_built = l.h <= r.h;
      const Front& b = left_built ? l : r;
      const Front& s = left_built ? r : l;
      en.slot = b.slot;
      en.identity = 0;
      en.begin = b.begin;
      en.len = b.len;
      rows = b.len;
      tr.parent = front[k].slot;
      tr.built = b.slot;
      tr.sibling = s.slot;
    }
  }
  unsigned long long prefix = 0, total = 0;
  Scan(tmp).ExclusiveSum(rows, prefix, total);
  if (active) {
    const int p = dec[k].pair;
    en.prefix = prefix;
    entries[p] = en;
    pairs[p] = tr;
  }
  if (k == 0) {
    const int n = terminal ? 0 : ls->n_split;
    ls_next->n_hentries = n;
    ls_next->n_pairs = n;
    ls_next->hist_rows = total;
  }
}

__global__ void k_root_setup(uint64_t n_rows, Front* front, HEntry* entries, LevelState* ls) {
  pdl_wait();
  Front f{};
  f.node = 0;
  f.slot = 0;
  f.begin = 0;
  f.len = (uint32_t)n_rows;
  front[0] = f;
  HEntry e{};
  e.slot = 0;
  e.identity = 1;
  e.begin = 0;
  e.len = (uint32_t)n_rows;
  e.prefix = 0;
  entries[0] = e;
  ls->n_front = 1;
  ls->n_nodes = 1;
  ls->n_hentries = 1;
  ls->hist_rows = n_rows;
}

__global__ void k_root_stats(Front* front, const long long* totals) {
  pdl_wait();
  front[0].g = totals[0];
  front[0].h = totals[1];
}

__global__ void k_finish_tree(const hb_tree_node* __restrict__ tree, const LevelState* ls_last,
                              hb_tree_node* __restrict__ forest, uint32_t* counts,
                              int32_t* tree_counter, uint32_t max_nodes) {
  pdl_wait();
  const int t = *tree_counter;
  const int n = ls_last->n_nodes;
  for (int i = threadIdx.x; i < n; i += blockDim.x) forest[(uint64_t)t * max_nodes + i] = tree[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    counts[t] = (uint32_t)n;
    *tree_counter = t + 1;
  }
}

__global__ void k_dequantize(const longlong2* __restrict__ hist, uint32_t n,
                             const Scale* __restrict__ scale, double* __restrict__ out) {
  const double ig = scale->ig, ih = scale->ih;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const longlong2 v = hist[i];
    out[2 * i] = ll2d(v.x) * ig;
    out[2 * i + 1] = ll2d(v.y) * ih;
  }
}

__global__ void k_add_segment(const uint32_t* __restrict__ rows, uint32_t begin, uint32_t len,
                              float value, float* __restrict__ margin) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x) {
    const uint32_t r = rows[begin + i];
    margin[r] = __fadd_rn(margin[r], value);
  }
}

// RowEngine helpers (one launch each, in place of per-segment work on the
// host):
// rows[i] = first + i: the row list of a contiguous run, built on the device
// instead of copied from the host.
__global__ void k_fill(float* __restrict__ p, float v, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

__global__ void k_iota(uint32_t* __restrict__ rows, uint32_t first, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    rows[i] = first + (uint32_t)i;
}

// Each segment (offset, len) gets its value added to the margins of its
// rows: one CTA per segment, a grid-stride loop inside.
__global__ void k_add_segments(const uint32_t* __restrict__ rows, const uint4* __restrict__ tiles,
                               float* __restrict__ margin) {
  const uint4 t = tiles[blockIdx.x];  // first row position, length, leaf value bits
  const float v = __uint_as_float(t.z);
  for (uint32_t i = threadIdx.x; i < t.y; i += blockDim.x) {
    const uint32_t r = rows[t.x + i];
    margin[r] = __fadd_rn(margin[r], v);
  }
}

// A partition's last step, one CTA per work item (a tile of a split's
// segment): the tile's rows, which the scatter wrote to rows_out, copied back
// to rows_in (where the children's segments then live); the CTA of each
// split's first tile also writes the children's first and last row ids to
// ends[4k .. 4k + 3] (the host tells contiguous segments from them).
__global__ void k_finish_partition(const PItem* __restrict__ items, const Front* __restrict__ parents,
                                   const Front* __restrict__ kids, const uint32_t* __restrict__ rows_out,
                                   uint32_t* __restrict__ rows_in, uint32_t* __restrict__ ends) {
  const PItem pi = items[blockIdx.x];
  const uint32_t base = parents[pi.k].begin + pi.off;
  for (uint32_t i = threadIdx.x; i < pi.len; i += blockDim.x) rows_in[base + i] = rows_out[base + i];
  if (pi.off == 0 && threadIdx.x < 2) {
    const int k = pi.k;
    const Front f = kids[2 * k + threadIdx.x];
    ends[4 * k + 2 * threadIdx.x] = f.len ? rows_out[f.begin] : 0u;
    ends[4 * k + 2 * threadIdx.x + 1] = f.len ? rows_out[f.begin + f.len - 1] : 0u;
  }
}

// The fixed-point totals of a segment's rows (exact int64 sums, the order
// free): per-CTA sums added atomically into totals[0..1].
__global__ void k_seg_total(const uint32_t* __restrict__ rows, uint64_t begin, uint64_t len,
                            const float2* __restrict__ gpair, const Scale* __restrict__ scale,
                            long long* __restrict__ totals) {
  const double fg = scale->fg, fh = scale->fh;
  long long tg = 0, th = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (uint64_t)gridDim.x * blockDim.x) {
    const float2 p = gpair[rows[begin + i]];
    tg += __double2ll_rn((double)p.x * fg);
    th += __double2ll_rn((double)p.y * fh);
  }
  using BR = cub::BlockReduce<long long, 256>;
  __shared__ typename BR::TempStorage tmp;
  const long long sg = BR(tmp).Sum(tg);
  __syncthreads();
  const long long sh = BR(tmp).Sum(th);
  if (threadIdx.x == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&totals[0]), (unsigned long long)sg);
    atomicAdd(reinterpret_cast<unsigned long long*>(&totals[1]), (unsigned long long)sh);
  }
}

}  // namespace

void launch_fill(float* p, float v, uint64_t n, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8));
  k_fill<<<grid, 256, 0, s>>>(p, v, n);
}

void launch_iota(uint32_t* rows, uint32_t first, uint64_t n, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8));
  k_iota<<<grid, 256, 0, s>>>(rows, first, n);
}

void launch_add_segments(const uint32_t* rows, const uint4* tiles, uint32_t n_tiles, float* margin,
                         cudaStream_t s) {
  if (n_tiles) k_add_segments<<<n_tiles, 256, 0, s>>>(rows, tiles, margin);
}

void launch_finish_partition(const PItem* items, int n_items, const Front* parents, const Front* kids,
                             const uint32_t* rows_out, uint32_t* rows_in, uint32_t* ends, cudaStream_t s) {
  if (n_items > 0) k_finish_partition<<<n_items, 256, 0, s>>>(items, parents, kids, rows_out, rows_in, ends);
}

void launch_seg_total(const uint32_t* rows, uint64_t begin, uint64_t len, const float2* gpair,
                      const Scale* scale, long long* totals, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((len + 255) / 256, (uint64_t)n_sm * 4));
  k_seg_total<<<grid, 256, 0, s>>>(rows, begin, len, gpair, scale, totals);
}

// ---------------------------------------------------------------------------
// Launchers.
void launch_gradients(int kind, float* margin, const float* label, const float* weight, float spw,
                      float min_hess, uint64_t n, uint64_t vrows, float2* gpair, Scale* scale,
                      const WNode* wtree, const LevelState* ls_last, int max_nodes, int walk_depth,
                      uint8_t* rec, uint32_t stride, uint32_t mask_off, uint32_t blk, uint32_t blk_pair,
                      const int* pending, int n_sm, cudaStream_t s) {
  int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8);
  if (grid < 1) grid = 1;
  const size_t smem = wtree ? sizeof(WNode) * (size_t)max_nodes : 0;
  if (blk == 3 && blk_pair == 96 && stride == 32 && mask_off <= 28) {
    const uint64_t nblk = (n + 2) / 3;
    int g3 = (int)std::min<uint64_t>((nblk + kGradThreads - 1) / kGradThreads, (uint64_t)n_sm * 4);
    if (g3 < 1) g3 = 1;
    const int ct = (wtree && walk_depth > 0 && walk_depth <= kCtMaxDepth) ? walk_depth : 0;
    // (hist_configure granted the largest size: a depth-10 tree)
    const size_t sm3 = wtree ? gradients_b3_smem(max_nodes, ct) : 0;
    launch_pdl(k_gradients_b3, dim3(g3), dim3(kGradThreads), sm3, s, kind, margin, label, weight, spw, min_hess,
               n, vrows, gpair, scale, wtree, ls_last, max_nodes, ct, rec, mask_off >> 2, pending);
    return;
  }
  launch_pdl(k_gradients, dim3(grid), dim3(256), smem, s, kind, margin, label, weight, spw, min_hess, n, vrows, gpair, scale,
                                      wtree, ls_last, rec, stride, mask_off, blk, blk_pair, pending);
}

void launch_walk(const WNode* wtree, const LevelState* ls_last, int max_nodes, const uint8_t* rec,
                 uint32_t stride, uint32_t mask_off, uint32_t blk, uint64_t n, float* margin,
                 const int* pending, int n_sm, cudaStream_t s) {
  int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8);
  if (grid < 1) grid = 1;
  k_walk<<<grid, 256, sizeof(WNode) * (size_t)max_nodes, s>>>(wtree, ls_last, rec, stride, mask_off, blk,
                                                              n, margin, pending);
}

void hist_configure() {
  const char* np = std::getenv("HB_NO_PDL");
  g_pdl = !(np && np[0] == '1');
  cudaFuncSetAttribute(k_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 1024);
  cudaFuncSetAttribute(k_gradients_b3, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)gradients_b3_smem(2 << kCtMaxDepth, kCtMaxDepth));
  for (const void* f : h32_kernels())
    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 1024);
}

void launch_softmax_gradients(int K, float* margin, const float* label, uint64_t n, uint64_t vrows,
                              float min_hess, float2* gpair, Scale* scale, const WNode* wtree,
                              uint32_t wstride, const uint8_t* rec, uint32_t stride, uint32_t mask_off,
                              uint32_t blk, const int* pending, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8));
  if (K == 2) {
    launch_pdl(k_softmax_short<2>, dim3(grid), dim3(256), 0, s, margin, label, n, vrows, min_hess, gpair, scale,
               wtree, wstride, rec, stride, mask_off, blk, pending);
    return;
  }
  if (K == 4) {
    launch_pdl(k_softmax_short<4>, dim3(grid), dim3(256), 0, s, margin, label, n, vrows, min_hess, gpair, scale,
               wtree, wstride, rec, stride, mask_off, blk, pending);
    return;
  }
  launch_pdl(k_softmax_gradients, dim3(grid), dim3(256), 0, s, K, margin, label, n, min_hess, gpair, scale, wtree,
                                           wstride, rec, stride, mask_off, blk, pending);
}

void launch_walk_csr(const DevConst& c, int K, const WNode* wtree, uint32_t wstride, float* margin,
                     const int* pending, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((c.n_rows + 255) / 256, (uint64_t)n_sm * 8));
  if (c.csr_col)
    launch_pdl(k_walk_csr<true>, dim3(grid), dim3(256), 0, s, c, K, wtree, wstride, margin, pending);
  else
    launch_pdl(k_walk_csr<false>, dim3(grid), dim3(256), 0, s, c, K, wtree, wstride, margin, pending);
}

void launch_csr_columns(const DevConst& c, uint8_t* col, uint64_t* colmiss, int n_sm, cudaStream_t s) {
  if (!c.n_rows || !c.n_cols) return;
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((c.n_rows + 255) / 256, (uint64_t)n_sm * 8));
  k_csr_columns<<<grid, 256, 0, s>>>(c, col, reinterpret_cast<unsigned long long*>(colmiss));
}

void launch_walk_classes(int K, const WNode* wtree, uint32_t wstride, const uint8_t* rec,
                         uint32_t stride, uint32_t mask_off, uint32_t blk, uint64_t n, float* margin,
                         const int* pending, int n_sm, cudaStream_t s) {
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8));
  k_walk_classes<<<grid, 256, 0, s>>>(K, wtree, wstride, rec, stride, mask_off, blk, n, margin, pending);
}

void launch_pair_maxima(const float2* gpair, uint64_t n, Scale* scale, int n_sm, cudaStream_t s) {
  int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)n_sm * 8);
  if (grid < 1) grid = 1;
  k_pair_maxima<<<grid, 256, 0, s>>>(gpair, n, scale);
}

void launch_scale(Scale* scale, uint64_t global_rows, int* pending, cudaStream_t s) {
  launch_pdl(k_scale, dim3(1), dim3(1), 0, s, scale, global_rows, pending);
}

void launch_encode(const uint8_t* col, const uint64_t* colmiss, uint64_t n_rows, uint32_t n_cols,
                   uint32_t stride, uint32_t mask_off, uint32_t blk, uint8_t* rec, cudaStream_t s) {
  int grid = (int)std::min<uint64_t>((n_rows + 255) / 256, 4096);
  if (grid < 1) grid = 1;
  k_encode<<<grid, 256, 0, s>>>(col, colmiss, n_rows, n_cols, stride, mask_off, blk, rec);
}

// The split of the 32-bit kernel for `global_rows` rows: lo bits K and the
// rows between folds R (0: the 32-bit kernel does not apply). A value holds
// Q = kFixedTop - c bits (|q| <= 2^Q, c = ceil(log2 rows)); R = 2^r rows of
// lo parts (< 2^K each) stay below 2^32 and of hi parts (|hi| <= 2^(Q-K))
// within +-2^30.
static void split_for_rows(uint64_t global_rows, int& lo_bits, int& flush_rows) {
  int c = 0;
  while (c < 64 && (1ull << c) < global_rows) ++c;
  const int Q = kFixedTop - c;
  const int K = (Q + 3) / 2;
  const int r = std::min(32 - K, 30 - (Q - K));
  lo_bits = K;
  flush_rows = (r >= 10 && r < 31) ? (1 << r) : 0;  // at least two 512-row passes per fold
}

static bool use_hist32(const DevConst& c) {
  int K, R;
  split_for_rows(c.global_rows, K, R);
  return !c.hist64 && R > 0 && c.max_bins * 32 <= kNSlots;
}

// Feature groups per histogram CTA (k_hist32<G>).
static int hist_groups_per_cta(const DevConst& c) {
  return (c.max_bins <= 128 && c.n_groups >= 2) ? 2 : 1;
}

size_t hist_smem_bytes(const DevConst& c) {
  if (c.csr) return 0;
  if (use_hist32(c)) {
    return hist_groups_per_cta(c) == 2 ? H32<2>::smem() : H32<1>::smem();
  }
  return (size_t)c.max_bins * 32 * 16;
}

int hist_grid(int n_sm) { return n_sm; }

void launch_hist(const DevConst& c, const uint32_t* fo, const uint8_t* rec, const float2* gpair,
                 const Scale* scale, const uint32_t* rows, const HEntry* entries,
                 const LevelState* ls, longlong2* hist, long long* totals,
                 unsigned long long* row_stats, int grid_x, size_t smem, cudaStream_t s) {
  if (c.csr) {
    launch_pdl(k_hist_csr, dim3(grid_x * (2048 / kCsrThreads)), dim3(kCsrThreads), 0, s, c, gpair, scale, rows, entries, ls,
                                                                    hist, totals, row_stats);
    return;
  }
  // The dynamic shared memory this launch needs, granted per device (the
  // attribute is per device); the launch reports the error if it cannot be.
  static size_t granted[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || granted[dev] < smem) {
    if (cudaFuncSetAttribute(k_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
            cudaSuccess &&
        dev >= 0 && dev < 64)
      granted[dev] = smem;
  }
  dim3 grid(grid_x, c.n_groups);
  if (use_hist32(c)) {
    // every instantiation was granted its shared memory by hist_configure
    int G = hist_groups_per_cta(c);
    H32Fn f = h32_fn(G, c.blk, gpair == nullptr);
    if (!f) {
      G = 1;
      f = h32_fn(1, c.blk, gpair == nullptr);
    }
    int K, R;
    split_for_rows(c.global_rows, K, R);
    grid.y = (c.n_groups + G - 1) / G;
    launch_pdl(f, dim3(grid), dim3(kH32Threads), smem, s, c, fo, rec, gpair, scale, rows, entries, ls, hist, totals, row_stats,
                                      K, R);
    return;
  }
  launch_pdl(k_hist, dim3(grid), dim3(kHistThreads), smem, s, c, fo, rec, gpair, scale, rows, entries, ls, hist, totals,
                                          row_stats);
}

void launch_subtract(const Triple* pairs, const LevelState* ls, int max_pairs, uint32_t total_bins,
                     longlong2* hist, cudaStream_t s) {
  uint64_t work = (uint64_t)max_pairs * total_bins;
  int grid = (int)std::min<uint64_t>((work + 255) / 256, 148 * 16);
  if (grid < 1) grid = 1;
  k_subtract<<<grid, 256, 0, s>>>(pairs, ls, total_bins, hist);
}

void launch_scan(const DevConst& c, const uint32_t* fo, longlong2* hist, const Front* front,
                 const LevelState* ls, const Triple* pairs, int sib_base, const Scale* scale,
                 int max_front, Cand* cand, cudaStream_t s, const int8_t* dirs,
                 unsigned long long* best_key) {
  if (max_front < 1 || c.n_cols == 0) return;
  // features of <= 128 bins: a warp per (node, feature); wider: a CTA
  if (c.max_bins <= 128 && !c.scan_cta) {
    dim3 grid((c.n_cols + kScanWarps - 1) / kScanWarps, max_front);
    if (c.max_bins <= 32)
      launch_pdl(k_scan_w<1>, dim3(grid), dim3(kScanWarps * 32), 0, s, c, fo, hist, front, ls, pairs, sib_base, scale, cand, dirs, best_key);
    else if (c.max_bins <= 64)
      launch_pdl(k_scan_w<2>, dim3(grid), dim3(kScanWarps * 32), 0, s, c, fo, hist, front, ls, pairs, sib_base, scale, cand, dirs, best_key);
    else
      launch_pdl(k_scan_w<4>, dim3(grid), dim3(kScanWarps * 32), 0, s, c, fo, hist, front, ls, pairs, sib_base, scale, cand, dirs, best_key);
    return;
  }
  dim3 grid(c.n_cols, max_front);
  if (c.max_bins > (uint32_t)kSplitThreads) {
    launch_pdl(k_scan_wide, dim3(grid), dim3(kSplitThreads), 0, s, c, fo, hist, front, ls, pairs, sib_base, scale, cand, dirs, best_key);
    return;
  }
  launch_pdl(k_scan, dim3(grid), dim3(kSplitThreads), 0, s, c, fo, hist, front, ls, pairs, sib_base, scale, cand, dirs, best_key);
}

void launch_apply(const DevConst& c, const uint32_t* fo, const float* cuts, const Cand* cand,
                  const Front* front, Front* next, Decision* dec, PItem* items, LevelState* ls,
                  LevelState* ls_next, hb_tree_node* tree, WNode* wtree, const Scale* scale,
                  int depth, int leaf_only, unsigned long long* best_key, cudaStream_t s) {
  // the frontier at `depth` has at most 2^depth nodes
  if (depth <= 8)
    launch_pdl(k_apply<256>, dim3(1), dim3(256), 0, s, c, fo, cuts, cand, front, next, dec, items, ls, ls_next,
               tree, wtree, scale, depth, leaf_only, best_key);
  else
    launch_pdl(k_apply<kApplyThreads>, dim3(1), dim3(kApplyThreads), 0, s, c, fo, cuts, cand, front, next, dec,
               items, ls, ls_next, tree, wtree, scale, depth, leaf_only, best_key);
}

void launch_part_count(const DevConst& c, const uint8_t* col, const uint64_t* colmiss,
                       const uint8_t* rec, int use_record, const uint32_t* rows_in, int identity,
                       const Front* front, const Decision* dec, const PItem* items,
                       const LevelState* ls, int max_items, uint32_t* dirbits, uint32_t* item_left,
                       cudaStream_t s, uint32_t* rows_copy) {
  if (c.csr && !col)  // a CSR index held feature-major reads its columns like a dense one
    launch_pdl(k_part_count<true>, dim3(max_items), dim3(kPartThreads), 0, s, c, col, colmiss, rec, use_record, rows_in, identity,
                                                        front, dec, items, ls, dirbits, item_left, rows_copy);
  else
    launch_pdl(k_part_count<false>, dim3(max_items), dim3(kPartThreads), 0, s, c, col, colmiss, rec, use_record, rows_in, identity,
                                                         front, dec, items, ls, dirbits, item_left, rows_copy);
}

void launch_part_onepass(const DevConst& c, const uint8_t* col, const uint64_t* colmiss,
                         const uint32_t* rows_in, int identity, const Front* front, const Decision* dec,
                         const LevelState* ls, int max_items, uint32_t* fill, uint32_t* rows_out,
                         uint32_t half, cudaStream_t s) {
  if (c.csr && !col)
    launch_pdl(k_part_onepass<true>, dim3(max_items), dim3(kPartThreads), 0, s, c, col, colmiss, rows_in,
               identity, front, dec, ls, fill, rows_out, half);
  else
    launch_pdl(k_part_onepass<false>, dim3(max_items), dim3(kPartThreads), 0, s, c, col, colmiss, rows_in,
               identity, front, dec, ls, fill, rows_out, half);
}

void launch_part_plan(const Front* front, const Decision* dec, const LevelState* ls, uint32_t* fill,
                      Front* next, HEntry* entries, Triple* pairs, LevelState* ls_next, int max_front,
                      uint32_t half, cudaStream_t s) {
  if (max_front <= 256)
    launch_pdl(k_part_plan<256>, dim3(1), dim3(256), 0, s, front, dec, ls, fill, next, entries, pairs, ls_next,
               half);
  else
    launch_pdl(k_part_plan<kApplyThreads>, dim3(1), dim3(kApplyThreads), 0, s, front, dec, ls, fill, next, entries,
               pairs, ls_next, half);
}

void launch_part_scan(const Front* front, const Decision* dec, LevelState* ls, int max_front,
                      const uint32_t* item_left, uint32_t* item_left_off, Front* next,
                      HEntry* entries, Triple* pairs, LevelState* ls_next, cudaStream_t s) {
  launch_pdl(k_part_scan, dim3(max_front), dim3(kScanThreads), 0, s, front, dec, ls, item_left, item_left_off, next,
                                                 entries, pairs, ls_next);
}

void launch_part_scatter(const Front* front, const Decision* dec, const PItem* items,
                         const LevelState* ls, int max_items, const uint32_t* dirbits,
                         const uint32_t* item_left_off, const Front* next,
                         const uint32_t* rows_in, int identity, uint32_t* rows_out,
                         cudaStream_t s) {
  launch_pdl(k_part_scatter, dim3(max_items), dim3(kPartThreads), 0, s, front, dec, items, ls, dirbits, item_left_off,
                                                    next, rows_in, identity, rows_out);
}


void launch_lg_step(const DevConst& c, const uint32_t* fo, const float* cuts, const Cand* cand,
                    const Front* pend, Front* front, Front* next, Decision* dec, LevelState* ls,
                    LevelState* ls_next, hb_tree_node* tree, WNode* wtree, const Scale* scale,
                    LgKey* heap, LgNode* pool, int heap_cap, LgState* st, int32_t* ndepth,
                    int max_leaves, int depth_limit, int final_step, unsigned long long* best_key,
                    cudaStream_t s) {
  const size_t smem = sizeof(LgKey) * (size_t)heap_cap;
  static size_t granted[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && (dev < 0 || dev >= 64 || granted[dev] < smem)) {
    if (cudaFuncSetAttribute(k_lg_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
            cudaSuccess &&
        dev >= 0 && dev < 64)
      granted[dev] = smem;
  }
  launch_pdl(k_lg_step, dim3(1), dim3(kLgThreads), smem, s, c, fo, cuts, cand, pend, front, next, dec, ls, ls_next, tree,
                                        wtree, scale, heap, pool, st, ndepth, max_leaves, depth_limit,
                                        final_step, best_key);
}

void launch_lg_setup(LgState* st, int32_t* ndepth, hb_tree_node* tree, const Front* root,
                     const Scale* scale, LevelState* ls_next, cudaStream_t s) {
  launch_pdl(k_lg_setup, dim3(1), dim3(1), 0, s, st, ndepth, tree, root, scale, ls_next);
}


void launch_root_setup(uint64_t n_rows, Front* front, HEntry* entries, LevelState* ls,
                       cudaStream_t s) {
  launch_pdl(k_root_setup, dim3(1), dim3(1), 0, s, n_rows, front, entries, ls);
}

void launch_root_stats(Front* front, const long long* totals, cudaStream_t s) {
  launch_pdl(k_root_stats, dim3(1), dim3(1), 0, s, front, totals);
}

void launch_finish_tree(const hb_tree_node* tree, const LevelState* ls_last, hb_tree_node* forest,
                        uint32_t* counts, int32_t* tree_counter, uint32_t max_nodes,
                        cudaStream_t s) {
  launch_pdl(k_finish_tree, dim3(1), dim3(256), 0, s, tree, ls_last, forest, counts, tree_counter, max_nodes);
}

void launch_dequantize(const longlong2* hist, uint32_t n, const Scale* scale, double* out,
                       cudaStream_t s) {
  int grid = (int)std::min<uint32_t>((n + 255) / 256, 1024u);
  if (grid < 1) grid = 1;
  k_dequantize<<<grid, 256, 0, s>>>(hist, n, scale, out);
}

void launch_add_segment(const uint32_t* rows, uint32_t begin, uint32_t len, float value,
                        float* margin, cudaStream_t s) {
  int grid = (int)std::min<uint32_t>((len + 255) / 256, 2048u);
  if (grid < 1) grid = 1;
  k_add_segment<<<grid, 256, 0, s>>>(rows, begin, len, value, margin);
}

}  // namespace hb
