// Tree-ensemble batch prediction (BoostedModel::predict_margin,
// src/model/predict.rs:701, and the GPU model of src/backend/cuda/predict.rs).
//
// margin[row][out] = base[out] + sum over trees t in order of
// weight[t] * leaf_t(row), each term added in f32 to output tree_output[t].
// A node sends a row left when x[feature] < split_cond, and a missing (NaN)
// value the node's default direction (src/tree/regtree.rs:39).
#include <cuda_pipeline.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "hb_internal.h"

namespace {

// 16-byte node: a leaf stores its weighted value and marks itself with
// child = -1.
struct PNode {
  int32_t feature;   // bit 31: default_left
  float cond;        // threshold, or the leaf's value for a leaf
  int32_t left;      // absolute index of the left child (right = left + 1), -1 = leaf
  int32_t pad;
};

__global__ void k_predict(const PNode* __restrict__ nodes, const uint32_t* __restrict__ roots,
                          const uint32_t* __restrict__ order, const uint32_t* __restrict__ ostart,
                          const float* __restrict__ weights, int n_outputs,
                          const float* __restrict__ base, const float* __restrict__ x,
                          uint64_t n_rows, uint32_t n_cols, float* __restrict__ out) {
  // one output at a time over its trees in tree order (order[ostart[o] ..
  // ostart[o + 1]) lists them), so each output's sum is the reference's
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const float* row = x + r * n_cols;
    for (int o = 0; o < n_outputs; ++o) {
      float acc = base[o];
      for (uint32_t q = ostart[o]; q < ostart[o + 1]; ++q) {
        const uint32_t t = order[q];
        uint32_t id = roots[t];
        PNode nd = nodes[id];
        while (nd.left >= 0) {
          const int f = nd.feature & 0x7fffffff;
          const float v = __ldg(row + f);
          const bool left = isnan(v) ? (nd.feature < 0) : (v < nd.cond);
          id = (uint32_t)nd.left + (left ? 0u : 1u);
          nd = nodes[id];
        }
        acc = __fadd_rn(acc, __fmul_rn(weights[t], nd.cond));
      }
      out[r * n_outputs + o] = acc;
    }
  }
}

// ---- complete-tree path --------------------------------------------------
// A single-output forest whose trees are at most kCompleteMaxDepth deep is
// also laid out as complete trees: a tree of depth d becomes 2^d - 1
// internal nodes (CNode) in breadth-first order, children of i at 2i + 1 and
// 2i + 2, followed by its 2^d leaf values. A leaf shallower than d fills its
// whole subtree below: the padded internal nodes route anywhere and every
// leaf under them is that leaf, so each row reaches the same value. The
// walk is then d steps with no child pointers and no leaf test.
//
// k_predict_chunked keeps a tile of rows in shared memory (feature-major,
// stride tile, a multiple of 32: thread t reads its row's values from bank
// t % 32 whatever feature each lane's node asks for, so the walk's feature
// reads never conflict; only the tile's staging writes do) and
// streams the forest through two shared buffers of kChunkBytes with
// cp.async, the next chunk loading while the current one is walked. The
// margin is summed in tree order with the same f32 operations as k_predict.
constexpr int kCompleteMaxDepth = 10;
constexpr int kPredThreads = 512;
constexpr int kChunkBytes = 48 * 1024;
constexpr int kPredSmemBudget = 224 * 1024;

struct CNode {
  float cond;
  uint32_t meta;  // feature * tile: its row in the shared tile | default_left << 31
};
struct TreeHdr {
  uint32_t off;    // byte offset of the tree in its chunk
  uint32_t depth;
  uint32_t pad;
  float weight;
};
struct ChunkHdr {
  uint32_t off;    // byte offset of the chunk in the arena
  uint32_t bytes;  // a multiple of 16
  uint32_t t0, t1; // its trees
};

// One step of a complete-tree walk: left iff v < cond; a missing value
// follows default_left.
__device__ __forceinline__ uint32_t walk_step(const CNode q, const float* xr, uint32_t idx) {
  const float v = xr[q.meta & 0x7fffffffu];
  const bool right = (v != v) ? (q.meta >> 31) == 0u : !(v < q.cond);
  return 2u * idx + (right ? 2u : 1u);
}

__global__ void __launch_bounds__(kPredThreads, 1)
    k_predict_chunked(const unsigned char* __restrict__ arena, const ChunkHdr* __restrict__ chunks,
                      int n_chunks, const TreeHdr* __restrict__ trees, float base0,
                      const float* __restrict__ x, uint64_t n_rows, uint32_t n_cols, int tile,
                      uint32_t x_bytes, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char sm[];
  float* s_x = reinterpret_cast<float*>(sm);  // [n_cols][tile]
  unsigned char* const buf0 = sm + x_bytes;  // chunk c lives at buf0 + (c & 1) * kChunkBytes
  const int tid = threadIdx.x;
  const uint64_t n_tiles = (n_rows + tile - 1) / tile;
  for (uint64_t tl = blockIdx.x; tl < n_tiles; tl += gridDim.x) {
    const uint64_t r0 = tl * (uint64_t)tile;
    const uint64_t left = n_rows - r0;
    const int rows = left < (uint64_t)tile ? (int)left : tile;
    const float* xt = x + r0 * n_cols;
    const int nv = rows * (int)n_cols;
    for (int i = tid; i < nv; i += kPredThreads) {
      const int r = i / (int)n_cols, f = i - r * (int)n_cols;
      s_x[f * tile + r] = __ldg(xt + i);
    }
    auto issue = [&](int c) {
      const ChunkHdr ch = chunks[c];
      unsigned char* dst = buf0 + (c & 1) * kChunkBytes;
      for (uint32_t o = (uint32_t)tid * 16u; o < ch.bytes; o += kPredThreads * 16u)
        __pipeline_memcpy_async(dst + o, arena + ch.off + o, 16);
      __pipeline_commit();
    };
    issue(0);
    float acc = base0;
    const float* xr = s_x + tid;
    for (int c = 0; c < n_chunks; ++c) {
      if (c + 1 < n_chunks)
        issue(c + 1);
      else
        __pipeline_commit();  // an empty group keeps the wait count uniform
      __pipeline_wait_prior(1);
      __syncthreads();        // chunk c (and, at c = 0, the row tile) visible to all
      const ChunkHdr ch = chunks[c];
      if (tid < rows) {
        const unsigned char* cb = buf0 + (c & 1) * kChunkBytes;
        uint32_t t = ch.t0;
        // kLanes trees of one depth walked in lockstep: independent chains of
        // shared loads; their leaves still add in tree order
        constexpr int kLanes = 8;
        for (; t + kLanes <= ch.t1; t += kLanes) {
          TreeHdr h[kLanes];
          bool same = true;
#pragma unroll
          for (int j = 0; j < kLanes; ++j) {
            h[j] = trees[t + j];
            same = same && h[j].depth == h[0].depth;
          }
          if (!same) break;
          uint32_t ix[kLanes];
#pragma unroll
          for (int j = 0; j < kLanes; ++j) ix[j] = 0;
          for (uint32_t k = 0; k < h[0].depth; ++k) {
#pragma unroll
            for (int j = 0; j < kLanes; ++j)
              ix[j] = walk_step(reinterpret_cast<const CNode*>(cb + h[j].off)[ix[j]], xr, ix[j]);
          }
          const uint32_t internal = (1u << h[0].depth) - 1u;
#pragma unroll
          for (int j = 0; j < kLanes; ++j) {
            const CNode* nd = reinterpret_cast<const CNode*>(cb + h[j].off);
            acc = __fadd_rn(acc, __fmul_rn(h[j].weight, reinterpret_cast<const float*>(nd + internal)[ix[j] - internal]));
          }
        }
        for (; t < ch.t1; ++t) {
          const TreeHdr th = trees[t];
          const CNode* nd = reinterpret_cast<const CNode*>(cb + th.off);
          uint32_t idx = 0;
          for (uint32_t k = 0; k < th.depth; ++k) idx = walk_step(nd[idx], xr, idx);
          const uint32_t internal = (1u << th.depth) - 1u;
          const float leaf = reinterpret_cast<const float*>(nd + internal)[idx - internal];
          acc = __fadd_rn(acc, __fmul_rn(th.weight, leaf));
        }
      }
      __syncthreads();  // buffer c & 1 is free for chunk c + 2; the tile for the next one
    }
    if (tid < rows) out[r0 + tid] = acc;
  }
}

}  // namespace

struct hb_predictor {
  int device = 0;
  cudaStream_t stream = nullptr;
  PNode* nodes = nullptr;
  uint32_t* roots = nullptr;
  uint32_t* outs = nullptr;    // trees grouped by output, in tree order within an output
  uint32_t* ostart = nullptr;  // [n_outputs + 1] offsets into outs
  float* weights = nullptr;
  float* base = nullptr;
  uint32_t n_trees = 0;
  int n_outputs = 1;
  uint32_t n_features = 0;
  int n_sm = 148;
  // host-row prediction: two staging sets, block b on stream b & 1 (the
  // predictor's stream and a second one), so one block's copies overlap
  // the other's kernel
  cudaStream_t stream2 = nullptr;
  float* stage_x[2] = {nullptr, nullptr};
  float* stage_out[2] = {nullptr, nullptr};
  size_t stage_rows = 0;
  // the complete-tree layout (empty when the forest does not qualify)
  unsigned char* carena = nullptr;
  ChunkHdr* chunks = nullptr;
  TreeHdr* theads = nullptr;
  int n_chunks = 0;
  int tile = 0;
  uint32_t x_bytes = 0;
  size_t smem = 0;
  float base0 = 0.0f;
};

namespace {

// The complete-tree layout of a forest, or false when a tree is deeper than
// kCompleteMaxDepth, there is more than one output, or a row tile would not
// fit in shared memory.
bool build_complete(const hb_tree_node* nodes, const uint64_t* tree_ptr, uint64_t n_trees,
                    const float* ws, int n_outputs, uint32_t n_features, int& tile,
                    std::vector<unsigned char>& arena, std::vector<ChunkHdr>& chunks,
                    std::vector<TreeHdr>& heads) {
  if (n_outputs != 1 || n_features == 0 || n_trees == 0) return false;
  const int budget_rows = (kPredSmemBudget - 2 * kChunkBytes) / (4 * (int)n_features) - 1;
  tile = std::min(kPredThreads, budget_rows) & ~31;
  if (tile < 32) return false;
  heads.resize(n_trees);
  std::vector<int> depth_of;
  std::vector<std::pair<int32_t, int>> stack;
  ChunkHdr cur{0, 0, 0, 0};
  for (uint64_t t = 0; t < n_trees; ++t) {
    const hb_tree_node* tn = nodes + tree_ptr[t];
    const int64_t n = (int64_t)(tree_ptr[t + 1] - tree_ptr[t]);
    // depth of the tree (the trees were checked by the caller)
    int d = 0;
    stack.assign(1, {0, 0});
    while (!stack.empty()) {
      const auto [id, k] = stack.back();
      stack.pop_back();
      if (id < 0 || id >= n || k > kCompleteMaxDepth) return false;
      if (tn[id].left < 0) {
        d = std::max(d, k);
      } else {
        stack.push_back({tn[id].left, k + 1});
        stack.push_back({tn[id].right, k + 1});
      }
    }
    const uint32_t internal = (1u << d) - 1u, leaves = 1u << d;
    const uint32_t bytes = ((8u * internal + 4u * leaves) + 15u) & ~15u;
    std::vector<unsigned char> rec(bytes, 0);
    CNode* cn = reinterpret_cast<CNode*>(rec.data());
    float* lf = reinterpret_cast<float*>(rec.data() + 8u * internal);
    // fill position p (depth k) of the complete tree from node id
    struct Item { uint32_t p; int32_t id; int k; };
    std::vector<Item> work{{0u, 0, 0}};
    while (!work.empty()) {
      const Item it = work.back();
      work.pop_back();
      const hb_tree_node& s = tn[it.id];
      if (it.k == d) {
        lf[it.p - internal] = s.leaf_value;
        continue;
      }
      if (s.left < 0) {  // a shallow leaf: pad its subtree
        cn[it.p].cond = INFINITY;
        cn[it.p].meta = 0u;
        work.push_back({2 * it.p + 1, it.id, it.k + 1});
        work.push_back({2 * it.p + 2, it.id, it.k + 1});
      } else {
        cn[it.p].cond = s.split_cond;
        cn[it.p].meta = s.split_feature * (uint32_t)tile | (s.default_left ? 0x80000000u : 0u);
        work.push_back({2 * it.p + 1, s.left, it.k + 1});
        work.push_back({2 * it.p + 2, s.right, it.k + 1});
      }
    }
    if (cur.bytes + bytes > (uint32_t)kChunkBytes) {
      chunks.push_back(cur);
      cur = ChunkHdr{(uint32_t)arena.size(), 0, (uint32_t)t, (uint32_t)t};
    }
    heads[t] = TreeHdr{cur.bytes, (uint32_t)d, 0u, ws[t]};
    arena.insert(arena.end(), rec.begin(), rec.end());
    cur.bytes += bytes;
    cur.t1 = (uint32_t)t + 1;
  }
  chunks.push_back(cur);
  return true;
}

}  // namespace

extern "C" {

hb_status hb_predictor_create(int32_t device_ordinal, const hb_tree_node* nodes,
                              const uint64_t* tree_ptr, uint64_t n_trees,
                              const uint32_t* tree_output, const float* tree_weight,
                              int32_t n_outputs, const float* base, uint32_t n_features,
                              hb_predictor** out) {
  if (!out || !tree_ptr || !base || n_outputs < 1 || n_outputs > 4096 || (!nodes && n_trees))
    return HB_INVALID_ARGUMENT;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device_ordinal < 0 || device_ordinal >= ndev)
    return HB_REFUSED;
  if (cudaSetDevice(device_ordinal) != cudaSuccess) return HB_DEVICE_FAILED;
  // Re-lay the trees: children adjacent (left, left + 1), leaves carrying
  // their value; node ids become absolute arena indices.
  std::vector<PNode> arena;
  std::vector<uint32_t> roots(n_trees), outs(n_trees);
  std::vector<float> ws(n_trees);
  for (uint64_t t = 0; t < n_trees; ++t) {
    const hb_tree_node* tn = nodes + tree_ptr[t];
    const uint64_t n = tree_ptr[t + 1] - tree_ptr[t];
    if (n == 0) return HB_INVALID_ARGUMENT;
    roots[t] = (uint32_t)arena.size();
    outs[t] = tree_output ? tree_output[t] : (uint32_t)(t % (uint64_t)n_outputs);
    if (outs[t] >= (uint32_t)n_outputs) return HB_INVALID_ARGUMENT;
    ws[t] = tree_weight ? tree_weight[t] : 1.0f;
    // breadth-first: a node's children get consecutive slots
    std::vector<int32_t> order{0};
    std::vector<uint32_t> slot_of(n, 0);
    arena.push_back(PNode{});
    for (size_t q = 0; q < order.size(); ++q) {
      const int32_t id = order[q];
      if (id < 0 || (uint64_t)id >= n) return HB_INVALID_ARGUMENT;
      PNode pn{};
      const hb_tree_node& s = tn[id];
      if (s.left < 0) {
        pn.feature = 0;
        pn.cond = s.leaf_value;
        pn.left = -1;
      } else {
        if (s.split_feature >= n_features) return HB_INVALID_ARGUMENT;
        pn.feature = (int32_t)s.split_feature | (s.default_left ? (int32_t)0x80000000 : 0);
        pn.cond = s.split_cond;
        pn.left = (int32_t)arena.size();
        order.push_back(s.left);
        order.push_back(s.right);
        arena.push_back(PNode{});
        arena.push_back(PNode{});
      }
      arena[roots[t] + q] = pn;
      if (order.size() > n + 1) return HB_INVALID_ARGUMENT;
    }
  }
  // trees grouped by output, stable: output o's trees in tree order
  std::vector<uint32_t> ostart(n_outputs + 1, 0), grouped(n_trees);
  for (uint64_t t = 0; t < n_trees; ++t) ++ostart[outs[t] + 1];
  for (int o = 0; o < n_outputs; ++o) ostart[o + 1] += ostart[o];
  {
    std::vector<uint32_t> at(ostart.begin(), ostart.end() - 1);
    for (uint64_t t = 0; t < n_trees; ++t) grouped[at[outs[t]]++] = (uint32_t)t;
  }
  hb_predictor* p = new hb_predictor();
  p->device = device_ordinal;
  p->n_trees = (uint32_t)n_trees;
  p->n_outputs = n_outputs;
  p->n_features = n_features;
  cudaDeviceGetAttribute(&p->n_sm, cudaDevAttrMultiProcessorCount, device_ordinal);
  bool ok = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking) == cudaSuccess &&
            cudaMalloc(&p->nodes, sizeof(PNode) * std::max<size_t>(arena.size(), 1)) == cudaSuccess &&
            cudaMalloc(&p->roots, 4 * std::max<uint64_t>(n_trees, 1)) == cudaSuccess &&
            cudaMalloc(&p->outs, 4 * std::max<uint64_t>(n_trees, 1)) == cudaSuccess &&
            cudaMalloc(&p->ostart, 4 * (size_t)(n_outputs + 1)) == cudaSuccess &&
            cudaMalloc(&p->weights, 4 * std::max<uint64_t>(n_trees, 1)) == cudaSuccess &&
            cudaMalloc(&p->base, 4 * n_outputs) == cudaSuccess;
  if (ok && !arena.empty())
    ok = cudaMemcpy(p->nodes, arena.data(), sizeof(PNode) * arena.size(), cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && n_trees)
    ok = cudaMemcpy(p->roots, roots.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->outs, grouped.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->weights, ws.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok) ok = cudaMemcpy(p->base, base, 4 * n_outputs, cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemcpy(p->ostart, ostart.data(), 4 * (size_t)(n_outputs + 1), cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok) {
    std::vector<unsigned char> carena;
    std::vector<ChunkHdr> chunks;
    std::vector<TreeHdr> heads;
    int tile = 0;
    if (build_complete(nodes, tree_ptr, n_trees, ws.data(), n_outputs, n_features, tile, carena,
                       chunks, heads)) {
      p->tile = tile;
      p->n_chunks = (int)chunks.size();
      p->x_bytes = (uint32_t)((4ull * n_features * tile + 15) & ~15ull);
      p->smem = p->x_bytes + 2 * (size_t)kChunkBytes;
      p->base0 = base[0];
      ok = cudaMalloc(&p->carena, carena.size()) == cudaSuccess &&
           cudaMalloc(&p->chunks, sizeof(ChunkHdr) * chunks.size()) == cudaSuccess &&
           cudaMalloc(&p->theads, sizeof(TreeHdr) * heads.size()) == cudaSuccess &&
           cudaMemcpy(p->carena, carena.data(), carena.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaMemcpy(p->chunks, chunks.data(), sizeof(ChunkHdr) * chunks.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaMemcpy(p->theads, heads.data(), sizeof(TreeHdr) * heads.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaFuncSetAttribute(k_predict_chunked, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)p->smem) == cudaSuccess;
    }
  }
  if (!ok) {
    hb_predictor_destroy(p);
    return HB_DEVICE_FAILED;
  }
  *out = p;
  return HB_OK;
}

hb_status hb_predictor_destroy(hb_predictor* p) {
  if (!p) return HB_INVALID_ARGUMENT;
  cudaSetDevice(p->device);
  if (p->stream) cudaStreamSynchronize(p->stream);
  cudaFree(p->nodes);
  cudaFree(p->roots);
  cudaFree(p->outs);
  cudaFree(p->ostart);
  cudaFree(p->weights);
  cudaFree(p->base);
  if (p->stream2) cudaStreamSynchronize(p->stream2);
  for (int b = 0; b < 2; ++b) {
    cudaFree(p->stage_x[b]);
    cudaFree(p->stage_out[b]);
  }
  cudaFree(p->carena);
  cudaFree(p->chunks);
  cudaFree(p->theads);
  if (p->stream) cudaStreamDestroy(p->stream);
  if (p->stream2) cudaStreamDestroy(p->stream2);
  delete p;
  return HB_OK;
}

hb_status hb_predict_margin_device(hb_predictor* p, const float* d_rows, uint64_t n_rows,
                                   float* d_out, void* stream) {
  if (!p || (!d_rows && n_rows) || (!d_out && n_rows)) return HB_INVALID_ARGUMENT;
  if (cudaSetDevice(p->device) != cudaSuccess) return HB_DEVICE_FAILED;
  if (!n_rows) return HB_OK;
  cudaStream_t s = stream ? (cudaStream_t)stream : p->stream;
  if (p->n_chunks > 0) {
    const uint64_t tiles = (n_rows + p->tile - 1) / p->tile;
    const int grid = (int)std::min<uint64_t>(tiles, (uint64_t)p->n_sm);
    k_predict_chunked<<<grid, kPredThreads, p->smem, s>>>(p->carena, p->chunks, p->n_chunks,
                                                          p->theads, p->base0, d_rows, n_rows,
                                                          p->n_features, p->tile, p->x_bytes, d_out);
    return cudaGetLastError() == cudaSuccess ? HB_OK : HB_DEVICE_FAILED;
  }
  int grid = (int)std::min<uint64_t>((n_rows + 127) / 128, (uint64_t)p->n_sm * 16);
  k_predict<<<grid, 128, 0, s>>>(p->nodes, p->roots, p->outs, p->ostart, p->weights, p->n_outputs,
                                 p->base, d_rows, n_rows, p->n_features, d_out);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_DEVICE_FAILED;
}

// Host rows in, host margins out (GpuModel::predict_margin, :401): blocks of
// rows copied in, predicted and copied back, alternating between two
// streams and two staging sets so that a block's transfers overlap the
// neighbouring block's kernel (with pageable host memory the copies are
// staged by the driver and overlap less). Returns once every margin is back.
hb_status hb_predict_margin(hb_predictor* p, const float* rows, uint64_t n_rows, float* out) {
  if (!p || (!rows && n_rows) || (!out && n_rows)) return HB_INVALID_ARGUMENT;
  if (cudaSetDevice(p->device) != cudaSuccess) return HB_DEVICE_FAILED;
  const uint64_t block = 1ull << 21;
  const uint64_t want = std::min<uint64_t>(std::max<uint64_t>(n_rows, 1), block);
  if (!p->stream2 && cudaStreamCreateWithFlags(&p->stream2, cudaStreamNonBlocking) != cudaSuccess)
    return HB_DEVICE_FAILED;
  if (p->stage_rows < want) {
    for (int b = 0; b < 2; ++b) {
      cudaFree(p->stage_x[b]);
      cudaFree(p->stage_out[b]);
      p->stage_x[b] = p->stage_out[b] = nullptr;
    }
    p->stage_rows = 0;
    for (int b = 0; b < 2; ++b)
      if (cudaMalloc(&p->stage_x[b], 4 * want * p->n_features) != cudaSuccess ||
          cudaMalloc(&p->stage_out[b], 4 * want * p->n_outputs) != cudaSuccess)
        return HB_DEVICE_FAILED;
    p->stage_rows = want;
  }
  uint64_t k = 0;
  for (uint64_t at = 0; at < n_rows; at += block, ++k) {
    const int b = (int)(k & 1);
    cudaStream_t s = b ? p->stream2 : p->stream;
    const uint64_t m = std::min(block, n_rows - at);
    if (cudaMemcpyAsync(p->stage_x[b], rows + at * p->n_features, 4 * m * p->n_features,
                        cudaMemcpyHostToDevice, s) != cudaSuccess)
      return HB_DEVICE_FAILED;
    hb_status st = hb_predict_margin_device(p, p->stage_x[b], m, p->stage_out[b], s);
    if (st != HB_OK) return st;
    if (cudaMemcpyAsync(out + at * p->n_outputs, p->stage_out[b], 4 * m * p->n_outputs,
                        cudaMemcpyDeviceToHost, s) != cudaSuccess)
      return HB_DEVICE_FAILED;
  }
  const bool ok = cudaStreamSynchronize(p->stream) == cudaSuccess &&
                  cudaStreamSynchronize(p->stream2) == cudaSuccess;
  return ok ? HB_OK : HB_DEVICE_FAILED;
}

}  // extern "C"
