// Tree-ensemble batch prediction (BoostedModel::predict_margin,
// src/model/predict.rs:701, and the GPU model of src/backend/cuda/predict.rs).
//
// margin[row][out] = base[out] + sum over trees t in order of
// weight[t] * leaf_t(row), each term added in f32 to output tree_output[t].
// A node sends a row left when x[feature] < split_cond, and a missing (NaN)
// value the node's default direction (src/tree/regtree.rs:39).
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
                          const uint32_t* __restrict__ outs, const float* __restrict__ weights,
                          uint32_t n_trees, int n_outputs, const float* __restrict__ base,
                          const float* __restrict__ x, uint64_t n_rows, uint32_t n_cols,
                          float* __restrict__ out) {
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const float* row = x + r * n_cols;
    float acc[8];
    for (int o = 0; o < n_outputs && o < 8; ++o) acc[o] = base[o];
    for (uint32_t t = 0; t < n_trees; ++t) {
      uint32_t id = roots[t];
      PNode nd = nodes[id];
      while (nd.left >= 0) {
        const int f = nd.feature & 0x7fffffff;
        const float v = __ldg(row + f);
        const bool left = isnan(v) ? (nd.feature < 0) : (v < nd.cond);
        id = (uint32_t)nd.left + (left ? 0u : 1u);
        nd = nodes[id];
      }
      const uint32_t o = outs[t];
      acc[o] = __fadd_rn(acc[o], __fmul_rn(weights[t], nd.cond));
    }
    for (int o = 0; o < n_outputs && o < 8; ++o) out[r * n_outputs + o] = acc[o];
  }
}

}  // namespace

struct hb_predictor {
  int device = 0;
  cudaStream_t stream = nullptr;
  PNode* nodes = nullptr;
  uint32_t* roots = nullptr;
  uint32_t* outs = nullptr;
  float* weights = nullptr;
  float* base = nullptr;
  uint32_t n_trees = 0;
  int n_outputs = 1;
  uint32_t n_features = 0;
  int n_sm = 148;
  float* stage_x = nullptr;
  float* stage_out = nullptr;
  size_t stage_rows = 0;
};

extern "C" {

hb_status hb_predictor_create(int32_t device_ordinal, const hb_tree_node* nodes,
                              const uint64_t* tree_ptr, uint64_t n_trees,
                              const uint32_t* tree_output, const float* tree_weight,
                              int32_t n_outputs, const float* base, uint32_t n_features,
                              hb_predictor** out) {
  if (!out || !tree_ptr || !base || n_outputs < 1 || n_outputs > 8 || (!nodes && n_trees))
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
            cudaMalloc(&p->weights, 4 * std::max<uint64_t>(n_trees, 1)) == cudaSuccess &&
            cudaMalloc(&p->base, 4 * n_outputs) == cudaSuccess;
  if (ok && !arena.empty())
    ok = cudaMemcpy(p->nodes, arena.data(), sizeof(PNode) * arena.size(), cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && n_trees)
    ok = cudaMemcpy(p->roots, roots.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->outs, outs.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->weights, ws.data(), 4 * n_trees, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok) ok = cudaMemcpy(p->base, base, 4 * n_outputs, cudaMemcpyHostToDevice) == cudaSuccess;
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
  cudaFree(p->weights);
  cudaFree(p->base);
  cudaFree(p->stage_x);
  cudaFree(p->stage_out);
  if (p->stream) cudaStreamDestroy(p->stream);
  delete p;
  return HB_OK;
}

hb_status hb_predict_margin_device(hb_predictor* p, const float* d_rows, uint64_t n_rows,
                                   float* d_out, void* stream) {
  if (!p || (!d_rows && n_rows) || (!d_out && n_rows)) return HB_INVALID_ARGUMENT;
  if (cudaSetDevice(p->device) != cudaSuccess) return HB_DEVICE_FAILED;
  if (!n_rows) return HB_OK;
  cudaStream_t s = stream ? (cudaStream_t)stream : p->stream;
  int grid = (int)std::min<uint64_t>((n_rows + 127) / 128, (uint64_t)p->n_sm * 16);
  k_predict<<<grid, 128, 0, s>>>(p->nodes, p->roots, p->outs, p->weights, p->n_trees, p->n_outputs,
                                 p->base, d_rows, n_rows, p->n_features, d_out);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_DEVICE_FAILED;
}

// Host rows in, host margins out: blocks of rows copied in, predicted and
// copied back on the predictor's stream (GpuModel::predict_margin, :401).
hb_status hb_predict_margin(hb_predictor* p, const float* rows, uint64_t n_rows, float* out) {
  if (!p || (!rows && n_rows) || (!out && n_rows)) return HB_INVALID_ARGUMENT;
  if (cudaSetDevice(p->device) != cudaSuccess) return HB_DEVICE_FAILED;
  const uint64_t block = 1ull << 22;
  const uint64_t want = std::min<uint64_t>(std::max<uint64_t>(n_rows, 1), block);
  if (p->stage_rows < want) {
    cudaFree(p->stage_x);
    cudaFree(p->stage_out);
    p->stage_x = p->stage_out = nullptr;
    if (cudaMalloc(&p->stage_x, 4 * want * p->n_features) != cudaSuccess ||
        cudaMalloc(&p->stage_out, 4 * want * p->n_outputs) != cudaSuccess)
      return HB_DEVICE_FAILED;
    p->stage_rows = want;
  }
  for (uint64_t at = 0; at < n_rows; at += block) {
    const uint64_t m = std::min(block, n_rows - at);
    if (cudaMemcpyAsync(p->stage_x, rows + at * p->n_features, 4 * m * p->n_features,
                        cudaMemcpyHostToDevice, p->stream) != cudaSuccess)
      return HB_DEVICE_FAILED;
    hb_status st = hb_predict_margin_device(p, p->stage_x, m, p->stage_out, p->stream);
    if (st != HB_OK) return st;
    if (cudaMemcpyAsync(out + at * p->n_outputs, p->stage_out, 4 * m * p->n_outputs,
                        cudaMemcpyDeviceToHost, p->stream) != cudaSuccess)
      return HB_DEVICE_FAILED;
  }
  return cudaStreamSynchronize(p->stream) == cudaSuccess ? HB_OK : HB_DEVICE_FAILED;
}

}  // extern "C"
