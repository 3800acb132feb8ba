// hb_probe_smem: the shared-memory throughput the histogram kernels are bound
// by, measured on this GPU. Each kind is one shared-memory operation pattern
// of a histogram update, issued by every warp of one CTA per SM for `iters`
// iterations; the kernel counts SM clock cycles (clock64) around the loop,
// so the result is lane operations per SM clock, independent of the clock
// rate the GPU runs at.
//
// Kinds (all addresses inside the CTA's own 64 KiB of shared memory):
//   0  red.shared.add.u32, lane l at word l of a 32-word row (one bank each)
//   1  red.shared.add.u64, lane l at double-word l (two wavefronts a warp)
//   2  atom.shared.add.u32 whose result feeds the next address (latency)
//   3  ld.shared.u32 + add + st.shared.u32 (a non-atomic update)
//   4  the 32-bit histogram update: four red.shared.add.u32 per lane at one
//      random row of 256 and the lane's diagonal column (the k_hist32 loop)
//   5  the 64-bit histogram update: two red.shared.add.u64 (g, h) per lane at
//      one random row of 128 and the lane's diagonal column
//   6  red.shared.add.u32 with every lane of a warp on one word (a 32-way
//      conflict: the serialised worst case)
// A lane operation is one lane's access of one instruction; kind 4 counts
// four and kind 5 two per update.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "../../include/hb_backend.h"

namespace {

constexpr int kWords = 16384;  // 64 KiB of u32

__device__ __forceinline__ uint32_t lcg(uint32_t x) { return x * 1664525u + 1013904223u; }

template <int K>
__global__ void k_probe(int iters, unsigned long long* cycles, uint32_t* sink) {
  extern __shared__ __align__(16) uint32_t sm[];
  for (int i = threadIdx.x; i < kWords; i += blockDim.x) sm[i] = 0u;
  __syncthreads();
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(sm);
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  uint32_t r = 0x9e3779b9u * (threadIdx.x + 1u) + blockIdx.x;
  uint32_t acc = 0;
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    if (K == 0) {
      const uint32_t ad = base + 4u * (((warp + (uint32_t)it) & 127u) * 32u + lane);
      asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(ad), "r"(1u) : "memory");
    } else if (K == 1) {
      const uint32_t ad = base + 8u * (((warp + (uint32_t)it) & 63u) * 32u + lane);
      asm volatile("red.shared.add.u64 [%0], %1;" ::"r"(ad), "l"(1ull) : "memory");
    } else if (K == 2) {
      const uint32_t ad = base + 4u * (((acc + warp + (uint32_t)it) & 127u) * 32u + lane);
      uint32_t old;
      asm volatile("atom.shared.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(ad), "r"(1u) : "memory");
      acc += old & 1u;
    } else if (K == 3) {
      const uint32_t ad = base + 4u * (((warp + (uint32_t)it) & 127u) * 32u + lane);
      uint32_t v;
      asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(ad) : "memory");
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(ad), "r"(v + 1u) : "memory");
    } else if (K == 4) {
      r = lcg(r);
      const uint32_t row = r >> 24;  // 0..255
      const uint32_t ad = base + row * 128u + 4u * ((lane + (uint32_t)it) & 31u);
      // the four accumulator arrays 8 KiB apart (they overlap in this
      // 64 KiB buffer, which changes neither the banks nor the wavefronts)
      asm volatile(
          "red.shared.add.u32 [%0], %1;\n\t"
          "red.shared.add.u32 [%0+8192], %1;\n\t"
          "red.shared.add.u32 [%0+16384], %1;\n\t"
          "red.shared.add.u32 [%0+24576], %1;" ::"r"(ad),
          "r"(r & 0xffu)
          : "memory");
    } else if (K == 5) {
      r = lcg(r);
      const uint32_t row = r >> 25;  // 0..127
      const uint32_t ad = base + row * 256u + 8u * ((lane + (uint32_t)it) & 31u);
      asm volatile(
          "red.shared.add.u64 [%0], %1;\n\t"
          "red.shared.add.u64 [%0+32768], %1;" ::"r"(ad),
          "l"((unsigned long long)(r & 0xffu))
          : "memory");
    } else {
      const uint32_t ad = base + 4u * ((warp + (uint32_t)it) & 127u) * 32u;
      asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(ad), "r"(1u) : "memory");
    }
  }
  __syncthreads();
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
  if (acc == 0xffffffffu) sink[0] = sm[threadIdx.x];
}

template <int K>
cudaError_t run(int grid, int threads, int iters, unsigned long long* cyc, uint32_t* sink, cudaStream_t s) {
  const size_t smem = kWords * sizeof(uint32_t);
  cudaError_t rc = cudaFuncSetAttribute(k_probe<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (rc != cudaSuccess) return rc;
  k_probe<K><<<grid, threads, smem, s>>>(iters, cyc, sink);
  return cudaGetLastError();
}

}  // namespace

extern "C" hb_status hb_probe_smem(int32_t device, int32_t kind, int32_t threads, int32_t iters,
                                   double* lane_ops_per_clk) {
  if (!lane_ops_per_clk || kind < 0 || kind > 6 || threads < 32 || threads > 1024 || threads % 32 ||
      iters < 1 || iters > (1 << 24))
    return HB_INVALID_ARGUMENT;
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev) {
    cudaGetLastError();
    return HB_REFUSED;
  }
  if (cudaSetDevice(device) != cudaSuccess) return HB_DEVICE_FAILED;
  int n_sm = 0;
  if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return HB_DEVICE_FAILED;
  unsigned long long* cyc = nullptr;
  uint32_t* sink = nullptr;
  if (cudaMalloc(&cyc, sizeof(unsigned long long) * n_sm) != cudaSuccess) return HB_DEVICE_FAILED;
  if (cudaMalloc(&sink, sizeof(uint32_t)) != cudaSuccess) {
    cudaFree(cyc);
    return HB_DEVICE_FAILED;
  }
  cudaError_t rc = cudaSuccess;
  for (int pass = 0; pass < 2 && rc == cudaSuccess; ++pass) {  // the first pass warms up
    switch (kind) {
      case 0: rc = run<0>(n_sm, threads, iters, cyc, sink, 0); break;
      case 1: rc = run<1>(n_sm, threads, iters, cyc, sink, 0); break;
      case 2: rc = run<2>(n_sm, threads, iters, cyc, sink, 0); break;
      case 3: rc = run<3>(n_sm, threads, iters, cyc, sink, 0); break;
      case 4: rc = run<4>(n_sm, threads, iters, cyc, sink, 0); break;
      case 5: rc = run<5>(n_sm, threads, iters, cyc, sink, 0); break;
      default: rc = run<6>(n_sm, threads, iters, cyc, sink, 0); break;
    }
    if (rc == cudaSuccess) rc = cudaDeviceSynchronize();
  }
  std::vector<unsigned long long> h(n_sm);
  if (rc == cudaSuccess)
    rc = cudaMemcpy(h.data(), cyc, sizeof(unsigned long long) * n_sm, cudaMemcpyDeviceToHost);
  cudaFree(cyc);
  cudaFree(sink);
  if (rc != cudaSuccess) return HB_DEVICE_FAILED;
  const unsigned long long worst = *std::max_element(h.begin(), h.end());
  const double ops_per_update = kind == 4 ? 4.0 : kind == 5 ? 2.0 : 1.0;
  *lane_ops_per_clk = worst ? (double)threads * iters * ops_per_update / (double)worst : 0.0;
  return HB_OK;
}
