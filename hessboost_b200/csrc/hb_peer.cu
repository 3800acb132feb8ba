// Level histogram allreduce over NVLink peer memory (the multi-GPU exchange
// step of the hist path: after each rank builds its local int64 histograms
// of a level's built children, every rank needs their sum over ranks;
// hist/mod.rs builds one histogram per node, the row-sharded trainer sums
// the shards' exact integer histograms).
//
// Every rank's histogram buffer and barrier block are mapped into every
// other rank's address space (CUDA IPC, set up by the engine). One launch
// per level:
//   1. arrive: this rank's histograms are complete (the launch follows the
//      histogram kernel on the stream); its CTA 0 raises its flag in every
//      peer's `arrive` array, and every CTA waits until all peers' flags
//      reach this launch's epoch;
//   2. reduce: rank r owns the r-th 1/N of the words; each thread loads its
//      words from all N ranks (N independent 16-byte loads), adds them
//      (int64, so the order of ranks does not matter) and stores the sum
//      into all N ranks' buffers;
//   3. depart: the last CTA to finish raises this rank's flag in every
//      peer's `depart` array and waits for all peers', so when the launch
//      completes every rank's buffer holds the full sums.
// Plain peer loads and stores only (no multicast, no TMA). Every wait is
// bounded by `timeout_ns` of the global timer; on expiry the kernel sets
// the sticky status word, stops waiting and returns, and the engine
// reports the failure when it next reads the status.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "hb_internal.h"
#include "hb_kernels.cuh"

namespace hb {
namespace {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait until bar[slot * kPeerMax + j] >= epoch for every rank j != self.
// Returns false (and raises the status word) when the time runs out.
__device__ bool wait_all(const PeerSet& ps, int slot, unsigned long long epoch, uint64_t t0) {
  unsigned long long* mine = ps.bar[ps.rank];
  for (int j = 0; j < ps.n; ++j) {
    if (j == ps.rank) continue;
    const unsigned long long* f = mine + (size_t)slot * kPeerMax + j;
    while (ld_acquire_sys(f) < epoch) {
      if (ld_acquire_sys(mine + kPeerStatus) != 0) return false;
      if (global_ns() - t0 > ps.timeout_ns) {
        atomicExch(mine + kPeerStatus, 1ull);
        return false;
      }
      __nanosleep(32);
    }
  }
  return true;
}

// Raise this rank's flag `slot` to `epoch` in every peer's barrier block.
__device__ void signal_all(const PeerSet& ps, int slot, unsigned long long epoch) {
  __threadfence_system();
  for (int j = 0; j < ps.n; ++j) {
    if (j == ps.rank) continue;
    st_release_sys(ps.bar[j] + (size_t)slot * kPeerMax + ps.rank, epoch);
  }
}

// N ranks (a compile-time count, so each thread keeps U units' loads from
// every rank in flight at once: remote loads cost a round trip over NVLink).
template <int N>
__global__ void __launch_bounds__(kPeerThreads)
    k_peer_allreduce(PeerSet ps, uint64_t first, uint64_t count) {
  constexpr int U = N <= 2 ? 4 : N <= 4 ? 2 : 1;
  pdl_wait();
  unsigned long long* mine = ps.bar[ps.rank];
  __shared__ int s_ok;
  __shared__ unsigned long long s_epoch;
  const uint64_t t0 = global_ns();
  if (threadIdx.x == 0) {
    // every CTA reads the epoch before the last one advances it
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(mine + kPeerEpoch) + 1;
    s_epoch = e;
    int ok = ld_acquire_sys(mine + kPeerStatus) == 0;
    if (ok && blockIdx.x == 0) signal_all(ps, kPeerArrive, e);
    if (ok) ok = wait_all(ps, kPeerArrive, e, t0);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  __threadfence_system();  // this thread's peer loads after the arrive flags
  const unsigned long long epoch = s_epoch;

  // this rank's share of the words, split over the CTAs
  const uint64_t lo = first + count * (uint64_t)ps.rank / (uint64_t)N;
  const uint64_t hi = first + count * (uint64_t)(ps.rank + 1) / (uint64_t)N;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t u0 = lo + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; u0 < hi; u0 += U * stride) {
    longlong2 v[U][N];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint64_t u = u0 + k * stride;
#pragma unroll
      for (int j = 0; j < N; ++j) v[k][j] = u < hi ? ps.hist[j][u] : make_longlong2(0, 0);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint64_t u = u0 + k * stride;
      if (u >= hi) break;
      long long sx = 0, sy = 0;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        sx += v[k][j].x;
        sy += v[k][j].y;
      }
      const longlong2 sum = make_longlong2(sx, sy);
#pragma unroll
      for (int j = 0; j < N; ++j) ps.hist[j][u] = sum;
    }
  }

  // depart: the last CTA of this rank waits for every peer's last CTA
  __threadfence_system();  // this thread's peer stores before the CTA's count
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long done = atomicAdd(mine + kPeerCount, 1ull) + 1;
    if (done == gridDim.x) {
      signal_all(ps, kPeerDepart, epoch);
      wait_all(ps, kPeerDepart, epoch, t0);
      mine[kPeerCount] = 0ull;
      *reinterpret_cast<volatile unsigned long long*>(mine + kPeerEpoch) = epoch;
      __threadfence();
    }
  }
}

// A self-test of the bounded wait: one CTA waits on a flag that nothing
// raises (a peer set of two ranks whose "peer" block is `bar` itself) and
// must give up after timeout_ns with the status word set.
__global__ void k_peer_wait_probe(PeerSet ps) {
  if (threadIdx.x == 0) wait_all(ps, kPeerArrive, ~0ull, global_ns());
}

}  // namespace

void launch_peer_allreduce(const PeerSet& ps, uint64_t first, uint64_t count, int n_sm, cudaStream_t s) {
  const uint64_t share = (count + ps.n - 1) / ps.n;
  int grid = (int)std::min<uint64_t>((share + kPeerThreads - 1) / kPeerThreads, (uint64_t)n_sm * 2);
  if (grid < 1) grid = 1;
  const dim3 g(grid), b(kPeerThreads);
  switch (ps.n) {
    case 2: launch_pdl(k_peer_allreduce<2>, g, b, 0, s, ps, first, count); break;
    case 3: launch_pdl(k_peer_allreduce<3>, g, b, 0, s, ps, first, count); break;
    case 4: launch_pdl(k_peer_allreduce<4>, g, b, 0, s, ps, first, count); break;
    case 5: launch_pdl(k_peer_allreduce<5>, g, b, 0, s, ps, first, count); break;
    case 6: launch_pdl(k_peer_allreduce<6>, g, b, 0, s, ps, first, count); break;
    case 7: launch_pdl(k_peer_allreduce<7>, g, b, 0, s, ps, first, count); break;
    default: launch_pdl(k_peer_allreduce<8>, g, b, 0, s, ps, first, count); break;
  }
}

void launch_peer_wait_probe(const PeerSet& ps, cudaStream_t s) { k_peer_wait_probe<<<1, 32, 0, s>>>(ps); }

}  // namespace hb

extern "C" hb_status hb_peer_wait_probe(int32_t device, int32_t timeout_ms, uint64_t* status, double* waited_ms) {
  if (!status || !waited_ms || timeout_ms < 1 || timeout_ms > 10000) return HB_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return HB_REFUSED;
  unsigned long long* blk = nullptr;
  if (cudaMalloc(&blk, sizeof(unsigned long long) * hb::kPeerWords) != cudaSuccess) return HB_DEVICE_FAILED;
  cudaEvent_t a = nullptr, b = nullptr;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  hb::PeerSet ps{};
  ps.n = 2;
  ps.rank = 0;
  ps.bar[0] = ps.bar[1] = blk;  // the "peer" is this block, whose flag nothing raises
  ps.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  bool ok = cudaMemset(blk, 0, sizeof(unsigned long long) * hb::kPeerWords) == cudaSuccess;
  if (ok) {
    cudaEventRecord(a, 0);
    hb::launch_peer_wait_probe(ps, 0);
    cudaEventRecord(b, 0);
    ok = cudaEventSynchronize(b) == cudaSuccess && cudaGetLastError() == cudaSuccess;
  }
  float ms = 0.0f;
  unsigned long long st = 0;
  if (ok) ok = cudaEventElapsedTime(&ms, a, b) == cudaSuccess &&
               cudaMemcpy(&st, blk + hb::kPeerStatus, sizeof(st), cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaFree(blk);
  if (!ok) return HB_DEVICE_FAILED;
  *status = st;
  *waited_ms = ms;
  return HB_OK;
}
