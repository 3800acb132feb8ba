// hb_build_noalloc: the node histogram of hb_build for callers that cannot
// allocate device memory at call time, for instance a host framework that
// hands every byte of HBM to its own pool and forbids cudaMalloc once
// training runs. The row ids come from, and the histogram goes to, device
// buffers the caller owns; the call's own working memory is one static
// device array of this file, so the call allocates nothing.
//
// Scratch: g_scratch, kScratchBytes (512 KiB + 1 KiB) per device and process:
//   [0, 512 KiB)           fixed-point (g, h) accumulators, at most
//                          kNoAllocMaxBins = 32,768 bins (128 features of
//                          256 bins); zeroed by every call
//   [512 KiB, +256)        the one histogram entry (HEntry)
//   [512 KiB + 256, +256)  the level state the histogram kernels read
//   [512 KiB + 512, +8)    bad-row counter and the status word the host
//                          reads back; both are set to zero at the start of
//                          every call (cudaMemsetAsync, which allocates
//                          nothing), so a call that failed half way cannot
//                          leave a stale verdict for the next one
// An index with more bins than kNoAllocMaxBins is refused.
//
// Ordering: the kernels run on the engine's stream. `rows_dev` must hold its
// final values before the call starts: a caller that produced it on another
// stream synchronises that stream (or the device) first.
//
// The first call on a device (with that device current) looks up the
// scratch's device address with cudaGetSymbolAddress; that may load this
// file's device code, so make the first call before any stream capture.
//
// There is one scratch per device per process, shared by every engine on
// that device: two calls that overlapped on one device would race on it.
// The calls therefore take a per-device lock and wait for their own kernels
// before returning, so that within one process they never overlap.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "hb_engine_view.h"
#include "hb_internal.h"
#include "hb_kernels.cuh"

using namespace hb;

namespace {

constexpr uint32_t kNoAllocMaxBins = 32768;
constexpr size_t kHistBytes = sizeof(longlong2) * kNoAllocMaxBins;
constexpr size_t kEntryOff = kHistBytes;
constexpr size_t kLevelOff = kHistBytes + 256;
constexpr size_t kFlagOff = kHistBytes + 512;
constexpr size_t kScratchBytes = kHistBytes + 1024;
static_assert(sizeof(HEntry) <= 256 && sizeof(LevelState) <= 256, "scratch layout");

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock[kMaxDevices];
unsigned char* g_base[kMaxDevices] = {};  // device address of g_scratch, per device

// Zero the accumulators, check the row ids (ascending, distinct, inside the
// index) and write the single histogram entry.
__global__ void k_na_prepare(longlong2* __restrict__ hist, uint32_t total_bins,
                             const uint32_t* __restrict__ rows, uint64_t n, uint64_t n_rows,
                             HEntry* __restrict__ entry, unsigned* __restrict__ bad) {
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (uint64_t i = t; i < total_bins; i += step) hist[i] = make_longlong2(0, 0);
  unsigned mine = 0;
  for (uint64_t i = t; i < n; i += step) {
    const uint32_t r = rows[i];
    if (r >= n_rows || (i > 0 && rows[i - 1] >= r)) mine = 1;
  }
  if (mine) atomicOr(bad, 1u);
  if (t == 0) {
    HEntry x;
    x.slot = 0;
    x.identity = 0;
    x.begin = 0;
    x.len = (uint32_t)n;
    x.prefix = 0;
    *entry = x;
  }
}

// One entry over all n rows, or, when a row id was bad, no entry at all (the
// histogram kernels then read no row). Publishes the verdict.
__global__ void k_na_gate(uint64_t n, LevelState* __restrict__ ls, const unsigned* __restrict__ bad,
                          unsigned* __restrict__ status) {
  const unsigned b = *bad;
  LevelState s{};
  s.n_hentries = b ? 0 : 1;
  s.hist_rows = b ? 0 : n;
  *ls = s;
  *status = b;
}

bool on_device(const void* p, int device) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice && a.device == device) || a.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" hb_status hb_build_noalloc(hb_engine* e, const uint32_t* rows_dev, uint64_t n,
                                      hb_grad_stats* out_dev) {
  if (!e) return HB_INVALID_ARGUMENT;
  EngineView v;
  engine_view(e, &v);
  if (v.failed) return HB_REFUSED;
  if (v.device < 0 || v.device >= kMaxDevices) return engine_refuse(e, "device ordinal out of range");
  cudaError_t rc = cudaSetDevice(v.device);
  if (rc != cudaSuccess) return engine_fail(e, "cudaSetDevice", rc);
  if (!v.uploaded || !v.staged) return engine_refuse(e, "no staged gradients");
  const DevConst& c = *v.c;
  if (c.total_bins > kNoAllocMaxBins)
    return engine_refuse(e, "hb_build_noalloc: the index has more than 32768 bins, the scratch limit");
  if (!out_dev) return engine_invalid(e, "hb_build_noalloc: out_dev is NULL");
  if (n && !rows_dev) return engine_invalid(e, "hb_build_noalloc: rows_dev is NULL");
  if (n > c.n_rows) return engine_invalid(e, "hb_build_noalloc: more row ids than the index has rows");
  if (reinterpret_cast<uintptr_t>(out_dev) % 8 || reinterpret_cast<uintptr_t>(rows_dev) % 4)
    return engine_invalid(e, "hb_build_noalloc: out_dev must be 8-byte and rows_dev 4-byte aligned");
  if (!on_device(out_dev, v.device) || (n && !on_device(rows_dev, v.device)))
    return engine_refuse(e, "hb_build_noalloc: rows and out must be device memory of the engine's GPU");

  std::lock_guard<std::mutex> hold(g_lock[v.device]);
  if (!g_base[v.device]) {
    void* p = nullptr;
    rc = cudaGetSymbolAddress(&p, g_scratch);
    if (rc != cudaSuccess) return engine_fail(e, "cudaGetSymbolAddress(g_scratch)", rc);
    g_base[v.device] = static_cast<unsigned char*>(p);
  }
  unsigned char* base = g_base[v.device];
  longlong2* hist = reinterpret_cast<longlong2*>(base);
  HEntry* entry = reinterpret_cast<HEntry*>(base + kEntryOff);
  LevelState* ls = reinterpret_cast<LevelState*>(base + kLevelOff);
  unsigned* bad = reinterpret_cast<unsigned*>(base + kFlagOff);
  unsigned* status = bad + 1;

  cudaStream_t s = v.stream;
  // the counter and the verdict start at zero whatever an earlier call left
  rc = cudaMemsetAsync(bad, 0, 2 * sizeof(unsigned), s);
  if (rc != cudaSuccess) return engine_fail(e, "hb_build_noalloc: clear the verdict", rc);
  const uint64_t work = std::max<uint64_t>(n, c.total_bins);
  const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((work + 255) / 256, 4ull * v.n_sm));
  k_na_prepare<<<grid, 256, 0, s>>>(hist, c.total_bins, rows_dev, n, c.n_rows, entry, bad);
  k_na_gate<<<1, 1, 0, s>>>(n, ls, bad, status);
  launch_hist(c, v.fo, v.rec, v.gpair, v.scale, rows_dev, entry, ls, hist, nullptr, nullptr,
              hist_grid(v.n_sm), hist_smem_bytes(c), s);
  launch_dequantize(hist, c.total_bins, v.scale, reinterpret_cast<double*>(out_dev), s);
  rc = cudaGetLastError();
  if (rc != cudaSuccess) return engine_fail(e, "hb_build_noalloc launch", rc);
  unsigned verdict = 0;
  rc = cudaMemcpyAsync(&verdict, status, sizeof(verdict), cudaMemcpyDeviceToHost, s);
  if (rc == cudaSuccess) rc = cudaStreamSynchronize(s);
  if (rc != cudaSuccess) return engine_fail(e, "hb_build_noalloc", rc);
  if (verdict) return engine_refuse(e, "rows must ascend within the index");
  return HB_OK;
}
