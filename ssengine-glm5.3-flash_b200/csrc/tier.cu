// Copies between a stage's cache views in HBM and its DRAM tier (pinned host memory, addressed by the device through
// unified virtual addressing): a list of runs {src, dst, bytes} -- a context's KV pages and state rows -- moved by SM
// loads and stores, one kernel for a whole tier op.
//
// Reference behaviour (ssengine/kvpool/mover.py): the reference moves the same pieces with copy-engine batch calls
// issued from the host, two hops through an HBM ring. Here the runs are gathered by one kernel on the stage's stream,
// so a write-back reads the evicted pages before any later forward on that stream reuses them and a read lands before
// the forward that needs it, with no event bookkeeping; host memory is read or written straight over the host link.
#include "../../include/ssengine_b200.h"
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kCopyThreads = 256;
constexpr int kUnroll = 4;                       // 16-byte loads in flight per thread before their stores

// run r = (src, dst, bytes) at runs[3 r .. 3 r + 2]; each CTA takes runs r = blockIdx.x, blockIdx.x + gridDim.x, ...
// A run whose pointers are not 16-byte aligned or whose size is not a multiple of 16 is skipped and raises kErrArgs.
__global__ void __launch_bounds__(kCopyThreads) copy_runs_kernel(const int64_t* __restrict__ runs, int64_t n,
                                                                 int32_t* status) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t s = runs[3 * r], d = runs[3 * r + 1], bytes = runs[3 * r + 2];
    if (((s | d | bytes) & 15) != 0 || bytes < 0) {
      if (threadIdx.x == 0) raise_status(status, kErrArgs);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(s);
    uint4* dst = reinterpret_cast<uint4*>(d);
    const int64_t n16 = bytes >> 4;
    int64_t i = threadIdx.x;
    for (; i + (kUnroll - 1) * kCopyThreads < n16; i += kUnroll * kCopyThreads) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = src[i + u * kCopyThreads];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[i + u * kCopyThreads] = v[u];
    }
    for (; i < n16; i += kCopyThreads) dst[i] = src[i];
  }
}

}  // namespace
}  // namespace ssb

extern "C" {

int ssb_copy_runs(const int64_t* runs, int64_t n, int32_t* status, void* stream) {
  if (n < 0 || (n > 0 && runs == nullptr)) return ssb::kErrArgs;
  if (n == 0) return ssb::kOk;
  const int sms = ssb::device_sm_count();
  const int64_t want = 2LL * sms;
  const int grid = static_cast<int>(n < want ? n : want);
  ssb::copy_runs_kernel<<<grid, ssb::kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(runs, n, status);
  return cudaGetLastError() == cudaSuccess ? ssb::kOk : ssb::kErrCuda;
}

}  // extern "C"
