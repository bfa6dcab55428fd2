// ssb_moe_route_permute_noalloc: MoE routing + permutation for callers that cannot allocate device memory.
//
// Who cannot allocate: a stage process whose KV pool already took the free HBM at start-up (the reference sizes its
// pool from the memory left after a profile pass, so a later cudaMalloc can fail), code that must not stall the GPU
// mid-microbatch (a cudaMalloc synchronizes the device and costs milliseconds; the reference keeps allocations out
// of the microbatch for that reason), and hosts that only hold buffers another process mapped for them. Such a
// caller passes inputs and outputs only; the routing's scratch (per-256-token expert bit masks, per-block bases, the
// GEMM tile table) lives in one file-scope __device__ array of kScratchBytes (about 1.25 MiB), which every GPU that
// loads the library holds until the process exits.
//
// Limits: T <= kMaxTokens (16384), E <= kMaxExperts (512), k < 32; larger sizes return kErrNoAllocLimit (7) before
// any launch. Every call shares the one array and leaves its contents behind: each scratch word a call reads is
// written earlier in the same call (masks and block counts for every block of the call, the scan in place, the tile
// table and its count), so nothing needs clearing; but calls whose work overlaps on the GPU (two streams, or two
// threads on one device without ordering) race on the array. The first call on a device looks up the array's
// device address (cudaGetSymbolAddress, with that device current) and caches it; make that first call before any
// stream capture. `status` may be null (the offsets step then drops its table-overflow report). With T == 0 the call
// still writes `counts` (all zero) and `offsets` (all zero).

#include <mutex>

#include "../../include/ssengine_b200.h"
#include "common.cuh"
#include "ops.h"

namespace {

constexpr int64_t kMaxTokens = 16384;
constexpr int64_t kMaxExperts = 512;
constexpr int64_t kMaxTopK = 31;
constexpr int64_t kBlockTokens = 256;
constexpr int64_t kMaxBlocks = kMaxTokens / kBlockTokens;
constexpr int64_t kMasksBytes = kMaxBlocks * kMaxExperts * 8 * 4;
constexpr int64_t kCountsBytes = kMaxBlocks * kMaxExperts * 4;
constexpr int64_t kMaxTiles = (kMaxTokens * (kMaxTopK + 1) + (kMaxExperts + 1) * 127 + 127) / 128;
constexpr int64_t kTilesBytes = (kMaxTiles * 16 + 255) / 256 * 256;
constexpr int64_t kOffMasks = 0;
constexpr int64_t kOffCounts = kOffMasks + kMasksBytes;
constexpr int64_t kOffTiles = kOffCounts + kCountsBytes;
constexpr int64_t kOffNumTiles = kOffTiles + kTilesBytes;
constexpr int64_t kScratchBytes = kOffNumTiles + 256;
constexpr int kMaxDevices = 64;
constexpr int kErrNoAllocLimit = 7;

__device__ __align__(256) uint8_t g_route_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Device address of g_route_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return ssb::kErrCuda;
  if (dev < 0 || dev >= kMaxDevices) return ssb::kErrArgs;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) return ssb::kErrCuda;
    g_scratch[dev] = p;
  }
  *out = g_scratch[dev];
  return ssb::kOk;
}

// rows[t, j] = offsets[e] + (block base of e) + (tokens of the block before t that route to e), e = ids[t, j]
__global__ void moe_rows_kernel(const int32_t* __restrict__ ids, int64_t T, int E, int k,
                                const uint32_t* __restrict__ masks, const int32_t* __restrict__ block_base,
                                const int32_t* __restrict__ offsets, int32_t* __restrict__ rows) {
  const int64_t n = T * k;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / k;
    const int e = ids[idx];
    const int64_t b = t / kBlockTokens;
    const int i = static_cast<int>(t % kBlockTokens);
    const uint32_t* m = masks + (b * E + e) * 8;
    int rank = block_base[b * E + e];
    for (int q = 0; q < (i >> 5); ++q) rank += __popc(m[q]);
    rank += __popc(m[i >> 5] & ((1u << (i & 31)) - 1u));
    rows[idx] = offsets[e] + rank;
  }
}

}  // namespace

extern "C" int ssb_moe_route_permute_noalloc(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids,
                                             float* weights, int32_t* rows, int32_t* counts, int32_t* offsets,
                                             int32_t* status, void* stream_) {
  if (T < 0 || E <= 0 || k <= 0 || k > E) return ssb::kErrArgs;
  if (T > kMaxTokens || E > kMaxExperts || k > kMaxTopK) return kErrNoAllocLimit;
  if (logits == nullptr || ids == nullptr || weights == nullptr || rows == nullptr || counts == nullptr ||
      offsets == nullptr)
    return ssb::kErrArgs;
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc != ssb::kOk) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  uint8_t* s = static_cast<uint8_t*>(base);
  uint32_t* masks = reinterpret_cast<uint32_t*>(s + kOffMasks);
  int32_t* block_counts = reinterpret_cast<int32_t*>(s + kOffCounts);
  int32_t* tiles = reinterpret_cast<int32_t*>(s + kOffTiles);
  int32_t* num_tiles = reinterpret_cast<int32_t*>(s + kOffNumTiles);
  const int32_t cap = static_cast<int32_t>((T * (k + 1) + (static_cast<int64_t>(E) + 1) * 127 + 127) / 128);
  // with no tokens only the offsets step runs: it writes zero counts and offsets (no block reads)
  if (T > 0) {
    rc = ssb::launch_moe_route(logits, T, E, k, ids, weights, stream);
    if (rc != ssb::kOk) return rc;
    rc = ssb::launch_moe_count(ids, T, E, k, masks, block_counts, stream);
    if (rc != ssb::kOk) return rc;
  }
  rc = ssb::launch_moe_offsets(T, E, block_counts, counts, offsets, tiles, num_tiles, cap, nullptr, 0, status, stream);
  if (rc != ssb::kOk) return rc;
  if (T == 0) return ssb::kOk;
  const int64_t n = T * k;
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  moe_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(ids, T, E, k, masks, block_counts, offsets,
                                                                         rows);
  return cudaGetLastError() == cudaSuccess ? ssb::kOk : ssb::kErrCuda;
}
