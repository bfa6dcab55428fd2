// DSA indexer key pools for sm_100a: compress every pool of 4 tokens that a prefill chunk completes and write it into
// the paged pool-key cache, then keep the chunk's trailing incomplete pool in the request's tail ring.
//
//   pool[p, c] = sum_{j<4} softmax_j(gate[4p+j, c] + ape[j, c]) * k[4p+j, c]        (per channel c < 128, fp32)
//
// Reference behaviour (ssengine/model/pp_patch.py:415-534 `kpool_compress_insert`, `kpool_seed_tail_cache`; the
// reference ops in tests/test_kpool_cpu.py:20-41): a pool whose first tokens belong to an earlier chunk (the chunk
// starts inside it) takes those tokens' k and gate from the tail ring, so a prompt prefilled in any chunking writes
// the pools of the unsplit prefill. Here the pool-key cache is bf16 rows in pages of 32 pools (pool p of a request at
// row pages[p / 32] * 32 + p % 32, the request's KV pages), the ring bf16 [blocks][2 (k, gate)][4][128].
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kDim = 128;

// One block per (request, completed pool of the chunk); thread = channel.
__global__ void kpool_compress_kernel(KpoolArgs a) {
  const int r = blockIdx.x;
  const int4 q = reinterpret_cast<const int4*>(a.reqs)[r];     // first row, rows, start position, tail block
  const int64_t start = q.z, n = q.y;
  if (start + n < 4) return;
  const int64_t p_first = start / 4, p_last = (start + n - 4) / 4;
  const int64_t p = p_first + blockIdx.y;
  if (p > p_last) return;
  const int c = threadIdx.x;
  float lg[4], kv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t pos = 4 * p + j;
    if (pos < start) {
      const __nv_bfloat16* ring = a.tail + ((int64_t)q.w * 2 * 4 + j) * kDim;
      kv[j] = __bfloat162float(ring[c]);
      lg[j] = __bfloat162float(ring[4 * kDim + c]);
    } else {
      const int64_t row = q.x + (pos - start);
      kv[j] = __bfloat162float(a.k[row * a.ld + c]);
      lg[j] = __bfloat162float(a.gate[row * a.ld + c]);
    }
    lg[j] += a.ape[j * kDim + c];
  }
  const float m = fmaxf(fmaxf(lg[0], lg[1]), fmaxf(lg[2], lg[3]));
  float e[4], s = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    e[j] = expf(lg[j] - m);
    s += e[j];
  }
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc = __fmaf_rn(e[j] / s, kv[j], acc);
  const int32_t page = (p / 32) < a.width ? a.table[(int64_t)r * a.width + p / 32] : -1;
  if (page < 0) return;
  a.pool[((int64_t)page * 32 + p % 32) * kDim + c] = __float2bfloat16_rn(acc);
}

// The chunk's trailing incomplete pool (positions 4 * ((start + n) / 4) .. start + n - 1 inside this chunk) -> ring.
__global__ void kpool_seed_kernel(KpoolArgs a) {
  const int r = blockIdx.x;
  const int4 q = reinterpret_cast<const int4*>(a.reqs)[r];
  const int64_t start = q.z, end = (int64_t)q.z + q.y;
  const int64_t from = (end / 4) * 4 > start ? (end / 4) * 4 : start;
  const int c = threadIdx.x;
  for (int64_t pos = from; pos < end; ++pos) {
    const int64_t row = q.x + (pos - start);
    __nv_bfloat16* ring = a.tail + ((int64_t)q.w * 2 * 4 + (pos & 3)) * kDim;
    ring[c] = a.k[row * a.ld + c];
    ring[4 * kDim + c] = a.gate[row * a.ld + c];
  }
}

}  // namespace

int launch_kpool_insert(const KpoolArgs& a, int32_t max_rows, cudaStream_t stream) {
  if (a.k == nullptr || a.gate == nullptr || a.ape == nullptr || a.reqs == nullptr || a.table == nullptr ||
      a.pool == nullptr || a.tail == nullptr || a.R < 0 || a.ld < kDim || a.width <= 0 || max_rows < 0)
    return kErrArgs;
  if (a.R == 0) return kOk;
  const int pools = max_rows / 4 + 1;                   // a chunk of n rows completes at most n / 4 + 1 pools
  kpool_compress_kernel<<<dim3((unsigned)a.R, (unsigned)pools), kDim, 0, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  kpool_seed_kernel<<<(unsigned)a.R, kDim, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
