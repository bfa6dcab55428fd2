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

// One block per (request, completed pool of the chunk); thread = channel. FP8: the pool row is stored as e4m3 codes
// of x / s with s = 2^ceil(log2(max(1e-4, amax) / 448)) (ue8m0; the division rounded to nearest as vLLM's
// `indexer_k_quant_and_cache` computes it) in the request's page of 33 rows of 128 bytes: row p % 32 the codes, row
// 32 the page's 32 fp32 scales.
template <bool FP8>
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
  if (page < 0) return;                                // uniform over the block: r and p are the block's
  if (!FP8) {
    a.pool[((int64_t)page * 32 + p % 32) * kDim + c] = __float2bfloat16_rn(acc);
    return;
  }
  __shared__ float red[kDim / 32];
  float am = fabsf(acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if ((c & 31) == 0) red[c >> 5] = am;
  __syncthreads();
  am = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const uint32_t b = __float_as_uint(__fdiv_rn(fmaxf(1e-4f, am), 448.0f));
  const uint32_t ex = ((b >> 23) & 0xffu) + ((b & 0x7fffffu) != 0u ? 1u : 0u);   // ceil(log2 s) + 127
  const float scale = __uint_as_float(ex << 23), inv = __uint_as_float((254u - ex) << 23);
  uint16_t code;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(code) : "f"(0.0f), "f"(acc * inv));
  uint8_t* pg = a.pool8 + (int64_t)page * (33 * kDim);
  pg[(p % 32) * kDim + c] = static_cast<uint8_t>(code & 0xffu);
  if (c == 0) reinterpret_cast<float*>(pg + 32 * kDim)[p % 32] = scale;
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
  const bool fp8 = a.pool8 != nullptr;
  const bool one_cache = fp8 ? a.pool == nullptr : a.pool != nullptr;     // exactly one of the two forms
  if (a.k == nullptr || a.gate == nullptr || a.ape == nullptr || a.reqs == nullptr || a.table == nullptr ||
      !one_cache || a.tail == nullptr || a.R < 0 || a.ld < kDim || a.width <= 0 || max_rows < 0 ||
      (fp8 && (reinterpret_cast<uintptr_t>(a.pool8) & 3)))
    return kErrArgs;
  if (a.R == 0) return kOk;
  const int pools = max_rows / 4 + 1;                   // a chunk of n rows completes at most n / 4 + 1 pools
  if (fp8)
    kpool_compress_kernel<true><<<dim3((unsigned)a.R, (unsigned)pools), kDim, 0, stream>>>(a);
  else
    kpool_compress_kernel<false><<<dim3((unsigned)a.R, (unsigned)pools), kDim, 0, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  kpool_seed_kernel<<<(unsigned)a.R, kDim, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
