// Small data-movement kernels of the DSA attention block (sm_100a): RMSNorm of a column slice, rotary embedding of the
// rope slices, head-major <-> row-major transposes around the per-head (absorb / v_up) GEMMs, column concatenation of
// the latent-cache rows. All HBM-bound, 16-byte accesses where the shapes allow.
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

// y[r, :w] = x[r, :w] * rsqrt(mean(x^2) + eps) * g[:w]; one block per row.
__global__ void rmsnorm_cols_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int width,
                                    const __nv_bfloat16* __restrict__ g, float eps, __nv_bfloat16* __restrict__ y,
                                    int64_t ldy) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* xr = x + r * ldx;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    const float v = __bfloat162float(xr[c]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(width) + eps);
  for (int c = threadIdx.x; c < width; c += blockDim.x)
    y[r * ldy + c] = __float2bfloat16(__bfloat162float(xr[c]) * inv * __bfloat162float(g[c]));
}

// In-place rotary embedding of a 64-dim slice per head with interleaved pairs (the MLA rope of DeepSeek-V3.2-style
// DSA layers, GPT-J pairing): for i < 32, with angle = pos * theta^(-i / 32):
// (a, b) = (x[2i], x[2i + 1]) -> (a cos - b sin, b cos + a sin).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int64_t ldx, int heads, int64_t head_stride,
                            const int64_t* __restrict__ positions, int64_t rows, float theta) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * heads * 32) return;
  const int d = static_cast<int>(i & 31);
  const int64_t rh = i >> 5;
  const int64_t r = rh / heads;
  const int h = static_cast<int>(rh - r * heads);
  __nv_bfloat16* p = x + r * ldx + h * head_stride;
  const float inv_freq = powf(theta, -static_cast<float>(d) / 32.0f);
  const float ang = static_cast<float>(positions[r]) * inv_freq;
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const __nv_bfloat162 ab = *reinterpret_cast<const __nv_bfloat162*>(p + 2 * d);
  const float a = __low2float(ab), b = __high2float(ab);
  *reinterpret_cast<__nv_bfloat162*>(p + 2 * d) = __floats2bfloat162_rn(a * cs - b * sn, b * cs + a * sn);
}

// dst[h, r, :dim] = src[r, h * src_head_stride + :dim] (to_heads) or dst[r, h * dst_head_stride + :dim] =
// src[h, r, :dim] (from heads); head-major rows padded to rows_pad (pad rows written as zeros when to_heads).
__global__ void transpose_heads_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                       int64_t rows, int64_t rows_pad, int heads, int dim16, int64_t row_ld,
                                       int64_t head_stride, int to_heads) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(heads) * rows_pad * dim16;
  if (i >= total) return;
  const int c = static_cast<int>(i % dim16);
  const int64_t hr = i / dim16;
  const int64_t r = hr % rows_pad;
  const int h = static_cast<int>(hr / rows_pad);
  const int64_t hm = (static_cast<int64_t>(h) * rows_pad + r) * dim16 + c;        // head-major, 16-byte units
  if (to_heads) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows) v = reinterpret_cast<const uint4*>(src + r * row_ld + h * head_stride)[c];
    reinterpret_cast<uint4*>(dst)[hm] = v;
  } else if (r < rows) {
    reinterpret_cast<uint4*>(dst + r * row_ld + h * head_stride)[c] = reinterpret_cast<const uint4*>(src)[hm];
  }
}

// out[r, :wa + wb] = [a[r, :wa], b[r, :wb]] (16-byte units).
__global__ void concat_cols_kernel(const __nv_bfloat16* __restrict__ a, int64_t lda, int wa16,
                                   const __nv_bfloat16* __restrict__ b, int64_t ldb, int wb16,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo, int64_t rows) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int w = wa16 + wb16;
  if (i >= rows * w) return;
  const int64_t r = i / w;
  const int c = static_cast<int>(i - r * w);
  const uint4 v = c < wa16 ? reinterpret_cast<const uint4*>(a + r * lda)[c]
                           : reinterpret_cast<const uint4*>(b + r * ldb)[c - wa16];
  reinterpret_cast<uint4*>(out + r * ldo)[c] = v;
}

// Tile table of a per-head grouped GEMM over head-major rows padded to rows_pad: tile i = {head, first row, 128, 0}
// with head = i / (rows_pad / 128); *num = heads * rows_pad / 128.
__global__ void head_tiles_kernel(int heads, int64_t rows_pad, int32_t* __restrict__ tiles, int32_t* __restrict__ num) {
  const int64_t per = rows_pad / 128;
  const int64_t n = per * heads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t h = i / per;
    const int64_t m = i - h * per;
    reinterpret_cast<int4*>(tiles)[i] =
        make_int4(static_cast<int>(h), static_cast<int>(h * rows_pad + 128 * m), 128, 0);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *num = static_cast<int32_t>(n);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

unsigned blocks_for(int64_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

int launch_rmsnorm_cols(const void* x, int64_t ldx, int width, int64_t rows, const void* g, float eps, void* y,
                        int64_t ldy, cudaStream_t stream) {
  if (x == nullptr || g == nullptr || y == nullptr || width <= 0 || rows < 0 || ldx < width || ldy < width)
    return kErrArgs;
  if (rows == 0) return kOk;
  rmsnorm_cols_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, width, static_cast<const __nv_bfloat16*>(g), eps,
      static_cast<__nv_bfloat16*>(y), ldy);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_rope(void* x, int64_t ldx, int heads, int64_t head_stride, const int64_t* positions, int64_t rows,
                float theta, cudaStream_t stream) {
  if (x == nullptr || positions == nullptr || heads <= 0 || rows < 0 || theta <= 0.0f) return kErrArgs;
  // each lane moves one bf16 pair with a 4-byte access: every slice must start on an even element
  if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0 || (ldx & 1) != 0 || (head_stride & 1) != 0) return kErrArgs;
  if (rows == 0) return kOk;
  const int64_t n = rows * heads * 32;
  rope_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), ldx, heads, head_stride,
                                                      positions, rows, theta);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_transpose_heads(const void* src, void* dst, int64_t rows, int64_t rows_pad, int heads, int dim,
                           int64_t row_ld, int64_t head_stride, bool to_heads, cudaStream_t stream) {
  if (src == nullptr || dst == nullptr || rows < 0 || rows_pad < rows || heads <= 0 || dim <= 0 || dim % 8 != 0 ||
      row_ld % 8 != 0 || head_stride % 8 != 0 || !al16(src) || !al16(dst))
    return kErrArgs;
  const int64_t total = static_cast<int64_t>(heads) * rows_pad * (dim / 8);
  if (total == 0) return kOk;
  transpose_heads_kernel<<<blocks_for(total, 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), rows, rows_pad, heads, dim / 8, row_ld,
      head_stride, to_heads ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_head_tiles(int heads, int64_t rows_pad, int32_t* tiles, int64_t tile_cap, int32_t* num,
                      cudaStream_t stream) {
  if (tiles == nullptr || num == nullptr || heads <= 0 || rows_pad < 0 || rows_pad % 128 != 0 || !al16(tiles))
    return kErrArgs;
  const int64_t n = rows_pad / 128 * heads;
  if (n > tile_cap || rows_pad * heads >= (int64_t(1) << 31)) return kErrArgs;
  head_tiles_kernel<<<static_cast<unsigned>(n / 256 + 1), 256, 0, stream>>>(heads, rows_pad, tiles, num);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_concat_cols(const void* a, int64_t lda, int wa, const void* b, int64_t ldb, int wb, void* out, int64_t ldo,
                       int64_t rows, cudaStream_t stream) {
  if (a == nullptr || b == nullptr || out == nullptr || wa % 8 != 0 || wb % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 ||
      ldo % 8 != 0 || !al16(a) || !al16(b) || !al16(out) || rows < 0 || ldo < wa + wb)
    return kErrArgs;
  const int64_t n = rows * ((wa + wb) / 8);
  if (n == 0) return kOk;
  concat_cols_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(a), lda, wa / 8,
                                                             static_cast<const __nv_bfloat16*>(b), ldb, wb / 8,
                                                             static_cast<__nv_bfloat16*>(out), ldo, rows);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
