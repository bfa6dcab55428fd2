// Stage-level kernels around the layers (sm_100a): device-side microbatch metadata, the stage-0 embedding gather,
// RMSNorm and the last stage's greedy argmax.
//
// Metadata (the reference builds it on the host with numpy and copies one packed buffer, ssengine/model/metadata.py:
// 79-96, 210-313): from the compact per-request arrays of a plan in row order -- qsl [R+1] (first row of each
// request), starts [R] (tokens already in KV), page_ptr [R+1] and pages (each request's 128-token KV pages) --
// this builds on the device, bit-exact with the reference's `g0_table` / `graph_rows`:
//   positions[t] = starts[r] + t - qsl[r]                         (pad rows of a graph bucket: 0)
//   slots[t]     = pages[r][pos / P] * P + pos % P                (pad rows: -1, they write no KV)
//   table[r, c]  = pages[r][c / kpp] * kpp + c % kpp  for c < ceil(seq_len / P) * kpp, else 0   (kpp = P / 64)
// so only the plan's page ids cross PCIe, not the expanded tables.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

__global__ void stage_rows_kernel(const int32_t* __restrict__ qsl, const int32_t* __restrict__ starts,
                                  const int32_t* __restrict__ page_ptr, const int32_t* __restrict__ pages, int R,
                                  int64_t T, int64_t bucket, int page_tokens, int64_t* __restrict__ positions,
                                  int64_t* __restrict__ slots) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < bucket; t += (int64_t)gridDim.x * blockDim.x) {
    if (t >= T) {
      positions[t] = 0;
      slots[t] = -1;
      continue;
    }
    int lo = 0, hi = R;                          // last r with qsl[r] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (qsl[mid] <= t) lo = mid; else hi = mid;
    }
    const int64_t pos = starts[lo] + (t - qsl[lo]);
    positions[t] = pos;
    slots[t] = static_cast<int64_t>(pages[page_ptr[lo] + pos / page_tokens]) * page_tokens + pos % page_tokens;
  }
}

__global__ void stage_table_kernel(const int32_t* __restrict__ qsl, const int32_t* __restrict__ starts,
                                   const int32_t* __restrict__ page_ptr, const int32_t* __restrict__ pages, int R,
                                   int width, int page_tokens, int kpp, int32_t* __restrict__ table) {
  const int64_t total = static_cast<int64_t>(R) * width;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(idx / width);
    const int c = static_cast<int>(idx - static_cast<int64_t>(r) * width);
    const int64_t seq = starts[r] + (qsl[r + 1] - qsl[r]);
    const int64_t n = (seq + page_tokens - 1) / page_tokens;
    table[idx] = c < n * kpp ? pages[page_ptr[r] + c / kpp] * kpp + c % kpp : 0;
  }
}

// out[t, :] = table[ids[t], :] (bf16 rows, 16-byte vectors); ids outside [0, vocab) give a zero row.
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ table, int64_t vocab, int64_t H,
                                  const int64_t* __restrict__ ids, int64_t T, __nv_bfloat16* __restrict__ out) {
  const int64_t nvec = H / 8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < T * nvec;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / nvec, v = idx - t * nvec;
    const int64_t id = ids[t];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab) val = reinterpret_cast<const uint4*>(table + id * H)[v];
    reinterpret_cast<uint4*>(out + t * H)[v] = val;
  }
}

// y[r] = x[rows[r]] * rsqrt(mean(x^2) + eps) * w, one block per output row (rows == nullptr: row r).
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t H, const int64_t* __restrict__ rows,
                               int64_t n, const __nv_bfloat16* __restrict__ w, float eps,
                               __nv_bfloat16* __restrict__ y) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  const int64_t src = rows != nullptr ? rows[r] : r;
  const __nv_bfloat16* xr = x + src * H;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __bfloat162float(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(H) + eps);
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x)
    y[r * H + i] = __float2bfloat16(__bfloat162float(xr[i]) * inv * __bfloat162float(w[i]));
}

// out[r] = the lowest column holding the maximum of logits[r, :N] (NaN never wins), one block per row.
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t ld, int64_t N, int64_t n,
                              int64_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  const float* row = logits + r * ld;
  float bv = -INFINITY;
  int64_t bi = N;
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
    const float v = row[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
    const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    bv = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : N;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
      const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) out[r] = bi < N ? bi : 0;
  }
}

int grid_of(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

// Gated RMSNorm per 128-channel head group: y = x * rsqrt(mean(x^2) + eps) * w[c] * sigmoid(gate) (bf16 out); one warp
// per (row, head), 4 channels a lane. The reference's KDA output norm (FusedRMSNormGated, activation sigmoid).
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* gate, int64_t ldg,
                                     const __nv_bfloat16* w, float eps, __nv_bfloat16* y, int64_t ldy, int64_t rows,
                                     int heads) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * heads) return;
  const int64_t t = gw / heads;
  const int h = static_cast<int>(gw - t * heads);
  const int c = h * 128 + lane * 4;
  const uint2 xv = *reinterpret_cast<const uint2*>(x + t * ldx + c);
  const uint2 gv = *reinterpret_cast<const uint2*>(gate + t * ldg + c);
  const uint2 wv = *reinterpret_cast<const uint2*>(w + lane * 4);
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
  float f[4], ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[i] = __bfloat162float(xb[i]);
    ss = fmaf(f[i], f[i], ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / 128.0f + eps);
  uint2 ov;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float gt = __bfloat162float(gb[i]);
    ob[i] = __float2bfloat16(f[i] * inv * __bfloat162float(wb[i]) / (1.0f + expf(-gt)));
  }
  *reinterpret_cast<uint2*>(y + t * ldy + c) = ov;
}

// The same arithmetic with 16 elements a lane (two 16-byte loads and stores; 8 lanes a head, 4 heads a warp): lane j
// of a head holds the elements of the 4 lanes 4 j .. 4 j + 3 of the warp-per-head form above, and its sum of squares
// is reduced in that form's tree order (lane xor 16, 8, 4 across the 8 lanes, then xor 2, 1 inside the lane), so the
// results are identical.
__global__ void gated_rmsnorm16_kernel(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* gate, int64_t ldg,
                                       const __nv_bfloat16* w, float eps, __nv_bfloat16* y, int64_t ldy,
                                       int64_t rows, int heads) {
  const int lane = threadIdx.x & 31;
  const int64_t grp = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 4 + (lane >> 3);
  const bool live = grp < rows * heads;
  const int64_t t = live ? grp / heads : 0;
  const int h = live ? static_cast<int>(grp - t * heads) : 0;
  const int j = lane & 7;
  const int c = h * 128 + j * 16;
  uint4 xv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, gv[2] = {xv[0], xv[0]}, wv[2] = {xv[0], xv[0]};
  if (live) {
    xv[0] = *reinterpret_cast<const uint4*>(x + t * ldx + c);
    xv[1] = *reinterpret_cast<const uint4*>(x + t * ldx + c + 8);
    gv[0] = *reinterpret_cast<const uint4*>(gate + t * ldg + c);
    gv[1] = *reinterpret_cast<const uint4*>(gate + t * ldg + c + 8);
    wv[0] = *reinterpret_cast<const uint4*>(w + j * 16);
    wv[1] = *reinterpret_cast<const uint4*>(w + j * 16 + 8);
  }
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(xv);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(gv);
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(wv);
  float f[16], p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    p[q] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[4 * q + i] = __bfloat162float(xb[4 * q + i]);
      p[q] = fmaf(f[4 * q + i], f[4 * q + i], p[q]);
    }
  }
#pragma unroll
  for (int o = 4; o; o >>= 1)                          // the per-head form's lane xor 16, 8, 4
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], o);
  float p2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) p2[q] = p[q] + p[q ^ 2];  // lane xor 2
  const float ss = p2[0] + p2[1];                      // lane xor 1
  const float inv = rsqrtf(ss / 128.0f + eps);
  uint4 ov[2];
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(ov);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float gt = __bfloat162float(gb[i]);
    ob[i] = __float2bfloat16(f[i] * inv * __bfloat162float(wb[i]) / (1.0f + expf(-gt)));
  }
  if (live) {
    *reinterpret_cast<uint4*>(y + t * ldy + c) = ov[0];
    *reinterpret_cast<uint4*>(y + t * ldy + c + 8) = ov[1];
  }
}

// The gated RMSNorm with its output quantized to NVFP4 for the next GEMM (the KDA o_proj): the arithmetic of
// gated_rmsnorm16_kernel up to the bf16 rounding of each element, then each lane's 16 elements (one NVFP4 block) are
// quantized exactly as the activation quantizer does (nvfp4_quant16 on the bf16 values, global scale gs), so the codes
// and scale atoms equal those of the two-step path; the 4 scale bytes of an atom column come from lanes j .. j + 3 of
// the head. Codes [rows, ldc] bytes, scale atoms of the 128-row blocks (sf_atom_offset layout, ncb atom columns).
__global__ void gated_rmsnorm_nvfp4_kernel(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* gate,
                                           int64_t ldg, const __nv_bfloat16* w, float eps, float gs, uint8_t* codes,
                                           int64_t ldc, uint8_t* sf, int64_t ncb, int64_t rows, int heads) {
  const int lane = threadIdx.x & 31;
  const int64_t grp = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 4 + (lane >> 3);
  const bool live = grp < rows * heads;
  const int64_t t = live ? grp / heads : 0;
  const int h = live ? static_cast<int>(grp - t * heads) : 0;
  const int j = lane & 7;
  const int c = h * 128 + j * 16;
  uint4 xv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, gv[2] = {xv[0], xv[0]}, wv[2] = {xv[0], xv[0]};
  if (live) {
    xv[0] = *reinterpret_cast<const uint4*>(x + t * ldx + c);
    xv[1] = *reinterpret_cast<const uint4*>(x + t * ldx + c + 8);
    gv[0] = *reinterpret_cast<const uint4*>(gate + t * ldg + c);
    gv[1] = *reinterpret_cast<const uint4*>(gate + t * ldg + c + 8);
    wv[0] = *reinterpret_cast<const uint4*>(w + j * 16);
    wv[1] = *reinterpret_cast<const uint4*>(w + j * 16 + 8);
  }
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(xv);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(gv);
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(wv);
  float f[16], p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    p[q] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[4 * q + i] = __bfloat162float(xb[4 * q + i]);
      p[q] = fmaf(f[4 * q + i], f[4 * q + i], p[q]);
    }
  }
#pragma unroll
  for (int o = 4; o; o >>= 1)
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], o);
  float p2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) p2[q] = p[q] + p[q ^ 2];
  const float ss = p2[0] + p2[1];
  const float inv = rsqrtf(ss / 128.0f + eps);
  float yv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float gt = __bfloat162float(gb[i]);
    yv[i] = __bfloat162float(__float2bfloat16(f[i] * inv * __bfloat162float(wb[i]) / (1.0f + expf(-gt))));
  }
  uint32_t pk[2];
  const uint32_t s8 = live ? nvfp4_quant16(yv, gs, pk) : 0u;
  uint32_t word = s8;
  word |= __shfl_down_sync(0xffffffffu, s8, 1) << 8;
  word |= __shfl_down_sync(0xffffffffu, s8, 2) << 16;
  word |= __shfl_down_sync(0xffffffffu, s8, 3) << 24;
  if (live) {
    *reinterpret_cast<uint2*>(codes + t * ldc + c / 2) = make_uint2(pk[0], pk[1]);
    if ((j & 3) == 0) *reinterpret_cast<uint32_t*>(sf + sf_atom_offset(t, c / 16, ncb)) = word;
  }
}

// hc_expand: the 4 residual streams of a stage-0 row all start as its embedding (16-byte pieces).
__global__ void hc_expand_kernel(const uint4* __restrict__ x, int64_t n16_row, int64_t T, uint4* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * n16_row) return;
  const int64_t t = i / n16_row, c = i - t * n16_row;
  const uint4 v = x[i];
#pragma unroll
  for (int s = 0; s < 4; ++s) out[(t * 4 + s) * n16_row + c] = v;
}

// hc mean: out[r] = bf16(mean over the 4 streams of res[rows[r]]) (rows == nullptr: row r).
__global__ void hc_mean_kernel(const __nv_bfloat16* __restrict__ res, int64_t H, const int64_t* __restrict__ rows,
                               int64_t n, __nv_bfloat16* __restrict__ out) {
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  const int64_t t = rows != nullptr ? rows[r] : r;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
    float v = 0.0f;
#pragma unroll
    for (int s = 0; s < 4; ++s) v += __bfloat162float(res[(t * 4 + s) * H + h]);
    out[r * H + h] = __float2bfloat16(v * 0.25f);
  }
}

}  // namespace

int launch_stage_metadata(const int32_t* qsl, const int32_t* starts, const int32_t* page_ptr, const int32_t* pages,
                          int32_t R, int64_t T, int64_t bucket, int32_t page_tokens, int32_t width,
                          int64_t* positions, int64_t* slots, int32_t* table, cudaStream_t stream) {
  if (R < 0 || T < 0 || bucket < T || page_tokens <= 0 || page_tokens % 64 != 0 || width < 0) return kErrArgs;
  if (R == 0 && T > 0) return kErrArgs;
  if (bucket > 0)
    stage_rows_kernel<<<grid_of(bucket, 256), 256, 0, stream>>>(qsl, starts, page_ptr, pages, R, T, bucket,
                                                                 page_tokens, positions, slots);
  if (R > 0 && width > 0 && table != nullptr)
    stage_table_kernel<<<grid_of(static_cast<int64_t>(R) * width, 256), 256, 0, stream>>>(
        qsl, starts, page_ptr, pages, R, width, page_tokens, page_tokens / 64, table);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_embed_rows(const void* table, int64_t vocab, int64_t H, const int64_t* ids, int64_t T, void* out,
                      cudaStream_t stream) {
  if (H % 8 != 0 || T < 0) return kErrArgs;
  if (T == 0) return kOk;
  embed_rows_kernel<<<grid_of(T * (H / 8), 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(table), vocab, H, ids, T, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_rmsnorm(const void* x, int64_t H, const int64_t* rows, int64_t n, const void* w, float eps, void* y,
                   cudaStream_t stream) {
  if (H <= 0 || n < 0) return kErrArgs;
  if (n == 0) return kOk;
  rmsnorm_kernel<<<static_cast<unsigned>(n), 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), H, rows, n,
                                                                reinterpret_cast<const __nv_bfloat16*>(w), eps,
                                                                reinterpret_cast<__nv_bfloat16*>(y));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_argmax_rows(const float* logits, int64_t ld, int64_t N, int64_t n, int64_t* out, cudaStream_t stream) {
  if (N <= 0 || n < 0 || ld < N) return kErrArgs;
  if (n == 0) return kOk;
  argmax_kernel<<<static_cast<unsigned>(n), 256, 0, stream>>>(logits, ld, N, n, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_gated_rmsnorm(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps, void* y,
                         int64_t ldy, int64_t rows, int heads, cudaStream_t stream) {
  if (x == nullptr || gate == nullptr || w == nullptr || y == nullptr || rows < 0 || heads <= 0 || ldx < heads * 128 ||
      ldg < heads * 128 || ldy < heads * 128 || (ldx | ldg | ldy) % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(w) |
        reinterpret_cast<uintptr_t>(y)) & 7))
    return kErrArgs;
  if (rows == 0) return kOk;
  if ((ldx | ldg | ldy) % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate) |
                                       reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
    const int64_t warps16 = (rows * heads + 3) / 4;
    gated_rmsnorm16_kernel<<<static_cast<unsigned>((warps16 * 32 + 255) / 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(gate), ldg,
        static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
  }
  const int64_t warps = rows * heads;
  gated_rmsnorm_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(gate), ldg,
      static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_gated_rmsnorm_nvfp4(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps,
                               float gs, uint8_t* codes, int64_t ldc, uint8_t* sf, int64_t rows, int heads,
                               cudaStream_t stream) {
  if (x == nullptr || gate == nullptr || w == nullptr || codes == nullptr || sf == nullptr || rows < 0 || heads <= 0 ||
      ldx < heads * 128 || ldg < heads * 128 || ldc < heads * 64 || (ldx | ldg) % 8 != 0 || ldc % 8 != 0 ||
      !(gs > 0.0f) ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(w)) & 15) ||
      (reinterpret_cast<uintptr_t>(codes) & 7) || (reinterpret_cast<uintptr_t>(sf) & 3))
    return kErrArgs;
  if (rows == 0) return kOk;
  const int64_t warps = (rows * heads + 3) / 4;
  gated_rmsnorm_nvfp4_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(gate), ldg,
      static_cast<const __nv_bfloat16*>(w), eps, gs, codes, ldc, sf, sf_atom_cols(static_cast<int64_t>(heads) * 128),
      rows, heads);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_hc_expand(const void* x, int64_t T, int64_t H, void* out, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || T < 0 || H <= 0 || H % 8 != 0 ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15))
    return kErrArgs;
  if (T == 0) return kOk;
  const int64_t n16 = H / 8, total = T * n16;
  hc_expand_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(static_cast<const uint4*>(x), n16, T,
                                                                                    static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_hc_mean(const void* res, int64_t H, const int64_t* rows, int64_t n, void* out, cudaStream_t stream) {
  if (res == nullptr || out == nullptr || n < 0 || H <= 0) return kErrArgs;
  if (n == 0) return kOk;
  hc_mean_kernel<<<static_cast<unsigned>(n), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(res), H, rows, n,
                                                               static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
