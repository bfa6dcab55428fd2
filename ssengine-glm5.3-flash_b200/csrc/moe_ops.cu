// MoE routing / permutation / combine and the NVFP4 activation quantizer (sm_100a, HBM-bound integer and byte
// work: coalesced vector loads and stores, grids sized in multiples of the SM count where the work allows).
//
// Permutation contract (bit-exact): expert-major, tokens ascending inside an expert, the shared expert (index E)
// last with every token; expert e's rows start at offsets[e] = sum over e' < e of ceil(n_e' / 128) * 128, so every
// 128-row GEMM tile belongs to one expert. The rank of token t inside expert e is the number of tokens before t that
// route to e: per 256-token block a bit mask per expert (built with shared-memory atomicOr, order independent),
// block bases by an exclusive scan over blocks, and popcounts inside the block -- deterministic, no global atomics.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

constexpr int kBlockTokens = 256;
constexpr int kMaskWords = kBlockTokens / 32;

// ---- NVFP4 activation quantizer: one thread per (row, atom column) = 64 elements, 4 scale bytes ----------------
// The 128 input bytes are loaded before any arithmetic (8 independent 16-byte loads in flight per thread).
__global__ void nvfp4_quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t K, int64_t ldx,
                                      float gs, uint8_t* __restrict__ codes, int64_t ldc, uint8_t* __restrict__ sf,
                                      int64_t ncb) {
  // one warp per 512 elements of a row, lane l quantizing the 16-element block l: its two 16-byte loads are half of
  // a 1 KB span per instruction, its 8 code bytes a quarter of a 256-byte store; the 4 scale bytes of each atom column
  // (64 elements) are assembled in the column's first lane. Atom columns past K (up to the 256-element padding) get
  // zero scale words.
  const int lane = threadIdx.x & 31;
  const int64_t chunks = (K + 511) / 512;
  const int64_t total = rows * chunks;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
    const int64_t r = w / chunks;
    const int64_t k0 = (w - r * chunks) * 512 + lane * 16;
    const bool valid = k0 + 16 <= K;
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
    if (valid) {
      const uint4* src = reinterpret_cast<const uint4*>(x + r * ldx + k0);
      v0 = __ldg(src);
      v1 = __ldg(src + 1);
    }
    float f[16];
    const __nv_bfloat16* b0 = reinterpret_cast<const __nv_bfloat16*>(&v0);
    const __nv_bfloat16* b1 = reinterpret_cast<const __nv_bfloat16*>(&v1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      f[i] = __bfloat162float(b0[i]);
      f[8 + i] = __bfloat162float(b1[i]);
    }
    uint32_t p[2];
    const uint32_t sc = valid ? nvfp4_quant16(f, gs, p) : 0u;
    if (valid) *reinterpret_cast<uint2*>(codes + r * ldc + k0 / 2) = make_uint2(p[0], p[1]);
    uint32_t word = sc;
    word |= __shfl_down_sync(0xFFFFFFFFu, sc, 1) << 8;
    word |= __shfl_down_sync(0xFFFFFFFFu, sc, 2) << 16;
    word |= __shfl_down_sync(0xFFFFFFFFu, sc, 3) << 24;
    if ((lane & 3) == 0 && k0 < ncb * 64) *reinterpret_cast<uint32_t*>(sf + sf_atom_offset(r, k0 / 16, ncb)) = word;
  }
}

// ---- routing: softmax top-k, one warp per token -------------------------------------------------------------------
// Selection: k rounds of a warp arg-max with (value desc, expert index asc); weights softmax over the selected.
template <int EPL>
__global__ void moe_route_kernel(const float* __restrict__ logits, int64_t T, int E, int k, int32_t* __restrict__ ids,
                                 float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  float v[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    float x = e < E ? logits[t * E + e] : -INFINITY;
    if (x != x) x = -INFINITY;   // NaN never outranks a number
    v[j] = e < E ? x : -INFINITY;
  }
  uint32_t taken = 0;
  int my_id = -1;
  float my_val = 0.0f, top = 0.0f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((taken >> j) & 1u) && (v[j] > bv || (v[j] == bv && e < bi))) {
        bv = v[j];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == r) {
      my_id = bi;
      my_val = bv;
    }
    if (r == 0) top = bv;
  }
  const float p = lane < k ? expf(my_val - top) : 0.0f;
  // sum in rank order (lane 0 .. k-1), the same order on every call
  float s = 0.0f;
  for (int r = 0; r < k; ++r) s += __shfl_sync(0xFFFFFFFFu, p, r);
  if (lane < k) {
    ids[t * k + lane] = my_id;
    weights[t * k + lane] = p / s;
  }
}

// ---- routing: sigmoid scores + correction bias, grouped top-k (the DeepSeek-V3 rule), one warp per token -----------
// score[e] = sigmoid(logit[e]) (evaluated in double and rounded to fp32 once, so that the CPU restatement reproduces
// every bit); choice[e] = score[e] + bias[e] (fp32). With n_group > 1 the experts form n_group equal groups, a group's
// rank is the sum of its two largest choices, and only the topk_group best groups (ties: lower group) stay eligible.
// Selection: k rounds of a warp arg-max over the eligible choices with (value desc, expert index asc), slots in that
// rank order. Weights: the unbiased scores of the selected experts, divided by their sum (summed in rank order) and
// multiplied by `scale` (the routed scaling factor).
template <int EPL>
__global__ void moe_route_sigmoid_kernel(const float* __restrict__ logits, int64_t T, int E, int k,
                                         const float* __restrict__ bias, int n_group, int topk_group, float scale,
                                         int32_t* __restrict__ ids, float* __restrict__ weights) {
  extern __shared__ float choice_sh[];          // [warps][E] (only with n_group > 1)
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  float sc[EPL], v[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    sc[j] = 0.0f;
    v[j] = -INFINITY;
    if (e < E) {
      const float x = logits[t * E + e];
      if (x == x) {                              // NaN never outranks a number
        sc[j] = static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(x))));
        v[j] = __fadd_rn(sc[j], bias[e]);
      }
    }
  }
  if (n_group > 1) {
    float* ch = choice_sh + (threadIdx.x >> 5) * E;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (lane + 32 * j < E) ch[lane + 32 * j] = v[j];
    __syncwarp();
    const int gsize = E / n_group;
    float gscore = -INFINITY;
    if (lane < n_group) {
      float a = -INFINITY, b = -INFINITY;       // the group's two largest choices
      for (int i = 0; i < gsize; ++i) {
        const float c = ch[lane * gsize + i];
        if (c > a) {
          b = a;
          a = c;
        } else if (c > b) {
          b = c;
        }
      }
      gscore = __fadd_rn(a, b);
    }
    uint32_t keep = 0;
    for (int r = 0; r < topk_group; ++r) {
      float bv = (keep >> lane) & 1u ? -INFINITY : gscore;
      int bi = lane < n_group && !((keep >> lane) & 1u) ? lane : 0x7FFFFFFF;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi < 32) keep |= 1u << bi;
    }
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((keep >> (e / gsize)) & 1u)) v[j] = -INFINITY;
    }
  }
  uint32_t taken = 0;
  int my_id = -1;
  float my_w = 0.0f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    float bs = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((taken >> j) & 1u) && (v[j] > bv || (v[j] == bv && e < bi))) {
        bv = v[j];
        bi = e;
        bs = sc[j];
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
      const float os = __shfl_xor_sync(0xFFFFFFFFu, bs, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bs = os;
      }
    }
    if (bi < E && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == r) {
      my_id = bi < E ? bi : -1;
      my_w = bi < E ? bs : 0.0f;
    }
  }
  float sum = 0.0f;
  for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xFFFFFFFFu, my_w, r));
  if (lane < k) {
    ids[t * k + lane] = my_id;
    weights[t * k + lane] = __fmul_rn(__fdiv_rn(my_w, sum), scale);
  }
}

// ---- per-block expert masks and counts ------------------------------------------------------------------------------
__global__ void moe_count_kernel(const int32_t* __restrict__ ids, int64_t T, int E, int k, uint32_t* __restrict__ masks,
                                 int32_t* __restrict__ block_counts) {
  extern __shared__ uint32_t sm[];   // [E][kMaskWords]
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < E * kMaskWords; i += blockDim.x) sm[i] = 0u;
  __syncthreads();
  const int64_t t = (int64_t)b * kBlockTokens + threadIdx.x;
  if (t < T) {
    for (int j = 0; j < k; ++j) {
      const int e = ids[t * k + j];
      if (e >= 0 && e < E) atomicOr(&sm[e * kMaskWords + (threadIdx.x >> 5)], 1u << (threadIdx.x & 31));
    }
  }
  __syncthreads();
  uint32_t* gm = masks + (int64_t)b * E * kMaskWords;
  for (int i = threadIdx.x; i < E * kMaskWords; i += blockDim.x) gm[i] = sm[i];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < kMaskWords; ++w) c += __popc(sm[e * kMaskWords + w]);
    block_counts[(int64_t)b * E + e] = c;
  }
}

// ---- expert offsets, block bases, GEMM tile table (one block) ------------------------------------------------------
// With `mpairs`, also the CTA-pair table of the grouped GEMM: per expert ceil(tiles / 2) entries {expert, first row,
// rows of the first 128, rows of the next 128} (the second half may be 0 rows: the next expert's first tile), count
// in num_mtiles[1].
__global__ void moe_offsets_kernel(int64_t T, int E, int nblocks, int32_t* __restrict__ block_counts,
                                   int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                   int32_t* __restrict__ mtiles, int32_t* __restrict__ num_mtiles, int cap,
                                   int32_t* __restrict__ mpairs, int pair_cap, int32_t* status) {
  extern __shared__ int32_t sh[];     // [E + 1] padded sizes, then [E + 1] first pair per expert
  int32_t* psh = sh + (E + 1);
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    int run = 0;
    if (e < E) {
      // exclusive base of block b inside expert e; the counts of 16 blocks are loaded before any is overwritten, so
      // the loads overlap instead of each waiting for the previous store
      for (int b0 = 0; b0 < nblocks; b0 += 16) {
        int c[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) c[j] = b0 + j < nblocks ? block_counts[(int64_t)(b0 + j) * E + e] : 0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (b0 + j < nblocks) block_counts[(int64_t)(b0 + j) * E + e] = run;
          run += c[j];
        }
      }
    } else {
      run = static_cast<int>(T);                  // the shared expert takes every token
    }
    counts[e] = run;
    sh[e] = (run + 127) / 128 * 128;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, pacc = 0;
    for (int e = 0; e <= E; ++e) {
      const int p = sh[e];
      sh[e] = acc;
      offsets[e] = acc;
      acc += p;
      psh[e] = pacc;
      pacc += (p / 128 + 1) / 2;
    }
    offsets[E + 1] = acc;
    const int n = acc / 128;
    *num_mtiles = n;
    if (n > cap) raise_status(status, kErrCapacity);
    if (mpairs != nullptr) {
      num_mtiles[1] = pacc;
      if (pacc > pair_cap) raise_status(status, kErrCapacity);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    const int c = counts[e];
    const int base = sh[e];
    for (int i = 0; i * 128 < c; ++i) {
      const int tile = base / 128 + i;
      if (tile < cap) {
        int4 v = make_int4(e, base + 128 * i, min(128, c - 128 * i), 0);
        reinterpret_cast<int4*>(mtiles)[tile] = v;
      }
    }
    if (mpairs != nullptr) {
      for (int j = 0; j * 256 < c; ++j) {
        const int pair = psh[e] + j;
        if (pair < pair_cap)
          reinterpret_cast<int4*>(mpairs)[pair] =
              make_int4(e, base + 256 * j, min(128, c - 256 * j), max(0, min(128, c - 256 * j - 128)));
      }
    }
  }
}

// ---- permuted rows, the row map and the code rows of the token's k + 1 rows ----------------------------------------
// One warp per token: lanes 0..k-1 rank the token's routed slots, lane k takes the shared expert row; every row records
// its source token in row_src, and the warp copies the token's code row (16-byte vectors) into each destination row.
__global__ void moe_scatter_kernel(const int32_t* __restrict__ ids, int64_t T, int E, int k,
                                   const uint32_t* __restrict__ masks, const int32_t* __restrict__ block_base,
                                   const int32_t* __restrict__ offsets, int32_t* __restrict__ rows,
                                   int32_t* __restrict__ row_src, const uint8_t* __restrict__ xq, int64_t H,
                                   uint8_t* __restrict__ xq_perm) {
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int64_t row_bytes = H / 2;
  const int64_t b = t / kBlockTokens;
  const int i = static_cast<int>(t - b * kBlockTokens);
  int my_row = -1;
  if (lane < k) {
    const int e = ids[t * k + lane];
    const uint32_t* m = masks + (b * E + e) * kMaskWords;
    const int w = i >> 5;
    int rank = block_base[b * E + e];
    for (int q = 0; q < w; ++q) rank += __popc(m[q]);
    rank += __popc(m[w] & ((1u << (i & 31)) - 1u));
    my_row = offsets[e] + rank;
    rows[t * k + lane] = my_row;
  }
  if (lane == k) my_row = offsets[E] + static_cast<int>(t);   // shared expert
  if (lane <= k) row_src[my_row] = static_cast<int32_t>(t);
  const uint4* src = reinterpret_cast<const uint4*>(xq + t * row_bytes);
  const int nvec = static_cast<int>(row_bytes / 16);
  constexpr int kVecPerLane = 8;                               // up to H = 8192 in registers
  uint4 reg[kVecPerLane];
#pragma unroll
  for (int j = 0; j < kVecPerLane; ++j)
    if (lane + 32 * j < nvec) reg[j] = __ldg(src + lane + 32 * j);
  for (int d = 0; d <= k; ++d) {
    const int64_t dst_row = __shfl_sync(0xFFFFFFFFu, my_row, d);
    uint4* dst = reinterpret_cast<uint4*>(xq_perm + dst_row * row_bytes);
#pragma unroll
    for (int j = 0; j < kVecPerLane; ++j)
      if (lane + 32 * j < nvec) dst[lane + 32 * j] = reg[j];
    for (int v = lane + 32 * kVecPerLane; v < nvec; v += 32) dst[v] = src[v];
  }
}

// ---- permuted scale atoms, gathered: one thread per 16-byte atom line -------------------------------------------------
// Atom (row block rb, column c) line l holds the words of rows 128 rb + l + 32 q, q = 0..3; the thread reads those four
// rows' source-token words (token order, L2-resident) and writes the line, so a warp writes one whole 512-byte atom.
// Rows past the tile's valid rows (the expert's padding) get zeros.
__global__ void moe_sf_gather_kernel(const int32_t* __restrict__ row_src, const int32_t* __restrict__ mtiles,
                                     const int32_t* __restrict__ num_mtiles, int cap, const uint8_t* __restrict__ xsf,
                                     int64_t ncb, uint8_t* __restrict__ xsf_perm) {
  const int64_t rb = blockIdx.x;
  if (rb >= min(*num_mtiles, cap)) return;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= ncb) return;
  const int l = threadIdx.x & 31;
  const int valid = mtiles[rb * 4 + 2];
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int r = l + 32 * q;
    w[q] = r < valid ? *reinterpret_cast<const uint32_t*>(xsf + sf_atom_offset(row_src[rb * 128 + r], c * 4, ncb)) : 0u;
  }
  *reinterpret_cast<uint4*>(xsf_perm + (rb * ncb + c) * 512 + l * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

// ---- weighted combine: out[t] = (x[t]) + sum_j w[t, j] y[rows[t, j]] + y[shared row of t], fp32 accumulate -----
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int64_t H, const int32_t* __restrict__ rows,
                                   const float* __restrict__ weights, const int32_t* __restrict__ offsets, int64_t T,
                                   int E, int k, const __nv_bfloat16* __restrict__ residual,
                                   __nv_bfloat16* __restrict__ out) {
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  const int64_t srow = offsets[E] + t;
  const int nvec = static_cast<int>(H / 8);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[8];
    if (residual != nullptr) {
      const uint4 q = reinterpret_cast<const uint4*>(residual + t * H)[v];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __bfloat162float(b[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    }
    for (int j = 0; j < k; ++j) {
      const int64_t r = rows[t * k + j];
      const float w = weights[t * k + j];
      const uint4 q = reinterpret_cast<const uint4*>(y + r * H)[v];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, __bfloat162float(b[i]), acc[i]);
    }
    const uint4 q = reinterpret_cast<const uint4*>(y + srow * H)[v];
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&q);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 p = __floats2bfloat162_rn(acc[2 * i] + __bfloat162float(b[2 * i]),
                                               acc[2 * i + 1] + __bfloat162float(b[2 * i + 1]));
      o[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    reinterpret_cast<uint4*>(out + t * H)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The same combine with the top-k width known at compile time: each thread reads its token's K rows and weights once,
// then issues the K + 1 row loads of a vector together before any arithmetic (K + 1 16-byte loads in flight per
// thread instead of one at a time); the register cap keeps two 512-thread blocks per SM. Same fma order as
// moe_combine_kernel, so the same bits.
template <int K>
__global__ void __launch_bounds__(512, 2)
moe_combine_k_kernel(const __nv_bfloat16* __restrict__ y, int64_t H, const int32_t* __restrict__ rows,
                     const float* __restrict__ weights, const int32_t* __restrict__ offsets, int64_t T, int E,
                     const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out) {
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  const int64_t srow = offsets[E] + t;
  int64_t r[K];
  float w[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    r[j] = rows[t * K + j];
    w[j] = weights[t * K + j];
  }
  const int nvec = static_cast<int>(H / 8);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 q[K + 1];
#pragma unroll
    for (int j = 0; j < K; ++j) q[j] = __ldg(reinterpret_cast<const uint4*>(y + r[j] * H) + v);
    q[K] = __ldg(reinterpret_cast<const uint4*>(y + srow * H) + v);
    float acc[8];
    if (residual != nullptr) {
      const uint4 rq = reinterpret_cast<const uint4*>(residual + t * H)[v];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&rq);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __bfloat162float(b[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&q[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w[j], __bfloat162float(b[i]), acc[i]);
    }
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&q[K]);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 p = __floats2bfloat162_rn(acc[2 * i] + __bfloat162float(b[2 * i]),
                                               acc[2 * i + 1] + __bfloat162float(b[2 * i + 1]));
      o[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    reinterpret_cast<uint4*>(out + t * H)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t sms = device_sm_count();
  int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = sms * 16;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

int last_error() { return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda; }

}  // namespace

int launch_nvfp4_quantize(const void* x, int64_t rows, int64_t K, int64_t ldx, float gs, uint8_t* codes, int64_t ldc,
                          uint8_t* sf, cudaStream_t stream) {
  if (K <= 0 || K % 16 != 0 || ldx % 8 != 0 || ldc % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(codes) & 7) || (reinterpret_cast<uintptr_t>(sf) & 3))
    return kErrArgs;
  if (rows == 0) return kOk;
  const int64_t ncb = sf_atom_cols(K);
  const int threads = 256;
  nvfp4_quantize_kernel<<<grid_for(rows * ((K + 511) / 512) * 32, threads), threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), rows, K, ldx, gs, codes, ldc, sf, ncb);
  return last_error();
}

int launch_moe_route(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids, float* weights,
                     cudaStream_t stream) {
  if (E <= 0 || E > 512 || k <= 0 || k > 32 || k > E) return kErrArgs;
  if (T == 0) return kOk;
  const int threads = 256;
  const int64_t blocks = (T + 7) / 8;
  const int epl = (E + 31) / 32;
  if (epl <= 4)
    moe_route_kernel<4><<<blocks, threads, 0, stream>>>(logits, T, E, k, ids, weights);
  else if (epl <= 8)
    moe_route_kernel<8><<<blocks, threads, 0, stream>>>(logits, T, E, k, ids, weights);
  else
    moe_route_kernel<16><<<blocks, threads, 0, stream>>>(logits, T, E, k, ids, weights);
  return last_error();
}

int launch_moe_route_sigmoid(const float* logits, int64_t T, int32_t E, int32_t k, const float* bias, int32_t n_group,
                             int32_t topk_group, float scale, int32_t* ids, float* weights, cudaStream_t stream) {
  if (E <= 0 || E > 512 || k <= 0 || k > 32 || k > E || bias == nullptr) return kErrArgs;
  if (n_group < 1 || n_group > 32 || E % n_group != 0 || topk_group < 1 || topk_group > n_group) return kErrArgs;
  if (n_group > 1 && (E / n_group < 2 || (E / n_group) * topk_group < k)) return kErrArgs;
  if (T == 0) return kOk;
  const int threads = 256;
  const int64_t blocks = (T + 7) / 8;
  const size_t sm = n_group > 1 ? static_cast<size_t>(threads / 32) * E * 4 : 0;
  const int epl = (E + 31) / 32;
  if (epl <= 4)
    moe_route_sigmoid_kernel<4><<<blocks, threads, sm, stream>>>(logits, T, E, k, bias, n_group, topk_group, scale, ids,
                                                                 weights);
  else if (epl <= 8)
    moe_route_sigmoid_kernel<8><<<blocks, threads, sm, stream>>>(logits, T, E, k, bias, n_group, topk_group, scale, ids,
                                                                 weights);
  else
    moe_route_sigmoid_kernel<16><<<blocks, threads, sm, stream>>>(logits, T, E, k, bias, n_group, topk_group, scale,
                                                                  ids, weights);
  return last_error();
}

int launch_moe_count(const int32_t* ids, int64_t T, int32_t E, int32_t k, uint32_t* masks, int32_t* block_counts,
                     cudaStream_t stream) {
  if (T == 0) return kOk;
  const int nblocks = static_cast<int>((T + kBlockTokens - 1) / kBlockTokens);
  const size_t sm = static_cast<size_t>(E) * kMaskWords * 4;
  moe_count_kernel<<<nblocks, kBlockTokens, sm, stream>>>(ids, T, E, k, masks, block_counts);
  return last_error();
}

int launch_moe_offsets(int64_t T, int32_t E, int32_t* block_counts, int32_t* counts, int32_t* offsets,
                       int32_t* mtiles, int32_t* num_mtiles, int32_t mtile_cap, int32_t* mpairs, int32_t mpair_cap,
                       int32_t* status, cudaStream_t stream) {
  const int nblocks = static_cast<int>((T + kBlockTokens - 1) / kBlockTokens);
  moe_offsets_kernel<<<1, 512, (E + 1) * 8, stream>>>(T, E, nblocks, block_counts, counts, offsets, mtiles,
                                                      num_mtiles, mtile_cap, mpairs, mpair_cap, status);
  return last_error();
}

int launch_moe_scatter(const int32_t* ids, int64_t T, int32_t E, int32_t k, const uint32_t* masks,
                       const int32_t* block_base, const int32_t* offsets, int32_t* rows, int32_t* row_src,
                       const uint8_t* xq, int64_t H, uint8_t* xq_perm, cudaStream_t stream) {
  if (k >= 32 || H % 32 != 0) return kErrArgs;
  if (T == 0) return kOk;
  const int64_t blocks = (T + 7) / 8;   // 8 warps per block, one token per warp
  moe_scatter_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(ids, T, E, k, masks, block_base, offsets, rows,
                                                                        row_src, xq, H, xq_perm);
  return last_error();
}

int launch_moe_sf_gather(const int32_t* row_src, const int32_t* mtiles, const int32_t* num_mtiles, int32_t mtile_cap,
                         const uint8_t* xsf, int64_t H, uint8_t* xsf_perm, cudaStream_t stream) {
  if (H % 64 != 0 || mtile_cap <= 0) return kErrArgs;
  const int64_t ncb = sf_atom_cols(H);
  const dim3 grid(static_cast<unsigned>(mtile_cap), static_cast<unsigned>((ncb + 7) / 8));
  moe_sf_gather_kernel<<<grid, 256, 0, stream>>>(row_src, mtiles, num_mtiles, mtile_cap, xsf, ncb, xsf_perm);
  return last_error();
}

int launch_moe_combine(const void* y, int64_t H, const int32_t* rows, const float* weights, const int32_t* offsets,
                       int64_t T, int32_t E, int32_t k, const void* residual, void* out, cudaStream_t stream) {
  if (H % 8 != 0) return kErrArgs;
  if (T == 0) return kOk;
  const int threads = H / 8 >= 512 ? 512 : static_cast<int>((H / 8 + 31) / 32 * 32);
  if (k == 8) {
    moe_combine_k_kernel<8><<<static_cast<unsigned>(T), threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(y), H, rows, weights, offsets, T, E,
        reinterpret_cast<const __nv_bfloat16*>(residual), reinterpret_cast<__nv_bfloat16*>(out));
    return last_error();
  }
  moe_combine_kernel<<<static_cast<unsigned>(T), threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(y), H, rows, weights, offsets, T, E, k,
      reinterpret_cast<const __nv_bfloat16*>(residual), reinterpret_cast<__nv_bfloat16*>(out));
  return last_error();
}

}  // namespace ssb
