// Sparse MLA prefill for sm_100a (absorbed-latent attention of one DSA layer) and the latent-cache append.
//
//   out[t, h, :] = sum_j softmax_j(scale * q[t, h, :] . kv[s_j, :]) * kv[s_j, 0:512]      (h < 64 heads)
//
// over the row's selected tokens j (the indexer's expanded indices, -1 = none), each read from the paged latent cache
// (latent 512 + rope 64 per token, bf16 rows of 576) at slot = pages[pos / 128] * 128 + pos % 128 of the row's
// request. Reference: the TRTLLM sparse MLA called through `trtllm_batch_decode_with_kv_cache_mla` (ssengine/kernels.py
// config 25; split at 32,768 rows, ssengine/model/pp_patch.py:643-672).
//
// One CTA per query row, 16 warps: the row's 64 x 576 query stays in shared memory; the selected tokens stream in
// blocks of 32 gathered rows (cp.async 16-byte pieces, a 3-stage ring keeping two blocks in flight, missing tokens
// zero-filled): the kernel is bound by the latency of those gathers, so bytes in flight matter more than the tensor
// pipe. Per block: S = Q K^T (warp (head group, 8 tokens): 36 mma.sync m16n8k16 over 4 accumulators), an online
// softmax per head row (one warp per 4 rows, one token per lane, exp2 with the scale folded), O += P V (warp (head
// group, 128 latent columns): 32 mma);
// O stays in registers (64 fp32 per thread) until the row's last block, then is normalised and stored as bf16.
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kHeads = 64, kDq = 576, kDv = 512, kBlk = 32;
constexpr int kMlaThreads = 512;
constexpr int kRowBytes = kDq * 2;                       // 1152
constexpr int kChunks = kRowBytes / 16;                  // 72 16-byte chunks per row
constexpr int kQBytes = kHeads * kRowBytes;              // 73728
constexpr int kKvBytes = kBlk * kRowBytes;               // 36864
constexpr int kOffQ = 0;
constexpr int kStagesKv = 3;                             // gather ring: two blocks in flight while one is used
constexpr int kOffKv = kQBytes;
constexpr int kOffS = kOffKv + kStagesKv * kKvBytes;     // fp32 [64][33] scores
constexpr int kOffP = kOffS + kHeads * 33 * 4;           // bf16 [64][32] (swizzled, 64-byte rows)
constexpr int kOffAlpha = kOffP + kHeads * kBlk * 2;     // fp32 [64]
constexpr int kOffL = kOffAlpha + kHeads * 4;            // fp32 [64]
constexpr int kMlaSmem = kOffL + kHeads * 4;

// [rows][576] bf16 with the 16-byte chunk index XOR-ed by (row & 7) (72 chunks = 9 groups of 8)
SSB_DEVICE int swq(int r, int c) { return r * kDq + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }
// [64][32] bf16: 4 chunks per row, XOR by ((row >> 1) & 3) so 8 rows of one ldmatrix hit distinct banks
SSB_DEVICE int swp(int r, int c) { return r * kBlk + ((((c >> 3) ^ ((r >> 1) & 3))) << 3) + (c & 7); }

SSB_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
SSB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SSB_DEVICE void cp_async_wait2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }
SSB_DEVICE void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

SSB_DEVICE void ldsm4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
SSB_DEVICE void ldsm2(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
SSB_DEVICE void ldsm4t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
SSB_DEVICE void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Gather block b's 32 token rows into buffer `buf` (token slot -1 -> zeros).
SSB_DEVICE void gather_block(uint8_t* smem, int buf, const __nv_bfloat16* kv, const int64_t* slot_of, int tid) {
  const uint32_t base = smem_u32(smem + kOffKv + buf * kKvBytes);
  for (int c = tid; c < kBlk * kChunks; c += kMlaThreads) {
    const int r = c / kChunks, ch = c - r * kChunks;
    const int64_t slot = slot_of[r];
    const int sch = (ch & ~7) | ((ch & 7) ^ (r & 7));
    cp_async16(base + r * kRowBytes + sch * 16, kv + (slot >= 0 ? slot : 0) * kDq + ch * 8, slot >= 0);
  }
}

__global__ void __launch_bounds__(kMlaThreads, 1) sparse_mla_kernel(MlaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int64_t slots[kStagesKv][kBlk];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int64_t t = blockIdx.x;
  const __nv_bfloat16* Q = reinterpret_cast<const __nv_bfloat16*>(smem + kOffQ);
  float* S = reinterpret_cast<float*>(smem + kOffS);
  __nv_bfloat16* Pm = reinterpret_cast<__nv_bfloat16*>(smem + kOffP);
  float* ALPHA = reinterpret_cast<float*>(smem + kOffAlpha);
  float* LSUM = reinterpret_cast<float*>(smem + kOffL);

  // the row's request (binary search of the query start list) and its pages
  int lo = 0, hi = a.R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.qsl[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int32_t* pages = a.table + (int64_t)lo * a.width;
  const int32_t* idx = a.indices + t * a.ld_idx;
  const int nblk = (a.n_idx + kBlk - 1) / kBlk;

  auto fill_slots = [&](int b, int buf) {
    if (tid < kBlk) {
      const int j = b * kBlk + tid;
      int64_t s = -1;
      if (j < a.n_idx) {
        const int32_t pos = idx[j];
        if (pos >= 0 && (pos >> 7) < a.width) {
          const int32_t pg = pages[pos >> 7];
          if (pg >= 0) s = (int64_t)pg * 128 + (pos & 127);
        }
      }
      slots[buf][tid] = s;
    }
  };

  // Q -> shared (swizzled), block 0's slots
  {
    const __nv_bfloat16* qrow = a.q + t * (int64_t)kHeads * kDq;
    const uint32_t qb = smem_u32(smem + kOffQ);
    for (int c = tid; c < kHeads * kChunks; c += kMlaThreads) {
      const int r = c / kChunks, ch = c - r * kChunks;
      const int sch = (ch & ~7) | ((ch & 7) ^ (r & 7));
      cp_async16(qb + r * kRowBytes + sch * 16, qrow + r * kDq + ch * 8, true);
    }
    fill_slots(0, 0);
  }
  if (nblk > 1) fill_slots(1, 1);
  __syncthreads();
  if (nblk > 0) gather_block(smem, 0, a.kv, slots[0], tid);
  cp_async_commit();                       // group: Q + block 0
  if (nblk > 1) gather_block(smem, 1, a.kv, slots[1], tid);
  cp_async_commit();                       // group: block 1

  const int rg = warp & 3;                 // head rows 16 rg .. 16 rg + 15
  const int cg = warp >> 2;                // S: tokens 8 cg .. 8 cg + 7 of the block; PV: latent columns 128 cg ..
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[4], l_run[4];                // softmax state of rows 4 warp .. 4 warp + 3 (lane-uniform)
#pragma unroll
  for (int i = 0; i < 4; ++i) { m_run[i] = -INFINITY; l_run[i] = 0.0f; }
  const float sc = a.scale * 1.4426950408889634f;    // exp2 domain

  for (int b = 0; b < nblk; ++b) {
    const int buf = b % kStagesKv;
    if (b + 2 < nblk) {                    // stage (b + 2) % 3 held block b - 1, finished last iteration
      const int nb = (b + 2) % kStagesKv;
      fill_slots(b + 2, nb);
      __syncthreads();
      gather_block(smem, nb, a.kv, slots[nb], tid);
    }
    cp_async_commit();
    cp_async_wait2();                      // block b (and Q) landed
    __syncthreads();
    const __nv_bfloat16* KV = reinterpret_cast<const __nv_bfloat16*>(smem + kOffKv + buf * kKvBytes);

    // ---- S = Q K^T for head rows 16 rg.., tokens 8 cg.. (4 accumulators over the 36 k-steps) ----
    {
      float s4[4][4] = {};
#pragma unroll
      for (int ks = 0; ks < kDq / 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1;
        ldsm4(Q + swq(16 * rg + (lane & 15), 16 * ks + (lane >> 4) * 8), a0, a1, a2, a3);
        ldsm2(KV + swq(8 * cg + (lane & 7), 16 * ks + ((lane >> 3) & 1) * 8), b0, b1);
        mma_bf16(s4[ks & 3], a0, a1, a2, a3, b0, b1);
      }
      const int j0 = 8 * cg + 2 * t4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = 16 * rg + g8 + 8 * (q >> 1);
        S[row * 33 + j0 + (q & 1)] = s4[0][q] + s4[1][q] + s4[2][q] + s4[3][q];
      }
    }
    __syncthreads();

    // ---- online softmax: warp w owns rows 4w .. 4w+3, lane = token ----
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = 4 * warp + i;
      const float x = slots[buf][lane] >= 0 ? S[row * 33 + lane] * sc : -INFINITY;
      float mb = x;
#pragma unroll
      for (int off = 16; off; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      const float m_new = fmaxf(m_run[i], mb);
      const float p = (m_new == -INFINITY) ? 0.0f : exp2f(x - m_new);
      float ps = p;
#pragma unroll
      for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      const float alpha = (m_run[i] == -INFINITY) ? 0.0f : exp2f(m_run[i] - m_new);
      l_run[i] = l_run[i] * alpha + ps;
      m_run[i] = m_new;
      Pm[swp(row, lane)] = __float2bfloat16_rn(p);
      if (lane == 0) ALPHA[row] = alpha;
    }
    __syncthreads();

    // ---- O = alpha O + P V for head rows 16 rg.., latent columns 128 cg .. ----
    {
      const float al = ALPHA[16 * rg + g8], ah = ALPHA[16 * rg + g8 + 8];
#pragma unroll
      for (int i = 0; i < 16; ++i) { o[i][0] *= al; o[i][1] *= al; o[i][2] *= ah; o[i][3] *= ah; }
#pragma unroll
      for (int ks = 0; ks < kBlk / 16; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm4(Pm + swp(16 * rg + (lane & 15), 16 * ks + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm4t(KV + swq(16 * ks + (lane & 7) + ((lane >> 3) & 1) * 8, 128 * cg + 16 * p + (lane >> 4) * 8), b0, b1, b2,
                 b3);
          mma_bf16(o[2 * p], a0, a1, a2, a3, b0, b1);
          mma_bf16(o[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();                       // buffer `buf`, S and P are reused by the next block
  }
  cp_async_wait0();

  // ---- normalise and store ----
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) LSUM[4 * warp + i] = l_run[i];
  }
  __syncthreads();
  const float ll = LSUM[16 * rg + g8], lh = LSUM[16 * rg + g8 + 8];
  const float il = ll > 0.0f ? 1.0f / ll : 0.0f, ih = lh > 0.0f ? 1.0f / lh : 0.0f;
  __nv_bfloat16* orow = a.out + t * (int64_t)kHeads * kDv;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 128 * cg + 8 * i + 2 * t4;
    *reinterpret_cast<__nv_bfloat162*>(orow + (16 * rg + g8) * kDv + c) = __floats2bfloat162_rn(o[i][0] * il, o[i][1] * il);
    *reinterpret_cast<__nv_bfloat162*>(orow + (16 * rg + g8 + 8) * kDv + c) =
        __floats2bfloat162_rn(o[i][2] * ih, o[i][3] * ih);
  }
}

// Latent cache append: row t of src (bf16 [T, 576], row pitch lds) -> cache row slots[t] (skipped when < 0).
__global__ void mla_append_kernel(const __nv_bfloat16* src, int64_t lds, const int64_t* slots, int64_t T,
                                  __nv_bfloat16* cache) {
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  const int64_t s = slots[t];
  if (s < 0) return;
  for (int c = threadIdx.x; c < kChunks; c += blockDim.x)
    reinterpret_cast<uint4*>(cache + s * kDq)[c] = reinterpret_cast<const uint4*>(src + t * lds)[c];
}

}  // namespace

int launch_sparse_mla(const MlaArgs& a, cudaStream_t stream) {
  if (a.q == nullptr || a.kv == nullptr || a.indices == nullptr || a.qsl == nullptr || a.table == nullptr ||
      a.out == nullptr || a.T < 0 || a.R <= 0 || a.width <= 0 || a.n_idx < 0 || a.ld_idx < a.n_idx ||
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.kv) | reinterpret_cast<uintptr_t>(a.out)) &
       15))
    return kErrArgs;
  if (a.T == 0) return kOk;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(sparse_mla_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlaSmem) != cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  sparse_mla_kernel<<<(unsigned)a.T, kMlaThreads, kMlaSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_mla_append(const void* src, int64_t lds, const int64_t* slots, int64_t T, void* cache,
                      cudaStream_t stream) {
  if (src == nullptr || slots == nullptr || cache == nullptr || T < 0 || lds < kDq || (lds % 8) ||
      ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(cache)) & 15))
    return kErrArgs;
  if (T == 0) return kOk;
  mla_append_kernel<<<(unsigned)T, 96, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), lds, slots, T,
                                                    static_cast<__nv_bfloat16*>(cache));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
