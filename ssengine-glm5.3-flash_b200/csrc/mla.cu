// Sparse MLA prefill for sm_100a (absorbed-latent attention of one DSA layer) and the latent-cache append.
//
//   out[t, h, :] = sum_j softmax_j(scale * q[t, h, :] . kv[s_j, :]) * kv[s_j, 0:512]      (h < 64 heads)
//
// over the row's selected tokens j (the indexer's expanded indices, -1 = none), each read from the paged latent cache
// (latent 512 + rope 64 per token, bf16 rows of 576) at slot = pages[pos / 128] * 128 + pos % 128 of the row's
// request. Reference: the TRTLLM sparse MLA called through `trtllm_batch_decode_with_kv_cache_mla` (ssengine/kernels.py
// config 25; split at 32,768 rows, ssengine/model/pp_patch.py:643-672).
//
// One CTA (4 warps) per query row; tcgen05 with the 64 heads as M = 64 (accumulator rows in lanes 0-15 of each
// 32-lane sub-partition; a second M = 64 accumulator sits in lanes 16-31 of the same columns):
//   Q [64 x 576] bf16 stays in shared memory (TMA, 9 K-major 128-byte-swizzled chunks);
//   the index columns are taken in blocks of 64; blocks without a selected token are skipped (listed up front), so a
//   row near its request's start costs its own tokens, not the full top-k width;
//   per block, the selected tokens' rows are gathered by cp.async into 9 chunks [64 tokens x 64 dims] with the same
//   swizzle (missing tokens zero-filled without a read), double-buffered (block b+1 lands while block b is used);
//   S [64 x 64] = Q K^T as two N = 32 halves (tokens 0-31 in lanes 0-15, 32-63 in lanes 16-31 of columns 0-31;
//   2 x 36 MMAs kind::f16); softmax by all 128 threads (a head row's two halves combine max and sum with a shuffle;
//   exp2, scale folded) with the running max kept stale until a block raises it by more than 2^8, so the accumulator
//   is rescaled in TMEM only then;
//   P [64 x 64] bf16 to shared memory (K-major); O += P V with V = the same chunks read MN-major: O columns 256-511,
//   latent dims 0-255 in lanes 0-15 and dims 256-511 in lanes 16-31 (2 x 4 MMAs of N = 256 per block).
// Bounded waits; on expiry the status word holds kErrTimeout, in-flight MMAs are drained and TMEM is freed.
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kHeads = 64, kDq = 576, kDv = 512, kBlk = 64;
constexpr int kMlaThreads = 128;
constexpr int kChunk = kBlk * 128;                       // [64 rows x 64 bf16], 8 KB
constexpr int kNChunks = kDq / 64;                       // 9
constexpr int kQBytes = kNChunks * kChunk;               // 73728
constexpr int kKvBytes = kNChunks * kChunk;              // 73728 per block buffer
constexpr int kOffQ = 0;
constexpr int kOffKv = kQBytes;                          // 2 buffers
constexpr int kOffP = kOffKv + 2 * kKvBytes;             // P [64 x 64] bf16, K-major swizzled
constexpr int kOffSlots = kOffP + kChunk;                // int64 [2][64]
constexpr int kOffBar = kOffSlots + 2 * kBlk * 8;        // bar_q, bar_s, bar_pv, bar_drain
constexpr int kOffMisc = kOffBar + 32;                   // tmem slot, abort flag, block count
constexpr int kMaxBlocks = 256;                          // n_idx <= 16384
constexpr int kOffMask = kOffMisc + 16;                  // uint64 [4]: blocks holding a selected token
constexpr int kOffList = kOffMask + 32;                  // uint16 [256]: those blocks in order
constexpr int kMlaSmem = kOffList + 2 * kMaxBlocks + 1024;   // + alignment slack
constexpr uint32_t kSCol = 0, kOCol = 256;

SSB_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
SSB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SSB_DEVICE void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

SSB_DEVICE void drain_bar(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) break;
  }
}

// Block b's 64 token rows -> the 9 chunks of a buffer (a missing token is zero-filled without a read; its score is
// masked): thread t copies half (t & 1) of row t >> 1, four 16-byte pieces per chunk, offsets fixed at compile time.
SSB_DEVICE void gather_block(uint32_t kvb, const __nv_bfloat16* kv, const int64_t* slot_of, int tid) {
  const int r = tid >> 1, hi = tid & 1;
  const int64_t slot = slot_of[r];
  const bool valid = slot >= 0;
  const __nv_bfloat16* src = kv + (valid ? slot : 0) * kDq + hi * 32;
  const uint32_t dst = kvb + r * 128;
  const int sw = r & 7;
#pragma unroll
  for (int ch = 0; ch < kNChunks; ++ch)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = 4 * hi + jj;
      cp_async16(dst + ch * kChunk + ((j ^ sw) << 4), src + ch * 64 + jj * 8, valid);
    }
}

__global__ void __launch_bounds__(kMlaThreads, 1)
    sparse_mla_kernel(const __grid_constant__ CUtensorMap mq, const MlaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t = blockIdx.x;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_q = sbase + kOffBar, bar_s = bar_q + 8, bar_pv = bar_q + 16, bar_drain = bar_q + 24;
  int64_t* slots = reinterpret_cast<int64_t*>(smem + kOffSlots);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + kOffMisc + 4);
  uint8_t* Pb = smem + kOffP;

  // the row's request (binary search of the query start list) and its pages
  int lo = 0, hi = a.R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.qsl[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int32_t* pages = a.table + (int64_t)lo * a.width;
  const int32_t* idx = a.indices + t * a.ld_idx;
  unsigned long long* mask = reinterpret_cast<unsigned long long*>(smem + kOffMask);
  uint16_t* blist = reinterpret_cast<uint16_t*>(smem + kOffList);
  volatile int32_t* nblk_s = reinterpret_cast<volatile int32_t*>(smem + kOffMisc + 8);
  auto slot_at = [&](int j) -> int64_t {
    const int32_t pos = idx[j];
    if (pos >= 0 && (pos >> 7) < a.width) {
      const int32_t pg = pages[pos >> 7];
      if (pg >= 0) return (int64_t)pg * 128 + (pos & 127);
    }
    return -1;
  };
  // list entry i (the i-th block of 64 index columns that holds a selected token) -> slot buffer (i & 1)
  auto fill_slots = [&](int i) {
    if (tid < kBlk) {
      const int j = blist[i] * kBlk + tid;
      slots[(i & 1) * kBlk + tid] = j < a.n_idx ? slot_at(j) : -1;
    }
  };

  if (tid == 0) {                                       // Q lands while the index columns are scanned
    mbar_init(bar_q, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_pv, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar_q, kQBytes);
    for (int c = 0; c < kNChunks; ++c) tma_load_2d(sbase + kOffQ + c * kChunk, &mq, 64 * c, (int32_t)(t * kHeads), bar_q);
  }
  // blocks of index columns without a selected token are skipped: mark the others, then list them in order
  if (tid < 4) mask[tid] = 0ull;
  __syncthreads();
  for (int j = tid; j < a.n_idx; j += kMlaThreads)
    if (slot_at(j) >= 0) atomicOr(mask + (j >> 12), 1ull << ((j >> 6) & 63));
  __syncthreads();
  if (tid == 0) {
    int n = 0;
    for (int w = 0; w < 4; ++w)
      for (unsigned long long m = mask[w]; m; m &= m - 1) blist[n++] = static_cast<uint16_t>(64 * w + __ffsll(m) - 1);
    *nblk_s = n;
  }
  __syncthreads();
  const int nblk = *nblk_s;

  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (nblk > 0) fill_slots(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (nblk > 0) gather_block(sbase + kOffKv, a.kv, slots, tid);
  cp_async_commit();

  constexpr uint32_t idesc_s = idesc_bf16(64, 32);                     // tokens 0-31 -> lanes 0-15, 32-63 -> 16-31
  constexpr uint32_t idesc_pv = idesc_bf16(64, 256) | (1u << 16);      // B (V) MN-major
  const float sc = a.scale * 1.4426950408889634f;                        // exp2 domain
  const uint32_t tq = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float m_used = -INFINITY, l_sum = 0.0f;
  bool ok = true, any_mma = false;

  for (int b = 0; b < nblk && ok; ++b) {
    const int kb = b & 1;
    const uint32_t kvb = sbase + kOffKv + kb * kKvBytes;
    cp_async_wait0();                                    // block b landed (this thread's pieces)
    fence_proxy_async_smem();                            // generic-proxy writes -> visible to the tensor core
    __syncthreads();
    if (tid == 0) {
      if (b == 0) mbar_wait(bar_q, 0, abort_flag, a.status);
      if (!*abort_flag) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kNChunks; ++c) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = smem_desc(sbase + kOffQ + c * kChunk + ks * 32, 0, 1024, 2);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint64_t bd = smem_desc(kvb + c * kChunk + hh * 4096 + ks * 32, 0, 1024, 2);
              tc_mma_f16(tmem + (static_cast<uint32_t>(16 * hh) << 16) + kSCol, ad, bd, idesc_s, (c | ks) != 0 ? 1u : 0u);
            }
          }
        }
        any_mma = true;
        tc_commit(bar_s);
      }
    }
    // PV of block b-1 done: its KV buffer, P and O are free / stable; gather block b+1 into that buffer
    if (b >= 1) mbar_wait(bar_pv, (b - 1) & 1, abort_flag, a.status);
    if (b + 1 < nblk) fill_slots(b + 1);
    __syncthreads();
    if (*abort_flag) { ok = false; break; }
    if (b + 1 < nblk) gather_block(sbase + kOffKv + (kb ^ 1) * kKvBytes, a.kv, slots + (kb ^ 1) * kBlk, tid);
    cp_async_commit();
    mbar_wait(bar_s, b & 1, abort_flag, a.status);      // a timeout raises the abort flag, checked after the next barrier
    tc_fence_after();

    // ---- softmax: lane l holds row 16 warp + (l & 15), tokens 32 (l >> 4) .. + 31; the two halves of a row combine
    //      their max and sum with one shuffle and keep identical running state ----
    float v[32];
    tmem_ld_32x32b_x32(tq + kSCol, v);
    tmem_ld_wait();
    const int half = lane >> 4;
    float alpha = 1.0f;
    bool rescale = false;
    {
      const int64_t* sl = slots + kb * kBlk + 32 * half;
      float mb = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = sl[j] >= 0 ? v[j] * sc : -INFINITY;
        mb = fmaxf(mb, v[j]);
      }
      mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 16));
      if (m_used == -INFINITY) {
        m_used = mb;                                     // nothing accumulated yet (O = 0, l = 0)
      } else if (mb > m_used + 8.0f) {
        alpha = exp2f(m_used - mb);
        m_used = mb;
        l_sum *= alpha;
        rescale = true;
      }
      const int row = 16 * warp + (lane & 15);
      float ps = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = (m_used == -INFINITY) ? 0.0f : exp2f(v[8 * c + e] - m_used);
          ps += p[e];
        }
        uint4 pk;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(p[2 * e], p[2 * e + 1]);
          pw[e] = *reinterpret_cast<uint32_t*>(&h2);
        }
        const int chunk = 4 * half + c;
        *reinterpret_cast<uint4*>(Pb + row * 128 + ((chunk ^ (row & 7)) << 4)) = pk;
      }
      l_sum += ps + __shfl_xor_sync(0xffffffffu, ps, 16);
    }
    // rescale O rows in TMEM when a row's max moved (warp-collective; lanes 0-15 hold dims 0-255, 16-31 dims 256-511)
    if (__any_sync(0xffffffffu, rescale) && b > 0) {
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        float o[32];
        tmem_ld_32x32b_x32(tq + kOCol + 32 * c, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= alpha;
        tmem_st_32x32b_x32(tq + kOCol + 32 * c, o);
      }
      tmem_st_wait();
    }
    fence_proxy_async_smem();                            // P (generic stores) -> visible to the tensor core
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) { ok = false; break; }
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ad = smem_desc(sbase + kOffP + ks * 32, 0, 1024, 2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint64_t bd = smem_desc(kvb + 4 * h * kChunk + ks * 2048, kChunk, 1024, 2);
          tc_mma_f16(tmem + (static_cast<uint32_t>(16 * h) << 16) + kOCol, ad, bd, idesc_pv,
                     (b > 0 || ks > 0) ? 1u : 0u);
        }
      }
      tc_commit(bar_pv);
    }
  }
  cp_async_wait0();

  // ---- normalise and store (lanes 0-15: dims 0-255 of row 16 warp + lane; lanes 16-31: dims 256-511) ----
  const bool have = ok && nblk > 0;
  if (have) mbar_wait(bar_pv, (nblk - 1) & 1, abort_flag, a.status);
  if (nblk == 0 && tid == 0) mbar_wait(bar_q, 0, abort_flag, a.status);   // no copy in flight at exit
  __syncthreads();
  if (*abort_flag) ok = false;
  tc_fence_after();
  const float inv = (ok && have && l_sum > 0.0f) ? 1.0f / l_sum : 0.0f;
  const int row = 16 * warp + (lane & 15);
  __nv_bfloat16* orow = a.out + (t * kHeads + row) * kDv + (lane >> 4) * 256;
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    float o[32];
    if (have && ok) {
      tmem_ld_32x32b_x32(tq + kOCol + 32 * c, o);
      tmem_ld_wait();
    }
    uint4 pk[4];
    uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float x0 = (have && ok) ? o[2 * e] * inv : 0.0f, x1 = (have && ok) ? o[2 * e + 1] * inv : 0.0f;
      __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
      pw[e] = *reinterpret_cast<uint32_t*>(&h2);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(orow + 32 * c)[e] = pk[e];
  }
  if (*abort_flag && any_mma && tid == 0) {
    tc_commit(bar_drain);
    drain_bar(bar_drain, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Latent cache append: row t of src (bf16 [T, 576], row pitch lds) -> cache row slots[t] (skipped when < 0).
__global__ void mla_append_kernel(const __nv_bfloat16* src, int64_t lds, const int64_t* slots, int64_t T,
                                  __nv_bfloat16* cache) {
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  const int64_t s = slots[t];
  if (s < 0) return;
  for (int c = threadIdx.x; c < kDq / 8; c += blockDim.x)
    reinterpret_cast<uint4*>(cache + s * kDq)[c] = reinterpret_cast<const uint4*>(src + t * lds)[c];
}

}  // namespace

int launch_sparse_mla(const MlaArgs& a, cudaStream_t stream) {
  if (a.q == nullptr || a.kv == nullptr || a.indices == nullptr || a.qsl == nullptr || a.table == nullptr ||
      a.out == nullptr || a.T < 0 || a.R <= 0 || a.width <= 0 || a.n_idx < 0 || a.n_idx > kMaxBlocks * kBlk ||
      a.ld_idx < a.n_idx ||
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.kv) | reinterpret_cast<uintptr_t>(a.out)) &
       15))
    return kErrArgs;
  if (a.T == 0) return kOk;
  CUtensorMap mq;
  const int rc = make_map_2d_swizzled(&mq, a.q, a.T * kHeads, kDq, kDq * 2, 64);
  if (rc != kOk) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(sparse_mla_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlaSmem) != cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  sparse_mla_kernel<<<(unsigned)a.T, kMlaThreads, kMlaSmem, stream>>>(mq, a);
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
