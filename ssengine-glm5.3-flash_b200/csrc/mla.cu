// Sparse MLA prefill for sm_100a (absorbed-latent attention of one DSA layer) over an FP8 latent cache, the cache
// append and the FP8 query pack.
//
//   out[t, h, :] = bmm2 * sum_j softmax_j(bmm1 * q8[t, h, :] . kv8[s_j, :]) * kv8[s_j, 0:512]      (h < 64 heads)
//
// over the row's selected tokens j (the indexer's expanded indices, -1 = none), each read from the paged latent cache
// (e4m3 rows of 576 bytes: latent 512 + rope 64) at slot = pages[pos / 128] * 128 + pos % 128 of the row's request.
// q8 = e4m3(q / q_scale), kv8 = e4m3(kv / k_scale), bmm1 = softmax scale * q_scale * k_scale, bmm2 = k_scale: the
// reference's FP8 query and cache (vLLM kv_cache_dtype fp8_e4m3, `concat_and_cache_mla`; TRTLLM sparse MLA with
// bmm1 / bmm2 scales: ssengine/kernels.py configs 23 and 25, ssengine/model/pp_patch.py:643-672).
//
// One CTA per query row, 352 threads. Up front, every index column (n_idx <= 2304) is resolved to its cache row in
// shared memory with all loads in flight; then three roles run over blocks of 128 index columns (blocks without a
// selected token skipped):
//   warps 5-10 gather: each block's 128 token rows by cp.async into 5 K-major 128-byte-swizzled chunks [128 x 128 B]
//            (the 5th holds the 64 rope bytes), two buffers; missing tokens zero-filled without a read; each
//            thread's arrive on the buffer's full barrier fires when its copies land (cp.async.mbarrier.arrive), so
//            the next block's copies are issued while the previous block's are in flight;
//   warp 4 issues the MMAs (one thread, kind::f8f6f4, M = 64 heads): S [64 x 128] = Q K^T as two N = 64 halves
//            (tokens 0-63 in lanes 0-15, 64-127 in lanes 16-31 of TMEM columns 0-63; 36 MMAs), then
//            O += P V with V the same chunks read MN-major (dims 0-255 in lanes 0-15, 256-511 in lanes 16-31 of
//            columns 256-511; 8 MMAs of N = 256);
//   warps 0-3 softmax: one head row half per thread (64 scores), base-2 weights, running max kept stale
//            until a block raises it by more than 2^3 (O rescaled in TMEM only then), so p <= 8 and 32 p fits e4m3
//            (448) with normals down to p = 2^-11; P to e4m3 (K-major, swizzled) for the PV MMA; then the epilogue
//            (O * bmm2 / (32 l) -> bf16).
// Each tcgen05.commit tracks every earlier MMA of the issuing thread, so "S of block i done" also means "PV of block
// i - 1 done": one S accumulator and one P buffer suffice, and O is stable whenever the softmax warps touch it.
// Bounded waits; on expiry the status word holds kErrTimeout, in-flight MMAs are drained and TMEM is freed.
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kHeads = 64, kDq = 576, kDv = 512, kBlk = 128;
constexpr int kMlaThreads = 352;                  // warps 0-3 softmax + epilogue, warp 4 MMA, warps 5-10 gather
constexpr int kGather = 192;                      // gather threads
constexpr int kPro = 256;                         // threads 0-255 load Q and resolve the index columns
constexpr int kNC = 5;                            // 128-byte chunks of a 576-byte row
constexpr int kQChunk = kHeads * 128;             // [64 heads x 128 B], 8 KB
constexpr int kKvChunk = kBlk * 128;              // [128 tokens x 128 B], 16 KB
constexpr int kKvBuf = kNC * kKvChunk;            // 80 KB
constexpr int kOffQ = 0;
constexpr int kOffKv = kNC * kQChunk;             // 2 buffers
constexpr int kOffP = kOffKv + 2 * kKvBuf;        // P [64 heads x 128 tokens] e4m3, K-major swizzled
constexpr int kMaxBlocks = 18;                    // n_idx <= 2304 (the reference selects 2,176)
constexpr int kMaxIdx = kMaxBlocks * kBlk;
constexpr int kOffSlots = kOffP + kHeads * 128;   // int32 [2304]: cache row of each index column (-1: none)
constexpr int kOffMask = kOffSlots + 4 * kMaxIdx; // uint32 [72] (read as uint64 [36]): selected columns
constexpr int kOffBar = kOffMask + 8 * 2 * kMaxBlocks;   // kv_full[2], kv_empty[2], s_full, p_full, o_done
constexpr int kOffMisc = kOffBar + 64;            // tmem slot, abort flag, block count
constexpr int kOffList = kOffMisc + 16;           // uint16 [18]: the blocks holding a selected column, in order
constexpr int kMlaSmem = kOffList + 2 * kMaxBlocks + 1024;   // + alignment slack
static_assert(kMlaSmem <= 232448, "shared memory");
constexpr uint32_t kSCol = 0, kOCol = 256;
constexpr float kLazy = 3.0f;                     // a block raising a row's max by more than 2^3 rescales O
constexpr float kPScale = 32.0f;                  // P stored as e4m3(32 p): p <= 2^3 over a stale max -> <= 256

SSB_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
SSB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// an arrive on `bar` (one of its expected arrivals) once this thread's earlier cp.async copies have landed
SSB_DEVICE void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
SSB_DEVICE void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Two floats -> two e4m3 bytes (round to nearest even, saturating to +-448): lo in the low byte.
SSB_DEVICE uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Softmax in base 2 with log2(e) folded into the score scale (the FlashAttention-2 formulation, Dao 2023): 2^x by
// the PTX ex2.approx.ftz instruction (flush-to-zero, a few ulp), ample for weights that are rounded to e4m3 next.
SSB_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

SSB_DEVICE void drain_bar(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) break;
  }
}

SSB_DEVICE void tmem_ld_x64(uint32_t taddr, float (&v)[64]) {
  float a[32], b[32];
  tmem_ld_32x32b_x32(taddr, a);
  tmem_ld_32x32b_x32(taddr + 32, b);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = a[i];
    v[32 + i] = b[i];
  }
}

// Byte offset of 16-byte granule g (0-35) of row r in a buffer of 5 K-major 128-byte-swizzled chunks of `rows` rows.
SSB_DEVICE uint32_t chunk_off(int r, int g, int chunk_bytes) {
  const int c = g < 32 ? (g >> 3) : 4, gg = g < 32 ? (g & 7) : g - 32;
  return c * chunk_bytes + r * 128 + ((gg ^ (r & 7)) << 4);
}

__global__ void __launch_bounds__(kMlaThreads, 1) sparse_mla_kernel(const MlaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t = blockIdx.x;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  const uint32_t kv_full = bar0, kv_empty = bar0 + 16, s_full = bar0 + 32, p_full = bar0 + 40, o_done = bar0 + 48;
  int32_t* slots = reinterpret_cast<int32_t*>(smem + kOffSlots);
  unsigned long long* tmask = reinterpret_cast<unsigned long long*>(smem + kOffMask);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + kOffMisc + 4);
  volatile int32_t* nblk_s = reinterpret_cast<volatile int32_t*>(smem + kOffMisc + 8);
  uint16_t* blist = reinterpret_cast<uint16_t*>(smem + kOffList);

  // the row's request (binary search of the query start list) and its pages
  int lo = 0, hi = a.R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.qsl[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int32_t* pages = a.table + (int64_t)lo * a.width;
  const int32_t* idx = a.indices + t * a.ld_idx;

  // Q (64 heads x 576 bytes) by cp.async into the 5 swizzled chunks, 9 granules a thread
  {
    const uint8_t* q = a.q + t * (kHeads * kDq);
    if (tid < kPro) {
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const int p = tid + kPro * k, h = p / 36, g = p - h * 36;
        cp_async16(sbase + kOffQ + chunk_off(h, g, kQChunk), q + h * kDq + g * 16, true);
      }
    }
    cp_async_commit();
  }
  if (tid == 0) {
    mbar_init(kv_full, kGather);
    mbar_init(kv_full + 8, kGather);
    mbar_init(kv_empty, 1);
    mbar_init(kv_empty + 8, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  // every index column -> its cache row (the loads of all columns in flight at once), and the selected-column bits
  if (tid < kPro) {
    constexpr int kPer = (kMaxIdx + kPro - 1) / kPro;   // 9
    int32_t pos[kPer], pg[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int j = tid + kPro * k;
      pos[k] = j < a.n_idx ? idx[j] : -1;
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) pg[k] = (pos[k] >= 0 && (pos[k] >> 7) < a.width) ? pages[pos[k] >> 7] : -1;
    static_assert(kPer * kPro == kMaxIdx, "every column written");
    static_assert(kPro % 32 == 0 && kPro <= kMlaThreads, "whole warps resolve the columns");
    uint32_t* tm32 = reinterpret_cast<uint32_t*>(tmask);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int j = tid + kPro * k;                  // a warp's 32 lanes: the 32 columns of word j >> 5
      const bool v = pg[k] >= 0 && pg[k] < (1 << 24);
      slots[j] = v ? pg[k] * 128 + (pos[k] & 127) : -1;
      const uint32_t bits = __ballot_sync(0xffffffffu, v);
      if (lane == 0) tm32[j >> 5] = bits;
    }
  }
  __syncthreads();
  // blocks of index columns without a selected token are skipped: list the others in order
  if (tid == 0) {
    int n = 0;
    for (int b = 0; b < kMaxBlocks; ++b)
      if (tmask[2 * b] | tmask[2 * b + 1]) blist[n++] = static_cast<uint16_t>(b);
    *nblk_s = n;
  }
  cp_async_wait0();
  fence_proxy_async_smem();                              // Q (generic-proxy writes) -> visible to the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int nblk = *nblk_s;
  const uint32_t tmem = *tmem_slot;

  if (warp >= 5) {
    // ---------------------------------------------------------------- gather
    const int gt = tid - 160;
    for (int i = 0; i < nblk; ++i) {
      const int buf = i & 1;
      bool ok = true;
      if (i >= 2) ok = mbar_wait(kv_empty + 8 * buf, ((i >> 1) - 1) & 1, abort_flag, a.status);   // PV of i - 2
      if (named_bar_or(1, kGather, !ok)) break;
      const uint32_t kvb = sbase + kOffKv + buf * kKvBuf;
      const int32_t* bs = slots + blist[i] * kBlk;
#pragma unroll 4
      for (int p = gt; p < kBlk * 36; p += kGather) {
        const int tok = p / 36, g = p - tok * 36;
        const int32_t sl = bs[tok];
        const bool v = sl >= 0;
        cp_async16(kvb + chunk_off(tok, g, kKvChunk), a.kv + (int64_t)(v ? sl : 0) * kDq + g * 16, v);
      }
      // the arrive fires when this thread's copies have landed: the gather moves on to the other buffer meanwhile
      // (the MMA thread orders the copies before its tensor-core reads with a proxy fence)
      cp_async_arrive_noinc(kv_full + 8 * buf);
    }
    cp_async_wait0();
  } else if (warp == 4) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_e4m3(64, 64);                   // tokens 0-63 -> lanes 0-15, 64-127 -> 16-31
      constexpr uint32_t idesc_pv = idesc_e4m3(64, 256) | (1u << 16);    // B (V) MN-major
      int issued = 0;
      for (int i = 0; i < nblk; ++i) {
        const int buf = i & 1;
        if (!mbar_wait(kv_full + 8 * buf, (i >> 1) & 1, abort_flag, a.status)) break;
        fence_proxy_async_smem();                          // the gathered rows (cp.async) -> the tensor core
        tc_fence_after();
        const uint32_t kvb = sbase + kOffKv + buf * kKvBuf;
#pragma unroll
        for (int c = 0; c < kNC; ++c) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (c == kNC - 1 && ks >= 2) break;                            // the rope chunk holds 64 bytes
            const uint64_t ad = smem_desc(sbase + kOffQ + c * kQChunk + ks * 32, 0, 1024, 2);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint64_t bd = smem_desc(kvb + c * kKvChunk + hh * 8192 + ks * 32, 0, 1024, 2);
              tc_mma_f8(tmem + (static_cast<uint32_t>(16 * hh) << 16) + kSCol, ad, bd, idesc_s, (c | ks) != 0 ? 1u : 0u);
            }
          }
        }
        tc_commit(s_full);
        issued = 1;
        if (!mbar_wait(p_full, i & 1, abort_flag, a.status)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = smem_desc(sbase + kOffP + ks * 32, 0, 1024, 2);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t bd = smem_desc(kvb + 2 * h * kKvChunk + ks * 4096, kKvChunk, 1024, 2);
            tc_mma_f8(tmem + (static_cast<uint32_t>(16 * h) << 16) + kOCol, ad, bd, idesc_pv,
                      (i > 0 || ks > 0) ? 1u : 0u);
          }
        }
        tc_commit(kv_empty + 8 * buf);
      }
      tc_commit(o_done);                                 // every MMA issued above has completed when this arrives
      if (issued) drain_bar(o_done, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 0-3)
    const int half = lane >> 4, row = 16 * warp + (lane & 15);
    const uint32_t tq = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float sc = a.scale * 1.4426950408889634f;      // log2(e) folded in: weights are 2^(s - m)
    uint8_t* Pb = smem + kOffP;
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = true;
    for (int i = 0; i < nblk; ++i) {
      const bool w = mbar_wait(s_full, i & 1, abort_flag, a.status);
      if (named_bar_or(2, 128, !w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[64];
      tmem_ld_x64(tq + kSCol, v);
      tmem_ld_wait();
      const unsigned long long vm = tmask[2 * blist[i] + half];
      float mb = -INFINITY;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        v[j] = ((vm >> j) & 1ull) ? v[j] * sc : -INFINITY;
        mb = fmaxf(mb, v[j]);
      }
      mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 16));
      float alpha = 1.0f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        m_used = mb;                                     // nothing accumulated yet (O = 0, l = 0)
      } else if (mb > m_used + kLazy) {
        alpha = ex2_approx(m_used - mb);
        m_used = mb;
        l_sum *= alpha;
        rescale = true;
      }
      // rescale O rows in TMEM when a row's max moved (warp-collective; PV of the previous block has completed)
      if (__any_sync(0xffffffffu, rescale) && i > 0) {
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
      float ps = 0.0f;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t wd[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float p[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float x = v[16 * g + 4 * e + u];
            p[u] = (m_used == -INFINITY) ? 0.0f : ex2_approx(x - m_used);
            ps += p[u];
          }
          wd[e] = e4m3x2(p[0] * kPScale, p[1] * kPScale) | (e4m3x2(p[2] * kPScale, p[3] * kPScale) << 16);
        }
        const int gg = 4 * half + g;                     // 16-token granule of the row
        *reinterpret_cast<uint4*>(Pb + row * 128 + ((gg ^ (row & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
      l_sum += ps + __shfl_xor_sync(0xffffffffu, ps, 16);
      fence_proxy_async_smem();                          // P (generic stores) -> visible to the tensor core
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---- epilogue: lanes 0-15 dims 0-255 of head row 16 warp + lane, lanes 16-31 dims 256-511 ----
    const bool have = ok && nblk > 0;
    if (have && !mbar_wait(o_done, 0, abort_flag, a.status)) ok = false;
    tc_fence_after();
    const bool good = have && ok && !*abort_flag;
    const float inv = (good && l_sum > 0.0f) ? a.bmm2 / (l_sum * kPScale) : 0.0f;
    __nv_bfloat16* orow = a.out + (t * kHeads + row) * kDv + half * 256;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      float o[32];
      if (good) {
        tmem_ld_32x32b_x32(tq + kOCol + 32 * c, o);
        tmem_ld_wait();
      }
      uint4 pk[4];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x0 = good ? o[2 * e] * inv : 0.0f, x1 = good ? o[2 * e + 1] * inv : 0.0f;
        __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
        pw[e] = *reinterpret_cast<uint32_t*>(&h2);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(orow + 32 * c)[e] = pk[e];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Latent cache append: row t of src (bf16 [T, 576], row pitch lds) -> e4m3(x / k_scale) at cache row slots[t] (576
// bytes; skipped when the slot is < 0). One warp per row, 8 values per lane step.
__global__ void mla_append_kernel(const __nv_bfloat16* src, int64_t lds, const int64_t* slots, int64_t T,
                                  uint8_t* cache, float inv_scale) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int64_t s = slots[t];
  if (s < 0) return;
  const int lane = threadIdx.x & 31;
  for (int c = lane; c < kDq / 8; c += 32) {             // 72 groups of 8 values
    const uint4 v = reinterpret_cast<const uint4*>(src + t * lds)[c];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float2 f0 = __bfloat1622float2(b[2 * k]), f1 = __bfloat1622float2(b[2 * k + 1]);
      w[k] = e4m3x2(f0.x * inv_scale, f0.y * inv_scale) | (e4m3x2(f1.x * inv_scale, f1.y * inv_scale) << 16);
    }
    reinterpret_cast<uint2*>(cache + s * kDq)[c] = make_uint2(w[0], w[1]);
  }
}

// Query pack: q8[t, h, 0:512] = e4m3(lat[h, t, :] / q_scale) (head-major latent rows, rows_pad rows a head) and
// q8[t, h, 512:576] = e4m3(rope[t, h * rope_stride + :64] / q_scale). One thread per 8 values.
__global__ void mla_q_pack_kernel(const __nv_bfloat16* lat, int64_t rows_pad, const __nv_bfloat16* rope, int64_t ldr,
                                  int64_t rope_stride, int64_t T, uint8_t* q8, float inv_scale) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * kHeads * (kDq / 8)) return;
  const int g = static_cast<int>(i % (kDq / 8));
  const int64_t th = i / (kDq / 8);
  const int h = static_cast<int>(th % kHeads);
  const int64_t t = th / kHeads;
  const uint4 v = g < kDv / 8 ? reinterpret_cast<const uint4*>(lat + ((int64_t)h * rows_pad + t) * kDv)[g]
                              : reinterpret_cast<const uint4*>(rope + t * ldr + h * rope_stride)[g - kDv / 8];
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint32_t w[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float2 f0 = __bfloat1622float2(b[2 * k]), f1 = __bfloat1622float2(b[2 * k + 1]);
    w[k] = e4m3x2(f0.x * inv_scale, f0.y * inv_scale) | (e4m3x2(f1.x * inv_scale, f1.y * inv_scale) << 16);
  }
  reinterpret_cast<uint2*>(q8 + th * kDq)[g] = make_uint2(w[0], w[1]);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int launch_sparse_mla(const MlaArgs& a, cudaStream_t stream) {
  if (a.q == nullptr || a.kv == nullptr || a.indices == nullptr || a.qsl == nullptr || a.table == nullptr ||
      a.out == nullptr || a.T < 0 || a.R <= 0 || a.width <= 0 || a.n_idx < 0 || a.n_idx > kMaxIdx ||
      a.ld_idx < a.n_idx || !al16(a.q) || !al16(a.kv) || !al16(a.out))
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

int launch_mla_append(const void* src, int64_t lds, const int64_t* slots, int64_t T, void* cache, float k_scale,
                      cudaStream_t stream) {
  if (src == nullptr || slots == nullptr || cache == nullptr || T < 0 || lds < kDq || (lds % 8) || !al16(src) ||
      !al16(cache) || !(k_scale > 0.0f))
    return kErrArgs;
  if (T == 0) return kOk;
  mla_append_kernel<<<(unsigned)((T + 7) / 8), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), lds, slots, T,
                                                                 static_cast<uint8_t*>(cache), 1.0f / k_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_mla_q_pack(const void* lat, int64_t rows_pad, const void* rope, int64_t ldr, int64_t rope_stride,
                      int64_t T, void* q8, float q_scale, cudaStream_t stream) {
  if (lat == nullptr || rope == nullptr || q8 == nullptr || T < 0 || rows_pad < T || (ldr % 8) || (rope_stride % 8) ||
      !al16(lat) || !al16(rope) || !al16(q8) || !(q_scale > 0.0f))
    return kErrArgs;
  const int64_t n = T * kHeads * (kDq / 8);
  if (n == 0) return kOk;
  mla_q_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(lat), rows_pad, static_cast<const __nv_bfloat16*>(rope), ldr, rope_stride, T,
      static_cast<uint8_t*>(q8), 1.0f / q_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
