// DSA lightning indexer for sm_100a: the per-query pool logits over the paged pool-key cache, and the expansion of
// the selected pools into token indices.
//
//   logit[t, p] = sum_h w[t, h] * relu(q[t, h, :] . k_pool[p, :])     (h < 32 heads, dim 128, pools p < (pos_t+1)/4)
//
// Pool keys are paged like the KV: the request's KV page j (128 tokens) holds its pools 32j .. 32j+31, pool row
// page * 32 + p % 32 of the [pages * 32, 128] bf16 cache, so the pool pages are the chunk's `kv_pages`.
//
// One tcgen05 tile: D[128 pools x 256] = K_pool[128 x 128] . Q[8 queries x 32 heads, 128]^T (kind::f16, bf16 in,
// fp32 in TMEM). Pools are the MMA's M, so each TMEM lane is one pool and its 256 columns are the 8 queries' 32 heads:
// the weighted ReLU sum over heads runs in one thread's registers, with no cross-lane reduction.
// Work unit: a group of <= 8 consecutive query rows of one request (host table, longest first); its Q tile stays in
// shared memory while its pool tiles stream through a 4-stage ring. Roles (320 threads, persistent):
//   warp 0 TMA producer (Q tile: 2 boxes of 256 x 64; pool tile: 2 x 4 page boxes of 32 x 64, 128-byte swizzle),
//   warp 1 TMEM owner + MMA issuer (8 MMAs of K = 16 per tile; two 256-column accumulators alternate),
//   warps 2-9 epilogue (lane quadrant = warp % 4, two warps a quadrant taking 4 of the 8 queries each): tcgen05.ld of
//   two queries' 32 heads at a time, ReLU, weights, four partial sums over the heads, fp32 logits rows.
// Every wait is bounded; on expiry the roles leave, in-flight copies / MMAs are drained, TMEM is freed and the
// status word holds kErrTimeout. No cluster multicast.
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kIdxEpiWarps = 8;             // two per TMEM lane quadrant, 4 of the 8 queries each
constexpr int kIdxThreads = 64 + 32 * kIdxEpiWarps;
constexpr int kStages = 4;
constexpr int kAChunk = 128 * 128;          // one 128-byte k-chunk of a pool tile: 128 rows x 128 B
constexpr int kBChunk = 256 * 128;          // one k-chunk of the Q tile: 256 rows x 128 B
constexpr int kFp8PageRows = 33;            // an FP8 pool page: 32 rows of 128 e4m3 codes, then 32 fp32 scales

// Shared-memory plan of the bf16 form (128 dims = two 128-byte k-chunks of 64 values) and of the FP8 form (one chunk
// of 128 codes): Q tile, a 4-stage pool-tile ring, barriers, the staged head weights.
template <bool FP8>
struct IdxCfg {
  static constexpr int kChunks = FP8 ? 1 : 2;
  static constexpr int kABytes = kChunks * kAChunk;     // 16 / 32 KB
  static constexpr int kBBytes = kChunks * kBChunk;     // 32 / 64 KB
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kBBytes;
  static constexpr int kOffBar = kOffA + kStages * kABytes;
  // bars: full[S], empty[S], q_full, q_empty, acc_full[2], acc_empty[2], drain
  static constexpr int kOffMisc = kOffBar + (2 * kStages + 7) * 8;
  static constexpr int kOffW = (kOffMisc + 16 + 127) & ~127;   // fp32 head weights of 8 queries, two buffers [2][8][32]
  static constexpr int kSmem = kOffW + 2 * 8 * 32 * 4 + 1024;
  static_assert(kOffA % 1024 == 0 && kABytes % 1024 == 0, "128-byte swizzle atoms of the tiles");
  static_assert(kOffW % 16 == 0, "float4 reads of the staged weights");
};

SSB_DEVICE void drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) break;
  }
}

template <bool FP8>
__global__ void __launch_bounds__(kIdxThreads, 1)
    indexer_logits_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                          const IdxArgs a) {
  using C = IdxCfg<FP8>;
  constexpr int kOffB = C::kOffB, kOffA = C::kOffA, kOffBar = C::kOffBar, kOffMisc = C::kOffMisc, kOffW = C::kOffW;
  constexpr int kABytes = C::kABytes, kBBytes = C::kBBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + kOffBar;
  const uint32_t bar_empty = bar_full + kStages * 8;
  const uint32_t bar_qfull = bar_empty + kStages * 8;
  const uint32_t bar_qempty = bar_qfull + 8;
  const uint32_t bar_accf = bar_qempty + 8;        // [2]
  const uint32_t bar_acce = bar_accf + 16;         // [2]
  const uint32_t bar_drain = bar_acce + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + kOffMisc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_qfull, 1);
    mbar_init(bar_qempty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8 * b, 1);
      mbar_init(bar_acce + 8 * b, kIdxEpiWarps);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&mq);
      tma_prefetch_desc(&mk);
      int stage = 0, issued = 0, qissued = 0;
      uint32_t phase = 0, qphase = 0;
      bool ok = true;
      for (int gi = blockIdx.x; ok && gi < a.G; gi += gridDim.x) {
        const int4 gr = reinterpret_cast<const int4*>(a.groups)[gi];
        if (gr.w <= 0) continue;
        if (!mbar_wait(bar_qempty, qphase ^ 1, abort_flag, a.status)) { ok = false; break; }
        mbar_arrive_expect_tx(bar_qfull, kBBytes);
        tma_load_2d(sbase + kOffB, &mq, 0, gr.y * 32, bar_qfull);
        if (!FP8) tma_load_2d(sbase + kOffB + kBChunk, &mq, 64, gr.y * 32, bar_qfull);
        ++qissued;
        qphase ^= 1;
        const int32_t* pages = a.table + (int64_t)gr.x * a.width;
        for (int m = 0; m < gr.w; ++m) {
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, abort_flag, a.status)) { ok = false; break; }
          const uint32_t fb = bar_full + 8 * stage;
          mbar_arrive_expect_tx(fb, kABytes);
          const uint32_t sa = sbase + kOffA + stage * kABytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = 4 * m + i;
            const int page = j < a.width ? pages[j] : -1;
            // a page's 32 pool rows (FP8: the first 32 of its 33 rows); a missing page reads as zeros
            const int row = page >= 0 ? page * (FP8 ? kFp8PageRows : 32) : -32;
            tma_load_2d(sa + i * 4096, &mk, 0, row, fb);
            if (!FP8) tma_load_2d(sa + kAChunk + i * 4096, &mk, 64, row, fb);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        int s = stage;
        uint32_t p = phase;
        for (int i = 0; i < min(issued, kStages); ++i) {
          if (--s < 0) { s = kStages - 1; p ^= 1; }
          drain(bar_full + 8 * s, p);
        }
        if (qissued > 0) drain(bar_qfull, qphase ^ 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = FP8 ? idesc_e4m3(128, 256) : idesc_bf16(128, 256);
      int stage = 0;
      uint32_t phase = 0, qphase = 0, iter = 0;
      bool ok = true, any = false;
      for (int gi = blockIdx.x; ok && gi < a.G; gi += gridDim.x) {
        const int4 gr = reinterpret_cast<const int4*>(a.groups)[gi];
        if (gr.w <= 0) continue;
        if (!mbar_wait(bar_qfull, qphase, abort_flag, a.status)) { ok = false; break; }
        qphase ^= 1;
        tc_fence_after();
        for (int m = 0; m < gr.w; ++m) {
          const int buf = iter & 1;
          if (!mbar_wait(bar_acce + 8 * buf, ((iter >> 1) & 1) ^ 1, abort_flag, a.status)) { ok = false; break; }
          if (!mbar_wait(bar_full + 8 * stage, phase, abort_flag, a.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + kOffA + stage * kABytes;
          // 32 bytes of K a step: 16 bf16 values (kind::f16) or 32 e4m3 codes (kind::f8f6f4)
#pragma unroll
          for (int kc = 0; kc < C::kChunks; ++kc) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = smem_desc(sa + kc * kAChunk + ks * 32, 0, 1024, 2);
              const uint64_t bd = smem_desc(sbase + kOffB + kc * kBChunk + ks * 32, 0, 1024, 2);
              if (FP8)
                tc_mma_f8(tmem + buf * 256, ad, bd, idesc, (kc | ks) != 0 ? 1u : 0u);
              else
                tc_mma_f16(tmem + buf * 256, ad, bd, idesc, (kc | ks) != 0 ? 1u : 0u);
            }
          }
          any = true;
          tc_commit(bar_empty + 8 * stage);
          tc_commit(bar_accf + 8 * buf);
          ++iter;
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(bar_qempty);
      }
      if (!ok && any) {
        tc_commit(bar_drain);
        drain(bar_drain, 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9: lane quadrant warp % 4, queries 4 half .. 4 half + 3) ----------------
    const int quad = warp & 3, half = (warp - 2) >> 2, et = threadIdx.x - 64;
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float* wsm = reinterpret_cast<float*>(smem + kOffW);
    uint32_t iter = 0, gcount = 0;
    bool ok = true;
    for (int gi = blockIdx.x; gi < a.G; gi += gridDim.x) {
      const int4 gr = reinterpret_cast<const int4*>(a.groups)[gi];
      if (gr.w <= 0) continue;
      // the group's head weights (bf16, read in place) -> fp32 in shared memory, one per epilogue thread; buffer
      // gcount & 1 was last read two groups ago, by warps that have all passed the previous group's barrier. The
      // barrier also carries a failed wait of any epilogue warp, so that all of them leave together.
      float* wg = wsm + (gcount & 1) * 256;
      {
        const int j = et >> 5, hd = et & 31;
        if (ok && j < gr.z) {
          const uint16_t wb = static_cast<const uint16_t*>(a.w)[(int64_t)(gr.y + j) * a.ldw + hd];
          float wv = __uint_as_float(static_cast<uint32_t>(wb) << 16);
          if (FP8) wv *= a.q_scale[(int64_t)(gr.y + j) * 32 + hd];      // the query's scale folds into its weight
          wg[et] = wv;
        }
      }
      if (named_bar_or(3, 32 * kIdxEpiWarps, !ok)) break;
      ++gcount;
      for (int m = 0; m < gr.w; ++m) {
        const int buf = iter & 1;
        if (!mbar_wait(bar_accf + 8 * buf, (iter >> 1) & 1, abort_flag, a.status)) { ok = false; break; }
        tc_fence_after();
        const int64_t pool = (int64_t)m * 128 + quad * 32 + lane;
        float kscale = 1.0f;                   // FP8: the pool's scale, row 32 of its page, entry lane
        if (FP8) {
          const int jp = 4 * m + quad;
          const int page = jp < a.width ? a.table[(int64_t)gr.x * a.width + jp] : -1;
          kscale = page >= 0 ? a.kscale[(int64_t)page * (kFp8PageRows * 32) + 32 * 32 + lane] : 0.0f;
        }
        // two queries per TMEM wait; four partial sums over the heads (h % 4), added in a fixed order
        for (int j0 = 4 * half; j0 < min(gr.z, 4 * half + 4); j0 += 2) {
          const bool two = j0 + 1 < gr.z;
          float v[2][32];
          tmem_ld_32x32b_x32(tq + buf * 256 + j0 * 32, v[0]);
          if (two) tmem_ld_32x32b_x32(tq + buf * 256 + (j0 + 1) * 32, v[1]);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;
            const int64_t q = gr.y + j0 + u;
            const float4* wq = reinterpret_cast<const float4*>(wg + (j0 + u) * 32);
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 w4 = wq[i];                        // heads 4i .. 4i + 3 (a broadcast read)
              acc[0] = __fmaf_rn(fmaxf(v[u][4 * i], 0.0f), w4.x, acc[0]);
              acc[1] = __fmaf_rn(fmaxf(v[u][4 * i + 1], 0.0f), w4.y, acc[1]);
              acc[2] = __fmaf_rn(fmaxf(v[u][4 * i + 2], 0.0f), w4.z, acc[2]);
              acc[3] = __fmaf_rn(fmaxf(v[u][4 * i + 3], 0.0f), w4.w, acc[3]);
            }
            if (pool < a.ldl) a.logits[q * a.ldl + pool] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * kscale;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_acce + 8 * buf);
        ++iter;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Pool ids -> token indices (pure index arithmetic): columns < 4k: pool * 4 + c % 4 (or -1); then the tokens of the
// query's incomplete last pool, seq_len = pos + 1, tail = [4 * (seq_len / 4), seq_len), up to 3 columns (or -1).
__global__ void indexer_expand_kernel(const int32_t* pool_ids, int64_t ldp, int32_t k, const int64_t* positions,
                                      int32_t* out, int64_t ldo, int64_t rows) {
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  const int64_t seq_len = positions[row] + 1;
  const int64_t tail_start = (seq_len / 4) * 4;
  const int64_t tail_count = seq_len - tail_start;
  const int cols = 4 * k + 3;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    int32_t v;
    if (c < 4 * k) {
      const int32_t pid = pool_ids[row * ldp + c / 4];
      v = pid >= 0 ? pid * 4 + (c & 3) : -1;
    } else {
      const int off = c - 4 * k;
      v = off < tail_count ? static_cast<int32_t>(tail_start + off) : -1;
    }
    out[row * ldo + c] = v;
  }
}

}  // namespace

int launch_indexer_logits(const void* q, const void* k_cache, int64_t pool_rows, const IdxArgs& a,
                          cudaStream_t stream) {
  if (q == nullptr || k_cache == nullptr || a.w == nullptr || a.table == nullptr || a.groups == nullptr ||
      a.logits == nullptr || a.T <= 0 || pool_rows <= 0 || a.width <= 0 || a.G < 0 || a.ldl <= 0 ||
      (reinterpret_cast<uintptr_t>(a.w) & 15) || a.ldw < 32 || (a.ldw % 8))
    return kErrArgs;
  if (a.G == 0) return kOk;
  CUtensorMap mq, mk;
  int rc = make_map_2d_swizzled(&mq, q, a.T * 32, 128, 256, 256);
  if (rc != kOk) return rc;
  rc = make_map_2d_swizzled(&mk, k_cache, pool_rows, 128, 256, 32);
  if (rc != kOk) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(indexer_logits_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             IdxCfg<false>::kSmem) != cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  const int sms = device_sm_count();
  const int grid = a.G < sms ? a.G : sms;
  indexer_logits_kernel<false><<<grid, kIdxThreads, IdxCfg<false>::kSmem, stream>>>(mq, mk, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_indexer_logits_fp8(const uint8_t* q8, const float* q_scale, const uint8_t* k_pages, int64_t pages,
                              const IdxArgs& a_in, cudaStream_t stream) {
  IdxArgs a = a_in;
  if (q8 == nullptr || q_scale == nullptr || k_pages == nullptr || a.w == nullptr || a.table == nullptr ||
      a.groups == nullptr || a.logits == nullptr || a.T <= 0 || pages <= 0 || a.width <= 0 || a.G < 0 ||
      a.ldl <= 0 || (reinterpret_cast<uintptr_t>(a.w) & 15) || a.ldw < 32 || (a.ldw % 8) ||
      (reinterpret_cast<uintptr_t>(k_pages) & 127) || (reinterpret_cast<uintptr_t>(q8) & 127))
    return kErrArgs;
  if (a.G == 0) return kOk;
  a.q_scale = q_scale;
  a.kscale = reinterpret_cast<const float*>(k_pages);
  CUtensorMap mq, mk;
  // e4m3 codes as bytes: Q [T * 32, 128] (one box of 256 rows), the pool pages [pages * 33, 128] (boxes of 32 rows)
  int rc = make_map_2d_ex(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, q8, a.T * 32, 128, 128, 128, 256,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != kOk) return rc;
  rc = make_map_2d_ex(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_pages, pages * kFp8PageRows, 128, 128, 128, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != kOk) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(indexer_logits_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             IdxCfg<true>::kSmem) != cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  const int sms = device_sm_count();
  const int grid = a.G < sms ? a.G : sms;
  indexer_logits_kernel<true><<<grid, kIdxThreads, IdxCfg<true>::kSmem, stream>>>(mq, mk, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

namespace {

// Indexer queries to e4m3 per (token, head) row of 128 (the FP8 indexer): one warp a row, 4 values a lane; scale =
// 2^ceil(log2(max(amax, 1e-10) * fl(1 / 448))) (ue8m0, from the exponent bits), codes = e4m3(x / scale) (exact
// quotients, rounded to nearest even by cvt.rn.satfinite).
__global__ void idx_q_quant_kernel(const __nv_bfloat16* __restrict__ q, int64_t rows, uint8_t* __restrict__ q8,
                                   float* __restrict__ qs) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint2 raw = *reinterpret_cast<const uint2*>(q + row * 128 + lane * 4);
  float x[4];
  x[0] = __uint_as_float(raw.x << 16);
  x[1] = __uint_as_float(raw.x & 0xffff0000u);
  x[2] = __uint_as_float(raw.y << 16);
  x[3] = __uint_as_float(raw.y & 0xffff0000u);
  float am = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float s = fmaxf(am, 1e-10f) * (1.0f / 448.0f);
  const uint32_t b = __float_as_uint(s);
  const uint32_t e = ((b >> 23) & 0xffu) + ((b & 0x7fffffu) != 0u ? 1u : 0u);   // ceil(log2 s) + 127
  const float scale = __uint_as_float(e << 23), inv = __uint_as_float((254u - e) << 23);
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(x[1] * inv), "f"(x[0] * inv));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(x[3] * inv), "f"(x[2] * inv));
  *reinterpret_cast<uint32_t*>(q8 + row * 128 + lane * 4) = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  if (lane == 0) qs[row] = scale;
}

}  // namespace

int launch_indexer_q_quant(const void* q, int64_t rows, uint8_t* q8, float* q_scale, cudaStream_t stream) {
  if (q == nullptr || q8 == nullptr || q_scale == nullptr || rows < 0 || (reinterpret_cast<uintptr_t>(q) & 7) ||
      (reinterpret_cast<uintptr_t>(q8) & 3))
    return kErrArgs;
  if (rows == 0) return kOk;
  idx_q_quant_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(q), rows, q8,
                                                                     q_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_indexer_expand(const int32_t* pool_ids, int64_t ldp, int32_t k, const int64_t* positions, int32_t* out,
                          int64_t ldo, int64_t rows, cudaStream_t stream) {
  if (pool_ids == nullptr || positions == nullptr || out == nullptr || k <= 0 || rows < 0 || ldp < k ||
      ldo < 4 * (int64_t)k + 3)
    return kErrArgs;
  if (rows == 0) return kOk;
  indexer_expand_kernel<<<(unsigned)rows, 256, 0, stream>>>(pool_ids, ldp, k, positions, out, ldo, rows);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
