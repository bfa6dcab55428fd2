// Canonical per-row top-k of the DSA indexer (sm_100a).
//
// For row r the keys are columns [ks[r], ke[r]) of `logits`; the selected set is every key strictly above the k-th
// largest value plus, among the keys equal to it, the lowest columns; the output holds the selected columns minus
// ks[r] in ascending order, -1 past the number selected (rows of at most k keys select all their keys). This is the
// rule of the reference's `canonicalize` (ssengine/model/topk_canon.py:1-52), computed here from the logits directly,
// so the select and the canonical rewrite (the reference's top-k kernel + 3 rewrite kernels) are one kernel.
//
// One CTA per row (grid-stride over rows), 256 threads, several CTAs per SM:
//  1. keys = order-preserving uint32 images of the floats (NaN sorts below every number), cached in shared memory
//     for rows of up to 4096 keys, else re-read from global memory (L2) in each pass;
//  2. radix select of the k-th largest key, MSB first, digits of 11, 11 and 10 bits: a 2048-bin shared-memory
//     histogram of the first digit (sign, exponent and two mantissa bits: logits spread over many bins, so the
//     atomics rarely collide), then the keys in the chosen bin are compacted into a candidate list (when it fits)
//     and the two remaining digits are resolved on the candidates only; each bin choice is a block-wide scan from
//     the top bin down;
//  3. compaction in column order with two block barriers: each warp owns a contiguous segment of the row, counts its
//     selected keys, and after a prefix over warps writes them with ballot + popcount ranks.
// Memory bound by design: one HBM read of the row plus k int32 writes (later passes hit L2 or shared memory).
// Rows longer than the shared-memory cache (the indexer's long contexts: tens of thousands of pools) take a two-pass
// form with 16-byte loads, four in flight per thread: pass 1 builds the first-digit histogram; pass 2 collects the
// columns above the chosen bin (all selected) and the keys and columns inside it (the candidates); the remaining
// digits are resolved on the candidates in shared memory, the ties at the threshold are taken lowest column first
// (a bitonic sort when more tie than are needed), and the k selected columns are sorted ascending (bitonic) before
// the store. A bin holding more candidates than the list fits falls back to the streaming passes above.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

constexpr int kTopkThreads = 256;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kCand = 4096;                    // candidate list capacity (keys + columns)
constexpr int kMaxK = 2048;                    // largest k of the two-pass long-row form (selected-column buffer)

SSB_DEVICE uint32_t order_key(float f) {
  if (f != f) return 0u;                       // NaN: below every number
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// From the top bin down, find the bin of `hist` (nbins, a multiple of 256) where the running count reaches `need`;
// thread t scans bins [nbins - (t + 1) * per, nbins - t * per); publishes the bin and the count still needed in it.
SSB_DEVICE void pick_bin(const uint32_t* hist, int nbins, uint32_t need, int tid, int lane, int warp,
                         uint32_t* w_sum, uint32_t* s_bin, uint32_t* s_need) {
  const int per = nbins / kTopkThreads;
  const int top = nbins - 1 - tid * per;      // this thread's bins: top, top - 1, ..., top - per + 1
  uint32_t local = 0;
  for (int j = 0; j < per; ++j) local += hist[top - j];
  uint32_t incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) w_sum[warp] = incl;
  __syncthreads();
  uint32_t before = 0;
  for (int w = 0; w < warp; ++w) before += w_sum[w];
  const uint32_t excl = before + incl - local;
  if (excl < need && need <= excl + local) {
    uint32_t run = excl;
    for (int j = 0; j < per; ++j) {
      const uint32_t c = hist[top - j];
      if (run + c >= need) {
        *s_bin = static_cast<uint32_t>(top - j);
        *s_need = need - run;
        break;
      }
      run += c;
    }
  }
  __syncthreads();
}

// Bitonic sort of v[0, n) ascending (n a power of two, <= 4096), all threads of the block; barriers inside.
SSB_DEVICE void bitonic_sort(uint32_t* v, int n, int tid) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n / 2; i += kTopkThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint32_t a = v[lo], b = v[hi];
        if ((a > b) == up) {
          v[lo] = b;
          v[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// fn(i, key) for every i in [0, n) of `row`: 16-byte loads, four in flight per thread, scalar head and tail around the
// 16-byte-aligned body. Keys are order_key images.
template <class Fn>
SSB_DEVICE void for_keys(const float* __restrict__ row, int n, int tid, Fn fn) {
  const int head = min(n, static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) >> 2));
  for (int i = tid; i < head; i += kTopkThreads) fn(i, order_key(__ldg(row + i)));
  const float4* body = reinterpret_cast<const float4*>(row + head);
  const int nv = (n - head) >> 2;
  for (int v0 = tid; v0 < nv; v0 += 4 * kTopkThreads) {
    float4 f[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = v0 + u * kTopkThreads;
      f[u] = v < nv ? __ldg(body + v) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = v0 + u * kTopkThreads;
      if (v < nv) {
        const int i = head + 4 * v;
        fn(i, order_key(f[u].x));
        fn(i + 1, order_key(f[u].y));
        fn(i + 2, order_key(f[u].z));
        fn(i + 3, order_key(f[u].w));
      }
    }
  }
  for (int i = head + 4 * nv + tid; i < n; i += kTopkThreads) fn(i, order_key(__ldg(row + i)));
}

__global__ void __launch_bounds__(kTopkThreads)
    topk_canon_kernel(const float* __restrict__ logits, int64_t rows, int64_t ld, const int32_t* __restrict__ ks,
                      const int32_t* __restrict__ ke, int k, int32_t* __restrict__ out, int cache_keys) {
  extern __shared__ uint32_t sm_keys[];        // [cache_keys] row cache, then the long-row lists
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t w_sum[kTopkWarps];
  __shared__ uint32_t cand_key[kCand];
  uint32_t* cand_col = sm_keys + cache_keys;  // dynamic shared memory after the row cache: [kCand] then [kMaxK]
  uint32_t* sel = cand_col + kCand;
  __shared__ uint32_t s_bin, s_need, s_ncand, s_nsel, s_ntie;
  __shared__ uint32_t w_above[kTopkWarps], w_tie[kTopkWarps];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int lo = ks[r];
    const int hi = ke[r];
    const int n = hi > lo ? hi - lo : 0;
    int32_t* orow = out + r * k;
    const float* row = logits + r * ld + lo;
    if (n <= k) {
      for (int i = tid; i < k; i += kTopkThreads) orow[i] = i < n ? i : -1;
      continue;
    }
    const bool cached = n <= cache_keys;
    auto key_at = [&](int i) -> uint32_t { return cached ? sm_keys[i] : order_key(__ldg(row + i)); };
    const int n_pad = (n + kTopkThreads - 1) / kTopkThreads * kTopkThreads;   // uniform trip counts per warp

    if (!cached && k <= kMaxK) {
      // ---- long rows: pass 1, the first-digit histogram ----
      for (int i = tid; i < 2048; i += kTopkThreads) hist[i] = 0;
      if (tid == 0) {
        s_ncand = 0;
        s_nsel = 0;
        s_ntie = 0;
      }
      __syncthreads();
      for_keys(row, n, tid, [&](int, uint32_t key) { atomicAdd(&hist[key >> 21], 1u); });
      __syncthreads();
      pick_bin(hist, 2048, static_cast<uint32_t>(k), tid, lane, warp, w_sum, &s_bin, &s_need);
      const uint32_t b1 = s_bin;
      // ---- pass 2: columns above the bin (selected), keys and columns in it (candidates) ----
      for_keys(row, n, tid, [&](int i, uint32_t key) {
        const uint32_t d = key >> 21;
        if (d > b1) {
          sel[atomicAdd(&s_nsel, 1u)] = static_cast<uint32_t>(i);          // fewer than k: the bin holds the k-th
        } else if (d == b1) {
          const uint32_t c = atomicAdd(&s_ncand, 1u);
          if (c < static_cast<uint32_t>(kCand)) {
            cand_key[c] = key;
            cand_col[c] = static_cast<uint32_t>(i);
          }
        }
      });
      __syncthreads();
      const uint32_t nc = s_ncand;
      if (nc <= static_cast<uint32_t>(kCand)) {
        uint32_t prefix = b1 << 21, need = s_need, mask = 0xFFE00000u;
        for (int pass = 0; pass < 2; ++pass) {
          const int shift = pass == 0 ? 10 : 0;
          const int nbins = pass == 0 ? 2048 : 1024;
          for (int i = tid; i < nbins; i += kTopkThreads) hist[i] = 0;
          __syncthreads();
          for (int i = tid; i < static_cast<int>(nc); i += kTopkThreads) {
            const uint32_t key = cand_key[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & static_cast<uint32_t>(nbins - 1)], 1u);
          }
          __syncthreads();
          pick_bin(hist, nbins, need, tid, lane, warp, w_sum, &s_bin, &s_need);
          prefix |= s_bin << shift;
          need = s_need;
          mask |= static_cast<uint32_t>(nbins - 1) << shift;
        }
        // candidates above the threshold join the selected columns; the ties at it are counted
        for (int i = tid; i < static_cast<int>(nc); i += kTopkThreads) {
          const uint32_t key = cand_key[i];
          if (key > prefix) sel[atomicAdd(&s_nsel, 1u)] = cand_col[i];
          else if (key == prefix) atomicAdd(&s_ntie, 1u);
        }
        __syncthreads();
        const uint32_t nt = s_ntie;
        if (nt > 2048u) {                          // more ties than the tie buffer holds: the streaming passes below
          __syncthreads();
          goto streaming;
        }
        if (tid == 0) s_ntie = 0;
        __syncthreads();
        for (int i = tid; i < static_cast<int>(nc); i += kTopkThreads)
          if (cand_key[i] == prefix) hist[atomicAdd(&s_ntie, 1u)] = cand_col[i];   // hist is free: the tie columns
        __syncthreads();
        if (nt > need) {                                                   // lowest columns first
          int np2 = 1;
          while (np2 < static_cast<int>(nt)) np2 <<= 1;
          for (int i = static_cast<int>(nt) + tid; i < np2; i += kTopkThreads) hist[i] = 0xFFFFFFFFu;
          __syncthreads();
          bitonic_sort(hist, np2, tid);
        }
        const uint32_t base = s_nsel;
        for (int i = tid; i < static_cast<int>(need); i += kTopkThreads) sel[base + i] = hist[i];
        __syncthreads();
        // k selected columns, ascending
        int kp2 = 1;
        while (kp2 < k) kp2 <<= 1;
        for (int i = k + tid; i < kp2; i += kTopkThreads) sel[i] = 0xFFFFFFFFu;
        __syncthreads();
        bitonic_sort(sel, kp2, tid);
        for (int i = tid; i < k; i += kTopkThreads) orow[i] = static_cast<int32_t>(sel[i]);
        __syncthreads();                                                   // the next row reuses the buffers
        continue;
      }
      // more candidates than the list holds: the streaming passes below
    }
  streaming:

    // ---- digit 1 (bits 21..31) over the whole row (and the row into shared memory) ----
    for (int i = tid; i < 2048; i += kTopkThreads) hist[i] = 0;
    if (tid == 0) s_ncand = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kTopkThreads) {
      const uint32_t key = order_key(__ldg(row + i));
      if (cached) sm_keys[i] = key;
      atomicAdd(&hist[key >> 21], 1u);
    }
    __syncthreads();
    pick_bin(hist, 2048, static_cast<uint32_t>(k), tid, lane, warp, w_sum, &s_bin, &s_need);
    uint32_t prefix = s_bin << 21, need = s_need, mask = 0xFFE00000u;

    // ---- candidates: the keys in that bin ----
    for (int i = tid; i < n_pad; i += kTopkThreads) {
      const bool v = i < n;
      const uint32_t key = v ? key_at(i) : 0u;
      const bool c = v && (key & mask) == prefix;
      const uint32_t b = __ballot_sync(0xFFFFFFFFu, c);
      uint32_t base = 0;
      if (lane == 0 && b) base = atomicAdd(&s_ncand, static_cast<uint32_t>(__popc(b)));
      base = __shfl_sync(0xFFFFFFFFu, base, 0);
      const uint32_t slot = base + __popc(b & ((1u << lane) - 1u));
      if (c && slot < kCand) cand_key[slot] = key;
    }
    __syncthreads();
    const uint32_t ncand = s_ncand;
    const bool use_cand = ncand <= static_cast<uint32_t>(kCand);
    const int m = use_cand ? static_cast<int>(ncand) : n;

    // ---- digits 2 (bits 10..20) and 3 (bits 0..9) on the candidates (or the whole row when they overflow) ----
    for (int pass = 0; pass < 2; ++pass) {
      const int shift = pass == 0 ? 10 : 0;
      const int nbins = pass == 0 ? 2048 : 1024;
      for (int i = tid; i < nbins; i += kTopkThreads) hist[i] = 0;
      __syncthreads();
      for (int i = tid; i < m; i += kTopkThreads) {
        const uint32_t key = use_cand ? cand_key[i] : key_at(i);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & static_cast<uint32_t>(nbins - 1)], 1u);
      }
      __syncthreads();
      pick_bin(hist, nbins, need, tid, lane, warp, w_sum, &s_bin, &s_need);
      prefix |= s_bin << shift;
      need = s_need;
      mask |= static_cast<uint32_t>(nbins - 1) << shift;
    }
    // prefix = key of the k-th largest; need = keys equal to it to take, lowest columns first

    // ---- compaction in column order: warp w owns columns [w * seg, (w + 1) * seg) ----
    const int seg = (n + kTopkWarps - 1) / kTopkWarps;
    const int s0 = warp * seg;
    const int s1 = min(n, s0 + seg);
    uint32_t above = 0, ties = 0;
    for (int c0 = s0; c0 < s1; c0 += 32) {
      const int i = c0 + lane;
      const bool v = i < s1;
      const uint32_t key = v ? key_at(i) : 0u;
      above += __popc(__ballot_sync(0xFFFFFFFFu, v && key > prefix));
      ties += __popc(__ballot_sync(0xFFFFFFFFu, v && key == prefix));
    }
    if (lane == 0) {
      w_above[warp] = above;
      w_tie[warp] = ties;
    }
    __syncthreads();
    uint32_t tie_run = 0, sel_run = 0;
    for (int w = 0; w < warp; ++w) {
      const uint32_t t = w_tie[w];
      const uint32_t taken = min(t, need > tie_run ? need - tie_run : 0u);
      sel_run += w_above[w] + taken;
      tie_run += t;
    }
    for (int c0 = s0; c0 < s1; c0 += 32) {
      const int i = c0 + lane;
      const bool v = i < s1;
      const uint32_t key = v ? key_at(i) : 0u;
      const bool tie = v && key == prefix;
      const uint32_t bt = __ballot_sync(0xFFFFFFFFu, tie);
      const uint32_t tie_rank = tie_run + __popc(bt & ((1u << lane) - 1u));
      const bool sel = (v && key > prefix) || (tie && tie_rank < need);
      const uint32_t bs = __ballot_sync(0xFFFFFFFFu, sel);
      const uint32_t pos = sel_run + __popc(bs & ((1u << lane) - 1u));
      if (sel && pos < static_cast<uint32_t>(k)) orow[pos] = i;
      sel_run += __popc(bs);
      tie_run += __popc(bt);
    }
    __syncthreads();   // the next row reuses the shared buffers
  }
}

}  // namespace

int launch_topk_canonical(const float* logits, int64_t rows, int64_t ld, const int32_t* ks, const int32_t* ke,
                          int32_t k, int32_t* out, int32_t max_keys, cudaStream_t stream) {
  if (rows < 0 || k <= 0 || ld <= 0 || max_keys < 0) return kErrArgs;
  if (rows == 0) return kOk;
  // cache rows of up to 4096 keys (16 KB) in shared memory; longer rows are re-read from L2 in each pass, which keeps
  // 8 CTAs resident per SM (measured at 16 Ki-key rows: 1.0 ms streaming vs 1.9 ms with a 64 KB row cache that
  // leaves 2 CTAs per SM: the passes are latency-bound and need the warps)
  const int cache = max_keys < 4096 ? max_keys : 4096;
  const size_t smem = static_cast<size_t>(cache + kCand + kMaxK) * 4;
  // static (~25 KB) + dynamic shared memory passes the 48 KB a launch gets without opting in
  if (cudaFuncSetAttribute(topk_canon_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return kErrCuda;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, topk_canon_kernel, kTopkThreads, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t grid = static_cast<int64_t>(device_sm_count()) * per_sm;
  if (grid > rows) grid = rows;
  topk_canon_kernel<<<static_cast<unsigned>(grid), kTopkThreads, smem, stream>>>(logits, rows, ld, ks, ke, k, out,
                                                                                   cache);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
