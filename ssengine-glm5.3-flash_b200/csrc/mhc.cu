// mHC (4-stream hyper-connections) at a layer boundary (sm_100a).
//
// The reference runs DeepGEMM `mega_mhc` here (ssengine/model/pp_patch.py:125-153: the previous layer's post, the
// next layer's pre and its RMSNorm in one persistent launch); the stage edge uses a standalone pre (edge_recv) and a
// standalone post (edge_send), :156-163. Arithmetic (the published mHC algorithm):
//   post: new_res[j] = post[j] * x + sum_i comb[i][j] * res[i]                     (bf16 out)
//   pre:  mixes = (z @ fn^T) * rsqrt(mean(z^2) + rms_eps), z = new_res flattened [4H] (fp32 of the bf16 values)
//         pre = sigmoid(mixes[0:4] s0 + b) + pre_eps; post' = sigmoid(mixes[4:8] s1 + b) * post_mult;
//         comb' = Sinkhorn(softmax_row(mixes[8:24] s2 + b)); y = RMSNorm(bf16(sum_i pre[i] new_res[i])) * w
// Layout: x [T, H] bf16, res / new_res [T, 4, H] bf16, post [T, 4] fp32, comb [T, 4, 4] fp32, fn [24, 4H] fp32.
//
// A pre step (post + pre, or pre only) is two launches: the persistent TMA-fed mix kernel (the new residual and the
// partial mixes) and the finalize kernel (Sinkhorn, the layer input and its RMSNorm), described at their definitions
// below. A post-only boundary (the stage edge's send) is one launch of `mhc_kernel<true, false>`:
// CTA = 32 tokens, 256 threads, up to 2 CTAs per SM. Main loop: warp w takes 16 tokens (tile w & 1) and a quarter of
// the hidden positions (w >> 1); each lane covers 2 tokens x 8 consecutive positions of every 32-position group
// (coalesced 16-byte loads of x and the 4 residual streams), forms the 4 new residual streams (bf16, stored) and feeds
// them directly as tf32 mma.sync fragments against the fn rows (read through the read-only cache with the same
// permutation of positions): no shared-memory staging and no block barrier in the loop. The quarters' partial mixes
// are summed in a fixed order in shared memory; then per token the pre / post / Sinkhorn scalars and two passes for
// the layer input and its RMSNorm. HBM traffic per token: 40 KB in (x + res), 32 KB new residual and 8 KB y out; the
// new residual is re-read for the layer input.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

constexpr int kMhcTok = 32;       // tokens per CTA
constexpr int kMhcThreads = 256;
constexpr int kMhcH = 64;         // hidden positions per y-pass step of a thread group
constexpr int kMhcMix = 24;

struct MhcArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* res;
  const float* post_in;
  const float* comb_in;
  __nv_bfloat16* new_res;
  const float* fn;
  const float* scale;
  const float* base;
  const __nv_bfloat16* norm_w;
  float* post_out;
  float* comb_out;
  __nv_bfloat16* y;
  int64_t T, H;
  float rms_eps, pre_eps, sinkhorn_eps, post_mult, norm_eps;
  int repeat;
  int32_t* status;
  int ranges;                // pre step: position ranges of a mix work item (8, or 4 when H % 512 != 0)
};

SSB_DEVICE float sigmoidf(float v) { return 1.0f / (1.0f + expf(-v)); }


template <bool POST, bool PRE>
__global__ void __launch_bounds__(kMhcThreads, 2) mhc_kernel(const MhcArgs a) {
  __shared__ float part[4][kMhcTok][kMhcMix];          // per K-quarter partial mixes
  __shared__ float ssp[4][kMhcTok];
  __shared__ __align__(16) float coef[kMhcTok][4][8];  // token, output stream j: post[j], comb[0..3][j]
  __shared__ float mix[kMhcTok][kMhcMix];
  __shared__ float ssq[kMhcTok];
  __shared__ float pre_s[kMhcTok][4];
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kMhcTok;
  const int64_t H = a.H;
  const int warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  if (POST) {
    for (int i = tid; i < kMhcTok * 4; i += kMhcThreads) {
      const int tk = i >> 2, j = i & 3;
      const int64_t tt = t0 + tk;
      float* d = coef[tk][j];
      const bool ok = tt < a.T;
      d[0] = ok ? a.post_in[tt * 4 + j] : 0.0f;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) d[1 + ii] = ok ? a.comb_in[tt * 16 + ii * 4 + j] : 0.0f;
    }
    __syncthreads();
  }
  // ---- main loop: warp -> 16 tokens (tile w & 1) x one quarter of the hidden positions (w >> 1); lane -> tokens
  //      g8 and g8 + 8 of the tile and 8 consecutive positions h = g + 8 t4 .. + 7 of each 32-position group g, so a
  //      quad of lanes reads 64 contiguous bytes of a row. The new residual goes straight into tf32 mma.sync
  //      fragments: within stream j's 4 k-steps s of a group, MMA k index c < 4 is position g + 8 c + 2 s and c >= 4
  //      is g + 8 (c - 4) + 2 s + 1 (a permutation of the 32 positions, applied to the fn rows alike). ----
  const int tr0 = 16 * (warp & 1) + g8, tr1 = tr0 + 8, kq = warp >> 1;
  const int64_t r0 = t0 + tr0, r1 = t0 + tr1;
  const bool v0 = r0 < a.T, v1 = r1 < a.T;
  float macc[3][4] = {};
  float ss0 = 0.0f, ss1 = 0.0f;
  const uint4 zero4 = make_uint4(0, 0, 0, 0);
  for (int64_t g = kq * (H / 4); g < (kq + 1) * (H / 4); g += 32) {
    const int64_t h = g + 8 * t4;
    uint4 rv0[4], rv1[4], xv0 = zero4, xv1 = zero4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rv0[i] = v0 ? *reinterpret_cast<const uint4*>(a.res + (r0 * 4 + i) * H + h) : zero4;
      rv1[i] = v1 ? *reinterpret_cast<const uint4*>(a.res + (r1 * 4 + i) * H + h) : zero4;
    }
    if (POST) {
      if (v0) xv0 = *reinterpret_cast<const uint4*>(a.x + r0 * H + h);
      if (v1) xv1 = *reinterpret_cast<const uint4*>(a.x + r1 * H + h);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float z0[8], z1[8];
      if (POST) {
        auto mixrow = [&](const uint4& xv, const uint4 (&rv)[4], const float* c, float (&z)[8]) -> uint4 {
          const float4 ca = *reinterpret_cast<const float4*>(c), cb = *reinterpret_cast<const float4*>(c + 4);
          const float cm[4] = {ca.y, ca.z, ca.w, cb.x};
          const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float v = ca.x * __bfloat162float(xb[e]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              v = fmaf(cm[i], __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv[i])[e]), v);
            const __nv_bfloat16 bv = __float2bfloat16(v);
            z[e] = __bfloat162float(bv);
            if (e & 1) w[e >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(bv)) << 16;
            else w[e >> 1] = __bfloat16_as_ushort(bv);
          }
          return make_uint4(w[0], w[1], w[2], w[3]);
        };
        const uint4 n0 = mixrow(xv0, rv0, coef[tr0][j], z0);
        const uint4 n1 = mixrow(xv1, rv1, coef[tr1][j], z1);
        if (v0) *reinterpret_cast<uint4*>(a.new_res + (r0 * 4 + j) * H + h) = n0;
        if (v1) *reinterpret_cast<uint4*>(a.new_res + (r1 * 4 + j) * H + h) = n1;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          z0[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv0[j])[e]);
          z1[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv1[j])[e]);
        }
      }
      if (PRE) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ss0 = fmaf(z0[e], z0[e], ss0);
          ss1 = fmaf(z1[e], z1[e], ss1);
        }
#pragma unroll
        for (int nt = 0; nt < 3; ++nt) {
          const float* fr = a.fn + static_cast<int64_t>(8 * nt + g8) * 4 * H + j * H + h;
          const float4 f0 = __ldg(reinterpret_cast<const float4*>(fr)), f1 = __ldg(reinterpret_cast<const float4*>(fr + 4));
          const float fb[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            uint32_t b0, b1;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b0) : "f"(fb[2 * st]));
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b1) : "f"(fb[2 * st + 1]));
            // z is bf16-exact, so its fp32 bits are already tf32
            asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                         "{%0,%1,%2,%3};"
                         : "+f"(macc[nt][0]), "+f"(macc[nt][1]), "+f"(macc[nt][2]), "+f"(macc[nt][3])
                         : "r"(__float_as_uint(z0[2 * st])), "r"(__float_as_uint(z1[2 * st])),
                           "r"(__float_as_uint(z0[2 * st + 1])), "r"(__float_as_uint(z1[2 * st + 1])), "r"(b0), "r"(b1));
          }
        }
      }
    }
  }
  if (!PRE) return;
  // ---- the 4 K-quarters' partials of the [32 x 24] mixes and of the sums of squares, summed in a fixed order ----
  ss0 += __shfl_xor_sync(0xFFFFFFFFu, ss0, 1);
  ss0 += __shfl_xor_sync(0xFFFFFFFFu, ss0, 2);
  ss1 += __shfl_xor_sync(0xFFFFFFFFu, ss1, 1);
  ss1 += __shfl_xor_sync(0xFFFFFFFFu, ss1, 2);
  if (t4 == 0) {
    ssp[kq][tr0] = ss0;
    ssp[kq][tr1] = ss1;
  }
#pragma unroll
  for (int nt = 0; nt < 3; ++nt) {
    part[kq][tr0][8 * nt + 2 * t4] = macc[nt][0];
    part[kq][tr0][8 * nt + 2 * t4 + 1] = macc[nt][1];
    part[kq][tr1][8 * nt + 2 * t4] = macc[nt][2];
    part[kq][tr1][8 * nt + 2 * t4 + 1] = macc[nt][3];
  }
  __syncthreads();
  for (int i = tid; i < kMhcTok * kMhcMix; i += kMhcThreads) {
    const int tk = i / kMhcMix, c = i % kMhcMix;
    mix[tk][c] = ((part[0][tk][c] + part[1][tk][c]) + part[2][tk][c]) + part[3][tk][c];
  }
  if (tid < kMhcTok) ssq[tid] = ((ssp[0][tid] + ssp[1][tid]) + ssp[2][tid]) + ssp[3][tid];
  __syncthreads();
  if (tid < kMhcTok && t0 + tid < a.T) {
    const int64_t tt = t0 + tid;
    const float rinv = rsqrtf(ssq[tid] / static_cast<float>(4 * H) + a.rms_eps);
    float mx[kMhcMix];
#pragma unroll
    for (int c = 0; c < kMhcMix; ++c) mx[c] = mix[tid][c] * rinv;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pre_s[tid][i] = sigmoidf(mx[i] * a.scale[0] + a.base[i]) + a.pre_eps;
      a.post_out[tt * 4 + i] = sigmoidf(mx[4 + i] * a.scale[1] + a.base[4 + i]) * a.post_mult;
    }
    float cb[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cb[i][j] = mx[8 + i * 4 + j] * a.scale[2] + a.base[8 + i * 4 + j];
        m = fmaxf(m, cb[i][j]);
      }
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cb[i][j] = expf(cb[i][j] - m);
        s += cb[i][j];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) cb[i][j] = cb[i][j] / s + a.sinkhorn_eps;
    }
    auto col_norm = [&]() {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s = cb[0][j] + cb[1][j] + cb[2][j] + cb[3][j] + a.sinkhorn_eps;
#pragma unroll
        for (int i = 0; i < 4; ++i) cb[i][j] /= s;
      }
    };
    col_norm();
    for (int r = 1; r < a.repeat; ++r) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float s = cb[i][0] + cb[i][1] + cb[i][2] + cb[i][3] + a.sinkhorn_eps;
#pragma unroll
        for (int j = 0; j < 4; ++j) cb[i][j] /= s;
      }
      col_norm();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) a.comb_out[tt * 16 + i * 4 + j] = cb[i][j];
  }
  __syncthreads();
  const int tl = tid >> 3;                             // this thread's token in the tile (y passes)
  const int seg = (tid & 7) * 8;                       // its 8 hidden positions in each 64-position step
  const int64_t t = t0 + tl;
  const bool tv = t < a.T;
  // ---- layer input and its RMSNorm: token tl, positions seg + 64 m (two passes over the new residual, from L2) ----
  // (no early return: the 8 lanes of a token reduce with shuffles, so every lane of the warp stays)
  const __nv_bfloat16* src = POST ? a.new_res : a.res;
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = tv ? pre_s[tl][i] : 0.0f;
  float ls = 0.0f;
  // two positions groups per iteration, all loads issued before the stores (the stores to y could alias src for all
  // the compiler knows)
  for (int64_t hh = seg; tv && hh < H; hh += 2 * kMhcH) {
    const bool two = hh + kMhcH < H;
    uint4 rv[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        rv[u][i] = (u == 0 || two) ? *reinterpret_cast<const uint4*>(src + (t * 4 + i) * H + hh + u * kMhcH)
                                   : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (u == 1 && !two) break;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          v = fmaf(p[i], __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv[u][i])[e]), v);
        const __nv_bfloat16 b = __float2bfloat16(v);
        const float bv = __bfloat162float(b);
        ls = fmaf(bv, bv, ls);
        if (e & 1) w[e >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16;
        else w[e >> 1] = __bfloat16_as_ushort(b);
      }
      *reinterpret_cast<uint4*>(a.y + t * H + hh + u * kMhcH) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) ls += __shfl_xor_sync(0xFFFFFFFFu, ls, off);
  const float inv = rsqrtf(ls / static_cast<float>(H) + a.norm_eps);
  for (int64_t hh = seg; tv && hh < H; hh += 4 * kMhcH) {
    uint4 v[4], wv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (hh + u * kMhcH < H) {
        v[u] = *reinterpret_cast<const uint4*>(a.y + t * H + hh + u * kMhcH);
        wv[u] = *reinterpret_cast<const uint4*>(a.norm_w + hh + u * kMhcH);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (hh + u * kMhcH >= H) break;
      __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&v[u]);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) vb[e] = __float2bfloat16(__bfloat162float(vb[e]) * inv * __bfloat162float(wb[e]));
      *reinterpret_cast<uint4*>(a.y + t * H + hh + u * kMhcH) = v[u];
    }
  }
}

// ---- split pre path: the mix kernel (post + partial mixes) and the finalize kernel (the partials summed in a fixed
//      order, Sinkhorn, the layer input and its RMSNorm) ----
//
// Mix: persistent, one CTA per SM over work items of 64 tokens x one eighth of the hidden positions (of every
// stream). A producer thread streams each 32-position group of an item through a 4-stage ring by TMA: the 4 residual
// streams [64 tokens x 32 positions] bf16 (one box per stream, so a stream's rows are adjacent: conflict-free reads),
// x (post) and the fn rows [24 x 32] fp32 of the 4 streams (128-byte swizzle). Eight consumer warps: warp w takes
// tokens 16 (w & 3) .. + 15 and output streams 2 (w >> 2), + 1; each lane covers 2 tokens x 8 consecutive positions
// (the MMA fragment layout), forms the new residual of its streams (bf16, stored straight to HBM) and feeds it as tf32
// mma.sync fragments against the fn rows; the sums of squares go alongside. Partial mixes of (eighth, stream half)
// go to the workspace: kMixParts partials per token, summed by the finalize kernel in a fixed order.
constexpr int kMixTok = 64;                      // tokens per work item
constexpr int kMixEighths = 8;                   // position ranges per item row
constexpr int kMixParts = 2 * kMixEighths;       // partials per token: (eighth, stream half)
constexpr int kMixStages = 3;
constexpr int kMixConsumers = 8;                 // consumer warps
constexpr int kMixThreads = 32 * (kMixConsumers + 1);
constexpr int kMixHalves = 2;                    // a stage holds 2 x 32 positions: 128 contiguous bytes of every row
constexpr int kMixRes = 0;                       // stage: res [half][4][64][32] bf16, 4 KB a box
constexpr int kMixX = kMixHalves * 4 * 4096;     // x [half][64][32] bf16
constexpr int kMixFn = kMixX + kMixHalves * 4096;        // fn [half][4][24][32] fp32, 3 KB a box, 128-byte swizzle
constexpr int kMixStage = kMixFn + kMixHalves * 4 * 3072;   // 64 KB
constexpr int kMixBar = kMixStages * kMixStage;  // full[4], empty[4], abort flag
constexpr int kMixSmem = kMixBar + 128 + 1024;   // + alignment slack (1024-byte aligned stages)

template <bool POST>
__global__ void __launch_bounds__(kMixThreads, 1)
    mhc_mix_kernel(const __grid_constant__ CUtensorMap mres, const __grid_constant__ CUtensorMap mx,
                   const __grid_constant__ CUtensorMap mfn, const MhcArgs a, float* part, float* part_ss) {
  extern __shared__ uint8_t mix_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mix_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t full0 = sb + kMixBar, empty0 = full0 + 8 * kMixStages;
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + kMixBar + 16 * kMixStages);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int64_t H = a.H;
  const int ranges = a.ranges;                                     // position ranges an item row is cut into
  const int groups = static_cast<int>(H / ranges / (32 * kMixHalves));    // 64-position groups of an item
  const int64_t n_items = (a.T + kMixTok - 1) / kMixTok * ranges;
  if (tid == 0) {
    for (int s = 0; s < kMixStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kMixConsumers);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kMixConsumers) {
    // ---------------------------------------------------------------- producer (one thread)
    if (lane == 0) {
      tma_prefetch_desc(&mres);
      tma_prefetch_desc(&mfn);
      if (POST) tma_prefetch_desc(&mx);
      constexpr uint32_t kBytes = kMixHalves * (4 * 4096 + (POST ? 4096 : 0) + 4 * 3072);
      int64_t n = 0;                                           // groups issued so far
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
        const int32_t t0 = static_cast<int32_t>((it / ranges) * kMixTok);
        const int32_t g0 = static_cast<int32_t>((it % ranges) * (H / ranges));
        for (int gi = 0; gi < groups; ++gi, ++n) {
          const int s = static_cast<int>(n % kMixStages);
          if (n >= kMixStages &&
              !mbar_wait(empty0 + 8 * s, static_cast<uint32_t>((n / kMixStages - 1) & 1), abort_flag, a.status)) {
            ok = false;
            break;
          }
          const uint32_t st = sb + s * kMixStage, fb = full0 + 8 * s;
          const int32_t g = g0 + 32 * kMixHalves * gi;
          mbar_arrive_expect_tx(fb, kBytes);
          // the two halves of a row back to back: one 128-byte run of each row per stage
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int hb = 0; hb < kMixHalves; ++hb)
              tma_load_2d(st + kMixRes + (hb * 4 + i) * 4096, &mres, static_cast<int32_t>(i * H) + g + 32 * hb, t0, fb);
          if (POST)
#pragma unroll
            for (int hb = 0; hb < kMixHalves; ++hb) tma_load_2d(st + kMixX + hb * 4096, &mx, g + 32 * hb, t0, fb);
#pragma unroll
          for (int hb = 0; hb < kMixHalves; ++hb)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              tma_load_2d(st + kMixFn + (hb * 4 + i) * 3072, &mfn, static_cast<int32_t>(i * H) + g + 32 * hb, 0, fb);
        }
      }
      // the copies in flight land before the CTA exits (bounded; normally every stage was consumed already)
      for (int64_t m = n > kMixStages ? n - kMixStages : 0; m < n; ++m) {
        const uint32_t fb = full0 + 8 * static_cast<int>(m % kMixStages);
        const uint32_t par = static_cast<uint32_t>((m / kMixStages) & 1);
        const unsigned long long w0 = globaltimer();
        while (!mbar_try_wait(fb, par) && globaltimer() - w0 < kWaitNs) {
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int tr0 = 16 * (warp & 3) + g8, tr1 = tr0 + 8, sh = warp >> 2;
  int64_t n = 0;
  for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x) {
    const int64_t t0 = (it / ranges) * kMixTok;
    const int e = static_cast<int>(it % ranges);
    const int64_t r0 = t0 + tr0, r1 = t0 + tr1;
    const bool v0 = r0 < a.T, v1 = r1 < a.T;
    // post[j] and comb[i][j] of this lane's two tokens for its two output streams j = 2 sh, 2 sh + 1, as pairs
    uint64_t c0[2][5], c1[2][5];
    if (POST) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * sh + jj;
        const float p0 = v0 ? a.post_in[r0 * 4 + j] : 0.0f, p1 = v1 ? a.post_in[r1 * 4 + j] : 0.0f;
        c0[jj][0] = f2pack(p0, p0);
        c1[jj][0] = f2pack(p1, p1);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float q0 = v0 ? a.comb_in[r0 * 16 + i * 4 + j] : 0.0f, q1 = v1 ? a.comb_in[r1 * 16 + i * 4 + j] : 0.0f;
          c0[jj][1 + i] = f2pack(q0, q0);
          c1[jj][1 + i] = f2pack(q1, q1);
        }
      }
    }
    float macc[3][4] = {};
    uint64_t ss0 = 0, ss1 = 0;                                  // packed sums of squares (even, odd positions)
    bool ok = true;
    for (int gi = 0; gi < groups; ++gi, ++n) {
      const int s = static_cast<int>(n % kMixStages);
      if (!mbar_wait(full0 + 8 * s, static_cast<uint32_t>((n / kMixStages) & 1), abort_flag, a.status)) {
        ok = false;
        break;
      }
#pragma unroll 1
      for (int hb = 0; hb < kMixHalves; ++hb) {
      const uint8_t* st0 = smem + s * kMixStage;
      const uint8_t* st = st0 + kMixRes + hb * (4 * 4096);              // this half's residual boxes
      const uint8_t* stx = st0 + kMixX + hb * 4096;                     // its x box
      const uint8_t* stf = st0 + kMixFn + hb * (4 * 3072);              // its fn boxes
      const int64_t h = e * (H / ranges) + 32 * (kMixHalves * gi + hb) + 8 * t4;   // this lane's first position
      // the new residual of this lane's two output streams, bf16 pairs: w[token][stream][pair]
      uint32_t w[2][2][4];
      if (POST) {
        auto mix_token = [&](int tr, const uint64_t (&c)[2][5], uint32_t (&wt)[2][4]) {
          const uint4 xv = *reinterpret_cast<const uint4*>(stx + tr * 64 + t4 * 16);
          uint4 rv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) rv[i] = *reinterpret_cast<const uint4*>(st + i * 4096 + tr * 64 + t4 * 16);
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint64_t xf = bf2_f2(xw[q]);
            uint64_t rf[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) rf[i] = bf2_f2(reinterpret_cast<const uint32_t*>(&rv[i])[q]);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              uint64_t acc = mul2(c[jj][0], xf);                // post[j] x + sum_i comb[i][j] res_i, in that order
#pragma unroll
              for (int i = 0; i < 4; ++i) acc = fma2(c[jj][1 + i], rf[i], acc);
              wt[jj][q] = f2_bf2(acc);
            }
          }
        };
        mix_token(tr0, c0, w[0]);
        mix_token(tr1, c1, w[1]);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * sh + jj;
          if (v0) *reinterpret_cast<uint4*>(a.new_res + (r0 * 4 + j) * H + h) = make_uint4(w[0][jj][0], w[0][jj][1], w[0][jj][2], w[0][jj][3]);
          if (v1) *reinterpret_cast<uint4*>(a.new_res + (r1 * 4 + j) * H + h) = make_uint4(w[1][jj][0], w[1][jj][1], w[1][jj][2], w[1][jj][3]);
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * sh + jj;
          const uint4 q0 = *reinterpret_cast<const uint4*>(st + j * 4096 + tr0 * 64 + t4 * 16);
          const uint4 q1 = *reinterpret_cast<const uint4*>(st + j * 4096 + tr1 * 64 + t4 * 16);
          w[0][jj][0] = q0.x; w[0][jj][1] = q0.y; w[0][jj][2] = q0.z; w[0][jj][3] = q0.w;
          w[1][jj][0] = q1.x; w[1][jj][1] = q1.y; w[1][jj][2] = q1.z; w[1][jj][3] = q1.w;
        }
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * sh + jj;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint64_t z0 = bf2_f2(w[0][jj][q]), z1 = bf2_f2(w[1][jj][q]);
          ss0 = fma2(z0, z0, ss0);
          ss1 = fma2(z1, z1, ss1);
        }
        const uint8_t* fs = stf + j * 3072;
#pragma unroll
        for (int nt = 0; nt < 3; ++nt) {
          const int row = 8 * nt + g8;
          const float4 f0 = *reinterpret_cast<const float4*>(fs + row * 128 + (((2 * t4) ^ (row & 7)) << 4));
          const float4 f1 = *reinterpret_cast<const float4*>(fs + row * 128 + (((2 * t4 + 1) ^ (row & 7)) << 4));
          const float fb[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2) {
            uint32_t b0, b1;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b0) : "f"(fb[2 * s2]));
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b1) : "f"(fb[2 * s2 + 1]));
            // k index t4: position 2 s2 of the lane's 8, k index t4 + 4: position 2 s2 + 1 (bf16 bits are exact tf32)
            asm volatile(
                "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(macc[nt][0]), "+f"(macc[nt][1]), "+f"(macc[nt][2]), "+f"(macc[nt][3])
                : "r"(w[0][jj][s2] << 16), "r"(w[1][jj][s2] << 16), "r"(w[0][jj][s2] & 0xFFFF0000u),
                  "r"(w[1][jj][s2] & 0xFFFF0000u), "r"(b0), "r"(b1));
          }
        }
      }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);               // this warp is done with the stage
    }
    if (!ok) break;
    // this item's partial (eighth e, stream half sh): mixes [T][24] and the sum of squares [T]
    float ssa, ssb, sq0, sq1;
    f2unpack(ss0, ssa, ssb);
    sq0 = ssa + ssb;
    f2unpack(ss1, ssa, ssb);
    sq1 = ssa + ssb;
    sq0 += __shfl_xor_sync(0xFFFFFFFFu, sq0, 1);
    sq0 += __shfl_xor_sync(0xFFFFFFFFu, sq0, 2);
    sq1 += __shfl_xor_sync(0xFFFFFFFFu, sq1, 1);
    sq1 += __shfl_xor_sync(0xFFFFFFFFu, sq1, 2);
    const int p = 2 * e + sh;
    float* pq = part + static_cast<int64_t>(p) * a.T * kMhcMix;
    if (t4 == 0) {
      if (v0) part_ss[p * a.T + r0] = sq0;
      if (v1) part_ss[p * a.T + r1] = sq1;
    }
#pragma unroll
    for (int nt = 0; nt < 3; ++nt) {
      if (v0) *reinterpret_cast<float2*>(pq + r0 * kMhcMix + 8 * nt + 2 * t4) = make_float2(macc[nt][0], macc[nt][1]);
      if (v1) *reinterpret_cast<float2*>(pq + r1 * kMhcMix + 8 * nt + 2 * t4) = make_float2(macc[nt][2], macc[nt][3]);
    }
  }
}

// Finalize: 16 tokens per CTA, 16 threads a token in the y passes (two 128-position steps of loads in flight), up
// to four CTAs an SM: at T = 8192 every CTA is resident at once.
constexpr int kFinTok = 16;

template <bool POST>
__global__ void __launch_bounds__(kMhcThreads, 4) mhc_final_kernel(const MhcArgs a, const float* part,
                                                                    const float* part_ss) {
  __shared__ float mix[kFinTok][kMhcMix];
  __shared__ float ssq[kFinTok];
  __shared__ float pre_s[kFinTok][4];
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kFinTok;
  const int64_t H = a.H;
  const int64_t QT = a.T * kMhcMix;
  for (int i = tid; i < kFinTok * kMhcMix; i += kMhcThreads) {
    const int tk = i / kMhcMix, c = i % kMhcMix;
    const int64_t o = (t0 + tk) * kMhcMix + c;
    float v = 0.0f;                                    // the mix kernel's partials in a fixed order
    if (t0 + tk < a.T) {
#pragma unroll
      for (int q = 0; q < kMixParts; ++q)
        if (q < 2 * a.ranges) v += part[q * QT + o];
    }
    mix[tk][c] = v;
  }
  if (tid < kFinTok) {
    const int64_t tt = t0 + tid;
    float v = 0.0f;
    if (tt < a.T) {
#pragma unroll
      for (int q = 0; q < kMixParts; ++q)
        if (q < 2 * a.ranges) v += part_ss[q * a.T + tt];
    }
    ssq[tid] = v;
  }
  __syncthreads();
  if (tid < kFinTok && t0 + tid < a.T) {
    const int64_t tt = t0 + tid;
    const float rinv = rsqrtf(ssq[tid] / static_cast<float>(4 * H) + a.rms_eps);
    float mx[kMhcMix];
#pragma unroll
    for (int c = 0; c < kMhcMix; ++c) mx[c] = mix[tid][c] * rinv;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pre_s[tid][i] = sigmoidf(mx[i] * a.scale[0] + a.base[i]) + a.pre_eps;
      a.post_out[tt * 4 + i] = sigmoidf(mx[4 + i] * a.scale[1] + a.base[4 + i]) * a.post_mult;
    }
    float cb[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cb[i][j] = mx[8 + i * 4 + j] * a.scale[2] + a.base[8 + i * 4 + j];
        m = fmaxf(m, cb[i][j]);
      }
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cb[i][j] = expf(cb[i][j] - m);
        s += cb[i][j];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) cb[i][j] = cb[i][j] / s + a.sinkhorn_eps;
    }
    auto col_norm = [&]() {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s = cb[0][j] + cb[1][j] + cb[2][j] + cb[3][j] + a.sinkhorn_eps;
#pragma unroll
        for (int i = 0; i < 4; ++i) cb[i][j] /= s;
      }
    };
    col_norm();
    for (int r = 1; r < a.repeat; ++r) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float s = cb[i][0] + cb[i][1] + cb[i][2] + cb[i][3] + a.sinkhorn_eps;
#pragma unroll
        for (int j = 0; j < 4; ++j) cb[i][j] /= s;
      }
      col_norm();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) a.comb_out[tt * 16 + i * 4 + j] = cb[i][j];
  }
  __syncthreads();
  const int tl = tid >> 4;                             // this thread's token in the tile (y passes)
  const int seg = (tid & 15) * 8;                      // its 8 hidden positions in each 128-position step
  const int64_t t = t0 + tl;
  const bool tv = t < a.T;
  constexpr int kStep = 128, kU = 2;
  // ---- layer input and its RMSNorm: token tl, positions seg + 128 m (two passes over the new residual, from L2) ----
  // (no early return: the 16 lanes of a token reduce with shuffles, so every lane of the warp stays)
  const __nv_bfloat16* src = POST ? a.new_res : a.res;
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = tv ? pre_s[tl][i] : 0.0f;
  float ls = 0.0f;
  // kU steps per iteration, all loads issued before the stores (the stores to y could alias src for all the compiler
  // knows)
  for (int64_t hh = seg; tv && hh < H; hh += kU * kStep) {
    uint4 rv[kU][4];
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        rv[u][i] = hh + u * kStep < H ? *reinterpret_cast<const uint4*>(src + (t * 4 + i) * H + hh + u * kStep)
                                      : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (hh + u * kStep >= H) break;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          v = fmaf(p[i], __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv[u][i])[e]), v);
        const __nv_bfloat16 b = __float2bfloat16(v);
        const float bv = __bfloat162float(b);
        ls = fmaf(bv, bv, ls);
        if (e & 1) w[e >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16;
        else w[e >> 1] = __bfloat16_as_ushort(b);
      }
      *reinterpret_cast<uint4*>(a.y + t * H + hh + u * kStep) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ls += __shfl_xor_sync(0xFFFFFFFFu, ls, off);
  const float inv = rsqrtf(ls / static_cast<float>(H) + a.norm_eps);
  for (int64_t hh = seg; tv && hh < H; hh += kU * kStep) {
    uint4 v[kU], wv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (hh + u * kStep < H) {
        v[u] = *reinterpret_cast<const uint4*>(a.y + t * H + hh + u * kStep);
        wv[u] = *reinterpret_cast<const uint4*>(a.norm_w + hh + u * kStep);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (hh + u * kStep >= H) break;
      __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&v[u]);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) vb[e] = __float2bfloat16(__bfloat162float(vb[e]) * inv * __bfloat162float(wb[e]));
      *reinterpret_cast<uint4*>(a.y + t * H + hh + u * kStep) = v[u];
    }
  }
}

}  // namespace

int64_t mhc_workspace_bytes(int64_t T) {
  return T <= 0 ? 0 : kMixParts * T * (kMhcMix + 1) * static_cast<int64_t>(sizeof(float));
}

int launch_mhc(bool do_post, bool do_pre, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, const float* fn, const float* scale, const float* base, const void* norm_w,
               float* post_out, float* comb_out, void* y, int64_t T, int64_t H, float rms_eps, float pre_eps,
               float sinkhorn_eps, float post_mult, int repeat, float norm_eps, void* ws, int64_t ws_bytes,
               int32_t* status, cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % 128 != 0 || repeat < 1 || (!do_post && !do_pre)) return kErrArgs;
  if (T == 0) return kOk;
  MhcArgs a{reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(res), post_in, comb_in,
            reinterpret_cast<__nv_bfloat16*>(new_res), fn, scale, base,
            reinterpret_cast<const __nv_bfloat16*>(norm_w), post_out, comb_out, reinterpret_cast<__nv_bfloat16*>(y),
            T, H, rms_eps, pre_eps, sinkhorn_eps, post_mult, norm_eps, repeat, status,
            H % (kMixEighths * 64) == 0 ? kMixEighths : kMixEighths / 2};
  if (!do_pre) {
    mhc_kernel<true, false><<<static_cast<unsigned>((T + kMhcTok - 1) / kMhcTok), kMhcThreads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
  }
  if (H % (kMixEighths / 2 * 64) != 0) return kErrArgs;   // a pre step covers H in 4 or 8 ranges of 64-wide groups
  const int64_t need = mhc_workspace_bytes(T);
  bool own = false;
  if (ws == nullptr) {                                   // no caller workspace: a stream-ordered allocation
    if (cudaMallocAsync(&ws, need, stream) != cudaSuccess) return kErrCuda;
    own = true;
  } else if (ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 15)) {
    return kErrWorkspace;
  }
  float* part = static_cast<float*>(ws);
  float* part_ss = part + kMixParts * T * kMhcMix;
  int rc = kOk;
  // tensor maps: the residual as [T, 4H] bf16 (one 32 x 64 box per stream), x as [T, H], fn as [24, 4H] fp32 (one
  // 32 x 24 box per stream, 128-byte swizzle); T and H are the only extents (rows past T read as zeros)
  CUtensorMap mres, mx, mfn;
  if (reinterpret_cast<uintptr_t>(fn) & 15) rc = kErrArgs;
  if (rc == kOk)
    rc = make_map_2d(&mres, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, res, T, 4 * H, 4 * H * 2, 32, kMixTok);
  if (rc == kOk)
    rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, do_post ? x : res, T, H, (do_post ? H : 4 * H) * 2, 32,
                     kMixTok);
  if (rc == kOk) rc = make_map_2d_ex(&mfn, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, fn, kMhcMix, 4 * H, 4 * H * 4, 32,
                                     kMhcMix, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == kOk) {
    static bool attr = false;
    if (!attr) {
      if (cudaFuncSetAttribute(mhc_mix_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMixSmem) !=
              cudaSuccess ||
          cudaFuncSetAttribute(mhc_mix_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMixSmem) !=
              cudaSuccess)
        rc = kErrCuda;
      else
        attr = true;
    }
  }
  if (rc == kOk) {
    const int64_t items = (T + kMixTok - 1) / kMixTok * a.ranges;
    const unsigned gmix = static_cast<unsigned>(std::min<int64_t>(items, device_sm_count()));
    const unsigned gfin = static_cast<unsigned>((T + kFinTok - 1) / kFinTok);
    if (do_post) {
      mhc_mix_kernel<true><<<gmix, kMixThreads, kMixSmem, stream>>>(mres, mx, mfn, a, part, part_ss);
      mhc_final_kernel<true><<<gfin, kMhcThreads, 0, stream>>>(a, part, part_ss);
    } else {
      mhc_mix_kernel<false><<<gmix, kMixThreads, kMixSmem, stream>>>(mres, mx, mfn, a, part, part_ss);
      mhc_final_kernel<false><<<gfin, kMhcThreads, 0, stream>>>(a, part, part_ss);
    }
    rc = cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
  }
  if (own && cudaFreeAsync(ws, stream) != cudaSuccess && rc == kOk) rc = kErrCuda;
  return rc;
}

}  // namespace ssb
