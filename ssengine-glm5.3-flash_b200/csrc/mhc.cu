// mHC (4-stream hyper-connections) at a layer boundary, one fused kernel (sm_100a).
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

// ---- split pre path: the mix kernel (post + partial mixes over one quarter of the hidden positions for 128 tokens,
//      the fn rows of each 32-position group staged once in shared memory for all 8 warps) and the finalize kernel
//      (the quarters' partials summed in a fixed order, Sinkhorn, the layer input and its RMSNorm) ----
constexpr int kMixTok = 128;                     // tokens per CTA of the mix kernel: 8 warps x 16
constexpr int kFnStride = 132;                   // floats per staged fn row: 528 B, conflict-free 16-byte fragment loads
constexpr int kFnStage = kMhcMix * kFnStride;    // one group: 24 rows x [4 streams x 32 positions]

SSB_DEVICE void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <bool POST>
__global__ void __launch_bounds__(kMhcThreads, 2) mhc_mix_kernel(const MhcArgs a, float* part, float* part_ss) {
  __shared__ __align__(16) float fns[2][kFnStage];
  __shared__ __align__(16) float coef[POST ? kMixTok : 1][4][8];   // token, output stream j: post[j], comb[0..3][j]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kMixTok;
  const int kq = blockIdx.y;
  const int64_t H = a.H;
  const int64_t gb = kq * (H / 4), ge = gb + H / 4;
  auto stage_fn = [&](int64_t g, int st) {           // 768 pieces of 16 B: row, stream, 4 positions
    for (int i = tid; i < kMhcMix * 32; i += kMhcThreads) {
      const int row = i >> 5, j = (i >> 3) & 3, pc = i & 7;
      cp_async16(smem_u32(&fns[st][row * kFnStride + j * 32 + pc * 4]),
                 a.fn + static_cast<int64_t>(row) * 4 * H + j * H + g + pc * 4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  stage_fn(gb, 0);
  if (POST) {
    for (int i = tid; i < kMixTok * 4; i += kMhcThreads) {
      const int tk = i >> 2, j = i & 3;
      const int64_t tt = t0 + tk;
      float* d = coef[tk][j];
      const bool ok = tt < a.T;
      d[0] = ok ? a.post_in[tt * 4 + j] : 0.0f;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) d[1 + ii] = ok ? a.comb_in[tt * 16 + ii * 4 + j] : 0.0f;
    }
  }
  const int tr0 = 16 * warp + g8, tr1 = tr0 + 8;
  const int64_t r0 = t0 + tr0, r1 = t0 + tr1;
  const bool v0 = r0 < a.T, v1 = r1 < a.T;
  float macc[3][4] = {};
  float ss0 = 0.0f, ss1 = 0.0f;
  const uint4 zero4 = make_uint4(0, 0, 0, 0);
  int st = 0;
  for (int64_t g = gb; g < ge; g += 32, st ^= 1) {
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
    if (g + 32 < ge) {
      stage_fn(g + 32, st ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();                                   // this group's fn rows (and the coefficients) visible
    const float* fs = fns[st];
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
        const uint4 n0 = mixrow(xv0, rv0, coef[POST ? tr0 : 0][j], z0);
        const uint4 n1 = mixrow(xv1, rv1, coef[POST ? tr1 : 0][j], z1);
        if (v0) *reinterpret_cast<uint4*>(a.new_res + (r0 * 4 + j) * H + h) = n0;
        if (v1) *reinterpret_cast<uint4*>(a.new_res + (r1 * 4 + j) * H + h) = n1;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          z0[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv0[j])[e]);
          z1[e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv1[j])[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss0 = fmaf(z0[e], z0[e], ss0);
        ss1 = fmaf(z1[e], z1[e], ss1);
      }
#pragma unroll
      for (int nt = 0; nt < 3; ++nt) {
        const float* fr = fs + (8 * nt + g8) * kFnStride + j * 32 + 8 * t4;
        const float4 f0 = *reinterpret_cast<const float4*>(fr), f1 = *reinterpret_cast<const float4*>(fr + 4);
        const float fb[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
          uint32_t b0, b1;
          asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b0) : "f"(fb[2 * s2]));
          asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b1) : "f"(fb[2 * s2 + 1]));
          asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                       "{%0,%1,%2,%3};"
                       : "+f"(macc[nt][0]), "+f"(macc[nt][1]), "+f"(macc[nt][2]), "+f"(macc[nt][3])
                       : "r"(__float_as_uint(z0[2 * s2])), "r"(__float_as_uint(z1[2 * s2])),
                         "r"(__float_as_uint(z0[2 * s2 + 1])), "r"(__float_as_uint(z1[2 * s2 + 1])), "r"(b0), "r"(b1));
        }
      }
    }
    __syncthreads();                                   // all warps done with this stage before it is refilled
  }
  // partials of this quarter: mixes [T][24] and sums of squares [T]
  ss0 += __shfl_xor_sync(0xFFFFFFFFu, ss0, 1);
  ss0 += __shfl_xor_sync(0xFFFFFFFFu, ss0, 2);
  ss1 += __shfl_xor_sync(0xFFFFFFFFu, ss1, 1);
  ss1 += __shfl_xor_sync(0xFFFFFFFFu, ss1, 2);
  float* pq = part + static_cast<int64_t>(kq) * a.T * kMhcMix;
  if (t4 == 0) {
    if (v0) part_ss[kq * a.T + r0] = ss0;
    if (v1) part_ss[kq * a.T + r1] = ss1;
  }
#pragma unroll
  for (int nt = 0; nt < 3; ++nt) {
    if (v0) *reinterpret_cast<float2*>(pq + r0 * kMhcMix + 8 * nt + 2 * t4) = make_float2(macc[nt][0], macc[nt][1]);
    if (v1) *reinterpret_cast<float2*>(pq + r1 * kMhcMix + 8 * nt + 2 * t4) = make_float2(macc[nt][2], macc[nt][3]);
  }
}

template <bool POST>
__global__ void __launch_bounds__(kMhcThreads, 2) mhc_final_kernel(const MhcArgs a, const float* part,
                                                                    const float* part_ss) {
  __shared__ float mix[kMhcTok][kMhcMix];
  __shared__ float ssq[kMhcTok];
  __shared__ float pre_s[kMhcTok][4];
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kMhcTok;
  const int64_t H = a.H;
  const int64_t QT = a.T * kMhcMix;
  for (int i = tid; i < kMhcTok * kMhcMix; i += kMhcThreads) {
    const int tk = i / kMhcMix, c = i % kMhcMix;
    const int64_t o = (t0 + tk) * kMhcMix + c;
    mix[tk][c] = t0 + tk < a.T ? ((part[o] + part[QT + o]) + part[2 * QT + o]) + part[3 * QT + o] : 0.0f;
  }
  if (tid < kMhcTok) {
    const int64_t tt = t0 + tid;
    ssq[tid] = tt < a.T ? ((part_ss[tt] + part_ss[a.T + tt]) + part_ss[2 * a.T + tt]) + part_ss[3 * a.T + tt] : 0.0f;
  }
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

}  // namespace

int64_t mhc_workspace_bytes(int64_t T) { return T <= 0 ? 0 : 4 * T * (kMhcMix + 1) * static_cast<int64_t>(sizeof(float)); }

int launch_mhc(bool do_post, bool do_pre, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, const float* fn, const float* scale, const float* base, const void* norm_w,
               float* post_out, float* comb_out, void* y, int64_t T, int64_t H, float rms_eps, float pre_eps,
               float sinkhorn_eps, float post_mult, int repeat, float norm_eps, void* ws, int64_t ws_bytes,
               cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % 128 != 0 || repeat < 1 || (!do_post && !do_pre)) return kErrArgs;
  if (T == 0) return kOk;
  MhcArgs a{reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(res), post_in, comb_in,
            reinterpret_cast<__nv_bfloat16*>(new_res), fn, scale, base,
            reinterpret_cast<const __nv_bfloat16*>(norm_w), post_out, comb_out, reinterpret_cast<__nv_bfloat16*>(y),
            T, H, rms_eps, pre_eps, sinkhorn_eps, post_mult, norm_eps, repeat};
  if (!do_pre) {
    mhc_kernel<true, false><<<static_cast<unsigned>((T + kMhcTok - 1) / kMhcTok), kMhcThreads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
  }
  const int64_t need = mhc_workspace_bytes(T);
  bool own = false;
  if (ws == nullptr) {                                   // no caller workspace: a stream-ordered allocation
    if (cudaMallocAsync(&ws, need, stream) != cudaSuccess) return kErrCuda;
    own = true;
  } else if (ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 15)) {
    return kErrWorkspace;
  }
  float* part = static_cast<float*>(ws);
  float* part_ss = part + 4 * T * kMhcMix;
  const dim3 gmix(static_cast<unsigned>((T + kMixTok - 1) / kMixTok), 4);
  const unsigned gfin = static_cast<unsigned>((T + kMhcTok - 1) / kMhcTok);
  if (do_post) {
    mhc_mix_kernel<true><<<gmix, kMhcThreads, 0, stream>>>(a, part, part_ss);
    mhc_final_kernel<true><<<gfin, kMhcThreads, 0, stream>>>(a, part, part_ss);
  } else {
    mhc_mix_kernel<false><<<gmix, kMhcThreads, 0, stream>>>(a, part, part_ss);
    mhc_final_kernel<false><<<gfin, kMhcThreads, 0, stream>>>(a, part, part_ss);
  }
  int rc = cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
  if (own && cudaFreeAsync(ws, stream) != cudaSuccess && rc == kOk) rc = kErrCuda;
  return rc;
}

}  // namespace ssb
