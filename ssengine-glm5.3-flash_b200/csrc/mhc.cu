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
// CTA = 32 tokens, 256 threads; K (= 4H) is walked in chunks of 64 hidden positions x 4 streams: each thread
// computes 8 positions x 4 streams of one token (16-byte vector loads of x and the 4 residual streams), stores the
// new residual, and stages the chunk (fp32) and the chunk's 24 fn rows in shared memory; then each thread
// accumulates 3 of the 32 x 24 mix dot products. HBM traffic per token: 40 KB in (x + res), 32 KB new residual and
// 8 KB y out; the new residual is re-read from L2 for the layer input.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

constexpr int kMhcTok = 32;       // tokens per CTA
constexpr int kMhcThreads = 256;
constexpr int kMhcH = 64;         // hidden positions per K chunk (x 4 streams = 256 K)
constexpr int kMhcK = 4 * kMhcH;
constexpr int kMhcMix = 24;
constexpr int kFnPitch = kMhcK + 4;   // 16-byte rows; 260 = 4 (mod 32) spreads the 8 column groups' rows over the banks
constexpr int kZPitch = kMhcK + 4;    // 16-byte rows; the 4 tokens of a warp read 4 different bank groups

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
  extern __shared__ __align__(16) float smem_f[];
  float* zs = smem_f;                                  // [32][257]
  float* fs = zs + kMhcTok * kZPitch;                  // [24][257]
  __shared__ float mix[kMhcTok][kMhcMix];
  __shared__ float ssq[kMhcTok];
  __shared__ float pre_s[kMhcTok][4];
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kMhcTok;
  const int tl = tid >> 3;                             // this thread's token in the tile (chunk phase)
  const int seg = (tid & 7) * 8;                       // its 8 hidden positions inside the chunk
  const int64_t t = t0 + tl;
  const bool tv = t < a.T;
  const int64_t H = a.H;
  float pm[4] = {0, 0, 0, 0}, cm[4][4];
  if (POST && tv) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pm[i] = a.post_in[t * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) cm[i][j] = a.comb_in[t * 16 + i * 4 + j];
    }
  }
  float macc[2][3][4] = {};                            // mix partials: token tiles x mix tiles (mma accumulators)
  const int warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  float ss = 0.0f;
  // x / res rows of the next chunk are loaded while the current one is mixed (software pipeline over the K chunks)
  uint4 rv_next[4], xv_next = make_uint4(0, 0, 0, 0);
  if (tv) {
#pragma unroll
    for (int i = 0; i < 4; ++i) rv_next[i] = *reinterpret_cast<const uint4*>(a.res + (t * 4 + i) * H + seg);
    if (POST) xv_next = *reinterpret_cast<const uint4*>(a.x + t * H + seg);
  }
  for (int64_t h0 = 0; h0 < H; h0 += kMhcH) {
    // ---- new residual of this chunk (all 4 streams, 8 positions per thread) ----
    float nr[4][8];
    if (tv) {
      const int64_t hh = h0 + seg;
      uint4 rv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rv[i] = rv_next[i];
      const uint4 xv = xv_next;
      if (h0 + kMhcH < H) {
#pragma unroll
        for (int i = 0; i < 4; ++i) rv_next[i] = *reinterpret_cast<const uint4*>(a.res + (t * 4 + i) * H + hh + kMhcH);
        if (POST) xv_next = *reinterpret_cast<const uint4*>(a.x + t * H + hh + kMhcH);
      }
      if (POST) {
        const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float v = pm[j] * __bfloat162float(xb[e]);
#pragma unroll
            for (int i = 0; i < 4; ++i) v = fmaf(cm[i][j], __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv[i])[e]), v);
            const __nv_bfloat16 b = __float2bfloat16(v);
            nr[j][e] = __bfloat162float(b);
            if (e & 1) w[e >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16;
            else w[e >> 1] = __bfloat16_as_ushort(b);
          }
          *reinterpret_cast<uint4*>(a.new_res + (t * 4 + j) * H + hh) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) nr[j][e] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&rv[j])[e]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) nr[j][e] = 0.0f;
    }
    if (PRE) {
      // stage the chunk: z[tl][j * 64 + seg + e], fn rows [c][j * 64 + hh]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(nr[j][e], nr[j][e], ss);
        *reinterpret_cast<float4*>(zs + tl * kZPitch + j * kMhcH + seg) = make_float4(nr[j][0], nr[j][1], nr[j][2], nr[j][3]);
        *reinterpret_cast<float4*>(zs + tl * kZPitch + j * kMhcH + seg + 4) =
            make_float4(nr[j][4], nr[j][5], nr[j][6], nr[j][7]);
      }
      for (int i = tid; i < kMhcMix * kMhcK / 4; i += kMhcThreads) {
        const int c = i / (kMhcK / 4), kk = (i - c * (kMhcK / 4)) * 4;
        const int j = kk / kMhcH, hh = kk - j * kMhcH;
        *reinterpret_cast<float4*>(fs + c * kFnPitch + kk) =
            __ldg(reinterpret_cast<const float4*>(a.fn + static_cast<int64_t>(c) * 4 * H + j * H + h0 + hh));
      }
      __syncthreads();
      // mixes[32 tokens x 24] += z[32 x 256] fn_chunk^T on the tensor cores (tf32 m16n8k8; z is bf16-exact in tf32):
      // warp w takes k-steps 4w .. 4w + 3 for all 2 x 3 (token, mix) tiles
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        const int k0 = (4 * warp + kq) * 8;
        uint32_t af[2][4], bf[3][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const float* zr0 = zs + (16 * mt + g8) * kZPitch + k0 + t4;
          const float* zr1 = zr0 + 8 * kZPitch;
          af[mt][0] = __float_as_uint(zr0[0]);
          af[mt][1] = __float_as_uint(zr1[0]);
          af[mt][2] = __float_as_uint(zr0[4]);
          af[mt][3] = __float_as_uint(zr1[4]);
        }
#pragma unroll
        for (int nt = 0; nt < 3; ++nt) {
          const float* fr = fs + (8 * nt + g8) * kFnPitch + k0 + t4;
          asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(bf[nt][0]) : "f"(fr[0]));
          asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(bf[nt][1]) : "f"(fr[4]));
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 3; ++nt)
            asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                         "{%0,%1,%2,%3};"
                         : "+f"(macc[mt][nt][0]), "+f"(macc[mt][nt][1]), "+f"(macc[mt][nt][2]), "+f"(macc[mt][nt][3])
                         : "r"(af[mt][0]), "r"(af[mt][1]), "r"(af[mt][2]), "r"(af[mt][3]), "r"(bf[nt][0]),
                           "r"(bf[nt][1]));
      }
      __syncthreads();
    }
  }
  if (!PRE) return;
  // ---- per-token scalars ----
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);   // the 8 threads of a token
  if ((tid & 7) == 0) ssq[tl] = ss;
  // the 8 warps' K-slice partials of the [32 x 24] mixes, summed through shared memory (fs is free now)
  __syncthreads();
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        fs[warp * (kMhcTok * kMhcMix) + (16 * mt + g8 + 8 * (q >> 1)) * kMhcMix + 8 * nt + 2 * t4 + (q & 1)] =
            macc[mt][nt][q];
  __syncthreads();
  for (int i = tid; i < kMhcTok * kMhcMix; i += kMhcThreads) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kMhcThreads / 32; ++w) v += fs[w * (kMhcTok * kMhcMix) + i];
    mix[i / kMhcMix][i % kMhcMix] = v;
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

int launch_mhc(bool do_post, bool do_pre, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, const float* fn, const float* scale, const float* base, const void* norm_w,
               float* post_out, float* comb_out, void* y, int64_t T, int64_t H, float rms_eps, float pre_eps,
               float sinkhorn_eps, float post_mult, int repeat, float norm_eps, cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % kMhcH != 0 || repeat < 1 || (!do_post && !do_pre)) return kErrArgs;
  if (T == 0) return kOk;
  MhcArgs a{reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(res), post_in, comb_in,
            reinterpret_cast<__nv_bfloat16*>(new_res), fn, scale, base,
            reinterpret_cast<const __nv_bfloat16*>(norm_w), post_out, comb_out, reinterpret_cast<__nv_bfloat16*>(y),
            T, H, rms_eps, pre_eps, sinkhorn_eps, post_mult, norm_eps, repeat};
  const int blocks = static_cast<int>((T + kMhcTok - 1) / kMhcTok);
  const size_t smem = (static_cast<size_t>(kMhcTok) * kZPitch + kMhcMix * kFnPitch) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(mhc_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(mhc_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  if (do_post && do_pre)
    mhc_kernel<true, true><<<blocks, kMhcThreads, smem, stream>>>(a);
  else if (do_pre)
    mhc_kernel<false, true><<<blocks, kMhcThreads, smem, stream>>>(a);
  else
    mhc_kernel<true, false><<<blocks, kMhcThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
