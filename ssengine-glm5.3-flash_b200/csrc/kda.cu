// KDA prefill for sm_100a: the width-4 causal conv over the packed q|k|v projection rows, fused into a chunked
// gated delta-rule scan that reads and writes each request's FP32 recurrent state block in place.
//
// Reference behaviour (ssengine/model/pp_patch.py:215-244 `kda_prefill_forward`): conv (kda_conv.py:56-132) into
// contiguous q, k, v; state gather (zero for a fresh request, kda_state.py:19-36); FlashInfer persistent KDA (gate
// lower_bound * sigmoid(exp(A_log) * (g + dt_bias)) and beta sigmoid in kernel, q/k L2-normalised, scale D^-0.5);
// state scatter.
//
// Chunked form, 64-token chunks, with G the per-channel cumulative log decay (G_i includes token i) and S the
// [key, value] state at the chunk start:
//   L[i][j]  = beta_i sum_c k_i[c] k_j[c] exp(G_i[c] - G_j[c])      (j < i)
//   Aqk[i][j] = scale sum_c q_i[c] k_j[c] exp(G_i[c] - G_j[c])      (j <= i)
//   T = (I + L)^-1 diag(beta);  W = T (k * exp(G));  u = T v;  U = u - W S
//   O = scale (q * exp(G)) S + Aqk U;  S' = diag(exp(G_63)) S + (k * exp(G_63 - G))^T U
// Everything up to W and u is independent of S, so one call is three launches:
//   prep  -- one CTA per (chunk, head), all chunks of all sequences at once (two CTAs per SM): conv from TMA tiles,
//            norms, gates, the A blocks, the blocked solve; writes the chunk's image (W, scale q exp G,
//            k exp(G_63 - G), u, Aqk, exp(G_63)) into the workspace;
//   conv state -- each sequence's last 3 x rows into its conv state block (after prep has read the old ones);
//   scan  -- one CTA per (sequence, head, value half): the chunks in order, images double-buffered by bulk copies,
//            the state fp32 in registers, written back at the end.
// The exp(G_i - G_j) factors are split at 16-row block starts r (j <= r <= i), so that every factor stays <= 1 off
// the diagonal blocks and <= exp(-16 * lower_bound) on them: no overflow, tensor-core operands in bf16
// (mma.sync m16n8k16, fp32 accumulate).
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kD = 128;        // key = value head dim
constexpr int kC = 64;         // chunk tokens
constexpr int kKdaThreads = 256;

// bf16 [rows][64] tiles in shared memory, 16-byte chunks XOR-swizzled by (row & 7)
SSB_DEVICE int sw64(int r, int c) { return r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }

SSB_DEVICE void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
SSB_DEVICE void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
SSB_DEVICE void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                         uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
SSB_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
SSB_DEVICE uint32_t scale_bf16x2(uint32_t v, float lo, float hi) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  float2 f = __bfloat1622float2(b);
  return pack_bf16(f.x * lo, f.y * hi);
}

// SiLU of the conv accumulator, a / (1 + e^-a), with CUDA's fast intrinsics (__expf, __fdividef); for a -> -inf the
// quotient goes to 0 (e^-a overflows to inf). Checked against the oracle's exact SiLU within one bf16 step.
SSB_DEVICE float silu_conv(float a) { return __fdividef(a, 1.0f + __expf(-a)); }

SSB_DEVICE void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(b[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// 8 conv outputs (one 16-byte group of channels) from 4 input rows, oldest first; w[c * 4 + tap] (bf16 as f32).
SSB_DEVICE uint4 conv8(const uint4& x0, const uint4& x1, const uint4& x2, const uint4& x3, const float (&w)[32]) {
  float a[8], b[8], c[8], d[8];
  bf16x8_to_f32(x0, a);
  bf16x8_to_f32(x1, b);
  bf16x8_to_f32(x2, c);
  bf16x8_to_f32(x3, d);
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float y[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int ch = 2 * i + j;
      float acc = __fmaf_rn(w[ch * 4 + 0], a[ch], 0.0f);
      acc = __fmaf_rn(w[ch * 4 + 1], b[ch], acc);
      acc = __fmaf_rn(w[ch * 4 + 2], c[ch], acc);
      acc = __fmaf_rn(w[ch * 4 + 3], d[ch], acc);
      y[j] = silu_conv(acc);
    }
    op[i] = pack_bf16(y[0], y[1]);
  }
  return o;
}

SSB_DEVICE void load_w8(const __nv_bfloat16* w, int64_t ch, float (&wf)[32]) {
  const uint4* p = reinterpret_cast<const uint4*>(w + ch * 4);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float f[8];
    bf16x8_to_f32(__ldg(p + i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) wf[8 * i + j] = f[j];
  }
}

// Row t of one sequence [s, e) for the 8 channels at column `col` (< 3P): x for s <= t < e, the conv state row
// t - s + 3 for t < s when the request has one, else 0.
SSB_DEVICE uint4 conv_row(const KdaArgs& a, int64_t t, int s, int e, int blk, int init, int64_t col) {
  if (t >= s && t < e) return __ldg(reinterpret_cast<const uint4*>(a.x + t * a.ldx + col));
  if (t < s && init) {
    return *reinterpret_cast<const uint4*>(a.conv_state + (int64_t)blk * a.cs_stride + (t - s + 3) * (3 * a.P) + col);
  }
  return make_uint4(0, 0, 0, 0);
}

// ---- operand images ------------------------------------------------------------------------------------------------
// [64][128] bf16 matrices as two [64][64] halves (columns 0-63, then 64-127) of 128-byte rows whose 16-byte chunks are
// XOR-swizzled by (row & 7): the layout a 128-byte-swizzled TMA tile lands in (1024-byte aligned); ldmatrix rows of
// one column chunk fall in 8 different bank groups.
SSB_DEVICE int t128(int r, int c) { return ((c >> 6) << 12) + r * 64 + ((((c >> 3) & 7) ^ (r & 7)) << 3) + (c & 7); }
SSB_DEVICE int sw256(int r, int c) { return r * 256 + (((c >> 3) ^ (r & 7)) << 3) + (c & 7); }

SSB_DEVICE float2 ld_bf2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
SSB_DEVICE void st_bf2(__nv_bfloat16* p, float lo, float hi) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16(lo, hi);
}

// Workspace: the chunk bases int32 [R + 1] (header, a 1024-byte multiple), then one image per (chunk slot, head), all
// written by the prep kernel and read by the scan kernel.
struct KdaImg {
  static constexpr int W = 0;          // W = T (beta k exp G), bf16 [64][128] t128
  static constexpr int QT = 16384;     // scale q exp G, bf16 [64][128] t128
  static constexpr int KT = 32768;     // k exp(G_63 - G), bf16 [64][128] t128
  static constexpr int U = 49152;      // u = T (beta v), bf16 [64][128] t128 = value columns 0-63 | 64-127, [64][64] each
  static constexpr int AQK = 65536;    // scale A_qk, bf16 [64][64] sw64 (lower-triangle blocks)
  static constexpr int GC = 73728;     // exp(G_63), fp32 [128]
  static constexpr int BYTES = 74240;
};
__host__ __device__ inline int64_t kda_ws_header(int R) { return ((int64_t)4 * (R + 1) + 1023) / 1024 * 1024; }

// Chunk bases: base[r] = sum over r' < r of ceil(rows_r' / 64); a sequence outside [0, T) gets no chunks and raises
// kErrArgs in the status word. One block of 256 threads.
__global__ void kda_chunk_table_kernel(const int32_t* seqs, int R, int64_t T, int32_t* base, int32_t* status) {
  __shared__ int32_t part[256];
  const int per = (R + 255) / 256;
  const int r0 = threadIdx.x * per, r1 = min(R, r0 + per);
  auto chunks = [&](int r) -> int32_t {
    const int s = seqs[4 * r], e = seqs[4 * r + 1];
    if (s < 0 || e < s || e > T) {
      raise_status(status, kErrArgs);
      return 0;
    }
    return (e - s + kC - 1) / kC;
  };
  int32_t sum = 0;
  for (int r = r0; r < r1; ++r) sum += chunks(r);
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int o = 1; o < 256; o <<= 1) {
    const int32_t v = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t acc = part[threadIdx.x] - sum;
  for (int r = r0; r < r1; ++r) {
    base[r] = acc;
    acc += chunks(r);
  }
  if (threadIdx.x == 255) base[R] = part[255];
}

SSB_DEVICE int dpair(int I, int J) { return I == 1 ? 0 : (I == 2 ? 1 + J : 3 + J); }   // (1,0)(2,0)(2,1)(3,0..2)

SSB_DEVICE float sigmoid_fast(float z) {
  const float ez = __expf(-fminf(fmaxf(z, -80.0f), 80.0f));
  return __fdividef(1.0f, 1.0f + ez);
}

SSB_DEVICE void ldsm_x2_t(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}

// ---- prep: one CTA per (chunk, head), independent of the recurrent state ---------------------------------------
struct PrepSmem {
  static constexpr int XQ = 0;          // q tiles (TMA) -> conv q -> q exp(G - G_r) -> W
  static constexpr int XK = 16384;      // k tiles -> conv k -> k exp(G - G_r) -> u
  static constexpr int XV = 32768;      // v tiles -> conv v -> beta v
  static constexpr int GT = 49152;      // gate tiles -> k exp(G_r - G) -> R rows bf16 [16][256]
  static constexpr int KG = 65536;      // beta k exp G
  static constexpr int NP = 81920;      // per-row, per-group sums of squares fp32 [64][32] -> T_II bf16 [64][64] sw64
  static constexpr int LN = 90112;      // -L off the diagonal blocks, bf16 [64][64] sw64
  static constexpr int AD = 98304;      // L on the diagonal blocks, fp32 [4][16][16]
  static constexpr int BETA = 102400;   // fp32 [64]
  static constexpr int RQ = 102656;     // fp32 [64]
  static constexpr int RK = 102912;     // fp32 [64]
  static constexpr int GB = 103168;     // G at the 16-row block starts [4][128]
  static constexpr int DD = 105216;     // exp(G_rI - G_rJ) [6][128]
  static constexpr int XCH = 108288;    // per-quarter gate sums [4][128]
  static constexpr int MBAR = 110336;   // mbarrier (8 B) + abort flag
  static constexpr int BYTES = MBAR + 16 + 1024;   // + slack for the 1024-byte alignment of the swizzled tiles
  static_assert(2 * (BYTES + 1024) <= 233472, "two CTAs per SM");
};

// Conv, norms, gates, A_kk / A_qk, the blocked triangular solve -> the chunk's image. Two CTAs per SM.
__global__ void __launch_bounds__(kKdaThreads, 2)
    kda_prep_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mg, KdaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using S = PrepSmem;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int slot = blockIdx.x, h = blockIdx.y;
  const int32_t* cbase = reinterpret_cast<const int32_t*>(a.ws);
  if (slot >= cbase[a.R]) return;
  int lo = 0, hi = a.R - 1;                              // the sequence: the last r with base[r] <= slot
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cbase[mid] <= slot) lo = mid; else hi = mid - 1;
  }
  const int s = a.seqs[4 * lo], e = a.seqs[4 * lo + 1], blk = a.seqs[4 * lo + 2], init = a.seqs[4 * lo + 3];
  const int t0 = s + kC * (slot - cbase[lo]);
  const int n = min(kC, e - t0);
  const int P = a.P;
  uint8_t* img = a.ws + kda_ws_header(a.R) + ((int64_t)slot * a.H + h) * KdaImg::BYTES;

  __nv_bfloat16* XQ = reinterpret_cast<__nv_bfloat16*>(smem + S::XQ);
  __nv_bfloat16* XK = reinterpret_cast<__nv_bfloat16*>(smem + S::XK);
  __nv_bfloat16* XV = reinterpret_cast<__nv_bfloat16*>(smem + S::XV);
  __nv_bfloat16* GTs = reinterpret_cast<__nv_bfloat16*>(smem + S::GT);
  __nv_bfloat16* KGs = reinterpret_cast<__nv_bfloat16*>(smem + S::KG);
  float* NP = reinterpret_cast<float*>(smem + S::NP);
  __nv_bfloat16* TBs = reinterpret_cast<__nv_bfloat16*>(smem + S::NP);
  __nv_bfloat16* LN = reinterpret_cast<__nv_bfloat16*>(smem + S::LN);
  float* AD = reinterpret_cast<float*>(smem + S::AD);
  float* BETA = reinterpret_cast<float*>(smem + S::BETA);
  float* RQ = reinterpret_cast<float*>(smem + S::RQ);
  float* RK = reinterpret_cast<float*>(smem + S::RK);
  float* GB = reinterpret_cast<float*>(smem + S::GB);
  float* DD = reinterpret_cast<float*>(smem + S::DD);
  float* XCH = reinterpret_cast<float*>(smem + S::XCH);
  const uint32_t bar = smem_u32(smem + S::MBAR);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + S::MBAR + 8);

  if (tid == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    mbar_arrive_expect_tx(bar, 8 * 8192);
    const uint32_t sb = smem_u32(smem);
    const int hc = h * kD;
    tma_load_2d(sb + S::XQ, &mx, hc, t0, bar);
    tma_load_2d(sb + S::XQ + 8192, &mx, hc + 64, t0, bar);
    tma_load_2d(sb + S::XK, &mx, P + hc, t0, bar);
    tma_load_2d(sb + S::XK + 8192, &mx, P + hc + 64, t0, bar);
    tma_load_2d(sb + S::XV, &mx, 2 * P + hc, t0, bar);
    tma_load_2d(sb + S::XV + 8192, &mx, 2 * P + hc + 64, t0, bar);
    tma_load_2d(sb + S::GT, &mg, hc, t0, bar);
    tma_load_2d(sb + S::GT + 8192, &mg, hc + 64, t0, bar);
  }
  // conv items: 48 channel groups of 8 (q 0-15, k 16-31, v 32-47) x 5 row segments; segment 0 takes the 3 rows
  // before the chunk from x (or the conv state block / zeros at the sequence start), the others from the tile
  const bool item = tid < 240;
  const int grp = tid % 48, seg = tid / 48;
  const int i0 = 13 * seg, i1 = min(kC, i0 + 13);
  const int64_t col = (int64_t)(grp >> 4) * P + h * kD + (grp & 15) * 8;
  float wf[32];
  uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0, x2 = x0;
  if (item) {
    load_w8(a.conv_w, col, wf);
    if (seg == 0) {
      x0 = conv_row(a, (int64_t)t0 - 3, s, e, blk, init, col);
      x1 = conv_row(a, (int64_t)t0 - 2, s, e, blk, init, col);
      x2 = conv_row(a, (int64_t)t0 - 1, s, e, blk, init, col);
    }
  }
  float braw = 0.0f;
  if (tid >= 128 && tid < 192 && tid - 128 < n) braw = __bfloat162float(a.beta[(int64_t)(t0 + tid - 128) * a.ldb + h]);
  __syncthreads();
  mbar_wait(bar, 0, abort_flag, a.status);

  // ---- P1: conv in place (each item reads its 3 halo rows before any row is overwritten) -----------------------
  uint8_t* tb = smem + (grp >> 3) * 8192;                // tiles q0 q1 k0 k1 v0 v1
  const int ck = grp & 7;
  auto trow = [&](int i) { return reinterpret_cast<uint4*>(tb + i * 128 + ((ck ^ (i & 7)) << 4)); };
  if (item && seg > 0) {
    x0 = *trow(i0 - 3);
    x1 = *trow(i0 - 2);
    x2 = *trow(i0 - 1);
  }
  __syncthreads();
  if (*abort_flag) return;
  if (item) {
    // the taps of each channel pair and the window rows as packed fp32 pairs: every row is unpacked once, the four
    // products of a pair run as fp32x2 FMAs (each element rounded as the scalar chain w0 a + w1 b + w2 c + w3 d)
    uint64_t w2[16], xa[4], xb[4], xc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int tap = 0; tap < 4; ++tap) w2[4 * q + tap] = f2pack(wf[(2 * q) * 4 + tap], wf[(2 * q + 1) * 4 + tap]);
      xa[q] = bf2_f2((&x0.x)[q]);
      xb[q] = bf2_f2((&x1.x)[q]);
      xc[q] = bf2_f2((&x2.x)[q]);
    }
#pragma unroll 1
    for (int i = i0; i < i1; ++i) {
      const uint4 x3 = *trow(i);
      uint64_t xd[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) xd[q] = bf2_f2((&x3.x)[q]);
      uint4 y = make_uint4(0, 0, 0, 0);
      if (i < n) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint64_t acc = fma2(w2[4 * q], xa[q], 0ull);
          acc = fma2(w2[4 * q + 1], xb[q], acc);
          acc = fma2(w2[4 * q + 2], xc[q], acc);
          acc = fma2(w2[4 * q + 3], xd[q], acc);
          float lo, hi;
          f2unpack(acc, lo, hi);
          (&y.x)[q] = pack_bf16(silu_conv(lo), silu_conv(hi));
        }
      }
      *trow(i) = y;
      if (grp < 32) {
        float f[8];
        bf16x8_to_f32(y, f);
        float ss = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) ss = __fmaf_rn(f[c], f[c], ss);
        NP[i * 32 + grp] = ss;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        xa[q] = xb[q];
        xb[q] = xc[q];
        xc[q] = xd[q];
      }
    }
  }
  __syncthreads();

  // ---- P2: L2 norms of the q / k rows, beta, the gate's cumulative sum (per channel pair, 16-row quarters) -------
  if (tid < 128) {
    const float* np = NP + (tid & 63) * 32 + (tid >> 6) * 16;
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) ss += np[c];
    (tid < 64 ? RQ : RK)[tid & 63] = rsqrtf(ss + 1e-6f);
  } else if (tid < 192) {
    BETA[tid - 128] = (tid - 128 < n) ? sigmoid_fast(braw) : 0.0f;
  }
  const int cp = tid & 63, qt = tid >> 6, c0 = 2 * cp;
  const float eA = expf(a.a_log[h]);
  const float dtb0 = a.dt_bias[h * kD + c0], dtb1 = a.dt_bias[h * kD + c0 + 1];
  const float lb = a.lower_bound, scale = a.scale;
  float G0[16], G1[16];
  {
    float r0 = 0.0f, r1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int i = 16 * qt + j;
      const float2 gv = ld_bf2(GTs + t128(i, c0));
      float k0 = 0.0f, k1 = 0.0f;
      if (i < n) {
        k0 = lb * sigmoid_fast(eA * (gv.x + dtb0));
        k1 = lb * sigmoid_fast(eA * (gv.y + dtb1));
      }
      r0 += k0;
      r1 += k1;
      G0[j] = r0;
      G1[j] = r1;
    }
    XCH[qt * 128 + c0] = r0;
    XCH[qt * 128 + c0 + 1] = r1;
  }
  __syncthreads();
  float gc0 = 0.0f, gc1 = 0.0f;                          // G_63: every thread sums the quarters in the same order
  {
    float b0 = 0.0f, b1 = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float v0 = XCH[q * 128 + c0], v1 = XCH[q * 128 + c0 + 1];
      if (q < qt) {
        b0 += v0;
        b1 += v1;
      }
      gc0 += v0;
      gc1 += v1;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      G0[j] += b0;
      G1[j] += b1;
    }
  }
  GB[qt * 128 + c0] = G0[0];
  GB[qt * 128 + c0 + 1] = G1[0];
  if (qt == 0) {
    float* gcw = reinterpret_cast<float*>(img + KdaImg::GC);
    gcw[c0] = __expf(gc0);
    gcw[c0 + 1] = __expf(gc1);
  }
  __syncthreads();
  {
    const int c = tid & 127, hf = tid >> 7;
    const float g0 = GB[c], g1 = GB[128 + c], g2 = GB[256 + c], g3 = GB[384 + c];
    if (hf == 0) {
      DD[0 * 128 + c] = __expf(g1 - g0);   // (1,0)
      DD[1 * 128 + c] = __expf(g2 - g0);   // (2,0)
      DD[2 * 128 + c] = __expf(g2 - g1);   // (2,1)
    } else {
      DD[3 * 128 + c] = __expf(g3 - g0);   // (3,0)
      DD[4 * 128 + c] = __expf(g3 - g1);   // (3,1)
      DD[5 * 128 + c] = __expf(g3 - g2);   // (3,2)
    }
  }
  // operands: q exp(G - G_r), k exp(G - G_r) in place, k exp(G_r - G) over the gate tiles, beta k exp G; scale q exp G
  // and k exp(G_63 - G) straight into the image; beta v in place (G_r: G at the row's 16-row block start)
  {
    __nv_bfloat16* qtg = reinterpret_cast<__nv_bfloat16*>(img + KdaImg::QT);
    __nv_bfloat16* ktg = reinterpret_cast<__nv_bfloat16*>(img + KdaImg::KT);
    const float gr0 = G0[0], gr1 = G1[0];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int i = 16 * qt + j;
      const int o = t128(i, c0);
      const float2 qv = ld_bf2(XQ + o), kv = ld_bf2(XK + o), vv = ld_bf2(XV + o);
      const float rq = RQ[i], rk = RK[i], bt = BETA[i];
      const float qn0 = qv.x * rq, qn1 = qv.y * rq, kn0 = kv.x * rk, kn1 = kv.y * rk;
      const float eI0 = __expf(G0[j] - gr0), eI1 = __expf(G1[j] - gr1);
      const float eR0 = __expf(gr0 - G0[j]), eR1 = __expf(gr1 - G1[j]);
      const float eG0 = __expf(G0[j]), eG1 = __expf(G1[j]);
      const float eC0 = __expf(gc0 - G0[j]), eC1 = __expf(gc1 - G1[j]);
      st_bf2(XQ + o, qn0 * eI0, qn1 * eI1);
      st_bf2(XK + o, kn0 * eI0, kn1 * eI1);
      st_bf2(GTs + o, kn0 * eR0, kn1 * eR1);
      st_bf2(KGs + o, bt * kn0 * eG0, bt * kn1 * eG1);
      st_bf2(qtg + o, scale * qn0 * eG0, scale * qn1 * eG1);
      st_bf2(ktg + o, kn0 * eC0, kn1 * eC1);
      st_bf2(XV + o, bt * vv.x, bt * vv.y);
    }
  }
  __syncthreads();

  // ---- P3: the 16x16 blocks of A_kk (strict lower, times beta_i: fp32 diagonal blocks, -bf16 off them) and A_qk
  //      (lower, times scale, into the image) ------------------------------------------------------------------------
  {
    __nv_bfloat16* aqk = reinterpret_cast<__nv_bfloat16*>(img + KdaImg::AQK);
#pragma unroll 1
    for (int tau = warp; tau < 20; tau += 8) {
      const bool qk = tau >= 10;
      const int p = qk ? tau - 10 : tau;
      const int I = (p >= 1) + (p >= 3) + (p >= 6), J = p - I * (I + 1) / 2;   // blocks (0,0) (1,0) (1,1) ...
      const __nv_bfloat16* left = qk ? XQ : XK;
      const float* dv = (I != J) ? DD + dpair(I, J) * 128 : nullptr;
      float acc[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldsm_x4(left + t128(16 * I + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
        if (dv != nullptr) {
          const int cc = 16 * kk + 2 * t4;
          const float d0 = dv[cc], d1 = dv[cc + 1], d8 = dv[cc + 8], d9 = dv[cc + 9];
          a0 = scale_bf16x2(a0, d0, d1);
          a1 = scale_bf16x2(a1, d0, d1);
          a2 = scale_bf16x2(a2, d8, d9);
          a3 = scale_bf16x2(a3, d8, d9);
        }
        ldsm_x4(GTs + t128(16 * J + (lane & 7) + ((lane >> 4) << 3), 16 * kk + ((lane >> 3) & 1) * 8), b0, b1, b2, b3);
        mma16816(acc[0], a0, a1, a2, a3, b0, b1);
        mma16816(acc[1], a0, a1, a2, a3, b2, b3);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 16 * I + g8 + 8 * hh, j = 16 * J + 8 * nt + 2 * t4;
          const float v0 = acc[nt][2 * hh], v1 = acc[nt][2 * hh + 1];
          if (qk) {
            st_bf2(aqk + sw64(i, j), j <= i ? v0 * scale : 0.0f, j + 1 <= i ? v1 * scale : 0.0f);
          } else {
            const float bi = BETA[i];
            if (I == J) {
              float* ad = AD + I * 256 + (i - 16 * I) * 16 + (j - 16 * J);
              ad[0] = j < i ? bi * v0 : 0.0f;
              ad[1] = j + 1 < i ? bi * v1 : 0.0f;
            } else {
              st_bf2(LN + sw64(i, j), -(bi * v0), -(bi * v1));
            }
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- P4: diagonal blocks T_II = (I + L_II)^-1 (fp32 forward substitution) -> bf16 ------------------------------
  if (warp < 4 && lane < 16) {
    const int I = warp, c = lane;
    const float* ad = AD + I * 256;
    float tcol[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = (i == c) ? 1.0f : 0.0f;
#pragma unroll
      for (int j = 0; j < i; ++j) acc -= ad[i * 16 + j] * tcol[j];
      tcol[i] = acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) TBs[sw64(16 * I + i, 16 * I + c)] = __float2bfloat16_rn(tcol[i]);
  }
  __syncthreads();

  // ---- P5: [W | u] = (I + L)^-1 [beta k exp G | beta v] by 16-row blocks: R_I = B_I - sum_J L_IJ X_J,
  //      X_I = T_II R_I; 32 column tiles of 8 (W 0-15, u 16-31), 4 per warp; W over the q tiles, u over the k tiles --
  __nv_bfloat16* Wsm = XQ;
  __nv_bfloat16* Usm = XK;
  __nv_bfloat16* RB = GTs;
#pragma unroll 1
  for (int I = 0; I < 4; ++I) {
    if (I > 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int nt = warp * 4 + q;
        const bool wcol = nt < 16;
        const int c = wcol ? 8 * nt : 8 * (nt - 16);
        const __nv_bfloat16* B = wcol ? KGs : XV;
        float acc[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float2 f = ld_bf2(B + t128(16 * I + g8 + 8 * hh, c + 2 * t4));
          acc[2 * hh] = f.x;
          acc[2 * hh + 1] = f.y;
        }
        for (int J = 0; J < I; ++J) {
          uint32_t a0, a1, a2, a3, b0, b1;
          ldsm_x4(LN + sw64(16 * I + (lane & 15), 16 * J + (lane >> 4) * 8), a0, a1, a2, a3);
          ldsm_x2_t((wcol ? Wsm : Usm) + t128(16 * J + (lane & 15), c), b0, b1);
          mma16816(acc, a0, a1, a2, a3, b0, b1);
        }
        st_bf2(RB + sw256(g8, 8 * nt + 2 * t4), acc[0], acc[1]);
        st_bf2(RB + sw256(g8 + 8, 8 * nt + 2 * t4), acc[2], acc[3]);
      }
      __syncthreads();
    }
    uint32_t a0, a1, a2, a3;
    ldsm_x4(TBs + sw64(16 * I + (lane & 15), 16 * I + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int nt = warp * 4 + q;
      const bool wcol = nt < 16;
      const int c = wcol ? 8 * nt : 8 * (nt - 16);
      uint32_t b0, b1;
      if (I > 0) {
        ldsm_x2_t(RB + sw256(lane & 15, 8 * nt), b0, b1);
      } else {
        ldsm_x2_t((wcol ? KGs : XV) + t128(lane & 15, c), b0, b1);
      }
      float acc[4] = {};
      mma16816(acc, a0, a1, a2, a3, b0, b1);
      __nv_bfloat16* X = wcol ? Wsm : Usm;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) st_bf2(X + t128(16 * I + g8 + 8 * hh, c + 2 * t4), acc[2 * hh], acc[2 * hh + 1]);
    }
    __syncthreads();
  }
  // W and u into the image (generic-proxy writes made visible to the bulk copy first)
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    bulk_store(img + KdaImg::W, smem_u32(Wsm), 16384);
    bulk_store(img + KdaImg::U, smem_u32(Usm), 16384);
    bulk_commit();
    bulk_wait0();
  }
}

// ---- scan: one CTA per (sequence, head, value half), the chunks in order ----------------------------------------
struct ScanSmem {
  static constexpr int W = 0, QT = 16384, KT = 32768, U = 49152, AQK = 57344, GC = 65536;
  static constexpr int BUF = GC + 512;  // one chunk: W | QT | KT (t128) | U half (sw64) | AQK (sw64) | exp(G_63)
  static constexpr int S0 = 2 * BUF;    // state bf16 [128 key][64 value] sw64
  static constexpr int US = S0 + 16384; // U = u - W S, bf16 [64][64] sw64
  static constexpr int MBAR = US + 8192;   // 2 mbarriers + abort flag
  static constexpr int BYTES = MBAR + 32;
  static_assert(AQK + 8192 == GC && KdaImg::GC - KdaImg::AQK == GC - AQK, "A_qk and exp(G_63) arrive in one copy");
  static_assert(BYTES <= 232448, "shared memory");
};

//   U = u - W S;  O = (scale q exp G) S + A_qk U;  S' = diag(exp G_63) S + (k exp(G_63 - G))^T U
// with the state fp32 in registers (warp w: key rows 16w..16w+15 x the 64 value columns) and a bf16 copy in shared
// memory for the products; the chunk images double-buffered by bulk copies.
__global__ void __launch_bounds__(kKdaThreads, 1) kda_scan_kernel(KdaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  using S = ScanSmem;
  constexpr int BV = 64;
  constexpr int UN = BV / 16;                             // n-tiles of 8 per warp in the [64 x BV] products
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int vb = blockIdx.x & 1, h = (blockIdx.x >> 1) % a.H, r = blockIdx.x / (2 * a.H);
  const int s = a.seqs[4 * r], e = a.seqs[4 * r + 1], blk = a.seqs[4 * r + 2], init = a.seqs[4 * r + 3];
  if (s < 0 || e < s || e > a.T) return;                 // rejected by the chunk table (status raised there)
  const int32_t* cbase = reinterpret_cast<const int32_t*>(a.ws);
  const int slot0 = cbase[r], nc = cbase[r + 1] - slot0;
  if ((int64_t)slot0 + nc > a.ws_slots) {
    raise_status(a.status, kErrCapacity);
    return;
  }
  const uint8_t* img0 = a.ws + kda_ws_header(a.R) + ((int64_t)slot0 * a.H + h) * KdaImg::BYTES;
  const int64_t img_step = (int64_t)a.H * KdaImg::BYTES;
  __nv_bfloat16* S0 = reinterpret_cast<__nv_bfloat16*>(smem + S::S0);
  __nv_bfloat16* Us = reinterpret_cast<__nv_bfloat16*>(smem + S::US);
  const uint32_t bar0 = smem_u32(smem + S::MBAR);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + S::MBAR + 16);

  float st[BV / 8][4];
  float* page = a.rec_state + (int64_t)blk * a.rs_stride + ((int64_t)h * kD + vb * BV) * kD;
#pragma unroll
  for (int nt = 0; nt < BV / 8; ++nt) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ch = 16 * warp + g8 + 8 * (q >> 1), v = 8 * nt + 2 * t4 + (q & 1);
      st[nt][q] = init ? page[(int64_t)v * kD + ch] : 0.0f;
    }
    st_bf2(S0 + sw64(16 * warp + g8, 8 * nt + 2 * t4), st[nt][0], st[nt][1]);
    st_bf2(S0 + sw64(16 * warp + g8 + 8, 8 * nt + 2 * t4), st[nt][2], st[nt][3]);
  }
  auto issue = [&](int c) {
    const uint8_t* im = img0 + (int64_t)c * img_step;
    const uint32_t sb = smem_u32(smem) + (c & 1) * S::BUF;
    const uint32_t b = bar0 + 8 * (c & 1);
    mbar_arrive_expect_tx(b, 49152 + 8192 + 8704);     // = ScanSmem::BUF bytes
    bulk_load(sb + S::W, im + KdaImg::W, 49152, b);                 // W | QT | KT
    bulk_load(sb + S::U, im + KdaImg::U + vb * 8192, 8192, b);      // this value half of u
    bulk_load(sb + S::AQK, im + KdaImg::AQK, 8704, b);              // A_qk | exp(G_63)
  };
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    *abort_flag = 0;
    fence_barrier_init();
    if (nc > 0) issue(0);
    if (nc > 1) issue(1);
  }
  __syncthreads();
  const int m = warp & 3, nh = warp >> 2;
  for (int c = 0; c < nc; ++c) {
    const int t0 = s + kC * c, n = min(kC, e - t0);
    const uint8_t* buf = smem + (c & 1) * S::BUF;
    const __nv_bfloat16* Wb = reinterpret_cast<const __nv_bfloat16*>(buf + S::W);
    const __nv_bfloat16* QTb = reinterpret_cast<const __nv_bfloat16*>(buf + S::QT);
    const __nv_bfloat16* KTb = reinterpret_cast<const __nv_bfloat16*>(buf + S::KT);
    const __nv_bfloat16* UCb = reinterpret_cast<const __nv_bfloat16*>(buf + S::U);
    const __nv_bfloat16* AQKb = reinterpret_cast<const __nv_bfloat16*>(buf + S::AQK);
    const float* GCb = reinterpret_cast<const float*>(buf + S::GC);
    mbar_wait(bar0 + 8 * (c & 1), (c >> 1) & 1, abort_flag, a.status);
    __syncthreads();                                     // the state copy of the previous chunk is complete
    if (*abort_flag) break;

    // ---- U = u - W S -> shared bf16 ----
    {
      float pacc[UN][4] = {};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(Wb + t128(16 * m + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(S0 + sw64(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(pacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(pacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < UN; ++nt) {
        const int cc = (BV / 2) * nh + 8 * nt + 2 * t4;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int o = sw64(16 * m + g8 + 8 * hh, cc);
          const float2 u = ld_bf2(UCb + o);
          st_bf2(Us + o, u.x - pacc[nt][2 * hh], u.y - pacc[nt][2 * hh + 1]);
        }
      }
    }
    __syncthreads();

    // ---- O = (scale q exp G) S + A_qk U -> global; S' = diag(exp G_63) S + (k exp(G_63 - G))^T U ----
    {
      float oacc[UN][4] = {};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(QTb + t128(16 * m + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(S0 + sw64(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(oacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(oacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        if (kb > m) break;
        uint32_t a0, a1, a2, a3;
        ldsm_x4(AQKb + sw64(16 * m + (lane & 15), 16 * kb + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(Us + sw64(16 * kb + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(oacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(oacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < UN; ++nt) {
        const int cc = h * kD + vb * BV + (BV / 2) * nh + 8 * nt + 2 * t4;
        const int i0 = 16 * m + g8;
        if (i0 < n) *reinterpret_cast<uint32_t*>(a.out + (int64_t)(t0 + i0) * a.ldo + cc) = pack_bf16(oacc[nt][0], oacc[nt][1]);
        if (i0 + 8 < n)
          *reinterpret_cast<uint32_t*>(a.out + (int64_t)(t0 + i0 + 8) * a.ldo + cc) = pack_bf16(oacc[nt][2], oacc[nt][3]);
      }
      const float d_lo = GCb[16 * warp + g8], d_hi = GCb[16 * warp + g8 + 8];
#pragma unroll
      for (int nt = 0; nt < BV / 8; ++nt) {
        st[nt][0] *= d_lo; st[nt][1] *= d_lo; st[nt][2] *= d_hi; st[nt][3] *= d_hi;
      }
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(KTb + t128(16 * kb + (lane & 7) + ((lane >> 4) << 3), 16 * warp + ((lane >> 3) & 1) * 8), a0, a1, a2,
                  a3);
#pragma unroll
        for (int p = 0; p < BV / 16; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(Us + sw64(16 * kb + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * p + (lane >> 4) * 8), b0, b1, b2, b3);
          mma16816(st[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(st[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();                                     // this buffer and the state copy are no longer read
    if (tid == 0 && c + 2 < nc) issue(c + 2);
#pragma unroll
    for (int nt = 0; nt < BV / 8; ++nt) {
      st_bf2(S0 + sw64(16 * warp + g8, 8 * nt + 2 * t4), st[nt][0], st[nt][1]);
      st_bf2(S0 + sw64(16 * warp + g8 + 8, 8 * nt + 2 * t4), st[nt][2], st[nt][3]);
    }
  }

  // ---- final state back into the request's block (left as it was when a copy wait gave up) -------------------------
  if (*abort_flag) return;
#pragma unroll
  for (int nt = 0; nt < BV / 8; ++nt) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ch = 16 * warp + g8 + 8 * (q >> 1), v = 8 * nt + 2 * t4 + (q & 1);
      page[(int64_t)v * kD + ch] = st[nt][q];
    }
  }
}

// Conv states: per sequence, its last 3 x rows (old state rows where the sequence is shorter), 8 channels a thread;
// in a prefill call, not for a sequence the scan rejects (its chunks beyond the workspace).
__global__ void kda_conv_state_kernel(KdaArgs a, int C) {
  const int r = blockIdx.x;
  const int64_t col = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (col >= C) return;
  const int s = a.seqs[4 * r], e = a.seqs[4 * r + 1], blk = a.seqs[4 * r + 2], init = a.seqs[4 * r + 3];
  if (s < 0 || e < s || e > a.T) return;
  if (a.ws != nullptr && reinterpret_cast<const int32_t*>(a.ws)[r + 1] > a.ws_slots) return;   // rejected by the scan
  uint4 v[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) v[j] = conv_row(a, (int64_t)e - 3 + j, s, e, blk, init, col);
  __nv_bfloat16* base = a.conv_state + (int64_t)blk * a.cs_stride + col;
#pragma unroll
  for (int j = 0; j < 3; ++j) *reinterpret_cast<uint4*>(base + (int64_t)j * C) = v[j];
}

// Standalone conv (the reference's `conv_qkv` boundary): 16 rows x 8 channels a thread; q, k, v [T][P] each.
__global__ void kda_conv_qkv_kernel(KdaArgs a, int64_t T, __nv_bfloat16* q, __nv_bfloat16* k, __nv_bfloat16* v) {
  const int C = 3 * a.P;
  const int64_t col = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (col >= C) return;
  float wf[32];
  load_w8(a.conv_w, col, wf);
  const int sec = (int)(col / a.P);
  __nv_bfloat16* dst = sec == 0 ? q : (sec == 1 ? k : v);
  const int64_t dcol = col - (int64_t)sec * a.P;
  int cs = 0, ce = 0, cb = 0, ci = 0, cur = -1;
  const int64_t t_end = (int64_t)blockIdx.x * 16 + 16 < T ? (int64_t)blockIdx.x * 16 + 16 : T;
  for (int64_t t = (int64_t)blockIdx.x * 16; t < t_end; ++t) {
    if (cur < 0 || t < cs || t >= ce) {
      cur = -1;
      for (int r = 0; r < a.R; ++r) {
        if (t >= a.seqs[4 * r] && t < a.seqs[4 * r + 1]) {
          cur = r; cs = a.seqs[4 * r]; ce = a.seqs[4 * r + 1]; cb = a.seqs[4 * r + 2]; ci = a.seqs[4 * r + 3];
          break;
        }
      }
    }
    uint4 y = make_uint4(0, 0, 0, 0);
    if (cur >= 0) {
      y = conv8(conv_row(a, t - 3, cs, ce, cb, ci, col), conv_row(a, t - 2, cs, ce, cb, ci, col),
                conv_row(a, t - 1, cs, ce, cb, ci, col), conv_row(a, t, cs, ce, cb, ci, col), wf);
    }
    *reinterpret_cast<uint4*>(dst + t * a.P + dcol) = y;
  }
}

int run_prefill(const KdaArgs& a, int64_t slots, cudaStream_t stream) {
  kda_chunk_table_kernel<<<1, 256, 0, stream>>>(a.seqs, a.R, a.T, reinterpret_cast<int32_t*>(a.ws), a.status);
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  CUtensorMap mx, mg;
  int rc = make_map_2d_swizzled(&mx, a.x, a.T, 3 * (int64_t)a.P, a.ldx * 2, kC);
  if (rc != kOk) return rc;
  rc = make_map_2d_swizzled(&mg, a.g, a.T, a.P, a.ldg * 2, kC);
  if (rc != kOk) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kda_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PrepSmem::BYTES) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kda_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess ||
        cudaFuncSetAttribute(kda_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ScanSmem::BYTES) !=
            cudaSuccess)
      return kErrCuda;
    attr = true;
  }
  kda_prep_kernel<<<dim3((unsigned)slots, (unsigned)a.H), kKdaThreads, PrepSmem::BYTES, stream>>>(mx, mg, a);
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  const int C = 3 * a.P;                                 // after the prep kernel, which reads the old conv states
  kda_conv_state_kernel<<<dim3((unsigned)a.R, (unsigned)((C / 8 + 127) / 128)), 128, 0, stream>>>(a, C);
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  kda_scan_kernel<<<(unsigned)((int64_t)a.R * a.H * 2), kKdaThreads, ScanSmem::BYTES, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int check_kda(const KdaArgs& a) {
  const uintptr_t mask = 15;
  if (a.H <= 0 || a.R < 0 || a.P != a.H * kD) return kErrArgs;
  if (a.x == nullptr || a.conv_w == nullptr || a.conv_state == nullptr || a.seqs == nullptr) return kErrArgs;
  if ((reinterpret_cast<uintptr_t>(a.x) & mask) || (a.ldx % 8) || a.ldx < 3 * (int64_t)a.P) return kErrArgs;
  if ((reinterpret_cast<uintptr_t>(a.conv_w) & mask) || (reinterpret_cast<uintptr_t>(a.conv_state) & mask)) return kErrArgs;
  if ((a.cs_stride % 8) || a.cs_stride < 9 * (int64_t)a.P) return kErrArgs;
  return kOk;
}

}  // namespace

int64_t kda_workspace_bytes(int H, int64_t T, int R) {
  if (H <= 0 || T < 0 || R < 0) return 0;
  const int64_t slots = T / kC + R + 1;                  // sum over sequences of ceil(rows / 64) when rows sum to <= T
  return kda_ws_header(R) + slots * H * KdaImg::BYTES;
}

int launch_kda_prefill(const KdaArgs& a_in, cudaStream_t stream) {
  KdaArgs a = a_in;
  int rc = check_kda(a);
  if (rc != kOk) return rc;
  if (a.g == nullptr || a.beta == nullptr || a.a_log == nullptr || a.dt_bias == nullptr || a.rec_state == nullptr ||
      a.out == nullptr || (a.ldo % 2) || a.ldo < a.P || (reinterpret_cast<uintptr_t>(a.out) & 3) ||
      (reinterpret_cast<uintptr_t>(a.g) & 15) || (a.ldg % 8) ||
      a.rs_stride < (int64_t)a.H * kD * kD)
    return kErrArgs;
  if (a.R == 0 || a.T == 0) return a.R == 0 ? kOk : kErrArgs;
  const int64_t slots = a.T / kC + a.R + 1;
  if (slots > 0x7fffffff || a.H > 65535) return kErrArgs;
  const int64_t need = kda_workspace_bytes(a.H, a.T, a.R);
  bool own = false;
  if (a.ws == nullptr) {                                 // no caller workspace: a stream-ordered allocation
    void* p = nullptr;
    if (cudaMallocAsync(&p, need, stream) != cudaSuccess) return kErrCuda;
    a.ws = static_cast<uint8_t*>(p);
    own = true;
  } else if (a.ws_bytes < need || (reinterpret_cast<uintptr_t>(a.ws) & 15)) {
    return kErrWorkspace;
  }
  a.ws_slots = slots;
  rc = run_prefill(a, slots, stream);
  if (own && cudaFreeAsync(a.ws, stream) != cudaSuccess && rc == kOk) rc = kErrCuda;
  return rc;
}

int launch_kda_conv(const KdaArgs& a_in, int64_t T, void* q, void* k, void* v, cudaStream_t stream) {
  KdaArgs a = a_in;
  a.T = T;
  int rc = check_kda(a);
  if (rc != kOk) return rc;
  if (q == nullptr || k == nullptr || v == nullptr || T < 0) return kErrArgs;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return kErrArgs;
  const int C = 3 * a.P;
  if (T > 0) {
    kda_conv_qkv_kernel<<<dim3((unsigned)((T + 15) / 16), (unsigned)((C / 8 + 127) / 128)), 128, 0, stream>>>(
        a, T, static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v));
    if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  }
  if (a.R == 0) return kOk;
  kda_conv_state_kernel<<<dim3((unsigned)a.R, (unsigned)((C / 8 + 127) / 128)), 128, 0, stream>>>(a, C);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace ssb
