// KDA prefill for sm_100a: the width-4 causal conv over the packed q|k|v projection rows, fused into a chunked
// gated delta-rule scan that reads and writes each request's FP32 recurrent state block in place.
//
// Reference behaviour (ssengine/model/pp_patch.py:215-244 `kda_prefill_forward`): conv (kda_conv.py:56-132) into
// contiguous q, k, v; state gather (zero for a fresh request, kda_state.py:19-36); FlashInfer persistent KDA (gate
// lower_bound * sigmoid(exp(A_log) * (g + dt_bias)) and beta sigmoid in kernel, q/k L2-normalised, scale D^-0.5);
// state scatter. Here one launch does conv + gates + scan + state write; a second small launch writes the requests'
// conv states (it must run after the scan has read the old ones).
//
// Scan: one CTA per (sequence, head, value block of BV columns), 8 warps, 64-token chunks. Within a chunk, with G
// the per-channel cumulative log decay (G_i includes token i) and S the [key, value] state at the chunk start:
//   L[i][j]  = beta_i sum_c k_i[c] k_j[c] exp(G_i[c] - G_j[c])      (j < i)
//   Aqk[i][j] = scale sum_c q_i[c] k_j[c] exp(G_i[c] - G_j[c])      (j <= i)
//   T = (I + L)^-1 diag(beta);  W = T (k * exp(G));  U = T v - W S
//   O = scale (q * exp(G)) S + Aqk U;  S' = diag(exp(G_63)) S + (k * exp(G_63 - G))^T U
// The exp(G_i - G_j) factors are split at 16-row block starts r (j <= r <= i), so that every factor stays <= 1 off
// the diagonal blocks and <= exp(-16 * lower_bound) on them: no overflow, tensor-core operands in bf16
// (mma.sync m16n8k16, fp32 accumulate; the state stays fp32 in registers across chunks).
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

constexpr int kD = 128;        // key = value head dim
constexpr int kC = 64;         // chunk tokens
constexpr int kKdaThreads = 256;

// bf16 tiles in shared memory, 16-byte chunks XOR-swizzled by (row & 7): [rows][128] and [rows][64]
SSB_DEVICE int sw128(int r, int c) { return r * 128 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }
SSB_DEVICE int sw64(int r, int c) { return r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }
template <int BV> SSB_DEVICE int swv(int r, int c) { return BV == 64 ? sw64(r, c) : sw128(r, c); }

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

// SiLU of the conv accumulator: a * 1 / (1 + 2^(-a log2 e)) with the approximate ex2 / rcp instructions and FTZ, the
// arithmetic the reference's conv kernel fixes in inline PTX (kda_conv.py:37-53).
SSB_DEVICE float silu_conv(float a) {
  float e;
  asm("{\n\t.reg .f32 t;\n\t"
      "mul.ftz.f32 t, %1, 0fBFB8AA3B;\n\t"
      "ex2.approx.ftz.f32 t, t;\n\t"
      "add.ftz.f32 t, t, 0f3F800000;\n\t"
      "rcp.approx.ftz.f32 t, t;\n\t"
      "mul.ftz.f32 %0, %1, t;\n\t}"
      : "=f"(e) : "f"(a));
  return e;
}

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

struct KdaSmem {
  static constexpr int QR = 0;             // raw conv q [64][128] bf16       | A_kk fp32 [64][64]
  static constexpr int KR = 16384;         // raw conv k                      | A_qk bf16 [64][64], T_II bf16 [64][64]
  static constexpr int TB = KR + 8192;
  static constexpr int QH = 32768;         // q exp(G - G_r)                  | W bf16 [64][128]
  static constexpr int KH = 49152;         // k exp(G - G_r)                  | -L bf16 [64][64], R bf16 [16][192]
  static constexpr int LN = KH;
  static constexpr int RB = KH + 8192;
  static constexpr int KRB = 65536;        // k exp(G_r - G)                  | U bf16 [64][BV], u bf16 [64][BV]
  static constexpr int UC = KRB + 8192;
  static constexpr int KG = 81920;         // beta k exp(G)
  static constexpr int QT = 98304;         // scale q exp(G)
  static constexpr int KT = 114688;        // k exp(G_63 - G)
  static constexpr int VR = 131072;        // conv v [64][BV], then beta v
};

template <int BV>
struct KdaLayout {
  static constexpr int NG = 32 + BV / 8;                    // 16-byte channel groups: q 16, k 16, v BV/8
  static constexpr int XW = 8 * NG;                         // halo row: q 128 | k 128 | v BV
  static constexpr int S0 = KdaSmem::VR + kC * BV * 2;      // state bf16 [128][BV]
  static constexpr int BETA = S0 + kD * BV * 2;             // fp32 [64]
  static constexpr int RQ = BETA + 256;                     // fp32 [64]
  static constexpr int RK = RQ + 256;                       // fp32 [64]
  static constexpr int GC = RK + 256;                       // exp(G_63) [128]
  static constexpr int GB = GC + 512;                       // G at block starts [4][128]
  static constexpr int DD = GB + 2048;                      // exp(G_rI - G_rJ) [6][128]
  static constexpr int XCH = DD + 3072;                     // [2][128]
  static constexpr int XT = XCH + 1024;                     // raw rows: NG/8 x-tiles then 2 gate tiles, [64][64] bf16 each
  static constexpr int NXT = NG / 8;
  static constexpr int GT = XT + NXT * 8192;
  static constexpr int HX = GT + 2 * 8192;                  // the 3 x rows before the chunk [3][XW]
  static constexpr int WS = HX + ((3 * XW * 2 + 127) / 128) * 128;   // conv weights [NG][32] bf16
  static constexpr int MBAR = WS + NG * 64;                 // mbarrier (8 B) + abort flag
  static constexpr int BYTES = MBAR + 16;
  static constexpr int NP = KdaSmem::KG;                    // per-row, per-group sums of squares [64][32] (aliases KG)
  static constexpr uint32_t TX = (NXT + 2) * 8192;          // bytes landing per chunk
  static_assert(XT % 128 == 0 && GT % 128 == 0, "TMA destinations");
  static_assert(BYTES <= 232448, "shared memory");
};

SSB_DEVICE int dpair(int I, int J) { return I == 1 ? 0 : (I == 2 ? 1 + J : 3 + J); }   // (1,0)(2,0)(2,1)(3,0..2)

SSB_DEVICE float sigmoid_fast(float z) {
  const float ez = __expf(-fminf(fmaxf(z, -80.0f), 80.0f));
  return __fdividef(1.0f, 1.0f + ez);
}

SSB_DEVICE int sw192(int r, int c) { return r * 192 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7); }

SSB_DEVICE void ldsm_x2_t(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}

// x column (within the in_proj row) of channel group `grp` of this CTA: q 0..15, k 16..31, v 32..
template <int BV>
SSB_DEVICE int64_t group_col(int grp, int P, int h, int vb) {
  return grp < 16 ? (int64_t)h * kD + grp * 8
                  : (grp < 32 ? (int64_t)P + h * kD + (grp - 16) * 8 : 2 * (int64_t)P + h * kD + vb * BV + (grp - 32) * 8);
}

// One chunk's raw rows: the x tiles (q 0-63, q 64-127, k 0-63, k 64-127, v ...) and the 2 gate tiles, 64 rows from
// t0 (rows past the tensor read as zeros), all completing on `bar`. Called by one thread.
template <int BV>
SSB_DEVICE void issue_chunk_loads(const CUtensorMap* mx, const CUtensorMap* mg, uint8_t* smem, uint32_t bar, int t0,
                                  int P, int h, int vb) {
  using Ly = KdaLayout<BV>;
  mbar_arrive_expect_tx(bar, Ly::TX);
  const uint32_t xt = smem_u32(smem + Ly::XT), gt = smem_u32(smem + Ly::GT);
#pragma unroll
  for (int j = 0; j < Ly::NXT; ++j) {
    const int col = j < 2 ? h * kD + 64 * j : (j < 4 ? P + h * kD + 64 * (j - 2) : 2 * P + h * kD + vb * BV + 64 * (j - 4));
    tma_load_2d(xt + j * 8192, mx, col, t0, bar);
  }
  tma_load_2d(gt, mg, h * kD, t0, bar);
  tma_load_2d(gt + 8192, mg, h * kD + 64, t0, bar);
}

template <int BV>
__global__ void __launch_bounds__(kKdaThreads, 1)
    kda_prefill_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mg, KdaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using Ly = KdaLayout<BV>;
  constexpr int NVB = kD / BV;
  constexpr int NG = Ly::NG;
  constexpr int kSeg = 6;                    // conv row segments: NG x 6 items <= 256 threads
  static_assert(NG * kSeg <= kKdaThreads, "conv items");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int vb = blockIdx.x % NVB;
  const int h = (blockIdx.x / NVB) % a.H;
  const int r = blockIdx.x / (NVB * a.H);
  const int s = a.seqs[4 * r], e = a.seqs[4 * r + 1], blk = a.seqs[4 * r + 2], init = a.seqs[4 * r + 3];
  const int P = a.P;

  __nv_bfloat16* QRs = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::QR);
  __nv_bfloat16* KRs = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KR);
  float* AKK = reinterpret_cast<float*>(smem + KdaSmem::QR);
  __nv_bfloat16* AQK = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KR);
  __nv_bfloat16* TBs = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::TB);
  __nv_bfloat16* QH = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::QH);
  __nv_bfloat16* Ws = QH;
  __nv_bfloat16* KH = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KH);
  __nv_bfloat16* LN = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::LN);
  __nv_bfloat16* RB = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::RB);
  __nv_bfloat16* KRB = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KRB);
  __nv_bfloat16* Us = KRB;
  __nv_bfloat16* UC = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::UC);
  __nv_bfloat16* KG = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KG);
  __nv_bfloat16* QT = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::QT);
  __nv_bfloat16* KT = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::KT);
  __nv_bfloat16* VR = reinterpret_cast<__nv_bfloat16*>(smem + KdaSmem::VR);
  __nv_bfloat16* S0 = reinterpret_cast<__nv_bfloat16*>(smem + Ly::S0);
  float* BETA = reinterpret_cast<float*>(smem + Ly::BETA);
  float* RQ = reinterpret_cast<float*>(smem + Ly::RQ);
  float* RK = reinterpret_cast<float*>(smem + Ly::RK);
  float* GCs = reinterpret_cast<float*>(smem + Ly::GC);
  float* GB = reinterpret_cast<float*>(smem + Ly::GB);
  float* DD = reinterpret_cast<float*>(smem + Ly::DD);
  float* XCH = reinterpret_cast<float*>(smem + Ly::XCH);
  const __nv_bfloat16* XT = reinterpret_cast<const __nv_bfloat16*>(smem + Ly::XT);
  const __nv_bfloat16* GT = reinterpret_cast<const __nv_bfloat16*>(smem + Ly::GT);
  __nv_bfloat16* HX = reinterpret_cast<__nv_bfloat16*>(smem + Ly::HX);
  __nv_bfloat16* WSm = reinterpret_cast<__nv_bfloat16*>(smem + Ly::WS);
  float* NP = reinterpret_cast<float*>(smem + Ly::NP);
  const uint32_t bar = smem_u32(smem + Ly::MBAR);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + Ly::MBAR + 8);

  // ---- state: warp w holds key channels 16w..16w+15 x all BV value columns (fp32 mma accumulator layout) --------
  float st[BV / 8][4];
  float* page = a.rec_state + (int64_t)blk * a.rs_stride + ((int64_t)h * kD + vb * BV) * kD;
#pragma unroll
  for (int nt = 0; nt < BV / 8; ++nt) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ch = 16 * warp + g8 + 8 * (q >> 1), v = 8 * nt + 2 * t4 + (q & 1);
      st[nt][q] = init ? page[(int64_t)v * kD + ch] : 0.0f;
    }
    *reinterpret_cast<uint32_t*>(S0 + swv<BV>(16 * warp + g8, 8 * nt + 2 * t4)) = pack_bf16(st[nt][0], st[nt][1]);
    *reinterpret_cast<uint32_t*>(S0 + swv<BV>(16 * warp + g8 + 8, 8 * nt + 2 * t4)) = pack_bf16(st[nt][2], st[nt][3]);
  }
  // the 3 rows before the sequence (its conv state, or zeros) and this CTA's conv weights
  if (tid < 3 * NG) {
    const int j = tid / NG, grp = tid % NG;
    const int64_t col = group_col<BV>(grp, P, h, vb);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (init) v = *reinterpret_cast<const uint4*>(a.conv_state + (int64_t)blk * a.cs_stride + (int64_t)j * 3 * P + col);
    *reinterpret_cast<uint4*>(HX + j * Ly::XW + grp * 8) = v;
  }
  if (tid < 4 * NG) {
    const int grp = tid >> 2, part = tid & 3;
    reinterpret_cast<uint4*>(WSm + grp * 32)[part] =
        __ldg(reinterpret_cast<const uint4*>(a.conv_w + group_col<BV>(grp, P, h, vb) * 4) + part);
  }
  // raw beta of this thread's row of the coming chunk (threads 128..191)
  float braw = 0.0f;
  if (tid >= 128 && tid < 192 && s + (tid - 128) < e) braw = __bfloat162float(a.beta[(int64_t)(s + tid - 128) * a.ldb + h]);
  if (tid == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    if (e > s) issue_chunk_loads<BV>(&mx, &mg, smem, bar, s, P, h, vb);
  }
  __syncthreads();

  // per-thread constants of the gate phase: channel c, row half hf
  const int gc_c = tid & 127, hf = tid >> 7;
  const float eA = expf(a.a_log[h]);
  const float dtb = a.dt_bias[h * kD + gc_c];
  const float lb = a.lower_bound, scale = a.scale;
  uint32_t phase = 0;

  for (int t0 = s; t0 < e; t0 += kC, phase ^= 1) {
    const int n = min(kC, e - t0);
    const bool more = e - t0 > kC;                    // a chunk follows
    mbar_wait(bar, phase, abort_flag, a.status);
    // ---- P1: conv of q, k (all 128 channels) and v (this CTA's BV channels) from the landed tiles ---------------
    if (tid < NG * kSeg) {
      const int grp = tid % NG, seg = tid / NG;
      const int i0 = (kC * seg) / kSeg, i1 = (kC * (seg + 1)) / kSeg;
      float wf[32];
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        float f[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(WSm + grp * 32)[part], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) wf[8 * part + j] = f[j];
      }
      const __nv_bfloat16* tile = XT + (grp >> 3) * 4096 + (grp & 7) * 8;
      auto xrow = [&](int i) -> uint4 {
        return *reinterpret_cast<const uint4*>(i >= 0 ? tile + i * 64 : HX + (i + 3) * Ly::XW + grp * 8);
      };
      __nv_bfloat16* dst;
      int dcol;
      if (grp < 16) { dst = QRs; dcol = grp * 8; }
      else if (grp < 32) { dst = KRs; dcol = (grp - 16) * 8; }
      else { dst = VR; dcol = (grp - 32) * 8; }
      uint4 x0 = xrow(i0 - 3), x1 = xrow(i0 - 2), x2 = xrow(i0 - 1);
#pragma unroll 4
      for (int i = i0; i < i1; ++i) {
        const uint4 x3 = xrow(i);
        const uint4 y = (i < n) ? conv8(x0, x1, x2, x3, wf) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dst + (grp < 32 ? sw128(i, dcol) : swv<BV>(i, dcol))) = y;
        if (grp < 32) {
          float f[8];
          bf16x8_to_f32(y, f);
          float ss = 0.0f;
#pragma unroll
          for (int c = 0; c < 8; ++c) ss = __fmaf_rn(f[c], f[c], ss);
          NP[i * 32 + grp] = ss;
        }
        x0 = x1; x1 = x2; x2 = x3;
      }
    }
    __syncthreads();
    if (*abort_flag) break;

    // ---- P2: L2 norms of the q / k rows, beta; gate cumsum per channel (two 32-row halves); next chunk's loads ---
    if (tid < 128) {
      const float* np = NP + (tid & 63) * 32 + (tid >> 6) * 16;
      float ss = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) ss += np[c];
      (tid < 64 ? RQ : RK)[tid & 63] = rsqrtf(ss + 1e-6f);
    } else if (tid < 192) {
      BETA[tid - 128] = (tid - 128 < n) ? sigmoid_fast(braw) : 0.0f;
      if (more && tid - 128 < min(kC, e - t0 - kC))
        braw = __bfloat162float(a.beta[(int64_t)(t0 + kC + tid - 128) * a.ldb + h]);
    }
    float G[32];
    {
      const __nv_bfloat16* gcol = GT + (gc_c >> 6) * 4096 + (gc_c & 63);
      float run = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = 32 * hf + j;
        float gk = 0.0f;
        if (i < n) gk = lb * sigmoid_fast(eA * (__bfloat162float(gcol[i * 64]) + dtb));
        run += gk;
        G[j] = run;
      }
      if (hf == 0) XCH[gc_c] = run;
    }
    if (more && tid < 3 * NG) {                         // the next chunk's halo: this chunk's last 3 rows
      const int j = tid / NG, grp = tid % NG;
      *reinterpret_cast<uint4*>(HX + j * Ly::XW + grp * 8) =
          *reinterpret_cast<const uint4*>(XT + (grp >> 3) * 4096 + (kC - 3 + j) * 64 + (grp & 7) * 8);
    }
    __syncthreads();
    if (more && tid == 0) issue_chunk_loads<BV>(&mx, &mg, smem, bar, t0 + kC, P, h, vb);
    if (hf == 1) {
      const float base = XCH[gc_c];
#pragma unroll
      for (int j = 0; j < 32; ++j) G[j] += base;
      XCH[128 + gc_c] = G[31];
      GCs[gc_c] = __expf(G[31]);
    }
    GB[(2 * hf) * 128 + gc_c] = G[0];
    GB[(2 * hf + 1) * 128 + gc_c] = G[16];
    __syncthreads();
    {
      const float g0 = GB[gc_c], g1 = GB[128 + gc_c], g2 = GB[256 + gc_c], g3 = GB[384 + gc_c];
      if (hf == 0) {
        DD[0 * 128 + gc_c] = __expf(g1 - g0);   // (1,0)
        DD[1 * 128 + gc_c] = __expf(g2 - g0);   // (2,0)
        DD[2 * 128 + gc_c] = __expf(g2 - g1);   // (2,1)
      } else {
        DD[3 * 128 + gc_c] = __expf(g3 - g0);   // (3,0)
        DD[4 * 128 + gc_c] = __expf(g3 - g1);   // (3,1)
        DD[5 * 128 + gc_c] = __expf(g3 - g2);   // (3,2)
      }
      const float gC = XCH[128 + gc_c];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = 32 * hf + j;
        const float gr = (j < 16) ? (hf ? g2 : g0) : (hf ? g3 : g1);
        const int o = sw128(i, gc_c);
        const float qn = __bfloat162float(QRs[o]) * RQ[i];
        const float kn = __bfloat162float(KRs[o]) * RK[i];
        const float eI = __expf(G[j] - gr), eR = __expf(gr - G[j]);
        const float eG = __expf(G[j]), eC = __expf(gC - G[j]);
        QH[o] = __float2bfloat16_rn(qn * eI);
        KH[o] = __float2bfloat16_rn(kn * eI);
        KRB[o] = __float2bfloat16_rn(kn * eR);
        KG[o] = __float2bfloat16_rn(BETA[i] * kn * eG);
        QT[o] = __float2bfloat16_rn(scale * qn * eG);
        KT[o] = __float2bfloat16_rn(kn * eC);
        if (gc_c < BV) {
          const int ov = swv<BV>(i, gc_c);
          VR[ov] = __float2bfloat16_rn(BETA[i] * __bfloat162float(VR[ov]));
        }
      }
    }
    __syncthreads();

    // ---- P3: the 16x16 blocks of A_kk (strict lower, times beta_i) and A_qk (lower, times scale) -----------------
    {
#pragma unroll 1
      for (int tau = warp; tau < 20; tau += 8) {
        const bool qk = tau >= 10;
        const int p = qk ? tau - 10 : tau;
        const int I = (p >= 1) + (p >= 3) + (p >= 6), J = p - I * (I + 1) / 2;   // blocks (0,0) (1,0) (1,1) ...
        const __nv_bfloat16* left = qk ? QH : KH;
        const float* dv = (I != J) ? DD + dpair(I, J) * 128 : nullptr;
        float acc[2][4] = {};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          ldsm_x4(left + sw128(16 * I + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
          if (dv != nullptr) {
            const int c0 = 16 * kk + 2 * t4;
            const float d0 = dv[c0], d1 = dv[c0 + 1], d8 = dv[c0 + 8], d9 = dv[c0 + 9];
            a0 = scale_bf16x2(a0, d0, d1);
            a1 = scale_bf16x2(a1, d0, d1);
            a2 = scale_bf16x2(a2, d8, d9);
            a3 = scale_bf16x2(a3, d8, d9);
          }
          ldsm_x4(KRB + sw128(16 * J + (lane & 7) + ((lane >> 4) << 3), 16 * kk + ((lane >> 3) & 1) * 8), b0, b1, b2,
                  b3);
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
              *reinterpret_cast<uint32_t*>(AQK + sw64(i, j)) =
                  pack_bf16(j <= i ? v0 * scale : 0.0f, j + 1 <= i ? v1 * scale : 0.0f);
            } else {
              const float bi = BETA[i];
              AKK[i * 64 + j] = j < i ? bi * v0 : 0.0f;
              AKK[i * 64 + j + 1] = j + 1 < i ? bi * v1 : 0.0f;
            }
          }
        }
      }
    }
    __syncthreads();

    // ---- P4: diagonal blocks T_II = (I + L_II)^-1 (fp32 forward substitution) -> bf16; -L off the diagonal -------
    if (warp < 4 && lane < 16) {
      const int I = warp, c = lane;
      float tcol[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float acc = (i == c) ? 1.0f : 0.0f;
#pragma unroll
        for (int j = 0; j < i; ++j) acc -= AKK[(16 * I + i) * 64 + 16 * I + j] * tcol[j];
        tcol[i] = acc;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) TBs[sw64(16 * I + i, 16 * I + c)] = __float2bfloat16_rn(tcol[i]);
    }
    for (int el = tid; el < 64 * 32; el += kKdaThreads) {
      const int i = el >> 5, j = (el & 31) * 2;
      const bool off = (j >> 4) < (i >> 4);
      *reinterpret_cast<uint32_t*>(LN + sw64(i, j)) =
          off ? pack_bf16(-AKK[i * 64 + j], -AKK[i * 64 + j + 1]) : 0u;
    }
    __syncthreads();

    // ---- P5: [W | u] = (I + L)^-1 [beta k exp G | beta v] by 16-row blocks: R_I = B_I - sum_J L_IJ X_J,
    //      X_I = T_II R_I (X = W bf16 [64][128] and u bf16 [64][BV]); 24 (or 32) column tiles of 8 over the warps --
    constexpr int NT = (kD + BV) / 8;                   // column tiles of [W | u]
    constexpr int TPW = (NT + 7) / 8;                   // tiles per warp
#pragma unroll 1
    for (int I = 0; I < 4; ++I) {
      if (I > 0) {
#pragma unroll
        for (int q = 0; q < TPW; ++q) {
          const int nt = warp * TPW + q;
          if (nt >= NT) break;
          const bool wcol = nt < 16;
          const int c = wcol ? 8 * nt : 8 * (nt - 16);
          const __nv_bfloat16* B = wcol ? KG : VR;
          float acc[4];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int row = 16 * I + g8 + 8 * hh;
            const int o = wcol ? sw128(row, c + 2 * t4) : swv<BV>(row, c + 2 * t4);
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(B + o));
            acc[2 * hh] = f.x;
            acc[2 * hh + 1] = f.y;
          }
          for (int J = 0; J < I; ++J) {
            uint32_t a0, a1, a2, a3, b0, b1;
            ldsm_x4(LN + sw64(16 * I + (lane & 15), 16 * J + (lane >> 4) * 8), a0, a1, a2, a3);
            const int krow = 16 * J + (lane & 15);
            ldsm_x2_t(wcol ? Ws + sw128(krow, c) : UC + swv<BV>(krow, c), b0, b1);
            mma16816(acc, a0, a1, a2, a3, b0, b1);
          }
          *reinterpret_cast<uint32_t*>(RB + sw192(g8, 8 * nt + 2 * t4)) = pack_bf16(acc[0], acc[1]);
          *reinterpret_cast<uint32_t*>(RB + sw192(g8 + 8, 8 * nt + 2 * t4)) = pack_bf16(acc[2], acc[3]);
        }
        __syncthreads();
      }
      uint32_t a0, a1, a2, a3;
      ldsm_x4(TBs + sw64(16 * I + (lane & 15), 16 * I + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
      for (int q = 0; q < TPW; ++q) {
        const int nt = warp * TPW + q;
        if (nt >= NT) break;
        const bool wcol = nt < 16;
        const int c = wcol ? 8 * nt : 8 * (nt - 16);
        uint32_t b0, b1;
        if (I > 0) {
          ldsm_x2_t(RB + sw192(lane & 15, 8 * nt), b0, b1);
        } else {
          ldsm_x2_t(wcol ? KG + sw128(lane & 15, c) : VR + swv<BV>(lane & 15, c), b0, b1);
        }
        float acc[4] = {};
        mma16816(acc, a0, a1, a2, a3, b0, b1);
        __nv_bfloat16* X = wcol ? Ws : UC;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int row = 16 * I + g8 + 8 * hh;
          const int o = wcol ? sw128(row, c + 2 * t4) : swv<BV>(row, c + 2 * t4);
          *reinterpret_cast<uint32_t*>(X + o) = pack_bf16(acc[2 * hh], acc[2 * hh + 1]);
        }
      }
      __syncthreads();
    }

    const int m = warp & 3, nh = warp >> 2;
    constexpr int UN = BV / 16;              // n-tiles of 8 per warp in the [64 x BV] outputs (half the columns)
    // ---- P6: U = u - W S -> smem bf16 ----------------------------------------------------------------------------
    {
      float pacc[UN][4] = {};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(Ws + sw128(16 * m + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(S0 + swv<BV>(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(pacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(pacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < UN; ++nt) {
        const int c = (BV / 2) * nh + 8 * nt + 2 * t4;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int o = swv<BV>(16 * m + g8 + 8 * hh, c);
          const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(UC + o));
          *reinterpret_cast<uint32_t*>(Us + o) = pack_bf16(u.x - pacc[nt][2 * hh], u.y - pacc[nt][2 * hh + 1]);
        }
      }
    }
    __syncthreads();

    // ---- P7: O = (scale q exp G) S + A_qk U -> global; S' = diag(exp G_63) S + (k exp(G_63 - G))^T U ----------
    {
      float oacc[UN][4] = {};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(QT + sw128(16 * m + (lane & 15), 16 * kk + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(S0 + swv<BV>(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(oacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(oacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        if (kb > m) break;
        uint32_t a0, a1, a2, a3;
        ldsm_x4(AQK + sw64(16 * m + (lane & 15), 16 * kb + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int p = 0; p < UN / 2; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(Us + swv<BV>(16 * kb + (lane & 7) + ((lane >> 3) & 1) * 8, (BV / 2) * nh + 16 * p + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(oacc[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(oacc[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int nt = 0; nt < UN; ++nt) {
        const int c = h * kD + vb * BV + (BV / 2) * nh + 8 * nt + 2 * t4;
        const int i0 = 16 * m + g8;
        if (i0 < n) *reinterpret_cast<uint32_t*>(a.out + (int64_t)(t0 + i0) * a.ldo + c) = pack_bf16(oacc[nt][0], oacc[nt][1]);
        if (i0 + 8 < n)
          *reinterpret_cast<uint32_t*>(a.out + (int64_t)(t0 + i0 + 8) * a.ldo + c) = pack_bf16(oacc[nt][2], oacc[nt][3]);
      }
      const float d_lo = GCs[16 * warp + g8], d_hi = GCs[16 * warp + g8 + 8];
#pragma unroll
      for (int nt = 0; nt < BV / 8; ++nt) {
        st[nt][0] *= d_lo; st[nt][1] *= d_lo; st[nt][2] *= d_hi; st[nt][3] *= d_hi;
      }
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(KT + sw128(16 * kb + (lane & 7) + ((lane >> 4) << 3), 16 * warp + ((lane >> 3) & 1) * 8), a0, a1, a2,
                  a3);
#pragma unroll
        for (int p = 0; p < BV / 16; ++p) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(Us + swv<BV>(16 * kb + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * p + (lane >> 4) * 8), b0, b1, b2, b3);
          mma16816(st[2 * p], a0, a1, a2, a3, b0, b1);
          mma16816(st[2 * p + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < BV / 8; ++nt) {
      *reinterpret_cast<uint32_t*>(S0 + swv<BV>(16 * warp + g8, 8 * nt + 2 * t4)) = pack_bf16(st[nt][0], st[nt][1]);
      *reinterpret_cast<uint32_t*>(S0 + swv<BV>(16 * warp + g8 + 8, 8 * nt + 2 * t4)) = pack_bf16(st[nt][2], st[nt][3]);
    }
  }

  // ---- final state back into the request's block (left as it was when a copy wait gave up) ---------------------------
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

// Conv states: per sequence, its last 3 x rows (old state rows where the sequence is shorter), 8 channels a thread.
__global__ void kda_conv_state_kernel(KdaArgs a, int C) {
  const int r = blockIdx.x;
  const int64_t col = ((int64_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (col >= C) return;
  const int s = a.seqs[4 * r], e = a.seqs[4 * r + 1], blk = a.seqs[4 * r + 2], init = a.seqs[4 * r + 3];
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

template <int BV>
int launch_scan(const KdaArgs& a, cudaStream_t stream) {
  CUtensorMap mx, mg;
  int rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.T, 3 * (int64_t)a.P, a.ldx * 2, 64, kC);
  if (rc != kOk) return rc;
  rc = make_map_2d(&mg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.g, a.T, a.P, a.ldg * 2, 64, kC);
  if (rc != kOk) return rc;
  const int smem = KdaLayout<BV>::BYTES;
  if (cudaFuncSetAttribute(kda_prefill_kernel<BV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kErrCuda;
  const int64_t grid = (int64_t)a.R * a.H * (kD / BV);
  kda_prefill_kernel<BV><<<(unsigned)grid, kKdaThreads, smem, stream>>>(mx, mg, a);
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

int launch_kda_prefill(const KdaArgs& a, cudaStream_t stream) {
  int rc = check_kda(a);
  if (rc != kOk) return rc;
  if (a.g == nullptr || a.beta == nullptr || a.a_log == nullptr || a.dt_bias == nullptr || a.rec_state == nullptr ||
      a.out == nullptr || (a.ldo % 2) || a.ldo < a.P || (reinterpret_cast<uintptr_t>(a.out) & 3) ||
      (reinterpret_cast<uintptr_t>(a.g) & 15) || (a.ldg % 8) ||
      a.rs_stride < (int64_t)a.H * kD * kD)
    return kErrArgs;
  if (a.R == 0 || a.T == 0) return a.R == 0 ? kOk : kErrArgs;
  rc = launch_scan<64>(a, stream);
  if (rc != kOk) return rc;
  const int C = 3 * a.P;
  kda_conv_state_kernel<<<dim3((unsigned)a.R, (unsigned)((C / 8 + 127) / 128)), 128, 0, stream>>>(a, C);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int launch_kda_conv(const KdaArgs& a, int64_t T, void* q, void* k, void* v, cudaStream_t stream) {
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
