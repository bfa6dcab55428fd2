// Device-side building blocks shared by the sm_100a kernels of the prefill-stage library.
//
// - status codes written to the caller's device status word;
// - mbarrier / TMA / bulk-copy / tcgen05 wrappers as inline PTX (sm_100a only);
// - every mbarrier wait is bounded (SSB_WAIT_NS of %globaltimer): on expiry the waiter raises the CTA's abort flag
//   and the kernel's status word, and every role of the CTA leaves its loop at its next wait; no trap, no hang;
// - the NVFP4 codec (e2m1 elements, e4m3 per-16 scales, fp32 global scale) with each step a single IEEE fp32
//   operation, so that a CPU restatement with the same operations produces the same bytes.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SSB_DEVICE __device__ __forceinline__

namespace ssb {

// ---- status codes (device status word and C-ABI return values) ------------------------------------------------
enum Status : int32_t {
  kOk = 0,
  kErrArgs = 1,          // bad shape / pointer / alignment (host check)
  kErrCuda = 2,          // a CUDA runtime call failed (host)
  kErrWorkspace = 3,     // workspace too small
  kErrTimeout = 4,       // a bounded device wait expired (device)
  kErrNoDriver = 5,      // cuTensorMapEncodeTiled unavailable
  kErrCapacity = 6,      // a device-side table overflowed its capacity (device)
};

constexpr unsigned long long kWaitNs = 1000ull * 1000ull * 1000ull;   // 1 s per wait

SSB_DEVICE unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

SSB_DEVICE void raise_status(int32_t* status, int32_t code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

SSB_DEVICE uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---- mbarrier ---------------------------------------------------------------------------------------------------
SSB_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
SSB_DEVICE void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
SSB_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

SSB_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
SSB_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
SSB_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`, at most kWaitNs. Returns false (after raising the abort flag and the status
// word) on expiry, or at once when another role of the CTA already aborted.
SSB_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort_flag, int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      *abort_flag = 1;
      raise_status(status, kErrTimeout);
      return false;
    }
  }
}

// ---- named barriers (id 1..15) over a subset of the CTA's warps ------------------------------------------------
SSB_DEVICE void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Barrier that also returns the OR of `v` over the participating threads (a uniform decision for the group).
SSB_DEVICE bool named_bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// ---- TMA / bulk copies (no cluster multicast anywhere in this library) ---------------------------------------------
SSB_DEVICE void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
SSB_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* m, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
SSB_DEVICE void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// shared -> global bulk store (16-byte aligned addresses, size a multiple of 16), completed by bulk_wait0
SSB_DEVICE void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}
SSB_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
SSB_DEVICE void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- tcgen05 ------------------------------------------------------------------------------------------------------
SSB_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols));
}
SSB_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
SSB_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
SSB_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SSB_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
SSB_DEVICE void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Copy a 32-row x 16-byte scale atom (512 B, no swizzle) from shared memory to 4 TMEM columns, broadcast to the 4
// lane quadrants.
SSB_DEVICE void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// D[tmem] (+)= A[smem] x B[smem], e2m1 operands, ue4m3 scales per 16 elements in TMEM, fp32 accumulate.
SSB_DEVICE void tc_mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate,
                            uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// D[tmem] (+)= A[smem] x B[smem], bf16 operands (kind::f16), fp32 accumulate.
SSB_DEVICE void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] x B[smem], e4m3 operands (kind::f8f6f4), fp32 accumulate.
SSB_DEVICE void tc_mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
SSB_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
SSB_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SSB_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
SSB_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Instruction descriptor of kind::f8f6f4 with e4m3 A and B (format 0), fp32 D (1 in [4,6)), K-major both (bit 16 set
// by the caller for an MN-major B), N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor of kind::f16 with bf16 A and B (format 1 in [7,10) and [10,13)), fp32 D (1 in [4,6)),
// K-major both, N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory matrix descriptor (sm_100 format): start >> 4 in [0,14), LBO >> 4 in [16,30), SBO >> 4 in [32,46),
// version 1 in [46,48), layout type in [61,64) (0 = no swizzle, 2 = 128-byte swizzle).
SSB_DEVICE uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7) << 61;
  return d;
}

// Instruction descriptor of kind::mxf4nvf4 (block-scaled): e2m1 A and B (format 1), K-major both, ue4m3 scales
// (bit 23 = 0), N >> 3 in [17,23), M >> 4 in [24,29), scale-factor ids 0.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t M, uint32_t N) {
  return (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE single-precision operations per instruction, each rounded as
// the scalar one would be).
SSB_DEVICE uint64_t f2pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
SSB_DEVICE void f2unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
SSB_DEVICE uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
SSB_DEVICE uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// bf16 pair (low element in the low half) -> packed fp32 {lo, hi}; packed fp32 -> bf16 pair, round to nearest even
SSB_DEVICE uint64_t bf2_f2(uint32_t w) { return f2pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u)); }
SSB_DEVICE uint32_t f2_bf2(uint64_t v) {
  float lo, hi;
  f2unpack(v, lo, hi);
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// ---- NVFP4 codec --------------------------------------------------------------------------------------------------
SSB_DEVICE float e2m1_value(uint32_t code) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float v = mag[code & 7u];
  return (code & 8u) ? -v : v;
}

// e4m3 round to nearest even, saturating at 448 (cvt.rn.satfinite); value >= 0 here.
SSB_DEVICE uint32_t e4m3_encode(float v) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)) & 0xFFu;
}
SSB_DEVICE float e4m3_value(uint32_t code) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(code), __NV_E4M3);
  return __half2float(__half(h));
}

// Eight e2m1 codes (a 32-bit word, element i in nibble i) of a[0..7], round to nearest even, saturating at 6, by the
// hardware conversion (cvt.rn.satfinite.e2m1x2.f32); a value that rounds to zero keeps its sign (code 8 for a
// negative one), as vLLM's NVFP4 quantizer, which converts with the same instruction, writes it.
SSB_DEVICE uint32_t e2m1x8(const float* a) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w |= static_cast<uint32_t>(__nv_cvt_float2_to_fp4x2(make_float2(a[2 * i], a[2 * i + 1]), __NV_E2M1,
                                                        cudaRoundNearest)) << (8 * i);
  return w;
}

// Quantize 16 values with global scale gs: returns the scale byte, writes 8 bytes of packed codes (element 2i in the
// low nibble of byte i).
SSB_DEVICE uint32_t nvfp4_quant16(const float (&x)[16], float gs, uint32_t (&packed)[2]) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
  const float sf_f = __fmul_rn(__fdiv_rn(amax, 6.0f), gs);
  const uint32_t sf = e4m3_encode(sf_f);
  const float sfv = e4m3_value(sf);
  const float r = sfv > 0.0f ? __fdiv_rn(gs, sfv) : 0.0f;
  float y[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) y[i] = __fmul_rn(x[i], r);
  packed[0] = e2m1x8(y);
  packed[1] = e2m1x8(y + 8);
  return sf;
}

// Byte offset of scale (row r, scale column c) in the 128x4-atom layout with `ncb` atom columns per row block.
__host__ __device__ inline int64_t sf_atom_offset(int64_t r, int64_t c, int64_t ncb) {
  return ((r >> 7) * ncb + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// Atom columns per row block for K elements: K padded to 256 (one GEMM k-block), 4 atoms per 256.
__host__ __device__ constexpr int64_t sf_atom_cols(int64_t K) { return ((K + 255) / 256) * 4; }

}  // namespace ssb
