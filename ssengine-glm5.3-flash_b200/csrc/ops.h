// Internal host-side launchers of the sm_100a kernels (not part of the C ABI; see include/ssengine_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ssb {

// Output stage of the NVFP4 GEMM.
enum Epilogue : int {
  kEpiF32 = 0,     // fp32 [rows, ldo] = alpha * acc, columns < N stored (router logits)
  kEpiBF16 = 1,    // bf16 [rows, ldo] = alpha[g] * acc (expert down projection)
  kEpiSwiGLU = 2,  // a 256-wide tile holds 128 gate + 128 up columns; h = silu(alpha g) * (alpha u) quantized to
                   // NVFP4 (codes [rows, ldo bytes] + 128x4-atom scales) with global scale out_gs
};

struct GemmArgs {
  const uint8_t* sfa = nullptr;        // A scales, 128x4 atoms, sf_atom_cols(K) atom columns per row block
  const uint8_t* sfb = nullptr;        // B scales (all groups, group g's rows start at g * N)
  const int32_t* mtiles = nullptr;     // grouped: [cap][4] = {group, first A row, valid rows, 0}; nullptr = dense
  const int32_t* num_mtiles = nullptr; // grouped: device count of valid entries
  int32_t mtile_cap = 0;
  // grouped, CTA pairs (BN 256 epilogues): [cap][4] = {group, first row, rows of the first 128, rows of the next 128},
  // both 128-row halves inside the group's rows or its padding; when set, the GEMM runs on clusters of 2 CTAs that
  // share each MMA (M = 256), and `mtiles` is not read
  const int32_t* mpairs = nullptr;
  const int32_t* num_mpairs = nullptr;
  int32_t mpair_cap = 0;
  int32_t M = 0;                       // dense: rows of A
  int32_t K = 0;                       // reduction length (elements)
  int32_t N = 0;                       // B rows per group
  int32_t ncb_k = 0;                   // sf_atom_cols(K)
  const float* alpha = nullptr;        // per-group output scale (device), or nullptr -> alpha_scalar
  float alpha_scalar = 1.0f;
  void* out = nullptr;
  int64_t ldo = 0;                     // elements (F32 / BF16) or bytes (SwiGLU codes)
  uint8_t* out_sf = nullptr;           // SwiGLU: output scales
  int32_t out_ncb = 0;                 // SwiGLU: sf_atom_cols(N / 2)
  float out_gs = 1.0f;                 // SwiGLU: output global scale
  int32_t* status = nullptr;           // device status word
};

// Builds the TMA maps for A ([a_rows, K/2] bytes, row pitch lda bytes) and B ([b_rows, K/2], pitch ldb) and launches
// the persistent GEMM on `stream`. Returns a Status.
int launch_gemm_nvfp4(int epilogue, const uint8_t* a, int64_t a_rows, int64_t lda, const uint8_t* b, int64_t b_rows,
                      int64_t ldb, const GemmArgs& args, int num_sms, cudaStream_t stream);

int launch_nvfp4_quantize(const void* x, int64_t rows, int64_t K, int64_t ldx, float gs, uint8_t* codes, int64_t ldc,
                          uint8_t* sf, cudaStream_t stream);

int launch_moe_route(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids, float* weights,
                     cudaStream_t stream);
int launch_moe_route_sigmoid(const float* logits, int64_t T, int32_t E, int32_t k, const float* bias, int32_t n_group,
                             int32_t topk_group, float scale, int32_t* ids, float* weights, cudaStream_t stream);

int launch_moe_count(const int32_t* ids, int64_t T, int32_t E, int32_t k, uint32_t* masks, int32_t* block_counts,
                     cudaStream_t stream);

// mpairs (nullptr: none): the CTA-pair tile table of the grouped GEMM, count in num_mtiles[1]
int launch_moe_offsets(int64_t T, int32_t E, int32_t* block_counts, int32_t* counts, int32_t* offsets,
                       int32_t* mtiles, int32_t* num_mtiles, int32_t mtile_cap, int32_t* mpairs, int32_t mpair_cap,
                       int32_t* status, cudaStream_t stream);

// rows[t, j] = permuted row of (token t, slot j); row_src[row] = t and the token's code row copied for each of its
// k + 1 rows
int launch_moe_scatter(const int32_t* ids, int64_t T, int32_t E, int32_t k, const uint32_t* masks,
                       const int32_t* block_base, const int32_t* offsets, int32_t* rows, int32_t* row_src,
                       const uint8_t* xq, int64_t H, uint8_t* xq_perm, cudaStream_t stream);
// The permuted scale atoms of the *num_mtiles row tiles: row r's words from token row_src[r] of xsf, zeros past a
// tile's valid rows
int launch_moe_sf_gather(const int32_t* row_src, const int32_t* mtiles, const int32_t* num_mtiles, int32_t mtile_cap,
                         const uint8_t* xsf, int64_t H, uint8_t* xsf_perm, cudaStream_t stream);

// out = (residual if not null) + sum_j w[t, j] y[rows[t, j]] + y[shared row of t]
int launch_moe_combine(const void* y, int64_t H, const int32_t* rows, const float* weights, const int32_t* offsets,
                       int64_t T, int32_t E, int32_t k, const void* residual, void* out, cudaStream_t stream);

// Canonical per-row top-k of the indexer (csrc/topk.cu); max_keys bounds ke - ks (sizes the shared-memory row cache).
int launch_topk_canonical(const float* logits, int64_t rows, int64_t ld, const int32_t* ks, const int32_t* ke,
                          int32_t k, int32_t* out, int32_t max_keys, cudaStream_t stream);

// Stage kernels (csrc/stage.cu).
int launch_stage_metadata(const int32_t* qsl, const int32_t* starts, const int32_t* page_ptr, const int32_t* pages,
                          int32_t R, int64_t T, int64_t bucket, int32_t page_tokens, int32_t width,
                          int64_t* positions, int64_t* slots, int32_t* table, cudaStream_t stream);
int launch_embed_rows(const void* table, int64_t vocab, int64_t H, const int64_t* ids, int64_t T, void* out,
                      cudaStream_t stream);
int launch_rmsnorm(const void* x, int64_t H, const int64_t* rows, int64_t n, const void* w, float eps, void* y,
                   cudaStream_t stream);
int launch_gated_rmsnorm(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps, void* y,
                         int64_t ldy, int64_t rows, int heads, cudaStream_t stream);
// The gated RMSNorm quantized to NVFP4 (codes [rows, ldc] bytes, scale atoms of heads * 128 columns, global scale gs):
// the same codes and scales as launch_gated_rmsnorm followed by launch_nvfp4_quantize.
int launch_gated_rmsnorm_nvfp4(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps,
                               float gs, uint8_t* codes, int64_t ldc, uint8_t* sf, int64_t rows, int heads,
                               cudaStream_t stream);
int launch_hc_expand(const void* x, int64_t T, int64_t H, void* out, cudaStream_t stream);
int launch_hc_mean(const void* res, int64_t H, const int64_t* rows, int64_t n, void* out, cudaStream_t stream);
int launch_argmax_rows(const float* logits, int64_t ld, int64_t N, int64_t n, int64_t* out, cudaStream_t stream);

// mHC layer boundary (csrc/mhc.cu): do_post -> new_res; do_pre -> post_out, comb_out, y.
int64_t mhc_workspace_bytes(int64_t T);
int launch_mhc(bool do_post, bool do_pre, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, const float* fn, const float* scale, const float* base, const void* norm_w,
               float* post_out, float* comb_out, void* y, int64_t T, int64_t H, float rms_eps, float pre_eps,
               float sinkhorn_eps, float post_mult, int repeat, float norm_eps, void* ws, int64_t ws_bytes,
               int32_t* status, cudaStream_t stream);

// KDA prefill (csrc/kda.cu).
struct KdaArgs {
  const __nv_bfloat16* x = nullptr;    // in_proj rows [T, ldx]: q | k | v in columns [0, 3P)
  int64_t ldx = 0;
  const __nv_bfloat16* g = nullptr;    // raw gate rows [T, ldg], H * 128 columns
  int64_t ldg = 0;
  const __nv_bfloat16* beta = nullptr; // raw beta rows [T, ldb], H columns
  int64_t ldb = 0;
  const __nv_bfloat16* conv_w = nullptr;   // [3P][4]
  const float* a_log = nullptr;        // [H]
  const float* dt_bias = nullptr;      // [H * 128]
  float lower_bound = -5.0f;
  float scale = 0.0f;
  __nv_bfloat16* conv_state = nullptr; // blocks of [3][3P]
  int64_t cs_stride = 0;               // elements between blocks
  float* rec_state = nullptr;          // blocks of [H][128 value][128 key]
  int64_t rs_stride = 0;
  const int32_t* seqs = nullptr;       // [R][4] = {first row, end row, state block, has initial state}
  int32_t R = 0;
  int32_t H = 0;
  int32_t P = 0;                       // H * 128
  __nv_bfloat16* out = nullptr;        // [T, ldo], H * 128 columns
  int64_t ldo = 0;
  int32_t* status = nullptr;           // device status word (bounded copy waits)
  int64_t T = 0;                       // rows of x, g, beta, out
  uint8_t* ws = nullptr;               // chunk workspace (kda_workspace_bytes); null: allocated on the stream
  int64_t ws_bytes = 0;
  int64_t ws_slots = 0;                // chunk slots the workspace holds (set by the launcher)
};
int64_t kda_workspace_bytes(int H, int64_t T, int R);
int launch_kda_prefill(const KdaArgs& a, cudaStream_t stream);

// 2D tensor map (no swizzle) over [rows, width] elements of `dtype` (a CUtensorMapDataType) with row pitch ld_bytes;
// box = box_cols x box_rows (csrc/gemm_nvfp4.cu).
int make_map_2d(CUtensorMap* m, int dtype, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                int box_cols, int box_rows);
// The same with a CUtensorMapSwizzle mode (csrc/gemm_nvfp4.cu).
int make_map_2d_ex(CUtensorMap* m, int dtype, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                   int box_cols, int box_rows, int swizzle);
int launch_kda_conv(const KdaArgs& a, int64_t T, void* q, void* k, void* v, cudaStream_t stream);

// DSA indexer (csrc/indexer.cu).
struct IdxArgs {
  const void* w = nullptr;             // bf16 [T, ldw] head weights (32 used)
  int64_t ldw = 0;
  int64_t T = 0;                       // query rows
  const int32_t* table = nullptr;      // [R, width] pool pages (= KV pages) of each request
  int32_t width = 0;
  const int32_t* groups = nullptr;     // [G][4] = {request, first query row, query rows (<= 8), pool tiles of 128}
  int32_t G = 0;
  float* logits = nullptr;             // [T, ldl]
  int64_t ldl = 0;
  int32_t* status = nullptr;
  const float* q_scale = nullptr;      // FP8 form: fp32 [T, 32] query scales (folded into the head weights)
  const float* kscale = nullptr;       // FP8 form: the pool pages read as fp32 (each page's scale row)
};
int launch_indexer_logits(const void* q, const void* k_cache, int64_t pool_rows, const IdxArgs& a,
                          cudaStream_t stream);
// FP8 form: q8 e4m3 [T * 32, 128] with q_scale fp32 [T * 32]; the pool cache in pages of 33 rows of 128 bytes (32 rows
// of e4m3 codes, then the 32 fp32 scales), `pages` of them.
int launch_indexer_logits_fp8(const uint8_t* q8, const float* q_scale, const uint8_t* k_pages, int64_t pages,
                              const IdxArgs& a, cudaStream_t stream);
int launch_indexer_q_quant(const void* q, int64_t rows, uint8_t* q8, float* q_scale, cudaStream_t stream);
int launch_indexer_expand(const int32_t* pool_ids, int64_t ldp, int32_t k, const int64_t* positions, int32_t* out,
                          int64_t ldo, int64_t rows, cudaStream_t stream);
// bf16 map over [rows, width] elements (row pitch ld_bytes), box 64 x box_rows, 128-byte swizzle (csrc/gemm_nvfp4.cu).
int make_map_2d_swizzled(CUtensorMap* m, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                         int box_rows);

// Sparse MLA prefill and latent-cache append (csrc/mla.cu).
struct MlaArgs {
  const uint8_t* q = nullptr;          // e4m3 [T, 64, 576]
  const uint8_t* kv = nullptr;         // e4m3 latent cache [slots, 576]
  const int32_t* indices = nullptr;    // [T, ld_idx] token positions (-1 = none)
  int64_t ld_idx = 0;
  int32_t n_idx = 0;                   // columns used
  const int32_t* qsl = nullptr;        // [R + 1] first row of each request
  int32_t R = 0;
  const int32_t* table = nullptr;      // [R, width] KV pages (128 tokens)
  int32_t width = 0;
  float scale = 0.0f;                  // bmm1: softmax scale * q_scale * k_scale
  float bmm2 = 1.0f;                   // k_scale
  __nv_bfloat16* out = nullptr;        // [T, 64, 512]
  int64_t T = 0;
  int32_t* status = nullptr;           // device status word (bounded waits)
};
int launch_sparse_mla(const MlaArgs& a, cudaStream_t stream);
int launch_mla_append(const void* src, int64_t lds, const int64_t* slots, int64_t T, void* cache, float k_scale,
                      cudaStream_t stream);
int launch_mla_q_pack(const void* lat, int64_t rows_pad, const void* rope, int64_t ldr, int64_t rope_stride,
                      int64_t T, void* q8, float q_scale, cudaStream_t stream);

// Indexer key pools (csrc/kpool.cu).
struct KpoolArgs {
  const __nv_bfloat16* k = nullptr;    // [T, ld] (128 used)
  const __nv_bfloat16* gate = nullptr; // [T, ld]
  int64_t ld = 0;
  const float* ape = nullptr;          // [4, 128]
  const int32_t* reqs = nullptr;       // [R][4] = {first row, rows, start position, tail block}
  int32_t R = 0;
  const int32_t* table = nullptr;      // [R, width] KV pages = pool pages
  int32_t width = 0;
  __nv_bfloat16* pool = nullptr;       // [pages * 32, 128]
  __nv_bfloat16* tail = nullptr;       // [blocks][2][4][128]
  uint8_t* pool8 = nullptr;            // FP8 form instead of `pool`: pages of 33 rows x 128 bytes (32 code rows, scales)
};
int launch_kpool_insert(const KpoolArgs& a, int32_t max_rows, cudaStream_t stream);

// DSA block data movement (csrc/dsa.cu).
int launch_rmsnorm_cols(const void* x, int64_t ldx, int width, int64_t rows, const void* g, float eps, void* y,
                        int64_t ldy, cudaStream_t stream);
int launch_rope(void* x, int64_t ldx, int heads, int64_t head_stride, const int64_t* positions, int64_t rows,
                float theta, cudaStream_t stream);
int launch_transpose_heads(const void* src, void* dst, int64_t rows, int64_t rows_pad, int heads, int dim,
                           int64_t row_ld, int64_t head_stride, bool to_heads, cudaStream_t stream);
int launch_head_tiles(int heads, int64_t rows_pad, int32_t* tiles, int64_t tile_cap, int32_t* num,
                      cudaStream_t stream);
int launch_concat_cols(const void* a, int64_t lda, int wa, const void* b, int64_t ldb, int wb, void* out, int64_t ldo,
                       int64_t rows, cudaStream_t stream);

int device_sm_count();

}  // namespace ssb
