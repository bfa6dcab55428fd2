// extern "C" entry points of libssengine_b200.so (declared in include/ssengine_b200.h).
// Host-side argument checks, the MoE workspace layout and the launch sequence of one MoE layer.

#include <cstring>

#include "../../include/ssengine_b200.h"
#include "common.cuh"
#include "ops.h"

namespace {

using ssb::kErrArgs;
using ssb::kErrWorkspace;
using ssb::kOk;

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct MoeDims {
  int64_t T, H, F, E, k, Tpad, rcap, mtile_cap, mpair_cap, nblocks, ncbH, ncbF;
};

bool dims_of(const ssb_moe_layer* L, int64_t T, MoeDims& d) {
  if (L == nullptr || T < 0) return false;
  d.T = T;
  d.H = L->hidden;
  d.F = L->inter;
  d.E = L->num_experts;
  d.k = L->top_k;
  if (d.H <= 0 || d.H % 256 != 0 || d.F <= 0 || d.F % 128 != 0 || d.E <= 0 || d.E > 512 || d.k <= 0 || d.k >= 32 ||
      d.k > d.E)
    return false;
  d.Tpad = ceil_div(T > 0 ? T : 1, 128) * 128;
  d.rcap = ceil_div(T * (d.k + 1) + (d.E + 1) * 127, 128) * 128;
  if (d.rcap < 128) d.rcap = 128;
  d.mtile_cap = d.rcap / 128;
  d.mpair_cap = (d.mtile_cap + d.E + 1) / 2 + 1;   // sum over experts of ceil(tiles / 2)
  d.nblocks = ceil_div(T > 0 ? T : 1, 256);
  d.ncbH = ssb::sf_atom_cols(d.H);
  d.ncbF = ssb::sf_atom_cols(d.F);
  return true;
}

void layout(const MoeDims& d, int64_t* off) {
  int64_t sz[SSB_WS_END];
  sz[SSB_WS_XQ] = d.Tpad * d.H / 2;
  sz[SSB_WS_XSF] = (d.Tpad / 128) * d.ncbH * 512;
  sz[SSB_WS_LOGITS] = d.T * d.E * 4;
  sz[SSB_WS_IDS] = d.T * d.k * 4;
  sz[SSB_WS_WEIGHTS] = d.T * d.k * 4;
  sz[SSB_WS_ROWS] = d.T * d.k * 4;
  sz[SSB_WS_COUNTS] = (d.E + 1) * 4;
  sz[SSB_WS_OFFSETS] = (d.E + 2) * 4;
  sz[SSB_WS_MASKS] = d.nblocks * d.E * 8 * 4;
  sz[SSB_WS_BLOCKS] = d.nblocks * d.E * 4;
  sz[SSB_WS_MTILES] = (d.mtile_cap + d.mpair_cap) * 16;   // tile table, then the CTA-pair table
  sz[SSB_WS_NUM_MTILES] = 16;
  sz[SSB_WS_XQ_PERM] = d.rcap * d.H / 2;
  sz[SSB_WS_XSF_PERM] = (d.rcap / 128) * d.ncbH * 512;
  sz[SSB_WS_ACT] = d.rcap * d.F / 2;
  sz[SSB_WS_ACT_SF] = (d.rcap / 128) * d.ncbF * 512;
  sz[SSB_WS_Y] = d.rcap * d.H * 2;
  sz[SSB_WS_ROW_SRC] = d.rcap * 4;
  int64_t o = 0;
  for (int i = 0; i < SSB_WS_END; ++i) {
    off[i] = o;
    o += align256(sz[i] > 0 ? sz[i] : 16);
  }
  off[SSB_WS_END] = o;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

const char* ssb_version(void) { return "ssengine_b200 0.1 (sm_100a)"; }

int64_t ssb_sf_atom_cols(int64_t K) { return ssb::sf_atom_cols(K); }

int ssb_nvfp4_quantize(const void* x, int64_t rows, int64_t K, int64_t ldx, float gs, uint8_t* codes, int64_t ldc,
                       uint8_t* sf, void* stream) {
  if (x == nullptr || codes == nullptr || sf == nullptr || rows < 0) return kErrArgs;
  return ssb::launch_nvfp4_quantize(x, rows, K, ldx, gs, codes, ldc, sf, static_cast<cudaStream_t>(stream));
}

int ssb_nvfp4_gemm(int32_t epilogue, const uint8_t* a_codes, const uint8_t* a_sf, int64_t M, int64_t K,
                   const uint8_t* b_codes, const uint8_t* b_sf, int64_t N, float alpha, void* out, int64_t ldo,
                   uint8_t* out_sf, float out_gs, int32_t* status, void* stream) {
  if (a_codes == nullptr || a_sf == nullptr || b_codes == nullptr || b_sf == nullptr || out == nullptr || M < 0 ||
      K <= 0 || N <= 0 || M > (1ll << 30) || N > (1ll << 30))
    return kErrArgs;
  if (!aligned16(a_codes) || !aligned16(b_codes) || !aligned16(out) || (K / 2) % 16 != 0) return kErrArgs;
  if (epilogue == SSB_EPI_F32 && (ldo % 4 != 0 || ldo < N)) return kErrArgs;
  if (epilogue == SSB_EPI_BF16 && ldo < N) return kErrArgs;
  if (epilogue == SSB_EPI_SWIGLU && (out_sf == nullptr || ldo < N / 4)) return kErrArgs;
  if (M == 0) return kOk;
  ssb::GemmArgs g;
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.M = static_cast<int32_t>(M);
  g.K = static_cast<int32_t>(K);
  g.N = static_cast<int32_t>(N);
  g.ncb_k = static_cast<int32_t>(ssb::sf_atom_cols(K));
  g.alpha_scalar = alpha;
  g.out = out;
  g.ldo = ldo;
  g.out_sf = out_sf;
  g.out_ncb = static_cast<int32_t>(ssb::sf_atom_cols(N / 2));
  g.out_gs = out_gs;
  g.status = status;
  const int64_t b_rows = epilogue == SSB_EPI_F32 ? ceil_div(N, 128) * 128 : N;
  return ssb::launch_gemm_nvfp4(epilogue, a_codes, M, K / 2, b_codes, b_rows, K / 2, g, ssb::device_sm_count(),
                                static_cast<cudaStream_t>(stream));
}

int ssb_nvfp4_gemm_grouped(int32_t epilogue, const uint8_t* a_codes, const uint8_t* a_sf, int64_t a_rows, int64_t K,
                           const uint8_t* b_codes, const uint8_t* b_sf, int64_t N, int32_t groups, const float* alpha,
                           const int32_t* tiles, const int32_t* num_tiles, int32_t tile_cap, void* out, int64_t ldo,
                           int32_t* status, void* stream) {
  if (a_codes == nullptr || a_sf == nullptr || b_codes == nullptr || b_sf == nullptr || out == nullptr ||
      tiles == nullptr || num_tiles == nullptr || alpha == nullptr || a_rows <= 0 || K <= 0 || N <= 0 || groups <= 0 ||
      tile_cap <= 0 || epilogue != SSB_EPI_BF16 || ldo < N)
    return kErrArgs;
  if (!aligned16(a_codes) || !aligned16(b_codes) || !aligned16(out) || (K / 2) % 16 != 0) return kErrArgs;
  ssb::GemmArgs g;
  g.sfa = a_sf;
  g.sfb = b_sf;
  g.mtiles = tiles;
  g.num_mtiles = num_tiles;
  g.mtile_cap = tile_cap;
  g.K = static_cast<int32_t>(K);
  g.N = static_cast<int32_t>(N);
  g.ncb_k = static_cast<int32_t>(ssb::sf_atom_cols(K));
  g.alpha = alpha;
  g.out = out;
  g.ldo = ldo;
  g.status = status;
  return ssb::launch_gemm_nvfp4(epilogue, a_codes, a_rows, K / 2, b_codes, static_cast<int64_t>(groups) * N, K / 2, g,
                                ssb::device_sm_count(), static_cast<cudaStream_t>(stream));
}

int ssb_rmsnorm_cols(const void* x, int64_t ldx, int32_t width, int64_t rows, const void* w, float eps, void* y,
                     int64_t ldy, void* stream) {
  return ssb::launch_rmsnorm_cols(x, ldx, width, rows, w, eps, y, ldy, static_cast<cudaStream_t>(stream));
}

int ssb_rope(void* x, int64_t ldx, int32_t heads, int64_t head_stride, const int64_t* positions, int64_t rows,
             float theta, void* stream) {
  return ssb::launch_rope(x, ldx, heads, head_stride, positions, rows, theta, static_cast<cudaStream_t>(stream));
}

int ssb_transpose_heads(const void* src, void* dst, int64_t rows, int64_t rows_pad, int32_t heads, int32_t dim,
                        int64_t row_ld, int64_t head_stride, int32_t to_heads, void* stream) {
  return ssb::launch_transpose_heads(src, dst, rows, rows_pad, heads, dim, row_ld, head_stride, to_heads != 0,
                                     static_cast<cudaStream_t>(stream));
}

int ssb_concat_cols(const void* a, int64_t lda, int32_t wa, const void* b, int64_t ldb, int32_t wb, void* out,
                    int64_t ldo, int64_t rows, void* stream) {
  return ssb::launch_concat_cols(a, lda, wa, b, ldb, wb, out, ldo, rows, static_cast<cudaStream_t>(stream));
}

int ssb_head_tiles(int32_t heads, int64_t rows_pad, int32_t* tiles, int64_t tile_cap, int32_t* num_tiles,
                   void* stream) {
  return ssb::launch_head_tiles(heads, rows_pad, tiles, tile_cap, num_tiles, static_cast<cudaStream_t>(stream));
}

int ssb_moe_route_sigmoid(const float* logits, int64_t T, int32_t E, int32_t k, const float* bias, int32_t n_group,
                          int32_t topk_group, float scale, int32_t* ids, float* weights, void* stream) {
  if (logits == nullptr || ids == nullptr || weights == nullptr || T < 0) return kErrArgs;
  return ssb::launch_moe_route_sigmoid(logits, T, E, k, bias, n_group, topk_group, scale, ids, weights,
                                       static_cast<cudaStream_t>(stream));
}

int ssb_moe_route(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids, float* weights, void* stream) {
  if (logits == nullptr || ids == nullptr || weights == nullptr || T < 0) return kErrArgs;
  return ssb::launch_moe_route(logits, T, E, k, ids, weights, static_cast<cudaStream_t>(stream));
}

int ssb_topk_canonical(const float* logits, int64_t rows, int64_t ld, const int32_t* ks, const int32_t* ke, int32_t k,
                       int32_t* out, int32_t max_keys, void* stream) {
  if (logits == nullptr || ks == nullptr || ke == nullptr || out == nullptr || rows < 0 || k <= 0 || ld <= 0 ||
      max_keys < 0)
    return kErrArgs;
  return ssb::launch_topk_canonical(logits, rows, ld, ks, ke, k, out, max_keys, static_cast<cudaStream_t>(stream));
}

int ssb_stage_metadata(const int32_t* qsl, const int32_t* starts, const int32_t* page_ptr, const int32_t* pages,
                       int32_t R, int64_t T, int64_t bucket, int32_t page_tokens, int32_t width, int64_t* positions,
                       int64_t* slots, int32_t* table, void* stream) {
  if (positions == nullptr || slots == nullptr || (R > 0 && (qsl == nullptr || starts == nullptr ||
                                                              page_ptr == nullptr || pages == nullptr)))
    return kErrArgs;
  return ssb::launch_stage_metadata(qsl, starts, page_ptr, pages, R, T, bucket, page_tokens, width, positions, slots,
                                    table, static_cast<cudaStream_t>(stream));
}

int ssb_embed_rows(const void* table, int64_t vocab, int64_t H, const int64_t* ids, int64_t T, void* out,
                   void* stream) {
  if (table == nullptr || ids == nullptr || out == nullptr) return kErrArgs;
  return ssb::launch_embed_rows(table, vocab, H, ids, T, out, static_cast<cudaStream_t>(stream));
}

int ssb_rmsnorm(const void* x, int64_t H, const int64_t* rows, int64_t n, const void* w, float eps, void* y,
                void* stream) {
  if (x == nullptr || w == nullptr || y == nullptr) return kErrArgs;
  return ssb::launch_rmsnorm(x, H, rows, n, w, eps, y, static_cast<cudaStream_t>(stream));
}

int ssb_gated_rmsnorm(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps, void* y,
                      int64_t ldy, int64_t rows, int32_t heads, void* stream) {
  return ssb::launch_gated_rmsnorm(x, ldx, gate, ldg, w, eps, y, ldy, rows, heads, static_cast<cudaStream_t>(stream));
}

int ssb_gated_rmsnorm_nvfp4(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps,
                            float gs, void* codes, int64_t ldc, void* sf, int64_t rows, int32_t heads, void* stream) {
  return ssb::launch_gated_rmsnorm_nvfp4(x, ldx, gate, ldg, w, eps, gs, static_cast<uint8_t*>(codes), ldc,
                                         static_cast<uint8_t*>(sf), rows, heads, static_cast<cudaStream_t>(stream));
}

int ssb_hc_expand(const void* x, int64_t T, int64_t H, void* out, void* stream) {
  return ssb::launch_hc_expand(x, T, H, out, static_cast<cudaStream_t>(stream));
}

int ssb_hc_mean(const void* res, int64_t H, const int64_t* rows, int64_t n, void* out, void* stream) {
  return ssb::launch_hc_mean(res, H, rows, n, out, static_cast<cudaStream_t>(stream));
}

int ssb_argmax_rows(const float* logits, int64_t ld, int64_t N, int64_t n, int64_t* out, void* stream) {
  if (logits == nullptr || out == nullptr) return kErrArgs;
  return ssb::launch_argmax_rows(logits, ld, N, n, out, static_cast<cudaStream_t>(stream));
}

int ssb_mhc(const ssb_mhc_params* p, const void* x, const void* res, const float* post_in, const float* comb_in,
            void* new_res, float* post_out, float* comb_out, void* y, int64_t T, void* stream) {
  return ssb_mhc_ws(p, x, res, post_in, comb_in, new_res, post_out, comb_out, y, T, nullptr, 0, stream);
}

int64_t ssb_mhc_workspace_bytes(int64_t T) { return T < 0 ? -1 : ssb::mhc_workspace_bytes(T); }

int ssb_mhc_ws(const ssb_mhc_params* p, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, float* post_out, float* comb_out, void* y, int64_t T, void* workspace,
               int64_t ws_bytes, void* stream) {
  if (p == nullptr || res == nullptr || T < 0) return kErrArgs;
  const bool do_post = x != nullptr;
  const bool do_pre = y != nullptr;
  if (do_post && (post_in == nullptr || comb_in == nullptr || new_res == nullptr)) return kErrArgs;
  if (do_pre && (p->fn == nullptr || p->scale == nullptr || p->base == nullptr || p->norm_weight == nullptr ||
                 post_out == nullptr || comb_out == nullptr))
    return kErrArgs;
  if (p->hc_mult != 4) return kErrArgs;
  return ssb::launch_mhc(do_post, do_pre, x, res, post_in, comb_in, new_res, p->fn, p->scale, p->base, p->norm_weight,
                         post_out, comb_out, y, T, p->hidden, p->rms_eps, p->pre_eps, p->sinkhorn_eps, p->post_mult,
                         p->sinkhorn_repeat, p->norm_eps, workspace, ws_bytes, p->status,
                         static_cast<cudaStream_t>(stream));
}

static bool kda_args(const ssb_kda_layer* L, const void* x, int64_t ldx, const int32_t* seqs, int64_t R,
                     ssb::KdaArgs& a) {
  if (L == nullptr || L->head_dim != 128 || L->heads <= 0 || L->heads > 1024 || R < 0 || R > (1 << 20)) return false;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.conv_w = static_cast<const __nv_bfloat16*>(L->conv_weight);
  a.a_log = L->a_log;
  a.dt_bias = L->dt_bias;
  a.lower_bound = L->lower_bound;
  a.scale = L->scale;
  a.conv_state = static_cast<__nv_bfloat16*>(L->conv_state);
  a.cs_stride = L->conv_state_stride;
  a.rec_state = L->rec_state;
  a.rs_stride = L->rec_state_stride;
  a.seqs = seqs;
  a.R = static_cast<int32_t>(R);
  a.H = L->heads;
  a.P = L->heads * 128;
  return true;
}

int ssb_kda_prefill_ws(const ssb_kda_layer* layer, const void* x, int64_t ldx, const void* g, int64_t ldg,
                       const void* beta, int64_t ldb, int64_t T, const int32_t* seqs, int64_t R, void* out,
                       int64_t ldo, void* workspace, int64_t ws_bytes, int32_t* status, void* stream) {
  ssb::KdaArgs a;
  if (T < 0 || !kda_args(layer, x, ldx, seqs, R, a)) return kErrArgs;
  a.g = static_cast<const __nv_bfloat16*>(g);
  a.ldg = ldg;
  a.beta = static_cast<const __nv_bfloat16*>(beta);
  a.ldb = ldb;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.status = status;
  a.T = T;
  a.ws = static_cast<uint8_t*>(workspace);
  a.ws_bytes = ws_bytes;
  if (ldg < a.P || ldb < a.H || (workspace != nullptr && ws_bytes <= 0)) return kErrArgs;
  return ssb::launch_kda_prefill(a, static_cast<cudaStream_t>(stream));
}

int ssb_kda_prefill(const ssb_kda_layer* layer, const void* x, int64_t ldx, const void* g, int64_t ldg,
                    const void* beta, int64_t ldb, int64_t T, const int32_t* seqs, int64_t R, void* out, int64_t ldo,
                    int32_t* status, void* stream) {
  return ssb_kda_prefill_ws(layer, x, ldx, g, ldg, beta, ldb, T, seqs, R, out, ldo, nullptr, 0, status, stream);
}

int64_t ssb_kda_workspace_bytes(int32_t heads, int64_t T, int64_t R) {
  if (heads <= 0 || T < 0 || R < 0 || R > (1 << 30)) return -1;
  return ssb::kda_workspace_bytes(heads, T, static_cast<int>(R));
}

int ssb_kda_conv(const ssb_kda_layer* layer, const void* x, int64_t ldx, int64_t T, const int32_t* seqs, int64_t R,
                 void* q, void* k, void* v, void* stream) {
  ssb::KdaArgs a;
  if (T < 0 || !kda_args(layer, x, ldx, seqs, R, a)) return kErrArgs;
  return ssb::launch_kda_conv(a, T, q, k, v, static_cast<cudaStream_t>(stream));
}

int ssb_indexer_logits(const void* q, const void* w, int64_t ldw, int64_t T, const void* k_cache, int64_t pool_rows,
                       const int32_t* page_table, int64_t width, const int32_t* groups, int64_t G, float* logits,
                       int64_t ldl, int32_t* status, void* stream) {
  if (width <= 0 || width > (1 << 24) || G < 0 || G > (1 << 28)) return kErrArgs;
  ssb::IdxArgs a;
  a.w = w;
  a.ldw = ldw;
  a.T = T;
  a.table = page_table;
  a.width = static_cast<int32_t>(width);
  a.groups = groups;
  a.G = static_cast<int32_t>(G);
  a.logits = logits;
  a.ldl = ldl;
  a.status = status;
  return ssb::launch_indexer_logits(q, k_cache, pool_rows, a, static_cast<cudaStream_t>(stream));
}

int ssb_indexer_logits_fp8(const uint8_t* q8, const float* q_scale, const void* w, int64_t ldw, int64_t T,
                           const uint8_t* k_pages, int64_t pages, const int32_t* page_table, int64_t width,
                           const int32_t* groups, int64_t G, float* logits, int64_t ldl, int32_t* status,
                           void* stream) {
  if (width <= 0 || width > (1 << 24) || G < 0 || G > (1 << 28) || pages > (1LL << 26)) return kErrArgs;
  ssb::IdxArgs a;
  a.w = w;
  a.ldw = ldw;
  a.T = T;
  a.table = page_table;
  a.width = static_cast<int32_t>(width);
  a.groups = groups;
  a.G = static_cast<int32_t>(G);
  a.logits = logits;
  a.ldl = ldl;
  a.status = status;
  return ssb::launch_indexer_logits_fp8(q8, q_scale, k_pages, pages, a, static_cast<cudaStream_t>(stream));
}

int ssb_indexer_q_quant(const void* q, int64_t rows, uint8_t* q8, float* q_scale, void* stream) {
  return ssb::launch_indexer_q_quant(q, rows, q8, q_scale, static_cast<cudaStream_t>(stream));
}

int ssb_indexer_expand(const int32_t* pool_ids, int64_t ldp, int32_t k, const int64_t* positions, int64_t rows,
                       int32_t* out, int64_t ldo, void* stream) {
  return ssb::launch_indexer_expand(pool_ids, ldp, k, positions, out, ldo, rows, static_cast<cudaStream_t>(stream));
}

int ssb_sparse_mla(const void* q, int64_t T, const void* kv_cache, const int32_t* indices, int64_t ld_idx,
                   int32_t n_idx, const int32_t* qsl, int32_t R, const int32_t* page_table, int64_t width,
                   float bmm1_scale, float bmm2_scale, void* out, int32_t* status, void* stream) {
  if (width <= 0 || width > (1 << 24)) return kErrArgs;
  ssb::MlaArgs a;
  a.q = static_cast<const uint8_t*>(q);
  a.kv = static_cast<const uint8_t*>(kv_cache);
  a.indices = indices;
  a.ld_idx = ld_idx;
  a.n_idx = n_idx;
  a.qsl = qsl;
  a.R = R;
  a.table = page_table;
  a.width = static_cast<int32_t>(width);
  a.scale = bmm1_scale;
  a.bmm2 = bmm2_scale;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.T = T;
  a.status = status;
  return ssb::launch_sparse_mla(a, static_cast<cudaStream_t>(stream));
}

int ssb_mla_cache_append(const void* src, int64_t lds, const int64_t* slots, int64_t T, void* cache, float k_scale,
                         void* stream) {
  return ssb::launch_mla_append(src, lds, slots, T, cache, k_scale, static_cast<cudaStream_t>(stream));
}

int ssb_mla_q_pack(const void* lat, int64_t rows_pad, const void* rope, int64_t ldr, int64_t rope_stride, int64_t T,
                   void* q8, float q_scale, void* stream) {
  return ssb::launch_mla_q_pack(lat, rows_pad, rope, ldr, rope_stride, T, q8, q_scale,
                                static_cast<cudaStream_t>(stream));
}

int ssb_kpool_insert(const void* k, const void* gate, int64_t ld, const float* ape, const int32_t* reqs, int64_t R,
                     int32_t max_rows, const int32_t* page_table, int64_t width, void* pool_cache, void* tail_ring,
                     void* stream) {
  if (R < 0 || R > (1 << 20) || width <= 0 || width > (1 << 24)) return kErrArgs;
  ssb::KpoolArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.ld = ld;
  a.ape = ape;
  a.reqs = reqs;
  a.R = static_cast<int32_t>(R);
  a.table = page_table;
  a.width = static_cast<int32_t>(width);
  a.pool = static_cast<__nv_bfloat16*>(pool_cache);
  a.tail = static_cast<__nv_bfloat16*>(tail_ring);
  return ssb::launch_kpool_insert(a, max_rows, static_cast<cudaStream_t>(stream));
}

int ssb_kpool_insert_fp8(const void* k, const void* gate, int64_t ld, const float* ape, const int32_t* reqs, int64_t R,
                         int32_t max_rows, const int32_t* page_table, int64_t width, uint8_t* pool_pages,
                         void* tail_ring, void* stream) {
  if (R < 0 || R > (1 << 20) || width <= 0 || width > (1 << 24) || pool_pages == nullptr) return kErrArgs;
  ssb::KpoolArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.ld = ld;
  a.ape = ape;
  a.reqs = reqs;
  a.R = static_cast<int32_t>(R);
  a.table = page_table;
  a.width = static_cast<int32_t>(width);
  a.pool8 = pool_pages;
  a.tail = static_cast<__nv_bfloat16*>(tail_ring);
  return ssb::launch_kpool_insert(a, max_rows, static_cast<cudaStream_t>(stream));
}

int64_t ssb_moe_workspace_bytes(const ssb_moe_layer* layer, int64_t T) {
  MoeDims d;
  if (!dims_of(layer, T, d)) return -1;
  int64_t off[SSB_WS_END + 1];
  layout(d, off);
  return off[SSB_WS_END];
}

int ssb_moe_workspace_offsets(const ssb_moe_layer* layer, int64_t T, int64_t* offsets, int32_t n) {
  MoeDims d;
  if (!dims_of(layer, T, d) || offsets == nullptr || n < 0) return kErrArgs;
  int64_t off[SSB_WS_END + 1];
  layout(d, off);
  for (int i = 0; i < n && i <= SSB_WS_END; ++i) offsets[i] = off[i];
  return kOk;
}

}  // extern "C"

namespace {

// The layer's launch sequence; when `events` is not null, events[i] is recorded before step i and events[9] after the
// last (steps: quantize, router GEMM, route, count, offsets, scatter, gate_up GEMM, down GEMM, combine).
int moe_forward(const ssb_moe_layer* L, const void* x, int64_t T, void* out, void* ws, int64_t ws_bytes,
                int32_t* status, void* stream_, void* const* events) {
  MoeDims d;
  if (!dims_of(L, T, d)) return kErrArgs;
  if (T == 0) return kOk;
  if (x == nullptr || out == nullptr || ws == nullptr) return kErrArgs;
  if (L->router_codes == nullptr || L->router_sf == nullptr || L->w1_codes == nullptr || L->w1_sf == nullptr ||
      L->w1_alpha == nullptr || L->w2_codes == nullptr || L->w2_sf == nullptr || L->w2_alpha == nullptr ||
      L->router_rows < d.E || L->router_rows % 128 != 0)
    return kErrArgs;
  if (!aligned16(x) || !aligned16(out) || (reinterpret_cast<uintptr_t>(ws) & 255)) return kErrArgs;
  int64_t off[SSB_WS_END + 1];
  layout(d, off);
  if (ws_bytes < off[SSB_WS_END]) return kErrWorkspace;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto at = [&](int i) { return w + off[i]; };
  uint8_t* xq = at(SSB_WS_XQ);
  uint8_t* xsf = at(SSB_WS_XSF);
  float* logits = reinterpret_cast<float*>(at(SSB_WS_LOGITS));
  int32_t* ids = reinterpret_cast<int32_t*>(at(SSB_WS_IDS));
  float* wts = reinterpret_cast<float*>(at(SSB_WS_WEIGHTS));
  int32_t* rows = reinterpret_cast<int32_t*>(at(SSB_WS_ROWS));
  int32_t* counts = reinterpret_cast<int32_t*>(at(SSB_WS_COUNTS));
  int32_t* offsets = reinterpret_cast<int32_t*>(at(SSB_WS_OFFSETS));
  uint32_t* masks = reinterpret_cast<uint32_t*>(at(SSB_WS_MASKS));
  int32_t* bcounts = reinterpret_cast<int32_t*>(at(SSB_WS_BLOCKS));
  int32_t* mtiles = reinterpret_cast<int32_t*>(at(SSB_WS_MTILES));
  int32_t* num_mtiles = reinterpret_cast<int32_t*>(at(SSB_WS_NUM_MTILES));
  uint8_t* xqp = at(SSB_WS_XQ_PERM);
  int32_t* row_src = reinterpret_cast<int32_t*>(at(SSB_WS_ROW_SRC));
  uint8_t* xsfp = at(SSB_WS_XSF_PERM);
  uint8_t* act = at(SSB_WS_ACT);
  uint8_t* asf = at(SSB_WS_ACT_SF);
  void* y = at(SSB_WS_Y);
  const int sms = ssb::device_sm_count();
  int rc;
  auto mark = [&](int i) {
    if (events != nullptr) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), stream);
  };

  // 1. input quantization (token order)
  mark(0);
  rc = ssb::launch_nvfp4_quantize(x, T, d.H, d.H, L->gs_x, xq, d.H / 2, xsf, stream);
  if (rc != kOk) return rc;
  // 2. router logits
  mark(1);
  {
    ssb::GemmArgs g;
    g.sfa = xsf;
    g.sfb = L->router_sf;
    g.M = static_cast<int32_t>(T);
    g.K = static_cast<int32_t>(d.H);
    g.N = static_cast<int32_t>(d.E);
    g.ncb_k = static_cast<int32_t>(d.ncbH);
    g.alpha_scalar = L->router_alpha;
    g.out = logits;
    g.ldo = d.E;
    g.status = status;
    if (d.E % 4 != 0) return kErrArgs;   // fp32 rows of the logits are stored as 16-byte vectors
    rc = ssb::launch_gemm_nvfp4(ssb::kEpiF32, xq, d.Tpad, d.H / 2, L->router_codes, L->router_rows, d.H / 2, g, sms,
                                stream);
    if (rc != kOk) return rc;
  }
  // 3. routing, 4. permutation
  mark(2);
  if (L->routing == SSB_ROUTE_SIGMOID_BIAS)
    rc = ssb::launch_moe_route_sigmoid(logits, T, static_cast<int32_t>(d.E), static_cast<int32_t>(d.k), L->route_bias,
                                       L->n_group, L->topk_group, L->routed_scale, ids, wts, stream);
  else if (L->routing == SSB_ROUTE_SOFTMAX)
    rc = ssb::launch_moe_route(logits, T, static_cast<int32_t>(d.E), static_cast<int32_t>(d.k), ids, wts, stream);
  else
    rc = kErrArgs;
  if (rc != kOk) return rc;
  mark(3);
  rc = ssb::launch_moe_count(ids, T, static_cast<int32_t>(d.E), static_cast<int32_t>(d.k), masks, bcounts, stream);
  if (rc != kOk) return rc;
  mark(4);
  int32_t* mpairs = mtiles + 4 * d.mtile_cap;
  rc = ssb::launch_moe_offsets(T, static_cast<int32_t>(d.E), bcounts, counts, offsets, mtiles, num_mtiles,
                               static_cast<int32_t>(d.mtile_cap), mpairs, static_cast<int32_t>(d.mpair_cap), status,
                               stream);
  if (rc != kOk) return rc;
  mark(5);
  rc = ssb::launch_moe_scatter(ids, T, static_cast<int32_t>(d.E), static_cast<int32_t>(d.k), masks, bcounts, offsets,
                               rows, row_src, xq, d.H, xqp, stream);
  if (rc != kOk) return rc;
  rc = ssb::launch_moe_sf_gather(row_src, mtiles, num_mtiles, static_cast<int32_t>(d.mtile_cap), xsf, d.H, xsfp,
                                 stream);
  if (rc != kOk) return rc;
  // 5. grouped gate_up GEMM, SwiGLU + NVFP4 requant epilogue. When F is not a multiple of 256 the down GEMM's last
  //    k-block reads scale atoms past F that the epilogue never writes: they must hold zeros (finite scales times the
  //    zero-filled codes), not stale bytes.
  mark(6);
  if (d.F % 256 != 0 &&
      cudaMemsetAsync(asf, 0, static_cast<size_t>((d.rcap / 128) * d.ncbF * 512), stream) != cudaSuccess)
    return ssb::kErrCuda;
  {
    ssb::GemmArgs g;
    g.sfa = xsfp;
    g.sfb = L->w1_sf;
    g.mtiles = mtiles;
    g.num_mtiles = num_mtiles;
    g.mtile_cap = static_cast<int32_t>(d.mtile_cap);
    g.K = static_cast<int32_t>(d.H);
    g.N = static_cast<int32_t>(2 * d.F);
    g.ncb_k = static_cast<int32_t>(d.ncbH);
    g.alpha = L->w1_alpha;
    g.out = act;
    g.ldo = d.F / 2;
    g.out_sf = asf;
    g.out_ncb = static_cast<int32_t>(d.ncbF);
    g.out_gs = L->gs_h;
    g.status = status;
    rc = ssb::launch_gemm_nvfp4(ssb::kEpiSwiGLU, xqp, d.rcap, d.H / 2, L->w1_codes, (d.E + 1) * 2 * d.F, d.H / 2, g,
                                sms, stream);
    if (rc != kOk) return rc;
  }
  // 6. grouped down GEMM -> bf16 rows
  mark(7);
  {
    ssb::GemmArgs g;
    g.sfa = asf;
    g.sfb = L->w2_sf;
    g.mtiles = mtiles;
    g.num_mtiles = num_mtiles;
    g.mtile_cap = static_cast<int32_t>(d.mtile_cap);
    // CTA pairs: five 38 KB stages instead of three 54 KB ones (this GEMM's bf16 staging takes a stage's room), which
    // its short K (4 k-blocks a tile) needs; the gate_up GEMM measured slower paired (half-empty pairs on odd tile
    // counts cost more than the deeper ring gives)
    g.mpairs = mpairs;
    g.num_mpairs = num_mtiles + 1;
    g.mpair_cap = static_cast<int32_t>(d.mpair_cap);
    g.K = static_cast<int32_t>(d.F);
    g.N = static_cast<int32_t>(d.H);
    g.ncb_k = static_cast<int32_t>(d.ncbF);
    g.alpha = L->w2_alpha;
    g.out = y;
    g.ldo = d.H;
    g.status = status;
    rc = ssb::launch_gemm_nvfp4(ssb::kEpiBF16, act, d.rcap, d.F / 2, L->w2_codes, (d.E + 1) * d.H, d.F / 2, g, sms,
                                stream);
    if (rc != kOk) return rc;
  }
  // 7. weighted combine + shared expert
  mark(8);
  rc = ssb::launch_moe_combine(y, d.H, rows, wts, offsets, T, static_cast<int32_t>(d.E), static_cast<int32_t>(d.k),
                               L->add_input ? x : nullptr, out, stream);
  if (rc != kOk) return rc;
  mark(9);
  return kOk;
}

}  // namespace

extern "C" {

int ssb_moe_forward(const ssb_moe_layer* L, const void* x, int64_t T, void* out, void* ws, int64_t ws_bytes,
                    int32_t* status, void* stream) {
  return moe_forward(L, x, T, out, ws, ws_bytes, status, stream, nullptr);
}

int ssb_moe_forward_profiled(const ssb_moe_layer* L, const void* x, int64_t T, void* out, void* ws, int64_t ws_bytes,
                             int32_t* status, void* stream, void* const* events) {
  if (events == nullptr) return kErrArgs;
  for (int i = 0; i <= SSB_MOE_STEPS; ++i)
    if (events[i] == nullptr) return kErrArgs;
  return moe_forward(L, x, T, out, ws, ws_bytes, status, stream, events);
}

}  // extern "C"
