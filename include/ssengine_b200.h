/* C ABI of the B200 prefill-stage library (libssengine_b200.so, sm_100a).
 *
 * Conventions (the style of the reference's only native ABI, ssengine/native/kda_split_heads.cpp:17-19: plain
 * pointers and sizes, an int return code, out-parameters):
 * - every pointer argument named *_codes, *_sf, x, out, ws, logits, ids, weights, status is DEVICE memory owned by
 *   the caller. Entry points that need scratch take it from the caller (`ws`, `workspace`), except three forms that
 *   allocate: ssb_kda_prefill and ssb_mhc (one stream-ordered cudaMallocAsync + cudaFreeAsync per call; their `_ws`
 *   forms take a caller workspace and allocate nothing) and ssb_ipc_open (maps a peer's buffer). No other entry point
 *   allocates device memory;
 * - `stream` is a cudaStream_t passed as void*; every entry point only enqueues work on it (no host sync);
 * - return 0 on success, else an ssb status code (1 bad arguments, 2 CUDA launch error, 3 workspace too small,
 *   5 driver entry point missing, 7 size beyond ssb_moe_route_permute_noalloc's limits); device-side failures (4 a bounded wait expired, 6 a table overflowed) are written
 *   to the caller's int32 device `status` word (first error wins), read by the caller after the stream's work ends;
 * - NVFP4 operands: e2m1 codes packed two per byte (even element in the low nibble), rows K/2 bytes apart; scales
 *   are e4m3 bytes in the 128x4-atom layout: rows padded to 128, K padded to 256, atom (row block rb, atom column
 *   cb) at ((rb * ssb_sf_atom_cols(K)) + cb) * 512, scale (r, c) at byte (r % 32) * 16 + ((r / 32) % 4) * 4 + c % 4.
 */
#ifndef SSENGINE_B200_H_
#define SSENGINE_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version string. */
const char* ssb_version(void);

/* Scale atom columns per 128-row block for a reduction length K (K padded to 256, 4 atoms per 256). */
int64_t ssb_sf_atom_cols(int64_t K);

/* NVFP4 quantization of bf16 rows with a static global scale `gs`:
 *   sf = e4m3((amax16 / 6) * gs), code = e2m1(x * (gs / sf)), each step one IEEE fp32 operation.
 * x [rows, K] bf16 (row pitch ldx elements), codes [rows, ldc bytes], sf atoms (rows padded to 128).
 * Replaces the reference's activation quantizers, vLLM `scaled_fp4_quant` at ssengine/kernels.py:109-111 (config 8),
 * :116-118 (config 10) and :179-181 (config 29). */
int ssb_nvfp4_quantize(const void* x, int64_t rows, int64_t K, int64_t ldx, float gs, uint8_t* codes, int64_t ldc,
                       uint8_t* sf, void* stream);

/* Output stage selectors of ssb_nvfp4_gemm. */
#define SSB_EPI_F32 0    /* out fp32 [M, ldo] = alpha * A x B^T, columns < N */
#define SSB_EPI_BF16 1   /* out bf16 [M, ldo] = alpha * A x B^T (N % 256 == 0) */
#define SSB_EPI_SWIGLU 2 /* B rows in 256-row tiles of 128 gate + 128 up rows; h = silu(alpha g) * (alpha u),
                            quantized to NVFP4 with global scale out_gs: out = codes [M, ldo bytes], out_sf atoms */

/* Dense NVFP4 GEMM D = alpha * A x B^T on tcgen05 tensor cores (e2m1 x e2m1, ue4m3 scales per 16 elements applied
 * in the MMA, fp32 accumulation in TMEM). A [M, K] codes + scales, B [N, K] codes + scales (rows padded to 128 in the
 * scale layout), K % 64 == 0. Replaces the reference's NVFP4 dense projections, FlashInfer `mm_fp4` at
 * ssengine/kernels.py:112-121 (configs 9, 11), and (with BASELINE's NVFP4 projections) the BF16 router / shared
 * expert / projection GEMMs at :174-178, :188-193. */
int ssb_nvfp4_gemm(int32_t epilogue, const uint8_t* a_codes, const uint8_t* a_sf, int64_t M, int64_t K,
                   const uint8_t* b_codes, const uint8_t* b_sf, int64_t N, float alpha, void* out, int64_t ldo,
                   uint8_t* out_sf, float out_gs, int32_t* status, void* stream);

/* MoE routing: softmax over the top-k logits of each token; selection by value descending, ties to the lower expert
 * index; slots in rank order. logits fp32 [T, E] (E <= 512), ids int32 [T, k], weights fp32 [T, k].
 * Replaces the routing stage of FlashInfer `trtllm_fp4_block_scale_moe` (ssengine/kernels.py:182-187, config 30). */
int ssb_moe_route(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids, float* weights, void* stream);

/* Canonical top-k of the DSA indexer, per row: over columns [ks[r], ke[r]) of logits (fp32, row pitch ld elements),
 * every key above the k-th largest value plus the lowest-column keys equal to it, as columns relative to ks[r] in
 * ascending order, -1 past the number selected; rows of at most k keys select all their keys. out int32 [rows, k].
 * max_keys: an upper bound of ke - ks (rows up to min(max_keys, 4096) keys are cached in shared memory, longer rows
 * are re-read from L2 per pass). NaN sorts below every number. Replaces the reference's per-row top-k kernels (DeepSelect /
 * vLLM top_k_per_row_prefill, ssengine/kernels.py:147-154, configs 20/21) followed by `topk_canon.canonicalize`
 * (ssengine/model/topk_canon.py:130-147): the canonical set is selected directly. */
int ssb_topk_canonical(const float* logits, int64_t rows, int64_t ld, const int32_t* ks, const int32_t* ke, int32_t k,
                       int32_t* out, int32_t max_keys, void* stream);

/* Device-side metadata of a microbatch (the reference builds it with numpy on the host: ssengine/model/metadata.py
 * `g0_table` :79-96 and `graph_rows` :65-76, inside `StageMetadata.build` :210-313). Inputs, device, the plan's
 * requests in row order: qsl int32 [R+1] (first row of each request, qsl[R] = T), starts int32 [R] (tokens already in
 * KV), page_ptr int32 [R+1] and pages int32 (each request's KV pages of page_tokens tokens, page p = kernel blocks
 * p * kpp .. p * kpp + kpp - 1, kpp = page_tokens / 64). Outputs: positions int64 [bucket] and slots int64 [bucket]
 * (rows >= T of a CUDA-graph bucket: position 0, slot -1), table int32 [R, width] (kernel-block table, zero past a
 * request's pages; may be null). Bit-exact with the reference's functions. */
int ssb_stage_metadata(const int32_t* qsl, const int32_t* starts, const int32_t* page_ptr, const int32_t* pages,
                       int32_t R, int64_t T, int64_t bucket, int32_t page_tokens, int32_t width, int64_t* positions,
                       int64_t* slots, int32_t* table, void* stream);

/* Stage-0 embedding: out bf16 [T, H] = table bf16 [vocab, H] rows ids int64 [T] (ids outside [0, vocab): zeros).
 * Replaces the fork's embedding lookup on stage 0 (ssengine/model/stage.py:725-734, `hidden_in is None`). */
int ssb_embed_rows(const void* table, int64_t vocab, int64_t H, const int64_t* ids, int64_t T, void* out,
                   void* stream);

/* y bf16 [n, H] = RMSNorm(x[rows[i]]) * w (rows int64 [n] or null for rows 0..n-1), fp32 statistics.
 * Replaces vLLM `rms_norm` of the final norm (ssengine/kernels.py:200-202, config 34). */
int ssb_rmsnorm(const void* x, int64_t H, const int64_t* rows, int64_t n, const void* w, float eps, void* y,
                void* stream);

/* KDA output norm per 128-channel head: y = x * rsqrt(mean(x^2) + eps) * w[c % 128] * sigmoid(gate) (x, gate, y bf16
 * [rows, ld*] with heads * 128 columns; w bf16 [128]). Replaces the fork's FusedRMSNormGated(head_dim,
 * activation="sigmoid") of the KDA layer (vLLM kimi_linear `o_norm`). */
int ssb_gated_rmsnorm(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps, void* y,
                      int64_t ldy, int64_t rows, int32_t heads, void* stream);

/* The same norm with its output quantized for the next NVFP4 GEMM (the KDA o_proj): codes uint8 [rows, ldc] (two e2m1
 * per byte, ldc >= heads * 64) and ue4m3 scale atoms (128x4 layout, heads * 128 columns) of y / gs, equal byte for
 * byte to ssb_gated_rmsnorm followed by ssb_nvfp4_quantize; scale atoms past heads * 128 columns (up to the
 * 256-column padding) and past `rows` are left as they are (pass a zeroed buffer); the bf16 y is not written.
 * Replaces, where ssb_gated_rmsnorm stands, the fork's o_norm followed by the o_proj's `scaled_fp4_quant` (vLLM
 * kimi_linear). */
int ssb_gated_rmsnorm_nvfp4(const void* x, int64_t ldx, const void* gate, int64_t ldg, const void* w, float eps,
                            float gs, void* codes, int64_t ldc, void* sf, int64_t rows, int32_t heads, void* stream);

/* Stage 0's 4-stream residual: out bf16 [T, 4, H] = 4 copies of each embedding row x bf16 [T, H] (H % 8 == 0).
 * Replaces `hc_expand_cat` (ssengine/model/pp_patch.py:169-183). */
int ssb_hc_expand(const void* x, int64_t T, int64_t H, void* out, void* stream);

/* out bf16 [n, H] = mean over the 4 streams of res bf16 [T, 4, H] at rows (int64 [n], or row r when NULL): the last
 * stage's stream merge before the final norm (ssengine/model/stage.py:746-762 `head_logits`). */
int ssb_hc_mean(const void* res, int64_t H, const int64_t* rows, int64_t n, void* out, void* stream);

/* out int64 [n] = the lowest column of the maximum of logits fp32 [n, N] (row pitch ld; NaN never wins): the last
 * stage's greedy token (ssengine/model/stage.py:746-762 `head_logits` + argmax). */
int ssb_argmax_rows(const float* logits, int64_t ld, int64_t N, int64_t n, int64_t* out, void* stream);

/* mHC (4-stream hyper-connection) parameters of one layer boundary (device pointers except the scalars). */
typedef struct ssb_mhc_params {
  int32_t hidden;              /* H, % 128 == 0 (% 256 == 0 for a pre step) */
  int32_t hc_mult;             /* streams: 4 */
  const float* fn;             /* [24, 4H] fp32: mixes = z @ fn^T */
  const float* scale;          /* [3] fp32 */
  const float* base;           /* [24] fp32 */
  const void* norm_weight;     /* [H] bf16, the next layer's input RMSNorm */
  float rms_eps, pre_eps, sinkhorn_eps, post_mult, norm_eps;
  int32_t sinkhorn_repeat;
  int32_t* status;             /* device int32 status word or NULL: receives 4 if a bounded wait of a pre step expired */
} ssb_mhc_params;

/* mHC at a layer boundary. With x != NULL (post): new_res bf16 [T, 4, H] = post_in[j] * x + sum_i
 * comb_in[i][j] * res[i] (x bf16 [T, H], post_in fp32 [T, 4], comb_in fp32 [T, 4, 4]). With y != NULL (pre, on new_res
 * or, without post, on res): post_out fp32 [T, 4], comb_out fp32 [T, 4, 4] (Sinkhorn) and y bf16 [T, H] = the next
 * layer's RMS-normed input. Both: the reference's fused boundary `MegaMhcPostPre` (ssengine/model/pp_patch.py:125-153,
 * DeepGEMM mega_mhc, configs 1 and 7 at ssengine/kernels.py:76-80, 104-108); post only: `edge_send` (:156-158,
 * config 33); pre only: `edge_recv` + hc_pre (:160-163). */
int ssb_mhc(const ssb_mhc_params* p, const void* x, const void* res, const float* post_in, const float* comb_in,
            void* new_res, float* post_out, float* comb_out, void* y, int64_t T, void* stream);

/* Device bytes of the partial-mix workspace of a pre step for T rows (16 x T x 25 fp32); -1 for T < 0. */
int64_t ssb_mhc_workspace_bytes(int64_t T);

/* ssb_mhc with a caller-owned workspace (16-byte aligned, >= ssb_mhc_workspace_bytes(T); returns 3 when smaller), so
 * that the call allocates nothing; ssb_mhc allocates one on `stream` when it runs a pre step. A pre step is two
 * launches: the partial mixes of 64-row tiles over eighths of the hidden positions (post fused; one persistent CTA per
 * SM fed by TMA), then the partials summed in a fixed order, Sinkhorn and the layer input. */
int ssb_mhc_ws(const ssb_mhc_params* p, const void* x, const void* res, const float* post_in, const float* comb_in,
               void* new_res, float* post_out, float* comb_out, void* y, int64_t T, void* workspace,
               int64_t ws_bytes, void* stream);

/* One KDA layer of this stage (device pointers except the scalars). Head dim 128 (key = value). */
typedef struct ssb_kda_layer {
  int32_t heads;               /* H: KDA heads of this stage's layer */
  int32_t head_dim;            /* 128 */
  const void* conv_weight;     /* bf16 [3 * H * 128][4]: q | k | v channels, taps oldest row first */
  const float* a_log;          /* fp32 [H] */
  const float* dt_bias;        /* fp32 [H * 128] */
  float lower_bound;           /* gate lower bound (-5) */
  float scale;                 /* head_dim^-0.5 */
  void* conv_state;            /* bf16 conv state blocks [blocks][3][3 * H * 128] (x rows end-3 .. end-1) */
  int64_t conv_state_stride;   /* elements between blocks, % 8 == 0 */
  float* rec_state;            /* fp32 recurrent state blocks [blocks][H][128 value][128 key] */
  int64_t rec_state_stride;    /* elements between blocks */
} ssb_kda_layer;

/* KDA prefill of one layer over a microbatch: short conv (width 4, SiLU) of the in_proj rows x bf16 [T, ldx] (q | k |
 * v in columns [0, 3 * H * 128)), gate lower_bound * sigmoid(exp(A_log) * (g + dt_bias)) from the raw rows g bf16 [T,
 * ldg], ldg % 8 == 0), beta = sigmoid(raw beta bf16 [T, ldb]), q / k L2-normalised, chunked (64) delta-rule scan;
 * out bf16 [T, ldo]
 * (H * 128 columns). seqs int32 [R][4] device = {first row, end row, state block, has initial state}; a sequence
 * without initial state starts from zero conv rows and a zero state. Each sequence's recurrent state block is read
 * and written in place, then its conv state block (the sequence's last 3 x rows). Sequences are processed in table
 * order (longest first balances the grid). Rows outside every sequence are not written. status (device int32, may be
 * NULL) receives 4 if a chunk's row copies did not land within 1 s (that sequence's state block is then left as it
 * was).
 * Replaces `kda_prefill_forward` (ssengine/model/pp_patch.py:215-244: kda_conv.conv_qkv + kda_state.gather +
 * FlashInfer persistent KDA `fwd` + kda_state.scatter; configs 4 and 5 at ssengine/kernels.py:87-101). */
int ssb_kda_prefill(const ssb_kda_layer* layer, const void* x, int64_t ldx, const void* g, int64_t ldg,
                    const void* beta, int64_t ldb, int64_t T, const int32_t* seqs, int64_t R, void* out, int64_t ldo,
                    int32_t* status, void* stream);

/* Device bytes of the chunk workspace of ssb_kda_prefill_ws for `heads` heads, T rows and R sequences whose rows sum
 * to at most T (one 72.5 KB image per 64-row chunk and head, plus a header); -1 on bad arguments. */
int64_t ssb_kda_workspace_bytes(int32_t heads, int64_t T, int64_t R);

/* ssb_kda_prefill with a caller-owned workspace (16-byte aligned, >= ssb_kda_workspace_bytes; returns 3 when smaller),
 * so that the call allocates nothing; ssb_kda_prefill allocates and frees one on `stream`. Sequences whose rows sum
 * above T, or that reach outside [0, T), are rejected on the device (status 6 or 1; their state blocks untouched). */
int ssb_kda_prefill_ws(const ssb_kda_layer* layer, const void* x, int64_t ldx, const void* g, int64_t ldg,
                       const void* beta, int64_t ldb, int64_t T, const int32_t* seqs, int64_t R, void* out,
                       int64_t ldo, void* workspace, int64_t ws_bytes, int32_t* status, void* stream);

/* The short conv alone: q, k, v bf16 [T, H * 128] each (contiguous) and the conv state blocks updated; rows outside
 * every sequence are written as 0. Replaces `kda_conv.conv_qkv` (ssengine/model/kda_conv.py:146-164). */
int ssb_kda_conv(const ssb_kda_layer* layer, const void* x, int64_t ldx, int64_t T, const int32_t* seqs, int64_t R,
                 void* q, void* k, void* v, void* stream);

/* DSA lightning-indexer logits: logits fp32 [T, ldl], row t, column p = sum_h w[t, h] * relu(q[t, h, :] . k[p, :]) for
 * the pools p of row t's request (q bf16 [T, 32, 128]; w bf16 [T, ldw], the 32 head weights of each row read in place
 * from the indexer projection's output, 16-byte aligned, ldw % 8 == 0; pool keys bf16 in pages of
 * 32 pools: pool p of request r at row page_table[r * width + p / 32] * 32 + p % 32 of k_cache [pool_rows, 128]).
 * groups int32 [G][4] device = {request, first query row, rows (<= 8, one request), pool tiles of 128 to compute};
 * columns of a computed tile past a row's visible pools ((pos + 1) / 4) hold values of later pools: the top-k's key
 * range [0, (pos + 1) / 4) excludes them. status (device int32, may be NULL) receives 4 if a bounded wait expired.
 * Replaces the fork's DeepGEMM `fp8_mqa_logits` call of the kpool indexer (ssengine/kernels.py config 19;
 * split `split_indexer_prefill_chunks`, ssengine/model/pp_patch.py:587-634). */
int ssb_indexer_logits(const void* q, const void* w, int64_t ldw, int64_t T, const void* k_cache, int64_t pool_rows,
                       const int32_t* page_table, int64_t width, const int32_t* groups, int64_t G, float* logits,
                       int64_t ldl, int32_t* status, void* stream);

/* The FP8 form of ssb_indexer_logits (the reference's indexer cache: DeepSeek-V3.2's indexer as vLLM runs it). Queries
 * q8 e4m3 [T * 32, 128] with q_scale fp32 [T * 32] from ssb_indexer_q_quant; pool keys in the 132-byte entries of the
 * reference's cache, a 128-token page of 32 pools = 33 rows of 128 bytes (32 rows of e4m3 codes, then the 32 fp32
 * scales), k_pages holding `pages` pages (128-byte aligned), pool p of request r in page page_table[r * width + p / 32]
 * at row p % 32. logit = sum_h w_h * q_scale_h * relu(q8_h . k8) * k_scale; the softmax scale and the head-count
 * factor belong to w. Other arguments as ssb_indexer_logits. */
int ssb_indexer_logits_fp8(const uint8_t* q8, const float* q_scale, const void* w, int64_t ldw, int64_t T,
                           const uint8_t* k_pages, int64_t pages, const int32_t* page_table, int64_t width,
                           const int32_t* groups, int64_t G, float* logits, int64_t ldl, int32_t* status,
                           void* stream);
/* Indexer queries (bf16 rows of 128, `rows` = tokens x heads, 8-byte aligned) -> e4m3 codes q8 [rows, 128] and fp32
 * scales [rows]: scale = 2^ceil(log2(max(amax, 1e-10) / 448)), the ue8m0 form of vLLM's per-token-group FP8
 * quantization with groups of 128. */
int ssb_indexer_q_quant(const void* q, int64_t rows, uint8_t* q8, float* q_scale, void* stream);

/* Indexer key pools of one prefill microbatch: every pool of 4 tokens that a request's chunk completes, pool[p, c] =
 * sum_j softmax_j(gate[4p+j, c] + ape[j, c]) * k[4p+j, c] (fp32, stored bf16) at row page_table[r * width + p / 32] *
 * 32 + p % 32 of pool_cache [rows, 128]; tokens of the pool before the chunk's start come from the request's tail ring
 * (bf16 [blocks][2 (k, gate)][4][128]); afterwards the ring holds the chunk's trailing incomplete pool. k, gate bf16
 * [T, ld] (128 used), ape fp32 [4, 128]; reqs int32 [R][4] device = {first row, rows, start position, tail block};
 * max_rows >= every request's rows (sizes the grid). Replaces `kpool_compress_insert` + `kpool_seed_tail_cache`
 * (ssengine/model/pp_patch.py:415-534; the fork's `kpool_compress_and_write_cache`, configs 17-18). */
int ssb_kpool_insert(const void* k, const void* gate, int64_t ld, const float* ape, const int32_t* reqs, int64_t R,
                     int32_t max_rows, const int32_t* page_table, int64_t width, void* pool_cache, void* tail_ring,
                     void* stream);
/* The FP8 form of ssb_kpool_insert: each completed pool row stored as e4m3 codes of x / s with s = 2^ceil(log2(
 * max(1e-4, amax) / 448)) in the request's 132-byte-entry page (33 rows of 128 bytes: row p % 32 the codes, row 32 the
 * fp32 scales) of pool_pages (4-byte aligned); the tail ring stays bf16. */
int ssb_kpool_insert_fp8(const void* k, const void* gate, int64_t ld, const float* ape, const int32_t* reqs, int64_t R,
                         int32_t max_rows, const int32_t* page_table, int64_t width, uint8_t* pool_pages,
                         void* tail_ring, void* stream);

/* Selected pools -> token indices: out int32 [rows, ldo >= 4k + 3]: column c < 4k = pool_ids[row, c / 4] * 4 + c % 4
 * (-1 where the pool id is -1), then the tokens of the row's incomplete last pool (seq_len = positions[row] + 1:
 * 4 * (seq_len / 4) .. seq_len - 1, -1 past them). Replaces `kpool_fast.expand_into` (ssengine/model/kpool_fast.py:
 * 48-59, the fork's `expand_pools_and_append_tail`). */
int ssb_indexer_expand(const int32_t* pool_ids, int64_t ldp, int32_t k, const int64_t* positions, int64_t rows,
                       int32_t* out, int64_t ldo, void* stream);

/* Sparse MLA prefill of one DSA layer (absorbed latent attention) over the FP8 latent cache: out bf16 [T, 64, 512],
 * row t, head h = bmm2_scale * softmax over the row's selected tokens of bmm1_scale * q[t, h, :] . kv[s, :], times
 * kv[s, 0:512]; q e4m3 [T, 64, 576] (latent 512 + rope 64, 16-byte aligned); kv_cache e4m3 [slots, 576];
 * bmm1_scale = softmax scale * q_scale * k_scale, bmm2_scale = k_scale (the per-tensor scales of the FP8 query and
 * cache); indices int32 [T, ld_idx], the first n_idx (<= 2304) columns used (token positions of the row's request,
 * -1 = none: the indexer's expanded selection); the request of row t is found in qsl int32 [R + 1] (first row of each
 * request, ascending, qsl[0] = 0); slot of position p = page_table[r * width + p / 128] * 128 + p % 128 (a negative
 * page drops the token). The softmax weights enter the P.V product as e4m3 (like the reference's FP8 kernel). A row
 * with no selected token gets zeros. status (device int32, may be NULL) receives 4 if a bounded wait expired.
 * Replaces the TRTLLM sparse MLA with FP8 q and cache (ssengine/kernels.py config 25, bmm1 / bmm2 scales as vLLM's
 * FlashInfer sparse MLA backend passes them; split at 32,768 rows ssengine/model/pp_patch.py:643-672). */
int ssb_sparse_mla(const void* q, int64_t T, const void* kv_cache, const int32_t* indices, int64_t ld_idx,
                   int32_t n_idx, const int32_t* qsl, int32_t R, const int32_t* page_table, int64_t width,
                   float bmm1_scale, float bmm2_scale, void* out, int32_t* status, void* stream);

/* MLA cache append: row t of src bf16 [T, 576] (row pitch lds elements, % 8 == 0) into kv_cache row slots[t] (int64,
 * skipped when < 0) as e4m3(x / k_scale), round to nearest even, saturating to +-448 (576 bytes a row). Replaces the
 * fork's `concat_and_cache_mla` with kv_cache_dtype fp8_e4m3 (ssengine/kernels.py config 23). */
int ssb_mla_cache_append(const void* src, int64_t lds, const int64_t* slots, int64_t T, void* cache, float k_scale,
                         void* stream);

/* FP8 query of the sparse MLA: q8[t, h, 0:512] = e4m3(lat[h * rows_pad + t, :] / q_scale) (the absorbed latent
 * queries, head-major bf16 rows of 512) and q8[t, h, 512:576] = e4m3(rope[t * ldr + h * rope_stride + 0:64] / q_scale)
 * (each head's rope slice of the q_b rows); e4m3 [T, 64, 576]. Replaces the reference's transpose into the query
 * buffer and `scaled_fp8_quant` before the sparse MLA (ssengine/kernels.py `q_fp8_quant`). */
int ssb_mla_q_pack(const void* lat, int64_t rows_pad, const void* rope, int64_t ldr, int64_t rope_stride, int64_t T,
                   void* q8, float q_scale, void* stream);

/* Grouped NVFP4 GEMM (bf16 epilogue): for each tile {group g, first A row, rows, 0} of tiles int32 [num_tiles][4]
 * (device; *num_tiles on the device, <= tile_cap), out[row, :N] = alpha[g] * A[row] . B[g * N + n] with A NVFP4
 * [a_rows, K] (128x4 scale atoms) and B the groups' stacked NVFP4 rows [groups * N, K]; N % 256 == 0, K % 64 == 0.
 * The per-head MLA GEMMs of a DSA layer: q absorb 64 x (k 192, n 512) and v_up 64 x (k 512, n 256) (the reference's
 * torch.bmm, ssengine/kernels.py configs 22 and 26). */
int ssb_nvfp4_gemm_grouped(int32_t epilogue, const uint8_t* a_codes, const uint8_t* a_sf, int64_t a_rows, int64_t K,
                           const uint8_t* b_codes, const uint8_t* b_sf, int64_t N, int32_t groups, const float* alpha,
                           const int32_t* tiles, const int32_t* num_tiles, int32_t tile_cap, void* out, int64_t ldo,
                           int32_t* status, void* stream);

/* y[r, :width] = x[r, :width] * rsqrt(mean(x^2) + eps) * w (bf16, row pitches ldx / ldy): the q and kv latent norms of
 * a DSA layer on column slices of the fused down-projection (the fork's fused_q_kv_rmsnorm, config 13). */
int ssb_rmsnorm_cols(const void* x, int64_t ldx, int32_t width, int64_t rows, const void* w, float eps, void* y,
                     int64_t ldy, void* stream);

/* In place: rotary embedding of the 64-dim slice at x + r * ldx + h * head_stride for each row r and head h < heads
 * (interleaved pairs (2i, 2i + 1), angle positions[r] * theta^(-i / 32), as DeepSeek-V3.2-style MLA applies it --
 * vLLM's GlmMoeDsa / DeepseekV2 attention, is_neox_style=False): the rope parts of the MLA query and key. x + r * ldx
 * + h * head_stride must be 4-byte aligned. */
int ssb_rope(void* x, int64_t ldx, int32_t heads, int64_t head_stride, const int64_t* positions, int64_t rows,
             float theta, void* stream);

/* Head-major <-> row-major copies around the per-head GEMMs: to_heads: dst [heads, rows_pad, dim] (pad rows zero) =
 * src[r, h * head_stride + :dim] (row pitch row_ld); else dst[r, h * head_stride + :dim] = src [heads, rows_pad, dim].
 * dim, row_ld, head_stride % 8 == 0. */
int ssb_transpose_heads(const void* src, void* dst, int64_t rows, int64_t rows_pad, int32_t heads, int32_t dim,
                        int64_t row_ld, int64_t head_stride, int32_t to_heads, void* stream);

/* Tile table of ssb_nvfp4_gemm_grouped for per-head GEMMs over head-major rows padded to rows_pad (% 128 == 0):
 * tiles int32 [heads * rows_pad / 128][4] = {head, head * rows_pad + 128 * m, 128, 0} and *num_tiles, written on the
 * device (tile_cap entries available; tiles 16-byte aligned), so a microbatch's table costs no host work or copy.
 * Replaces the batch strides the reference's torch.bmm takes (ssengine/kernels.py configs 22 and 26). */
int ssb_head_tiles(int32_t heads, int64_t rows_pad, int32_t* tiles, int64_t tile_cap, int32_t* num_tiles,
                   void* stream);

/* out[r] = [a[r, :wa], b[r, :wb]] (bf16; widths and pitches % 8 == 0): the latent-cache rows (latent | rope key). */
int ssb_concat_cols(const void* a, int64_t lda, int32_t wa, const void* b, int64_t ldb, int32_t wb, void* out,
                    int64_t ldo, int64_t rows, void* stream);

/* One NVFP4 MoE layer's device parameters (all pointers device memory, owned by the caller).
 * Experts 0..E-1 are routed, expert E is the shared expert (every token, weight 1). */
typedef struct ssb_moe_layer {
  int32_t hidden;              /* H, % 256 == 0 */
  int32_t inter;               /* F (expert intermediate), % 128 == 0 */
  int32_t num_experts;         /* E routed experts, <= 512 */
  int32_t top_k;               /* k, < 32 */
  float gs_x;                  /* global scale of the layer input's NVFP4 quantization */
  float gs_h;                  /* global scale of the SwiGLU output's NVFP4 quantization */
  const uint8_t* router_codes; /* [router_rows, H/2], rows >= E zero */
  const uint8_t* router_sf;    /* atoms of [router_rows, H] */
  int64_t router_rows;         /* E padded to a multiple of 128 */
  float router_alpha;          /* 1 / (gs_x * gs_router) */
  const uint8_t* w1_codes;     /* [(E+1) * 2F, H/2]; per expert 256-row tiles of 128 gate + 128 up rows */
  const uint8_t* w1_sf;        /* atoms of [(E+1) * 2F, H] */
  const float* w1_alpha;       /* [E+1]: 1 / (gs_x * gs_w1[e]) */
  const uint8_t* w2_codes;     /* [(E+1) * H, F/2] */
  const uint8_t* w2_sf;        /* atoms of [(E+1) * H, F] */
  const float* w2_alpha;       /* [E+1]: 1 / (gs_h * gs_w2[e]) */
  int32_t add_input;           /* nonzero: out = x + MoE(x) (the residual add fused into the combine) */
  int32_t routing;             /* SSB_ROUTE_SOFTMAX or SSB_ROUTE_SIGMOID_BIAS */
  int32_t n_group;             /* sigmoid routing: expert groups (1 = no grouping) */
  int32_t topk_group;          /* sigmoid routing: groups kept */
  float routed_scale;          /* sigmoid routing: routed scaling factor applied to the normalized weights */
  const float* route_bias;     /* sigmoid routing: [E] fp32 correction bias */
} ssb_moe_layer;

/* Routing rules of ssb_moe_layer.routing. */
#define SSB_ROUTE_SOFTMAX 0       /* BASELINE configs: softmax over the k largest logits */
#define SSB_ROUTE_SIGMOID_BIAS 1  /* the reference model's rule (DeepSeek-V3 style), see ssb_moe_route_sigmoid */

/* Workspace of ssb_moe_forward for T tokens, in bytes (one caller-owned device buffer, 256-byte aligned). */
int64_t ssb_moe_workspace_bytes(const ssb_moe_layer* layer, int64_t T);

/* Byte offsets of the workspace's buffers (SSB_WS_* below) for T tokens; n = entries to fill. Lets a caller read the
 * intermediate routing / permutation / activation buffers of the last forward. */
#define SSB_WS_XQ 0          /* uint8 [Tpad, H/2] input codes (token order) */
#define SSB_WS_XSF 1         /* input scale atoms */
#define SSB_WS_LOGITS 2      /* fp32 [T, E] router logits */
#define SSB_WS_IDS 3         /* int32 [T, k] routed experts */
#define SSB_WS_WEIGHTS 4     /* fp32 [T, k] routing weights */
#define SSB_WS_ROWS 5        /* int32 [T, k] permuted row of each (token, slot) */
#define SSB_WS_COUNTS 6      /* int32 [E+1] tokens per expert (shared last) */
#define SSB_WS_OFFSETS 7     /* int32 [E+2] first permuted row per expert (128-aligned), total rows last */
#define SSB_WS_MASKS 8
#define SSB_WS_BLOCKS 9
#define SSB_WS_MTILES 10     /* int32 [cap, 4] GEMM row tiles {expert, first row, rows, 0}, then int32 [pair cap, 4]
                                CTA-pair tiles {expert, first row, rows of the first 128, rows of the next 128} */
#define SSB_WS_NUM_MTILES 11 /* int32 [2]: row tiles, CTA-pair tiles */
#define SSB_WS_XQ_PERM 12    /* uint8 [cap*128, H/2] permuted input codes */
#define SSB_WS_XSF_PERM 13
#define SSB_WS_ACT 14        /* uint8 [cap*128, F/2] SwiGLU output codes */
#define SSB_WS_ACT_SF 15
#define SSB_WS_Y 16          /* bf16 [cap*128, H] expert outputs per permuted row */
#define SSB_WS_ROW_SRC 17    /* int32 [cap*128] source token of each permuted row (padding rows unwritten) */
#define SSB_WS_END 18
int ssb_moe_workspace_offsets(const ssb_moe_layer* layer, int64_t T, int64_t* offsets, int32_t n);

/* Sigmoid + correction-bias grouped routing (the reference model's rule: "DeepSeek-V3 routing, scale 5/2",
 * ssengine/kernels.py:182-187, checked by its CPU test as (logits.sigmoid() + bias).topk(8),
 * tests/test_moe_tuning_cpu.py:63 of the reference): score = sigmoid(logit) (double, rounded to fp32 once),
 * choice = score + bias[e]; with n_group > 1 only the topk_group groups with the largest sums of their two best
 * choices stay eligible (ties: lower group); ids = the k largest eligible choices (ties: lower expert), in rank order;
 * weights = score[id] / sum of the k scores (rank order) * scale. logits fp32 [T, E], bias fp32 [E]; E <= 512,
 * k <= 32, n_group <= 32 dividing E. Replaces the routing inside FlashInfer `trtllm_fp4_block_scale_moe`
 * (routing_method DeepSeekV3, ssengine/kernels.py config 30). */
int ssb_moe_route_sigmoid(const float* logits, int64_t T, int32_t E, int32_t k, const float* bias, int32_t n_group,
                          int32_t topk_group, float scale, int32_t* ids, float* weights, void* stream);

/* Whole MoE layer on `stream`: quantize x -> router GEMM -> top-k routing -> permutation + gather -> grouped NVFP4
 * gate_up GEMM with SwiGLU + NVFP4 requant epilogue -> grouped down GEMM -> weighted combine (+ shared expert).
 * x bf16 [T, H] (contiguous), out bf16 [T, H]. Replaces the MoE block of a reference MoE layer
 * (ssengine/kernels.py:174-193: configs 28-32, the router GEMM, the input quant, FlashInfer
 * `trtllm_fp4_block_scale_moe` and the shared expert's two GEMMs). */
int ssb_moe_forward(const ssb_moe_layer* layer, const void* x, int64_t T, void* out, void* ws, int64_t ws_bytes,
                    int32_t* status, void* stream);

/* ssb_moe_forward with a cudaEvent_t recorded on `stream` before each of its SSB_MOE_STEPS launch steps and one after
 * the last (events: SSB_MOE_STEPS + 1 created events; steps: input quant, router GEMM, route, count, offsets,
 * scatter, gate_up GEMM, down GEMM, combine). For per-kernel device timing; the same work as ssb_moe_forward.
 * No counterpart in the reference (its per-kernel timing comes from nsys traces, benchmarks/nsys_trace.py:121-160). */
#define SSB_MOE_STEPS 9
int ssb_moe_forward_profiled(const ssb_moe_layer* layer, const void* x, int64_t T, void* out, void* ws,
                             int64_t ws_bytes, int32_t* status, void* stream, void* const* events);

/* ---- stage edge over NVLink (replaces the reference's CePipe, ssengine/runtime/transport.py:205-335) ----------------
 * The receiver's ring and flag words are mapped into the sender's process by CUDA IPC; the sender's kernels store rows
 * straight into the peer slot, then a release write of ready[slot] = n; the receiver's stream waits on it with a
 * bounded kernel. Flags count microbatches from 1 (slot = (n - 1) % K). */

/* handle64 (64 bytes) = cudaIpcGetMemHandle of the allocation holding dev_ptr, *offset = dev_ptr - its base (a pointer
 * from a caching allocator may sit inside a larger block) (CePipe._export, transport.py:281-283). */
int ssb_ipc_export(const void* dev_ptr, uint8_t* handle64, int64_t* offset);
/* Map a peer's exported allocation (lazy peer access) into this process; *dev_ptr = its base (add the exporter's
 * offset) (CePipe._open, transport.py:285-290). */
int ssb_ipc_open(const uint8_t* handle64, void** dev_ptr);
int ssb_ipc_close(void* dev_ptr);
/* On `stream`: wait until (int32)(*flag - value) >= 0 (flag: local or peer device memory, read with acquire at system
 * scope). Replaces cuStreamWaitValue32 GEQ (CePipe._wait, transport.py:292-294), with a limit: after timeout_ns the
 * kernel writes 4 to status (device int32, may be NULL) and returns, so the stream and the context stay usable. */
int ssb_flag_wait(const uint32_t* flag, uint32_t value, int64_t timeout_ns, int32_t* status, void* stream);
/* On `stream`: *flag = value after everything the stream did before is visible system-wide (release store).
 * Replaces cuStreamWriteValue32 (CePipe._write, transport.py:296-298). */
int ssb_flag_write(uint32_t* flag, uint32_t value, void* stream);
/* On `stream`: copy bytes (% 16 == 0, both pointers 16-byte aligned) by SM stores; dst may be a peer mapping. Replaces
 * the copy-engine cudaMemcpyAsync of CePipe.send (transport.py:326-327) where the producing kernel cannot write the
 * peer slot itself. */
int ssb_p2p_copy(void* dst, const void* src, int64_t bytes, void* stream);

/* ---- DRAM tier copies (the reference's tier mover, ssengine/kvpool/mover.py) -------------------------------------
 * On `stream`: for r < n, copy runs[3r + 2] bytes from address runs[3r] to address runs[3r + 1] (runs: int64 [n, 3] in
 * device memory; every address and size a multiple of 16 bytes). Either side may be pinned host memory (addressed
 * through unified virtual addressing) or this device's memory: a context's KV pages and state rows between a stage's
 * cache views and its DRAM tier, one launch per tier op. Misaligned runs are skipped and raise 1 in `status`. */
int ssb_copy_runs(const int64_t* runs, int64_t n, int32_t* status, void* stream);

/* MoE routing + permutation that allocates nothing: the same routing as ssb_moe_route and the same permutation as
 * ssb_moe_forward (expert-major, tokens ascending, shared expert last, experts at 128-aligned offsets), for callers
 * that cannot allocate device memory -- a stage whose KV pool already took the free HBM at start-up, code that must
 * not stall the GPU with a cudaMalloc mid-microbatch, a host holding only buffers mapped from another process.
 * Inputs: logits fp32 [T, E]. Outputs: ids int32 [T, k], weights fp32 [T, k], rows int32 [T, k] (permuted row of each
 * (token, slot)), counts int32 [E+1], offsets int32 [E+2]. Its scratch is one static device array of about 1.25 MiB
 * that every GPU loading the library holds until exit; limits T <= 16384, E <= 512, k <= 31, beyond which it returns
 * 7 before any launch. Calls share that array: calls whose work overlaps on the GPU race. The first call on a device
 * looks up the array's address and should come before any stream capture. `status` may be null. With T == 0 it
 * writes zero counts and offsets and nothing else.
 * No counterpart in the reference. */
int ssb_moe_route_permute_noalloc(const float* logits, int64_t T, int32_t E, int32_t k, int32_t* ids, float* weights,
                                  int32_t* rows, int32_t* counts, int32_t* offsets, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSENGINE_B200_H_ */
