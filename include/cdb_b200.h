/*
 * C ABI of the B200 continuous-depth-batching (CDB) decode library, libcdb_b200.so.
 *
 * Every entry point takes raw device pointers, sizes and strides plus a cudaStream_t passed
 * as void*, returns an int status (CDB_OK or a CDB_ERR_* code below), allocates no device
 * memory, and only enqueues work on the given stream (safe inside CUDA-graph capture).
 * Tensors are row-major; "bf16" is IEEE bfloat16; element strides are in elements.
 *
 * Device-side failures (a bounded wait that ran out, an out-of-range index caught by a
 * kernel's own check) are written to the caller's `status` word in device memory (first
 * error wins) instead of trapping; the host reads it between launches.
 *
 * Reference interfaces these replace are cited per entry point as path:line inside the
 * reference project (ZH-Haoran/continuous-depth-batching, package looped_cdb), or inside
 * HF transformers 5.x where the reference calls into it.
 */
#ifndef CDB_B200_H_
#define CDB_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CDB_OK 0
#define CDB_ERR_INVALID_ARGUMENT 1
#define CDB_ERR_UNSUPPORTED 2
#define CDB_ERR_CUDA 3
#define CDB_ERR_DEVICE_TIMEOUT 4
#define CDB_ERR_TMA_ENCODE 5
#define CDB_ERR_INDEX 6
#define CDB_ERR_SCRATCH_LIMIT 7 /* call exceeds the fixed static scratch of a *_static entry point */

/* Attention work plan header: 4 ints + the first unit of each chunk (+ one end entry). */
#define CDB_ATTN_PLAN_MAX_CHUNKS 1024
#define CDB_ATTN_PLAN_HEADER_INTS (4 + CDB_ATTN_PLAN_MAX_CHUNKS + 1)

/* Library version (major*10000 + minor*100 + patch). */
int cdb_version(void);

/* Human-readable text for a status code (static storage). */
const char* cdb_status_string(int status);

/* ---------------------------------------------------------------------------------------
 * Paged KV pool. One bf16 allocation laid out
 *   kv[num_cache_layers][2 (K,V)][rows][num_kv_heads][head_dim],  rows = (num_blocks+2)*block_size
 * i.e. for each cache layer exactly the reference's per-layer key/value tensors
 * [(num_blocks+2)*block_size, Hkv, D] (continuous_batching/cache.py:131-145), stacked. A token
 * of request r at position p lives in row block_table[r][p / block_size]*block_size + p % block_size
 * of every cache layer; cache layer = kv_slot*num_layers + physical layer
 * (kv_cache_policy.py:106-128).
 * ------------------------------------------------------------------------------------- */

/* Balanced split-KV work plan for one recurrent launch; run once, reused by every layer.
 * The pages of every (row, head group) segment, rows in order and head groups inner, are cut
 * into about 2*num_sms equal chunks (one per attention CTA); a segment crossing chunk boundaries
 * becomes split-KV pieces that the attention kernel merges (the last warp of a (row, head)).
 *   item_pos    [num_items] int32: position of each row's query token; -1 = padding row.
 *               Row p attends over cached rows [0, p].
 *   append      accepted for compatibility, no effect (the append runs before the attention).
 *   plan_header [CDB_ATTN_PLAN_HEADER_INTS] int32 out: {num_units, num_chunks, max_splits,
 *               whole_segments, first unit of chunk 0 .. num_chunks}.
 *   units       [unit_capacity] int4 out: {row, head_group << 16 | split, first_page << 16 |
 *               end_page, num_splits}; unit_capacity >= rows * heads/heads_per_CTA + 2*num_sms.
 *   scratch_items: rows the split-combine scratch covers; larger launches never split (whole
 *               segments dealt round-robin).
 * Replaces the split decision inside FlashAttention-3's flash_attn_with_kvcache
 * (transformers integrations/flash_paged.py:107-118). */
int cdb_attn_plan(const int32_t* item_pos, int num_items, int append, int num_heads, int head_dim,
                  int block_size, int unit_capacity, int scratch_items, int num_sms, int32_t* plan_header,
                  void* units, void* stream);

/* Ragged-depth paged decode attention with fused RoPE and KV append (one cache layer).
 * Replaces paged_attention_forward's decode branch -> flash_attn_with_kvcache
 * (transformers integrations/flash_paged.py:84-122), reached from OuroAttention.forward
 * (models/ouro/modeling_ouro.py:377-432) and HuginnAttention.forward
 * (models/huginn/modeling_huginn.py:244-302).
 *   qkv        bf16 [num_items, qkv_stride]: q at column 0, k at k_col, v at v_col (H*D each);
 *              16-byte aligned, strides and column offsets multiples of 8 elements.
 *   rope_mode  0: q/k already rotated; 1: split-half rotate_half RoPE (Ouro, bf16 tables
 *              [max_positions, head_dim]); 2: interleaved-pair RoPE in fp32 (Huginn, fp32
 *              tables [max_positions, head_dim/2], apply_rotary_emb_complex_like
 *              modeling_huginn.py:175-197).
 *   qk_bias    NULL, or bf16 [2, num_heads, head_dim] (q bias, then k bias) added to q and k in
 *              bf16 before the rotation (Huginn's learned qk_bias, modeling_huginn.py:261-264).
 *   append     1: rotate q in place in `qkv`, rotate k, write k/v at the row's position (a
 *              separate kernel), then attend over [0,p]; 2: the same result in one kernel (q
 *              rotated in registers and `qkv` left unchanged; k/v written to the cache and used
 *              for position p directly; tables and qk_bias 16-byte aligned); 0: attend over
 *              cached rows [0,p] with q already rotated.
 *   out        bf16 [num_items, out_stride], heads concatenated.
 *   part_o/part_ml/counters: split-combine scratch sized for scratch_items rows
 *              (cdb_attn_scratch_bytes); counters must start zeroed, kernels leave them zeroed.
 */
int cdb_paged_decode_attn_append(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                 void* out, int64_t out_stride, void* kv_base, int num_cache_layers,
                                 int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                 int64_t block_table_stride, const int32_t* item_slot, const int32_t* item_pos,
                                 int rope_mode, const void* rope_cos, const void* rope_sin, const void* qk_bias,
                                 int append, const int32_t* plan_header, const void* units, float* part_o,
                                 float* part_ml,
                                 int32_t* counters, int scratch_items, int num_items, int num_heads, int head_dim,
                                 int block_size, float scale, int num_ctas, int32_t* status, void* stream);

/* Same attention as cdb_paged_decode_attn_append (plan included), but needing no scratch from
 * the caller: no plan buffers, no split-combine buffers. No counterpart in the reference; it
 * exists for callers that cannot allocate device memory, such as an attention hook that runs
 * while the host framework captures a CUDA graph (allocation is not permitted during capture)
 * or a plugin that is handed tensors but no allocator.
 *   Arguments mean what they mean for cdb_paged_decode_attn_append.
 *   Scratch: one file-scope device array of 4,788,992 bytes (about 4.8 MB) per GPU, held until
 *   the process exits.
 *   Its device address is looked up with cudaGetSymbolAddress on the first call made with that
 *   device current, so make one call per device (num_items = 0 is enough) before any stream
 *   capture. Each call clears the split counters (cudaMemsetAsync on `stream`) before using them.
 *   Limits: head_dim <= 128, num_heads <= 128, num_items * (num_heads / heads_per_CTA) <= 32768
 *   (heads_per_CTA 4 for head_dim 64/128, 5 for 96); beyond them it returns
 *   CDB_ERR_SCRATCH_LIMIT and enqueues nothing. KV splitting is used only while
 *   num_items * num_heads <= 128; larger launches run one unit per (row, head group).
 *   Every call on a device shares the one array: calls whose work can overlap (different
 *   streams, or different host threads, without ordering between them) race on it and give
 *   wrong results. Calls must be ordered, e.g. all on one stream. */
int cdb_paged_decode_attn_append_static(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                        void* out, int64_t out_stride, void* kv_base, int num_cache_layers,
                                        int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                        int64_t block_table_stride, const int32_t* item_slot,
                                        const int32_t* item_pos, int rope_mode, const void* rope_cos,
                                        const void* rope_sin, const void* qk_bias, int append, int num_items,
                                        int num_heads,
                                        int head_dim, int block_size, float scale, int num_ctas, int32_t* status,
                                        void* stream);

/* Bytes of split-combine scratch (part_o + part_ml + counters) for `scratch_items` rows. */
int64_t cdb_attn_scratch_bytes(int scratch_items, int num_heads, int head_dim);

/* Causal paged prefill attention over prompt-chunk tiles (the varlen branch of
 * paged_attention_forward, transformers integrations/flash_paged.py:50-81, after
 * PagedAttentionCache.update, continuous_batching/cache.py:284-318).
 *   tiles  int4 [num_tiles] {row_start, num_rows <= 64, resident slot, position of row_start}:
 *          consecutive rows of one request; each row attends to keys [0, its position] of that
 *          request through the block table. q must already be rotated and the chunk's k/v
 *          written (cdb_rope_append_kv). head_dim 64, 96 or 128. */
int cdb_prefill_attention(const void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* out,
                          int64_t out_stride, const void* kv_base, int num_cache_layers, int64_t kv_rows,
                          int cache_layer, const int32_t* block_table, int64_t block_table_stride, const void* tiles,
                          int num_tiles, int num_heads, int head_dim, int block_size, float scale, int32_t* status,
                          void* stream);

/* Rotate q in place and rotate+write k and v of every row into its cache row (prefill path).
 * Replaces apply_rotary_pos_emb (modeling_ouro.py:186-204) + PagedAttentionCache.update's
 * index_copy_ writes (continuous_batching/cache.py:284-318). */
int cdb_rope_append_kv(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* kv_base,
                       int num_cache_layers, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                       int64_t block_table_stride, const int32_t* item_slot, const int32_t* item_pos, int rope_mode,
                       const void* rope_cos, const void* rope_sin, const void* qk_bias, int num_items, int num_heads,
                       int head_dim, int block_size, void* stream);

/* bf16 tensor-core GEMM on tcgen05/TMEM: c[M,N] = x[M,K] * w[N,K]^T (fp32 accumulation, bf16
 * store). Replaces the nn.Linear projections of the shared block and the LM head
 * (OuroAttention q/k/v/o_proj modeling_ouro.py:371-374,431; OuroMLP gate/up/down :162-168;
 * Huginn Wqkv/proj/fc/mlp.proj modeling_huginn.py:239-242,310-316; lm_head adapters/ouro.py:321-329),
 * which the reference runs on cuBLAS through ATen.
 *   x, w       row-major bf16, leading dimensions ldx, ldw (multiples of 8), 16-byte aligned.
 *   max_ctas   persistent CTAs (<= 0: num_sms). The (tile, k block) iterations are divided
 *              evenly over them (stream-K); a tile split across CTAs is combined through
 *              `workspace` by the piece that finishes last, summing the pieces in k order
 *              (deterministic for a given M, N, K and CTA count).
 *   workspace  fp32, >= cdb_gemm_workspace_elems(M, N, K, num_sms) elements, 16-byte aligned.
 *   counters   int32, >= cdb_gemm_counter_elems(M, N, K) elements, zeroed before first use;
 *              every call leaves them zeroed. Calls sharing workspace/counters must be ordered
 *              (one stream). */
int cdb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M, int N, int K,
                  int max_ctas, float* workspace, int64_t workspace_elems, int32_t* counters, int num_counters,
                  int num_sms, int32_t* status, void* stream);

/* Fused MLP input half: act[M, inter] = silu(x * Wg^T) * (x * Wu^T) with the reference's bf16
 * rounding (gate and up rounded to bf16, silu rounded to bf16, product rounded to bf16), in one
 * tcgen05 GEMM whose epilogue applies SwiGLU. Replaces OuroMLP.forward's
 * act_fn(gate_proj(x)) * up_proj(x) (modeling_ouro.py:162-168) and Huginn's gated MLP
 * (modeling_huginn.py:310-316).
 *   w_gate_up  bf16 [2*inter, K] with rows interleaved: row 2j = gate_proj row j,
 *              row 2j+1 = up_proj row j. act 2-byte aligned, ld_act >= inter.
 *   max_ctas, workspace, counters, num_sms, status: as cdb_gemm_bf16 with N = 2*inter. */
int cdb_mlp_gateup_silu_gemm(const void* x, int64_t ldx, const void* w_gate_up, int64_t ldw, void* act,
                             int64_t ld_act, int M, int inter, int K, int max_ctas, float* workspace,
                             int64_t workspace_elems, int32_t* counters, int num_counters, int num_sms,
                             int32_t* status, void* stream);

/* LM head + greedy argmax in one tcgen05 GEMM, without storing logits (the coda's lm_head,
 * adapters/ouro.py:321-329, then argmax, _run_coda_forward_graphed model_runner.py:1064-1125):
 * id[r] = argmax_v bf16(x[r] . w[v]) over v < vocab, first index on ties (as torch.argmax).
 *   out_ids[out_rows ? out_rows[r] : r] = id[r] (skipped when out_rows[r] < 0); if token_rows is
 *   not NULL and token_rows[r] >= 0, also token_table[token_rows[r]] = id[r].
 *   keys [M] uint64 and done [1] int32: scratch that must start zeroed; the call leaves it zeroed.
 *   workspace/counters as cdb_gemm_bf16 with N = vocab. Calls sharing keys/done/workspace/
 *   counters must be ordered (one stream). x/w as cdb_gemm_bf16. */
int cdb_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int vocab, int K,
                       int64_t* out_ids, const int32_t* out_rows, const int32_t* token_rows, int32_t* token_table,
                       uint64_t* keys, int32_t* done, float* workspace, int64_t workspace_elems, int32_t* counters,
                       int num_counters, int num_sms, int32_t* status, void* stream);

/* fp32 workspace elements a GEMM of this shape needs (split partials: 2 per CTA, 128 x token-tile
 * floats each). */
int64_t cdb_gemm_workspace_elems(int M, int N, int K, int num_sms);

/* int32 tile counters a GEMM of this shape needs (one per 128-row x token-tile output tile). */
int cdb_gemm_counter_elems(int M, int N, int K);

/* Split-K GEMM left unreduced, for a consumer that sums the planes while it reads them
 * (cdb_add_rmsnorm_parts): parts[z * part_stride + m * N + n] = the fp32 sum over split z's k
 * blocks of x[m, k] * w[n, k], for z < splits. Split z covers k blocks [z * ceil(kb / splits),
 * ...) of the kb = ceil(K / 64) blocks, and a consumer summing the planes in z order gets exactly
 * the value the reduced split mode of cdb_gemm_bf16 would store for the same split count.
 * Serves decode-width projections (few 128-row tiles) without any cross-CTA reduction.
 * splits in [1, 16], no empty split (use cdb_gemm_partial_splits); part_stride >= M * N;
 * parts 4-byte aligned. Replaces the nn.Linear o_proj / down_proj (modeling_ouro.py) as the
 * producer half of a projection + residual-norm pair. */
int cdb_gemm_bf16_partials(const void* x, int64_t ldx, const void* w, int64_t ldw, float* parts, int64_t part_stride,
                           int M, int N, int K, int splits, int32_t* status, void* stream);

/* The split count cdb_gemm_bf16_partials should use for this shape on num_sms SMs (toward two
 * CTAs per SM for token tiles up to 128, at least two k blocks per split, at most 6: more planes
 * cost more in plane traffic than they gain in streaming CTAs). */
int cdb_gemm_partial_splits(int M, int N, int K, int num_sms);

/* ---------------------------------------------------------------------------------------
 * Row-wise fused elementwise kernels (bf16 activations, fp32 math, bf16 rounding at the
 * points PyTorch rounds). Optional index arrays (nullable) gather input rows / scatter output
 * rows; an index < 0 marks a padding row that is skipped.
 * ------------------------------------------------------------------------------------- */

/* y[r] = weight * bf16(x*rsqrt(mean(x^2)+eps)), x read from x[x_rows[r]] (OuroRMSNorm.forward,
 * modeling_ouro.py:445-450). If x_copy != NULL the gathered x row is also stored there. */
int cdb_rmsnorm(const void* x, int64_t x_stride, const int32_t* x_rows, const void* weight, void* y,
                int64_t y_stride, void* x_copy, int64_t x_copy_stride, int num_rows, int hidden, float eps,
                void* stream);

/* Sandwich-norm residual step of OuroDecoderLayer.forward (modeling_ouro.py:481-502):
 *   x[r] = x[r] + rmsnorm(a[r]; w_a)     (bf16 add)
 *   y[r] = rmsnorm(x[r]; w_next)         (next norm: the MLP input norm, the next layer's
 *                                         input norm, or the final model norm)
 * If gate_w != NULL also gate_out[r] = bf16(dot(y[r], gate_w) + gate_b[0]) (exit gate
 * Linear(H,1), adapters/ouro.py:262-291). If y_rows != NULL, y row r is written to
 * y[y_rows[r]] (the hidden-state bank scatter, model_runner.py:690-693). */
int cdb_add_rmsnorm(void* x, int64_t x_stride, const void* a, int64_t a_stride, const void* w_a,
                    const void* w_next, void* y, int64_t y_stride, const int32_t* y_rows, const void* gate_w,
                    const void* gate_b, void* gate_out, int num_rows, int hidden, float eps, void* stream);

/* cdb_add_rmsnorm with a[r] = bf16(sum over z < num_parts, in z order, of a_parts[z * part_stride +
 * r * hidden + d]): the unreduced planes of cdb_gemm_bf16_partials (N = hidden), so the pair
 * GEMM -> norm equals cdb_gemm_bf16 -> cdb_add_rmsnorm at the same split count. a_parts 16-byte
 * aligned, part_stride a multiple of 4 and >= num_rows * hidden. */
int cdb_add_rmsnorm_parts(void* x, int64_t x_stride, const float* a_parts, int num_parts, int64_t part_stride,
                          const void* w_a, const void* w_next, void* y, int64_t y_stride, const int32_t* y_rows,
                          const void* gate_w, const void* gate_b, void* gate_out, int num_rows, int hidden,
                          float eps, void* stream);

/* QKV projection with RoPE and the KV append: qkv[M, v_col + H*D] = x * w_qkv^T (cdb_gemm_bf16),
 * then q rotated in place, k rotated, and k/v written at each row's position (cdb_rope_append_kv;
 * same arguments). Replaces OuroAttention.forward's q/k/v_proj + apply_rotary_pos_emb + the
 * cache write of paged_attention_forward (modeling_ouro.py:377-410, flash_paged.py:84-106); the
 * cache-only attention (append 0) then reads the new row. Two launches chained with programmatic
 * dependent launch. */
int cdb_qkv_rope_append_gemm(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw, void* qkv,
                             int64_t qkv_stride, int64_t k_col, int64_t v_col, int num_items, int K, void* kv_base,
                             int num_cache_layers, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                             int64_t block_table_stride, const int32_t* item_slot, const int32_t* item_pos,
                             int rope_mode, const void* rope_cos, const void* rope_sin, const void* qk_bias,
                             int num_heads, int head_dim, int block_size, float* workspace, int64_t workspace_elems,
                             int32_t* counters, int num_counters, int num_sms, int32_t* status, void* stream);

/* O projection with Ouro's post-attention sandwich: proj = attn * w_o^T; x <- bf16(x +
 * norm_post(proj)); y = norm_next(x) (OuroDecoderLayer.forward, modeling_ouro.py:470-490:
 * input_layernorm_2 on the attention output, the residual add, post_attention_layernorm). The
 * tcgen05 GEMM, then cdb_add_rmsnorm, chained with programmatic dependent launch. */
int cdb_o_proj_residual_norm_gemm(const void* attn, int64_t ld_attn, const void* w_o, int64_t ldw, void* proj,
                                  int64_t ld_proj, void* x, int64_t x_stride, const void* w_norm_post,
                                  const void* w_norm_next, void* y, int64_t y_stride, int num_rows, int hidden,
                                  int K, float eps, float* workspace, int64_t workspace_elems, int32_t* counters,
                                  int num_counters, int num_sms, int32_t* status, void* stream);

/* Down projection with the MLP sandwich: proj = act * w_down^T; x <- bf16(x + norm_post(proj));
 * y[y_rows[r]] = norm_next(x[r]) (y_rows NULL: y[r]; rows with y_rows[r] < 0 skipped) and, with
 * gate_w, gate_out[r] = bf16(gate_w . y + gate_b) - the layer end of OuroDecoderLayer.forward
 * (modeling_ouro.py:492-503) and, after the last layer, the final norm, bank scatter and exit-gate
 * logit of OuroCDBAdapter.recurrent_step (adapters/ouro.py:240-262). */
int cdb_down_residual_norm_gemm(const void* act, int64_t ld_act, const void* w_down, int64_t ldw, void* proj,
                                int64_t ld_proj, void* x, int64_t x_stride, const void* w_norm_post,
                                const void* w_norm_next, void* y, int64_t y_stride, const int32_t* y_rows,
                                const void* gate_w, const void* gate_b, void* gate_out, int num_rows, int hidden,
                                int K, float eps, float* workspace, int64_t workspace_elems, int32_t* counters,
                                int num_counters, int num_sms, int32_t* status, void* stream);

/* act[r] = bf16(bf16(silu(g)) * u) with gu[r] = [g (inter) | u (inter)] (OuroMLP.forward,
 * modeling_ouro.py:166-169). */
int cdb_silu_mul(const void* gu, int64_t gu_stride, void* act, int64_t act_stride, int num_rows, int inter,
                 void* stream);

/* Greedy sampling: id_r = argmax_j logits[r][j] (first index among equal maxima, as
 * torch.argmax; model_runner.py:1062,1105), stored to out[out_rows[r]] (out[r] when out_rows is
 * NULL; skipped when out_rows[r] < 0). If token_rows != NULL and token_rows[r] >= 0 the id is
 * also stored to token_table[token_rows[r]] (device-resident next-token buffer). */
int cdb_argmax(const void* logits, int64_t stride, int num_rows, int vocab, int64_t* out, const int32_t* out_rows,
               const int32_t* token_rows, int32_t* token_table, void* stream);

/* Prelude embedding lookup (OuroCDBAdapter.prelude, adapters/ouro.py:199-212; Huginn's
 * wte(ids) * embed_scale, modeling_huginn.py:431):
 * out[out_rows[r]] = bf16(table[id_r] * scale); id_r = ids[r] if ids[r] >= 0 else
 * token_table[id_src[r]] (the on-device successor-token gather of model_runner.py:439-457).
 * scale = 1 copies the row exactly (Ouro). */
int cdb_embed(const void* table, int hidden, int vocab, const int32_t* ids, const int32_t* id_src,
              const int32_t* token_table, void* out, int64_t out_stride, const int32_t* out_rows, int num_rows,
              float scale, int32_t* status, void* stream);

/* Huginn sandwich-norm row step (HuginnBlock.forward, modeling_huginn.py:333-336; run_coda :454-460):
 *   v = x_src[x_rows ? x_rows[r] : r];  if add: v = bf16(v + add[r]);  if w1: v = rmsnorm(v; w1);
 *   if x_dst: x_dst[x_dst_rows ? x_dst_rows[r] : r] = v  (skipped when that index < 0);
 *   if w2: y[r] = rmsnorm(v; w2).
 * Every pointer but x_src may be NULL; rmsnorm is HuginnRMSNorm (fp32 normalise, bf16 cast, bf16
 * gain multiply). A row whose x_rows entry is < 0 is skipped. hidden % 8 == 0, <= 12288. */
int cdb_sandwich_norm(const void* x_src, int64_t x_src_stride, const int32_t* x_rows, const void* add,
                      int64_t add_stride, const void* w1, void* x_dst, int64_t x_dst_stride,
                      const int32_t* x_dst_rows, const void* w2, void* y, int64_t y_stride, int num_rows, int hidden,
                      float eps, void* stream);

/* Huginn exit signal (latent_diff, models/huginn/exit_gates.py:33-40, as HuginnCDBAdapter.exit_signal
 * computes it in bf16, adapters/huginn.py:171-175): out[r] = bf16(bf16(||bf16(new-old)||) /
 * max(bf16(||new||), 1e-9)) with new = new_state[rows[r]] (row r when rows is NULL) and
 * old = old_state[r]; rows[r] < 0 skips row r. */
int cdb_latent_diff(const void* new_state, int64_t new_stride, const void* old_state, int64_t old_stride,
                    const int32_t* rows, int num_rows, int hidden, void* out, void* stream);

/* Apply n block-table edits {row, column, block_id} (int32 triples) to a device block table
 * [rows, stride]. The device mirror of FullAttentionCacheAllocator.allocate_blocks /
 * _refresh_cached_block_table (cache_manager.py:150-165, continuous_depth_batching/cache.py:115-144). */
int cdb_block_table_update(int32_t* table, int64_t stride, const int32_t* edits, int num_edits, void* stream);

/* Offload preemption: copy num KV blocks between the paged device pool kv_base
 * [num_cache_layers][2][kv_rows][row_bytes] and a host pool host_pool
 * [num_host_blocks][2 * num_cache_layers][block_size * row_bytes] (pinned, so the copies run
 * asynchronously). Block i moves between device block device_blocks[i] and host block
 * host_blocks[i], all cache layers, K and V; to_host = 1 copies device -> host, 0 host -> device.
 * device_blocks and host_blocks are HOST arrays; every id is range-checked (CDB_ERR_INDEX, nothing
 * queued) before the copies are queued on stream. Enqueues copies only, no kernel.
 * Replaces OffloadingManager._offload_to_cpu / restore_scheduled_requests
 * (offloading_manager.py:216-306), whose per-block, per-layer copy_ loops become one 2-D copy per block. */
int cdb_kv_blocks_host_copy(void* kv_base, int num_cache_layers, int64_t kv_rows, int64_t row_bytes, int block_size,
                            int num_device_blocks, const int32_t* device_blocks, void* host_pool, int num_host_blocks,
                            const int32_t* host_blocks, int num, int to_host, void* stream);

/* last_exited copy-on-exit: for each token row in rows[n] copy K and V of cache layer
 * src_layers[i] into dst_layers[i] (num_pairs pairs). PagedAttentionCache.copy_kv_rows driven by
 * _flush_exit_kv_copies (continuous_depth_batching/cache.py:105-113, continuous_api.py:1225-1245). */
int cdb_exit_kv_copy(void* kv_base, int num_cache_layers, int64_t kv_rows, int num_kv_heads, int head_dim,
                     const int32_t* rows, int num_rows, const int32_t* src_layers, const int32_t* dst_layers,
                     int num_pairs, void* stream);

/* dst[r] = src[rows[r]] for bf16 rows of `hidden` elements; rows[r] < 0 zeroes row r. The
 * gather of exited tokens' hidden states from the bank before the LM head
 * (`_run_coda_forward_graphed`, model_runner.py:1064-1125) and of the prefill rows whose logits
 * are kept (`logits_to_keep`, continuous_batching/model_runner.py:304-333). */
int cdb_gather_rows(const void* src, int64_t src_stride, const int32_t* rows, int num_rows, int hidden, void* dst,
                    int64_t dst_stride, void* stream);

/* Cumulative-hazard exit decision on device (ExitPolicy.should_exit, exit_policy.py:150-169):
 * for row r with hidden slot s = slots[r] (>= 0): h = float(bf16(sigmoid(signal[r]))) when
 * signal_bf16 else sigmoid in fp32; cdf[s] += h*surv[s]; surv[s] *= 1-h;
 * exit[r] = (steps[r]+1 >= min_steps) && cdf[s] >= threshold. cdf/surv are fp64 per slot and
 * must be reset (cdf=0, surv=1) when a slot starts a new token (reset[r] != 0 does that first). */
int cdb_exit_hazard(const void* signal, int signal_bf16, const int32_t* slots, const int32_t* steps,
                    const int8_t* reset, double* cdf, double* surv, int8_t* exit_out, int num_rows,
                    int min_steps, double threshold, void* stream);

/* ---------------------------------------------------------------- device scheduling primitives */

/* Exit-gate evaluation plus routing and compaction of one recurrent launch on device: the
 * decision of ExitPolicy.should_exit (exit_policy.py:150-169) and the routing of
 * _run_mixed_recurrent_batch / the delayed consumption path (continuous_api.py:1090-1203,
 * 1250-1280, 1699-1724). Row r: policy-state slot hidden[r] (< 0: padding, not routed), step[r],
 * replay depth depth[r] (NULL or < 0: none), reset[r] (NULL, or nonzero when the row starts a
 * new token: its slot's state is cleared first), signal = bf16 signal[r * signal_stride].
 *   policy 0 none, 1 cumulative hazard (h = bf16(sigmoid(x)); cdf += h*surv; surv *= 1-h;
 *          d = step+1 >= min_steps && cdf >= threshold), 2 direct threshold (d = step+1 >=
 *          min_steps && x < threshold). cdf/surv fp64 per slot.
 *   delayed 0: exit = step == max_steps-1 || (replay ? step >= depth : d).
 *   delayed 1 (use_async_batching with delay_gate_consumption): exit = step == max_steps-1 ||
 *          (replay ? step >= depth+1 : pending[slot] == 1); then pending[slot] = d (-1 without a
 *          policy). pending is int8 per slot, -1 = none.
 * Outputs: exit_flag[r] (1 exit, 0 continue, -1 padding); survivors / exits: row indices in row
 * order (survivors return to the depth-queue head in that order, exits join the coda queue in
 * it); counts = {num_survivors, num_exits}. One CTA; n any size. */
int cdb_exit_gate_route(const void* signal, int64_t signal_stride, const int32_t* hidden, const int32_t* step,
                        const int32_t* depth, const int8_t* reset, double* cdf, double* surv, int8_t* pending,
                        int num_rows, int policy, int delayed, int min_steps, int max_steps, double threshold,
                        int8_t* exit_flag, int32_t* survivors, int32_t* exits, int32_t* counts, void* stream);

/* Device FIFO KV block allocator, the order-exact mirror of BlockManager
 * (continuous_batching/cache_manager.py:33-91): ring[num_blocks] of free ids, popped at the head
 * and appended at the tail; state int32[4] = {head, free count, num_blocks, peak allocated};
 * row_len[num_rows] = blocks held by each block-table row. cdb_block_pool_init fills the ring
 * with 0..num_blocks-1 (the deque(range(num_blocks)) start) and zeroes row_len. */
int cdb_block_pool_init(int32_t* ring, int32_t* state, int32_t* row_len, int num_rows, int num_blocks, void* stream);

/* Requests in order: request j appends counts[j] blocks from the ring's head to block-table row
 * slots[j] (after its row_len blocks), or, when fewer blocks are free than it asks for or the row
 * would pass `width`, takes none and gets granted[j] = 0 while later requests still try
 * (get_free_blocks, cache_manager.py:72-81; exact-ceil counts as in _allocate_blocks_if_needed,
 * scheduler_base.py:416-433). slots must lie in [0, num_rows). */
int cdb_block_alloc(int32_t* ring, int32_t* state, int32_t* row_len, int32_t* block_table,
                    int64_t block_table_stride, int width, const int32_t* slots, const int32_t* counts,
                    int num_requests, int32_t* granted, void* stream);

/* Rows slots[j], in the order given: their blocks in column order are appended at the ring's tail
 * (a finished request's block list released, BlockManager.free_blocks), the row is reset to -1
 * and its row_len to 0. Each slot at most once per call. */
int cdb_block_free(int32_t* ring, int32_t* state, int32_t* row_len, int32_t* block_table,
                   int64_t block_table_stride, const int32_t* slots, int num_slots, void* stream);

/* One CDB scheduler tick on device-resident queues (CDBScheduler.schedule_next, scheduler.py:101-140,
 * with enqueue_depth / enqueue_depth_front / enqueue_coda, :142-186, and the slot-homogeneous FIFO
 * pop of _schedule_recurrent_batch, :322-346), applied in the engine's order:
 *   1. routed[i] (the last recurrent batch, in batch order): exit_flag[i] != 0 joins the coda
 *      queue; the others return to the head of the depth queue in batch order, item_step += 1;
 *   2. back[]: appended to the depth queue (prefill successors);
 *   3. front[]: to the head of the depth queue, in order (coda successors);
 *   then the work: a coda batch (up to max_num_seqs from the coda queue's head) when it holds
 *   min_coda_batch_size items, else prefill when prefill_admit (the host's admission), else a
 *   recurrent batch of up to max_num_seqs items whose KV slot min(step, kv_slots_per_layer - 1)
 *   equals the head item's (the others keep their order), else a coda flush.
 * queue_state int32[8] = {ready head, ready count, coda head, coda count, capacity, refill events,
 * 0, 0} (cdb_schedule_queues_init); ready / coda: int32 rings of `capacity` <= 2048 item ids;
 * item_step: int32 per item id. A step-0 item joining a non-empty depth queue counts a refill.
 * out: int32 [2 + max_num_seqs] = {kind (0 idle, 1 coda, 2 prefill, 3 recurrent; -1 a queue would
 * overflow or the state is invalid, nothing changed), count, item ids of the batch}. */
int cdb_schedule_tick(int32_t* queue_state, int32_t* ready, int32_t* coda, int32_t* item_step, const int32_t* routed,
                      const int8_t* exit_flag, int num_routed, const int32_t* back, int num_back, const int32_t* front,
                      int num_front, int min_coda_batch_size, int max_num_seqs, int prefill_admit,
                      int kv_slots_per_layer, int32_t* out, void* stream);

/* Empty queues of `capacity` (<= 2048) items each for cdb_schedule_tick. */
int cdb_schedule_queues_init(int32_t* queue_state, int capacity, void* stream);

/* The per-launch metadata FlashAttention's kvcache branch takes (_prepare_recurrent_stage_buffers,
 * model_runner.py:704-754, gather_block_table_host_rows, continuous_depth_batching/cache.py:66-91):
 * out_table[i] = the full block row of slot item_slot[i] (-1 past its row_len blocks, `width`
 * columns), cu_seq_lens_q = 0,1,..,num_items then plateaued, cu_seq_lens_k[i+1] =
 * cu_seq_lens_k[i] + item_pos[i] + 1 then plateaued; padding rows num_items <= i < bucket get
 * all -1. cu arrays hold bucket+1 entries. A row whose position lies past its blocks sets
 * CDB_ERR_INDEX in *status (the reference raises ValueError). */
int cdb_build_tables(const int32_t* block_table, int64_t block_table_stride, const int32_t* row_len, int width,
                     int block_size, const int32_t* item_slot, const int32_t* item_pos, int num_items, int bucket,
                     int32_t* out_table, int64_t out_stride, int32_t* cu_seq_lens_q, int32_t* cu_seq_lens_k,
                     int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CDB_B200_H_ */
