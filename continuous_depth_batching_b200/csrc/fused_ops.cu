// Projection entry points that carry the row work following them: QKV + RoPE + KV append, and the
// O / down projections with Ouro's residual sandwich norm. Each is the tcgen05 GEMM followed by the
// row kernel on the same stream; the row kernel is launched with programmatic dependent launch, so
// its launch and weight loads overlap the GEMM's tail. The norm needs whole output rows, which the
// GEMM spreads over ~16 weight tiles; folding it into the GEMM's epilogue would take two grid-wide
// barriers per call (sum of squares of the projection, then of the updated residual), which cost
// more than the second launch at decode sizes.
#include "cdb_common.cuh"
#include "cdb_b200.h"

extern "C" int cdb_qkv_rope_append_gemm(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw, void* qkv,
                                        int64_t qkv_stride, int64_t k_col, int64_t v_col, int num_items, int K,
                                        void* kv_base, int num_cache_layers, int64_t kv_rows, int cache_layer,
                                        const int32_t* block_table, int64_t block_table_stride,
                                        const int32_t* item_slot, const int32_t* item_pos, int rope_mode,
                                        const void* rope_cos, const void* rope_sin, const void* qk_bias,
                                        int num_heads, int head_dim, int block_size, float* workspace,
                                        int64_t workspace_elems, int32_t* counters, int num_counters, int num_sms,
                                        int32_t* status, void* stream) {
  if (num_items < 0 || num_heads <= 0 || head_dim <= 0 || k_col < (int64_t)num_heads * head_dim ||
      v_col < k_col + (int64_t)num_heads * head_dim)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_items == 0) return CDB_OK;
  const int n_out = (int)(v_col + (int64_t)num_heads * head_dim);
  int rc = cdb_gemm_bf16(x, ldx, w_qkv, ldw, qkv, qkv_stride, num_items, n_out, K, 0, workspace, workspace_elems,
                         counters, num_counters, num_sms, status, stream);
  if (rc != CDB_OK) return rc;
  return cdb_rope_append_kv(qkv, qkv_stride, k_col, v_col, kv_base, num_cache_layers, kv_rows, cache_layer,
                            block_table, block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin,
                            qk_bias, num_items, num_heads, head_dim, block_size, stream);
}

// o = a * W^T (the projection, written to `proj`); x <- bf16(x + norm_a(o)); y[y_rows[r]] =
// norm_next(x[r]) (rows with y_rows[r] < 0 skipped); optionally gate_out[r] = gate_w . y[r] + gate_b.
static int residual_norm_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, void* proj, int64_t ld_proj,
                              void* x, int64_t x_stride, const void* w_a, const void* w_next, void* y,
                              int64_t y_stride, const int32_t* y_rows, const void* gate_w, const void* gate_b,
                              void* gate_out, int num_rows, int hidden, int K, float eps, float* workspace,
                              int64_t workspace_elems, int32_t* counters, int num_counters, int num_sms,
                              int32_t* status, void* stream) {
  if (num_rows < 0 || hidden <= 0 || K <= 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  int rc = cdb_gemm_bf16(a, lda, w, ldw, proj, ld_proj, num_rows, hidden, K, 0, workspace, workspace_elems, counters,
                         num_counters, num_sms, status, stream);
  if (rc != CDB_OK) return rc;
  return cdb_add_rmsnorm(x, x_stride, proj, ld_proj, w_a, w_next, y, y_stride, y_rows, gate_w, gate_b, gate_out,
                         num_rows, hidden, eps, stream);
}

extern "C" int cdb_o_proj_residual_norm_gemm(const void* attn, int64_t ld_attn, const void* w_o, int64_t ldw,
                                             void* proj, int64_t ld_proj, void* x, int64_t x_stride,
                                             const void* w_norm_post, const void* w_norm_next, void* y,
                                             int64_t y_stride, int num_rows, int hidden, int K, float eps,
                                             float* workspace, int64_t workspace_elems, int32_t* counters,
                                             int num_counters, int num_sms, int32_t* status, void* stream) {
  return residual_norm_gemm(attn, ld_attn, w_o, ldw, proj, ld_proj, x, x_stride, w_norm_post, w_norm_next, y,
                            y_stride, nullptr, nullptr, nullptr, nullptr, num_rows, hidden, K, eps, workspace,
                            workspace_elems, counters, num_counters, num_sms, status, stream);
}

extern "C" int cdb_down_residual_norm_gemm(const void* act, int64_t ld_act, const void* w_down, int64_t ldw,
                                           void* proj, int64_t ld_proj, void* x, int64_t x_stride,
                                           const void* w_norm_post, const void* w_norm_next, void* y,
                                           int64_t y_stride, const int32_t* y_rows, const void* gate_w,
                                           const void* gate_b, void* gate_out, int num_rows, int hidden, int K,
                                           float eps, float* workspace, int64_t workspace_elems, int32_t* counters,
                                           int num_counters, int num_sms, int32_t* status, void* stream) {
  return residual_norm_gemm(act, ld_act, w_down, ldw, proj, ld_proj, x, x_stride, w_norm_post, w_norm_next, y,
                            y_stride, y_rows, gate_w, gate_b, gate_out, num_rows, hidden, K, eps, workspace,
                            workspace_elems, counters, num_counters, num_sms, status, stream);
}
