// Declarations of the host launchers exported by the native extension.
#pragma once

#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <vector>

void gsb_switched_gemm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                       int64_t epi_kind, int64_t bn, const c10::optional<at::Tensor>& residual,
                       double scale, const c10::optional<at::Tensor>& s,
                       const c10::optional<at::Tensor>& lb,
                       const c10::optional<at::Tensor>& tile_mask, int64_t rank,
                       int64_t num_adapters, std::vector<int64_t> slice_bounds,
                       const c10::optional<at::Tensor>& row_adapter, int64_t mask_rank,
                       int64_t mask_num_adapters, const at::Tensor& err, int64_t mc_out,
                       const c10::optional<at::Tensor>& tile_expert);

int64_t gsb_gemm_pair_min_m(int64_t m);
int64_t gsb_gemm_decode_max_m(int64_t v);
void gsb_gemm_decode_force_split(int64_t acc, int64_t ks);
void gsb_gemm_decode_trace(const at::Tensor& buf);
void gsb_lora_shrink_small(const at::Tensor& x, const at::Tensor& a_all, const at::Tensor& row_adapter,
                           const at::Tensor& s, int64_t rank, int64_t num_adapters);
void gsb_quantize_fp8_rows(const at::Tensor& x, const at::Tensor& x8, const at::Tensor& sfa, const at::Tensor& err);
void gsb_fp8_gemm(const at::Tensor& x8, const at::Tensor& sfa, const at::Tensor& w8, const at::Tensor& sfb,
                  const at::Tensor& out, int64_t epi, double scale, const c10::optional<at::Tensor>& residual,
                  const c10::optional<at::Tensor>& s, const c10::optional<at::Tensor>& lb,
                  const c10::optional<at::Tensor>& tile_mask, int64_t rank, int64_t num_adapters,
                  std::vector<int64_t> slice_bounds, const at::Tensor& err);
void gsb_rope_kv_fp8(const at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                     const at::Tensor& slots, const at::Tensor& k8, const at::Tensor& v8, const at::Tensor& k_scale,
                     const at::Tensor& v_scale, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                     const at::Tensor& err);
void gsb_kv_write_fp8(const at::Tensor& qkv, const at::Tensor& slots, const at::Tensor& k8, const at::Tensor& v8,
                      const at::Tensor& k_scale, const at::Tensor& v_scale, int64_t num_q_heads,
                      int64_t num_kv_heads, int64_t head_dim, const at::Tensor& err);
std::vector<int64_t> gsb_gemm_decode_plan(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t swiglu_tile);

void gsb_rmsnorm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                 const c10::optional<at::Tensor>& rows, double eps);
void gsb_embed(const at::Tensor& ids, const at::Tensor& table, const c10::optional<at::Tensor>& lut,
               double mult, const at::Tensor& out, const at::Tensor& err);
void gsb_rope_kv(const at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                 const c10::optional<at::Tensor>& k_cache, const c10::optional<at::Tensor>& v_cache,
                 const c10::optional<at::Tensor>& slots, int64_t num_q_heads, int64_t num_kv_heads,
                 int64_t head_dim, const at::Tensor& err);
void gsb_argmax(const at::Tensor& logits, const at::Tensor& out);
void gsb_routing(const at::Tensor& ids, const at::Tensor& seq_starts, const c10::optional<at::Tensor>& carry_in,
                 const at::Tensor& expert_tbl, const c10::optional<at::Tensor>& lut,
                 const c10::optional<at::Tensor>& kind_lut, int64_t num_adapters,
                 const c10::optional<at::Tensor>& remap, const at::Tensor& adapter_idx,
                 const at::Tensor& lora_idx, const at::Tensor& modified_ids,
                 const c10::optional<at::Tensor>& carry_out, const c10::optional<at::Tensor>& row_adapter,
                 const c10::optional<at::Tensor>& tile_mask);
void gsb_paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                         const at::Tensor& block_table, const at::Tensor& q_start, const at::Tensor& kv_len,
                         const at::Tensor& work_seq, const at::Tensor& work_row0, int64_t rows_per_tile,
                         int64_t num_q_heads, double scale, const at::Tensor& out, int64_t nsplit,
                         const c10::optional<at::Tensor>& ws_o, const c10::optional<at::Tensor>& ws_lse,
                         const at::Tensor& err, const c10::optional<at::Tensor>& k_scale,
                         const c10::optional<at::Tensor>& v_scale);
void gsb_sample(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                const at::Tensor& top_p, const at::Tensor& seeds, const at::Tensor& offsets, const at::Tensor& out);
void gsb_prefill_attention_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                              const at::Tensor& block_table, const at::Tensor& q_start, const at::Tensor& kv_len,
                              const at::Tensor& work_seq, const at::Tensor& work_row0, int64_t num_q_heads,
                              double scale, const at::Tensor& out, const at::Tensor& err, int64_t rows_per_tile,
                              int64_t nsplit, const c10::optional<at::Tensor>& ws_o,
                              const c10::optional<at::Tensor>& ws_lse);
void gsb_peer_barrier(const at::Tensor& pad_ptrs_dev, int64_t rank, int64_t tp, const at::Tensor& epoch_ctr, int64_t budget_ns,
                      const at::Tensor& err);
void gsb_rmsnorm_residual_from(const at::Tensor& y, const at::Tensor& h, const at::Tensor& w, const at::Tensor& x,
                               double eps);
void gsb_probe_verdict(const at::Tensor& hidden, const at::Tensor& rows, const at::Tensor& slots,
                       const at::Tensor& out_rows, const at::Tensor& w, const at::Tensor& bias,
                       const at::Tensor& verdict);
void gsb_probe_rewrite(const at::Tensor& logits, int64_t vocab_lo, const at::Tensor& out_rows,
                       const at::Tensor& slots, const at::Tensor& labels, const at::Tensor& verdict);
void gsb_moe_route(const at::Tensor& logits, int64_t num_experts, int64_t top_k, const at::Tensor& ids,
                   const at::Tensor& wts, const at::Tensor& counts, const at::Tensor& offsets, const at::Tensor& cursor,
                   const at::Tensor& tile_expert);
void gsb_moe_scatter(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& offsets, const at::Tensor& cursor,
                     const at::Tensor& slot, const at::Tensor& xp);
void gsb_moe_scatter_slots(const at::Tensor& x, const at::Tensor& slot, int64_t top_k, const at::Tensor& xp);
void gsb_moe_combine(const at::Tensor& yp, const at::Tensor& slot, const at::Tensor& wts, int64_t top_k,
                     const c10::optional<at::Tensor>& shared, const c10::optional<at::Tensor>& residual, double scale,
                     const at::Tensor& out);
void gsb_residual_axpy(const at::Tensor& h, const at::Tensor& y, double scale);
int64_t gsb_attn_packed(int64_t v);
int64_t gsb_gemm_splitk_max_tiles(int64_t v);
int64_t gsb_attn_fp8t_stages(int64_t v);
int64_t gsb_attn_decode_stages(int64_t v);
