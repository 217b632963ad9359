// extern "C" entry points declared in include/lmoe.h.
#include "../../include/lmoe.h"
#include "lmoe_internal.h"
#include "ptx.cuh"



namespace {
inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }
constexpr int kEpiBf16 = 0, kEpiF32 = 1, kEpiBf16Add = 2, kEpiSitu = 3;
}  // namespace

extern "C" {

int lmoe_version(void) { return 100; }

int lmoe_ragged_dot_bf16(const void* lhs, const void* rhs, const int32_t* group_sizes, void* out,
                         int64_t m, int64_t k, int64_t n, int64_t num_groups, int rhs_layout,
                         int out_f32, int zero_tail, int32_t* dev_status, void* stream) {
  if (group_sizes == nullptr) return LMOE_BAD_SHAPE;
  return lmoe::grouped_gemm_bf16(lhs, rhs, group_sizes, out, m, k, n, num_groups, rhs_layout,
                                 out_f32 ? kEpiF32 : kEpiBf16, nullptr, 0, 0, 0.f, 0.f, 0,
                                 zero_tail ? 1 : 0, dev_status, S(stream));
}

int lmoe_ragged_dot_f32(const float* lhs, const float* rhs, const int32_t* group_sizes, float* out,
                        int64_t m, int64_t k, int64_t n, int64_t num_groups, int rhs_layout,
                        int32_t* dev_status, void* stream) {
  if (group_sizes == nullptr) return LMOE_BAD_SHAPE;
  return lmoe::simt_grouped_gemm_f32(lhs, rhs, group_sizes, out, nullptr, m, k, n, num_groups,
                                     rhs_layout, 1, dev_status, S(stream));
}

int lmoe_gemm_f32(const float* lhs, const float* rhs, const float* addend, float* out, int64_t m,
                  int64_t k, int64_t n, int rhs_layout, int32_t* dev_status, void* stream) {
  return lmoe::simt_grouped_gemm_f32(lhs, rhs, nullptr, out, addend, m, k, n, 1, rhs_layout, 0,
                                     dev_status, S(stream));
}

int lmoe_gemm_bf16(const void* lhs, const void* rhs, const void* addend, void* out, int64_t m,
                   int64_t k, int64_t n, int rhs_layout, int out_f32, int32_t* dev_status,
                   void* stream) {
  // out_f32: 0 = bf16 out, 1 = f32 out, 2 = bf16-rounded values stored as f16
  if (out_f32 < 0 || out_f32 > 2 || (addend != nullptr && out_f32 != 0)) return LMOE_UNSUPPORTED;
  const int epi = addend ? kEpiBf16Add : (out_f32 == 1 ? kEpiF32 : kEpiBf16);
  return lmoe::grouped_gemm_bf16(lhs, rhs, nullptr, out, m, k, n, 1, rhs_layout, epi, addend, n,
                                 0, 0.f, 0.f, 0, 0, dev_status, S(stream), nullptr, 0,
                                 out_f32 == 2 ? 1 : 0);
}

int lmoe_gateup_situ_bf16(const void* lhs, const void* w_gateup, const int32_t* group_sizes,
                          void* out, int64_t m, int64_t k, int64_t intermediate,
                          int64_t num_groups, int rhs_layout, float beta, float linear_beta,
                          int round_gate_up, const int32_t* lhs_row_index, int64_t lhs_src_rows,
                          int zero_tail, int32_t* dev_status, void* stream) {
  return lmoe::grouped_gemm_bf16(lhs, w_gateup, group_sizes, out, m, k, intermediate,
                                 group_sizes ? num_groups : 1, rhs_layout, kEpiSitu, nullptr, 0,
                                 intermediate, beta, linear_beta, round_gate_up,
                                 (group_sizes && zero_tail) ? 1 : 0, dev_status, S(stream),
                                 lhs_row_index, lhs_src_rows);
}

int lmoe_mxfp4_ragged_dot(const void* lhs, const void* weight_packed, const void* weight_scale,
                          const int32_t* group_sizes, void* out, int64_t m, int64_t k, int64_t n,
                          int64_t num_groups, int lhs_f16, int out_f32, int zero_tail,
                          int32_t* dev_status, void* stream) {
  if (group_sizes == nullptr) return LMOE_BAD_SHAPE;
  return lmoe::grouped_gemm_mxfp4(lhs, weight_packed, weight_scale, group_sizes, out, m, k, n,
                                  num_groups, out_f32 ? kEpiF32 : kEpiBf16, 0, 0.f, 0.f, 0,
                                  zero_tail ? 1 : 0, lhs_f16, 0, dev_status, S(stream));
}

int lmoe_mxfp4_gateup_situ(const void* lhs, const void* weight_packed, const void* weight_scale,
                           const int32_t* group_sizes, void* out, int64_t m, int64_t k,
                           int64_t intermediate, int64_t num_groups, float beta, float linear_beta,
                           int round_gate_up, int lhs_f16, int out_f16,
                           const int32_t* lhs_row_index, int64_t lhs_src_rows, int zero_tail,
                           int32_t* dev_status, void* stream) {
  return lmoe::grouped_gemm_mxfp4(lhs, weight_packed, weight_scale, group_sizes, out, m, k,
                                  intermediate, group_sizes ? num_groups : 1, kEpiSitu,
                                  intermediate, beta, linear_beta, round_gate_up,
                                  (group_sizes && zero_tail) ? 1 : 0, lhs_f16, out_f16,
                                  dev_status, S(stream), lhs_row_index, lhs_src_rows);
}

int lmoe_mxfp4_ragged_dot_scatter(const void* lhs, const void* weight_packed,
                                  const void* weight_scale, const int32_t* group_sizes,
                                  const uint64_t* row_dest, int64_t m, int64_t k, int64_t n,
                                  int64_t num_groups, int lhs_f16, int32_t* dev_status,
                                  void* stream) {
  return lmoe::grouped_gemm_mxfp4_scatter(lhs, weight_packed, weight_scale, group_sizes, row_dest,
                                          m, k, n, num_groups, lhs_f16, dev_status, S(stream));
}

int lmoe_fp8_ragged_dot(const void* lhs, const void* rhs_q, const float* rhs_scale,
                        const int32_t* group_sizes, void* out, int64_t m, int64_t k, int64_t n,
                        int64_t num_groups, int64_t block_size, int out_f32, int zero_tail,
                        int32_t* dev_status, void* stream) {
  return lmoe::grouped_gemm_fp8(lhs, rhs_q, rhs_scale, group_sizes, out, m, k, n, num_groups,
                                block_size, out_f32, zero_tail, dev_status, S(stream));
}

int lmoe_situ_and_mul(const void* gate, const void* up, int64_t ld_in, void* out, int64_t rows,
                      int64_t intermediate, float beta, float linear_beta, int bf16, void* stream) {
  return lmoe::situ_and_mul(gate, up, ld_in, out, rows, intermediate, beta, linear_beta, bf16,
                            S(stream));
}

int lmoe_router_topk(const float* logits, const float* bias, int64_t num_tokens,
                     int64_t num_experts, int64_t top_k, int activation, int renormalize,
                     float routed_scaling_factor, int32_t* topk_idx, float* topk_w, void* stream) {
  return lmoe::router_topk(logits, bias, num_tokens, num_experts, top_k, activation, renormalize,
                           routed_scaling_factor, topk_idx, topk_w, S(stream));
}

size_t lmoe_router_fused_workspace_size(int64_t num_tokens, int64_t num_experts, int64_t top_k) {
  return lmoe::router_fused_workspace_size(num_tokens, num_experts, top_k);
}

int lmoe_router_fused_bf16(const void* hidden, const void* router_weight, const float* bias,
                           int64_t num_tokens, int64_t hidden_size, int64_t num_experts,
                           int64_t top_k, int renormalize, float routed_scaling_factor,
                           int32_t* topk_idx, float* topk_w, void* workspace,
                           size_t workspace_bytes, int32_t* dev_status, void* stream) {
  return lmoe::router_fused_bf16(hidden, router_weight, bias, num_tokens, hidden_size, num_experts,
                                 top_k, renormalize, routed_scaling_factor, topk_idx, topk_w,
                                 workspace, workspace_bytes, dev_status, S(stream));
}

size_t lmoe_dispatch_workspace_size(int64_t num_entries, int64_t num_local_experts) {
  if (num_entries < 0 || num_local_experts <= 0) return 0;
  return lmoe::dispatch_workspace_bytes(num_entries, num_local_experts);
}

int lmoe_dispatch(const int32_t* topk_idx, const float* topk_w, int64_t num_tokens,
                  int64_t top_k, int64_t expert_start, int64_t num_local_experts, int64_t m_out,
                  int pad_bucket, int32_t* order, int32_t* token_idx, float* weight,
                  int32_t* slot_pos, int32_t* group_sizes, int32_t* per_expert_counts,
                  uint8_t* valid, void* workspace, size_t workspace_bytes, void* stream) {
  if (num_tokens < 0 || top_k <= 0) return LMOE_BAD_SHAPE;
  if (token_idx == nullptr || group_sizes == nullptr) return LMOE_BAD_SHAPE;
  lmoe::DispatchOut o{order, token_idx, weight, slot_pos, group_sizes, per_expert_counts, valid};
  return lmoe::dispatch_sort(topk_idx, topk_w, num_tokens * top_k, top_k, expert_start,
                             num_local_experts, m_out, pad_bucket, o, workspace, workspace_bytes,
                             S(stream));
}

int lmoe_gather_rows(const void* x, int64_t x_rows, const int32_t* token_idx, void* out,
                     int64_t rows, int64_t row_bytes, int convert, int32_t* dev_status,
                     void* stream) {
  return lmoe::gather_rows(x, x_rows, token_idx, out, rows, row_bytes, convert, dev_status,
                           S(stream));
}

int lmoe_scatter_rows(const void* x, const int32_t* slot_pos, int64_t num_tokens, int64_t top_k,
                      void* out, int64_t out_rows, int64_t row_bytes, int convert,
                      int32_t* dev_status, void* stream) {
  return lmoe::scatter_rows(x, slot_pos, num_tokens, top_k, out, out_rows, row_bytes, convert,
                            dev_status, S(stream));
}

int lmoe_combine_rmsnorm(const void* expert_out, const int32_t* slot_pos, const float* topk_w,
                         const void* norm_scale, int64_t num_tokens, int64_t top_k,
                         int64_t latent, float eps, int bf16, void* routed_out, void* normed_out,
                         void* stream) {
  return lmoe::combine_rmsnorm(expert_out, slot_pos, topk_w, norm_scale, num_tokens, top_k, latent,
                               eps, bf16, routed_out, normed_out, S(stream));
}

int lmoe_ep_reorder(const int32_t* recv_counts, int64_t world, int64_t num_local_experts,
                    int64_t rows_cap, int32_t* em_src, int32_t* sm_src, int32_t* group_sizes,
                    void* stream) {
  return lmoe::ep_reorder(recv_counts, world, num_local_experts, rows_cap, em_src, sm_src,
                          group_sizes, S(stream));
}

int lmoe_combine_scatter_add(const void* shard_out, const int32_t* padded_token_idx,
                             const float* padded_combine_weight, void* routed_out, int64_t rows,
                             int64_t latent, int64_t num_tokens, int bf16, void* stream) {
  return lmoe::scatter_add(shard_out, padded_token_idx, padded_combine_weight, routed_out, rows,
                           latent, num_tokens, bf16, S(stream));
}

}  // extern "C"
