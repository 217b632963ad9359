// Internal host-side declarations shared by the CUDA translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace lmoe {

int num_sms(int device);

// Tensor maps for bf16 tiles with 128-byte swizzle (box inner extent = 64
// elements = 128 bytes).  Out-of-range elements read as zero.
bool encode_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_outer);
bool encode_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                         uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                         uint32_t box1);
// 2D uint8 tensor map (e4m3 rows) with 128-byte swizzle; box {box_inner bytes, box_outer rows}.
bool encode_tmap_u8_2d_sw128(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                             uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_outer);
// 3D tensor map over packed 4-bit codes (groups, rows, k codes; k/2 bytes per
// row) that the TMA unpacks into the block-scaled MMA's shared-memory form
// (16 codes per 16 bytes), 128-byte swizzle, box {128 codes, 128 rows, 1}.
bool encode_tmap_fp4_unpacked_3d(CUtensorMap* map, const void* base, uint64_t k, uint64_t rows,
                                 uint64_t groups);
// Tensor map for raw bytes (uint8), no swizzle, 3D.
bool encode_tmap_u8_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                       uint32_t box1);
// The same with 128-byte swizzle (box0 = 128 bytes): packed e2m1 operand rows
// for the kind::mxf4 MMA.
bool encode_tmap_u8_3d_sw128(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                             uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                             uint32_t box0, uint32_t box1);

int grouped_gemm_bf16(const void* lhs, const void* rhs, const int32_t* group_sizes, void* out,
                      int64_t M, int64_t K, int64_t N_out, int64_t G, int rhs_layout, int epi,
                      const void* addend, int64_t ld_add, int64_t up_offset, float beta,
                      float linear_beta, int round_gate_up, int zero_tail, int32_t* status,
                      cudaStream_t stream, const int32_t* a_rows = nullptr,
                      int64_t a_src_rows = 0, int out_f16 = 0);

int grouped_gemm_mxfp4(const void* lhs, const void* packed, const void* scales,
                       const int32_t* group_sizes, void* out, int64_t M, int64_t K, int64_t N_out,
                       int64_t G, int epi, int64_t up_offset, float beta, float linear_beta,
                       int round_gate_up, int zero_tail, int lhs_f16, int out_f16,
                       int32_t* status, cudaStream_t stream, const int32_t* a_rows = nullptr,
                       int64_t a_src_rows = 0);

int grouped_gemm_fp8(const void* lhs, const void* rhs_q, const float* rhs_scale,
                     const int32_t* group_sizes, void* out, int64_t M, int64_t K, int64_t N,
                     int64_t G, int64_t block_size, int out_f32, int zero_tail, int32_t* status,
                     cudaStream_t stream);

int grouped_gemm_mxfp4_scatter(const void* lhs, const void* packed, const void* scales,
                               const int32_t* group_sizes, const uint64_t* row_dest, int64_t M,
                               int64_t K, int64_t N, int64_t G, int lhs_f16, int32_t* status,
                               cudaStream_t stream);

inline int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int simt_grouped_gemm_f32(const float* lhs, const float* rhs, const int32_t* group_sizes,
                          float* out, const float* addend, int64_t M, int64_t K, int64_t N,
                          int64_t G, int rhs_layout, int zero_tail, int32_t* status,
                          cudaStream_t stream);
int router_topk(const float* logits, const float* bias, int64_t T, int64_t E, int64_t k,
                int activation, int renormalize, float rsf, int32_t* topk_idx, float* topk_w,
                cudaStream_t stream);

size_t router_fused_workspace_size(int64_t T, int64_t E, int64_t k);
int router_fused_bf16(const void* hidden, const void* router_w, const float* bias, int64_t T,
                      int64_t K, int64_t E, int64_t k, int renormalize, float rsf,
                      int32_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                      int32_t* status, cudaStream_t stream);

// Dispatch outputs (device pointers; optional ones may be null).
struct DispatchOut {
  int32_t* order;              // [m_out] entry index at each sorted position
  int32_t* token_idx;          // [m_out] source token, -1 for padding
  float* weight;               // [m_out] combine weight, 0 for padding
  int32_t* slot_pos;           // [S]     sorted position of entry i, -1 if not kept
  int32_t* group_sizes;        // [num_keys (+1 with the padding bucket)]
  int32_t* per_expert_counts;  // [num_keys]
  uint8_t* valid;              // [m_out]
};
size_t dispatch_workspace_bytes(int64_t n_ext, int64_t num_keys);
int dispatch_sort(const int32_t* flat_ids, const float* flat_w, int64_t S, int64_t top_k,
                  int64_t start, int64_t num_keys, int64_t m_out, int pad_bucket, DispatchOut o,
                  void* workspace, size_t ws_bytes, cudaStream_t stream);
int scatter_rows(const void* x, const int32_t* slot_pos, int64_t T, int64_t k, void* out,
                 int64_t out_rows, int64_t row_bytes, int convert, int32_t* status,
                 cudaStream_t stream);
int gather_rows(const void* x, int64_t x_rows, const int32_t* token_idx, void* out, int64_t rows,
                int64_t row_bytes, int convert, int32_t* status, cudaStream_t stream);
int combine_rmsnorm(const void* expert_out, const int32_t* slot_pos, const float* topk_w,
                    const void* norm_scale, int64_t T, int64_t k, int64_t L, float eps, int bf16,
                    void* routed_out, void* normed_out, cudaStream_t stream);
int scatter_add(const void* shard_out, const int32_t* idx, const float* w, void* routed,
                int64_t rows, int64_t L, int64_t T, int bf16, cudaStream_t stream);
int ep_reorder(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t rows_cap,
               int32_t* em_src, int32_t* sm_src, int32_t* group_sizes, cudaStream_t stream);
int situ_and_mul(const void* gate, const void* up, int64_t ld_in, void* out, int64_t rows,
                 int64_t I, float beta, float lbeta, int bf16, cudaStream_t stream);

}  // namespace lmoe
