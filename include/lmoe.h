/*
 * lmoe.h -- C ABI of the B200 (sm_100a) LatentMoE expert path.
 *
 * Drop-in boundary for the reference's JAX-facing operators
 * (Yog-Sothothftgn/tokamax-tpu-kernel-lab, paths below relative to its root).
 * Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream (`stream` is a
 *     cudaStream_t passed as void*; NULL = the legacy default stream);
 *   - is stream-ordered and asynchronous, allocates nothing and never
 *     synchronises the host (group sizes live in device memory and are read
 *     only on the device) -- except the exchange-buffer setup calls
 *     lmoe_ep_buffer_alloc / _open / _close / _free, which exist to allocate
 *     and map memory and are synchronous;
 *   - returns LMOE_OK or a host-detected error code;
 *   - optionally records a device-detected error (group sizes that exceed the
 *     row count, a bounded wait that timed out) in `dev_status`, a device
 *     int32 the caller zeroes and reads back when it chooses (may be NULL).
 * Layouts are row-major.  bf16 = IEEE bfloat16 stored as uint16.
 */
#ifndef LMOE_H_
#define LMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LMOE_API __attribute__((visibility("default")))
#else
#define LMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LMOE_OK = 0,
  LMOE_BAD_SHAPE = 1,      /* sizes out of range / inconsistent */
  LMOE_UNSUPPORTED = 2,    /* alignment or divisibility the kernels need */
  LMOE_LAUNCH_FAILED = 3,  /* CUDA launch or tensor-map encode failed */
  LMOE_DEVICE_BOUNDS = 4,  /* (dev_status) group sizes invalid on the device */
  LMOE_WAIT_TIMEOUT = 5,   /* (dev_status) a bounded device wait gave up */
  LMOE_SCRATCH_TOO_SMALL = 6, /* request exceeds the library's built-in scratch */
  LMOE_F16_RANGE = 7       /* (dev_status) a value written as an f16 operand was
                              outside f16's finite range (|x| > 65504) */
};

enum { LMOE_RHS_GKN = 0, LMOE_RHS_GNK = 1 };
enum { LMOE_ROUTER_SIGMOID = 0, LMOE_ROUTER_SOFTMAX = 1 };

/* Library version (major*10000 + minor*100 + patch). */
LMOE_API int lmoe_version(void);

/* Grouped matmul, bf16 in, f32 accumulate (tcgen05), bf16 or f32 out.
 *   out[r] = lhs[r] @ rhs[g]  for r in group g's contiguous row range; with
 *   zero_tail = 1 rows at or past sum(group_sizes) are written as zero (the
 *   ragged_dot contract); 0 leaves them untouched (an exchange buffer sized by
 *   capacity, whose tail nobody reads).
 * lhs (m, k); rhs (g, k, n) [LMOE_RHS_GKN] or (g, n, k) [LMOE_RHS_GNK];
 * group_sizes (g,) int32 device; out (m, n).  k, n multiples of 8.
 * Replaces tokamax.ragged_dot(lhs, rhs, group_sizes, implementation=...)
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:358-369, 604-607). */
LMOE_API int lmoe_ragged_dot_bf16(const void* lhs, const void* rhs, const int32_t* group_sizes, void* out,
                         int64_t m, int64_t k, int64_t n, int64_t num_groups, int rhs_layout,
                         int out_f32, int zero_tail, int32_t* dev_status, void* stream);

/* Same semantics in IEEE float32 on the CUDA cores (f32 compute dtype).
 * Replaces ragged_dot with f32 operands (the reference's f32 configs,
 * 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:383-406). */
LMOE_API int lmoe_ragged_dot_f32(const float* lhs, const float* rhs, const int32_t* group_sizes, float* out,
                        int64_t m, int64_t k, int64_t n, int64_t num_groups, int rhs_layout,
                        int32_t* dev_status, void* stream);

/* Dense f32 GEMM on the CUDA cores with an optional fused f32 residual add:
 *   out = lhs @ rhs (+ addend).  The f32 form of lmoe_gemm_bf16 below. */
LMOE_API int lmoe_gemm_f32(const float* lhs, const float* rhs, const float* addend, float* out,
                           int64_t m, int64_t k, int64_t n, int rhs_layout, int32_t* dev_status,
                           void* stream);

/* Dense bf16 GEMM with a fused bf16 residual add:
 *   out = bf16(bf16(lhs @ rhs) + addend)       (addend may equal nothing: pass NULL
 *   for a plain bf16(lhs @ rhs)).  rhs layout as above with g = 1.
 *   out_f32: 0 = bf16 out, 1 = f32 out, 2 = the bf16-rounded result stored as
 *   f16 (the lhs form of the f16-operand MXFP4 kernels); 1 and 2 need addend NULL.
 * Replaces `up + shared_out` after `normed @ up_proj` / `... @ shared_down`
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:422-435). */
LMOE_API int lmoe_gemm_bf16(const void* lhs, const void* rhs, const void* addend, void* out, int64_t m,
                   int64_t k, int64_t n, int rhs_layout, int out_f32, int32_t* dev_status,
                   void* stream);

/* Fused gate/up grouped matmul + SiTU-GLU epilogue, bf16 out (m, intermediate).
 * w_gateup is the plain concatenation [gate | up] along N:
 *   (g, k, 2*intermediate) [LMOE_RHS_GKN] or (g, 2*intermediate, k) [LMOE_RHS_GNK].
 * round_gate_up = 1 rounds gate/up to bf16 before the activation (the unfused
 * reference's convention); 0 applies it to the f32 accumulator (tokamax fuse_act).
 * lhs_row_index (optional, device int32, m entries): the dispatch gather fused
 * into the operand load -- logical row r is row lhs_row_index[r] of lhs, which
 * then has lhs_src_rows rows (index -1 reads as zeros), so the sorted copy of
 * the tokens is never materialised.  NULL: lhs is read directly (m rows).
 * zero_tail as in lmoe_ragged_dot_bf16 (ignored when group_sizes is NULL).
 * Replaces PallasMosaicTpuV2RaggedDot()(..., fuse_gateup_activation="situ:b:lb")
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:610-723) and the
 * dense own kernel (05_ragged_dot_on_tpu/own_gateup_situ_pallas_kernel.py:79-199). */
LMOE_API int lmoe_gateup_situ_bf16(const void* lhs, const void* w_gateup, const int32_t* group_sizes,
                          void* out, int64_t m, int64_t k, int64_t intermediate,
                          int64_t num_groups, int rhs_layout, float beta, float linear_beta,
                          int round_gate_up, const int32_t* lhs_row_index,
                          int64_t lhs_src_rows, int zero_tail, int32_t* dev_status,
                          void* stream);

/* Grouped matmul against MXFP4 weights: e2m1 codes (g, n, k/2) uint8, low nibble
 * = even k, and one E8M0 scale byte per 32-element k block (g, n, k/32) -- the
 * checkpoint's (out, in) layout.  The weights stay packed in HBM; each tile is
 * expanded to bf16 in shared memory and multiplied on the tensor cores with f32
 * accumulation.  Result = lhs @ dequant(w)^T, exactly the dequant-then-matmul
 * of 05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67 (code 8 = -0.0, scale byte 0 =
 * 2^-127).  k a multiple of 64, n a multiple of 8; bf16 or f32 out.
 * lhs_f16 = 1: lhs holds f16 (bf16 values carried in f16, e.g. from
 * lmoe_gather_rows with convert = 1); the codes are then expanded with the
 * hardware e2m1 -> f16 conversion and the MMA runs on f16 operands, which needs
 * every scale byte in [104, 140] (weights of magnitude 2^-23 .. 2^13 x 6).
 * zero_tail as in lmoe_ragged_dot_bf16.
 * Replaces the MXFP4 dequant matmul
 * (05_ragged_dot_on_tpu/mxfp4_online_dequant_matmul_pallas.py:120-157). */
LMOE_API int lmoe_mxfp4_ragged_dot(const void* lhs, const void* weight_packed,
                                   const void* weight_scale, const int32_t* group_sizes, void* out,
                                   int64_t m, int64_t k, int64_t n, int64_t num_groups,
                                   int lhs_f16, int out_f32, int zero_tail, int32_t* dev_status,
                                   void* stream);

/* lmoe_mxfp4_ragged_dot with bf16 output rows stored at arbitrary addresses:
 * output row r (r < sum(group_sizes)) goes to the byte address row_dest[r]
 * (uint64 device array of m entries, each 16-byte aligned; a peer GPU's
 * mapped buffer included), rows past sum(group_sizes) are not written.  The
 * expert-parallel down projection uses it to write each result straight into
 * the exchange buffer of the rank the row came from.  Replaces the down
 * ragged_dot of KRD:367-369 followed by the scatter back of KR:413, in one
 * kernel. */
LMOE_API int lmoe_mxfp4_ragged_dot_scatter(const void* lhs, const void* weight_packed,
                                           const void* weight_scale, const int32_t* group_sizes,
                                           const uint64_t* row_dest, int64_t m, int64_t k,
                                           int64_t n, int64_t num_groups, int lhs_f16,
                                           int32_t* dev_status, void* stream);

/* Fused gate/up + SiTU-GLU against MXFP4 weights: the packed rows are
 * [gate (intermediate rows) | up (intermediate rows)] per group, i.e.
 * (g, 2*intermediate, k/2) codes and (g, 2*intermediate, k/32) scales (the
 * checkpoint's w1 and w3 stacked).  group_sizes NULL = one dense group.
 * lhs_f16 as above; out_f16 = 1 stores the bf16-rounded activation as f16
 * (the lhs of a following lhs_f16 down-projection); lhs_row_index /
 * lhs_src_rows fuse the dispatch gather and zero_tail behaves as in
 * lmoe_gateup_situ_bf16. */
LMOE_API int lmoe_mxfp4_gateup_situ(const void* lhs, const void* weight_packed,
                                    const void* weight_scale, const int32_t* group_sizes,
                                    void* out, int64_t m, int64_t k, int64_t intermediate,
                                    int64_t num_groups, float beta, float linear_beta,
                                    int round_gate_up, int lhs_f16, int out_f16,
                                    const int32_t* lhs_row_index, int64_t lhs_src_rows,
                                    int zero_tail, int32_t* dev_status, void* stream);

/* Grouped matmul against e4m3 (float8_e4m3fn) weights with block scales:
 *   out[r] = lhs[r] @ bf16(f32(rhs_q[g]) * rhs_scale[g][k / block_size])
 * rhs_q (g, k, n) e4m3 -- the reference's (G, K, N) layout; rhs_scale
 * (g, k / block_size, 1, n) f32 (one scale per column per K block; block_size
 * a multiple of 32 dividing k, or k itself).  lhs bf16 (m, k); bf16 or f32
 * out; the e4m3 tile is expanded to bf16 in shared memory (the dequantised
 * weight, bit for bit) and multiplied on the tensor cores with f32
 * accumulation.  k a multiple of 64, n a multiple of 16.  zero_tail as in
 * lmoe_ragged_dot_bf16.
 * Replaces PallasMosaicTpuV2RaggedDot()(lhs, rhs, group_sizes=..., rhs_scale=...,
 * maybe_quantize_lhs=False) (05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:2804-2811,
 * 2914-2921); its check compares against ragged_dot with the dequantised
 * bf16 weight (same file, 2815-2827, 2923-2934). */
LMOE_API int lmoe_fp8_ragged_dot(const void* lhs, const void* rhs_q, const float* rhs_scale,
                                 const int32_t* group_sizes, void* out, int64_t m, int64_t k,
                                 int64_t n, int64_t num_groups, int64_t block_size, int out_f32,
                                 int zero_tail, int32_t* dev_status, void* stream);

/* Elementwise SiTU-GLU: out = dtype(beta*tanh(g/beta)*sigmoid(g) * lb*tanh(u/lb)).
 * gate/up rows have pitch ld_in elements; bf16 = 1 for bf16 I/O, 0 for f32.
 * Replaces _situ_and_mul (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:296-310). */
LMOE_API int lmoe_situ_and_mul(const void* gate, const void* up, int64_t ld_in, void* out, int64_t rows,
                      int64_t intermediate, float beta, float linear_beta, int bf16, void* stream);

/* Router epilogue from f32 logits (T, E): sigmoid (or softmax), + bias for
 * selection only, top-k descending with ties to the lower expert id, gather of
 * the un-biased scores, renormalise (sum + 1e-20) when k > 1 and renormalize,
 * times routed_scaling_factor.  topk_idx (T, k) int32, topk_w (T, k) f32.
 * E <= 1024, k <= 32.  bias may be NULL.
 * Replaces the gate of latent_moe_forward
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-356, 601-631). */
LMOE_API int lmoe_router_topk(const float* logits, const float* bias, int64_t num_tokens,
                     int64_t num_experts, int64_t top_k, int activation, int renormalize,
                     float routed_scaling_factor, int32_t* topk_idx, float* topk_w, void* stream);

/* Workspace bytes lmoe_router_fused_bf16 needs (0 for unsupported shapes). */
LMOE_API size_t lmoe_router_fused_workspace_size(int64_t num_tokens, int64_t num_experts,
                                                 int64_t top_k);

/* Router gate straight from the hidden states, sigmoid activation: the logits
 * h @ W_router^T run on the tensor cores (bf16 products, f32 accumulation)
 * and the selection of lmoe_router_topk (activation 0) runs in the GEMM's
 * epilogue on the accumulator, so the f32 logits are never stored.  topk_idx
 * and topk_w equal lmoe_gemm_bf16(out f32) followed by lmoe_router_topk bit
 * for bit.  hidden (T, d) bf16, router_weight (E, d) bf16 (d contiguous, the
 * nn.Linear layout), bias (E,) f32 or NULL; d % 8 == 0, E <= 1024,
 * top_k <= 16, 16-byte aligned pointers.  workspace: device scratch of
 * lmoe_router_fused_workspace_size bytes (LMOE_SCRATCH_TOO_SMALL otherwise).
 * Replaces the gate of latent_moe_forward
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-356). */
LMOE_API int lmoe_router_fused_bf16(const void* hidden, const void* router_weight, const float* bias,
                           int64_t num_tokens, int64_t hidden_size, int64_t num_experts,
                           int64_t top_k, int renormalize, float routed_scaling_factor,
                           int32_t* topk_idx, float* topk_w, void* workspace,
                           size_t workspace_bytes, int32_t* dev_status, void* stream);

/* Workspace bytes lmoe_dense_input_phase needs (0 for unsupported shapes). */
LMOE_API size_t lmoe_dense_input_workspace_size(int64_t num_tokens, int64_t hidden_size,
                                                int64_t num_experts, int64_t latent_size,
                                                int64_t shared_intermediate);

/* The input phase of the layer for small token counts, one persistent split-K
 * kernel: the three projections of the hidden states in one launch --
 *   logits     = h @ W_router^T                       (T, E) f32
 *   latent_out = bf16(h @ W_down^T)                   (T, L) bf16
 *   shared_act = bf16(situ(bf16(h @ W_g^T), bf16(h @ W_u^T)))   (T, Is) bf16
 *                (round_gate_up 0: g and u unrounded)
 * with the SiTU-GLU of lmoe_gateup_situ_bf16 (beta, linear_beta).  hidden
 * (T, d) bf16; router_w (E, d), down_w (L, d) and shared_gu_w (2*Is, d) =
 * [gate rows | up rows] are bf16 with d contiguous (the nn.Linear layout).
 * The K steps of each 128-column tile are split over the SMs (a split count
 * that depends on the weight shapes and the SM count, not on T, so each
 * token's result is independent of T); the CTA that finishes a tile's last
 * split sums the f32 partials in split order.  d % 64 == 0, E % 4 == 0,
 * L and Is % 8 == 0, 16-byte aligned pointers (LMOE_UNSUPPORTED otherwise).
 * workspace: device scratch of lmoe_dense_input_workspace_size bytes,
 * 256-byte aligned (LMOE_SCRATCH_TOO_SMALL otherwise); calls that share a
 * workspace must not overlap on the GPU.  Replaces the router gate, the
 * down-projection and the shared expert's gate/up of latent_moe_forward
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-365, 428-433). */
LMOE_API int lmoe_dense_input_phase(const void* hidden, const void* router_w, const void* down_w,
                                    const void* shared_gu_w, float* logits, void* latent_out,
                                    void* shared_act, int64_t num_tokens, int64_t hidden_size,
                                    int64_t num_experts, int64_t latent_size,
                                    int64_t shared_intermediate, float beta, float linear_beta,
                                    int round_gate_up, void* workspace, size_t workspace_bytes,
                                    int32_t* dev_status, void* stream);

/* Workspace bytes lmoe_dense_output_phase needs (0 for unsupported shapes). */
LMOE_API size_t lmoe_dense_output_workspace_size(int64_t num_tokens, int64_t latent_size,
                                                 int64_t shared_intermediate, int64_t hidden_size);

/* The output phase of the layer for small token counts, one persistent split-K
 * kernel over two K segments:
 *   out = bf16(normed @ W_up^T + shared_act @ W_sd^T)       (T, d) bf16
 * i.e. the up-projection, the shared expert's down projection and the output
 * sum with one rounding of the f32 sum (the reference rounds each branch to
 * bf16 before adding: the results differ by at most about one bf16 spacing of
 * the output).  normed (T, L), shared_act (T, Is) bf16; up_w (d, L) and
 * shared_down_w (d, Is) bf16 with K contiguous.  L and Is % 64 == 0,
 * d % 8 == 0, 16-byte aligned pointers; workspace as for the input phase.
 * Replaces the up-projection, the shared expert's output and the sum of
 * latent_moe_forward (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:419-435). */
LMOE_API int lmoe_dense_output_phase(const void* normed, const void* up_w, const void* shared_act,
                                     const void* shared_down_w, void* out, int64_t num_tokens,
                                     int64_t latent_size, int64_t shared_intermediate,
                                     int64_t hidden_size, void* workspace, size_t workspace_bytes,
                                     int32_t* dev_status, void* stream);

/* Workspace bytes lmoe_dispatch needs for max(num_tokens*top_k, m_out) entries. */
LMOE_API size_t lmoe_dispatch_workspace_size(int64_t num_entries, int64_t num_local_experts);

/* Dispatch metadata: stable counting sort of the flattened (token, slot)
 * entries by local expert id.  Entries whose expert is outside
 * [expert_start, expert_start + num_local_experts) (and padding entries up to
 * m_out) sort after every real entry; the first m_out sorted positions are kept
 * (tail drop on overflow).
 *   full dropless dispatch:   expert_start 0, num_local_experts E, m_out T*k, pad_bucket 0
 *                             -> order = argsort(flat_ids, stable), group_sizes = bincount
 *                             (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:370-378)
 *   shard, capacity padded:   m_out = m_padded, pad_bucket 1 -> group_sizes has
 *                             num_local_experts + 1 entries, the last one the
 *                             padding bucket (kimi_k3_latent_moe_reference.py:754-877)
 * Outputs (device; NULL to skip where marked optional):
 *   order[m_out]        (optional) flat entry index at each sorted position
 *   token_idx[m_out]    source token, -1 for padding positions
 *   weight[m_out]       (optional) topk_w of the entry, 0 for padding
 *   slot_pos[T*k]       (optional) sorted position of each entry, -1 if not kept
 *   group_sizes[...]    kept count per local expert (+ padding bucket)
 *   per_expert_counts   (optional) kept count per local expert
 *   valid[m_out]        (optional) 1 for real rows, 0 for padding
 * topk_w may be NULL (weights then read as 0).  num_local_experts <= 2048. */
LMOE_API int lmoe_dispatch(const int32_t* topk_idx, const float* topk_w, int64_t num_tokens,
                  int64_t top_k, int64_t expert_start, int64_t num_local_experts, int64_t m_out,
                  int pad_bucket, int32_t* order, int32_t* token_idx, float* weight,
                  int32_t* slot_pos, int32_t* group_sizes, int32_t* per_expert_counts,
                  uint8_t* valid, void* workspace, size_t workspace_bytes, void* stream);

/* lmoe_dispatch without a workspace argument, for callers that cannot allocate
 * device memory where they dispatch (a framework that owns the whole memory
 * pool, or a latency-critical loop that must not call cudaMalloc, which can
 * block on the device).  Same arguments and outputs as lmoe_dispatch minus the
 * workspace; the scratch is a fixed ~2.1 MB array inside the library, one per
 * device, resident until the process exits.  Limit: max(num_tokens*top_k, m_out)
 * <= 262144 and num_local_experts <= 2048, else LMOE_SCRATCH_TOO_SMALL with no
 * launch.  All calls on a device share the array: calls that overlap on the
 * GPU race and must be ordered.  The first call on each device looks up the
 * array's address; make it before any stream capture.
 * No counterpart in the reference. */
LMOE_API int lmoe_dispatch_static_scratch(const int32_t* topk_idx, const float* topk_w,
                                          int64_t num_tokens, int64_t top_k,
                                          int64_t expert_start, int64_t num_local_experts,
                                          int64_t m_out, int pad_bucket, int32_t* order,
                                          int32_t* token_idx, float* weight, int32_t* slot_pos,
                                          int32_t* group_sizes, int32_t* per_expert_counts,
                                          uint8_t* valid, void* stream);

/* Row gather: out[p] = token_idx[p] >= 0 ? x[token_idx[p]] : 0, rows of row_bytes
 * (a multiple of 16).  convert = 1 reads bf16 rows and writes them as f16
 * (exact in f16's normal range), the lhs_f16 form of the MXFP4 kernels; a
 * value above 65504 in magnitude becomes inf there and records LMOE_F16_RANGE
 * in dev_status (may be NULL).
 * Replaces `x[sorted_token_idx]` / `where(valid, x[idx], 0)`
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:372-374, 867-868). */
LMOE_API int lmoe_gather_rows(const void* x, int64_t x_rows, const int32_t* token_idx, void* out,
                              int64_t rows, int64_t row_bytes, int convert, int32_t* dev_status,
                              void* stream);

/* The gather in token order: out[slot_pos[t*k + s]] = x[t] for every token t
 * and slot s with slot_pos >= 0 (rows of row_bytes; convert as in
 * lmoe_gather_rows).  Each source row is read (and converted) once and
 * stored k times; rows that no slot points at are left untouched, so for a
 * dropless dispatch (every sorted position is some slot's) the output equals
 * lmoe_gather_rows(x, token_idx) bit for bit.  A position >= out_rows is
 * skipped and records LMOE_DEVICE_BOUNDS.  top_k <= 32.
 * Replaces `x[sorted_token_idx]` of the dropless forward
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:372-374). */
LMOE_API int lmoe_scatter_rows(const void* x, const int32_t* slot_pos, int64_t num_tokens,
                               int64_t top_k, void* out, int64_t out_rows, int64_t row_bytes,
                               int convert, int32_t* dev_status, void* stream);

/* Weighted combine + RMSNorm:
 *   routed[t] = dtype(sum_s expert_out[slot_pos[t*k+s]] * topk_w[t,s])   (f32, slot order)
 *   normed[t] = dtype(dtype(routed[t] / sqrt(mean(routed[t]^2) + eps)) * norm_scale)
 * slot_pos < 0 contributes nothing.  routed_out / normed_out may be NULL.
 * Replaces kimi_k3_latent_moe_reference.py:413-419 and _rms_norm (286-293). */
LMOE_API int lmoe_combine_rmsnorm(const void* expert_out, const int32_t* slot_pos, const float* topk_w,
                         const void* norm_scale, int64_t num_tokens, int64_t top_k,
                         int64_t latent, float eps, int bf16, void* routed_out, void* normed_out,
                         void* stream);

/* Expert-parallel receive-side reordering.  After the payload all-to-all the
 * rows are grouped by source rank, each source block ordered by local expert;
 * recv_counts (world, num_local_experts) int32 device holds the per-(source,
 * expert) row counts.  Writes em_src[p] (received row feeding expert-major
 * position p), its inverse sm_src[q], and group_sizes (num_local_experts) for
 * the grouped GEMMs.  rows_cap bounds the number of rows written.
 * No counterpart in the reference, which only simulates expert shards in one
 * process (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:1531-1674). */
LMOE_API int lmoe_ep_reorder(const int32_t* recv_counts, int64_t world, int64_t num_local_experts,
                             int64_t rows_cap, int32_t* em_src, int32_t* sm_src,
                             int32_t* group_sizes, void* stream);

/* Expert-parallel exchange over NVLink peer memory (one process per GPU).
 * peers_dev is a device array of `world` pointers to every rank's symmetric
 * buffer of lmoe_ep_buffer_bytes(...) bytes (same layout on every rank; index
 * `rank` = this rank's own buffer).  Each counts exchange advances an epoch
 * word kept in the buffer itself (every rank runs the same exchanges, so the
 * epochs agree; the calls are capturable in a CUDA graph).  Rank r owns
 * global experts [r*E/world, (r+1)*E/world).  Sequence per forward:
 *   lmoe_ep_exchange_counts  publish this rank's per-expert row counts
 *                            (group_sizes, E int32, from lmoe_dispatch over all E
 *                            experts) to every peer, wait for all, write
 *                            local_group_sizes (E/world int32)
 *   lmoe_ep_dispatch_put     copy row x[token_idx[p]] of every dispatched row p
 *                            straight into its owner's receive region, expert-major,
 *                            then wait until every source's rows have landed here
 *   (grouped GEMMs on the receive region, group sizes local_group_sizes)
 *   lmoe_ep_return_put       copy each output row back into its source's return
 *                            region at the row's original dispatch position, then
 *                            wait for this rank's rows to come back
 * Offsets are computed on the device from the exchanged counts: no host
 * synchronisation.  Waits are bounded (LMOE_WAIT_TIMEOUT in dev_status).
 * Region byte offsets within the buffer: lmoe_ep_region_offset (0 receive,
 * 1 return, 2 counts).  No counterpart in the reference (its expert shards are
 * simulated in one process, 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:1531-1674). */
LMOE_API int64_t lmoe_ep_buffer_bytes(int64_t world, int64_t num_experts,
                                      int64_t recv_capacity_rows, int64_t back_capacity_rows,
                                      int64_t row_bytes);
/* Limit, in nanoseconds, of every device-side wait on another rank's signal
 * (counts, rows, returns) in the exchange calls enqueued (or captured into a
 * CUDA graph) after this call; 0 restores the default of 2 s.  Accepted range
 * 1 us .. 60 s (LMOE_BAD_SHAPE otherwise).  A wait that runs out records
 * LMOE_WAIT_TIMEOUT in dev_status, empties the offset tables (so the puts and
 * the expert GEMMs that follow do no work) and returns; the CUDA context stays
 * usable.  Process-wide setting.  lmoe_peer_wait_timeout_ns reads it back.
 * No counterpart in the reference (it has no cross-device waits). */
LMOE_API int lmoe_set_peer_wait_timeout_ns(uint64_t ns);
LMOE_API uint64_t lmoe_peer_wait_timeout_ns(void);
/* The exchange buffer and its peer mappings, over CUDA IPC on the current
 * device (plain point-to-point peer mappings): lmoe_ep_buffer_alloc
 * allocates and zeroes `bytes`, returning the pointer and an IPC handle of
 * LMOE_EP_IPC_HANDLE_BYTES bytes to send to every peer; lmoe_ep_buffer_open
 * maps a peer's handle; close / free undo them (after every rank is done with
 * the exchange). */
#define LMOE_EP_IPC_HANDLE_BYTES 64
LMOE_API int lmoe_ep_buffer_alloc(int64_t bytes, void** buffer, void* ipc_handle);
LMOE_API int lmoe_ep_buffer_open(const void* ipc_handle, void** peer_buffer);
LMOE_API int lmoe_ep_buffer_close(void* peer_buffer);
LMOE_API int lmoe_ep_buffer_free(void* buffer);
LMOE_API int64_t lmoe_ep_region_offset(int64_t world, int64_t num_experts,
                                       int64_t recv_capacity_rows, int64_t back_capacity_rows,
                                       int64_t row_bytes, int region);
LMOE_API int lmoe_ep_exchange_counts(void* const* peers_dev, int64_t rank, int64_t world,
                                     int64_t num_experts, int64_t recv_capacity_rows,
                                     int64_t back_capacity_rows, int64_t row_bytes,
                                     const int32_t* group_sizes,
                                     int32_t* local_group_sizes, int32_t* dev_status,
                                     void* stream);
LMOE_API int lmoe_ep_dispatch_put(void* const* peers_dev, int64_t rank, int64_t world,
                                  int64_t num_experts, int64_t recv_capacity_rows,
                                  int64_t back_capacity_rows, int64_t row_bytes,
                                  const void* x, int64_t x_rows, const int32_t* token_idx,
                                  int64_t num_routed_rows, int32_t* dev_status, void* stream);
LMOE_API int lmoe_ep_return_put(void* const* peers_dev, int64_t rank, int64_t world,
                                int64_t num_experts, int64_t recv_capacity_rows,
                                int64_t back_capacity_rows, int64_t row_bytes,
                                const void* y, int64_t num_rows, int32_t* dev_status,
                                void* stream);

/* The fused return (an alternative to lmoe_ep_return_put): after
 * lmoe_ep_dispatch_put, lmoe_ep_return_destinations writes, for each of the
 * first num_rows received (expert-major) rows, the byte address in its source
 * rank's return region where that row's result belongs (uint64 device array);
 * the down-projection GEMM then stores its output rows there directly
 * (lmoe_mxfp4_ragged_dot_scatter), over NVLink, while it runs; and
 * lmoe_ep_return_signal tells every source this rank's rows are in place and
 * waits (bounded) until every rank's rows for this rank have arrived.  No
 * counterpart in the reference (see above). */
LMOE_API int lmoe_ep_return_destinations(void* const* peers_dev, int64_t rank, int64_t world,
                                         int64_t num_experts, int64_t recv_capacity_rows,
                                         int64_t back_capacity_rows, int64_t row_bytes,
                                         uint64_t* row_dest, int64_t num_rows,
                                         int32_t* dev_status, void* stream);
LMOE_API int lmoe_ep_return_signal(void* const* peers_dev, int64_t rank, int64_t world,
                                   int64_t num_experts, int64_t recv_capacity_rows,
                                   int64_t back_capacity_rows, int64_t row_bytes,
                                   int32_t* dev_status, void* stream);

/* Block-scaled fast path: MXFP8 activations x MXFP4 weights on
 * tcgen05.mma kind::mxf8f6f4.block_scale (opt-in; the activations are
 * rounded to e4m3 with one E8M0 scale per 32 K values, so results differ
 * from the exact MXFP4 path by that rounding, ~3% normwise on N(0,1) rows).
 * Activation rows live in a padded layout: every group's rows start at a
 * multiple of 128 (lmoe_mxfp8_padded_rows gives the capacity for num_rows
 * rows in num_groups groups); scale factors live in 512-byte atoms of 128
 * rows x 4 K blocks (byte r0*16 + r1*4 + kb for row r0 + 32*r1), the layout
 * the tensor core's scale copies read.
 * The reference's operator has the hook for quantising the activations
 * (`maybe_quantize_lhs`, 05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:257-263)
 * but never uses it; its MXFP4 weights are dequantised first
 * (05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67). */
LMOE_API int64_t lmoe_mxfp8_padded_rows(int64_t num_rows, int64_t num_groups);
/* One-time weight preparation: MXFP4 codes (g, n, k/2) + E8M0 scales (g, n,
 * k/32) -> scale atoms (g, n/128, k/128, 512) and, with interleave_gateup = 1
 * (a fused [gate | up] weight of n = 2I rows), the codes with gate/up rows
 * interleaved (row 2i = gate i, 2i+1 = up i; out_packed, same size);
 * interleave_gateup = 0 leaves the codes as they are (out_packed unused). */
LMOE_API int lmoe_mxfp4_repack_blockscaled(const void* weight_packed, const void* weight_scale,
                                           int64_t g, int64_t n, int64_t k, int interleave_gateup,
                                           void* out_packed, void* out_sf, void* stream);
/* Quantise rows to MXFP8: row p of the output is x[token_idx[p]] (token_idx
 * NULL: x[p]; an index < 0 gives a zero row), stored at its padded position
 * (group_sizes NULL: position p) as e4m3 (out_q, m_pad_capacity x k bytes)
 * with its scales in atoms (out_sf, k/128 x m_pad_capacity/128 x 512: K-step
 * major, so the atoms of consecutive row blocks are adjacent).  x is
 * bf16 (x_f16 = 0) or f16.  k a multiple of 128. */
LMOE_API int lmoe_mxfp8_quantize_rows(const void* x, int64_t x_rows, int x_f16,
                                      const int32_t* token_idx, const int32_t* group_sizes,
                                      int64_t num_groups, int64_t rows, int64_t k, void* out_q,
                                      void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                      void* stream);
/* The same in token order for a dropless dispatch: token t's row x[t] is
 * quantised once and stored at the padded position of each of its sorted
 * positions slot_pos[t*top_k + s] (the rows lmoe_mxfp8_quantize_rows writes
 * with token_idx the dispatch's, bit for bit).  Padding rows are left
 * untouched; a destination past m_pad_capacity is skipped and records
 * LMOE_DEVICE_BOUNDS.  top_k <= 32, k a multiple of 128, group_sizes required. */
LMOE_API int lmoe_mxfp8_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                         int64_t num_tokens, int64_t top_k, int64_t k,
                                         const int32_t* group_sizes, int64_t num_groups,
                                         void* out_q, void* out_sf, int64_t m_pad_capacity,
                                         int32_t* dev_status, void* stream);
/* positions (n int32, sorted-order rows; < 0 passes through as -1) -> their
 * padded positions (the slot positions the combine reads the padded expert
 * outputs with). */
LMOE_API int lmoe_mxfp8_pad_positions(const int32_t* positions, int64_t n,
                                      const int32_t* group_sizes, int64_t num_groups, int32_t* out,
                                      void* stream);
/* Grouped GEMM of padded MXFP8 rows against prepared MXFP4 weights:
 *   epi 0: out[r] = act[r] @ W[g]^T, out_dtype 0 bf16 / 1 f32 / 2 f16 (bf16 values)
 *   epi 3: SiTU-GLU over interleaved gate/up rows (n_out = intermediate size),
 *          out_dtype 0 bf16 / 2 f16; beta, linear_beta, round_gate_up as in
 *          lmoe_gateup_situ_bf16
 * Output rows are the padded rows (out has m_pad rows); only each group's
 * first group_sizes[g] rows are written.  g <= 1024.  Replaces the quantised
 * form of PallasMosaicTpuV2RaggedDot (kimi_k3_latent_moe_ragged_dot.py:2714-2953)
 * for MXFP4 weights with MXFP8 activations. */
LMOE_API int lmoe_mxfp8_mxfp4_grouped_gemm(const void* act_q, const void* act_sf,
                                           const void* w_packed, const void* w_sf,
                                           const int32_t* group_sizes, void* out, int64_t m_pad,
                                           int64_t k, int64_t n_out, int64_t g, int epi,
                                           float beta, float linear_beta, int round_gate_up,
                                           int out_dtype, int32_t* dev_status, void* stream);

/* The MXFP4-activation form of the same path (kind::mxf4 on the tensor core,
 * both operands e2m1, twice the MMA rate of the MXFP8 form and half its
 * activation bytes, at a larger rounding error: ~10% normwise on N(0,1) rows).
 * Rows are quantised to MXFP4: e2m1 values (two per byte, the even K index in
 * the low nibble, out_q m_pad_capacity x k/2 bytes), one E8M0 scale per 32 K
 * values, the smallest power of two 2^e with amax <= 6 * 2^e, values rounded
 * to nearest even; the padded layout and the scale atoms are those of the
 * MXFP8 functions.  Same arguments and errors as lmoe_mxfp8_quantize_rows /
 * lmoe_mxfp8_quantize_scatter. */
LMOE_API int lmoe_mxfp4_quantize_rows(const void* x, int64_t x_rows, int x_f16,
                                      const int32_t* token_idx, const int32_t* group_sizes,
                                      int64_t num_groups, int64_t rows, int64_t k, void* out_q,
                                      void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                      void* stream);
LMOE_API int lmoe_mxfp4_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                         int64_t num_tokens, int64_t top_k, int64_t k,
                                         const int32_t* group_sizes, int64_t num_groups,
                                         void* out_q, void* out_sf, int64_t m_pad_capacity,
                                         int32_t* dev_status, void* stream);
/* The exact MXFP4 matmul on the block-scaled tensor core: bf16/f16 rows split
 * into two e4m3 planes under one E8M0 scale per 32 K values (the MXFP8 scale
 * rule): hi = e4m3(x / 2^e), lo = e4m3(x / 2^e - hi), both rounded to nearest
 * even.  hi + lo holds every bf16 value with |x| >= 2^-2 of its block's scale
 * unit exactly (smaller ones to within 2^-10 of that unit), so the GEMM below
 * multiplies the activations themselves: ~1e-6 normwise from the
 * dequant-then-matmul result, at the MXFP8 MMA rate and with no weight
 * expansion.  out_q holds 2 x m_pad_capacity x k bytes (plane hi, then lo);
 * otherwise the arguments, layouts and errors of lmoe_mxfp8_quantize_rows /
 * lmoe_mxfp8_quantize_scatter. */
LMOE_API int lmoe_bf16split_quantize_rows(const void* x, int64_t x_rows, int x_f16,
                                          const int32_t* token_idx, const int32_t* group_sizes,
                                          int64_t num_groups, int64_t rows, int64_t k,
                                          void* out_q, void* out_sf, int64_t m_pad_capacity,
                                          int32_t* dev_status, void* stream);
LMOE_API int lmoe_bf16split_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                             int64_t num_tokens, int64_t top_k, int64_t k,
                                             const int32_t* group_sizes, int64_t num_groups,
                                             void* out_q, void* out_sf, int64_t m_pad_capacity,
                                             int32_t* dev_status, void* stream);
/* lmoe_bf16split_quantize_scatter that also writes, for every slot s of every
 * token t, padded_slot_pos[t * top_k + s] = the slot's row in the padded
 * layout (-1 where the slot has none): the output of lmoe_mxfp8_pad_positions
 * on slot_pos, produced by the gather that already computes it, so the combine
 * after the padded GEMMs needs no separate kernel.  padded_slot_pos: device
 * int32 [num_tokens * top_k].  Replaces, with the split rows' GEMMs, the
 * gather and scatter-back positions of latent_moe_forward
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:370-378, 413). */
LMOE_API int lmoe_bf16split_quantize_scatter_positions(const void* x, int x_f16,
                                                       const int32_t* slot_pos,
                                                       int64_t num_tokens, int64_t top_k,
                                                       int64_t k, const int32_t* group_sizes,
                                                       int64_t num_groups, void* out_q,
                                                       void* out_sf, int64_t m_pad_capacity,
                                                       int32_t* padded_slot_pos,
                                                       int32_t* dev_status, void* stream);
/* The block-scaled gate/up + SiTU-GLU GEMM with its activations written
 * quantised for the down GEMM (no bf16 activation tensor): input rows of
 * act_kind 0 (MXFP8), 1 (MXFP4, k a multiple of 256) or 2 (split), weights
 * prepared with interleave_gateup = 1 (n = 2 * inter); the SiTU output of
 * each padded row (rounded to bf16) is quantised per 32 features to out_fmt 0
 * (MXFP8), 1 (MXFP4, inter a multiple of 256) or 2 (split; out_q 2 x m_pad x
 * inter bytes) with the scale rule of the matching quantise function, codes
 * at the same padded rows of out_q, scale atoms (inter/128, m_pad/128, 512)
 * to out_sf: the bytes that quantising the bf16 activations would give.
 * inter a multiple of 128. */
LMOE_API int lmoe_blockscaled_gateup_situ_quantized(const void* act_q, const void* act_sf,
                                                    int act_kind, const void* w_packed,
                                                    const void* w_sf, const int32_t* group_sizes,
                                                    int64_t m_pad, int64_t k, int64_t inter,
                                                    int64_t g, float beta, float linear_beta,
                                                    int round_gate_up, int out_fmt, void* out_q,
                                                    void* out_sf, int32_t* dev_status,
                                                    void* stream);
/* Grouped GEMM of split rows against prepared MXFP4 weights: arguments as
 * lmoe_mxfp8_mxfp4_grouped_gemm, plus m_out: 0 writes the padded rows (out
 * has m_pad rows); m_out > 0 writes row r of group g at its unpadded position
 * (the sum of the earlier groups' sizes + r; out has m_out rows, those at or
 * past sum(group_sizes) are zeroed) -- the ragged_dot output layout.  m_out < 0:
 * the same with -m_out rows and the rows past sum(group_sizes) left
 * unwritten (an output sized by capacity, such as an expert-parallel receive
 * region). */
LMOE_API int lmoe_bf16split_mxfp4_grouped_gemm(const void* act_q, const void* act_sf,
                                               const void* w_packed, const void* w_sf,
                                               const int32_t* group_sizes, void* out,
                                               int64_t m_pad, int64_t k, int64_t n_out, int64_t g,
                                               int epi, float beta, float linear_beta,
                                               int round_gate_up, int out_dtype, int64_t m_out,
                                               int32_t* dev_status, void* stream);
/* Grouped GEMM of padded MXFP4 rows against prepared MXFP4 weights; arguments
 * as lmoe_mxfp8_mxfp4_grouped_gemm, k a multiple of 256. */
LMOE_API int lmoe_mxfp4_mxfp4_grouped_gemm(const void* act_q, const void* act_sf,
                                           const void* w_packed, const void* w_sf,
                                           const int32_t* group_sizes, void* out, int64_t m_pad,
                                           int64_t k, int64_t n_out, int64_t g, int epi,
                                           float beta, float linear_beta, int round_gate_up,
                                           int out_dtype, int32_t* dev_status, void* stream);

/* Scatter-add combine of one expert shard:
 *   routed[idx[p]] += dtype(shard_out[p] * w[p])   for idx[p] >= 0
 * Replaces _combine_shard_contribution
 * (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:1113-1141). */
LMOE_API int lmoe_combine_scatter_add(const void* shard_out, const int32_t* padded_token_idx,
                             const float* padded_combine_weight, void* routed_out, int64_t rows,
                             int64_t latent, int64_t num_tokens, int bf16, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LMOE_H_ */
