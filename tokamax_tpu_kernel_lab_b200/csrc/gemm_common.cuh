// Shared pieces of the tcgen05 grouped GEMM kernels: argument block, the
// in-CTA tile schedule over device-resident group sizes, and the MXFP4 code
// expansion helpers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace lmoe {

constexpr int kBK = 64;
constexpr int kMaxGroups = 2048;
// the weights-major MXFP4 kernel keeps its schedule in shared memory for up
// to this many groups; more groups take the token-major kernel
constexpr int kSwapMaxGroups = 1536;

enum EpiKind { EPI_BF16 = 0, EPI_F32 = 1, EPI_BF16_ADD = 2, EPI_SITU = 3 };
// B_MXFP4F16: the same packed MXFP4 weights, but the activations arrive as f16
// (bf16 values, which convert to f16 exactly in f16's normal range) and the
// codes are expanded with the hardware e2m1x2 -> f16x2 conversion; the UMMA
// runs kind::f16 with f16 operands.  The f16 scale 2^(s-127) and every scaled
// code stay exact for scale bytes in [104, 140] (the caller checks the range).
// B_FP8: e4m3 weights in the reference's (G, K, N) layout with one f32 scale
// per (group, K block, column), expanded to bf16 (the dequantised weight
// bf16(q * scale)) into the MN-major UMMA operand.
enum BFmt { B_KMAJOR = 0, B_NMAJOR = 1, B_MXFP4 = 2, B_MXFP4F16 = 3, B_FP8 = 4 };

__host__ __device__ constexpr bool is_mx(int bf) { return bf == B_MXFP4 || bf == B_MXFP4F16; }
// formats whose B operand is expanded in shared memory by dequant warps
__host__ __device__ constexpr bool is_expand(int bf) { return is_mx(bf) || bf == B_FP8; }

struct GemmArgs {
  const int32_t* group_sizes;  // nullptr: a single group of M rows
  int32_t* status;
  void* out;
  const __nv_bfloat16* addend;  // EPI_BF16_ADD
  const uint8_t* scales;        // B_MXFP4: (G, n_weight, K/32) E8M0 bytes
  int64_t ldo;                  // output row pitch, elements
  int64_t ld_add;               // addend row pitch, elements
  int M, N, K, G;               // N = output columns (EPI_SITU: the intermediate size I)
  int n_tiles;                  // ceil(N / output tile width)
  int up_offset;                // EPI_SITU: row/col offset of the up half in the fused weight
  int n_weight;                 // rows (N extent) of one group's weight
  float beta, linear_beta, inv_beta, inv_linear_beta;
  int round_gate_up;
  int zero_tail;
  int out_f16;  // EPI_BF16 / EPI_SITU: store the bf16-rounded value as f16
  // Row gather of the A operand: logical row r of lhs is source row a_rows[r]
  // of the tensor map (a_src_rows rows); -1 reads as zeros.  nullptr: A is
  // read directly (row r of the map).
  const int32_t* a_rows;
  int a_src_rows;
  // B_FP8: f32 scales (G, n_blocks, N) at `scales`, one per block_size rows of K
  int block_size, n_blocks;
  // weights-major MXFP4 kernel, plain epilogue: when set, output row r is
  // stored at the byte address row_dest[r] (any address the GPU can write, a
  // peer GPU's buffer included) instead of out + r * ldo
  const uint64_t* row_dest;
};

// Shared-memory pipeline.  bf16 B: STAGES load stages of [A | B].  MXFP4 B:
// STAGES load stages of [A | packed B] (24 KB, so the ring is deep enough to
// hide TMA latency) and a separate ring of kDStages expanded bf16/f16 B
// tiles written by the dequant warps.
// In-CTA schedule: row_off[g] = sum(gs[:g]), tile_start[g] = sum(tiles[:g]).
// Returns the total tile count, or -1 when group_sizes is invalid.
template <int TM>
__device__ int build_schedule(const GemmArgs& a, int32_t* row_off, int32_t* tile_start,
                              int32_t* scan_rows, int32_t* scan_tiles) {
  const int G = a.G;
  const int nthr = blockDim.x;
  const int per = (G + nthr - 1) / nthr;
  const int g0 = min(G, static_cast<int>(threadIdx.x) * per);
  const int g1 = min(G, g0 + per);
  long long rows = 0, tiles = 0;
  int bad = 0;
  for (int g = g0; g < g1; ++g) {
    const int s = a.group_sizes ? __ldg(a.group_sizes + g) : a.M;
    if (s < 0) bad = 1;
    const int ss = max(s, 0);
    rows += ss;
    tiles += static_cast<long long>((ss + TM - 1) / TM) * a.n_tiles;
  }
  scan_rows[threadIdx.x] = bad ? -1 : static_cast<int32_t>(min(rows, (long long)INT32_MAX));
  scan_tiles[threadIdx.x] = static_cast<int32_t>(min(tiles, (long long)INT32_MAX));
  __syncthreads();
  __shared__ int s_total;
  if (threadIdx.x == 0) {
    long long r = 0, t = 0;
    int invalid = 0;
    for (int i = 0; i < nthr; ++i) {
      const int rr = scan_rows[i];
      const int tt = scan_tiles[i];
      if (rr < 0) invalid = 1;
      scan_rows[i] = static_cast<int32_t>(r);
      scan_tiles[i] = static_cast<int32_t>(t);
      r += max(rr, 0);
      t += tt;
    }
    if (invalid || r > a.M || t > INT32_MAX) {
      record_status(a.status, kDeviceBounds);
      s_total = -1;
    } else {
      s_total = static_cast<int>(t);
      row_off[G] = static_cast<int32_t>(r);
      tile_start[G] = static_cast<int32_t>(t);
    }
  }
  __syncthreads();
  if (s_total >= 0) {
    int r = scan_rows[threadIdx.x];
    int t = scan_tiles[threadIdx.x];
    for (int g = g0; g < g1; ++g) {
      row_off[g] = r;
      tile_start[g] = t;
      const int s = a.group_sizes ? __ldg(a.group_sizes + g) : a.M;
      r += s;
      t += ((s + TM - 1) / TM) * a.n_tiles;
    }
  }
  __syncthreads();
  return s_total;
}

// last g with tile_start[g] <= t (groups with no tiles are skipped naturally)
__device__ __forceinline__ int find_group(const int32_t* tile_start, int G, int t) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct TileCoord {
  int g, m_tile, n_tile, row0, row_end;
};

template <int TM>
__device__ __forceinline__ TileCoord decode_tile(const int32_t* tile_start, const int32_t* row_off,
                                                 int G, int n_tiles, int t) {
  TileCoord c;
  c.g = find_group(tile_start, G, t);
  const int local = t - tile_start[c.g];
  c.m_tile = local / n_tiles;
  c.n_tile = local - c.m_tile * n_tiles;
  c.row0 = row_off[c.g] + c.m_tile * TM;
  c.row_end = row_off[c.g + 1];
  return c;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// 8 e2m1 codes (one u32, low nibble first) -> 8 bf16 (uint4), times 2^(s-127).
// Magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} are looked up bytewise with prmt
// (high and low byte tables), the code's bit 3 becomes the bf16 sign bit (so
// code 8 gives -0.0), and the power-of-two scale is one exact bf16x2 multiply.
__device__ __forceinline__ uint4 dequant_e2m1x8(uint32_t x, __nv_bfloat162 scale2) {
  const uint32_t sel = x & 0x77777777u;
  const uint32_t kHi0 = 0x3F3F3F00u, kHi1 = 0x40404040u;
  const uint32_t kLo0 = 0xC0800000u, kLo1 = 0xC0804000u;
  const uint32_t hi_a = prmt(kHi0, kHi1, sel & 0xFFFFu), hi_b = prmt(kHi0, kHi1, sel >> 16);
  const uint32_t lo_a = prmt(kLo0, kLo1, sel & 0xFFFFu), lo_b = prmt(kLo0, kLo1, sel >> 16);
  uint32_t w0 = prmt(lo_a, hi_a, 0x5140u), w1 = prmt(lo_a, hi_a, 0x7362u);
  uint32_t w2 = prmt(lo_b, hi_b, 0x5140u), w3 = prmt(lo_b, hi_b, 0x7362u);
  w0 |= ((x << 12) & 0x00008000u) | ((x << 24) & 0x80000000u);
  w1 |= ((x << 4) & 0x00008000u) | ((x << 16) & 0x80000000u);
  w2 |= ((x >> 4) & 0x00008000u) | ((x << 8) & 0x80000000u);
  w3 |= ((x >> 12) & 0x00008000u) | (x & 0x80000000u);
  uint32_t r[4] = {w0, w1, w2, w3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&r[i]);
    v = __hmul2(v, scale2);
    r[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// bf16 bit pattern of 2^(s-127) for an E8M0 byte s (s = 0 -> 2^-127, subnormal)
__device__ __forceinline__ uint32_t e8m0_to_bf16_bits(uint32_t s) {
  return s == 0 ? 0x0040u : (s << 7);
}

// f16 bit pattern of 2^(s-127), exact for s in [103, 142] (subnormal below 113)
__device__ __forceinline__ uint32_t e8m0_to_f16_bits(uint32_t s) {
  const int e = static_cast<int>(s) - 127;
  return e >= -14 ? static_cast<uint32_t>(e + 15) << 10 : 1u << (e + 24);
}

// 8 e2m1 codes -> 8 f16 (uint4) with the hardware conversion (low nibble ->
// low half), times the f16x2 scale (an exact power of two).
__device__ __forceinline__ uint4 dequant_e2m1x8_f16(uint32_t x, uint32_t scale2) {
  uint32_t r[4];
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(x));
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(r[i]) : "r"(scale2));
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// bf16-rounded value stored as f16 (exact for |v| in f16's normal range)
__device__ __forceinline__ uint32_t pack_f16x2_of_bf16(float lo, float hi) {
  const __half2 v = __floats2half2_rn(bf16_round_f(lo), bf16_round_f(hi));
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Weights-major MXFP4 grouped GEMM (mxfp4_swap.cu): lhs (a.M, a.K) tokens,
// packed (a.G, a.n_weight, a.K/2) codes; epilogue EPI_BF16, EPI_F32 or
// EPI_SITU.  The caller validates shapes; n_tiles is derived inside.
int mxfp4_swap_gemm(const void* lhs, const void* packed, GemmArgs a, int epi, int lhs_f16,
                    cudaStream_t stream);

// The same on CTA pairs (mxfp4_pair.cu): one MMA over two SMs, 256 weight
// rows x 256 tokens per pair tile, each SM staging half of the tokens.
int mxfp4_pair_gemm(const void* lhs, const void* packed, GemmArgs a, int epi, int lhs_f16,
                    cudaStream_t stream);

}  // namespace lmoe
