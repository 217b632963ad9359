// Block-scaled paths: MXFP4 weights on the block-scaled tensor core
// (tcgen05.mma kind::mxf8f6f4.block_scale / kind::mxf4.block_scale).
//
// The exact MXFP4 kernels (mxfp4_swap.cu) expand every weight tile to f16 or
// bf16 in shared memory and multiply on kind::f16.  These kernels instead
// feed the e2m1 codes to the tensor core as they are, with their E8M0 block
// scales in tensor memory, against activations quantised per 32 K values
// under one E8M0 scale each (the MMA kinds below):
//   MXFP8 rows   e4m3 (scale: the smallest power of two that fits the block's
//                absolute maximum under 448, so no element saturates);
//                kind::mxf8f6f4, the codes unpacked by the TMA (16 codes into
//                16 bytes); an opt-in path with a measured error (~3%)
//   MXFP4 rows   e2m1 (amax <= 6 * 2^e); kind::mxf4, both operands packed, at
//                twice the MMA rate; opt-in, ~12% error
//   split rows   the bf16 activations as two e4m3 planes under the MXFP8
//                scale (hi and the rounding remainder lo, which together hold
//                the bf16 value), two kind::mxf8f6f4 MMAs per K slice: the
//                exact product, with no weight expansion
// The reference's operator carries the hook for quantising the activations
// (`maybe_quantize_lhs`,
// 05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:257-263) but never
// exercises it.
//
// Layouts (all prepared once, or produced by the kernels here):
//   weights     codes (G, N, K/2) u8, the checkpoint's (out, in) layout; for a
//               fused gate/up weight the rows are interleaved (row 2i = gate
//               feature i, 2i+1 = up feature i) so a (gate, up) pair lands in
//               adjacent accumulator lanes
//   weight SF   (G, N/128, K/128) atoms of 512 bytes: the scales of 128 rows
//               x 4 K blocks, byte r0*16 + r1*4 + kb for row r0 + 32*r1,
//               the layout tcgen05.cp 32x128b.warpx4 copies to tensor memory
//               (row r's scales for the MMA's 4 K blocks land in TMEM column
//               r/32 of every lane quarter, byte kb)
//   activations rows (M_pad, K) e4m3, (M_pad, K/2) e2m1 pairs or (2, M_pad, K)
//               e4m3 planes; every expert's rows start at a multiple of 128
//               (rows past an expert's count up to that boundary are padding
//               nobody reads), so a 128-row tile owns whole atoms
//   act SF      (K/128, M_pad/128) atoms, the same byte layout per 128 rows,
//               K-step major so a tile's consecutive row blocks are one copy
//
// GEMM tile: 128 weight rows (UMMA M) x 192 token rows (UMMA N, or the tile's
// row count rounded up to 16), 128-byte operand rows per ring stage (K 128 =
// 4 MMAs of K 32, or K 256 = 4 MMAs of K 64 for kind::mxf4).  Two 192-column
// accumulators (at columns 0 and 256) leave room for the scale columns, and
// every tile of a group starts 64-row aligned inside its 128-aligned group, so
// the tokens' scales for the tile are whole atoms starting 0 or 2 columns in
// (64 rows = 2 columns).
//   warp 0     weight producer: TMA (codes) and the weight-scale atoms
//   warp 6     token producer: TMA (one 192-row box per plane for a full
//              tile) and the token-scale atoms (one bulk copy per quad)
//              (one thread issues a copy only every few hundred cycles, so
//              the copies of a step are split over two threads and kept few)
//   warp 1     TMEM owner and MMA issuer; copies each stage's scale atoms into
//              tensor memory (tcgen05.cp) ahead of its MMAs
//   warps 2-5  epilogue (tensor-memory lane = weight row, column = token);
//              the SiTU epilogue can write its activations already quantised
//              for the next GEMM
#include <cuda.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "../../include/lmoe.h"
#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

namespace {

constexpr int kMxRowBytes = 128;  // bytes of an operand row per stage (one 128-byte swizzle row)
constexpr int kMxRows = 128;   // weight rows per tile (UMMA M)
constexpr int kMxTok = 192;    // token rows per tile (UMMA N at most)
constexpr int kMxAlign = 128;  // row alignment of every expert's activation rows
constexpr int kMxMaxGroups = 1024;
constexpr int kMxThreads = 32 * 7;
constexpr int kMxTokWarp = 6;

// MMA kinds of this kernel:
//   KIND_F8F6F4  kind::mxf8f6f4, A e2m1 (the TMA unpacks 64 bytes of codes to a
//                128-byte row), B e4m3; K 128 per stage = 4 MMAs of K 32; one
//                E8M0 scale byte per operand row per MMA (scale_vec::1X)
//   KIND_F4      kind::mxf4, A and B e2m1, both packed (a 128-byte row holds
//                256 codes, low nibble first); K 256 per stage = 4 MMAs of K 64
//                at twice the rate of the former; two scale bytes per row per
//                MMA (scale_vec::2X, selected by scale id 0 or 2)
//   KIND_F8_SPLIT  kind::mxf8f6f4 as KIND_F8F6F4, with the token operand in two
//                e4m3 planes that share the block scale: hi = e4m3(x / 2^e) and
//                lo = e4m3(x / 2^e - hi).  hi + lo carries all 8 significant
//                bits of a bf16 value (exactly, for |x| >= 2^-2 of the scale
//                unit), so two MMAs into one accumulator give the product of
//                the bf16 activations themselves: the exact MXFP4 matmul on the
//                block-scaled tensor core, with no weight expansion
enum { KIND_F8F6F4 = 0, KIND_F4 = 1, KIND_F8_SPLIT = 2 };

template <int KIND>
struct MxCfg {
  static constexpr int kBK = KIND == KIND_F4 ? 256 : 128;  // K elements per stage
  static constexpr int kQuads = kBK / 128;                   // scale atoms (4 K blocks) per row block
  static constexpr int kPlanes = KIND == KIND_F8_SPLIT ? 2 : 1;  // token operand planes
  static constexpr int kStages = KIND == KIND_F8_SPLIT ? 3 : 4;
  static constexpr int kABytes = kMxRows * kMxRowBytes;      // 16 KB in shared memory
  static constexpr int kATx = KIND == KIND_F4 ? kABytes : kABytes / 2;  // bytes moved
  static constexpr int kBoxRows = 64;
  static constexpr int kBoxBytes = kBoxRows * kMxRowBytes;  // 8 KB
  static constexpr int kBPlaneBytes = 3 * kBoxBytes;        // up to 192 token rows
  static constexpr int kBBytes = kPlanes * kBPlaneBytes;
  static constexpr int kSfBytes = 512;
  static constexpr int kSfbAtoms = 2;                       // 192 rows from a 0- or 64-row offset
  static constexpr int kSfaOff = kABytes + kBBytes;         // kQuads weight-scale atoms
  static constexpr int kSfbOff = kSfaOff + kQuads * kSfBytes;  // kQuads x kSfbAtoms token-scale atoms
  // 41.5 (KIND_F8F6F4), 43 (KIND_F4) or 65.5 KB (KIND_F8_SPLIT) of operands, every
  // stage 1024-byte aligned
  static constexpr int kStageBytes =
      (kSfbOff + kQuads * kSfbAtoms * kSfBytes + 1023) / 1024 * 1024;
  static constexpr int kWarpStage = 1024;
  static constexpr int kOutStageBytes = 4 * kWarpStage;
  // the quantising SiTU epilogue's block maxima: 4 warps x 2 slots x 32 tokens
  static constexpr int kXchgBytes = 4 * 2 * 32 * 4;
  static constexpr int kSchedBytes = 3 * (kMxMaxGroups + 1) * 4;
  static constexpr int kNumBars = 2 * kStages + 7;
  static constexpr size_t kSmem = 1024 + size_t(kStages) * kStageBytes + kOutStageBytes +
                                  kXchgBytes + kSchedBytes + 16 + 8 * kNumBars + 16;
  static constexpr int kTmemCols = 512;  // accumulators at columns 0 and 256 (192 wide)
  static constexpr int kAccStride = 256;
  // scales in the gap after accumulator 0: 4 columns per atom, weight atoms
  // of the stage's quads first, then each quad's (up to) two token atoms
  static constexpr int kSfaCol = kMxTok;
  static constexpr int kSfbCol = kMxTok + 4 * kQuads;
  static_assert(kSfbCol + 4 * kSfbAtoms * kQuads <= kAccStride, "scale columns in the gap");
  static_assert(kStageBytes % 1024 == 0, "1024-byte aligned stages");
  static_assert(kOutStageBytes >= 3 * kMxThreads * 4, "scan scratch");
  static_assert(kSmem <= 232448, "shared memory");
};

// ------------------------------------------------------------------ PTX
// D (+)= A x B with per-32-K E8M0 scales of A rows and B columns read from
// tensor memory; A = e2m1 weights, B = e4m3 (KIND_F8F6F4) or e2m1 (KIND_F4)
// tokens (formats in idesc).
template <int KIND>
__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                        uint32_t accumulate) {
  if constexpr (KIND == KIND_F4) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
            "r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
            "r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
        : "memory");
  }
}

// 32 rows x 16 bytes of shared memory -> tensor-memory lanes 0-31 of every
// lane quarter, 4 columns
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// contiguous global -> shared copy counted on an mbarrier (16-byte aligned)
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Shared-memory descriptor of a scale atom for tcgen05.cp: no swizzle,
// 8-row core matrices of 16-byte rows 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(16 >> 4) << 16;
  d |= static_cast<uint64_t>(128 >> 4) << 32;
  d |= 1ull << 46;
  return d;
}

// Instruction descriptor with block scales: A format in bits 7-9, B format in
// bits 10-12 (kind::mxf8f6f4: e2m1 = 5, e4m3 = 0; kind::mxf4: e2m1 = 1), both
// K-major, N >> 3 in bits 17-22, E8M0 scales (bit 23), M >> 4 in bits 24-28,
// bit 31 clear (dense K: 32 for mxf8f6f4, 64 for mxf4); the first scale byte
// of each operand's TMEM word this MMA reads goes in bits 29-30 (A) and 4-5 (B).
template <int KIND>
__host__ __device__ constexpr uint32_t idesc_mx(uint32_t m, uint32_t n) {
  return (KIND == KIND_F4 ? (1u << 7) | (1u << 10) : (5u << 7) | (0u << 10)) |
         ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24);
}

struct MxArgs {
  const int32_t* group_sizes;
  int32_t* status;
  void* out;
  const uint8_t* w_sf;    // (G, n_weight/128, K/128, 512)
  const uint8_t* act_sf;  // (M_pad/128, K/128, 512)
  int64_t ldo;
  int M_pad, N, K, G;
  int n_tiles;
  int n_weight;
  float beta, linear_beta, inv_beta, inv_linear_beta;
  int round_gate_up;
  int out_f16;
  int m_out;  // 0: output rows at the padded positions; > 0: unpadded, m_out rows
  int zero_tail;  // unpadded output: rows at or past sum(group_sizes) are zeroed
  // EPI_SITU only: with q_out set, the activations are written quantised for
  // the next block-scaled GEMM instead of to `out` -- format q_fmt (MX_E4M3,
  // MX_E2M1 or MX_E4M3_SPLIT) at the same padded rows, scale atoms to q_sf
  uint8_t* q_out;
  uint8_t* q_sf;
  int q_fmt;
};

struct MxTile {
  int g, n_tile, row0, rows;
};

// ------------------------------------------------------------------ quantise
// Element formats of the quantised activation rows: MX_E4M3 (one byte per
// value, MXFP8), MX_E2M1 (two values per byte, low nibble first, MXFP4) or
// MX_E4M3_SPLIT (two e4m3 planes under the MXFP8 scale: hi, and lo = the
// rounding remainder of hi, so hi + lo carries the value's 8 significant bits).
enum { MX_E4M3 = 0, MX_E2M1 = 1, MX_E4M3_SPLIT = 2 };

// Exponent e of a block with absolute maximum `amax`: the smallest with
// amax <= emax * 2^e, where emax is the format's largest finite value (e4m3:
// 448 = 1.75 * 2^8; e2m1: 6 = 1.5 * 2^2), so no element saturates; E8M0 byte
// e + 127, clamped to [0, 254]; 0 for an all-zero block.
template <int FMT>
__device__ __forceinline__ int mx_scale_exp(float amax) {
  if (!(amax > 0.f)) return -127;
  const uint32_t b = __float_as_uint(amax);
  const int E = static_cast<int>((b >> 23) & 0xFF) - 127;
  const int e = FMT == MX_E2M1 ? E - 2 + ((b & 0x7FFFFF) > 0x400000 ? 1 : 0)
                               : E - 8 + ((b & 0x7FFFFF) > 0x600000 ? 1 : 0);  // e4m3, both planes
  return max(-127, min(127, e));
}

// The quantising gathers give each 32-value block to two lanes: lane l holds
// values [16 l, 16 l + 16) of each 512-value chunk of a row, so a warp's store
// of one plane's codes covers 512 contiguous bytes (e4m3; 256 for e2m1), and
// an 8-lane group holds one K group (4 blocks = one scale word).
template <int FMT>
struct MxHalf {
  uint32_t hi[4];  // 16 e4m3 codes, or 16 e2m1 codes in hi[0..1]
  uint32_t lo[4];  // MX_E4M3_SPLIT: the lo plane's 16 codes
  uint32_t sfw;    // scale word of the lane's K group (every lane of the 8-lane group)
};

// 2^-e as a float for e in [-127, 127] (exact powers of two; 2^-127 is subnormal)
__device__ __forceinline__ float mx_inv_scale(int e) {
  const int x = -e;
  return x >= -126 ? __uint_as_float(static_cast<uint32_t>(x + 127) << 23)
                   : __uint_as_float(1u << (x + 149));
}

// 16 bf16 or f16 values (two uint4) as floats.
template <bool F16>
__device__ __forceinline__ void mx_unpack16(const uint4 (&raw)[2], float (&v)[16]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint32_t ws[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if (F16)
        f = __half22float2(*reinterpret_cast<const __half2*>(&ws[i]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
      v[i * 2 + c * 8] = f.x;
      v[i * 2 + c * 8 + 1] = f.y;
    }
  }
}

// The 16 values' codes under the block exponent e, rounded to nearest even:
// e4m3 pairs, or e2m1 pairs (value 2i in the low nibble of byte i); for
// MX_E4M3_SPLIT also the remainders x * inv - e4m3(x * inv) (exact in f32)
// rounded to e4m3.
template <int FMT>
__device__ __forceinline__ void mx_encode16(const float (&v)[16], int e, MxHalf<FMT>& o) {
  const float inv = mx_inv_scale(e);
  if constexpr (FMT == MX_E2M1) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float* x = v + 8 * i;
      asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
          "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
          : "=r"(o.hi[i])
          : "f"(x[0] * inv), "f"(x[1] * inv), "f"(x[2] * inv), "f"(x[3] * inv),
            "f"(x[4] * inv), "f"(x[5] * inv), "f"(x[6] * inv), "f"(x[7] * inv));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = v[i * 4] * inv, x1 = v[i * 4 + 1] * inv;
      const float x2 = v[i * 4 + 2] * inv, x3 = v[i * 4 + 3] * inv;
      uint16_t p01, p23;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p01) : "f"(x1), "f"(x0));
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p23) : "f"(x3), "f"(x2));
      o.hi[i] = static_cast<uint32_t>(p01) | (static_cast<uint32_t>(p23) << 16);
      if constexpr (FMT == MX_E4M3_SPLIT) {
        // the rounded pairs back to f32 (through f16, exact for e4m3)
        uint32_t h01, h23;
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(p01));
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(p23));
        const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
        const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
        uint16_t l01, l23;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(l01) : "f"(x1 - f01.y), "f"(x0 - f01.x));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(l23) : "f"(x3 - f23.y), "f"(x2 - f23.x));
        o.lo[i] = static_cast<uint32_t>(l01) | (static_cast<uint32_t>(l23) << 16);
      }
    }
  }
}

// Quantise the lane's 16 values (raw: two uint4 of bf16 or f16; the partner
// lane l ^ 1 holds the other half of the block).  All 32 lanes must call.
template <bool F16, int FMT>
__device__ __forceinline__ void mx_quantize_half(const uint4 (&raw)[2], int lane, MxHalf<FMT>& o) {
  float v[16];
  mx_unpack16<F16>(raw, v);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const int e = mx_scale_exp<FMT>(amax);
  mx_encode16<FMT>(v, e, o);
  // the K group's 4 scale bytes (block (lane / 2) % 4 of the group)
  uint32_t w = static_cast<uint32_t>(e + 127) << (8 * ((lane >> 1) & 3));
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  w |= __shfl_xor_sync(0xffffffffu, w, 4);
  o.sfw = w;
}

// Store the lane's codes of value index vi (a multiple of 16) of padded row
// dst: each plane's codes at its byte offset, the scale word by the first
// lane of each 8-lane group.
template <int FMT>
__device__ __forceinline__ void mx_store_half(const MxHalf<FMT>& o, int lane, int vi, int64_t dst,
                                              int K, int64_t m_pad_cap, uint8_t* q, uint8_t* sf) {
  if constexpr (FMT == MX_E2M1) {
    __stcs(reinterpret_cast<uint2*>(q + dst * (K / 2) + vi / 2), make_uint2(o.hi[0], o.hi[1]));
  } else {
    uint8_t* qd = q + dst * K + vi;
    __stcs(reinterpret_cast<uint4*>(qd), make_uint4(o.hi[0], o.hi[1], o.hi[2], o.hi[3]));
    if constexpr (FMT == MX_E4M3_SPLIT)  // the lo plane, m_pad_cap rows further
      __stcs(reinterpret_cast<uint4*>(qd + m_pad_cap * K),
             make_uint4(o.lo[0], o.lo[1], o.lo[2], o.lo[3]));
  }
  if ((lane & 7) == 0) {
    // atom (K group, row block), bytes r0*16 + r1*4 for row r0 + 32*r1
    const int rr = static_cast<int>(dst % 128);
    const int64_t atom = static_cast<int64_t>(vi / 128) * (m_pad_cap / 128) + dst / 128;
    *reinterpret_cast<uint32_t*>(sf + atom * 512 + (rr & 31) * 16 + (rr >> 5) * 4) = o.sfw;
  }
}

// One scale byte (block exponent e) of padded row r, K block blk, in the atom
// layout of a tensor with m_pad_cap padded rows.
__device__ __forceinline__ void mx_store_scale_byte(uint8_t* sf, int64_t r, int blk, int e,
                                                    int64_t m_pad_cap) {
  const int rr = static_cast<int>(r % 128);
  const int64_t atom = static_cast<int64_t>(blk / 4) * (m_pad_cap / 128) + r / 128;
  sf[atom * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + (blk & 3)] = static_cast<uint8_t>(e + 127);
}

// Schedule: padded row starts (multiples of 128), unpadded row starts (the
// exclusive prefix sums of the group sizes, row_src[G] = their sum), tile
// starts.  `scan` holds 3 x blockDim.x ints of scratch.
__device__ int mx_schedule(const MxArgs& a, int32_t* row_off, int32_t* row_src,
                           int32_t* tile_start, int32_t* scan) {
  const int G = a.G;
  const int nthr = blockDim.x;
  int32_t* scan_rows = scan;
  int32_t* scan_src = scan + nthr;
  int32_t* scan_tiles = scan + 2 * nthr;
  const int per = (G + nthr - 1) / nthr;
  const int g0 = min(G, static_cast<int>(threadIdx.x) * per);
  const int g1 = min(G, g0 + per);
  long long rows = 0, src = 0, tiles = 0;
  int bad = 0;
  for (int g = g0; g < g1; ++g) {
    const int s = __ldg(a.group_sizes + g);
    if (s < 0) bad = 1;
    const int ss = max(s, 0);
    rows += (ss + kMxAlign - 1) / kMxAlign * kMxAlign;
    src += ss;
    tiles += static_cast<long long>((ss + kMxTok - 1) / kMxTok) * a.n_tiles;
  }
  scan_rows[threadIdx.x] = bad ? -1 : static_cast<int32_t>(min(rows, (long long)INT32_MAX));
  scan_src[threadIdx.x] = static_cast<int32_t>(min(src, (long long)INT32_MAX));
  scan_tiles[threadIdx.x] = static_cast<int32_t>(min(tiles, (long long)INT32_MAX));
  __syncthreads();
  __shared__ int s_total;
  if (threadIdx.x == 0) {
    long long r = 0, u = 0, t = 0;
    int invalid = 0;
    for (int i = 0; i < nthr; ++i) {
      const int rr = scan_rows[i];
      const int uu = scan_src[i];
      const int tt = scan_tiles[i];
      if (rr < 0) invalid = 1;
      scan_rows[i] = static_cast<int32_t>(r);
      scan_src[i] = static_cast<int32_t>(u);
      scan_tiles[i] = static_cast<int32_t>(t);
      r += max(rr, 0);
      u += uu;
      t += tt;
    }
    if (invalid || r > a.M_pad || t > INT32_MAX || (a.m_out > 0 && u > a.m_out)) {
      record_status(a.status, kDeviceBounds);
      s_total = -1;
    } else {
      s_total = static_cast<int>(t);
      row_off[G] = static_cast<int32_t>(r);
      row_src[G] = static_cast<int32_t>(u);
      tile_start[G] = static_cast<int32_t>(t);
    }
  }
  __syncthreads();
  if (s_total >= 0) {
    int r = scan_rows[threadIdx.x];
    int u = scan_src[threadIdx.x];
    int t = scan_tiles[threadIdx.x];
    for (int g = g0; g < g1; ++g) {
      const int s = max(__ldg(a.group_sizes + g), 0);
      row_off[g] = r;
      row_src[g] = u;
      tile_start[g] = t;
      r += (s + kMxAlign - 1) / kMxAlign * kMxAlign;
      u += s;
      t += ((s + kMxTok - 1) / kMxTok) * a.n_tiles;
    }
  }
  __syncthreads();
  return s_total;
}

__device__ __forceinline__ MxTile mx_tile(const int32_t* tile_start, const int32_t* row_off,
                                          const int32_t* row_src, int G, int n_tiles, int t) {
  MxTile c;
  c.g = find_group(tile_start, G, t);
  const int local = t - tile_start[c.g];
  const int m_tile = local / n_tiles;
  c.n_tile = local - m_tile * n_tiles;
  c.row0 = row_off[c.g] + m_tile * kMxTok;
  c.rows = min(kMxTok, row_src[c.g + 1] - row_src[c.g] - m_tile * kMxTok);
  return c;
}

__device__ __forceinline__ uint16_t mx_out16(float v, int out_f16) {
  if (out_f16) {
    const __half h = __float2half_rn(bf16_round_f(v));
    return *reinterpret_cast<const uint16_t*>(&h);
  }
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&b);
}

template <int kChunks>
__device__ __forceinline__ int mx_swz(int row) {
  return kChunks == 4 ? ((row >> 1) & 3) : (row & 7);
}

template <int EPI, int KIND>
__global__ void __launch_bounds__(kMxThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmT,
                   const __grid_constant__ CUtensorMap tmT64, const MxArgs args) {
  using C = MxCfg<KIND>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* stages = smem;
  uint8_t* ostage = stages + C::kStages * C::kStageBytes;
  const uint32_t xchg = smem_u32(ostage + C::kOutStageBytes);
  int32_t* row_off = reinterpret_cast<int32_t*>(ostage + C::kOutStageBytes + C::kXchgBytes);
  int32_t* row_src = row_off + (kMxMaxGroups + 1);
  int32_t* tile_start = row_src + (kMxMaxGroups + 1);
  // mbarriers need 8-byte alignment (three schedule arrays of 1025 ints end at 4 mod 8)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_align_up<16>(tile_start + (kMxMaxGroups + 1)));
  uint64_t* full = bars;
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* xbar = drain + 1;  // epilogue warps 2 and 3 (4 and 5) exchange block maxima
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = args.G;
  if (threadIdx.x == 0) *abort_flag = 0;
  int32_t* scan = reinterpret_cast<int32_t*>(ostage);
  const int total = mx_schedule(args, row_off, row_src, tile_start, scan);
  if (total < 0) return;  // uniform across the CTA; nothing allocated yet

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(full + s), 2);  // the weight and the token producer
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(acc_full + b), 1);
      mbar_init(smem_u32(acc_empty + b), 128);
    }
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(xbar), 2);
    mbar_init(smem_u32(xbar + 1), 2);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmT);
    tma_prefetch_desc(&tmT64);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = args.K / C::kBK;
  const int num_kq = args.K / 128;  // scale atoms along K per row block
  const int64_t w_sf_per_g = static_cast<int64_t>(args.n_weight / kMxRows) * num_kq * C::kSfBytes;

  if (warp == 0 || warp == kMxTokWarp) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      const bool tok = warp == kMxTokWarp;
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      const int64_t row_blocks = args.M_pad / kMxAlign;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const MxTile tc = mx_tile(tile_start, row_off, row_src, G, args.n_tiles, t);
        const int n_box = (tc.rows + C::kBoxRows - 1) / C::kBoxRows;
        const uint8_t* wsf = args.w_sf + tc.g * w_sf_per_g +
                             static_cast<int64_t>(tc.n_tile) * num_kq * C::kSfBytes;
        // token-scale atoms from the one holding row0 through the tile's last row
        const int n_atoms = ((tc.row0 % kMxAlign) + tc.rows + kMxAlign - 1) / kMxAlign;
        const int64_t rb0 = tc.row0 / kMxAlign;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          const uint32_t base = smem_u32(stages + stage * C::kStageBytes);
          // x coordinate of the stage's 128-byte rows: 128 per stage in both
          // kinds (codes of the unpacking weight map, bytes of the others)
          const int x0 = kb * kMxRowBytes;
          if (!tok) {
            // the weight-scale atoms of the stage's quads are consecutive
            mbar_arrive_expect_tx(fb, C::kATx + C::kQuads * C::kSfBytes);
            tma_load_3d(base, &tmW, fb, x0, tc.n_tile * kMxRows, tc.g);
            bulk_load(base + C::kSfaOff, wsf + kb * C::kQuads * C::kSfBytes,
                      C::kQuads * C::kSfBytes, fb);
          } else {
            const uint32_t b_dst = base + C::kABytes;
            if (tc.rows == kMxTok) {
              mbar_arrive_expect_tx(fb, C::kBBytes + C::kQuads * n_atoms * C::kSfBytes);
              for (int p = 0; p < C::kPlanes; ++p) {
                if (C::kPlanes > 1)
                  tma_load_3d(b_dst + p * C::kBPlaneBytes, &tmT, fb, x0, tc.row0, p);
                else
                  tma_load_2d(b_dst, &tmT, fb, x0, tc.row0);
              }
            } else {
              mbar_arrive_expect_tx(fb, C::kPlanes * n_box * C::kBoxBytes +
                                            C::kQuads * n_atoms * C::kSfBytes);
              for (int p = 0; p < C::kPlanes; ++p)
                for (int i = 0; i < n_box; ++i) {
                  const uint32_t dst = b_dst + p * C::kBPlaneBytes + i * C::kBoxBytes;
                  if (C::kPlanes > 1)
                    tma_load_3d(dst, &tmT64, fb, x0, tc.row0 + i * C::kBoxRows, p);
                  else
                    tma_load_2d(dst, &tmT64, fb, x0, tc.row0 + i * C::kBoxRows);
                }
            }
            // per quad, the tile's token-scale atoms are consecutive
            for (int q = 0; q < C::kQuads; ++q)
              bulk_load(base + C::kSfbOff + q * C::kSfbAtoms * C::kSfBytes,
                        args.act_sf +
                            (static_cast<int64_t>(kb * C::kQuads + q) * row_blocks + rb0) * C::kSfBytes,
                        n_atoms * C::kSfBytes, fb);
          }
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < C::kStages; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(full + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t sfa_t = tmem_base + C::kSfaCol;
      const uint32_t sfb_t = tmem_base + C::kSfbCol;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const MxTile tc = mx_tile(tile_start, row_off, row_src, G, args.n_tiles, t);
        const uint32_t n_mma = (tc.rows + 15) & ~15;
        const uint32_t idesc = idesc_mx<KIND>(kMxRows, n_mma);
        const int n_atoms = ((tc.row0 % kMxAlign) + tc.rows + kMxAlign - 1) / kMxAlign;
        // token n's scales sit in column (row0 % 128 + n) / 32 of the copied
        // atoms; row0 % 128 is 0 or 64 (tiles of 192 from 128-aligned group starts)
        const uint32_t sfb_mma = sfb_t + static_cast<uint32_t>((tc.row0 % kMxAlign) / 32);
        if (!mbar_wait(smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::kAccStride;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(stages + stage * C::kStageBytes);
          // this stage's scales into tensor memory; the tensor pipe runs them
          // in order, after the previous stage's MMAs and before these
#pragma unroll
          for (int q = 0; q < C::kQuads; ++q) {
            tmem_cp_sf(sfa_t + 4 * q, sf_desc(base + C::kSfaOff + q * C::kSfBytes));
            for (int i = 0; i < n_atoms; ++i)
              tmem_cp_sf(sfb_t + 4 * (q * C::kSfbAtoms + i),
                         sf_desc(base + C::kSfbOff + (q * C::kSfbAtoms + i) * C::kSfBytes));
          }
          // 4 MMAs of 32 bytes of each operand row: K 32 (one scale byte,
          // id k) or K 64 (two scale bytes of quad k/2, id 0 or 2); with two
          // token planes, one MMA per plane into the same accumulator
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t adesc = smem_desc_sw128(base + k * 32, 16, 1024);
            const uint32_t q = KIND == KIND_F4 ? static_cast<uint32_t>(k >> 1) : 0u;
            const uint32_t id = KIND == KIND_F4 ? static_cast<uint32_t>((k & 1) << 1)
                                                : static_cast<uint32_t>(k);
#pragma unroll
            for (int p = 0; p < C::kPlanes; ++p) {
              const uint64_t bdesc =
                  smem_desc_sw128(base + C::kABytes + p * C::kBPlaneBytes + k * 32, 16, 1024);
              umma_mx<KIND>(d_tmem, adesc, bdesc, idesc | (id << 29) | (id << 4),
                            (sfa_t + 4 * q) | (id << 30),
                            (sfb_mma + 4 * C::kSfbAtoms * q) | (id << 30),
                            (kb | k | p) != 0 ? 1u : 0u);
            }
          }
          umma_commit(smem_u32(empty + stage));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(acc_full + acc));
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        umma_commit(smem_u32(drain));
        mbar_drain(smem_u32(drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const uint32_t stg = smem_u32(ostage + q * C::kWarpStage);
    constexpr int esize = (EPI == EPI_F32) ? 4 : 2;
    uint32_t acc = 0, acc_phase = 0;
    uint32_t xcount = 0;  // block-maximum exchanges so far (the pair barrier's phases)
    bool xok = true;
    for (int t = blockIdx.x; t < total && xok; t += gridDim.x) {
      const MxTile tc = mx_tile(tile_start, row_off, row_src, G, args.n_tiles, t);
      if (!mbar_wait(smem_u32(acc_full + acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * C::kAccStride;
      // padded row -> output row (the unpadded position when m_out > 0)
      const int64_t out_shift = args.m_out > 0 ? row_src[tc.g] - row_off[tc.g] : 0;
#pragma unroll 1
      for (int c = 0; c < kMxTok / 32; ++c) {
        if (c * 32 >= tc.rows) break;  // warp-uniform
        const int tok0 = tc.row0 + c * 32;
        const int tok_end = tc.row0 + tc.rows;
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        if (EPI == EPI_SITU) {
          // lanes 2i / 2i+1 hold gate / up of feature i (interleaved weight rows)
          const int odd = lane & 1;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t send = odd ? v[j] : v[16 + j];
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
            float g = __uint_as_float(odd ? recv : v[j]);
            float u = __uint_as_float(odd ? v[16 + j] : recv);
            if (args.round_gate_up) {
              g = bf16_round_f(g);
              u = bf16_round_f(u);
            }
            const float o = situ_fast(g, u, args.beta, args.inv_beta, args.linear_beta,
                                      args.inv_linear_beta);
            sts_u16(stg + 2u * ((odd * 16 + j) * 16 + (lane >> 1)), mx_out16(o, args.out_f16));
          }
          __syncwarp();
          const int tok = tok0 + lane;
          const int f0 = tc.n_tile * (kMxRows / 2) + q * 16;
          if (args.q_out != nullptr) {
            // quantised activations: lane = token, its 16 features (bf16
            // values); their 32-feature block spans this warp and warp q ^ 1,
            // which meet through shared memory and a pair barrier
            const uint4 raw[2] = {lds_v4(stg + lane * 32), lds_v4(stg + lane * 32 + 16)};
            float fv[16];
            mx_unpack16<false>(raw, fv);
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(fv[i]));
            const uint32_t slot = xcount & 1u;
            sts_u32(xchg + ((q * 2 + slot) * 32 + lane) * 4, __float_as_uint(amax));
            __syncwarp();
            const uint32_t xb = smem_u32(xbar + (q >> 1));
            if (lane == 0) mbar_arrive(xb);
            if (!mbar_wait(xb, slot, abort_flag, args.status)) {
              xok = false;
              break;
            }
            amax = fmaxf(amax, lds_f32(xchg + (((q ^ 1) * 2 + slot) * 32 + lane) * 4));
            ++xcount;
            if (tok < tok_end) {
              const int64_t plane = static_cast<int64_t>(args.M_pad) * args.N;
              if (args.q_fmt == MX_E2M1) {
                const int e = mx_scale_exp<MX_E2M1>(amax);
                MxHalf<MX_E2M1> o;
                mx_encode16<MX_E2M1>(fv, e, o);
                *reinterpret_cast<uint2*>(args.q_out + static_cast<int64_t>(tok) * (args.N / 2) +
                                          f0 / 2) = make_uint2(o.hi[0], o.hi[1]);
                if ((q & 1) == 0) mx_store_scale_byte(args.q_sf, tok, tc.n_tile * 2 + (q >> 1), e, args.M_pad);
              } else {
                const int e = mx_scale_exp<MX_E4M3>(amax);
                uint8_t* qd = args.q_out + static_cast<int64_t>(tok) * args.N + f0;
                if (args.q_fmt == MX_E4M3_SPLIT) {
                  MxHalf<MX_E4M3_SPLIT> o;
                  mx_encode16<MX_E4M3_SPLIT>(fv, e, o);
                  *reinterpret_cast<uint4*>(qd) = make_uint4(o.hi[0], o.hi[1], o.hi[2], o.hi[3]);
                  *reinterpret_cast<uint4*>(qd + plane) = make_uint4(o.lo[0], o.lo[1], o.lo[2], o.lo[3]);
                } else {
                  MxHalf<MX_E4M3> o;
                  mx_encode16<MX_E4M3>(fv, e, o);
                  *reinterpret_cast<uint4*>(qd) = make_uint4(o.hi[0], o.hi[1], o.hi[2], o.hi[3]);
                }
                if ((q & 1) == 0) mx_store_scale_byte(args.q_sf, tok, tc.n_tile * 2 + (q >> 1), e, args.M_pad);
              }
            }
          } else if (tok < tok_end) {
            uint16_t* orow = reinterpret_cast<uint16_t*>(args.out) +
                             (tok + out_shift) * args.ldo + f0;
            if (f0 + 8 <= args.N) *reinterpret_cast<uint4*>(orow) = lds_v4(stg + lane * 32);
            if (f0 + 16 <= args.N) *reinterpret_cast<uint4*>(orow + 8) = lds_v4(stg + lane * 32 + 16);
          }
          __syncwarp();
        } else {
          constexpr int kRowBytes = 32 * esize;
          constexpr int kChunks = kRowBytes / 16;
          constexpr int kRows = C::kWarpStage / kRowBytes;
          const int byte = lane * esize;
          const int f0 = tc.n_tile * kMxRows + q * 32;
#pragma unroll
          for (int p0 = 0; p0 < 32; p0 += kRows) {
            const uint32_t dst0 = stg + (byte & 15);
#pragma unroll
            for (int jj = 0; jj < kRows; ++jj) {
              const uint32_t d = dst0 + jj * kRowBytes + (((byte >> 4) ^ mx_swz<kChunks>(jj)) << 4);
              if (EPI == EPI_F32)
                sts_u32(d, v[p0 + jj]);
              else
                sts_u16(d, mx_out16(__uint_as_float(v[p0 + jj]), args.out_f16));
            }
            __syncwarp();
            const int tok = tok0 + p0 + lane;
            if (lane < kRows && tok < tok_end) {
              uint8_t* orow = reinterpret_cast<uint8_t*>(args.out) +
                              ((tok + out_shift) * args.ldo + f0) * esize;
#pragma unroll
              for (int cc = 0; cc < kChunks; ++cc) {
                if (f0 + (cc + 1) * (16 / esize) <= args.N)
                  *reinterpret_cast<uint4*>(orow + cc * 16) =
                      lds_v4(stg + lane * kRowBytes + ((cc ^ mx_swz<kChunks>(lane)) * 16));
              }
            }
            __syncwarp();
          }
        }
      }
      if (!xok) break;
      tc_fence_before();
      mbar_arrive(smem_u32(acc_empty + acc));
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    // unpadded output: rows at or past sum(group_sizes) are zero (ragged_dot
    // semantics), written by the epilogue warps of all CTAs
    if (args.m_out > 0 && args.zero_tail) {
      const int64_t row_bytes = static_cast<int64_t>(args.N) * esize;
      const int64_t chunks_per_row = row_bytes / 16;
      const int64_t first = row_src[G];
      const int64_t n_chunks = (args.m_out - first) * chunks_per_row;
      const int etid = threadIdx.x - 64;  // epilogue warps 2-5
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * 128 + etid; i < n_chunks;
           i += static_cast<int64_t>(gridDim.x) * 128) {
        const int64_t rr = first + i / chunks_per_row;
        const int64_t cc = i % chunks_per_row;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(args.out) +
                                  (rr * args.ldo) * esize + cc * 16) = make_uint4(0, 0, 0, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int EPI, int KIND>
int launch_mx(const CUtensorMap& tw, const CUtensorMap& tt, const CUtensorMap& tt64,
              const MxArgs& a, int max_tiles, cudaStream_t stream) {
  auto kern = mx_gemm_kernel<EPI, KIND>;
  using C = MxCfg<KIND>;
  const int dev = current_device();
  static std::mutex mu;
  static uint64_t configured = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(configured & (1ull << dev))) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(C::kSmem)) != cudaSuccess)
        return kLaunchFailed;
      configured |= 1ull << dev;
    }
  }
  const int grid = max(1, min(num_sms(dev), max_tiles));
  kern<<<grid, kMxThreads, C::kSmem, stream>>>(tw, tt, tt64, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// ------------------------------------------------------------------ repack
// Weight repack, once per weight set: rows optionally interleaved (gate/up),
// scales gathered into 512-byte atoms, one warp per atom (lane r0 writes the
// 16 bytes of atom row r0).
__global__ void mx_repack_sf_kernel(const uint8_t* __restrict__ scales, int G, int N, int K,
                                    int interleave, uint8_t* __restrict__ sf_out) {
  const int kg_n = K / 128, rb_n = N / 128, kblocks = K / 32;
  const int64_t atoms = static_cast<int64_t>(G) * rb_n * kg_n;
  const int half = N / 2;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < atoms;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int lane = threadIdx.x & 31;
    const int kg = static_cast<int>(w % kg_n);
    const int rb = static_cast<int>((w / kg_n) % rb_n);
    const int g = static_cast<int>(w / (static_cast<int64_t>(kg_n) * rb_n));
    uint32_t words[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int r = rb * 128 + lane + 32 * r1;  // row of the repacked matrix
      const int src = interleave ? ((r & 1) ? half + (r >> 1) : (r >> 1)) : r;
      const uint8_t* s = scales + (static_cast<int64_t>(g) * N + src) * kblocks + kg * 4;
      words[r1] = static_cast<uint32_t>(s[0]) | (static_cast<uint32_t>(s[1]) << 8) |
                  (static_cast<uint32_t>(s[2]) << 16) | (static_cast<uint32_t>(s[3]) << 24);
    }
    *reinterpret_cast<uint4*>(sf_out + w * 512 + lane * 16) =
        make_uint4(words[0], words[1], words[2], words[3]);
  }
}

__global__ void mx_repack_rows_kernel(const uint8_t* __restrict__ packed, int G, int N, int K,
                                      uint8_t* __restrict__ out) {
  // interleave gate/up rows: out row 2i = in row i, 2i+1 = in row N/2 + i
  const int rb = K / 2 / 16;  // 16-byte chunks per row
  const int64_t total = static_cast<int64_t>(G) * N * rb;
  const int half = N / 2;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % rb);
    const int64_t row = i / rb;
    const int r = static_cast<int>(row % N);
    const int64_t g = row / N;
    const int src = (r & 1) ? half + (r >> 1) : (r >> 1);
    reinterpret_cast<uint4*>(out)[i] =
        reinterpret_cast<const uint4*>(packed)[(g * N + src) * rb + c];
  }
}

// Padded start of every group (multiples of 128) from the group sizes, in
// shared memory: pad_off[g] = padded_start[g] - start[g]; start[g] also kept.
// start[g] = sum of the counts before group g, pad_off[g] = (the same sum of
// the counts rounded up to kMxAlign) - start[g], start[G] = the total.  A
// block-wide exclusive scan, blockDim.x (a multiple of 32, at most 1024)
// groups at a time: warp scans by shuffles, then the warps' totals.
__device__ void mx_group_offsets(const int32_t* gs, int G, int32_t* start, int32_t* pad_off) {
  __shared__ int32_t warp_tot[2][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int32_t carry_s = 0, carry_p = 0;
  for (int base = 0; base < G; base += blockDim.x) {
    const int g = base + threadIdx.x;
    const int32_t n = g < G ? max(gs[g], 0) : 0;
    const int32_t np = (n + kMxAlign - 1) / kMxAlign * kMxAlign;
    int32_t is = n, ip = np;  // inclusive scans within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t ts = __shfl_up_sync(0xffffffffu, is, o);
      const int32_t tp = __shfl_up_sync(0xffffffffu, ip, o);
      if (lane >= o) {
        is += ts;
        ip += tp;
      }
    }
    if (lane == 31) {
      warp_tot[0][warp] = is;
      warp_tot[1][warp] = ip;
    }
    __syncthreads();
    int32_t before_s = 0, before_p = 0, all_s = 0, all_p = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) {
        before_s += warp_tot[0][w];
        before_p += warp_tot[1][w];
      }
      all_s += warp_tot[0][w];
      all_p += warp_tot[1][w];
    }
    if (g < G) {
      const int32_t s_excl = carry_s + before_s + is - n;
      start[g] = s_excl;
      pad_off[g] = carry_p + before_p + ip - np - s_excl;
    }
    carry_s += all_s;
    carry_p += all_p;
    __syncthreads();  // warp_tot is rewritten by the next chunk
  }
  if (threadIdx.x == 0) start[G] = carry_s;
  __syncthreads();
}

__device__ __forceinline__ int mx_group_of(const int32_t* start, int G, int p) {
  int lo = 0, hi = G - 1;  // last g with start[g] <= p
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= p) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One warp per row: gather (optional), quantise (FMT), store the row at its
// padded position and its scales in the atom layout.  The row is read 1024
// values (two chunks per lane) at a time; K is a multiple of 128, so an 8-lane
// group is inside the row or past it as a whole.
template <bool F16, int FMT>
__global__ void __launch_bounds__(256, 4) mx_quantize_kernel(
    const uint16_t* __restrict__ x, int64_t x_rows, const int32_t* __restrict__ token_idx,
    const int32_t* __restrict__ gs, int G, int64_t rows, int K, int64_t m_pad_cap,
    uint8_t* __restrict__ q, uint8_t* __restrict__ sf, int32_t* status) {
  extern __shared__ int32_t sh[];
  int32_t* start = sh;
  int32_t* pad_off = sh + G + 1;
  if (gs != nullptr) mx_group_offsets(gs, G, start, pad_off);
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < rows;
       p += nwarps) {
    int64_t dst = p;
    if (gs != nullptr) {
      if (p >= start[G]) continue;  // past sum(group_sizes): nothing to place
      dst = p + pad_off[mx_group_of(start, G, static_cast<int>(p))];
    }
    if (dst >= m_pad_cap) {
      if (lane == 0) record_status(status, kDeviceBounds);
      continue;
    }
    const int64_t src_row = token_idx != nullptr ? token_idx[p] : p;
    const bool zero = src_row < 0 || src_row >= x_rows;
    const uint4* src = reinterpret_cast<const uint4*>(x + (zero ? 0 : src_row) * K);
    for (int c0 = 0; c0 < K; c0 += 1024) {
      uint4 raw[2][2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int vi = c0 + 512 * i + 16 * lane;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          raw[i][c] = (zero || vi >= K) ? make_uint4(0, 0, 0, 0) : __ldg(src + vi / 8 + c);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int vi = c0 + 512 * i + 16 * lane;
        MxHalf<FMT> o;
        mx_quantize_half<F16, FMT>(raw[i], lane, o);
        if (vi < K) mx_store_half<FMT>(o, lane, vi, dst, K, m_pad_cap, q, sf);
      }
    }
  }
}

// The quantising gather in token order: a warp takes one 1024-value chunk of
// token t's row, quantises it once and stores the codes and scale words at
// the padded position of each of t's k sorted positions slot_pos[t*k + s] --
// the rows mx_quantize_kernel writes for a dropless dispatch, each source row
// read and quantised once instead of k times (the codes of the chunk's two
// halves kept in registers across the k stores).
// Positions past sum(group_sizes) or outside the capacity are skipped (the
// latter records LMOE_DEVICE_BOUNDS).
template <bool F16, int FMT>
__global__ void __launch_bounds__(256, 4) mx_quantize_scatter_kernel(
    const uint16_t* __restrict__ x, const int32_t* __restrict__ slot_pos, int64_t T, int k,
    const int32_t* __restrict__ gs, int G, int K, int64_t m_pad_cap, uint8_t* __restrict__ q,
    uint8_t* __restrict__ sf, int32_t* __restrict__ padded_pos, int32_t* status) {
  extern __shared__ int32_t sh[];
  int32_t* start = sh;
  int32_t* pad_off = sh + G + 1;
  mx_group_offsets(gs, G, start, pad_off);
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  bool bad = false;
  // a work item is one token's 1024-value chunk, so a few hundred tokens
  // still spread over many warps
  const int nchunks = (K + 1023) / 1024;
  const int64_t items = T * nchunks;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < items;
       w += nwarps) {
    const int64_t t = w / nchunks;
    const int c0 = static_cast<int>(w % nchunks) * 1024;
    // lane s < k: the padded destination row of slot s (-1: none)
    int64_t my_dst = -1;
    if (lane < k) {
      const int32_t p = slot_pos[t * k + lane];
      if (p >= 0 && p < start[G]) {
        my_dst = p + pad_off[mx_group_of(start, G, p)];
        if (my_dst >= m_pad_cap) {
          bad = true;
          my_dst = -1;
        }
      }
      // the padded position of each slot (lmoe_mxfp8_pad_positions' output),
      // written once per token by the warp of its first chunk
      if (padded_pos != nullptr && c0 == 0) padded_pos[t * k + lane] = static_cast<int32_t>(my_dst);
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + t * K);
    {
      uint4 raw[2][2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int vi = c0 + 512 * i + 16 * lane;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          raw[i][c] = vi < K ? __ldg(src + vi / 8 + c) : make_uint4(0, 0, 0, 0);
      }
      MxHalf<FMT> o[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) mx_quantize_half<F16, FMT>(raw[i], lane, o[i]);
      for (int s = 0; s < k; ++s) {
        const int64_t dst = __shfl_sync(0xffffffffu, my_dst, s);
        if (dst < 0) continue;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int vi = c0 + 512 * i + 16 * lane;
          if (vi < K) mx_store_half<FMT>(o[i], lane, vi, dst, K, m_pad_cap, q, sf);
        }
      }
    }
  }
  if (lane == 0 && __any_sync(0xffffffffu, bad)) record_status(status, kDeviceBounds);
}

// positions[i] -> padded positions (the combine's slot positions)
__global__ void mx_pad_positions_kernel(const int32_t* __restrict__ pos, int64_t n,
                                        const int32_t* __restrict__ gs, int G,
                                        int32_t* __restrict__ out) {
  extern __shared__ int32_t sh[];
  int32_t* start = sh;
  int32_t* pad_off = sh + G + 1;
  mx_group_offsets(gs, G, start, pad_off);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int p = pos[i];
    out[i] = (p < 0 || p >= start[G]) ? -1 : p + pad_off[mx_group_of(start, G, p)];
  }
}

// Quantising row gathers (the C entry points below): validation, launch.
template <int FMT>
int mx_quantize_rows_host(const void* x, int64_t x_rows, int x_f16, const int32_t* token_idx,
                             const int32_t* group_sizes, int64_t num_groups, int64_t rows,
                             int64_t k, void* out_q, void* out_sf, int64_t m_pad_capacity,
                             int32_t* dev_status, void* stream) {
  if (rows < 0 || k <= 0 || k % 128 || m_pad_capacity < 0 || m_pad_capacity % 128) return LMOE_BAD_SHAPE;
  if (group_sizes != nullptr && (num_groups <= 0 || num_groups > 4096)) return LMOE_BAD_SHAPE;
  if (group_sizes == nullptr && rows > m_pad_capacity) return LMOE_BAD_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out_q)) & 15)
    return LMOE_UNSUPPORTED;
  if (rows == 0) return LMOE_OK;
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t want = (rows * 32 + 255) / 256;
  const int blocks = static_cast<int>(std::min<int64_t>(want, int64_t(num_sms(current_device())) * 8));
  const size_t sh = group_sizes != nullptr ? static_cast<size_t>(2 * (num_groups + 1)) * 4 : 0;
  if (x_f16)
    mx_quantize_kernel<true, FMT><<<blocks, 256, sh, s>>>(
        static_cast<const uint16_t*>(x), x_rows, token_idx, group_sizes, (int)num_groups, rows,
        (int)k, m_pad_capacity, static_cast<uint8_t*>(out_q), static_cast<uint8_t*>(out_sf),
        dev_status);
  else
    mx_quantize_kernel<false, FMT><<<blocks, 256, sh, s>>>(
        static_cast<const uint16_t*>(x), x_rows, token_idx, group_sizes, (int)num_groups, rows,
        (int)k, m_pad_capacity, static_cast<uint8_t*>(out_q), static_cast<uint8_t*>(out_sf),
        dev_status);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

template <int FMT>
int mx_quantize_scatter_host(const void* x, int x_f16, const int32_t* slot_pos,
                                int64_t num_tokens, int64_t top_k, int64_t k,
                                const int32_t* group_sizes, int64_t num_groups, void* out_q,
                                void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                void* stream, int32_t* padded_pos = nullptr) {
  if (num_tokens < 0 || top_k <= 0 || top_k > 32 || k <= 0 || k % 128 || m_pad_capacity < 0 ||
      m_pad_capacity % 128)
    return LMOE_BAD_SHAPE;
  if (group_sizes == nullptr || slot_pos == nullptr || num_groups <= 0 || num_groups > 4096)
    return LMOE_BAD_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out_q)) & 15)
    return LMOE_UNSUPPORTED;
  if (num_tokens == 0) return LMOE_OK;
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t want = (num_tokens * ((k + 1023) / 1024) * 32 + 255) / 256;
  const int blocks = static_cast<int>(std::min<int64_t>(want, int64_t(num_sms(current_device())) * 8));
  const size_t sh = static_cast<size_t>(2 * (num_groups + 1)) * 4;
  if (x_f16)
    mx_quantize_scatter_kernel<true, FMT><<<blocks, 256, sh, s>>>(
        static_cast<const uint16_t*>(x), slot_pos, num_tokens, (int)top_k, group_sizes,
        (int)num_groups, (int)k, m_pad_capacity, static_cast<uint8_t*>(out_q),
        static_cast<uint8_t*>(out_sf), padded_pos, dev_status);
  else
    mx_quantize_scatter_kernel<false, FMT><<<blocks, 256, sh, s>>>(
        static_cast<const uint16_t*>(x), slot_pos, num_tokens, (int)top_k, group_sizes,
        (int)num_groups, (int)k, m_pad_capacity, static_cast<uint8_t*>(out_q),
        static_cast<uint8_t*>(out_sf), padded_pos, dev_status);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

// Grouped GEMM of padded block-scaled rows against prepared MXFP4 weights
// (the C entry points below): validation, tensor maps, launch.
template <int KIND>
int mx_grouped_gemm(const void* act_q, const void* act_sf, const void* w_packed, const void* w_sf,
                    const int32_t* group_sizes, void* out, int64_t m_pad, int64_t k, int64_t n_out,
                    int64_t g, int epi, float beta, float linear_beta, int round_gate_up,
                    int out_dtype, int64_t m_out, int32_t* dev_status, void* stream,
                    void* q_out = nullptr, void* q_sf = nullptr, int q_fmt = MX_E4M3) {
  // epi: 0 plain (out_dtype 0 bf16, 1 f32, 2 f16), 3 SiTU-GLU over interleaved
  // gate/up rows (n_out = intermediate; out_dtype 0 bf16, 2 f16)
  using C = MxCfg<KIND>;
  if (g <= 0 || g > kMxMaxGroups || m_pad < 0 || m_pad % 128 || k <= 0 || k % C::kBK ||
      n_out <= 0)
    return LMOE_BAD_SHAPE;
  if (epi != EPI_BF16 && epi != EPI_SITU) return LMOE_BAD_SHAPE;
  if (out_dtype < 0 || out_dtype > 2 || (epi == EPI_SITU && out_dtype == 1)) return LMOE_BAD_SHAPE;
  const int64_t n_weight = epi == EPI_SITU ? 2 * n_out : n_out;
  if (n_weight % 128 || (epi == EPI_SITU ? n_out % 16 : n_out % 8)) return LMOE_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w_packed) & 31) ||
      ((reinterpret_cast<uintptr_t>(act_q) | reinterpret_cast<uintptr_t>(out) |
        reinterpret_cast<uintptr_t>(act_sf) | reinterpret_cast<uintptr_t>(w_sf)) & 15))
    return LMOE_UNSUPPORTED;
  // m_out < 0: unpadded output of -m_out rows whose tail past sum(group_sizes)
  // is left as it is (a buffer sized by capacity)
  const bool zero_tail = m_out > 0;
  if (m_out < 0) m_out = -m_out;
  if (m_out >= (1ll << 31)) return LMOE_BAD_SHAPE;
  if (q_out != nullptr) {
    // quantised SiTU output: padded rows, bf16 values, the next GEMM's K
    // (the intermediate size) a multiple of 128 (of 256 for e2m1)
    if (epi != EPI_SITU || m_out != 0 || out_dtype != 0 || q_sf == nullptr) return LMOE_BAD_SHAPE;
    if (q_fmt != MX_E4M3 && q_fmt != MX_E2M1 && q_fmt != MX_E4M3_SPLIT) return LMOE_BAD_SHAPE;
    if (n_out % (q_fmt == MX_E2M1 ? 256 : 128)) return LMOE_BAD_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(q_sf)) & 15)
      return LMOE_UNSUPPORTED;
  }
  if (m_pad == 0) return LMOE_OK;
  if (m_pad >= (1ll << 31) || k >= (1 << 20)) return LMOE_BAD_SHAPE;
  MxArgs a{};
  a.m_out = static_cast<int>(m_out);
  a.zero_tail = zero_tail ? 1 : 0;
  a.q_out = static_cast<uint8_t*>(q_out);
  a.q_sf = static_cast<uint8_t*>(q_sf);
  a.q_fmt = q_fmt;
  a.group_sizes = group_sizes;
  a.status = dev_status;
  a.out = out;
  a.w_sf = static_cast<const uint8_t*>(w_sf);
  a.act_sf = static_cast<const uint8_t*>(act_sf);
  a.ldo = n_out;
  a.M_pad = static_cast<int>(m_pad);
  a.N = static_cast<int>(n_out);
  a.K = static_cast<int>(k);
  a.G = static_cast<int>(g);
  a.n_weight = static_cast<int>(n_weight);
  a.n_tiles = static_cast<int>(n_weight / kMxRows);
  a.beta = beta;
  a.linear_beta = linear_beta;
  a.inv_beta = beta != 0.f ? 1.f / beta : 0.f;
  a.inv_linear_beta = linear_beta != 0.f ? 1.f / linear_beta : 0.f;
  a.round_gate_up = round_gate_up;
  a.out_f16 = out_dtype == 2;
  CUtensorMap tw, tt, tt64;
  // activation row pitch in bytes: e4m3 (KIND_F8F6F4) or packed e2m1 (KIND_F4)
  const uint64_t act_pitch = KIND == KIND_F4 ? static_cast<uint64_t>(k / 2) : static_cast<uint64_t>(k);
  if (KIND == KIND_F4) {
    // packed codes as bytes, 128-byte rows of 256 codes, 128-byte swizzle
    const uint64_t kh = static_cast<uint64_t>(k / 2);
    if (!encode_tmap_u8_3d_sw128(&tw, w_packed, kh, static_cast<uint64_t>(n_weight),
                                 static_cast<uint64_t>(g), kh, static_cast<uint64_t>(n_weight) * kh,
                                 kMxRowBytes, kMxRows))
      return LMOE_LAUNCH_FAILED;
  } else if (!encode_tmap_fp4_unpacked_3d(&tw, w_packed, static_cast<uint64_t>(k),
                                          static_cast<uint64_t>(n_weight),
                                          static_cast<uint64_t>(g))) {
    return LMOE_LAUNCH_FAILED;
  }
  // token rows: one box of a full tile, or boxes of 64 rows for a partial one;
  // the split form's two planes (hi, lo) are the third coordinate
  if (C::kPlanes > 1) {
    const uint64_t mp = static_cast<uint64_t>(m_pad);
    if (!encode_tmap_u8_3d_sw128(&tt, act_q, act_pitch, mp, C::kPlanes, act_pitch,
                                 mp * act_pitch, kMxRowBytes, kMxTok) ||
        !encode_tmap_u8_3d_sw128(&tt64, act_q, act_pitch, mp, C::kPlanes, act_pitch,
                                 mp * act_pitch, kMxRowBytes, C::kBoxRows))
      return LMOE_LAUNCH_FAILED;
  } else if (!encode_tmap_u8_2d_sw128(&tt, act_q, act_pitch, static_cast<uint64_t>(m_pad),
                                      act_pitch, kMxRowBytes, kMxTok) ||
             !encode_tmap_u8_2d_sw128(&tt64, act_q, act_pitch, static_cast<uint64_t>(m_pad),
                                      act_pitch, kMxRowBytes, C::kBoxRows)) {
    return LMOE_LAUNCH_FAILED;
  }
  const int64_t tiles = (m_pad / kMxTok + g) * a.n_tiles;
  const int max_tiles = static_cast<int>(std::min<int64_t>(tiles, 1 << 30));
  auto s = static_cast<cudaStream_t>(stream);
  int rc;
  if (epi == EPI_SITU)
    rc = launch_mx<EPI_SITU, KIND>(tw, tt, tt64, a, max_tiles, s);
  else if (out_dtype == 1)
    rc = launch_mx<EPI_F32, KIND>(tw, tt, tt64, a, max_tiles, s);
  else
    rc = launch_mx<EPI_BF16, KIND>(tw, tt, tt64, a, max_tiles, s);
  return rc;
}

}  // namespace

}  // namespace lmoe

// --------------------------------------------------------------------------- C ABI
extern "C" {

int64_t lmoe_mxfp8_padded_rows(int64_t num_rows, int64_t num_groups) {
  if (num_rows < 0 || num_groups <= 0) return -1;
  // every group rounded up to 128 rows
  return (num_rows + 127 * (num_rows < num_groups ? num_rows : num_groups) + 127) / 128 * 128;
}

int lmoe_mxfp4_repack_blockscaled(const void* weight_packed, const void* weight_scale, int64_t g,
                                  int64_t n, int64_t k, int interleave_gateup,
                                  void* out_packed, void* out_sf, void* stream) {
  using namespace lmoe;
  if (g <= 0 || n <= 0 || k <= 0 || n % 128 || k % 128 || (interleave_gateup && n % 2))
    return LMOE_BAD_SHAPE;
  if (out_sf == nullptr || weight_scale == nullptr || (interleave_gateup && out_packed == nullptr))
    return LMOE_BAD_SHAPE;
  if ((reinterpret_cast<uintptr_t>(out_sf) | reinterpret_cast<uintptr_t>(weight_packed) |
       reinterpret_cast<uintptr_t>(out_packed)) & 15)
    return LMOE_UNSUPPORTED;
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t atoms = g * (n / 128) * (k / 128);
  const int blocks = static_cast<int>(std::min<int64_t>((atoms * 32 + 255) / 256, 4096));
  mx_repack_sf_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(weight_scale), (int)g,
                                             (int)n, (int)k, interleave_gateup,
                                             static_cast<uint8_t*>(out_sf));
  if (cudaGetLastError() != cudaSuccess) return LMOE_LAUNCH_FAILED;
  if (interleave_gateup) {
    mx_repack_rows_kernel<<<4096, 256, 0, s>>>(static_cast<const uint8_t*>(weight_packed), (int)g,
                                               (int)n, (int)k, static_cast<uint8_t*>(out_packed));
    if (cudaGetLastError() != cudaSuccess) return LMOE_LAUNCH_FAILED;
  }
  return LMOE_OK;
}

int lmoe_mxfp8_quantize_rows(const void* x, int64_t x_rows, int x_f16, const int32_t* token_idx,
                             const int32_t* group_sizes, int64_t num_groups, int64_t rows,
                             int64_t k, void* out_q, void* out_sf, int64_t m_pad_capacity,
                             int32_t* dev_status, void* stream) {
  return lmoe::mx_quantize_rows_host<lmoe::MX_E4M3>(x, x_rows, x_f16, token_idx, group_sizes,
                                                    num_groups, rows, k, out_q, out_sf,
                                                    m_pad_capacity, dev_status, stream);
}

int lmoe_mxfp4_quantize_rows(const void* x, int64_t x_rows, int x_f16, const int32_t* token_idx,
                             const int32_t* group_sizes, int64_t num_groups, int64_t rows,
                             int64_t k, void* out_q, void* out_sf, int64_t m_pad_capacity,
                             int32_t* dev_status, void* stream) {
  return lmoe::mx_quantize_rows_host<lmoe::MX_E2M1>(x, x_rows, x_f16, token_idx, group_sizes,
                                                    num_groups, rows, k, out_q, out_sf,
                                                    m_pad_capacity, dev_status, stream);
}

int lmoe_mxfp8_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                int64_t num_tokens, int64_t top_k, int64_t k,
                                const int32_t* group_sizes, int64_t num_groups, void* out_q,
                                void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                void* stream) {
  return lmoe::mx_quantize_scatter_host<lmoe::MX_E4M3>(x, x_f16, slot_pos, num_tokens, top_k, k,
                                                       group_sizes, num_groups, out_q, out_sf,
                                                       m_pad_capacity, dev_status, stream);
}

int lmoe_mxfp4_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                int64_t num_tokens, int64_t top_k, int64_t k,
                                const int32_t* group_sizes, int64_t num_groups, void* out_q,
                                void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                void* stream) {
  return lmoe::mx_quantize_scatter_host<lmoe::MX_E2M1>(x, x_f16, slot_pos, num_tokens, top_k, k,
                                                       group_sizes, num_groups, out_q, out_sf,
                                                       m_pad_capacity, dev_status, stream);
}

int lmoe_bf16split_quantize_rows(const void* x, int64_t x_rows, int x_f16,
                                 const int32_t* token_idx, const int32_t* group_sizes,
                                 int64_t num_groups, int64_t rows, int64_t k, void* out_q,
                                 void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                 void* stream) {
  return lmoe::mx_quantize_rows_host<lmoe::MX_E4M3_SPLIT>(
      x, x_rows, x_f16, token_idx, group_sizes, num_groups, rows, k, out_q, out_sf,
      m_pad_capacity, dev_status, stream);
}

int lmoe_bf16split_quantize_scatter(const void* x, int x_f16, const int32_t* slot_pos,
                                    int64_t num_tokens, int64_t top_k, int64_t k,
                                    const int32_t* group_sizes, int64_t num_groups, void* out_q,
                                    void* out_sf, int64_t m_pad_capacity, int32_t* dev_status,
                                    void* stream) {
  return lmoe::mx_quantize_scatter_host<lmoe::MX_E4M3_SPLIT>(
      x, x_f16, slot_pos, num_tokens, top_k, k, group_sizes, num_groups, out_q, out_sf,
      m_pad_capacity, dev_status, stream);
}

int lmoe_bf16split_quantize_scatter_positions(const void* x, int x_f16, const int32_t* slot_pos,
                                              int64_t num_tokens, int64_t top_k, int64_t k,
                                              const int32_t* group_sizes, int64_t num_groups,
                                              void* out_q, void* out_sf, int64_t m_pad_capacity,
                                              int32_t* padded_slot_pos, int32_t* dev_status,
                                              void* stream) {
  if (padded_slot_pos == nullptr) return LMOE_BAD_SHAPE;
  return lmoe::mx_quantize_scatter_host<lmoe::MX_E4M3_SPLIT>(
      x, x_f16, slot_pos, num_tokens, top_k, k, group_sizes, num_groups, out_q, out_sf,
      m_pad_capacity, dev_status, stream, padded_slot_pos);
}

int lmoe_mxfp8_pad_positions(const int32_t* positions, int64_t n, const int32_t* group_sizes,
                             int64_t num_groups, int32_t* out, void* stream) {
  using namespace lmoe;
  if (n < 0 || num_groups <= 0 || num_groups > 4096 || group_sizes == nullptr) return LMOE_BAD_SHAPE;
  if (n == 0) return LMOE_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 1024));
  mx_pad_positions_kernel<<<blocks, 256, static_cast<size_t>(2 * (num_groups + 1)) * 4,
                            static_cast<cudaStream_t>(stream)>>>(positions, n, group_sizes,
                                                                 (int)num_groups, out);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_mxfp8_mxfp4_grouped_gemm(const void* act_q, const void* act_sf, const void* w_packed,
                                  const void* w_sf, const int32_t* group_sizes, void* out,
                                  int64_t m_pad, int64_t k, int64_t n_out, int64_t g, int epi,
                                  float beta, float linear_beta, int round_gate_up, int out_dtype,
                                  int32_t* dev_status, void* stream) {
  return lmoe::mx_grouped_gemm<lmoe::KIND_F8F6F4>(act_q, act_sf, w_packed, w_sf, group_sizes, out,
                                                 m_pad, k, n_out, g, epi, beta, linear_beta,
                                                 round_gate_up, out_dtype, 0, dev_status, stream);
}

int lmoe_mxfp4_mxfp4_grouped_gemm(const void* act_q, const void* act_sf, const void* w_packed,
                                  const void* w_sf, const int32_t* group_sizes, void* out,
                                  int64_t m_pad, int64_t k, int64_t n_out, int64_t g, int epi,
                                  float beta, float linear_beta, int round_gate_up, int out_dtype,
                                  int32_t* dev_status, void* stream) {
  return lmoe::mx_grouped_gemm<lmoe::KIND_F4>(act_q, act_sf, w_packed, w_sf, group_sizes, out,
                                             m_pad, k, n_out, g, epi, beta, linear_beta,
                                             round_gate_up, out_dtype, 0, dev_status, stream);
}

int lmoe_blockscaled_gateup_situ_quantized(const void* act_q, const void* act_sf, int act_kind,
                                           const void* w_packed, const void* w_sf,
                                           const int32_t* group_sizes, int64_t m_pad, int64_t k,
                                           int64_t inter, int64_t g, float beta,
                                           float linear_beta, int round_gate_up, int out_fmt,
                                           void* out_q, void* out_sf, int32_t* dev_status,
                                           void* stream) {
  using namespace lmoe;
  if (out_q == nullptr) return LMOE_BAD_SHAPE;
  switch (act_kind) {
    case 0:
      return mx_grouped_gemm<KIND_F8F6F4>(act_q, act_sf, w_packed, w_sf, group_sizes, nullptr,
                                          m_pad, k, inter, g, EPI_SITU, beta, linear_beta,
                                          round_gate_up, 0, 0, dev_status, stream, out_q, out_sf,
                                          out_fmt);
    case 1:
      return mx_grouped_gemm<KIND_F4>(act_q, act_sf, w_packed, w_sf, group_sizes, nullptr, m_pad,
                                      k, inter, g, EPI_SITU, beta, linear_beta, round_gate_up, 0, 0,
                                      dev_status, stream, out_q, out_sf, out_fmt);
    case 2:
      return mx_grouped_gemm<KIND_F8_SPLIT>(act_q, act_sf, w_packed, w_sf, group_sizes, nullptr,
                                            m_pad, k, inter, g, EPI_SITU, beta, linear_beta,
                                            round_gate_up, 0, 0, dev_status, stream, out_q, out_sf,
                                            out_fmt);
    default:
      return LMOE_BAD_SHAPE;
  }
}

int lmoe_bf16split_mxfp4_grouped_gemm(const void* act_q, const void* act_sf, const void* w_packed,
                                      const void* w_sf, const int32_t* group_sizes, void* out,
                                      int64_t m_pad, int64_t k, int64_t n_out, int64_t g, int epi,
                                      float beta, float linear_beta, int round_gate_up,
                                      int out_dtype, int64_t m_out, int32_t* dev_status,
                                      void* stream) {
  return lmoe::mx_grouped_gemm<lmoe::KIND_F8_SPLIT>(act_q, act_sf, w_packed, w_sf, group_sizes,
                                                   out, m_pad, k, n_out, g, epi, beta,
                                                   linear_beta, round_gate_up, out_dtype, m_out,
                                                   dev_status, stream);
}

}  // extern "C"
