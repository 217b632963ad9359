// MXFP4 grouped GEMM with the weights as the UMMA A operand ("weights-major").
//
//   out[r, :] = lhs[r, :] @ dequant(w[g(r)])^T     r in group g's row range
//
// Same contract as the MXFP4 form of grouped_gemm.cu (the dequant-then-matmul
// of 05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67 and the fused SiTU-GLU of
// kimi_k3_latent_moe_ragged_dot.py:610-723), with the roles of the operands
// swapped: a tile is 128 weight rows (UMMA M) x 256 token rows (UMMA N), so
// each expanded weight tile feeds twice as many tokens as in the token-major
// kernel, halving the expansion work and the shared-memory bytes it writes
// per FLOP.
//
// Three rings, so that expanding the weights never waits on the token loads:
//   token ring   (4 x 32 KB)  256 token rows x 64 K, 128B swizzle  -> UMMA B
//   packed ring  (4 x 4 KB)   e2m1 codes of the tile's 128 weight rows
//   A ring       (4 x 16 KB)  expanded weights, K-major 128B swizzle -> UMMA A
// The packed ring has its own producer and runs ahead of the token ring, so a
// weight tile is expanded well before the MMA that needs it.
//
//   warp 0      token producer (TMA).
//   warp 1      TMEM owner and UMMA issuer: M=128, N=256, K=16, f32 in TMEM,
//               two accumulators (2 x 256 columns).  A tile with fewer token
//               rows (the last one of a group) runs its MMAs with N = its row
//               count rounded up to 16, and its token boxes cover only those
//               rows, so a group of 40 rows costs 48 columns of tensor time,
//               not 256.
//   warps 2-5   epilogue.  TMEM lane = weight row, column = token: each warp
//               reads its 32 lanes, transposes through a small shared-memory
//               tile and stores token-major rows.
//   warps 6-13  dequant: two groups of 4 warps on alternate K steps, one
//               thread per weight row, into the swizzled K-major A tile.
//   warp 14     packed-code producer (TMA).
// EPI_SITU: the A tile interleaves gate and up rows (row 2i = gate feature i,
// row 2i+1 = up feature i), so each (gate, up) pair sits in adjacent lanes of
// one warp and meets through one shuffle.
#include <cuda.h>

#include <cfloat>
#include <cstdlib>
#include <mutex>

#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

namespace {

constexpr int kTokTile = 256;  // UMMA N: token rows per tile
constexpr int kWRows = 128;    // UMMA M: weight rows per tile
constexpr int kTStages = 4;    // token ring
constexpr int kPStages = 4;    // packed-code ring
constexpr int kDStages = 4;    // expanded-weight (A) ring
constexpr int kSwMaxGroups = kSwapMaxGroups;  // schedule arrays in shared memory
constexpr int kDeqWarps = 8;           // two groups of 4, alternate K steps
constexpr int kPkWarp = 6 + kDeqWarps;  // packed-code producer
constexpr int kSwThreads = 32 * (kPkWarp + 1);
static_assert(kPStages % 2 == 0 && kDStages % 2 == 0, "each ring slot belongs to one dequant group");

struct SwCfg {
  static constexpr int kTokBytes = kTokTile * kBK * 2;     // 32 KB
  // A full tile's token rows are one 256-row box (32 KB); a partial tile
  // copies boxes of 64 rows (8 KB, a multiple of the 1 KB 128-byte-swizzle
  // atom, so stacked boxes form the same layout), only as many as it needs.
  // One thread issues a copy every few hundred cycles at best, so a step's
  // copies are kept few and large.
  static constexpr int kTokBoxRows = 64;
  static constexpr int kTokBoxBytes = kTokBoxRows * kBK * 2;
  static constexpr int kPackedBytes = kWRows * (kBK / 2);  // 4 KB
  static constexpr int kABytes = kWRows * kBK * 2;         // 16 KB
  static constexpr int kWarpStage = 1024;                  // epilogue transpose tile per warp
  static constexpr int kOutStageBytes = 4 * kWarpStage;
  static constexpr int kTmemCols = 2 * kTokTile;
  static constexpr int kSchedBytes = 2 * (kSwMaxGroups + 1) * 4;
  static constexpr int kNumBars = 2 * kTStages + 2 * kPStages + 2 * kDStages + 5;
  static constexpr size_t kSmem = 1024 + size_t(kTStages) * kTokBytes +
                                  size_t(kPStages) * kPackedBytes + size_t(kDStages) * kABytes +
                                  kOutStageBytes + kSchedBytes + 8 * kNumBars + 16;
  static_assert(kTokBytes % 1024 == 0 && kABytes % 1024 == 0 && kPackedBytes % 1024 == 0,
                "1024-byte aligned stages");
  // the schedule's scan scratch lives in the (not yet used) epilogue staging
  static_assert(kOutStageBytes >= 2 * kSwThreads * 4, "scan scratch");
  static_assert(kSmem <= 232448, "shared memory");
};

// weight row (N index of the checkpoint layout) behind row r of the A tile
template <int EPI>
__device__ __forceinline__ int weight_row(const GemmArgs& a, int n_tile, int r) {
  if (EPI == EPI_SITU) return ((r & 1) ? a.up_offset : 0) + n_tile * (kWRows / 2) + (r >> 1);
  return n_tile * kWRows + r;
}

// row of the packed stage holding A row r (the producer loads two 64-row boxes)
template <int EPI>
__device__ __forceinline__ int packed_row(int r) {
  return EPI == EPI_SITU ? (r & 1) * 64 + (r >> 1) : r;
}

// 16-byte chunk swizzle of a staged row: 8 consecutive rows (one quarter-warp
// of 16-byte reads) start on distinct banks
template <int kChunks>
__device__ __forceinline__ int swz_key(int row) {
  return kChunks == 4 ? ((row >> 1) & 3) : (row & 7);
}

__device__ __forceinline__ uint16_t out16(float v, int out_f16) {
  if (out_f16) {
    const __half h = __float2half_rn(bf16_round_f(v));
    return *reinterpret_cast<const uint16_t*>(&h);
  }
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<const uint16_t*>(&b);
}

struct RingPos {
  uint32_t stage = 0, phase = 0;
  template <int N>
  __device__ __forceinline__ void next() {
    if (++stage == N) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

template <int BF, int EPI>
__global__ void __launch_bounds__(kSwThreads, 1)
    mxfp4_swap_kernel(const __grid_constant__ CUtensorMap tmTok,
                      const __grid_constant__ CUtensorMap tmTok64,
                      const __grid_constant__ CUtensorMap tmW, const GemmArgs args) {
  using C = SwCfg;
  constexpr bool kF16 = BF == B_MXFP4F16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* tstages = smem;
  uint8_t* pstages = tstages + kTStages * C::kTokBytes;
  uint8_t* astages = pstages + kPStages * C::kPackedBytes;
  uint8_t* ostage = astages + kDStages * C::kABytes;
  int32_t* row_off = reinterpret_cast<int32_t*>(ostage + C::kOutStageBytes);
  int32_t* tile_start = row_off + (kSwMaxGroups + 1);
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_start + (kSwMaxGroups + 1));
  uint64_t* tok_full = bars;
  uint64_t* tok_empty = tok_full + kTStages;
  uint64_t* pk_full = tok_empty + kTStages;
  uint64_t* pk_empty = pk_full + kPStages;   // dequant warps done reading the codes
  uint64_t* a_ready = pk_empty + kPStages;   // expanded A tile written (dequant -> MMA)
  uint64_t* a_empty = a_ready + kDStages;    // expanded A tile consumed (MMA -> dequant)
  uint64_t* acc_full = a_empty + kDStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = args.G;

  if (threadIdx.x == 0) *abort_flag = 0;
  int32_t* scan = reinterpret_cast<int32_t*>(ostage);
  const int total = build_schedule<kTokTile>(args, row_off, tile_start, scan, scan + kSwThreads);
  if (total < 0) return;  // uniform across the CTA; nothing allocated yet

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(smem_u32(tok_full + s), 1);
      mbar_init(smem_u32(tok_empty + s), 1);
    }
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(smem_u32(pk_full + s), 1);
      mbar_init(smem_u32(pk_empty + s), kDeqWarps / 2);  // the step's dequant group
    }
    for (int s = 0; s < kDStages; ++s) {
      mbar_init(smem_u32(a_ready + s), kDeqWarps / 2);  // the step's dequant group
      mbar_init(smem_u32(a_empty + s), 1);  // UMMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(acc_full + b), 1);
      mbar_init(smem_u32(acc_empty + b), 128);
    }
    mbar_init(smem_u32(drain), 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmTok);
    tma_prefetch_desc(&tmTok64);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = args.K / kBK;

  if (warp == 0 || warp == kPkWarp) {
    // ------------------------------------------------------------ producers
    // warp 0: token tiles; warp kPkWarp: packed codes (two 64-row boxes per step)
    if (lane == 0) {
      const bool tok = warp == 0;
      uint64_t* fullb = tok ? tok_full : pk_full;
      uint64_t* emptyb = tok ? tok_empty : pk_empty;
      const uint32_t nst = tok ? kTStages : kPStages;
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile<kTokTile>(tile_start, row_off, G, args.n_tiles, t);
        const int wb0 = weight_row<EPI>(args, tc.n_tile, 0);
        const int wb1 = EPI == EPI_SITU ? weight_row<EPI>(args, tc.n_tile, 1) : wb0 + 64;
        // token boxes this tile needs (a tile holds at least one row)
        const int tile_rows = min(kTokTile, tc.row_end - tc.row0);
        const int n_box = (tile_rows + C::kTokBoxRows - 1) / C::kTokBoxRows;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(emptyb + stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(fullb + stage);
          if (tok) {
            const uint32_t t_dst = smem_u32(tstages + stage * C::kTokBytes);
            if (tile_rows == kTokTile) {
              mbar_arrive_expect_tx(fb, C::kTokBytes);
              tma_load_2d(t_dst, &tmTok, fb, kb * kBK, tc.row0);
            } else {
              mbar_arrive_expect_tx(fb, n_box * C::kTokBoxBytes);
              for (int i = 0; i < n_box; ++i)
                tma_load_2d(t_dst + i * C::kTokBoxBytes, &tmTok64, fb, kb * kBK,
                            tc.row0 + i * C::kTokBoxRows);
            }
          } else {
            mbar_arrive_expect_tx(fb, C::kPackedBytes);
            const uint32_t p_dst = smem_u32(pstages + stage * C::kPackedBytes);
            tma_load_3d(p_dst, &tmW, fb, kb * (kBK / 2), wb0, tc.g);
            tma_load_3d(p_dst + 64 * (kBK / 2), &tmW, fb, kb * (kBK / 2), wb1, tc.g);
          }
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == nst) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // abort: let every copy already issued land before the CTA retires
        for (uint32_t s = 0; s < nst; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(fullb + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      RingPos ts, ds;
      uint32_t acc = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        // UMMA N: the tile's token rows rounded up to 16 (N % 16 == 0 for M = 128)
        const TileCoord tc = decode_tile<kTokTile>(tile_start, row_off, G, args.n_tiles, t);
        const uint32_t n_mma = (min(kTokTile, tc.row_end - tc.row0) + 15) & ~15;
        const uint32_t idesc =
            kF16 ? idesc_f16_f32(kWRows, n_mma, false) : idesc_bf16_f32(kWRows, n_mma, false);
        if (!mbar_wait(smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTokTile;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(a_ready + ds.stage), ds.phase, abort_flag, args.status) ||
              !mbar_wait(smem_u32(tok_full + ts.stage), ts.phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(astages + ds.stage * C::kABytes);
          const uint32_t b_addr = smem_u32(tstages + ts.stage * C::kTokBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(tok_empty + ts.stage));
          umma_commit(smem_u32(a_empty + ds.stage));
          ts.next<kTStages>();
          ds.next<kDStages>();
        }
        if (!ok) break;
        umma_commit(smem_u32(acc_full + acc));
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        // abort: wait for every UMMA already issued before TMEM is released
        umma_commit(smem_u32(drain));
        mbar_drain(smem_u32(drain), 0);
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t stg = smem_u32(ostage + q * C::kWarpStage);
    constexpr int esize = (EPI == EPI_F32) ? 4 : 2;
    uint32_t acc = 0, acc_phase = 0;
    float f16_peak = 0.f;  // largest magnitude stored as f16 by the plain epilogue
    float f16_low = FLT_MAX;  // smallest nonzero peak of a stored f16 SiTU run
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileCoord tc = decode_tile<kTokTile>(tile_start, row_off, G, args.n_tiles, t);
      if (!mbar_wait(smem_u32(acc_full + acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kTokTile;
#pragma unroll 1
      for (int c = 0; c < kTokTile / 32; ++c) {
        const int tok0 = tc.row0 + c * 32;
        if (tok0 >= tc.row_end) break;  // warp-uniform
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        if (EPI == EPI_SITU) {
          // lanes 2i / 2i+1 hold gate / up of feature i; the even lane
          // finishes tokens 0-15 of the chunk, the odd lane tokens 16-31.
          // Staged [token][16 features] (32-byte rows).
          static_assert(C::kWarpStage >= 1024, "SiTU staging");
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
            sts_u16(stg + 2u * ((odd * 16 + j) * 16 + (lane >> 1)), out16(o, args.out_f16));
          }
          __syncwarp();
          const int tok = tok0 + lane;
          const int f0 = tc.n_tile * (kWRows / 2) + q * 16;
          if (tok < tc.row_end) {
            uint16_t* orow =
                reinterpret_cast<uint16_t*>(args.out) + static_cast<int64_t>(tok) * args.ldo + f0;
            const uint4 s0 = lds_v4(stg + lane * 32), s1 = lds_v4(stg + lane * 32 + 16);
            if (f0 + 8 <= args.N) *reinterpret_cast<uint4*>(orow) = s0;
            if (f0 + 16 <= args.N) *reinterpret_cast<uint4*>(orow + 8) = s1;
            if (args.out_f16) {
              // f16 range guard: this token's 16 activations all tiny
              const float run = fmaxf(f16x8_peak(s0), f16x8_peak(s1));
              if (run > 0.f) f16_low = fminf(f16_low, run);
            }
          }
          __syncwarp();
        } else {
          // lane = output feature, v[j] = token j.  Stage [token][feature]
          // rows of 32 features (64 B, or 128 B for f32) in passes of
          // kWarpStage bytes, 16-byte chunks swizzled by the staged row.
          constexpr int kRowBytes = 32 * esize;
          constexpr int kChunks = kRowBytes / 16;
          constexpr int kRows = C::kWarpStage / kRowBytes;  // token rows per pass
          static_assert(kRows >= 8 && 32 % kRows == 0, "staging rows");
          const int byte = lane * esize;
          const int f0 = tc.n_tile * kWRows + q * 32;
#pragma unroll
          for (int p0 = 0; p0 < 32; p0 += kRows) {
            const uint32_t dst0 = stg + (byte & 15);
            if (EPI == EPI_F32) {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj)
                sts_u32(dst0 + jj * kRowBytes + (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4), v[p0 + jj]);
            } else if (args.out_f16) {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj) {
                f16_peak = fmaxf(f16_peak, fabsf(__uint_as_float(v[p0 + jj])));
                sts_u16(dst0 + jj * kRowBytes + (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4),
                        out16(__uint_as_float(v[p0 + jj]), 1));
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj)
                sts_u16(dst0 + jj * kRowBytes + (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4),
                        out16(__uint_as_float(v[p0 + jj]), 0));
            }
            __syncwarp();
            const int tok = tok0 + p0 + lane;
            if (lane < kRows && tok < tc.row_end) {
              uint8_t* orow =
                  args.row_dest != nullptr
                      ? reinterpret_cast<uint8_t*>(args.row_dest[tok]) + static_cast<int64_t>(f0) * esize
                      : reinterpret_cast<uint8_t*>(args.out) +
                            (static_cast<int64_t>(tok) * args.ldo + f0) * esize;
#pragma unroll
              for (int cc = 0; cc < kChunks; ++cc) {
                if (f0 + (cc + 1) * (16 / esize) <= args.N)
                  *reinterpret_cast<uint4*>(orow + cc * 16) =
                      lds_v4(stg + lane * kRowBytes + ((cc ^ swz_key<kChunks>(lane)) * 16));
              }
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(acc_empty + acc));
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    // f16 range guard: above 65504 (the SiTU activations are bounded by
    // beta * linear_beta, so only the plain epilogue can overflow), or a run
    // of SiTU activations too small for f16 to carry accurately
    if (__any_sync(0xffffffffu, (EPI == EPI_BF16 && bf16_round_f(f16_peak) > kF16Max) ||
                                    (EPI == EPI_SITU && f16_low < kF16RunMin)) &&
        lane == 0)
      record_status(args.status, kF16Range);
    // rows scattered to other GPUs: make them visible system-wide before the
    // kernel ends (the next kernel on the stream signals their arrival)
    if (args.row_dest != nullptr) __threadfence_system();
    // rows at or past sum(group_sizes) are zero (ragged_dot semantics)
    if (args.zero_tail) {
      const int64_t row_bytes = static_cast<int64_t>(args.N) * esize;
      const int64_t chunks_per_row = row_bytes / 16;
      const int64_t first = row_off[G];
      const int64_t n_chunks = (args.M - first) * chunks_per_row;
      const int64_t pitch = args.ldo * esize;
      const int etid = threadIdx.x - 64;
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * 128 + etid; i < n_chunks;
           i += static_cast<int64_t>(gridDim.x) * 128) {
        const int64_t rr = first + i / chunks_per_row;
        const int64_t cc = i % chunks_per_row;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(args.out) + rr * pitch + cc * 16) =
            make_uint4(0, 0, 0, 0);
      }
    }
  } else if (warp < 6 + kDeqWarps) {
    // ------------------------------------------------------------ MXFP4 dequant
    // The CTA's K steps form one sequence (its tiles in schedule order, num_kb
    // steps each).  Two groups of 4 warps take alternate steps; within a
    // group, thread i expands A row i: 64 codes (32 packed bytes, two E8M0
    // blocks) -> the 8 16-byte chunks of its 128-byte swizzled row (chunk c
    // lands in slot c ^ (r & 7)).  Each group has two MMA steps' time per
    // step and fences once per step.  The packed and A slots of a step belong
    // to its group alone (both ring sizes are even), and the group uses them
    // in order, so the parity waits see their phases in order.
    // The codes are expanded into registers (and their packed slot released)
    // before waiting for a free A slot; the scale bytes of the group's next
    // step are fetched one step ahead.  The packed slot is refilled by TMA
    // (async proxy) after generic-proxy reads, so each thread consumes its
    // loaded codes and issues fence.proxy.async before the release: without
    // it a refill could land before a read and corrupt that row's K step.
    const int grp = (warp - 6) / 4;
    const int r = ((warp - 6) % 4) * 32 + lane;
    const int kgroups = args.K / 32;
    const int my_tiles = blockIdx.x < static_cast<unsigned>(total)
                             ? (total - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x
                             : 0;
    const int n_steps = my_tiles * num_kb;
    // scale row of A row r for the tile of the last looked-up step (decoded
    // once per tile); nullptr when the row lies past the weight
    int cached_tile = -1;
    const uint16_t* srow = nullptr;
    auto load_scale = [&](int st) -> uint32_t {  // two scale bytes of row r for step st
      const int ti = st / num_kb;
      if (ti != cached_tile) {
        cached_tile = ti;
        const TileCoord tc =
            decode_tile<kTokTile>(tile_start, row_off, G, args.n_tiles, blockIdx.x + ti * gridDim.x);
        const int w_row = weight_row<EPI>(args, tc.n_tile, r);
        const bool row_in = EPI == EPI_SITU
                                ? (tc.n_tile * (kWRows / 2) + (r >> 1)) < args.up_offset
                                : w_row < args.n_weight;
        srow = row_in ? reinterpret_cast<const uint16_t*>(
                            args.scales +
                            (static_cast<int64_t>(tc.g) * args.n_weight + w_row) * kgroups)
                      : nullptr;
      }
      return srow != nullptr ? __ldg(srow + (st - ti * num_kb)) : 0x7F7Fu;
    };
    // expand step st (scale bytes sc, loaded two of the group's steps earlier)
    auto expand = [&](int st, uint32_t sc) -> bool {
      const uint32_t pslot = st % kPStages, pph = (st / kPStages) & 1;
      if (!mbar_wait(smem_u32(pk_full + pslot), pph, abort_flag, args.status)) return false;
      const uint32_t src = smem_u32(pstages + pslot * C::kPackedBytes + packed_row<EPI>(r) * (kBK / 2));
      const uint4 p0 = lds_v4(src), p1 = lds_v4(src + 16);
      const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      uint4 dq[8];
      if (kF16) {
        const uint32_t b0 = e8m0_to_f16_bits(sc & 0xFFu), b1 = e8m0_to_f16_bits(sc >> 8);
        const uint32_t s0 = b0 | (b0 << 16), s1 = b1 | (b1 << 16);
#pragma unroll
        for (int c = 0; c < 8; ++c) dq[c] = dequant_e2m1x8_f16(words[c], c < 4 ? s0 : s1);
      } else {
        const uint32_t b0 = e8m0_to_bf16_bits(sc & 0xFFu), b1 = e8m0_to_bf16_bits(sc >> 8);
        const uint32_t s0 = b0 | (b0 << 16), s1 = b1 | (b1 << 16);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t sv = c < 4 ? s0 : s1;
          dq[c] = dequant_e2m1x8(words[c], *reinterpret_cast<const __nv_bfloat162*>(&sv));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(pk_empty + pslot));
      const uint32_t aslot = st % kDStages, aph = (st / kDStages) & 1;
      if (!mbar_wait(smem_u32(a_empty + aslot), aph ^ 1u, abort_flag, args.status)) return false;
      const uint32_t arow = smem_u32(astages + aslot * C::kABytes + r * 128);
#pragma unroll
      for (int c = 0; c < 8; ++c) sts_v4(arow + ((c ^ (r & 7)) << 4), dq[c]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(a_ready + aslot));
      return true;
    };
    // the group's steps are st0, st0 + 2, ...; scale bytes two steps ahead,
    // alternating between two registers (no copy that would wait on a load)
    uint32_t sa = grp < n_steps ? load_scale(grp) : 0x7F7Fu;
    uint32_t sb = grp + 2 < n_steps ? load_scale(grp + 2) : 0x7F7Fu;
    for (int st = grp; st < n_steps; st += 4) {
      if (!expand(st, sa)) break;
      if (st + 4 < n_steps) sa = load_scale(st + 4);
      if (st + 2 >= n_steps || !expand(st + 2, sb)) break;
      if (st + 6 < n_steps) sb = load_scale(st + 6);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int BF, int EPI>
int launch_swap(const CUtensorMap& tok, const CUtensorMap& tok64, const CUtensorMap& w,
                const GemmArgs& a, int max_tiles, cudaStream_t stream) {
  auto kern = mxfp4_swap_kernel<BF, EPI>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static uint64_t configured = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(configured & (1ull << dev))) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(SwCfg::kSmem)) != cudaSuccess)
        return kLaunchFailed;
      configured |= 1ull << dev;
    }
  }
  const int grid = max(1, min(num_sms(dev), max_tiles));
  kern<<<grid, kSwThreads, SwCfg::kSmem, stream>>>(tok, tok64, w, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

template <int BF>
int launch_swap_epi(int epi, const CUtensorMap& tok, const CUtensorMap& tok64,
                    const CUtensorMap& w, const GemmArgs& a, int max_tiles, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_swap<BF, EPI_BF16>(tok, tok64, w, a, max_tiles, s);
    case EPI_F32: return launch_swap<BF, EPI_F32>(tok, tok64, w, a, max_tiles, s);
    case EPI_SITU: return launch_swap<BF, EPI_SITU>(tok, tok64, w, a, max_tiles, s);
    default: return kUnsupported;
  }
}

}  // namespace

// Weights-major MXFP4 grouped GEMM.  `a` carries the shapes and epilogue
// parameters (validated by the caller); its n_tiles is set here.
int mxfp4_swap_gemm(const void* lhs, const void* packed, GemmArgs a, int epi, int lhs_f16,
                    cudaStream_t stream) {
  static const bool pair = [] {
    const char* e = std::getenv("LMOE_MXFP4_PAIR");
    return e != nullptr && e[0] == '1';
  }();
  if (pair) return mxfp4_pair_gemm(lhs, packed, a, epi, lhs_f16, stream);
  CUtensorMap tok, tok64, w;
  // tokens: dims {K, M}, boxes {64, 256} (full tiles) and {64, 64} (partial
  // tiles), 128-byte swizzle (K-major UMMA B)
  if (!encode_tmap_bf16_2d(&tok, lhs, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M),
                           static_cast<uint64_t>(a.K) * 2, kBK, kTokTile) ||
      !encode_tmap_bf16_2d(&tok64, lhs, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M),
                           static_cast<uint64_t>(a.K) * 2, kBK, SwCfg::kTokBoxRows))
    return kLaunchFailed;
  // packed codes: dims {K/2 bytes, n_weight, G}, box {32 bytes, 64 rows}
  const int64_t kh = a.K / 2;
  if (!encode_tmap_u8_3d(&w, packed, kh, a.n_weight, a.G, kh, static_cast<int64_t>(a.n_weight) * kh,
                         kBK / 2, 64))
    return kLaunchFailed;
  const int feat = epi == EPI_SITU ? kWRows / 2 : kWRows;  // output features per tile
  a.n_tiles = (a.N + feat - 1) / feat;
  const int64_t t = ((static_cast<int64_t>(a.M) + kTokTile - 1) / kTokTile + a.G) * a.n_tiles;
  const int max_tiles = static_cast<int>(t < (1 << 30) ? t : (1 << 30));
  return lhs_f16 ? launch_swap_epi<B_MXFP4F16>(epi, tok, tok64, w, a, max_tiles, stream)
                 : launch_swap_epi<B_MXFP4>(epi, tok, tok64, w, a, max_tiles, stream);
}

}  // namespace lmoe
