// Persistent grouped GEMM (ragged_dot) on sm_100a tensor cores.
//
//   out[r, :] = lhs[r, :] @ rhs[g(r)]        r in [off_g, off_g + group_sizes[g])
//
// Semantics follow `tokamax.ragged_dot(lhs, rhs, group_sizes)` as the reference
// calls it (05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:358-369),
// i.e. the per-expert loop of kimi_k3_latent_moe_reference.py:383-406: groups
// are contiguous row ranges in order, rows at or past sum(group_sizes) are
// zero.  group_sizes lives in device memory and is read only on the device
// (no host synchronisation).
//
// Design (one CTA per SM):
//   warp 0      TMA producer: A tile (128 rows x 64 K, bf16, 128B swizzle) and
//               the B operand of the stage, completion on an mbarrier.
//   warp 1      TMEM owner and UMMA issuer: tcgen05.mma kind::f16, M=128, N=BN,
//               K=16 per instruction, f32 accumulator in TMEM, two accumulator
//               buffers so the epilogue of tile i overlaps the MMAs of tile i+1.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns one
//               32-lane quarter of TMEM), fused activation, predicated stores of
//               the rows that belong to the tile's group.
//   warps 6-13  (MXFP4 weights only) dequant: expand the packed e2m1 codes the
//               TMA brought into shared memory, times their E8M0 block scale,
//               into the swizzled bf16 operand layout the UMMA reads.  The
//               weights stay packed in HBM (4.25 bits per weight read).
// B operand formats:
//   B_KMAJOR   bf16 (G, N, K)          one TMA box per half tile
//   B_NMAJOR   bf16 (G, K, N)          the reference's layout; MN-major UMMA operand
//   B_MXFP4    u8 (G, N, K/2) codes (low nibble = even k) + u8 (G, N, K/32) E8M0
//              scales (the checkpoint's (out, in) layout, 05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67)
// The tile schedule (group -> row offset, group -> first tile) is an in-CTA
// prefix sum over group_sizes; tiles are (group, m-tile, n-tile) with n
// fastest and are dealt round-robin to the persistent CTAs.  Empty groups own
// no tiles, so their weights are never read.
//
// Epilogues:
//   EPI_BF16      out = bf16(acc)
//   EPI_F32       out = acc (f32)
//   EPI_BF16_ADD  out = bf16(bf16(acc) + addend)    (residual add, bf16 rounding of each op)
//   EPI_SITU      B tile = [gate cols | up cols] of a fused [gate | up] weight;
//                 out = bf16(situ(g, u)) with g, u = acc (rounded to bf16 first
//                 when round_gate_up, the convention of
//                 kimi_k3_latent_moe_reference.py:296-310 / own_gateup_situ_pallas_kernel.py:116-125)
#include <cuda.h>

#include <cfloat>
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

constexpr int kBM = 128;

template <int BN, int STAGES, int BF, int EPI>
struct GemmCfg {
  static constexpr int kThreads = is_expand(BF) ? 448 : 192;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kPackedBytes = is_mx(BF) ? BN * (kBK / 2) : (BF == B_FP8 ? BN * kBK : 0);
  static constexpr int kStageBytes = kABytes + (is_expand(BF) ? kPackedBytes : kBBytes);
  static constexpr int kDStages = is_expand(BF) ? 2 : 0;
  static constexpr int kDAlloc = kDStages > 0 ? kDStages : 1;  // barrier slots
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSchedBytes = 2 * (kMaxGroups + 1) * 4 + 2 * kThreads * 4;
  static constexpr int kBarBytes = 8 * (2 * STAGES + 2 * kDAlloc + 5) + 16;
  static constexpr size_t kSmem = 1024 + size_t(STAGES) * kStageBytes +
                                  size_t(kDStages) * kBBytes + kSchedBytes + kBarBytes;
  static_assert(BN % 128 == 0 && BN <= 256, "BN");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM columns must be a power of two");
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned for SW128");
  static_assert(kSmem <= 232448, "shared memory");
};

// first weight row (N index) of half h of the B tile
template <int BN, int EPI>
__device__ __forceinline__ int b_half_base(const GemmArgs& a, int n_tile, int h) {
  if (EPI == EPI_SITU) return (h == 0 ? 0 : a.up_offset) + n_tile * (BN / 2);
  return n_tile * BN + h * (BN / 2);
}


template <int BN, int STAGES, int BF, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, BF, EPI>::kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = GemmCfg<BN, STAGES, BF, EPI>;
  constexpr bool kMx = is_expand(BF);  // B expanded by the dequant warps
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* stages = smem;
  uint8_t* dstages = smem + STAGES * C::kStageBytes;  // expanded B ring (MXFP4)
  int32_t* row_off = reinterpret_cast<int32_t*>(dstages + C::kDStages * C::kBBytes);
  int32_t* tile_start = row_off + (kMaxGroups + 1);
  int32_t* scan_rows = tile_start + (kMaxGroups + 1);
  int32_t* scan_tiles = scan_rows + C::kThreads;
  uint64_t* bars = reinterpret_cast<uint64_t*>(scan_tiles + C::kThreads);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* bready = bars + 2 * STAGES;       // expanded B tile ready (dequant -> MMA)
  uint64_t* bempty = bready + C::kDAlloc;     // expanded B tile consumed (MMA -> dequant)
  uint64_t* tfull = bempty + C::kDAlloc;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = args.G;

  if (threadIdx.x == 0) *abort_flag = 0;
  const int total = build_schedule<kBM>(args, row_off, tile_start, scan_rows, scan_tiles);
  if (total < 0) return;  // uniform across the CTA; nothing allocated yet

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int s = 0; s < C::kDAlloc; ++s) {
      mbar_init(smem_u32(bready + s), 8);  // one arrival per dequant warp
      mbar_init(smem_u32(bempty + s), 1);  // UMMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(tfull + b), 1);
      mbar_init(smem_u32(tempty + b), 128);
    }
    mbar_init(smem_u32(drain), 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (args.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Direct A: lane 0 issues one 128-row box per stage.  Gathered A: every
    // lane issues one tile::gather4 of 4 rows (lane i: tile rows 4i..4i+3),
    // the row indices read once per tile.
    const bool gather = args.a_rows != nullptr;
    if (gather || lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile<kBM>(tile_start, row_off, G, args.n_tiles, t);
        int32_t src[4] = {0, 0, 0, 0};
        if (gather) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int row = tc.row0 + 4 * lane + j;
            const int s = row < args.M ? __ldg(args.a_rows + row) : -1;
            src[j] = (s < 0 || s >= args.a_src_rows) ? args.a_src_rows : s;  // past the end: zeros
          }
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          bool w = true;
          if (lane == 0) w = mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.status);
          if (gather) w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
          if (!w) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          if (lane == 0) mbar_arrive_expect_tx(fb, C::kABytes + (kMx ? C::kPackedBytes : C::kBBytes));
          const uint32_t a_dst = smem_u32(stages + stage * C::kStageBytes);
          const uint32_t b_dst = a_dst + C::kABytes;  // bf16 B, or the packed codes (MXFP4)
          const uint32_t p_dst = b_dst;
          if (gather) {
            __syncwarp();  // the expected byte count is registered before any copy lands
            tma_gather4_2d(a_dst + lane * 4 * 128, &tmA, fb, kb * kBK, src[0], src[1], src[2],
                           src[3]);
          } else {
            tma_load_2d(a_dst, &tmA, fb, kb * kBK, tc.row0);
          }
          if (lane == 0)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int nbase = b_half_base<BN, EPI>(args, tc.n_tile, h);
            if (BF == B_NMAJOR) {
#pragma unroll
              for (int c = 0; c < BN / 128; ++c)
                tma_load_3d(b_dst + (h * (BN / 128) + c) * (kBK * 128), &tmB, fb, nbase + c * 64,
                            kb * kBK, tc.g);
            } else if (BF == B_KMAJOR) {
              tma_load_3d(b_dst + h * (BN / 2) * 128, &tmB, fb, kb * kBK, nbase, tc.g);
            } else if (BF == B_FP8) {
              // one box: BN columns (bytes) x 64 K rows of the (G, K, N) e4m3 weight
              if (h == 0) tma_load_3d(p_dst, &tmB, fb, tc.n_tile * BN, kb * kBK, tc.g);
            } else {
              tma_load_3d(p_dst + h * (BN / 2) * (kBK / 2), &tmB, fb, kb * (kBK / 2), nbase, tc.g);
            }
          }
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && lane == 0) {
        // abort: let every copy already issued land before the CTA retires
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(full + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = (BF == B_MXFP4F16)
                                     ? idesc_f16_f32(kBM, BN, false)
                                     : idesc_bf16_f32(kBM, BN, BF == B_NMAJOR || BF == B_FP8);
      uint32_t stage = 0, phase = 0, dstage = 0, dphase = 0;
      uint32_t acc = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        if (!mbar_wait(smem_u32(tempty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status) ||
              (kMx && !mbar_wait(smem_u32(bready + dstage), dphase, abort_flag, args.status))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * C::kStageBytes);
          const uint32_t b_addr = kMx ? smem_u32(dstages + dstage * C::kBBytes) : a_addr + C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = (BF == B_NMAJOR || BF == B_FP8)
                                       ? smem_desc_sw128(b_addr + k * 2048, kBK * 128, 1024)
                                       : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(empty + stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (kMx) {
            umma_commit(smem_u32(bempty + dstage));
            if (++dstage == C::kDAlloc) {
              dstage = 0;
              dphase ^= 1u;
            }
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(tfull + acc));
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
    uint32_t acc = 0, acc_phase = 0;
    // f16 range guard: the largest magnitude this thread stored as an f16
    // operand, and the smallest nonzero peak of its 32-value runs
    float f16_peak = 0.f, f16_low = FLT_MAX;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileCoord tc = decode_tile<kBM>(tile_start, row_off, G, args.n_tiles, t);
      if (!mbar_wait(smem_u32(tfull + acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const int r = tc.row0 + q * 32 + lane;
      const bool valid = r < tc.row_end;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (EPI == EPI_SITU) {
#pragma unroll 1
        for (int c = 0; c < (BN / 2) / 32; ++c) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tbase + c * 32, gv);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c * 32, uv);
          tmem_ld_wait();
          const int col0 = tc.n_tile * (BN / 2) + c * 32;
          if (valid && col0 < args.N) {
            float run_peak = 0.f;  // this run of 32 activations (f16 range guard)
            __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(args.out) + r * args.ldo + col0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (col0 + j * 8 < args.N) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float o[2];
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    float g = __uint_as_float(gv[j * 8 + e * 2 + h]);
                    float u = __uint_as_float(uv[j * 8 + e * 2 + h]);
                    if (args.round_gate_up) {
                      g = bf16_round_f(g);
                      u = bf16_round_f(u);
                    }
                    o[h] = situ_fast(g, u, args.beta, args.inv_beta, args.linear_beta, args.inv_linear_beta);
                  }
                  if (args.out_f16) run_peak = fmaxf(run_peak, fmaxf(fabsf(o[0]), fabsf(o[1])));
                  pk[e] = args.out_f16 ? pack_f16x2_of_bf16(o[0], o[1]) : pack_bf16x2(o[0], o[1]);
                }
                *reinterpret_cast<uint4*>(orow + j * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            }
            if (run_peak > 0.f) f16_low = fminf(f16_low, bf16_round_f(run_peak));
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col0 = tc.n_tile * BN + c * 32;
          // the residual's 32 columns are fetched before the accumulator is
          // read, so the global load overlaps the TMEM load
          uint4 addv[4];
          if (EPI == EPI_BF16_ADD) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              addv[j] = (valid && col0 + j * 8 < args.N)
                            ? *reinterpret_cast<const uint4*>(args.addend + r * args.ld_add + col0 + j * 8)
                            : make_uint4(0, 0, 0, 0);
          }
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + c * 32, v);
          tmem_ld_wait();
          if (valid && col0 < args.N) {
            if (EPI == EPI_F32) {
              float* orow = reinterpret_cast<float*>(args.out) + r * args.ldo + col0;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (col0 + j * 4 < args.N)
                  *reinterpret_cast<uint4*>(orow + j * 4) =
                      make_uint4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
            } else {
              __nv_bfloat16* orow =
                  reinterpret_cast<__nv_bfloat16*>(args.out) + r * args.ldo + col0;
              const float peak0 = f16_peak;
              if (EPI == EPI_BF16 && args.out_f16) f16_peak = 0.f;  // this run's peak
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (col0 + j * 8 < args.N) {
                  uint32_t pk[4];
                  if (EPI == EPI_BF16_ADD) {
                    const uint4 av = addv[j];
                    const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const __nv_bfloat162 ab = *reinterpret_cast<const __nv_bfloat162*>(&aw[e]);
                      const float x0 = bf16_round_f(__uint_as_float(v[j * 8 + e * 2]));
                      const float x1 = bf16_round_f(__uint_as_float(v[j * 8 + e * 2 + 1]));
                      pk[e] = pack_bf16x2(x0 + __low2float(ab), x1 + __high2float(ab));
                    }
                  } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const float x0 = __uint_as_float(v[j * 8 + e * 2]);
                      const float x1 = __uint_as_float(v[j * 8 + e * 2 + 1]);
                      if (args.out_f16) {
                        f16_peak = fmaxf(f16_peak, fmaxf(fabsf(x0), fabsf(x1)));
                        pk[e] = pack_f16x2_of_bf16(x0, x1);
                      } else {
                        pk[e] = pack_bf16x2(x0, x1);
                      }
                    }
                  }
                  *reinterpret_cast<uint4*>(orow + j * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
              }
              if (EPI == EPI_BF16 && args.out_f16) {
                if (f16_peak > 0.f) f16_low = fminf(f16_low, f16_peak);
                f16_peak = fmaxf(f16_peak, peak0);
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(tempty + acc));
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    // f16 range guard: a bf16 result above 65504 became inf in its f16 slot,
    // or a whole run of results was too small for f16 to carry accurately
    if ((EPI == EPI_BF16 || EPI == EPI_SITU) &&
        __any_sync(0xffffffffu, bf16_round_f(f16_peak) > kF16Max || f16_low < kF16RunMin) &&
        lane == 0)
      record_status(args.status, kF16Range);
    // rows at or past sum(group_sizes) are zero (ragged_dot semantics)
    if (args.zero_tail) {
      const int esize = (EPI == EPI_F32) ? 4 : 2;
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
  } else if (BF == B_FP8) {
    // ------------------------------------------------------------ fp8 expansion
    // The TMA stage holds the (64 K x BN) e4m3 tile, row k = BN bytes.  Thread d
    // expands columns n = 8 (d % 32) .. +7 of rows k = d / 32 + 8 i (i < 8):
    // bf16(f32(q) * scale[block(k)][n]) -- the reference's dequantised weight
    // -- written into the MN-major 128B-swizzled operand: 64-column chunks of
    // 64 rows x 128 B, the 16-byte group j of row k at slot j ^ (k & 7).
    const int d = threadIdx.x - 192;
    const int nc = d & 31;
    const int k0 = d >> 5;
    const int chunk = nc >> 3, sub = nc & 7;
    const float* scales = reinterpret_cast<const float*>(args.scales);
    uint32_t stage = 0, phase = 0, dstage = 0, dphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const TileCoord tc = decode_tile<kBM>(tile_start, row_off, G, args.n_tiles, t);
      const int n0 = tc.n_tile * BN + nc * 8;
      const bool col_in = n0 < args.N;
      const float* sg = scales + static_cast<int64_t>(tc.g) * args.n_blocks * args.N + n0;
      for (int kb = 0; kb < num_kb && ok; ++kb) {
        // scales of the (at most two) K blocks this step's rows fall in
        const int b_lo = (kb * kBK) / args.block_size;
        const int b_hi = (kb * kBK + kBK - 1) / args.block_size;
        float4 s_lo[2], s_hi[2];
        if (col_in) {
          s_lo[0] = __ldg(reinterpret_cast<const float4*>(sg + static_cast<int64_t>(b_lo) * args.N));
          s_lo[1] = __ldg(reinterpret_cast<const float4*>(sg + static_cast<int64_t>(b_lo) * args.N) + 1);
          s_hi[0] = __ldg(reinterpret_cast<const float4*>(sg + static_cast<int64_t>(b_hi) * args.N));
          s_hi[1] = __ldg(reinterpret_cast<const float4*>(sg + static_cast<int64_t>(b_hi) * args.N) + 1);
        } else {
          s_lo[0] = s_lo[1] = s_hi[0] = s_hi[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status) ||
            !mbar_wait(smem_u32(bempty + dstage), dphase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        const uint32_t src = smem_u32(stages + stage * C::kStageBytes + C::kABytes + nc * 8);
        const uint32_t dst = smem_u32(dstages + dstage * C::kBBytes + chunk * (kBK * 128));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = k0 + 8 * i;
          const bool hi = (kb * kBK + k) / args.block_size != b_lo;
          const float sc[8] = {hi ? s_hi[0].x : s_lo[0].x, hi ? s_hi[0].y : s_lo[0].y,
                               hi ? s_hi[0].z : s_lo[0].z, hi ? s_hi[0].w : s_lo[0].w,
                               hi ? s_hi[1].x : s_lo[1].x, hi ? s_hi[1].y : s_lo[1].y,
                               hi ? s_hi[1].z : s_lo[1].z, hi ? s_hi[1].w : s_lo[1].w};
          const uint2 q = lds_v2(src + k * BN);
          uint32_t h2[4];
          asm("{\n\t.reg .b16 l0, h0, l1, h1;\n\t"
              "mov.b32 {l0, h0}, %4;\n\t"
              "mov.b32 {l1, h1}, %5;\n\t"
              "cvt.rn.f16x2.e4m3x2 %0, l0;\n\t"
              "cvt.rn.f16x2.e4m3x2 %1, h0;\n\t"
              "cvt.rn.f16x2.e4m3x2 %2, l1;\n\t"
              "cvt.rn.f16x2.e4m3x2 %3, h1;\n\t}"
              : "=r"(h2[0]), "=r"(h2[1]), "=r"(h2[2]), "=r"(h2[3])
              : "r"(q.x), "r"(q.y));
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2[e]));
            o[e] = pack_bf16x2(f.x * sc[2 * e], f.y * sc[2 * e + 1]);
          }
          sts_v4(dst + k * 128 + ((sub ^ (k & 7)) << 4), make_uint4(o[0], o[1], o[2], o[3]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(bready + dstage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        if (++dstage == C::kDAlloc) {
          dstage = 0;
          dphase ^= 1u;
        }
      }
    }
  } else if (kMx) {
    // ------------------------------------------------------------ MXFP4 dequant
    // thread i of the 256 dequant threads expands row i of the B tile: 64 K
    // elements = 8 chunks of 8 bf16, written at the 128B-swizzled position
    // (chunk c of row r lands in 16-byte slot c ^ (r & 7)).
    const int r = threadIdx.x - 192;
    const int h = r / (BN / 2);
    const int kgroups = args.K / 32;
    uint32_t stage = 0, phase = 0, dstage = 0, dphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const TileCoord tc = decode_tile<kBM>(tile_start, row_off, G, args.n_tiles, t);
      const int n_row = b_half_base<BN, EPI>(args, tc.n_tile, h) + (r % (BN / 2));
      const bool row_in = n_row < args.n_weight;
      const uint16_t* srow = reinterpret_cast<const uint16_t*>(
          args.scales + (static_cast<int64_t>(tc.g) * args.n_weight + n_row) * kgroups);
      // scale bytes of this row's two 32-element blocks, fetched kPrefetch k steps
      // ahead (a global load outlives several 512-cycle MMA steps)
      constexpr int kPrefetch = 4;
      uint32_t sq[kPrefetch];
#pragma unroll
      for (int j = 0; j < kPrefetch; ++j) sq[j] = (row_in && j < num_kb) ? __ldg(srow + j) : 0x7F7Fu;
      for (int kb0 = 0; kb0 < num_kb && ok; kb0 += kPrefetch)
#pragma unroll
      for (int j = 0; j < kPrefetch; ++j) {
        const int kb = kb0 + j;
        if (kb >= num_kb) break;
        const uint32_t s01 = sq[j];
        if (kb + kPrefetch < num_kb) sq[j] = row_in ? __ldg(srow + kb + kPrefetch) : 0x7F7Fu;
        if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status) ||
            !mbar_wait(smem_u32(bempty + dstage), dphase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        const uint32_t prow = smem_u32(stages + stage * C::kStageBytes + C::kABytes + r * (kBK / 2));
        const uint4 p0 = lds_v4(prow), p1 = lds_v4(prow + 16);
        const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const uint32_t brow = smem_u32(dstages + dstage * C::kBBytes + r * 128);
        if (BF == B_MXFP4F16) {
          const uint32_t b0 = e8m0_to_f16_bits(s01 & 0xFFu), b1 = e8m0_to_f16_bits(s01 >> 8);
          const uint32_t sc0 = b0 | (b0 << 16), sc1 = b1 | (b1 << 16);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = dequant_e2m1x8_f16(words[c], c < 4 ? sc0 : sc1);
            sts_v4(brow + ((c ^ (r & 7)) << 4), v);
          }
        } else {
          const uint32_t b0 = e8m0_to_bf16_bits(s01 & 0xFFu), b1 = e8m0_to_bf16_bits(s01 >> 8);
          const uint32_t sc0 = b0 | (b0 << 16), sc1 = b1 | (b1 << 16);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t sc = c < 4 ? sc0 : sc1;
            const uint4 v = dequant_e2m1x8(words[c], *reinterpret_cast<const __nv_bfloat162*>(&sc));
            sts_v4(brow + ((c ^ (r & 7)) << 4), v);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(bready + dstage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        if (++dstage == C::kDAlloc) {
          dstage = 0;
          dphase ^= 1u;
        }
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

// --------------------------------------------------------------------------- host side

namespace {

template <int BN, int STAGES, int BF, int EPI>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int max_tiles,
                cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES, BF, EPI>;
  auto kern = grouped_gemm_kernel<BN, STAGES, BF, EPI>;
  int dev = 0;
  cudaGetDevice(&dev);
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
  const int sms = num_sms(dev);
  const int grid = max(1, min(sms, max_tiles));
  kern<<<grid, C::kThreads, C::kSmem, stream>>>(ta, tb, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

constexpr int kStagesBf16 = 4;
constexpr int kStagesMx = 5;
constexpr int kStagesFp8 = 4;
// Narrow tiles for dense GEMMs too small to fill the GPU (a few token blocks):
// 128-wide weight tiles give twice the CTAs, and their 32 KB stages fit a
// ring six deep in the same shared memory.  With few CTAs each one streams its
// weights from HBM and the ring's depth sets the rate (a ring microbenchmark:
// the round trip of a TMA copy from HBM is ~2700 clk, so four 512-clk stages
// leave the tensor pipe waiting).  Every output element sums its K products in
// the same order as with 256-wide tiles, so the results are the same bits.
constexpr int kNarrowBN = 128;
constexpr int kStagesNarrow = 6;

int launch_epi_narrow(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                      int max_tiles, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_gemm<kNarrowBN, kStagesNarrow, B_KMAJOR, EPI_BF16>(ta, tb, a, max_tiles, s);
    case EPI_F32: return launch_gemm<kNarrowBN, kStagesNarrow, B_KMAJOR, EPI_F32>(ta, tb, a, max_tiles, s);
    case EPI_BF16_ADD:
      return launch_gemm<kNarrowBN, kStagesNarrow, B_KMAJOR, EPI_BF16_ADD>(ta, tb, a, max_tiles, s);
    case EPI_SITU: return launch_gemm<kNarrowBN, kStagesNarrow, B_KMAJOR, EPI_SITU>(ta, tb, a, max_tiles, s);
    default: return kBadShape;
  }
}

template <int EPI>
int dispatch_format(int bf, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                    int max_tiles, cudaStream_t s) {
  switch (bf) {
    case B_NMAJOR: return launch_gemm<256, kStagesBf16, B_NMAJOR, EPI>(ta, tb, a, max_tiles, s);
    case B_KMAJOR: return launch_gemm<256, kStagesBf16, B_KMAJOR, EPI>(ta, tb, a, max_tiles, s);
    case B_MXFP4F16: return launch_gemm<256, kStagesMx, B_MXFP4F16, EPI>(ta, tb, a, max_tiles, s);
    case B_FP8:
      if constexpr (EPI == EPI_BF16 || EPI == EPI_F32)
        return launch_gemm<256, kStagesFp8, B_FP8, EPI>(ta, tb, a, max_tiles, s);
      else
        return kUnsupported;
    default: return launch_gemm<256, kStagesMx, B_MXFP4, EPI>(ta, tb, a, max_tiles, s);
  }
}

int launch_epi(int epi, int bf, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
               int max_tiles, cudaStream_t stream) {
  switch (epi) {
    case EPI_BF16: return dispatch_format<EPI_BF16>(bf, ta, tb, a, max_tiles, stream);
    case EPI_F32: return dispatch_format<EPI_F32>(bf, ta, tb, a, max_tiles, stream);
    case EPI_BF16_ADD: return dispatch_format<EPI_BF16_ADD>(bf, ta, tb, a, max_tiles, stream);
    case EPI_SITU: return dispatch_format<EPI_SITU>(bf, ta, tb, a, max_tiles, stream);
    default: return kBadShape;
  }
}

int common_checks(const void* lhs, const void* out, int64_t M, int64_t K, int64_t N_out, int64_t G,
                  int epi, const void* addend, int64_t ld_add, int64_t up_offset) {
  if (M < 0 || K <= 0 || N_out <= 0 || G <= 0 || G > kMaxGroups) return kBadShape;
  if (M >= (1ll << 31) || K >= (1ll << 31) || N_out >= (1ll << 31)) return kBadShape;
  if (K % 8 != 0 || N_out % 8 != 0) return kUnsupported;  // 16-byte TMA strides / vector stores
  if ((reinterpret_cast<uintptr_t>(lhs) | reinterpret_cast<uintptr_t>(out)) & 15) return kUnsupported;
  if (epi == EPI_BF16_ADD && (addend == nullptr || (reinterpret_cast<uintptr_t>(addend) & 15) ||
                              ld_add % 8 != 0))
    return kUnsupported;
  if (epi == EPI_SITU && up_offset != N_out) return kBadShape;
  return kOk;
}

GemmArgs make_args(const int32_t* group_sizes, void* out, const void* addend, int64_t ld_add,
                   int64_t M, int64_t K, int64_t N_out, int64_t G, int epi, int64_t up_offset,
                   int64_t n_weight, float beta, float linear_beta, int round_gate_up,
                   int zero_tail, int32_t* status) {
  GemmArgs a{};
  a.group_sizes = group_sizes;
  a.status = status;
  a.out = out;
  a.addend = static_cast<const __nv_bfloat16*>(addend);
  a.ldo = N_out;
  a.ld_add = ld_add;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N_out);
  a.K = static_cast<int>(K);
  a.G = group_sizes == nullptr ? 1 : static_cast<int>(G);
  const int out_tile = (epi == EPI_SITU) ? 128 : 256;
  a.n_tiles = static_cast<int>((N_out + out_tile - 1) / out_tile);
  a.up_offset = static_cast<int>(up_offset);
  a.n_weight = static_cast<int>(n_weight);
  a.beta = beta;
  a.linear_beta = linear_beta;
  a.inv_beta = beta != 0.f ? 1.0f / beta : 0.f;
  a.inv_linear_beta = linear_beta != 0.f ? 1.0f / linear_beta : 0.f;
  a.round_gate_up = round_gate_up;
  a.zero_tail = zero_tail;
  return a;
}

int max_tiles_of(const GemmArgs& a) {
  const int64_t t = ((static_cast<int64_t>(a.M) + kBM - 1) / kBM + a.G) * a.n_tiles;
  return static_cast<int>(std::min<int64_t>(t, 1 << 30));
}

// A operand map: a 128-row box over lhs (M, K), or, for a row gather, a
// one-row box over the source rows (the tile::gather4 form).
bool encode_a(CUtensorMap* ta, const void* lhs, int64_t M, int64_t K, const int32_t* a_rows,
              int64_t a_src_rows) {
  if (a_rows != nullptr)
    return encode_tmap_bf16_2d(ta, lhs, static_cast<uint64_t>(K),
                               static_cast<uint64_t>(a_src_rows), static_cast<uint64_t>(K) * 2,
                               kBK, 1);
  return encode_tmap_bf16_2d(ta, lhs, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                             static_cast<uint64_t>(K) * 2, kBK, kBM);
}

}  // namespace

// rhs_layout: 0 = (G, K, N) ("gkn", N contiguous, the reference's layout);
//             1 = (G, N, K) ("gnk", K contiguous, torch nn.Linear layout)
// a_rows (optional, device): logical lhs row r = source row a_rows[r] of lhs,
// which then has a_src_rows rows (-1 = zeros).
int grouped_gemm_bf16(const void* lhs, const void* rhs, const int32_t* group_sizes, void* out,
                      int64_t M, int64_t K, int64_t N_out, int64_t G, int rhs_layout, int epi,
                      const void* addend, int64_t ld_add, int64_t up_offset, float beta,
                      float linear_beta, int round_gate_up, int zero_tail, int32_t* status,
                      cudaStream_t stream, const int32_t* a_rows, int64_t a_src_rows,
                      int out_f16) {
  if (rhs_layout != 0 && rhs_layout != 1) return kBadShape;
  int rc = common_checks(lhs, out, M, K, N_out, G, epi, addend, ld_add, up_offset);
  if (rc != kOk) return rc;
  if (reinterpret_cast<uintptr_t>(rhs) & 15) return kUnsupported;
  if (a_rows != nullptr && (a_src_rows <= 0 || a_src_rows >= (1ll << 31))) return kBadShape;
  if (M == 0) return kOk;
  const bool b_mn = rhs_layout == 0;
  // width of the weight's N axis (the fused [gate|up] weight is 2I wide)
  const int64_t n_weight = (epi == EPI_SITU) ? 2 * up_offset : N_out;
  CUtensorMap ta, tb;
  if (!encode_a(&ta, lhs, M, K, a_rows, a_src_rows)) return kLaunchFailed;
  if (b_mn) {
    // dims {N, K, G}, box {64, 64, 1}
    if (!encode_tmap_bf16_3d(&tb, rhs, n_weight, K, G, n_weight * 2, n_weight * K * 2, 64, kBK))
      return kLaunchFailed;
  } else {
    // dims {K, N, G}, box {64, 128, 1}
    if (!encode_tmap_bf16_3d(&tb, rhs, K, n_weight, G, K * 2, n_weight * K * 2, kBK, 128))
      return kLaunchFailed;
  }
  GemmArgs a = make_args(group_sizes, out, addend, ld_add, M, K, N_out, G, epi, up_offset,
                         n_weight, beta, linear_beta, round_gate_up, zero_tail, status);
  a.a_rows = a_rows;
  a.a_src_rows = static_cast<int>(a_src_rows);
  a.out_f16 = (epi == EPI_BF16 || epi == EPI_SITU) ? out_f16 : 0;
  // a dense K-major GEMM whose 256-wide tiles would leave SMs idle takes the
  // narrow tiles (one group, no row gather: the tile count is exact)
  const int64_t m_blocks = (M + kBM - 1) / kBM;
  if (!b_mn && group_sizes == nullptr && a_rows == nullptr &&
      m_blocks * a.n_tiles < num_sms(current_device())) {
    // dims {K, N, G}, box {64, 64, 1}: each half of a 128-wide tile
    if (!encode_tmap_bf16_3d(&tb, rhs, K, n_weight, G, K * 2, n_weight * K * 2, kBK, kNarrowBN / 2))
      return kLaunchFailed;
    const int out_tile = (epi == EPI_SITU) ? kNarrowBN / 2 : kNarrowBN;
    a.n_tiles = static_cast<int>((N_out + out_tile - 1) / out_tile);
    return launch_epi_narrow(epi, ta, tb, a, static_cast<int>(m_blocks * a.n_tiles), stream);
  }
  return launch_epi(epi, b_mn ? B_NMAJOR : B_KMAJOR, ta, tb, a, max_tiles_of(a), stream);
}

// MXFP4 weights: packed (G, n_weight, K/2) u8, scales (G, n_weight, K/32) u8.
// lhs_f16: lhs holds f16 (bf16 values carried as f16) and the f16 operand path
// runs (scale bytes must lie in [104, 140]); out_f16: bf16-rounded results are
// stored as f16 (EPI_BF16 / EPI_SITU).
int grouped_gemm_mxfp4(const void* lhs, const void* packed, const void* scales,
                       const int32_t* group_sizes, void* out, int64_t M, int64_t K, int64_t N_out,
                       int64_t G, int epi, int64_t up_offset, float beta, float linear_beta,
                       int round_gate_up, int zero_tail, int lhs_f16, int out_f16,
                       int32_t* status, cudaStream_t stream, const int32_t* a_rows,
                       int64_t a_src_rows) {
  int rc = common_checks(lhs, out, M, K, N_out, G, epi, nullptr, 0, up_offset);
  if (rc != kOk) return rc;
  if (epi == EPI_BF16_ADD || (out_f16 && epi == EPI_F32)) return kUnsupported;
  if (K % 64 != 0) return kUnsupported;  // whole 32-element scale blocks per 64-wide K step
  if (reinterpret_cast<uintptr_t>(packed) & 15 || scales == nullptr ||
      (reinterpret_cast<uintptr_t>(scales) & 1))
    return kUnsupported;
  if (a_rows != nullptr && (a_src_rows <= 0 || a_src_rows >= (1ll << 31))) return kBadShape;
  if (M == 0) return kOk;
  const int64_t n_weight = (epi == EPI_SITU) ? 2 * up_offset : N_out;
  if (a_rows == nullptr && (group_sizes == nullptr || G <= kSwapMaxGroups)) {
    // direct operand: the weights-major kernel (expands each weight tile once
    // per 256 tokens instead of per 128)
    GemmArgs a = make_args(group_sizes, out, nullptr, 0, M, K, N_out, G, epi, up_offset, n_weight,
                           beta, linear_beta, round_gate_up, zero_tail, status);
    a.scales = static_cast<const uint8_t*>(scales);
    a.out_f16 = out_f16;
    return mxfp4_swap_gemm(lhs, packed, a, epi, lhs_f16, stream);
  }
  CUtensorMap ta, tb;
  if (!encode_a(&ta, lhs, M, K, a_rows, a_src_rows)) return kLaunchFailed;
  // dims {K/2 bytes, N, G}, box {32 bytes = 64 codes, 128 rows, 1}
  if (!encode_tmap_u8_3d(&tb, packed, K / 2, n_weight, G, K / 2, n_weight * (K / 2), kBK / 2, 128))
    return kLaunchFailed;
  GemmArgs a = make_args(group_sizes, out, nullptr, 0, M, K, N_out, G, epi, up_offset, n_weight,
                         beta, linear_beta, round_gate_up, zero_tail, status);
  a.scales = static_cast<const uint8_t*>(scales);
  a.out_f16 = out_f16;
  a.a_rows = a_rows;
  a.a_src_rows = static_cast<int>(a_src_rows);
  return launch_epi(epi, lhs_f16 ? B_MXFP4F16 : B_MXFP4, ta, tb, a, max_tiles_of(a), stream);
}


// e4m3 weights (G, K, N) -- the reference's layout -- with f32 scales
// (G, K / block_size, N): out = lhs @ bf16(f32(q) * scale) per group.
int grouped_gemm_fp8(const void* lhs, const void* rhs_q, const float* rhs_scale,
                     const int32_t* group_sizes, void* out, int64_t M, int64_t K, int64_t N,
                     int64_t G, int64_t block_size, int out_f32, int zero_tail, int32_t* status,
                     cudaStream_t stream) {
  const int epi = out_f32 ? EPI_F32 : EPI_BF16;
  int rc = common_checks(lhs, out, M, K, N, G, epi, nullptr, 0, 0);
  if (rc != kOk) return rc;
  if (group_sizes == nullptr || rhs_q == nullptr || rhs_scale == nullptr) return kBadShape;
  if (K % kBK != 0 || block_size <= 0 || block_size % 32 != 0 || K % block_size != 0)
    return kUnsupported;
  if ((reinterpret_cast<uintptr_t>(rhs_q) | reinterpret_cast<uintptr_t>(rhs_scale)) & 15)
    return kUnsupported;
  if (N % 16 != 0) return kUnsupported;  // 16-byte TMA rows of the (K, N) e4m3 weight
  if (M == 0) return kOk;
  CUtensorMap ta, tb;
  if (!encode_a(&ta, lhs, M, K, nullptr, 0)) return kLaunchFailed;
  // dims {N bytes, K, G}, box {256 columns, 64 K rows}
  if (!encode_tmap_u8_3d(&tb, rhs_q, N, K, G, N, N * K, 256, kBK)) return kLaunchFailed;
  GemmArgs a = make_args(group_sizes, out, nullptr, 0, M, K, N, G, epi, 0, N, 0.f, 0.f, 0,
                         zero_tail, status);
  a.scales = reinterpret_cast<const uint8_t*>(rhs_scale);
  a.block_size = static_cast<int>(block_size);
  a.n_blocks = static_cast<int>(K / block_size);
  return launch_epi(epi, B_FP8, ta, tb, a, max_tiles_of(a), stream);
}


// MXFP4 grouped matmul whose output row r goes to the byte address
// row_dest[r] (16-byte aligned; any GPU-writable address, a peer GPU's buffer
// included) -- the down projection writing straight into the exchange buffers
// of the ranks the rows came from.  bf16 out, rows past sum(group_sizes) are
// not written.
int grouped_gemm_mxfp4_scatter(const void* lhs, const void* packed, const void* scales,
                               const int32_t* group_sizes, const uint64_t* row_dest, int64_t M,
                               int64_t K, int64_t N, int64_t G, int lhs_f16, int32_t* status,
                               cudaStream_t stream) {
  if (group_sizes == nullptr || row_dest == nullptr || scales == nullptr) return kBadShape;
  if (M < 0 || K <= 0 || N <= 0 || G <= 0 || G > kSwapMaxGroups) return kBadShape;
  if (M >= (1ll << 31) || K >= (1ll << 31) || N >= (1ll << 31)) return kBadShape;
  if (K % 64 != 0 || N % 8 != 0) return kUnsupported;
  if ((reinterpret_cast<uintptr_t>(lhs) | reinterpret_cast<uintptr_t>(packed)) & 15 ||
      (reinterpret_cast<uintptr_t>(scales) & 1))
    return kUnsupported;
  if (M == 0) return kOk;
  GemmArgs a = make_args(group_sizes, nullptr, nullptr, 0, M, K, N, G, EPI_BF16, 0, N, 0.f, 0.f, 0,
                         0, status);
  a.scales = static_cast<const uint8_t*>(scales);
  a.row_dest = row_dest;
  return mxfp4_swap_gemm(lhs, packed, a, EPI_BF16, lhs_f16, stream);
}

}  // namespace lmoe
