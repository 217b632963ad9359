// MXFP4 grouped GEMM, weights-major, on CTA pairs (cluster of 2, one MMA over
// both SMs: `tcgen05.mma.cta_group::2`, M = 256 weight rows x N = 256 tokens).
//
//   out[r, :] = lhs[r, :] @ dequant(w[g(r)])^T     r in group g's row range
//
// Same contract and epilogues as the single-CTA weights-major kernel
// (mxfp4_swap.cu; reference: 05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67 and
// the fused SiTU-GLU of kimi_k3_latent_moe_ragged_dot.py:610-723).  A pair
// tile is 256 weight rows x 256 token rows.  Each CTA of the pair
//   - expands its own 128 weight rows (UMMA A rows 128*rank ...),
//   - loads its own 128 of the tile's 256 token rows (UMMA B columns),
//   - holds its 128 accumulator rows x 256 tokens in its own TMEM and runs the
//     epilogue for them.
// So per SM the token bytes per MMA FLOP halve: the token ring holds 8 K steps
// in the shared memory that held 4, and the L2 -> SM token traffic halves.
//
// Rings (identical offsets in both CTAs; the leader's tensor core reads the
// peer's A and B tiles at the leader's descriptor addresses):
//   token ring   (8 x 16 KB)  128 token rows x 64 K, 128B swizzle  -> B half
//   packed ring  (4 x 4 KB)   e2m1 codes of the CTA's 128 weight rows (local)
//   A ring       (4 x 16 KB)  expanded weights, K-major 128B swizzle -> A half
// Barriers the leader's MMA issuer waits on live in the leader: tok_full
// (both CTAs' token copies count their bytes on it), a_ready (4 dequant warps
// of each CTA), acc_empty (4 epilogue warps of each CTA).  Barriers each CTA's
// own roles wait on live in that CTA and the leader's MMA commits to both:
// tok_empty, a_empty, acc_full.  The packed ring is local to each CTA.
//
// Roles per CTA (480 threads): warp 0 token producer, warp 1 TMEM allocation
// (both CTAs, cta_group::2) and, in the leader, the MMA issuer; warps 2-5
// epilogue; warps 6-13 dequant (two groups of 4 on alternate K steps); warp 14
// packed-code producer.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

namespace {

constexpr int kPairTok = 256;   // tokens per pair tile (UMMA N)
constexpr int kHalfTok = 128;   // tokens per CTA
constexpr int kWRows = 128;     // weight rows per CTA (UMMA M = 256 over the pair)
constexpr int kTStages = 8;     // token ring
constexpr int kPStages = 4;     // packed-code ring
constexpr int kDStages = 4;     // expanded-weight (A) ring
constexpr int kDeqWarps = 8;
constexpr int kPkWarp = 6 + kDeqWarps;
constexpr int kThreads = 32 * (kPkWarp + 1);
constexpr int kMaxG = kSwapMaxGroups;
static_assert(kPStages % 2 == 0 && kDStages % 2 == 0, "each ring slot belongs to one dequant group");

struct PairCfg {
  static constexpr int kTokBytes = kHalfTok * kBK * 2;     // 16 KB
  static constexpr int kPackedBytes = kWRows * (kBK / 2);  // 4 KB
  static constexpr int kABytes = kWRows * kBK * 2;         // 16 KB
  static constexpr int kWarpStage = 1024;
  static constexpr int kOutStageBytes = 4 * kWarpStage;
  static constexpr int kTmemCols = 2 * kPairTok;
  static constexpr int kSchedBytes = 2 * (kMaxG + 1) * 4;
  static constexpr int kNumBars = 2 * kTStages + 2 * kPStages + 2 * kDStages + 5;
  static constexpr size_t kSmem = 1024 + size_t(kTStages) * kTokBytes +
                                  size_t(kPStages) * kPackedBytes + size_t(kDStages) * kABytes +
                                  kOutStageBytes + kSchedBytes + 8 * kNumBars + 16;
  static_assert(kTokBytes % 1024 == 0 && kABytes % 1024 == 0 && kPackedBytes % 1024 == 0,
                "1024-byte aligned stages");
  static_assert(kOutStageBytes >= 2 * kThreads * 4, "scan scratch");
  static_assert(kSmem <= 232448, "shared memory");
};

// weight row (N index of the checkpoint layout) behind row r of this CTA's A half
template <int EPI>
__device__ __forceinline__ int pair_weight_row(const GemmArgs& a, int n_tile, int rank, int r) {
  if (EPI == EPI_SITU)
    return ((r & 1) ? a.up_offset : 0) + n_tile * kWRows + rank * (kWRows / 2) + (r >> 1);
  return n_tile * 2 * kWRows + rank * kWRows + r;
}

template <int EPI>
__device__ __forceinline__ int pair_packed_row(int r) {
  return EPI == EPI_SITU ? (r & 1) * 64 + (r >> 1) : r;
}

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
__global__ void __launch_bounds__(kThreads, 1)
    mxfp4_pair_kernel(const __grid_constant__ CUtensorMap tmTok,
                      const __grid_constant__ CUtensorMap tmW, const GemmArgs args) {
  using C = PairCfg;
  constexpr bool kF16 = BF == B_MXFP4F16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* tstages = smem;
  uint8_t* pstages = tstages + kTStages * C::kTokBytes;
  uint8_t* astages = pstages + kPStages * C::kPackedBytes;
  uint8_t* ostage = astages + kDStages * C::kABytes;
  int32_t* row_off = reinterpret_cast<int32_t*>(ostage + C::kOutStageBytes);
  int32_t* tile_start = row_off + (kMaxG + 1);
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_start + (kMaxG + 1));
  uint64_t* tok_full = bars;                   // leader: both halves' bytes
  uint64_t* tok_empty = tok_full + kTStages;   // each CTA: leader's UMMA commit
  uint64_t* pk_full = tok_empty + kTStages;
  uint64_t* pk_empty = pk_full + kPStages;
  uint64_t* a_ready = pk_empty + kPStages;     // leader: 4 dequant warps of each CTA
  uint64_t* a_empty = a_ready + kDStages;      // each CTA: leader's UMMA commit
  uint64_t* acc_full = a_empty + kDStages;     // each CTA: leader's UMMA commit
  uint64_t* acc_empty = acc_full + 2;          // leader: 4 epilogue warps of each CTA
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = args.G;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) *abort_flag = 0;
  int32_t* scan = reinterpret_cast<int32_t*>(ostage);
  // both CTAs build the same schedule, so both return here or neither does
  const int total = build_schedule<kPairTok>(args, row_off, tile_start, scan, scan + kThreads);
  if (total < 0) return;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(smem_u32(tok_full + s), 1);
      mbar_init(smem_u32(tok_empty + s), 1);
    }
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(smem_u32(pk_full + s), 1);
      mbar_init(smem_u32(pk_empty + s), kDeqWarps / 2);
    }
    for (int s = 0; s < kDStages; ++s) {
      mbar_init(smem_u32(a_ready + s), kDeqWarps);  // 4 warps x 2 CTAs
      mbar_init(smem_u32(a_empty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(acc_full + b), 1);
      mbar_init(smem_u32(acc_empty + b), 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(smem_u32(drain), 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmTok);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // the peer's barriers exist and both TMEM allocations are done before any
  // remote arrive, remote copy completion or pair MMA
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = args.K / kBK;

  if (warp == 0 || warp == kPkWarp) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      const bool tok = warp == 0;
      uint64_t* fullb = tok ? tok_full : pk_full;
      uint64_t* emptyb = tok ? tok_empty : pk_empty;
      const uint32_t nst = tok ? kTStages : kPStages;
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        const TileCoord tc = decode_tile<kPairTok>(tile_start, row_off, G, args.n_tiles, t);
        const int wb0 = pair_weight_row<EPI>(args, tc.n_tile, rank, 0);
        const int wb1 = EPI == EPI_SITU ? pair_weight_row<EPI>(args, tc.n_tile, rank, 1) : wb0 + 64;
        const int tok_row = tc.row0 + static_cast<int>(rank) * kHalfTok;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(emptyb + stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          if (tok) {
            // both halves count on the leader's barrier; the leader registers
            // the bytes of both
            const uint32_t fb_local = smem_u32(fullb + stage);
            if (rank == 0) mbar_arrive_expect_tx(fb_local, 2 * C::kTokBytes);
            tma_load_2d_pair(smem_u32(tstages + stage * C::kTokBytes), &tmTok,
                             mapa_shared(fb_local, 0), kb * kBK, tok_row);
          } else {
            const uint32_t fb = smem_u32(fullb + stage);
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
      // abort: let every copy already issued land before the CTA retires (the
      // peer's token copies count on the leader's barrier: the leader waits)
      if (!ok && (!tok || rank == 0)) {
        for (uint32_t s = 0; s < nst; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(fullb + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = kF16 ? idesc_f16_f32(2 * kWRows, kPairTok, false)
                                      : idesc_bf16_f32(2 * kWRows, kPairTok, false);
      RingPos ts, ds;
      uint32_t acc = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        if (!mbar_wait(smem_u32(acc_empty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairTok;
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
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          const uint32_t te = smem_u32(tok_empty + ts.stage), ae = smem_u32(a_empty + ds.stage);
          umma_commit_pair(te);
          umma_commit_pair(mapa_shared(te, 1));
          umma_commit_pair(ae);
          umma_commit_pair(mapa_shared(ae, 1));
          ts.next<kTStages>();
          ds.next<kDStages>();
        }
        if (!ok) break;
        const uint32_t af = smem_u32(acc_full + acc);
        umma_commit_pair(af);
        umma_commit_pair(mapa_shared(af, 1));
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        // abort: wait for every UMMA already issued before TMEM is released
        umma_commit_pair(smem_u32(drain));
        mbar_drain(smem_u32(drain), 0);
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    uint8_t* stg = ostage + q * C::kWarpStage;
    constexpr int esize = (EPI == EPI_F32) ? 4 : 2;
    uint32_t acc = 0, acc_phase = 0;
    for (int t = pair; t < total; t += npairs) {
      const TileCoord tc = decode_tile<kPairTok>(tile_start, row_off, G, args.n_tiles, t);
      if (!mbar_wait(smem_u32(acc_full + acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kPairTok;
#pragma unroll 1
      for (int c = 0; c < kPairTok / 32; ++c) {
        const int tok0 = tc.row0 + c * 32;
        if (tok0 >= tc.row_end) break;  // warp-uniform
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        if (EPI == EPI_SITU) {
          // lanes 2i / 2i+1 hold gate / up of feature i
          static_assert(C::kWarpStage >= 1024, "SiTU staging");
          const int odd = lane & 1;
          uint16_t* s16 = reinterpret_cast<uint16_t*>(stg);
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
            s16[(odd * 16 + j) * 16 + (lane >> 1)] = out16(o, args.out_f16);
          }
          __syncwarp();
          const int tok = tok0 + lane;
          const int f0 = tc.n_tile * kWRows + static_cast<int>(rank) * (kWRows / 2) + q * 16;
          if (tok < tc.row_end) {
            const uint4* src = reinterpret_cast<const uint4*>(stg + lane * 32);
            uint16_t* orow =
                reinterpret_cast<uint16_t*>(args.out) + static_cast<int64_t>(tok) * args.ldo + f0;
            if (f0 + 8 <= args.N) *reinterpret_cast<uint4*>(orow) = src[0];
            if (f0 + 16 <= args.N) *reinterpret_cast<uint4*>(orow + 8) = src[1];
          }
          __syncwarp();
        } else {
          constexpr int kRowBytes = 32 * esize;
          constexpr int kChunks = kRowBytes / 16;
          constexpr int kRows = C::kWarpStage / kRowBytes;
          static_assert(kRows >= 8 && 32 % kRows == 0, "staging rows");
          const int byte = lane * esize;
          const int f0 = tc.n_tile * 2 * kWRows + static_cast<int>(rank) * kWRows + q * 32;
#pragma unroll
          for (int p0 = 0; p0 < 32; p0 += kRows) {
            uint8_t* dst0 = stg + (byte & 15);
            if (EPI == EPI_F32) {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj)
                *reinterpret_cast<uint32_t*>(dst0 + jj * kRowBytes +
                                             (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4)) = v[p0 + jj];
            } else if (args.out_f16) {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj)
                *reinterpret_cast<uint16_t*>(dst0 + jj * kRowBytes +
                                             (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4)) =
                    out16(__uint_as_float(v[p0 + jj]), 1);
            } else {
#pragma unroll
              for (int jj = 0; jj < kRows; ++jj)
                *reinterpret_cast<uint16_t*>(dst0 + jj * kRowBytes +
                                             (((byte >> 4) ^ swz_key<kChunks>(jj)) << 4)) =
                    out16(__uint_as_float(v[p0 + jj]), 0);
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
                  *reinterpret_cast<uint4*>(orow + cc * 16) = *reinterpret_cast<const uint4*>(
                      stg + lane * kRowBytes + ((cc ^ swz_key<kChunks>(lane)) * 16));
              }
            }
            __syncwarp();
          }
        }
      }
      // the accumulator is read: one arrival per warp on the leader's barrier
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t ae = smem_u32(acc_empty + acc);
        if (rank == 0) mbar_arrive(ae); else mbar_arrive_cluster(mapa_shared(ae, 0));
      }
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (args.row_dest != nullptr) __threadfence_system();
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
    // Same scheme as the single-CTA kernel: two groups of 4 warps on
    // alternate K steps, thread i expands row i of this CTA's A half, slot
    // ownership per group; the codes are expanded into registers and
    // fenced before their packed slot is released (TMA refills it), and the
    // expanded row is fenced for the async proxy before the leader's a_ready
    // counts it (the leader's tensor core reads this CTA's tile).
    const int grp = (warp - 6) / 4;
    const int r = ((warp - 6) % 4) * 32 + lane;
    const int kgroups = args.K / 32;
    const int my_tiles = pair < total ? (total - pair + npairs - 1) / npairs : 0;
    const int n_steps = my_tiles * num_kb;
    int cached_tile = -1;
    const uint16_t* srow = nullptr;
    auto load_scale = [&](int st) -> uint32_t {
      const int ti = st / num_kb;
      if (ti != cached_tile) {
        cached_tile = ti;
        const TileCoord tc =
            decode_tile<kPairTok>(tile_start, row_off, G, args.n_tiles, pair + ti * npairs);
        const int w_row = pair_weight_row<EPI>(args, tc.n_tile, rank, r);
        const bool row_in =
            EPI == EPI_SITU
                ? (tc.n_tile * kWRows + static_cast<int>(rank) * (kWRows / 2) + (r >> 1)) < args.up_offset
                : w_row < args.n_weight;
        srow = row_in ? reinterpret_cast<const uint16_t*>(
                            args.scales +
                            (static_cast<int64_t>(tc.g) * args.n_weight + w_row) * kgroups)
                      : nullptr;
      }
      return srow != nullptr ? __ldg(srow + (st - ti * num_kb)) : 0x7F7Fu;
    };
    auto expand = [&](int st, uint32_t sc) -> bool {
      const uint32_t pslot = st % kPStages, pph = (st / kPStages) & 1;
      if (!mbar_wait(smem_u32(pk_full + pslot), pph, abort_flag, args.status)) return false;
      const uint4* src = reinterpret_cast<const uint4*>(pstages + pslot * C::kPackedBytes +
                                                        pair_packed_row<EPI>(r) * (kBK / 2));
      const uint4 p0 = src[0], p1 = src[1];
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
      uint8_t* arow = astages + aslot * C::kABytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = dq[c];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const uint32_t ar = smem_u32(a_ready + aslot);
        if (rank == 0) mbar_arrive(ar); else mbar_arrive_cluster(mapa_shared(ar, 0));
      }
      return true;
    };
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
  // neither CTA retires (or frees TMEM) while the other may still touch its
  // shared memory or signal its barriers
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

template <int BF, int EPI>
int launch_pair(const CUtensorMap& tok, const CUtensorMap& w, const GemmArgs& a, int max_tiles,
                cudaStream_t stream) {
  auto kern = mxfp4_pair_kernel<BF, EPI>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static uint64_t configured = 0;
  static int max_pairs[64] = {0};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(configured & (1ull << dev))) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(PairCfg::kSmem)) != cudaSuccess)
        return kLaunchFailed;
      // how many CTA pairs can be resident at once with this shared memory
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * (num_sms(dev) / 2));
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = PairCfg::kSmem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &q) != cudaSuccess || clusters < 1)
        return kLaunchFailed;
      max_pairs[dev & 63] = clusters;
      configured |= 1ull << dev;
    }
  }
  const int pairs = max(1, min(max_pairs[dev & 63], max_tiles));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = PairCfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tok, w, a) != cudaSuccess) return kLaunchFailed;
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

template <int BF>
int launch_pair_epi(int epi, const CUtensorMap& tok, const CUtensorMap& w, const GemmArgs& a,
                    int max_tiles, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_pair<BF, EPI_BF16>(tok, w, a, max_tiles, s);
    case EPI_F32: return launch_pair<BF, EPI_F32>(tok, w, a, max_tiles, s);
    case EPI_SITU: return launch_pair<BF, EPI_SITU>(tok, w, a, max_tiles, s);
    default: return kUnsupported;
  }
}

}  // namespace

// Weights-major MXFP4 grouped GEMM on CTA pairs.  Same arguments as
// mxfp4_swap_gemm; its n_tiles is set here (a pair tile covers 256 weight rows).
int mxfp4_pair_gemm(const void* lhs, const void* packed, GemmArgs a, int epi, int lhs_f16,
                    cudaStream_t stream) {
  CUtensorMap tok, w;
  // tokens: dims {K, M}, box {64, 128} (one CTA's half of a pair tile), 128B swizzle
  if (!encode_tmap_bf16_2d(&tok, lhs, static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.M),
                           static_cast<uint64_t>(a.K) * 2, kBK, kHalfTok))
    return kLaunchFailed;
  const int64_t kh = a.K / 2;
  if (!encode_tmap_u8_3d(&w, packed, kh, a.n_weight, a.G, kh, static_cast<int64_t>(a.n_weight) * kh,
                         kBK / 2, 64))
    return kLaunchFailed;
  const int feat = epi == EPI_SITU ? kWRows : 2 * kWRows;  // output features per pair tile
  a.n_tiles = (a.N + feat - 1) / feat;
  const int64_t t = ((static_cast<int64_t>(a.M) + kPairTok - 1) / kPairTok + a.G) * a.n_tiles;
  const int max_tiles = static_cast<int>(t < (1 << 30) ? t : (1 << 30));
  return lhs_f16 ? launch_pair_epi<B_MXFP4F16>(epi, tok, w, a, max_tiles, stream)
                 : launch_pair_epi<B_MXFP4>(epi, tok, w, a, max_tiles, stream);
}

}  // namespace lmoe
