// Per-phase dense projections of the LatentMoE layer as one persistent,
// split-K tcgen05 kernel per phase, for token counts too small to fill the
// GPU with output tiles.
//
//   input phase  (kimi_k3_latent_moe_reference.py:347-365, 428-433): the three
//                projections of the hidden states h (T, d) in one launch --
//                router logits h @ Wr^T (f32), latent x = bf16(h @ Wd^T), and
//                the shared expert's SiTU-GLU activation
//                bf16(situ(bf16(h @ Wg^T), bf16(h @ Wu^T)));
//   output phase (kimi_k3_latent_moe_reference.py:419-435): the layer output
//                bf16(normed @ Wup^T + shared_act @ Wsd^T) -- the
//                up-projection, the shared expert's down projection and the
//                output sum -- as one GEMM over two K segments.
//
// Why split-K: with a few hundred tokens or fewer, the output tiles of these
// projections number a few dozen (one 128-token block x d / 128 weight
// columns), so an ordinary persistent GEMM leaves most of the 148 SMs idle and
// each busy SM streams its weights through a long serial K loop.  Here a work
// unit is (K split s, 128-column tile n, 128-token block m): the K steps of a
// tile are dealt over S splits (S depends on the weights' shapes and the SM
// count only, never on T, so a token's result does not depend on how many
// tokens share the call), every SM streams a disjoint slice of the weights
// once, and the f32 partial sums go to an L2-resident workspace.  The CTA
// that completes a tile's last split (an arrival counter per tile) sums the S
// partials in split order -- a fixed order, so the result is deterministic --
// and applies the tile's epilogue.  Nothing waits on another CTA.
//
// Roles per CTA (192 threads): warp 0 TMA producer (A box 128 tokens x 64 K,
// B two boxes of 64 weight rows x 64 K, 128-byte swizzle, 6-stage ring),
// warp 1 TMEM owner and MMA issuer (kind::f16, M 128 tokens x N 128 columns,
// two accumulators), warps 2-5 epilogue (partials out of TMEM, then the
// reduction of finished tiles).  Every mbarrier wait is bounded.
//
// Column ranges of the input phase (each padded to whole tiles):
//   PH_F32   router logits, out (T, E) f32, weight rows j*128 .. +127
//   PH_BF16  latent rows,   out (T, L) bf16
//   PH_SITU  shared expert, out (T, Is) bf16: tile j loads gate rows
//            j*64 .. +63 and up rows Is + j*64 .. +63 of the fused [gate | up]
//            weight, so each (gate, up) pair meets in one tile
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "../../include/lmoe.h"
#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {
namespace {

constexpr int PH_F32 = 0, PH_BF16 = 1, PH_SITU = 2;
constexpr int kPhBM = 128;       // tokens per tile (UMMA M)
constexpr int kPhBN = 128;       // weight columns per tile (UMMA N)
constexpr int kPhStages = 6;
constexpr int kPhThreads = 192;
constexpr int kPhABytes = kPhBM * kBK * 2;  // 16 KB
constexpr int kPhBBytes = kPhBN * kBK * 2;  // 16 KB
constexpr int kPhStageBytes = kPhABytes + kPhBBytes;
constexpr int kPhMaxRanges = 3;
constexpr size_t kPhSmem = 1024 + size_t(kPhStages) * kPhStageBytes + 256;
static_assert(kPhSmem <= 232448, "shared memory");

struct PhaseRange {
  int tile_end;      // first n-tile past this range
  int mode;          // PH_F32 / PH_BF16 / PH_SITU
  int n_valid;       // output columns of this range
  int up_offset;     // PH_SITU: first up row of the fused weight
  int64_t ld;        // output row pitch, elements
  void* out;
};

struct PhaseArgs {
  int T, m_tiles, n_tiles;
  int n_ranges;
  PhaseRange r[kPhMaxRanges];
  int seg_kb[2];      // K steps of each segment (segment 1: 0 when absent)
  int seg_splits[2];  // splits of each segment
  int seg_kps[2];     // K steps per split
  int splits;         // seg_splits[0] + seg_splits[1]
  float* partial;     // (splits, m_tiles, n_tiles, 128 columns, 128 rows)
  int* counters;      // (m_tiles * n_tiles), zero at launch
  float beta, linear_beta, inv_beta, inv_linear_beta;
  int round_gate_up;
  int32_t* status;
};

struct PhaseUnit {
  int s, n, m, seg, kb0, kb1, range;
};

__device__ __forceinline__ PhaseUnit phase_unit(const PhaseArgs& a, int u) {
  PhaseUnit p;
  p.m = u % a.m_tiles;
  const int rest = u / a.m_tiles;
  p.n = rest % a.n_tiles;
  p.s = rest / a.n_tiles;
  p.seg = p.s < a.seg_splits[0] ? 0 : 1;
  const int ls = p.seg == 0 ? p.s : p.s - a.seg_splits[0];
  p.kb0 = ls * a.seg_kps[p.seg];
  p.kb1 = min(a.seg_kb[p.seg], p.kb0 + a.seg_kps[p.seg]);
  p.range = 0;
#pragma unroll
  for (int i = 0; i < kPhMaxRanges - 1; ++i)
    if (i < a.n_ranges - 1 && p.n >= a.r[p.range].tile_end) ++p.range;
  return p;
}

// first weight row of half h (64 rows) of n-tile n
__device__ __forceinline__ int phase_b_row(const PhaseArgs& a, const PhaseUnit& p, int h) {
  const int first = p.range == 0 ? 0 : a.r[p.range - 1].tile_end;
  const int j = p.n - first;
  if (a.r[p.range].mode == PH_SITU) return (h == 0 ? 0 : a.r[p.range].up_offset) + j * 64;
  return j * kPhBN + h * 64;
}

__device__ __forceinline__ const CUtensorMap* pick_b(const CUtensorMap* b0, const CUtensorMap* b1,
                                                     const CUtensorMap* b2, const CUtensorMap* b3,
                                                     const PhaseUnit& p) {
  if (p.seg == 1) return b3;
  return p.range == 0 ? b0 : (p.range == 1 ? b1 : b2);
}

// Partials are stored tile by tile, column-major inside a tile: split s,
// tile (m, n), column c, token row r at
//   ((s * m_tiles + m) * n_tiles + n) * 128 * 128 + c * 128 + r,
// so the 32 lanes of a warp (32 consecutive rows) store and load whole
// 128-byte lines.
constexpr int kPhTileFloats = kPhBN * kPhBM;

__device__ __forceinline__ int64_t partial_tile(const PhaseArgs& a, int s, int m, int n) {
  return ((static_cast<int64_t>(s) * a.m_tiles + m) * a.n_tiles + n) * kPhTileFloats;
}

__device__ __forceinline__ void ldcg_col32(const float* src, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __ldcg(src + j * kPhBM);
}

// Sum of the `splits` partials of 32 consecutive columns (from col) of token
// row r of tile (m, n), in split order.
__device__ __forceinline__ void sum_partials(const PhaseArgs& a, const PhaseUnit& u, int r,
                                             int col, float (&acc)[32]) {
  const int64_t stride = partial_tile(a, 1, 0, 0);  // one split
  const float* p = a.partial + partial_tile(a, 0, u.m, u.n) + static_cast<int64_t>(col) * kPhBM + r;
  ldcg_col32(p, acc);
  int s = 1;
  for (; s + 1 < a.splits; s += 2) {
    float v0[32], v1[32];
    ldcg_col32(p + s * stride, v0);
    ldcg_col32(p + (s + 1) * stride, v1);
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = (acc[i] + v0[i]) + v1[i];
  }
  if (s < a.splits) {
    float v0[32];
    ldcg_col32(p + s * stride, v0);
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] += v0[i];
  }
}

// The finished tile (m, n): every split's partial is in memory.  Thread r of
// the 128 epilogue threads reduces token row m*128 + r and applies the
// range's epilogue.
__device__ void finish_tile(const PhaseArgs& a, const PhaseUnit& p, int r) {
  const int64_t row = static_cast<int64_t>(p.m) * kPhBM + r;
  if (row >= a.T) return;
  const PhaseRange& rg = a.r[p.range];
  const int first = p.range == 0 ? 0 : a.r[p.range - 1].tile_end;
  const int j = p.n - first;
  if (rg.mode == PH_SITU) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      float g[32], u[32];
      sum_partials(a, p, r, c * 32, g);
      sum_partials(a, p, r, 64 + c * 32, u);
      const int o0 = j * 64 + c * 32;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(rg.out) + row * rg.ld;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (o0 + q * 8 >= rg.n_valid) break;
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float o[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float gv = g[q * 8 + e * 2 + h], uv = u[q * 8 + e * 2 + h];
            if (a.round_gate_up) {
              gv = bf16_round_f(gv);
              uv = bf16_round_f(uv);
            }
            o[h] = situ_fast(gv, uv, a.beta, a.inv_beta, a.linear_beta, a.inv_linear_beta);
          }
          pk[e] = pack_bf16x2(o[0], o[1]);
        }
        *reinterpret_cast<uint4*>(orow + o0 + q * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float v[32];
    const int o0 = j * kPhBN + c * 32;
    if (o0 >= rg.n_valid) break;
    sum_partials(a, p, r, c * 32, v);
    if (rg.mode == PH_F32) {
      float* orow = static_cast<float*>(rg.out) + row * rg.ld;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (o0 + q * 4 < rg.n_valid)
          *reinterpret_cast<float4*>(orow + o0 + q * 4) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(rg.out) + row * rg.ld;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (o0 + q * 8 < rg.n_valid)
          *reinterpret_cast<uint4*>(orow + o0 + q * 8) =
              make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                         pack_bf16x2(v[8 * q + 4], v[8 * q + 5]),
                         pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
    }
  }
}

// AND of v over the 128 epilogue threads (named barrier 1): every epilogue
// thread takes the same branch after a bounded wait, so none is left behind
// at a later named barrier.
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kPhThreads, 1)
    dense_phase_kernel(const __grid_constant__ CUtensorMap tmA0,
                       const __grid_constant__ CUtensorMap tmA1,
                       const __grid_constant__ CUtensorMap tmB0,
                       const __grid_constant__ CUtensorMap tmB1,
                       const __grid_constant__ CUtensorMap tmB2,
                       const __grid_constant__ CUtensorMap tmB3, const PhaseArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kPhStages * kPhStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = full + kPhStages;
  uint64_t* tfull = empty + kPhStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = args.splits * args.n_tiles * args.m_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kPhStages; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(tfull + b), 1);
      mbar_init(smem_u32(tempty + b), 128);
    }
    mbar_init(smem_u32(drain), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * kPhBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const PhaseUnit p = phase_unit(args, u);
        const CUtensorMap* ta = p.seg == 0 ? &tmA0 : &tmA1;
        const CUtensorMap* tb = pick_b(&tmB0, &tmB1, &tmB2, &tmB3, p);
        const int brow0 = phase_b_row(args, p, 0), brow1 = phase_b_row(args, p, 1);
        for (int kb = p.kb0; kb < p.kb1; ++kb) {
          if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          mbar_arrive_expect_tx(fb, kPhStageBytes);
          const uint32_t a_dst = smem_u32(stages + stage * kPhStageBytes);
          tma_load_2d(a_dst, ta, fb, kb * kBK, p.m * kPhBM);
          tma_load_2d(a_dst + kPhABytes, tb, fb, kb * kBK, brow0);
          tma_load_2d(a_dst + kPhABytes + 64 * 128, tb, fb, kb * kBK, brow1);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPhStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < kPhStages; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(full + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kPhBM, kPhBN, false);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const PhaseUnit p = phase_unit(args, u);
        if (!mbar_wait(smem_u32(tempty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPhBN;
        for (int kb = p.kb0; kb < p.kb1; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * kPhStageBytes);
          const uint32_t b_addr = a_addr + kPhABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 16, 1024),
                     smem_desc_sw128(b_addr + k * 32, 16, 1024), idesc,
                     (kb != p.kb0 || k != 0) ? 1u : 0u);
          umma_commit(smem_u32(empty + stage));
          if (++stage == kPhStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(tfull + acc));
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
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;  // token row within the tile
    const int et = threadIdx.x - 64;  // 0..127
    uint32_t acc = 0, acc_phase = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const PhaseUnit p = phase_unit(args, u);
      if (!epi_all(mbar_wait(smem_u32(tfull + acc), acc_phase, abort_flag, args.status))) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(p.m) * kPhBM + r;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kPhBN;
      float* ptile = args.partial + partial_tile(args, p.s, p.m, p.n) + r;
#pragma unroll 1
      for (int c = 0; c < kPhBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        if (row < args.T) {
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(ptile + (c * 32 + j) * kPhBM, __uint_as_float(v[j]));
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(tempty + acc));
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
      // publish this split's partial; the tile's last split reduces all of them
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) {
        const int tile = p.n * args.m_tiles + p.m;
        const int prev = atomicAdd(args.counters + tile, 1);
        const int last = prev == args.splits - 1;
        if (last) args.counters[tile] = 0;  // ready for the next launch
        *last_flag = last;
        __threadfence();
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last_flag) finish_tile(args, p, r);
      asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag is reused by the next unit
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kPhBN);
  }
}

struct PhasePlan {
  PhaseArgs a;
  size_t counter_bytes = 0, partial_bytes = 0;
  size_t bytes() const { return counter_bytes + partial_bytes; }
};

// Splits of each K segment: the count that minimises the busiest SM's K steps
// (units per SM x steps per split) plus a charge per split for storing and
// reducing its partials, measured on B200 at about six K steps' time per
// split (128 tokens, d 7168: 2 splits 34.5 us, 4 splits 38.5, 8 splits 44.6
// for the input phase).  Chosen for one token block, so it does not depend on
// T.
void choose_splits(PhaseArgs& a, int sms) {
  int best_cost = 1 << 30;
  for (int s0 = 1; s0 <= std::min(a.seg_kb[0], 32); ++s0) {
    int s1 = 0;
    if (a.seg_kb[1] > 0)
      s1 = std::max(1, std::min(a.seg_kb[1], (s0 * a.seg_kb[1] + a.seg_kb[0] / 2) / a.seg_kb[0]));
    const int kps0 = (a.seg_kb[0] + s0 - 1) / s0;
    const int kps1 = s1 > 0 ? (a.seg_kb[1] + s1 - 1) / s1 : 0;
    const int n0 = (a.seg_kb[0] + kps0 - 1) / kps0;
    const int n1 = s1 > 0 ? (a.seg_kb[1] + kps1 - 1) / kps1 : 0;
    const int units = (n0 + n1) * a.n_tiles;
    const int waves = (units + sms - 1) / sms;
    const int cost = waves * std::max(kps0, kps1) + 6 * (n0 + n1);
    if (cost < best_cost) {
      best_cost = cost;
      a.seg_splits[0] = n0;
      a.seg_splits[1] = n1;
      a.seg_kps[0] = kps0;
      a.seg_kps[1] = std::max(kps1, 1);
    }
  }
  a.splits = a.seg_splits[0] + a.seg_splits[1];
}

PhasePlan make_plan(int64_t T, int n_tiles, int64_t k0, int64_t k1) {
  PhasePlan p;
  PhaseArgs& a = p.a;
  a.T = static_cast<int>(T);
  a.m_tiles = static_cast<int>((T + kPhBM - 1) / kPhBM);
  a.n_tiles = n_tiles;
  a.seg_kb[0] = static_cast<int>(k0 / kBK);
  a.seg_kb[1] = static_cast<int>(k1 / kBK);
  choose_splits(a, num_sms(current_device()));
  p.counter_bytes = (static_cast<size_t>(a.m_tiles) * n_tiles * 4 + 255) / 256 * 256;
  p.partial_bytes = static_cast<size_t>(a.splits) * a.m_tiles * n_tiles * kPhBN * kPhBM * 4;
  return p;
}

int launch_phase(PhasePlan& p, const CUtensorMap* maps, void* workspace, size_t ws_bytes,
                 int32_t* status, cudaStream_t stream) {
  if (workspace == nullptr || ws_bytes < p.bytes() ||
      (reinterpret_cast<uintptr_t>(workspace) & 255))
    return kScratchTooSmall;
  PhaseArgs& a = p.a;
  a.counters = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.counter_bytes);
  a.status = status;
  static std::mutex mu;
  static unsigned long long configured = 0;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(configured & (1ull << dev))) {
      if (cudaFuncSetAttribute(dense_phase_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kPhSmem)) != cudaSuccess)
        return kLaunchFailed;
      configured |= 1ull << dev;
    }
  }
  // arrival counters start at zero in every launch (the last arrival of a
  // tile also resets its counter, but a launch that stopped early would not)
  if (cudaMemsetAsync(a.counters, 0, p.counter_bytes, stream) != cudaSuccess) return kLaunchFailed;
  const int total = a.splits * a.n_tiles * a.m_tiles;
  const int grid = std::max(1, std::min(num_sms(dev), total));
  dense_phase_kernel<<<grid, kPhThreads, kPhSmem, stream>>>(maps[0], maps[1], maps[2], maps[3],
                                                             maps[4], maps[5], a);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// A operand map: (T, K) bf16 rows, box 128 rows x 64 K (rows past T read zero)
bool map_a(CUtensorMap* m, const void* base, int64_t T, int64_t K) {
  return encode_tmap_bf16_2d(m, base, static_cast<uint64_t>(K), static_cast<uint64_t>(T),
                             static_cast<uint64_t>(K) * 2, kBK, kPhBM);
}

// B operand map: (rows, K) K-major bf16 weight, box 64 rows x 64 K
bool map_b(CUtensorMap* m, const void* base, int64_t rows, int64_t K) {
  return encode_tmap_bf16_2d(m, base, static_cast<uint64_t>(K), static_cast<uint64_t>(rows),
                             static_cast<uint64_t>(K) * 2, kBK, 64);
}

PhasePlan input_plan(int64_t t, int64_t d, int64_t e, int64_t latent, int64_t shared_i) {
  const int nt_r = static_cast<int>((e + kPhBN - 1) / kPhBN);
  const int nt_l = static_cast<int>((latent + kPhBN - 1) / kPhBN);
  const int nt_s = static_cast<int>((shared_i + 63) / 64);
  PhasePlan p = make_plan(t, nt_r + nt_l + nt_s, d, 0);
  PhaseArgs& a = p.a;
  a.n_ranges = 3;
  a.r[0] = {nt_r, PH_F32, static_cast<int>(e), 0, e, nullptr};
  a.r[1] = {nt_r + nt_l, PH_BF16, static_cast<int>(latent), 0, latent, nullptr};
  a.r[2] = {nt_r + nt_l + nt_s, PH_SITU, static_cast<int>(shared_i), static_cast<int>(shared_i),
            shared_i, nullptr};
  return p;
}

PhasePlan output_plan(int64_t t, int64_t latent, int64_t shared_i, int64_t d) {
  PhasePlan p = make_plan(t, static_cast<int>((d + kPhBN - 1) / kPhBN), latent, shared_i);
  p.a.n_ranges = 1;
  p.a.r[0] = {p.a.n_tiles, PH_BF16, static_cast<int>(d), 0, d, nullptr};
  return p;
}

bool input_shape_ok(int64_t t, int64_t d, int64_t e, int64_t latent, int64_t shared_i) {
  return t >= 0 && t < (1ll << 24) && d > 0 && e > 0 && latent > 0 && shared_i > 0 &&
         d % kBK == 0 && e % 4 == 0 && latent % 8 == 0 && shared_i % 8 == 0 && d < (1ll << 24) &&
         e < (1ll << 20) && latent < (1ll << 20) && shared_i < (1ll << 20);
}

bool output_shape_ok(int64_t t, int64_t latent, int64_t shared_i, int64_t d) {
  return t >= 0 && t < (1ll << 24) && d > 0 && latent > 0 && shared_i > 0 &&
         latent % kBK == 0 && shared_i % kBK == 0 && d % 8 == 0 && d < (1ll << 20) &&
         latent < (1ll << 20) && shared_i < (1ll << 20);
}

}  // namespace
}  // namespace lmoe

extern "C" {

size_t lmoe_dense_input_workspace_size(int64_t t, int64_t d, int64_t e, int64_t latent,
                                       int64_t shared_i) {
  if (!lmoe::input_shape_ok(t, d, e, latent, shared_i)) return 0;
  return lmoe::input_plan(t, d, e, latent, shared_i).bytes();
}

int lmoe_dense_input_phase(const void* hidden, const void* router_w, const void* down_w,
                           const void* shared_gu_w, float* logits, void* latent_out,
                           void* shared_act, int64_t t, int64_t d, int64_t e, int64_t latent,
                           int64_t shared_i, float beta, float linear_beta, int round_gate_up,
                           void* workspace, size_t workspace_bytes, int32_t* dev_status,
                           void* stream) {
  using namespace lmoe;
  if (!input_shape_ok(t, d, e, latent, shared_i)) return LMOE_UNSUPPORTED;
  const void* ptrs[7] = {hidden, router_w, down_w, shared_gu_w, logits, latent_out, shared_act};
  for (const void* p : ptrs)
    if (p == nullptr) return LMOE_BAD_SHAPE;
  for (const void* p : ptrs)
    if (!aligned16(p)) return LMOE_UNSUPPORTED;
  if (t == 0) return LMOE_OK;
  PhasePlan p = input_plan(t, d, e, latent, shared_i);
  p.a.r[0].out = logits;
  p.a.r[1].out = latent_out;
  p.a.r[2].out = shared_act;
  p.a.beta = beta;
  p.a.linear_beta = linear_beta;
  p.a.inv_beta = beta != 0.f ? 1.0f / beta : 0.f;
  p.a.inv_linear_beta = linear_beta != 0.f ? 1.0f / linear_beta : 0.f;
  p.a.round_gate_up = round_gate_up ? 1 : 0;
  CUtensorMap maps[6];
  if (!map_a(&maps[0], hidden, t, d) || !map_b(&maps[2], router_w, e, d) ||
      !map_b(&maps[3], down_w, latent, d) || !map_b(&maps[4], shared_gu_w, 2 * shared_i, d))
    return LMOE_LAUNCH_FAILED;
  maps[1] = maps[0];  // one K segment
  maps[5] = maps[2];
  return launch_phase(p, maps, workspace, workspace_bytes, dev_status,
                      static_cast<cudaStream_t>(stream));
}

size_t lmoe_dense_output_workspace_size(int64_t t, int64_t latent, int64_t shared_i, int64_t d) {
  if (!lmoe::output_shape_ok(t, latent, shared_i, d)) return 0;
  return lmoe::output_plan(t, latent, shared_i, d).bytes();
}

int lmoe_dense_output_phase(const void* normed, const void* up_w, const void* shared_act,
                            const void* shared_down_w, void* out, int64_t t, int64_t latent,
                            int64_t shared_i, int64_t d, void* workspace, size_t workspace_bytes,
                            int32_t* dev_status, void* stream) {
  using namespace lmoe;
  if (!output_shape_ok(t, latent, shared_i, d)) return LMOE_UNSUPPORTED;
  const void* ptrs[5] = {normed, up_w, shared_act, shared_down_w, out};
  for (const void* p : ptrs)
    if (p == nullptr) return LMOE_BAD_SHAPE;
  for (const void* p : ptrs)
    if (!aligned16(p)) return LMOE_UNSUPPORTED;
  if (t == 0) return LMOE_OK;
  PhasePlan p = output_plan(t, latent, shared_i, d);
  p.a.r[0].out = out;
  CUtensorMap maps[6];
  if (!map_a(&maps[0], normed, t, latent) || !map_a(&maps[1], shared_act, t, shared_i) ||
      !map_b(&maps[2], up_w, d, latent) || !map_b(&maps[5], shared_down_w, d, shared_i))
    return LMOE_LAUNCH_FAILED;
  maps[3] = maps[2];
  maps[4] = maps[2];
  return launch_phase(p, maps, workspace, workspace_bytes, dev_status,
                      static_cast<cudaStream_t>(stream));
}

}  // extern "C"
