// Fused router gate: the logits GEMM h @ W_router^T on tcgen05 tensor cores
// with sigmoid, bias and a per-chunk top-k in its epilogue, then a per-token
// merge.  The f32 logits never reach global memory.
//
// Semantics: exactly router_topk (routing.cu, activation 0) applied to the f32
// logits of the dense GEMM, i.e. the gate of
// 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-356 -- score =
// sigmoid(logit), key = score + bias (selection only), top-k by key with
// ties to the lower expert id, weight = the selected scores, renormalised by
// (sum + 1e-20) in selection order when k > 1, times the routed scaling
// factor.
//
// Layout.  The experts are split into n_chunks = ceil(E / 256) column chunks
// of W = ceil(E / n_chunks) rounded up to 16 (896 experts: 4 chunks of 224).
// A tile is 128 tokens x one chunk; the chunks of a token block have
// consecutive tile ids, so the CTAs working on them read the same hidden
// rows from L2 at about the same time.
//   warp 0     TMA producer: hidden rows (128 x 64 bf16) and the chunk's
//              router rows (W x 64 bf16), 128B-swizzled, one stage per 64-wide
//              K step
//   warp 1     TMEM owner and MMA issuer: kind::f16, M = 128, N = W, f32
//              accumulators in two buffers (columns 0 and 256) so the
//              selection of one tile overlaps the MMAs of the next
//   warps 2-5  selection: thread = token row.  The chunk's logits come out
//              of tensor memory 32 columns at a time; the thread keeps the
//              chunk's best LIST (key, expert, score) entries in registers,
//              sorted in the selection order, and writes them to the
//              candidate buffer (T, n_chunks, LIST).  A first pass over
//              the chunk computes every score and key (the scores replace
//              the logits in tensor memory) and a lower bound tau of the
//              LIST-th largest key; a second pass inserts only the columns
//              whose key reaches tau (the insertion is the costly part; the
//              32 tokens of a warp have independent lists, so inserting
//              column by column would run the insertion for almost every
//              column)
// The merge kernel then runs the selection over each token's n_chunks x LIST
// candidates (one warp per token).  A chunk's top LIST >= k holds every
// expert of that chunk that is in the token's overall top-k, so the merge
// sees all winners and picks them in the same order as router_topk.
#include <cuda.h>

#include <cfloat>
#include <climits>
#include <mutex>

#include "gemm_common.cuh"
#include "lmoe_internal.h"
#include "ptx.cuh"
#include "router_select.cuh"

namespace lmoe {

namespace {

constexpr int kRtBM = 128;           // tokens per tile (TMEM lanes)
constexpr int kRtStages = 4;
constexpr int kRtThreads = 192;      // producer, issuer, 4 selection warps
constexpr int kRtMaxW = 256;         // widest chunk (one MMA N)
constexpr int kRtMaxE = 1024;
constexpr int kRtMaxK = 16;
constexpr int kRtAccStride = 256;    // TMEM columns per accumulator buffer
constexpr int kRtTmemCols = 512;
constexpr int kRtABytes = kRtBM * kBK * 2;                     // 16 KB
constexpr int kRtStageBytes = kRtABytes + kRtMaxW * kBK * 2;   // 48 KB
constexpr int kRtParkBytes = 128 * 32 * 4;                     // 32 scores per selection thread
constexpr size_t kRtSmem =
    1024 + size_t(kRtStages) * kRtStageBytes + kRtMaxE * 4 + kRtParkBytes + 256;
static_assert(kRtStageBytes % 1024 == 0, "stages stay 1024-byte aligned for SW128");
static_assert(kRtSmem <= 232448, "shared memory");

struct RtArgs {
  const float* bias;  // (E,) or nullptr
  int32_t* status;
  uint4* cand;        // (T, n_chunks, LIST) entries (key bits, expert, score bits, 0)
  uint32_t idesc;
  int T, E, K, W, n_chunks, total;
};

template <int LIST>
__global__ void __launch_bounds__(kRtThreads, 1)
    router_select_kernel(const __grid_constant__ CUtensorMap tmH,
                         const __grid_constant__ CUtensorMap tmR, const RtArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* stages = smem;
  float* bias_s = reinterpret_cast<float*>(stages + kRtStages * kRtStageBytes);
  float* park = bias_s + kRtMaxE;  // [128 selection threads][32 scores]
  uint64_t* bars = reinterpret_cast<uint64_t*>(park + kRtParkBytes / 4);
  uint64_t* full = bars;
  uint64_t* empty = full + kRtStages;
  uint64_t* tfull = empty + kRtStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < args.E; i += blockDim.x)
    bias_s[i] = args.bias != nullptr ? args.bias[i] : 0.f;
  if (threadIdx.x == 0) *abort_flag = 0;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(tfull + b), 1);
      mbar_init(smem_u32(tempty + b), 128);
    }
    mbar_init(smem_u32(drain), 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmH);
    tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kRtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (args.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t tx = kRtABytes + static_cast<uint32_t>(args.W) * kBK * 2;
      uint32_t stage = 0, phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.total && ok; t += gridDim.x) {
        const int mb = t / args.n_chunks;
        const int chunk = t - mb * args.n_chunks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(full + stage);
          const uint32_t dst = smem_u32(stages + stage * kRtStageBytes);
          mbar_arrive_expect_tx(fb, tx);
          tma_load_2d(dst, &tmH, fb, kb * kBK, mb * kRtBM);
          tma_load_2d(dst + kRtABytes, &tmR, fb, kb * kBK, chunk * args.W);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kRtStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // abort: let every copy already issued land before the CTA retires
        for (int s = 0; s < kRtStages; ++s)
          if (issued & (1u << s)) mbar_drain(smem_u32(full + s), (last_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.total && ok; t += gridDim.x) {
        if (!mbar_wait(smem_u32(tempty + acc), acc_phase ^ 1u, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kRtAccStride;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * kRtStageBytes);
          const uint32_t b_addr = a_addr + kRtABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32, 16, 1024),
                     smem_desc_sw128(b_addr + k * 32, 16, 1024), args.idesc,
                     (kb | k) != 0 ? 1u : 0u);
          umma_commit(smem_u32(empty + stage));
          if (++stage == kRtStages) {
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
        // abort: wait for every MMA already issued before TMEM is released
        umma_commit(smem_u32(drain));
        mbar_drain(smem_u32(drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ selection
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t acc = 0, acc_phase = 0;
    for (int t = blockIdx.x; t < args.total; t += gridDim.x) {
      const int mb = t / args.n_chunks;
      const int chunk = t - mb * args.n_chunks;
      if (!mbar_wait(smem_u32(tfull + acc), acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const int r = mb * kRtBM + q * 32 + lane;
      const int e0 = chunk * args.W;
      const int width = min(args.W, args.E - e0);  // experts in this chunk
      // the list starts with -inf keys: every finite key beats them (a -inf
      // or NaN key never enters, as in router_topk, which never selects one)
      float kv[LIST], ks[LIST];
      int ke[LIST];
#pragma unroll
      for (int j = 0; j < LIST; ++j) {
        kv[j] = -INFINITY;
        ke[j] = INT_MAX;
        ks[j] = 0.f;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kRtAccStride;
      const uint32_t bias_a = smem_u32(bias_s);
      // Pass A: scores and keys of every column.  The scores go back into
      // tensor memory over the logits; per group of columns (column mod LIST)
      // the two largest keys are kept.  The LIST-th largest of those 2 x LIST
      // keys is a lower bound tau of the token's LIST-th largest key in the
      // chunk (they are keys of 2 x LIST distinct experts), and usually close
      // to it: pass B only has to insert columns whose key reaches tau.
      float m1[LIST], m2[LIST];
#pragma unroll
      for (int g = 0; g < LIST; ++g) m1[g] = m2[g] = -INFINITY;
#pragma unroll 1
      for (int c = 0; c * 32 < width; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = c * 32 + j;
          const float sc = router_sigmoid(__uint_as_float(v[j]));
          float key = sc + lds_f32(bias_a + 4u * static_cast<uint32_t>(min(e0 + col, args.E - 1)));
          key = (col < width && key == key) ? key : -INFINITY;  // NaN keys never enter
          const int g = j % LIST;
          m2[g] = fmaxf(m2[g], fminf(m1[g], key));
          m1[g] = fmaxf(m1[g], key);
          v[j] = __float_as_uint(sc);
        }
        tmem_st_32x32b_x32(tbase + c * 32, v);
      }
      tmem_st_wait();
      sort_desc<LIST>(m1);
      sort_desc<LIST>(m2);
      const float tau = lth_largest_of_two<LIST>(m1, m2);
      // Pass B: the columns whose key reaches tau and beats the list's last
      // entry are parked (their scores in this thread's shared-memory row,
      // 16-byte group g of the row in slot g ^ (lane & 7) so a warp's vector
      // stores spread over the banks) and inserted one by one, the next
      // one's loads issued before the current insertion.
      const uint32_t row = smem_u32(park + (q * 32 + lane) * 32);
      const int sw = lane & 7;
#pragma unroll 1
      for (int c = 0; c * 32 < width; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        // experts arrive in increasing id order: a new key must beat the
        // last entry strictly (on an equal key the lower id already held wins)
        const float last = kv[LIST - 1];
        uint32_t marked = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = c * 32 + j;
          const float key =
              __uint_as_float(v[j]) + lds_f32(bias_a + 4u * static_cast<uint32_t>(min(e0 + col, args.E - 1)));
          marked |= (col < width && key >= tau && key > last) ? (1u << j) : 0u;
        }
        if (__any_sync(0xffffffffu, marked != 0u)) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            sts_v4(row + ((g ^ sw) << 4), make_uint4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]));
        }
        int j = marked != 0u ? __ffs(marked) - 1 : 0;
        float s_next = 0.f, b_next = 0.f;
        if (marked != 0u) {
          s_next = lds_f32(row + ((((j >> 2) ^ sw) << 4) | ((j & 3) << 2)));
          b_next = lds_f32(bias_a + 4u * static_cast<uint32_t>(e0 + c * 32 + j));
        }
        while (marked != 0u) {
          const int e = e0 + c * 32 + j;
          const float s = s_next;
          const float key = s + b_next;
          marked &= marked - 1u;
          if (marked != 0u) {
            j = __ffs(marked) - 1;
            s_next = lds_f32(row + ((((j >> 2) ^ sw) << 4) | ((j & 3) << 2)));
            b_next = lds_f32(bias_a + 4u * static_cast<uint32_t>(e0 + c * 32 + j));
          }
          if (key > kv[LIST - 1]) sel_insert_ascending<LIST>(kv, ke, ks, key, e, s);
        }
      }
      // the accumulator is free for the next tile before the candidates go out
      tc_fence_before();
      mbar_arrive(smem_u32(tempty + acc));
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
      if (r < args.T) {
        uint4* dst = args.cand + (static_cast<int64_t>(r) * args.n_chunks + chunk) * LIST;
#pragma unroll
        for (int j = 0; j < LIST; ++j)
          dst[j] = make_uint4(__float_as_uint(kv[j]), static_cast<uint32_t>(ke[j]),
                              __float_as_uint(ks[j]), 0u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kRtTmemCols);
  }
}

// One warp per token: the selection of router_topk over the token's
// candidates (lane l holds candidates l and l + 32, best first), then the
// weights with the same arithmetic: the selected scores summed in selection
// order, w / (sum + 1e-20) when k > 1 and renormalize, times rsf.
__global__ void __launch_bounds__(256) router_merge_kernel(const uint4* __restrict__ cand, int T,
                                                           int n_cand, int k, int renormalize,
                                                           float rsf, int32_t* __restrict__ topk_idx,
                                                           float* __restrict__ topk_w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const uint4* c = cand + static_cast<int64_t>(warp) * n_cand;
  float v1 = -FLT_MAX, v2 = -FLT_MAX, s1 = 0.f, s2 = 0.f;
  int e1 = INT_MAX, e2 = INT_MAX;
  if (lane < n_cand) {
    const uint4 a = c[lane];
    v1 = __uint_as_float(a.x);
    e1 = static_cast<int>(a.y);
    s1 = __uint_as_float(a.z);
  }
  if (lane + 32 < n_cand) {
    const uint4 b = c[lane + 32];
    v2 = __uint_as_float(b.x);
    e2 = static_cast<int>(b.y);
    s2 = __uint_as_float(b.z);
    if (sel_before(v2, e2, v1, e1)) {
      const float tv = v1, ts = s1;
      const int te = e1;
      v1 = v2; e1 = e2; s1 = s2;
      v2 = tv; e2 = te; s2 = ts;
    }
  }
  float wsum = 0.f, my_w = 0.f;
  int my_idx = 0;
  for (int s = 0; s < k; ++s) {
    // warp argmax: the largest key (as an order-preserving unsigned), then
    // the lowest expert id holding it
    const uint32_t fb = __float_as_uint(v1);
    const uint32_t ku = fb ^ ((fb & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, ku);
    const int bi = static_cast<int>(
        __reduce_min_sync(0xffffffffu, ku == kmax ? static_cast<uint32_t>(e1) : 0xFFFFFFFFu));
    const bool won = ku == kmax && bi == e1;
    const int wl = __ffs(__ballot_sync(0xffffffffu, won)) - 1;
    const float bw = __shfl_sync(0xffffffffu, s1, wl);
    wsum += bw;
    if (lane == s) {
      my_w = bw;
      my_idx = bi;
    }
    if (won) {
      v1 = v2; e1 = e2; s1 = s2;
      v2 = -FLT_MAX; e2 = INT_MAX; s2 = 0.f;
    }
  }
  if (lane < k) {
    float w = my_w;
    if (k > 1 && renormalize) w = w / (wsum + 1e-20f);
    w = w * rsf;
    topk_idx[static_cast<int64_t>(warp) * k + lane] = my_idx;
    topk_w[static_cast<int64_t>(warp) * k + lane] = w;
  }
}

struct RtShape {
  int n_chunks, W, list;
};

RtShape rt_shape(int64_t E, int64_t k) {
  RtShape s;
  s.n_chunks = static_cast<int>((E + kRtMaxW - 1) / kRtMaxW);
  const int64_t w = (E + s.n_chunks - 1) / s.n_chunks;
  s.W = static_cast<int>((w + 15) / 16 * 16);
  s.list = k <= 8 ? 8 : 16;
  return s;
}

template <int LIST>
int launch_select(const CUtensorMap& tmH, const CUtensorMap& tmR, const RtArgs& a,
                  cudaStream_t stream) {
  auto kern = router_select_kernel<LIST>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static uint64_t configured = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!(configured & (1ull << dev))) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kRtSmem)) != cudaSuccess)
        return kLaunchFailed;
      configured |= 1ull << dev;
    }
  }
  const int grid = max(1, min(num_sms(dev), a.total));
  kern<<<grid, kRtThreads, kRtSmem, stream>>>(tmH, tmR, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace

size_t router_fused_workspace_size(int64_t T, int64_t E, int64_t k) {
  if (T <= 0 || E <= 0 || E > kRtMaxE || k <= 0 || k > kRtMaxK) return 0;
  const RtShape s = rt_shape(E, k);
  return static_cast<size_t>(T) * s.n_chunks * s.list * sizeof(uint4);
}

int router_fused_bf16(const void* hidden, const void* router_w, const float* bias, int64_t T,
                      int64_t K, int64_t E, int64_t k, int renormalize, float rsf,
                      int32_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                      int32_t* status, cudaStream_t stream) {
  if (T < 0 || K <= 0 || E <= 0 || E > kRtMaxE || k <= 0 || k > kRtMaxK || k > E)
    return kBadShape;
  if (T >= (1ll << 31) / 32 || K >= (1ll << 31)) return kBadShape;
  if (K % 8 != 0) return kUnsupported;  // 16-byte TMA row strides
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(router_w) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return kUnsupported;
  if (T == 0) return kOk;
  if (workspace == nullptr || workspace_bytes < router_fused_workspace_size(T, E, k))
    return kScratchTooSmall;
  const RtShape s = rt_shape(E, k);
  CUtensorMap tmH, tmR;
  if (!encode_tmap_bf16_2d(&tmH, hidden, static_cast<uint64_t>(K), static_cast<uint64_t>(T),
                           static_cast<uint64_t>(K) * 2, kBK, kRtBM) ||
      !encode_tmap_bf16_2d(&tmR, router_w, static_cast<uint64_t>(K), static_cast<uint64_t>(E),
                           static_cast<uint64_t>(K) * 2, kBK, static_cast<uint32_t>(s.W)))
    return kLaunchFailed;
  RtArgs a{};
  a.bias = bias;
  a.status = status;
  a.cand = static_cast<uint4*>(workspace);
  a.idesc = idesc_bf16_f32(kRtBM, static_cast<uint32_t>(s.W), false);
  a.T = static_cast<int>(T);
  a.E = static_cast<int>(E);
  a.K = static_cast<int>(K);
  a.W = s.W;
  a.n_chunks = s.n_chunks;
  a.total = static_cast<int>((T + kRtBM - 1) / kRtBM) * s.n_chunks;
  const int rc = s.list == 8 ? launch_select<8>(tmH, tmR, a, stream)
                             : launch_select<16>(tmH, tmR, a, stream);
  if (rc != kOk) return rc;
  const int threads = 256;
  const int blocks = static_cast<int>((T * 32 + threads - 1) / threads);
  router_merge_kernel<<<blocks, threads, 0, stream>>>(a.cand, a.T, s.n_chunks * s.list,
                                                      static_cast<int>(k), renormalize, rsf,
                                                      topk_idx, topk_w);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace lmoe
