// Router top-k, dispatch (stable counting sort + capacity padding + row
// gather), weighted combine + RMSNorm, scatter-add combine and the unfused
// SiTU-GLU activation.  All HBM-bound integer/byte work: warp-level
// primitives, 16-byte vector accesses, no tensor cores.
//
// Reference semantics (paths relative to the reference project):
//   router        05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-356
//   dispatch      kimi_k3_latent_moe_reference.py:370-378 (full) and
//                 kimi_k3_latent_moe_reference.py:754-877 (shard, capacity padded)
//   combine       kimi_k3_latent_moe_reference.py:413-416, 286-293 (RMSNorm)
//   scatter-add   kimi_k3_latent_moe_reference.py:1113-1141
//   SiTU-GLU      kimi_k3_latent_moe_reference.py:296-310
#include <cuda_bf16.h>

#include <cfloat>

#include "lmoe_internal.h"
#include "ptx.cuh"
#include "router_select.cuh"

namespace lmoe {

// =========================================================================== router
// One warp per token.  Lane l holds experts e = l + 32*j, j < PER.
// Selection = top-k of scores_for_choice (descending, ties -> lower expert id,
// the `jax.lax.top_k` rule); weights = un-biased scores of the winners,
// renormalised in slot order, times routed_scaling_factor.
// Three blocks per SM (24 warps): at configuration 5 the selection is latency
// bound, and the extra resident warps pay for the few spilled registers
// (137 -> 115 us for 16384 tokens x 896 experts; four blocks spill more and
// lose again).
template <int PER>
__global__ void __launch_bounds__(256, 3) router_topk_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int T, int E, int k,
    int activation, int renormalize, float rsf, int32_t* __restrict__ topk_idx,
    float* __restrict__ topk_w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + static_cast<int64_t>(warp) * E;
  // key[j] first holds the logit of expert lane + 32j, then its selection key
  float key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    key[j] = (e < E) ? row[e] : -FLT_MAX;
  }
  // softmax normaliser: the max, then the sum of exp(x - max) in lane order
  // and a butterfly; kept so that a winner's score is recomputed from its
  // logit with the same operations instead of holding every score
  float m = -FLT_MAX, ssum = 0.f;
  if (activation != 0) {
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j < E) m = fmaxf(m, key[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
#pragma unroll
    for (int j = 0; j < PER; ++j) ssum += (lane + 32 * j < E) ? expf(key[j] - m) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
  }
  auto score = [&](float x) -> float {
    return activation == 0 ? router_sigmoid(x) : expf(x - m) / ssum;
  };
  // Selection order: key descending, expert id ascending on equal keys -- a
  // total order, so the winners leave in exactly one sequence.  Each lane
  // keeps its two best remaining (key, id, score) entries; a round is one
  // warp-wide argmax over the lanes' bests, after which the winning lane
  // promotes its second.  Only a lane that has used up both rescans its
  // entries, for the two best strictly after the last one it gave up (every
  // better entry of the lane is already taken).
  auto before = [](float av, int ae, float bv, int be) { return sel_before(av, ae, bv, be); };
  float v1 = -FLT_MAX, v2 = -FLT_MAX, s1 = 0.f, s2 = 0.f;
  int e1 = INT_MAX, e2 = INT_MAX;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      const float sj = score(key[j]);
      const float kj = sj + (bias ? bias[e] : 0.f);
      key[j] = kj;
      if (before(kj, e, v1, e1)) {
        v2 = v1; e2 = e1; s2 = s1;
        v1 = kj; e1 = e; s1 = sj;
      } else if (before(kj, e, v2, e2)) {
        v2 = kj; e2 = e; s2 = sj;
      }
    } else {
      key[j] = -FLT_MAX;
    }
  }
  auto refill = [&](float tv, int te) {  // two best entries strictly after (tv, te)
    v1 = v2 = -FLT_MAX;
    e1 = e2 = INT_MAX;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && before(tv, te, key[j], e)) {
        if (before(key[j], e, v1, e1)) {
          v2 = v1; e2 = e1;
          v1 = key[j]; e1 = e;
        } else if (before(key[j], e, v2, e2)) {
          v2 = key[j]; e2 = e;
        }
      }
    }
    // their scores, recomputed from the logits
    s1 = e1 < E ? score(row[e1]) : 0.f;
    s2 = e2 < E ? score(row[e2]) : 0.f;
  };
  bool have2 = true;  // (v2, e2) is this lane's next entry after (v1, e1)
  float wsum = 0.f;
  float my_w = 0.f;
  int my_idx = 0;
  for (int s = 0; s < k; ++s) {
    // warp argmax in two hardware reductions: the largest key (as an
    // order-preserving unsigned), then the lowest expert id holding it; the
    // winner's lane is its id mod 32 (lane l holds experts l + 32j)
    const uint32_t fb = __float_as_uint(v1);
    const uint32_t ku = fb ^ ((fb & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, ku);
    const int bi = static_cast<int>(
        __reduce_min_sync(0xffffffffu, ku == kmax ? static_cast<uint32_t>(e1) : 0xFFFFFFFFu));
    const bool won = bi == e1;  // exactly one lane
    const float bv = v1;        // the winner's key (used by the winner only)
    const float bw = __shfl_sync(0xffffffffu, s1, bi & 31);
    wsum += bw;
    if (lane == s) {
      my_w = bw;
      my_idx = bi;
    }
    if (won) {
      if (have2) {
        v1 = v2; e1 = e2; s1 = s2;
        have2 = false;
      } else {
        v1 = -FLT_MAX;
        e1 = INT_MAX;  // exhausted until the rescan below
      }
    }
    // the winner had no second left: it rescans after the entry it just gave up
    if (__any_sync(0xffffffffu, won && e1 == INT_MAX) && s + 1 < k) {
      if (won && e1 == INT_MAX) {
        refill(bv, bi);
        have2 = true;
      }
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

// The same selection for few tokens (sigmoid scores): one 256-thread CTA
// per token instead of one warp, so a token's k rounds run on 256 lanes
// (E <= 1024: at most 4 experts per thread, expert threadIdx.x + 256 j).
// Each round every thread offers its best remaining (key, id), the warps
// reduce them with the same order-preserving unsigned max / lowest-id min as
// router_topk_kernel, and the eight warp winners meet in shared memory.  The
// winners, their order and the weight arithmetic (scores summed in selection
// order by one thread, w / (sum + 1e-20) when k > 1 and renormalize, times
// rsf) equal router_topk_kernel's, bit for bit; with one warp per token that
// kernel runs its k rounds serially per token, which at a few hundred tokens
// leaves most SMs idle and takes ~20 us.
constexpr int kTopkBlockThreads = 256;
constexpr int64_t kTopkBlockMaxTokens = 1024;

__global__ void __launch_bounds__(kTopkBlockThreads) router_topk_block_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int E, int k,
    int renormalize, float rsf, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w) {
  __shared__ uint32_t s_key[kTopkBlockThreads / 32];
  __shared__ int s_id[kTopkBlockThreads / 32];
  __shared__ float s_score[32];
  __shared__ int s_win[32];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const float* row = logits + static_cast<int64_t>(blockIdx.x) * E;
  float key[4], sc[4];
  bool live[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = tid + kTopkBlockThreads * j;
    live[j] = e < E;
    sc[j] = live[j] ? router_sigmoid(row[e]) : 0.f;
    key[j] = live[j] ? sc[j] + (bias ? bias[e] : 0.f) : -FLT_MAX;
    live[j] = live[j] && key[j] == key[j];  // a NaN key never wins
  }
  for (int s = 0; s < k; ++s) {
    // this thread's best remaining entry (ids increase with j)
    float bv = -FLT_MAX;
    int be = INT_MAX;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (live[j] && sel_before(key[j], tid + kTopkBlockThreads * j, bv, be)) {
        bv = key[j];
        be = tid + kTopkBlockThreads * j;
      }
    const uint32_t fb = __float_as_uint(bv);
    const uint32_t ku = fb ^ ((fb & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, ku);
    const uint32_t emin =
        __reduce_min_sync(0xffffffffu, ku == kmax ? static_cast<uint32_t>(be) : 0xFFFFFFFFu);
    if (lane == 0) {
      s_key[warp] = kmax;
      s_id[warp] = static_cast<int>(emin);
    }
    __syncthreads();
    uint32_t wk = s_key[0];
    int we = s_id[0];
#pragma unroll
    for (int w = 1; w < kTopkBlockThreads / 32; ++w) {
      const uint32_t kw = s_key[w];
      const int ew = s_id[w];
      if (kw > wk || (kw == wk && ew < we)) {
        wk = kw;
        we = ew;
      }
    }
    if (we == INT_MAX && tid == 0) {  // fewer than k selectable experts (NaN keys)
      s_score[s] = 0.f;
      s_win[s] = -1;
    }
    if (we % kTopkBlockThreads == tid && we != INT_MAX) {
      const int j = we / kTopkBlockThreads;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        if (jj == j) {
          live[jj] = false;
          s_score[s] = sc[jj];
        }
      s_win[s] = we;
    }
    __syncthreads();  // s_key/s_id are rewritten next round; s_score/s_win are complete
  }
  if (tid == 0) {
    float wsum = 0.f;
    for (int s = 0; s < k; ++s) wsum += s_score[s];
    for (int s = 0; s < k; ++s) {
      float w = s_score[s];
      if (k > 1 && renormalize) w = w / (wsum + 1e-20f);
      w = w * rsf;
      topk_idx[static_cast<int64_t>(blockIdx.x) * k + s] = s_win[s];
      topk_w[static_cast<int64_t>(blockIdx.x) * k + s] = w;
    }
  }
}

int router_topk(const float* logits, const float* bias, int64_t T, int64_t E, int64_t k,
                int activation, int renormalize, float rsf, int32_t* topk_idx, float* topk_w,
                cudaStream_t stream) {
  if (T < 0 || E <= 0 || E > 1024 || k <= 0 || k > 32 || k > E) return kBadShape;
  if (activation != 0 && activation != 1) return kBadShape;
  if (T == 0) return kOk;
  if (activation == 0 && T <= kTopkBlockMaxTokens) {
    router_topk_block_kernel<<<static_cast<int>(T), kTopkBlockThreads, 0, stream>>>(
        logits, bias, static_cast<int>(E), static_cast<int>(k), renormalize, rsf, topk_idx,
        topk_w);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
  }
  const int threads = 256;
  const int blocks = static_cast<int>((T * 32 + threads - 1) / threads);
  const int per = static_cast<int>((E + 31) / 32);
#define LMOE_ROUTER(P)                                                                      \
  router_topk_kernel<P><<<blocks, threads, 0, stream>>>(logits, bias, (int)T, (int)E, (int)k, \
                                                         activation, renormalize, rsf,        \
                                                         topk_idx, topk_w)
  if (per <= 2) LMOE_ROUTER(2);
  else if (per <= 4) LMOE_ROUTER(4);
  else if (per <= 8) LMOE_ROUTER(8);
  else if (per <= 16) LMOE_ROUTER(16);
  else if (per <= 28) LMOE_ROUTER(28);
  else LMOE_ROUTER(32);
#undef LMOE_ROUTER
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// =========================================================================== dispatch
// Stable counting sort of the (token, slot) entries by key:
//   key(i) = flat_ids[i] - start   if the id is in [start, start + num_keys)
//          = num_keys (sentinel)   otherwise, and for the padding entries
//                                   i >= T*k that fill the sort up to m_padded
// Position of entry i = bin_start[key] + (#entries of the same key in earlier
// chunks) + (#entries of the same key earlier in its chunk); the first
// m_padded positions are kept (tail drop on overflow).
constexpr int kDispThreads = 256;
constexpr int kDispItems = 8;                                // entries per thread
constexpr int kDispChunk = kDispThreads * kDispItems;        // entries per block
constexpr int kMaxBins = 2049;                               // num_keys + 1

struct DispatchWs {
  int32_t* counts;  // [bins][nchunks]  per-chunk counts, then per-chunk exclusive prefix
  int32_t* totals;  // [bins]
  int32_t* rank;    // [n_ext]          rank of the entry within its chunk and key
};

__device__ __forceinline__ int entry_key(const int32_t* flat_ids, int64_t i, int64_t S, int start,
                                         int num_keys) {
  if (i >= S) return num_keys;
  const int id = flat_ids[i];
  const int local = id - start;
  return (local >= 0 && local < num_keys) ? local : num_keys;
}

// Kernel 1: per-chunk histogram and stable in-chunk ranks.  Each warp owns a
// contiguous run of 32*kDispItems entries, processed 32 at a time in order;
// __match_any_sync finds equal keys inside a 32-entry round.
__global__ void __launch_bounds__(kDispThreads) dispatch_rank_kernel(
    const int32_t* __restrict__ flat_ids, int64_t S, int64_t n_ext, int start, int num_keys,
    int nchunks, DispatchWs ws) {
  extern __shared__ uint16_t whist[];  // [8 warps][bins]
  const int bins = num_keys + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * bins; i += blockDim.x) whist[i] = 0;
  __syncthreads();
  uint16_t* h = whist + warp * bins;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kDispChunk + warp * 32 * kDispItems;
  int keys[kDispItems];
  int ranks[kDispItems];
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int it = 0; it < kDispItems; ++it) {
    const int64_t i = base + it * 32 + lane;
    const bool live = i < n_ext;
    const int key = live ? entry_key(flat_ids, i, S, start, num_keys) : -1 - lane;  // dead lanes unique
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int before = __popc(peers & lt);
    const int leader = __ffs(peers) - 1;
    int r = 0;
    if (live) r = h[key] + before;
    __syncwarp();
    if (live && lane == leader) h[key] = static_cast<uint16_t>(h[key] + __popc(peers));
    __syncwarp();
    keys[it] = key;
    ranks[it] = r;
  }
  __syncthreads();
  // exclusive prefix over the 8 warps for every bin; chunk total to global
  for (int b = threadIdx.x; b < bins; b += blockDim.x) {
    int run = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int c = whist[w * bins + b];
      whist[w * bins + b] = static_cast<uint16_t>(run);
      run += c;
    }
    ws.counts[static_cast<int64_t>(b) * nchunks + blockIdx.x] = run;
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < kDispItems; ++it) {
    const int64_t i = base + it * 32 + lane;
    if (i < n_ext) ws.rank[i] = whist[warp * bins + keys[it]] + ranks[it];
  }
}

// Kernel 2: one warp per bin: exclusive prefix of its per-chunk counts, total.
__global__ void dispatch_bin_scan_kernel(int bins, int nchunks, DispatchWs ws) {
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (b >= bins) return;
  int32_t* row = ws.counts + static_cast<int64_t>(b) * nchunks;
  int carry = 0;
  for (int c0 = 0; c0 < nchunks; c0 += 32) {
    const int c = c0 + lane;
    const int v = (c < nchunks) ? row[c] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (c < nchunks) row[c] = carry + incl - v;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) ws.totals[b] = carry;
}



// Kernel 3: every block rebuilds the bin starts (exclusive scan of the totals)
// in shared memory, then scatters its chunk's entries.  Block 0 also writes
// group_sizes (kept counts after the m_out cap, plus the padding bucket).
__global__ void __launch_bounds__(kDispThreads) dispatch_scatter_kernel(
    const int32_t* __restrict__ flat_ids, const float* __restrict__ flat_w, int64_t S,
    int64_t n_ext, int start, int num_keys, int top_k, int64_t m_out, int pad_bucket, int nchunks,
    DispatchWs ws, DispatchOut o) {
  __shared__ int bin_start[kMaxBins + 1];
  __shared__ int warp_sums[kDispThreads / 32];
  const int bins = num_keys + 1;
  // block-wide exclusive scan of totals[0..bins)
  const int per = (bins + kDispThreads - 1) / kDispThreads;
  const int b0 = min(bins, static_cast<int>(threadIdx.x) * per), b1 = min(bins, b0 + per);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += ws.totals[b];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += warp_sums[w];
  int run = wbase + incl - local;
  for (int b = b0; b < b1; ++b) {
    bin_start[b] = run;
    run += ws.totals[b];
  }
  if (threadIdx.x == kDispThreads - 1) bin_start[bins] = run;
  __syncthreads();

  if (blockIdx.x == 0) {
    int kept_local = 0;
    for (int b = threadIdx.x; b < num_keys; b += blockDim.x) {
      const int64_t s0 = bin_start[b];
      const int64_t room = m_out - s0;
      const int64_t tb = ws.totals[b];
      const int64_t kept = room <= 0 ? 0 : (tb < room ? tb : room);
      o.group_sizes[b] = static_cast<int32_t>(kept);
      if (o.per_expert_counts) o.per_expert_counts[b] = static_cast<int32_t>(kept);
      kept_local += static_cast<int>(kept);
    }
    if (pad_bucket) {
      // padding bucket = m_out - sum(kept): reduce kept_local over the block
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) kept_local += __shfl_xor_sync(0xffffffffu, kept_local, off);
      __syncthreads();
      if (lane == 0) warp_sums[warp] = kept_local;
      __syncthreads();
      if (threadIdx.x == 0) {
        int tot = 0;
        for (int w = 0; w < kDispThreads / 32; ++w) tot += warp_sums[w];
        o.group_sizes[num_keys] = static_cast<int32_t>(m_out - tot);
      }
    }
  }

  const int64_t base = static_cast<int64_t>(blockIdx.x) * kDispChunk;
  for (int it = 0; it < kDispItems; ++it) {
    const int64_t i = base + it * kDispThreads + threadIdx.x;
    if (i >= n_ext) break;
    const int key = entry_key(flat_ids, i, S, start, num_keys);
    const int64_t pos = static_cast<int64_t>(bin_start[key]) +
                        ws.counts[static_cast<int64_t>(key) * nchunks + blockIdx.x] + ws.rank[i];
    const bool in_range = pos < m_out;
    if (i < S && o.slot_pos) o.slot_pos[i] = (in_range && key < num_keys) ? static_cast<int32_t>(pos) : -1;
    if (!in_range) continue;
    const bool valid = key < num_keys;
    if (o.order) o.order[pos] = static_cast<int32_t>(i);
    o.token_idx[pos] = valid ? static_cast<int32_t>(i / top_k) : -1;
    if (o.weight) o.weight[pos] = (valid && flat_w) ? flat_w[i] : 0.f;
    if (o.valid) o.valid[pos] = valid ? 1 : 0;
  }
}

// All three steps in one block for dispatches of at most one chunk
// (n_ext <= kDispChunk: a few hundred tokens): the in-chunk ranks of kernel 1,
// the bin totals kept in shared memory (with one chunk, kernel 2's per-chunk
// prefix is zero) and kernel 3's bin starts, group sizes and scatter.  The
// same positions, bit for bit, with one launch and no workspace round trips:
// at 2048 entries the three kernels were latency chains of ~10-15 us each.
__global__ void __launch_bounds__(kDispThreads) dispatch_single_chunk_kernel(
    const int32_t* __restrict__ flat_ids, const float* __restrict__ flat_w, int64_t S,
    int64_t n_ext, int start, int num_keys, int top_k, int64_t m_out, int pad_bucket,
    DispatchOut o) {
  extern __shared__ uint16_t whist[];  // [8 warps][bins], then int32 totals / starts
  const int bins = num_keys + 1;
  int32_t* totals = reinterpret_cast<int32_t*>(whist + ((8 * bins + 1) & ~1));
  int32_t* bin_start = totals + bins;
  __shared__ int warp_sums[kDispThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * bins; i += blockDim.x) whist[i] = 0;
  __syncthreads();
  // kernel 1's ranks: warp w owns entries [w * 32 * kDispItems, ...), 32 at a time
  uint16_t* h = whist + warp * bins;
  const int64_t base = static_cast<int64_t>(warp) * 32 * kDispItems;
  int keys[kDispItems];
  int ranks[kDispItems];
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int it = 0; it < kDispItems; ++it) {
    const int64_t i = base + it * 32 + lane;
    const bool live = i < n_ext;
    const int key = live ? entry_key(flat_ids, i, S, start, num_keys) : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int before = __popc(peers & lt);
    const int leader = __ffs(peers) - 1;
    int r = 0;
    if (live) r = h[key] + before;
    __syncwarp();
    if (live && lane == leader) h[key] = static_cast<uint16_t>(h[key] + __popc(peers));
    __syncwarp();
    keys[it] = key;
    ranks[it] = r;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < bins; b += blockDim.x) {
    int run = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int c = whist[w * bins + b];
      whist[w * bins + b] = static_cast<uint16_t>(run);
      run += c;
    }
    totals[b] = run;
  }
  __syncthreads();
  // kernel 3's bin starts: exclusive scan of the totals
  const int per = (bins + kDispThreads - 1) / kDispThreads;
  const int b0 = min(bins, static_cast<int>(threadIdx.x) * per), b1 = min(bins, b0 + per);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += totals[b];
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += warp_sums[w];
  int run = wbase + incl - local;
  for (int b = b0; b < b1; ++b) {
    bin_start[b] = run;
    run += totals[b];
  }
  __syncthreads();
  // group sizes: kept counts after the m_out cap, plus the padding bucket
  int kept_local = 0;
  for (int b = threadIdx.x; b < num_keys; b += blockDim.x) {
    const int64_t s0 = bin_start[b];
    const int64_t room = m_out - s0;
    const int64_t tb = totals[b];
    const int64_t kept = room <= 0 ? 0 : (tb < room ? tb : room);
    o.group_sizes[b] = static_cast<int32_t>(kept);
    if (o.per_expert_counts) o.per_expert_counts[b] = static_cast<int32_t>(kept);
    kept_local += static_cast<int>(kept);
  }
  if (pad_bucket) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) kept_local += __shfl_xor_sync(0xffffffffu, kept_local, off);
    __syncthreads();  // warp_sums is reused
    if (lane == 0) warp_sums[warp] = kept_local;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < kDispThreads / 32; ++w) tot += warp_sums[w];
      o.group_sizes[num_keys] = static_cast<int32_t>(m_out - tot);
    }
  }
  // the scatter, from this warp's own entries and ranks
#pragma unroll
  for (int it = 0; it < kDispItems; ++it) {
    const int64_t i = base + it * 32 + lane;
    if (i >= n_ext) continue;
    const int key = keys[it];
    const int64_t pos = static_cast<int64_t>(bin_start[key]) + whist[warp * bins + key] + ranks[it];
    const bool in_range = pos < m_out;
    if (i < S && o.slot_pos) o.slot_pos[i] = (in_range && key < num_keys) ? static_cast<int32_t>(pos) : -1;
    if (!in_range) continue;
    const bool valid = key < num_keys;
    if (o.order) o.order[pos] = static_cast<int32_t>(i);
    o.token_idx[pos] = valid ? static_cast<int32_t>(i / top_k) : -1;
    if (o.weight) o.weight[pos] = (valid && flat_w) ? flat_w[i] : 0.f;
    if (o.valid) o.valid[pos] = valid ? 1 : 0;
  }
}

// 8 bf16 -> 8 f16 (exact for magnitudes in f16's normal range)
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    const __half2 h = __floats2half2_rn(f.x, f.y);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Kernel 4: row gather, one warp per output row, 16-byte vectors.
//   out[p, :] = token_idx[p] >= 0 ? x[token_idx[p], :] : 0      (CONVERT: bf16 -> f16)
// Largest bf16 magnitude among 8 packed bf16 (NaN compares false and is ignored).
__device__ __forceinline__ float bf16x8_peak(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

template <bool CONVERT>
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint4* __restrict__ x,
                                                          const int32_t* __restrict__ token_idx,
                                                          uint4* __restrict__ out, int64_t rows,
                                                          int vec_per_row, int64_t x_rows,
                                                          int32_t* status) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  // f16 range guard of the converting form: the largest magnitude of the
  // row being converted (per lane), checked once per row
  float peak = 0.f;
  bool out_of_range = false;
  auto cv = [&peak](uint4 v) {
    if (!CONVERT) return v;
    peak = fmaxf(peak, bf16x8_peak(v));
    return bf16x8_to_f16x8(v);
  };
  // the next row's source index is fetched while this row is copied, and each
  // lane keeps eight 16-byte loads in flight, so neither load latency is paid
  // once per row.  The gathered rows are stored evict-first: every source row
  // is read k times spread over the whole output, and plain stores of the
  // (much larger) output would push the source rows out of L2 and have them
  // re-read from memory.
  int t_next = warp < rows ? token_idx[warp] : -1;
  for (int64_t p = warp; p < rows; p += nwarps) {
    const int t = t_next;
    t_next = p + nwarps < rows ? token_idx[p + nwarps] : -1;
    uint4* dst = out + p * vec_per_row;
    if (t >= 0 && t < x_rows) {
      const uint4* src = x + static_cast<int64_t>(t) * vec_per_row;
      int v = lane;
      for (; v + 224 < vec_per_row; v += 256) {
        uint4 a[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = __ldg(src + v + 32 * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) __stcs(dst + v + 32 * i, cv(a[i]));
      }
      for (; v + 96 < vec_per_row; v += 128) {
        const uint4 a = __ldg(src + v), b = __ldg(src + v + 32), c = __ldg(src + v + 64),
                    d = __ldg(src + v + 96);
        __stcs(dst + v, cv(a));
        __stcs(dst + v + 32, cv(b));
        __stcs(dst + v + 64, cv(c));
        __stcs(dst + v + 96, cv(d));
      }
      for (; v < vec_per_row; v += 32) __stcs(dst + v, cv(__ldg(src + v)));
      if (CONVERT) {
        // the whole row above f16's range, or all of it too small for f16
        // to carry accurately (see kF16RunMin)
        // peaks are non-negative, so their bit patterns order like the values
        const float rp = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(peak)));
        out_of_range |= rp > kF16Max || (rp > 0.f && rp < kF16RunMin);
        peak = 0.f;
      }
    } else {
      for (int v = lane; v < vec_per_row; v += 32) __stcs(dst + v, make_uint4(0, 0, 0, 0));
    }
  }
  if (CONVERT && out_of_range && lane == 0) record_status(status, kF16Range);
}

// The same copy in token order: warp w takes token t = w, reads its row once
// (8 x 16 bytes per lane in flight) and stores it at the k sorted positions
// slot_pos[t*k + s].  For a dropless dispatch every output row is some
// (token, slot)'s position, so this writes exactly gather_rows' output while
// reading each source row once instead of k times (and converts it and
// checks its f16 range once).  Rows no slot points at are left untouched.
template <bool CONVERT>
__global__ void __launch_bounds__(256) scatter_rows_kernel(const uint4* __restrict__ x,
                                                           const int32_t* __restrict__ slot_pos,
                                                           int64_t T, int k,
                                                           uint4* __restrict__ out, int64_t out_rows,
                                                           int vec_per_row, int32_t* status) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  bool out_of_range = false, bad_pos = false;
  for (int64_t t = warp; t < T; t += nwarps) {
    // lane s < k holds slot s's position
    const int32_t my_pos = lane < k ? slot_pos[t * k + lane] : -1;
    const uint4* src = x + t * vec_per_row;
    float peak = 0.f;
    for (int v0 = 0; v0 < vec_per_row; v0 += 256) {
      uint4 a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = v0 + lane + 32 * i;
        a[i] = v < vec_per_row ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
        if (CONVERT) {
          peak = fmaxf(peak, bf16x8_peak(a[i]));
          a[i] = bf16x8_to_f16x8(a[i]);
        }
      }
      for (int s = 0; s < k; ++s) {
        const int32_t p = __shfl_sync(0xffffffffu, my_pos, s);
        if (p < 0) continue;
        if (p >= out_rows) {
          bad_pos = true;
          continue;
        }
        uint4* dst = out + static_cast<int64_t>(p) * vec_per_row;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int v = v0 + lane + 32 * i;
          if (v < vec_per_row) __stcs(dst + v, a[i]);
        }
      }
    }
    if (CONVERT) {
      const float rp = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(peak)));
      out_of_range |= rp > kF16Max || (rp > 0.f && rp < kF16RunMin);
    }
  }
  if (lane == 0 && bad_pos) record_status(status, kDeviceBounds);
  if (CONVERT && out_of_range && lane == 0) record_status(status, kF16Range);
}

int scatter_rows(const void* x, const int32_t* slot_pos, int64_t T, int64_t k, void* out,
                 int64_t out_rows, int64_t row_bytes, int convert, int32_t* status,
                 cudaStream_t stream) {
  if (T < 0 || k <= 0 || k > 32 || out_rows < 0 || row_bytes <= 0 || row_bytes % 16 != 0)
    return kBadShape;
  if (row_bytes / 16 >= (1ll << 31) || convert < 0 || convert > 1) return kBadShape;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) return kUnsupported;
  if (T == 0) return kOk;
  const int threads = 256;
  const int64_t want = (T * 32 + threads - 1) / threads;
  const int blocks =
      static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms(current_device())) * 16));
  const int vpr = static_cast<int>(row_bytes / 16);
  if (convert)
    scatter_rows_kernel<true><<<blocks, threads, 0, stream>>>(
        static_cast<const uint4*>(x), slot_pos, T, static_cast<int>(k), static_cast<uint4*>(out),
        out_rows, vpr, status);
  else
    scatter_rows_kernel<false><<<blocks, threads, 0, stream>>>(
        static_cast<const uint4*>(x), slot_pos, T, static_cast<int>(k), static_cast<uint4*>(out),
        out_rows, vpr, status);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

size_t dispatch_workspace_bytes(int64_t n_ext, int64_t num_keys) {
  const int64_t nchunks = (n_ext + kDispChunk - 1) / kDispChunk;
  const int64_t bins = num_keys + 1;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  return static_cast<size_t>(al(bins * nchunks * 4) + al(bins * 4) + al(n_ext * 4));
}

int dispatch_sort(const int32_t* flat_ids, const float* flat_w, int64_t S, int64_t top_k,
                  int64_t start, int64_t num_keys, int64_t m_out, int pad_bucket, DispatchOut o,
                  void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (S < 0 || top_k <= 0 || num_keys <= 0 || num_keys + 1 > kMaxBins || m_out < 0)
    return kBadShape;
  if (S >= (1ll << 31) || m_out >= (1ll << 31)) return kBadShape;
  const int64_t n_ext = std::max<int64_t>(S, m_out);
  if (ws_bytes < dispatch_workspace_bytes(n_ext, num_keys) || (n_ext > 0 && workspace == nullptr))
    return kBadShape;
  if (n_ext == 0) {
    // no entries: every group is empty
    if (cudaMemsetAsync(o.group_sizes, 0, (num_keys + (pad_bucket ? 1 : 0)) * 4, stream) != cudaSuccess)
      return kLaunchFailed;
    if (o.per_expert_counts && cudaMemsetAsync(o.per_expert_counts, 0, num_keys * 4, stream) != cudaSuccess)
      return kLaunchFailed;
    return kOk;
  }
  const int nchunks = static_cast<int>((n_ext + kDispChunk - 1) / kDispChunk);
  const int bins = static_cast<int>(num_keys + 1);
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* p = static_cast<uint8_t*>(workspace);
  DispatchWs ws;
  ws.counts = reinterpret_cast<int32_t*>(p);
  p += al(static_cast<int64_t>(bins) * nchunks * 4);
  ws.totals = reinterpret_cast<int32_t*>(p);
  p += al(bins * 4);
  ws.rank = reinterpret_cast<int32_t*>(p);
  if (n_ext <= kDispChunk) {
    // one chunk: the fused single-block form
    const size_t sh1 = static_cast<size_t>((8 * bins + 1) & ~1) * sizeof(uint16_t) +
                       static_cast<size_t>(2 * bins) * sizeof(int32_t);
    if (sh1 > 48 * 1024 &&
        cudaFuncSetAttribute(dispatch_single_chunk_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sh1)) != cudaSuccess)
      return kLaunchFailed;
    dispatch_single_chunk_kernel<<<1, kDispThreads, sh1, stream>>>(
        flat_ids, flat_w, S, n_ext, static_cast<int>(start), static_cast<int>(num_keys),
        static_cast<int>(top_k), m_out, pad_bucket, o);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
  }
  const size_t sh = static_cast<size_t>(8) * bins * sizeof(uint16_t);
  if (sh > 48 * 1024) {
    if (cudaFuncSetAttribute(dispatch_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sh)) != cudaSuccess)
      return kLaunchFailed;
  }
  dispatch_rank_kernel<<<nchunks, kDispThreads, sh, stream>>>(flat_ids, S, n_ext,
                                                              static_cast<int>(start),
                                                              static_cast<int>(num_keys), nchunks, ws);
  dispatch_bin_scan_kernel<<<(bins * 32 + 255) / 256, 256, 0, stream>>>(bins, nchunks, ws);
  dispatch_scatter_kernel<<<nchunks, kDispThreads, 0, stream>>>(
      flat_ids, flat_w, S, n_ext, static_cast<int>(start), static_cast<int>(num_keys),
      static_cast<int>(top_k), m_out, pad_bucket, nchunks, ws, o);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int gather_rows(const void* x, int64_t x_rows, const int32_t* token_idx, void* out, int64_t rows,
                int64_t row_bytes, int convert, int32_t* status, cudaStream_t stream) {
  if (rows < 0 || row_bytes <= 0 || row_bytes % 16 != 0) return kBadShape;
  if (convert != 0 && convert != 1) return kBadShape;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) return kUnsupported;
  if (rows == 0) return kOk;
  const int threads = 256;
  const int64_t want = (rows * 32 + threads - 1) / threads;
  const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms(current_device())) * 16));
  if (convert)
    gather_rows_kernel<true><<<blocks, threads, 0, stream>>>(
        static_cast<const uint4*>(x), token_idx, static_cast<uint4*>(out), rows,
        static_cast<int>(row_bytes / 16), x_rows, status);
  else
    gather_rows_kernel<false><<<blocks, threads, 0, stream>>>(
        static_cast<const uint4*>(x), token_idx, static_cast<uint4*>(out), rows,
        static_cast<int>(row_bytes / 16), x_rows, status);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// =========================================================================== combine
// routed[t] = bf16( sum_s out[slot_pos[t*k+s]] * w[t,s] )   (f32, slot order)
// normed[t] = bf16( bf16(routed * 1/sqrt(mean(routed^2) + eps)) * scale )
// One block per token; L elements staged in shared memory as f32.
template <bool BF16_IO>
__global__ void __launch_bounds__(256) combine_rmsnorm_kernel(
    const void* __restrict__ expert_out, const int32_t* __restrict__ slot_pos,
    const float* __restrict__ topk_w, const void* __restrict__ norm_scale, int T, int k, int L,
    float eps, void* __restrict__ routed_out, void* __restrict__ normed_out) {
  extern __shared__ float racc[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < L; c += blockDim.x) racc[c] = 0.f;
  // no barrier needed: each thread owns the same columns in every loop below
  for (int s = 0; s < k; ++s) {
    const int p = slot_pos[static_cast<int64_t>(t) * k + s];
    const float w = topk_w[static_cast<int64_t>(t) * k + s];
    if (p < 0) continue;
    if (BF16_IO) {
      const __nv_bfloat16* row = static_cast<const __nv_bfloat16*>(expert_out) + static_cast<int64_t>(p) * L;
      for (int c = threadIdx.x; c < L; c += blockDim.x)
        racc[c] = __fadd_rn(racc[c], __fmul_rn(__bfloat162float(row[c]), w));
    } else {
      const float* row = static_cast<const float*>(expert_out) + static_cast<int64_t>(p) * L;
      for (int c = threadIdx.x; c < L; c += blockDim.x)
        racc[c] = __fadd_rn(racc[c], __fmul_rn(row[c], w));
    }
  }
  float ss = 0.f;
  for (int c = threadIdx.x; c < L; c += blockDim.x) {
    float v = racc[c];
    if (BF16_IO) v = bf16_round_f(v);
    racc[c] = v;
    ss += v * v;
    if (routed_out) {
      if (BF16_IO)
        static_cast<__nv_bfloat16*>(routed_out)[static_cast<int64_t>(t) * L + c] = __float2bfloat16_rn(v);
      else
        static_cast<float*>(routed_out)[static_cast<int64_t>(t) * L + c] = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float var = red[0] / static_cast<float>(L);
  const float inv = 1.0f / sqrtf(var + eps);
  if (normed_out) {
    for (int c = threadIdx.x; c < L; c += blockDim.x) {
      float n = racc[c] * inv;
      if (BF16_IO) {
        n = bf16_round_f(n);
        const float sc = __bfloat162float(static_cast<const __nv_bfloat16*>(norm_scale)[c]);
        static_cast<__nv_bfloat16*>(normed_out)[static_cast<int64_t>(t) * L + c] = __float2bfloat16_rn(n * sc);
      } else {
        const float sc = static_cast<const float*>(norm_scale)[c];
        static_cast<float*>(normed_out)[static_cast<int64_t>(t) * L + c] = n * sc;
      }
    }
  }
}

// bf16 fast path: one block per token, each thread owns CH chunks of 8
// consecutive columns (16-byte loads and stores), accumulates the k slot rows
// in f32 registers in slot order (same arithmetic as the generic kernel), and
// the RMS statistic is a block reduction of the bf16-rounded routed values.
template <int CH>
__global__ void __launch_bounds__(256) combine_rmsnorm_bf16_vec_kernel(
    const __nv_bfloat16* __restrict__ expert_out, const int32_t* __restrict__ slot_pos,
    const float* __restrict__ topk_w, const __nv_bfloat16* __restrict__ norm_scale, int k, int L,
    float eps, __nv_bfloat16* __restrict__ routed_out, __nv_bfloat16* __restrict__ normed_out) {
  __shared__ float red[8];
  const int t = blockIdx.x;
  const int nchunk = L / 8;
  float acc[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[c][e] = 0.f;
  for (int s = 0; s < k; ++s) {
    const int p = __ldg(slot_pos + static_cast<int64_t>(t) * k + s);
    const float w = __ldg(topk_w + static_cast<int64_t>(t) * k + s);
    if (p < 0) continue;
    const uint4* row = reinterpret_cast<const uint4*>(expert_out + static_cast<int64_t>(p) * L);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int ch = threadIdx.x + c * 256;
      if (ch < nchunk) {
        const uint4 v = __ldg(row + ch);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
          acc[c][2 * e] = __fadd_rn(acc[c][2 * e], __fmul_rn(f.x, w));
          acc[c][2 * e + 1] = __fadd_rn(acc[c][2 * e + 1], __fmul_rn(f.y, w));
        }
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = threadIdx.x + c * 256;
    if (ch < nchunk) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc[c][e] = bf16_round_f(acc[c][e]);
        ss += acc[c][e] * acc[c][e];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) pk[e] = pack_bf16x2(acc[c][2 * e], acc[c][2 * e + 1]);
      if (routed_out)
        reinterpret_cast<uint4*>(routed_out + static_cast<int64_t>(t) * L)[ch] =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(L) + eps);
  if (normed_out == nullptr) return;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = threadIdx.x + c * 256;
    if (ch < nchunk) {
      const uint4 sv = __ldg(reinterpret_cast<const uint4*>(norm_scale) + ch);
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 sc = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sw[e]));
        const float n0 = bf16_round_f(acc[c][2 * e] * inv) * sc.x;
        const float n1 = bf16_round_f(acc[c][2 * e + 1] * inv) * sc.y;
        pk[e] = pack_bf16x2(n0, n1);
      }
      reinterpret_cast<uint4*>(normed_out + static_cast<int64_t>(t) * L)[ch] =
          make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

int combine_rmsnorm(const void* expert_out, const int32_t* slot_pos, const float* topk_w,
                    const void* norm_scale, int64_t T, int64_t k, int64_t L, float eps, int bf16,
                    void* routed_out, void* normed_out, cudaStream_t stream) {
  if (T < 0 || k <= 0 || L <= 0 || L > 12288) return kBadShape;  // L f32 values in 48 KB smem
  if (T == 0) return kOk;
  const bool aligned = ((reinterpret_cast<uintptr_t>(expert_out) |
                         reinterpret_cast<uintptr_t>(norm_scale) |
                         reinterpret_cast<uintptr_t>(routed_out) |
                         reinterpret_cast<uintptr_t>(normed_out)) & 15) == 0;
  if (bf16 && aligned && L % 8 == 0 && L <= 8 * 256 * 4) {
    const int ch = static_cast<int>((L / 8 + 255) / 256);
    auto eo = static_cast<const __nv_bfloat16*>(expert_out);
    auto ns = static_cast<const __nv_bfloat16*>(norm_scale);
    auto ro = static_cast<__nv_bfloat16*>(routed_out);
    auto no = static_cast<__nv_bfloat16*>(normed_out);
    const int grid = static_cast<int>(T);
    if (ch == 1)
      combine_rmsnorm_bf16_vec_kernel<1><<<grid, 256, 0, stream>>>(eo, slot_pos, topk_w, ns, (int)k, (int)L, eps, ro, no);
    else if (ch == 2)
      combine_rmsnorm_bf16_vec_kernel<2><<<grid, 256, 0, stream>>>(eo, slot_pos, topk_w, ns, (int)k, (int)L, eps, ro, no);
    else
      combine_rmsnorm_bf16_vec_kernel<4><<<grid, 256, 0, stream>>>(eo, slot_pos, topk_w, ns, (int)k, (int)L, eps, ro, no);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
  }
  const size_t sh = static_cast<size_t>(L) * sizeof(float);
  if (bf16)
    combine_rmsnorm_kernel<true><<<static_cast<int>(T), 256, sh, stream>>>(
        expert_out, slot_pos, topk_w, norm_scale, (int)T, (int)k, (int)L, eps, routed_out, normed_out);
  else
    combine_rmsnorm_kernel<false><<<static_cast<int>(T), 256, sh, stream>>>(
        expert_out, slot_pos, topk_w, norm_scale, (int)T, (int)k, (int)L, eps, routed_out, normed_out);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// =========================================================================== scatter-add
// routed[idx[p], :] += dtype(shard_out[p, :] * w[p])  for every padded row p
// with idx[p] >= 0 (idx == -1 rows carry weight 0 by construction).
// One warp per row, bf16x2 atomics (f32 atomics for the f32 variant).
template <bool BF16_IO>
__global__ void __launch_bounds__(256) scatter_add_kernel(const void* __restrict__ shard_out,
                                                          const int32_t* __restrict__ idx,
                                                          const float* __restrict__ w,
                                                          void* routed, int64_t rows, int L, int T) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int t = idx[warp];
  const float wv = w[warp];
  if (t < 0 || t >= T || wv == 0.f) return;
  if (BF16_IO) {
    const __nv_bfloat162* src =
        reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(shard_out) + warp * L);
    __nv_bfloat162* dst =
        reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(routed) + static_cast<int64_t>(t) * L);
    for (int c = lane; c < L / 2; c += 32) {
      const float2 v = __bfloat1622float2(src[c]);
      atomicAdd(dst + c, __floats2bfloat162_rn(v.x * wv, v.y * wv));
    }
  } else {
    const float* src = static_cast<const float*>(shard_out) + warp * L;
    float* dst = static_cast<float*>(routed) + static_cast<int64_t>(t) * L;
    for (int c = lane; c < L; c += 32) atomicAdd(dst + c, src[c] * wv);
  }
}

int scatter_add(const void* shard_out, const int32_t* idx, const float* w, void* routed,
                int64_t rows, int64_t L, int64_t T, int bf16, cudaStream_t stream) {
  if (rows < 0 || L <= 0 || T < 0 || (bf16 && L % 2)) return kBadShape;
  if (rows == 0) return kOk;
  const int blocks = static_cast<int>((rows * 32 + 255) / 256);
  if (bf16)
    scatter_add_kernel<true><<<blocks, 256, 0, stream>>>(shard_out, idx, w, routed, rows, (int)L, (int)T);
  else
    scatter_add_kernel<false><<<blocks, 256, 0, stream>>>(shard_out, idx, w, routed, rows, (int)L, (int)T);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// =========================================================================== EP reorder
// Expert-parallel receive side.  Rows arrive from the all-to-all grouped by
// source rank, and within a source block ordered by local expert (the sender's
// dispatch sorts by global expert id).  For recv_counts[s][e] (rows source s
// sent for local expert e):
//   em_src[p] = q   expert-major position p takes received row q
//   sm_src[q] = p   (inverse) expert-major row that returns to received row q
//   group_sizes[e] = sum_s recv_counts[s][e]
// Expert-major order is (expert, source, arrival), so each expert's rows keep
// their source-rank order and the grouped GEMM sees one contiguous group per
// local expert.
constexpr int kMaxEpBlocks = 4096;  // world * local experts

__global__ void __launch_bounds__(256) ep_reorder_kernel(const int32_t* __restrict__ recv_counts,
                                                         int world, int n_local, int64_t rows_cap,
                                                         int32_t* __restrict__ em_src,
                                                         int32_t* __restrict__ sm_src,
                                                         int32_t* __restrict__ group_sizes) {
  __shared__ int src_off[kMaxEpBlocks + 1];  // block (s, e) start in source-major order
  __shared__ int exp_off[kMaxEpBlocks];      // block (s, e) start in expert-major order
  const int nb = world * n_local;
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < nb; ++i) {
      src_off[i] = run;
      run += recv_counts[i];
    }
    src_off[nb] = run;
    run = 0;
    for (int e = 0; e < n_local; ++e)
      for (int s = 0; s < world; ++s) {
        exp_off[s * n_local + e] = run;
        run += recv_counts[s * n_local + e];
      }
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < n_local; e += blockDim.x) {
      int t = 0;
      for (int s = 0; s < world; ++s) t += recv_counts[s * n_local + e];
      group_sizes[e] = t;
    }
  }
  const int64_t received = src_off[nb];
  const int64_t total = received < rows_cap ? received : rows_cap;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < total;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int lo = 0, hi = nb - 1;  // last block with src_off <= q (empty blocks skipped)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (src_off[mid] <= q) lo = mid; else hi = mid - 1;
    }
    const int64_t p = exp_off[lo] + (q - src_off[lo]);
    em_src[p] = static_cast<int32_t>(q);
    sm_src[q] = static_cast<int32_t>(p);
  }
}

int ep_reorder(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t rows_cap,
               int32_t* em_src, int32_t* sm_src, int32_t* group_sizes, cudaStream_t stream) {
  if (world <= 0 || n_local <= 0 || world * n_local > kMaxEpBlocks || rows_cap < 0)
    return kBadShape;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((rows_cap + 255) / 256, 1024)));
  ep_reorder_kernel<<<blocks, 256, 0, stream>>>(recv_counts, (int)world, (int)n_local, rows_cap,
                                                em_src, sm_src, group_sizes);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

// =========================================================================== SiTU-GLU
// out = dtype(beta*tanh(g/beta)*sigmoid(g) * lb*tanh(u/lb)), f32 math.
// gate/up may be two arrays or the two halves of one fused [gate|up] row.
template <bool BF16_IO>
__global__ void situ_kernel(const void* __restrict__ gate, const void* __restrict__ up,
                            int64_t ld_in, void* __restrict__ out, int64_t rows, int64_t I,
                            float beta, float lbeta) {
  const int64_t n = rows * I;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / I, c = i - r * I;
    float g, u;
    if (BF16_IO) {
      g = __bfloat162float(static_cast<const __nv_bfloat16*>(gate)[r * ld_in + c]);
      u = __bfloat162float(static_cast<const __nv_bfloat16*>(up)[r * ld_in + c]);
    } else {
      g = static_cast<const float*>(gate)[r * ld_in + c];
      u = static_cast<const float*>(up)[r * ld_in + c];
    }
    const float v = situ_fast(g, u, beta, 1.0f / beta, lbeta, 1.0f / lbeta);
    if (BF16_IO) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else static_cast<float*>(out)[i] = v;
  }
}

int situ_and_mul(const void* gate, const void* up, int64_t ld_in, void* out, int64_t rows,
                 int64_t I, float beta, float lbeta, int bf16, cudaStream_t stream) {
  if (rows < 0 || I <= 0 || ld_in < I) return kBadShape;
  if (rows == 0) return kOk;
  const int blocks = static_cast<int>(std::min<int64_t>((rows * I + 255) / 256, 148 * 32));
  if (bf16) situ_kernel<true><<<blocks, 256, 0, stream>>>(gate, up, ld_in, out, rows, I, beta, lbeta);
  else situ_kernel<false><<<blocks, 256, 0, stream>>>(gate, up, ld_in, out, rows, I, beta, lbeta);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace lmoe
