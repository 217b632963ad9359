// Expert-parallel exchange over NVLink peer memory: the dispatch all-to-all
// fused with the row gather, and the return all-to-all, as device kernels
// that store straight into the peer GPUs' buffers (one process per GPU; every
// rank maps every peer's buffer through CUDA IPC).  No host synchronisation: the
// per-expert row counts travel through peer memory too, and every offset is
// computed on the device.  Plain peer stores only (no TMA on peer memory).
//
// Symmetric buffer layout (same byte offsets on every rank), see ep_layout():
//   flags   [3][world] u32   epoch of the last (counts, rows, returns) signal from each source
//   done    [3] u32          grid-completion counters of the two put kernels; the
//                            exchange epoch (bumped by each counts exchange)
//   counts  [world][E] i32   counts[s][g] = rows source s routes to global expert g
//   tables  (local use)      base[E], cum[E+1], exp_off[E+1], src_pos[E] (see below)
//   recv    [recv_cap][row_bytes]   rows this rank's experts receive, expert-major:
//                                   (local expert, source, arrival order)
//   back    [back_cap][row_bytes]   this rank's routed rows coming back, in its own
//                                   dispatch (global-expert-sorted) order
// Rank r owns global experts [r*El, (r+1)*El).  With cnt = counts:
//   exp_off_d(e, s) = sum_{e'<e} sum_s' cnt[s'][d*El+e'] + sum_{s'<s} cnt[s'][d*El+e]
//     (start of source s's rows for rank d's local expert e in d's recv buffer)
//   cum_s(g) = sum_{g'<g} cnt[s][g']   (start of global expert g in s's dispatch order)
//   base[g]       = exp_off_{g/El}(g%El, r)              (this rank sending)
//   cum[g]        = cum_r(g)
//   exp_off[e*world+s] = exp_off_r(e, s)                 (this rank receiving)
//   src_pos[e*world+s] = cum_s(r*El + e)
// Every wait on another rank is bounded: by LMOE_WAIT_TIMEOUT_NS unless
// lmoe_set_peer_wait_timeout_ns chose another limit; a timeout records
// LMOE_WAIT_TIMEOUT in the status word and the kernel returns.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <cstdint>

#include "../../include/lmoe.h"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

constexpr int kEpMaxExperts = 2048;
constexpr int kEpMaxWorld = 8;

struct EpLayout {
  int64_t flags, done, counts, tables, recv, back, total;
};

__host__ __device__ inline int64_t ep_align(int64_t v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline EpLayout ep_layout(int world, int E, int64_t recv_cap,
                                              int64_t back_cap, int64_t row_bytes) {
  EpLayout l;
  l.flags = 0;
  l.done = ep_align(3 * world * 4);
  l.counts = l.done + 256;
  l.tables = ep_align(l.counts + static_cast<int64_t>(world) * E * 4);
  l.recv = ep_align(l.tables + (4 * static_cast<int64_t>(E) + 2) * 4);
  l.back = ep_align(l.recv + recv_cap * row_bytes);
  l.total = ep_align(l.back + back_cap * row_bytes);
  return l;
}

struct EpArgs {
  uint8_t* const* peers;  // device array [world] of symmetric-buffer bases (peers[rank] = own)
  int rank, world, E, n_local;
  int64_t recv_cap, back_cap, row_bytes;
  uint32_t epoch;  // set on the device from the epoch word
  int32_t* status;
  uint64_t timeout_ns;  // limit of every wait on another rank's signal
};

struct EpTablePtrs {
  int32_t *base, *cum, *exp_off, *src_pos;
};

// this rank's exchange epoch: one more per counts exchange, the same count on
// every rank (each rank runs the same exchanges), so no host counter is needed
// and a captured CUDA graph replays correctly
__device__ __forceinline__ uint32_t* ep_epoch_word(const EpArgs& a, const EpLayout& l) {
  return reinterpret_cast<uint32_t*>(a.peers[a.rank] + l.done) + 2;
}

__device__ __forceinline__ EpTablePtrs ep_tables(const EpArgs& a, const EpLayout& l) {
  int32_t* t = reinterpret_cast<int32_t*>(a.peers[a.rank] + l.tables);
  return {t, t + a.E, t + 2 * a.E + 1, t + 3 * a.E + 2};
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// epochs grow by one per exchange; wrap-safe "reached" test
__device__ __forceinline__ bool epoch_reached(uint32_t seen, uint32_t want) {
  return static_cast<int32_t>(seen - want) >= 0;
}

// Bounded wait until flags[s] reached epoch for every source s (one thread).
__device__ bool wait_all_sources(const uint32_t* flags, int world, uint32_t epoch,
                                 int32_t* status, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while (!epoch_reached(ld_acquire_sys(flags + s), epoch)) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        record_status(status, kWaitTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// --------------------------------------------------------------------------- counts
// Exclusive prefix sum of v[0..n) in shared memory by the whole block (256
// threads, n <= 256 * kScanPer); returns the total.
constexpr int kScanPer = kEpMaxExperts / 256;

__device__ int block_exclusive_scan(int32_t* v, int n) {
  __shared__ int32_t warp_tot[8];
  __shared__ int32_t total;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int b0 = t * kScanPer;
  int local[kScanPer];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    local[i] = (b0 + i < n) ? v[b0 + i] : 0;
    sum += local[i];
  }
  int inc = sum;  // inclusive scan of the per-thread sums
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_tot[w] = inc;
  __syncthreads();
  if (t == 0) {
    int run = 0;
    for (int i = 0; i < 8; ++i) {
      const int x = warp_tot[i];
      warp_tot[i] = run;
      run += x;
    }
    total = run;
  }
  __syncthreads();
  int run = warp_tot[w] + inc - sum;
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    if (b0 + i < n) v[b0 + i] = run;
    run += local[i];
  }
  __syncthreads();
  return total;
}

// One block: publish this rank's per-expert counts into every peer's matrix,
// signal, wait for every source's counts, then build this rank's offset
// tables and local group sizes (rows per local expert over all sources), all
// with block-parallel prefix sums over the experts.
__global__ void __launch_bounds__(256) ep_counts_kernel(EpArgs a, const int32_t* __restrict__ gs,
                                                        int32_t* __restrict__ local_gs) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    uint32_t* w = ep_epoch_word(a, l);
    epoch = *w + 1u;
    *w = epoch;
  }
  __syncthreads();
  a.epoch = epoch;
  for (int d = 0; d < a.world; ++d) {
    int32_t* dst = reinterpret_cast<int32_t*>(a.peers[d] + l.counts) + a.rank * a.E;
    for (int g = threadIdx.x; g < a.E; g += blockDim.x) dst[g] = gs[g];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world) {
    uint32_t* f = reinterpret_cast<uint32_t*>(a.peers[threadIdx.x] + l.flags);
    st_release_sys(f + 0 * a.world + a.rank, a.epoch);
  }
  __shared__ int ok;
  if (threadIdx.x == 0)
    ok = wait_all_sources(reinterpret_cast<const uint32_t*>(a.peers[a.rank] + l.flags), a.world,
                          a.epoch, a.status, a.timeout_ns);
  __syncthreads();
  const EpTablePtrs t = ep_tables(a, l);
  const int El = a.n_local, W = a.world, E = a.E, r = a.rank;
  if (!ok) {
    // timed out: empty tables, so the puts and the expert GEMMs do no work
    for (int e = threadIdx.x; e < El; e += blockDim.x) local_gs[e] = 0;
    if (threadIdx.x == 0) {
      t.cum[E] = 0;
      t.exp_off[El * W] = 0;
    }
    return;
  }
  const int32_t* cnt = reinterpret_cast<const int32_t*>(a.peers[a.rank] + l.counts);
  __shared__ int32_t tot[kEpMaxExperts];     // rows all sources send to expert g -> its scan
  __shared__ int32_t mine[kEpMaxExperts];    // rows this rank sends to expert g -> its scan
  __shared__ int32_t before[kEpMaxExperts];  // rows sources < r send to expert g
  for (int g = threadIdx.x; g < E; g += blockDim.x) {
    int s_all = 0, s_before = 0;
    for (int s = 0; s < W; ++s) {
      const int c = cnt[s * E + g];
      s_all += c;
      if (s < r) s_before += c;
    }
    tot[g] = s_all;
    before[g] = s_before;
    mine[g] = cnt[r * E + g];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < El; e += blockDim.x) local_gs[e] = tot[r * El + e];
  const int recv_total_all = block_exclusive_scan(tot, E);  // tot -> exclusive scan
  const int send_total = block_exclusive_scan(mine, E);     // mine -> cum of this rank
  // sending side: row p of global expert g goes to rank d = g / El at
  // base[g] + (p - cum[g]) of d's receive region
  for (int g = threadIdx.x; g < E; g += blockDim.x) {
    t.base[g] = tot[g] - tot[(g / El) * El] + before[g];
    t.cum[g] = mine[g];
  }
  // receiving side: block (e, s) of this rank's region starts at exp_off[e*W+s]
  const int g0 = r * El;
  const int recv_total = (r + 1 < W ? tot[g0 + El] : recv_total_all) - tot[g0];
  for (int i = threadIdx.x; i < El * W; i += blockDim.x) {
    const int e = i / W, s = i % W;
    int pre = 0;
    for (int s2 = 0; s2 < s; ++s2) pre += cnt[s2 * E + g0 + e];
    t.exp_off[i] = tot[g0 + e] - tot[g0] + pre;
  }
  // src_pos[e*W+s] = rows source s routes to experts below g0 + e (the
  // dispatch-order position of its rows for this rank's expert e): warp s
  // reduces row s below g0, then scans it across the El local experts
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int s = warp; s < W; s += blockDim.x / 32) {
    const int32_t* row = cnt + s * E;
    int pre = 0;
    for (int g = lane; g < g0; g += 32) pre += row[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
    int run = pre;
    for (int e0 = 0; e0 < El; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < El ? row[g0 + e] : 0;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      if (e < El) t.src_pos[e * W + s] = run + inc - c;
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  __shared__ int over;
  if (threadIdx.x == 0) {
    over = recv_total > a.recv_cap || send_total > a.back_cap;
    t.cum[E] = over ? 0 : send_total;
    t.exp_off[El * W] = over ? 0 : recv_total;
    if (over) record_status(a.status, kDeviceBounds);  // run nothing downstream
  }
  __syncthreads();
  if (over)
    for (int e = threadIdx.x; e < El; e += blockDim.x) local_gs[e] = 0;
}

// --------------------------------------------------------------------------- dispatch put
// Row p of this rank's dispatch order (global-expert sorted) is x[token_idx[p]];
// it goes to rank d = g / El at position base[g] + (p - cum[g]) of d's recv
// buffer.  One warp per row, 16-byte vectors; the last block to finish
// signals every peer.
__global__ void __launch_bounds__(256) ep_dispatch_put_kernel(EpArgs a, const uint8_t* __restrict__ x,
                                                              int64_t x_rows,
                                                              const int32_t* __restrict__ token_idx,
                                                              int64_t S) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  a.epoch = *ep_epoch_word(a, l);  // set by this exchange's counts kernel
  const EpTablePtrs t = ep_tables(a, l);
  __shared__ int32_t base[kEpMaxExperts];
  __shared__ int32_t cum[kEpMaxExperts + 1];
  for (int g = threadIdx.x; g < a.E; g += blockDim.x) {
    base[g] = t.base[g];
    cum[g] = t.cum[g];
  }
  if (threadIdx.x == 0) cum[a.E] = t.cum[a.E];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int vec = static_cast<int>(a.row_bytes / 16);
  const int64_t S_eff = S < cum[a.E] ? S : cum[a.E];
  for (int64_t p = warp; p < S_eff; p += nwarps) {
    int lo = 0, hi = a.E - 1;  // global expert of row p: last g with cum[g] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cum[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int d = g / a.n_local;
    const int64_t pos = base[g] + (p - cum[g]);
    const int tok = token_idx[p];
    if (pos >= a.recv_cap || tok < 0 || tok >= x_rows) {
      if (lane == 0) record_status(a.status, kDeviceBounds);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * a.row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(a.peers[d] + l.recv + pos * a.row_bytes);
    for (int v = lane; v < vec; v += 32) dst[v] = __ldg(src + v);
  }
  // grid completion: the last block publishes the rows to every peer
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* done = reinterpret_cast<uint32_t*>(a.peers[a.rank] + l.done);
    if (atomicAdd(done + 0, 1u) == gridDim.x - 1) {
      done[0] = 0;
      __threadfence_system();
      for (int dd = 0; dd < a.world; ++dd)
        st_release_sys(reinterpret_cast<uint32_t*>(a.peers[dd] + l.flags) + 1 * a.world + a.rank,
                       a.epoch);
    }
  }
}

// --------------------------------------------------------------------------- waits
// One thread: wait until every source signalled `which` (1 rows, 2 returns)
// for this epoch.
__global__ void ep_wait_kernel(EpArgs a, int which) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  a.epoch = *ep_epoch_word(a, l);  // set by this exchange's counts kernel
  if (threadIdx.x == 0 && blockIdx.x == 0)
    wait_all_sources(reinterpret_cast<const uint32_t*>(a.peers[a.rank] + l.flags) + which * a.world,
                     a.world, a.epoch, a.status, a.timeout_ns);
}

// --------------------------------------------------------------------------- return put
// Expert-major row q of this rank (block (e, s), j-th) returns to source s at
// position src_pos[e*world+s] + j of s's dispatch order.
__global__ void __launch_bounds__(256) ep_return_put_kernel(EpArgs a, const uint8_t* __restrict__ y,
                                                            int64_t R) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  a.epoch = *ep_epoch_word(a, l);  // set by this exchange's counts kernel
  const EpTablePtrs t = ep_tables(a, l);
  __shared__ int32_t exp_off[kEpMaxExperts + 1];
  __shared__ int32_t src_pos[kEpMaxExperts];
  const int nb = a.n_local * a.world;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    exp_off[i] = t.exp_off[i];
    src_pos[i] = t.src_pos[i];
  }
  if (threadIdx.x == 0) exp_off[nb] = t.exp_off[nb];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int vec = static_cast<int>(a.row_bytes / 16);
  const int64_t R_eff = R < exp_off[nb] ? R : exp_off[nb];
  for (int64_t q = warp; q < R_eff; q += nwarps) {
    int lo = 0, hi = nb - 1;  // last block with exp_off <= q
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (exp_off[mid] <= q) lo = mid; else hi = mid - 1;
    }
    const int s = lo % a.world;
    const int64_t pos = src_pos[lo] + (q - exp_off[lo]);
    if (pos >= a.back_cap) {
      if (lane == 0) record_status(a.status, kDeviceBounds);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(y + q * a.row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(a.peers[s] + l.back + pos * a.row_bytes);
    for (int v = lane; v < vec; v += 32) dst[v] = __ldg(src + v);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* done = reinterpret_cast<uint32_t*>(a.peers[a.rank] + l.done);
    if (atomicAdd(done + 1, 1u) == gridDim.x - 1) {
      done[1] = 0;
      __threadfence_system();
      for (int dd = 0; dd < a.world; ++dd)
        st_release_sys(reinterpret_cast<uint32_t*>(a.peers[dd] + l.flags) + 2 * a.world + a.rank,
                       a.epoch);
    }
  }
}

// --------------------------------------------------------------------------- fused return
// Destination of every received row: expert-major row q (block (e, s),
// j-th) belongs at position src_pos[e*world+s] + j of source s's return
// region.  A GEMM given these addresses stores its output rows straight into
// the sources' buffers over NVLink, so the return needs no copy kernel.
__global__ void __launch_bounds__(256) ep_row_dest_kernel(EpArgs a, uint64_t* __restrict__ dest,
                                                          int64_t R) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  const EpTablePtrs t = ep_tables(a, l);
  __shared__ int32_t exp_off[kEpMaxExperts + 1];
  __shared__ int32_t src_pos[kEpMaxExperts];
  const int nb = a.n_local * a.world;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    exp_off[i] = t.exp_off[i];
    src_pos[i] = t.src_pos[i];
  }
  if (threadIdx.x == 0) exp_off[nb] = t.exp_off[nb];
  __syncthreads();
  const int64_t R_eff = R < exp_off[nb] ? R : exp_off[nb];
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < R_eff;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int lo = 0, hi = nb - 1;  // last block with exp_off <= q
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (exp_off[mid] <= q) lo = mid; else hi = mid - 1;
    }
    const int64_t pos = src_pos[lo] + (q - exp_off[lo]);
    if (pos >= a.back_cap) {
      record_status(a.status, kDeviceBounds);
      dest[q] = reinterpret_cast<uint64_t>(a.peers[a.rank] + l.back);  // a harmless own row
      continue;
    }
    dest[q] = reinterpret_cast<uint64_t>(a.peers[lo % a.world] + l.back + pos * a.row_bytes);
  }
}

// One thread: after the kernel that stored this rank's returned rows into the
// sources' buffers, signal every source, then wait (bounded) until every
// rank's rows for this rank have landed.
__global__ void ep_return_signal_kernel(EpArgs a) {
  const EpLayout l = ep_layout(a.world, a.E, a.recv_cap, a.back_cap, a.row_bytes);
  a.epoch = *ep_epoch_word(a, l);
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  for (int d = 0; d < a.world; ++d)
    st_release_sys(reinterpret_cast<uint32_t*>(a.peers[d] + l.flags) + 2 * a.world + a.rank,
                   a.epoch);
  wait_all_sources(reinterpret_cast<const uint32_t*>(a.peers[a.rank] + l.flags) + 2 * a.world,
                   a.world, a.epoch, a.status, a.timeout_ns);
}

// --------------------------------------------------------------------------- host

namespace {

// limit of the waits on other ranks, for every exchange enqueued after it is set
std::atomic<uint64_t> g_peer_wait_timeout_ns{LMOE_WAIT_TIMEOUT_NS};

int check_ep(const EpArgs& a) {
  if (a.world < 1 || a.world > kEpMaxWorld || a.rank < 0 || a.rank >= a.world) return kBadShape;
  if (a.E <= 0 || a.E > kEpMaxExperts || a.E % a.world != 0 || a.n_local * a.world != a.E)
    return kBadShape;
  if (a.row_bytes <= 0 || a.row_bytes % 16 != 0 || a.recv_cap < 0 || a.back_cap < 0)
    return kBadShape;
  if (a.recv_cap >= (1ll << 31) || a.back_cap >= (1ll << 31)) return kBadShape;
  if (a.peers == nullptr) return kBadShape;
  return kOk;
}

int grid_for(int64_t rows) {
  const int64_t want = (rows * 32 + 255) / 256;
  const int sms = num_sms(current_device());
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * 8)));
}

EpArgs make_ep(void* const* peers, int64_t rank, int64_t world, int64_t E, int64_t recv_cap,
               int64_t back_cap, int64_t row_bytes, int32_t* status) {
  EpArgs a;
  a.peers = reinterpret_cast<uint8_t* const*>(peers);
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.E = static_cast<int>(E);
  a.n_local = world > 0 ? static_cast<int>(E / world) : 0;
  a.recv_cap = recv_cap;
  a.back_cap = back_cap;
  a.row_bytes = row_bytes;
  a.epoch = 0;
  a.status = status;
  a.timeout_ns = g_peer_wait_timeout_ns.load(std::memory_order_relaxed);
  return a;
}

}  // namespace
}  // namespace lmoe

// --------------------------------------------------------------------------- C ABI
extern "C" {

int lmoe_set_peer_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) ns = LMOE_WAIT_TIMEOUT_NS;
  if (ns < 1000ull || ns > 60000000000ull) return LMOE_BAD_SHAPE;
  lmoe::g_peer_wait_timeout_ns.store(ns, std::memory_order_relaxed);
  return LMOE_OK;
}

uint64_t lmoe_peer_wait_timeout_ns(void) {
  return lmoe::g_peer_wait_timeout_ns.load(std::memory_order_relaxed);
}

int64_t lmoe_ep_buffer_bytes(int64_t world, int64_t num_experts, int64_t recv_capacity_rows,
                             int64_t back_capacity_rows, int64_t row_bytes) {
  if (world <= 0 || num_experts <= 0 || recv_capacity_rows < 0 || back_capacity_rows < 0 ||
      row_bytes <= 0)
    return -1;
  return lmoe::ep_layout(static_cast<int>(world), static_cast<int>(num_experts),
                         recv_capacity_rows, back_capacity_rows, row_bytes)
      .total;
}

int lmoe_ep_buffer_alloc(int64_t bytes, void** buffer, void* ipc_handle) {
  if (bytes <= 0 || buffer == nullptr || ipc_handle == nullptr) return LMOE_BAD_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) return LMOE_LAUNCH_FAILED;
  // flags and counters start at zero (epoch 0 = nothing signalled yet)
  if (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return LMOE_LAUNCH_FAILED;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return LMOE_LAUNCH_FAILED;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == LMOE_EP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return LMOE_OK;
}

int lmoe_ep_buffer_open(const void* ipc_handle, void** peer_buffer) {
  if (ipc_handle == nullptr || peer_buffer == nullptr) return LMOE_BAD_SHAPE;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return LMOE_LAUNCH_FAILED;
  *peer_buffer = p;
  return LMOE_OK;
}

int lmoe_ep_buffer_close(void* peer_buffer) {
  return cudaIpcCloseMemHandle(peer_buffer) == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_ep_buffer_free(void* buffer) {
  return cudaFree(buffer) == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int64_t lmoe_ep_region_offset(int64_t world, int64_t num_experts, int64_t recv_capacity_rows,
                              int64_t back_capacity_rows, int64_t row_bytes, int region) {
  const auto l = lmoe::ep_layout(static_cast<int>(world), static_cast<int>(num_experts),
                                 recv_capacity_rows, back_capacity_rows, row_bytes);
  switch (region) {
    case 0: return l.recv;
    case 1: return l.back;
    case 2: return l.counts;
    default: return -1;
  }
}

int lmoe_ep_exchange_counts(void* const* peers_dev, int64_t rank, int64_t world,
                            int64_t num_experts, int64_t recv_capacity_rows,
                            int64_t back_capacity_rows, int64_t row_bytes,
                            const int32_t* group_sizes, int32_t* local_group_sizes,
                            int32_t* dev_status, void* stream) {
  const auto a = lmoe::make_ep(peers_dev, rank, world, num_experts, recv_capacity_rows,
                               back_capacity_rows, row_bytes, dev_status);
  int rc = lmoe::check_ep(a);
  if (rc != lmoe::kOk) return rc;
  lmoe::ep_counts_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(a, group_sizes,
                                                                          local_group_sizes);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_ep_dispatch_put(void* const* peers_dev, int64_t rank, int64_t world, int64_t num_experts,
                         int64_t recv_capacity_rows, int64_t back_capacity_rows, int64_t row_bytes,
                         const void* x, int64_t x_rows, const int32_t* token_idx,
                         int64_t num_routed_rows, int32_t* dev_status, void* stream) {
  const auto a = lmoe::make_ep(peers_dev, rank, world, num_experts, recv_capacity_rows,
                               back_capacity_rows, row_bytes, dev_status);
  int rc = lmoe::check_ep(a);
  if (rc != lmoe::kOk) return rc;
  if (reinterpret_cast<uintptr_t>(x) & 15) return LMOE_UNSUPPORTED;
  auto s = static_cast<cudaStream_t>(stream);
  lmoe::ep_dispatch_put_kernel<<<lmoe::grid_for(num_routed_rows), 256, 0, s>>>(
      a, static_cast<const uint8_t*>(x), x_rows, token_idx, num_routed_rows);
  if (cudaGetLastError() != cudaSuccess) return LMOE_LAUNCH_FAILED;
  lmoe::ep_wait_kernel<<<1, 32, 0, s>>>(a, 1);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_ep_return_put(void* const* peers_dev, int64_t rank, int64_t world, int64_t num_experts,
                       int64_t recv_capacity_rows, int64_t back_capacity_rows, int64_t row_bytes,
                       const void* y, int64_t num_rows, int32_t* dev_status,
                       void* stream) {
  const auto a = lmoe::make_ep(peers_dev, rank, world, num_experts, recv_capacity_rows,
                               back_capacity_rows, row_bytes, dev_status);
  int rc = lmoe::check_ep(a);
  if (rc != lmoe::kOk) return rc;
  if (reinterpret_cast<uintptr_t>(y) & 15) return LMOE_UNSUPPORTED;
  auto s = static_cast<cudaStream_t>(stream);
  lmoe::ep_return_put_kernel<<<lmoe::grid_for(num_rows), 256, 0, s>>>(
      a, static_cast<const uint8_t*>(y), num_rows);
  if (cudaGetLastError() != cudaSuccess) return LMOE_LAUNCH_FAILED;
  lmoe::ep_wait_kernel<<<1, 32, 0, s>>>(a, 2);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_ep_return_destinations(void* const* peers_dev, int64_t rank, int64_t world,
                                int64_t num_experts, int64_t recv_capacity_rows,
                                int64_t back_capacity_rows, int64_t row_bytes, uint64_t* row_dest,
                                int64_t num_rows, int32_t* dev_status, void* stream) {
  const auto a = lmoe::make_ep(peers_dev, rank, world, num_experts, recv_capacity_rows,
                               back_capacity_rows, row_bytes, dev_status);
  int rc = lmoe::check_ep(a);
  if (rc != lmoe::kOk) return rc;
  if (row_dest == nullptr || num_rows < 0) return LMOE_BAD_SHAPE;
  const int64_t want = (num_rows + 255) / 256;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 1024)));
  lmoe::ep_row_dest_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a, row_dest,
                                                                                  num_rows);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

int lmoe_ep_return_signal(void* const* peers_dev, int64_t rank, int64_t world,
                          int64_t num_experts, int64_t recv_capacity_rows,
                          int64_t back_capacity_rows, int64_t row_bytes, int32_t* dev_status,
                          void* stream) {
  const auto a = lmoe::make_ep(peers_dev, rank, world, num_experts, recv_capacity_rows,
                               back_capacity_rows, row_bytes, dev_status);
  int rc = lmoe::check_ep(a);
  if (rc != lmoe::kOk) return rc;
  lmoe::ep_return_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? LMOE_OK : LMOE_LAUNCH_FAILED;
}

}  // extern "C"
