// Dispatch with built-in scratch: the same counting-sort kernels as
// lmoe_dispatch, but their scratch lives in a fixed array inside this library
// instead of a caller-provided workspace, so the call allocates nothing and
// takes no workspace argument.
//
// Who needs this: callers that cannot allocate device memory at the point
// where they dispatch -- for example code running under a framework that owns
// the whole device memory pool (a preallocating allocator leaves cudaMalloc
// nothing to give), or a latency-critical loop that must not call
// cudaMalloc/cudaFree because those calls can block on, or synchronise with,
// the device.
//
// Limits and sharing rules:
//   - capacity: max(num_tokens * top_k, m_out) <= kStaticMaxEntries (262144,
//     one full 16384-token top-16 batch) and num_local_experts + 1 <=
//     kStaticMaxBins (2049); larger requests return LMOE_SCRATCH_TOO_SMALL and
//     launch nothing.
//   - the array (about 2.1 MB) exists once per device and stays resident on
//     every GPU that loads this library until the process exits.
//   - every call on a device uses the same array and leaves its contents
//     behind.  Nothing in it has to start at zero: each call writes every
//     entry it later reads.  Two calls whose kernels overlap on the GPU (for
//     example on two streams without ordering between them) race on the array
//     and produce wrong results; keep such calls ordered.
//   - the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture begins.
#include <mutex>

#include "../../include/lmoe.h"
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace {

constexpr int64_t kStaticMaxEntries = 262144;
constexpr int64_t kStaticMaxBins = 2049;
constexpr int64_t kChunk = 2048;  // entries per block of the rank kernel
constexpr int64_t al256(int64_t b) { return (b + 255) / 256 * 256; }
constexpr int64_t kStaticScratchBytes =
    al256(kStaticMaxBins * ((kStaticMaxEntries + kChunk - 1) / kChunk) * 4) +
    al256(kStaticMaxBins * 4) + al256(kStaticMaxEntries * 4);

// The scratch itself.  In host code this name is only a stand-in for the
// device symbol, never a usable address: the kernels receive the address
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_dispatch_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_dispatch_scratch on the current device (looked up once).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return LMOE_LAUNCH_FAILED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dispatch_scratch) != cudaSuccess || p == nullptr)
      return LMOE_LAUNCH_FAILED;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LMOE_OK;
}

}  // namespace

extern "C" int lmoe_dispatch_static_scratch(const int32_t* topk_idx, const float* topk_w,
                                            int64_t num_tokens, int64_t top_k,
                                            int64_t expert_start, int64_t num_local_experts,
                                            int64_t m_out, int pad_bucket, int32_t* order,
                                            int32_t* token_idx, float* weight, int32_t* slot_pos,
                                            int32_t* group_sizes, int32_t* per_expert_counts,
                                            uint8_t* valid, void* stream) {
  if (num_tokens < 0 || top_k <= 0 || num_local_experts <= 0 || m_out < 0) return LMOE_BAD_SHAPE;
  if (token_idx == nullptr || group_sizes == nullptr) return LMOE_BAD_SHAPE;
  const int64_t entries = std::max(num_tokens * top_k, m_out);
  if (entries > kStaticMaxEntries || num_local_experts + 1 > kStaticMaxBins)
    return LMOE_SCRATCH_TOO_SMALL;
  const size_t need = lmoe::dispatch_workspace_bytes(entries, num_local_experts);
  if (need > static_cast<size_t>(kStaticScratchBytes)) return LMOE_SCRATCH_TOO_SMALL;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != LMOE_OK) return rc;
  lmoe::DispatchOut o{order, token_idx, weight, slot_pos, group_sizes, per_expert_counts, valid};
  return lmoe::dispatch_sort(topk_idx, topk_w, num_tokens * top_k, top_k, expert_start,
                             num_local_experts, m_out, pad_bucket, o, scratch,
                             static_cast<size_t>(kStaticScratchBytes),
                             static_cast<cudaStream_t>(stream));
}
