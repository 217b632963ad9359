// float32 grouped GEMM on the CUDA cores (FFMA), for the float32 compute
// dtype of the reduced-scale configuration and the float32 golden bundles.
// tcgen05 has no IEEE-f32 kind (kind::tf32 rounds the operands), so the f32
// path runs here; every output element accumulates its K products in order.
// Same ragged semantics as the tensor-core kernel (rows past sum(group_sizes)
// are zero), same device-side schedule (no host synchronisation).
#include "lmoe_internal.h"
#include "ptx.cuh"

namespace lmoe {

constexpr int kSBM = 64, kSBN = 64, kSBK = 16;
constexpr int kSimtMaxGroups = 4096;

__global__ void __launch_bounds__(256) simt_grouped_gemm_f32_kernel(
    const float* __restrict__ lhs, const float* __restrict__ rhs, const int32_t* __restrict__ gs,
    float* __restrict__ out, const float* __restrict__ addend, int M, int K, int N, int G,
    int rhs_gnk, int n_tiles, int zero_tail, int32_t* status) {
  __shared__ int32_t row_off[kSimtMaxGroups + 1];
  __shared__ int32_t tile_start[kSimtMaxGroups + 1];
  __shared__ float As[kSBK][kSBM + 4];
  __shared__ float Bs[kSBK][kSBN + 4];
  __shared__ int s_total;
  if (threadIdx.x == 0) {
    long long r = 0, t = 0;
    int bad = 0;
    for (int g = 0; g < G; ++g) {
      const int s = gs ? gs[g] : M;
      if (s < 0) bad = 1;
      row_off[g] = static_cast<int32_t>(r);
      tile_start[g] = static_cast<int32_t>(t);
      r += max(s, 0);
      t += static_cast<long long>((max(s, 0) + kSBM - 1) / kSBM) * n_tiles;
    }
    row_off[G] = static_cast<int32_t>(r);
    tile_start[G] = static_cast<int32_t>(t);
    if (bad || r > M) {
      record_status(status, kDeviceBounds);
      s_total = -1;
    } else {
      s_total = static_cast<int>(t);
    }
  }
  __syncthreads();
  const int total = s_total;
  if (total < 0) return;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int local = t - tile_start[g];
    const int mt = local / n_tiles, nt = local - mt * n_tiles;
    const int row0 = row_off[g] + mt * kSBM, row_end = row_off[g + 1];
    const int col0 = nt * kSBN;
    const float* B = rhs + static_cast<int64_t>(g) * K * N;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kSBK) {
      for (int i = threadIdx.x; i < kSBM * kSBK; i += 256) {
        const int r = i / kSBK, kk = i % kSBK;
        const int gr = row0 + r, gk = k0 + kk;
        As[kk][r] = (gr < row_end && gk < K) ? lhs[static_cast<int64_t>(gr) * K + gk] : 0.f;
      }
      for (int i = threadIdx.x; i < kSBN * kSBK; i += 256) {
        int kk, c;
        if (rhs_gnk) { c = i / kSBK; kk = i % kSBK; } else { kk = i / kSBN; c = i % kSBN; }
        const int gk = k0 + kk, gc = col0 + c;
        float v = 0.f;
        if (gk < K && gc < N)
          v = rhs_gnk ? B[static_cast<int64_t>(gc) * K + gk] : B[static_cast<int64_t>(gk) * N + gc];
        Bs[kk][c] = v;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kSBK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = row0 + ty * 4 + i;
      if (r >= row_end) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = col0 + tx * 4 + j;
        if (c < N) {
          const int64_t o = static_cast<int64_t>(r) * N + c;
          out[o] = addend ? acc[i][j] + addend[o] : acc[i][j];
        }
      }
    }
  }
  if (zero_tail) {
    const int64_t first = row_off[G];
    const int64_t n = (static_cast<int64_t>(M) - first) * N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * 256)
      out[first * N + i] = 0.f;
  }
}

int simt_grouped_gemm_f32(const float* lhs, const float* rhs, const int32_t* group_sizes,
                          float* out, const float* addend, int64_t M, int64_t K, int64_t N,
                          int64_t G, int rhs_layout, int zero_tail, int32_t* status,
                          cudaStream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || G <= 0 || G > kSimtMaxGroups) return kBadShape;
  if (M >= (1ll << 31) || K >= (1ll << 31) || N >= (1ll << 31)) return kBadShape;
  if (M == 0) return kOk;
  const int n_tiles = static_cast<int>((N + kSBN - 1) / kSBN);
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t max_tiles = ((M + kSBM - 1) / kSBM + G) * n_tiles;
  const int grid = static_cast<int>(std::min<int64_t>(max_tiles, static_cast<int64_t>(num_sms(dev)) * 4));
  simt_grouped_gemm_f32_kernel<<<std::max(grid, 1), 256, 0, stream>>>(
      lhs, rhs, group_sizes, out, addend, (int)M, (int)K, (int)N, group_sizes ? (int)G : 1,
      rhs_layout == 1 ? 1 : 0, n_tiles, zero_tail, status);
  return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace lmoe
