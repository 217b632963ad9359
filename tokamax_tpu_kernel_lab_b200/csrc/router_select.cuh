// Selection arithmetic shared by the router kernels (routing.cu: top-k from
// stored logits; router_fused.cu: top-k in the logits GEMM's epilogue).  Both
// must produce the same bits, so the score and the selection order live here.
//
// The gate of 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:347-356:
//   score = sigmoid(logit)           (f32)
//   key   = score + bias[e]          (selection only)
//   order = key descending, the lower expert id first on equal keys
#pragma once

#include <cfloat>
#include <climits>
#include <cstdint>

namespace lmoe {

// sigmoid(x) = 1 / (1 + exp(-x)): expf, a round-to-nearest add (the
// intrinsic keeps the compiler from fusing it into the exponential's last
// multiply) and the hardware reciprocal (rcp.approx, within 1 ulp; results
// below 2^-126 flush to zero).  Every router kernel calls this one function,
// so they all get the same bits; against the correctly rounded sigmoid the
// score is within a few ulp (~4e-7 relative).  The IEEE reciprocal costs
// several times more in the selection loop, where the sigmoid runs once per
// (token, expert).
__device__ __forceinline__ float router_sigmoid(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, expf(-x))));
  return r;
}

// true when (av, ae) comes before (bv, be) in the selection order
__device__ __forceinline__ bool sel_before(float av, int ae, float bv, int be) {
  return av > bv || (av == bv && ae < be);
}

// Insert (key, e, s) into a list kept sorted in the selection order, dropping
// its last entry; the caller has checked that the new entry beats that last
// entry.  Fully unrolled, so the list stays in registers.
template <int L>
__device__ __forceinline__ void sel_insert(float (&kv)[L], int (&ke)[L], float (&ks)[L], float key,
                                           int e, float s) {
  bool stay[L];  // entry j stays ahead of the new one
#pragma unroll
  for (int j = 0; j < L; ++j) stay[j] = sel_before(kv[j], ke[j], key, e);
#pragma unroll
  for (int j = L - 1; j >= 0; --j) {
    if (!stay[j]) {
      const int p = j > 0 ? j - 1 : 0;
      const bool here = j == 0 || stay[p];  // the new entry lands in slot j
      kv[j] = here ? key : kv[p];
      ke[j] = here ? e : ke[p];
      ks[j] = here ? s : ks[p];
    }
  }
}

// The same insertion for a caller that offers experts in increasing id order
// and starts its list with -inf keys: an entry already held comes first
// exactly when its key is >= the new key, so one compare per slot decides.
// (Finite keys only: a -inf or NaN key is never offered.)
template <int L>
__device__ __forceinline__ void sel_insert_ascending(float (&kv)[L], int (&ke)[L], float (&ks)[L],
                                                     float key, int e, float s) {
  bool stay[L];
#pragma unroll
  for (int j = 0; j < L; ++j) stay[j] = kv[j] >= key;
#pragma unroll
  for (int j = L - 1; j >= 0; --j) {
    const int p = j > 0 ? j - 1 : 0;
    const bool here = j == 0 || stay[p];
    kv[j] = stay[j] ? kv[j] : (here ? key : kv[p]);
    ke[j] = stay[j] ? ke[j] : (here ? e : ke[p]);
    ks[j] = stay[j] ? ks[j] : (here ? s : ks[p]);
  }
}

// Sort L values descending in place (bitonic network; L a power of two).
template <int L>
__device__ __forceinline__ void sort_desc(float (&v)[L]) {
#pragma unroll
  for (int size = 2; size <= L; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < L; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          // descending runs where bit `size` of i is clear, ascending where set,
          // so that each merge level sees a bitonic sequence
          const bool desc = (i & size) == 0;
          const float a = v[i], b = v[j];
          v[i] = desc ? fmaxf(a, b) : fminf(a, b);
          v[j] = desc ? fminf(a, b) : fmaxf(a, b);
        }
      }
    }
  }
}

// The L-th largest of the 2L values a[] u b[] (each sorted descending): the
// element-wise max of a and reversed b is the top L of the union.
template <int L>
__device__ __forceinline__ float lth_largest_of_two(const float (&a)[L], const float (&b)[L]) {
  float m = fmaxf(a[0], b[L - 1]);
#pragma unroll
  for (int i = 1; i < L; ++i) m = fminf(m, fmaxf(a[i], b[L - 1 - i]));
  return m;
}

}  // namespace lmoe
