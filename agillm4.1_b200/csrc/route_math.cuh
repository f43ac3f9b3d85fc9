// Gate arithmetic shared by the router (forward) and the routing backward.
//
// The backward recomputes the fp32 gates and the top-1 probabilities from the
// saved fp32 logits with these same functions, so its values are the exact
// values the forward used (agillm41.py:4402, 4419: softmax over all experts
// for top-1, softmax over the k chosen logits otherwise).
#pragma once

#include "common.cuh"

namespace agm {

// Sum of e[0..W) in the order of a butterfly (xor) reduction over W lanes,
// which is how torch's warp softmax reduces a row of W <= 32 elements.
template <int W>
__device__ __forceinline__ float butterfly_sum(const float* e) {
  float v[W];
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = e[i];
#pragma unroll
  for (int off = W / 2; off > 0; off /= 2) {
#pragma unroll
    for (int i = 0; i < off; ++i) v[i] = v[i] + v[i + off];
  }
  return v[0];
}

__device__ __forceinline__ int next_pow2_le32(int n) {
  int w = 1;
  while (w < n) w <<= 1;
  return w;
}

// Sum with the butterfly order for a runtime width w (power of two, <= 16).
__device__ __forceinline__ float butterfly_sum_rt(const float* e, int w) {
  switch (w) {
    case 1: return e[0];
    case 2: return butterfly_sum<2>(e);
    case 4: return butterfly_sum<4>(e);
    case 8: return butterfly_sum<8>(e);
    default: return butterfly_sum<16>(e);
  }
}

constexpr int pow2_ceil(int n) { return n <= 1 ? 1 : 2 * pow2_ceil((n + 1) / 2); }

// softmax over the k chosen logits val[0..k) (arrays of S >= k entries):
// gate[r] = exp(val[r] - max) / sum, the sum in butterfly order over
// next_pow2(k) lanes. KC > 0 is k known at compile time (S = pow2_ceil(KC)).
template <int KC, int S>
__device__ __forceinline__ void topk_gates(const float (&val)[S], int k, float (&gate)[S]) {
  float m = val[0];
#pragma unroll
  for (int r = 1; r < S; ++r)
    if (r < k) m = fmaxf(m, val[r]);
  float ex[S];
#pragma unroll
  for (int r = 0; r < S; ++r) ex[r] = (r < k) ? expf(val[r] - m) : 0.f;
  float s;
  if constexpr (KC > 0) {
    s = butterfly_sum<S>(ex);
  } else {
    s = butterfly_sum_rt(ex, next_pow2_le32(k));
  }
#pragma unroll
  for (int r = 0; r < S; ++r) gate[r] = (r < k) ? ex[r] / s : 0.f;
}

// Top-1 probabilities: softmax over all E logits (padding lanes of the
// next_pow2(E)-wide warp softmax contribute exp(-inf) = 0). ex[] receives the
// unnormalised terms, the return value is their sum; p_e = ex[e] / sum.
template <int NE>
__device__ __forceinline__ float softmax_terms(const float (&lg)[NE], int E, float (&ex)[NE]) {
  float m = lg[0];
#pragma unroll
  for (int e = 1; e < NE; ++e)
    if (e < E) m = fmaxf(m, lg[e]);
#pragma unroll
  for (int e = 0; e < NE; ++e) ex[e] = (e < E) ? expf(lg[e] - m) : 0.f;
  return butterfly_sum_rt(ex, next_pow2_le32(E));
}

}  // namespace agm
