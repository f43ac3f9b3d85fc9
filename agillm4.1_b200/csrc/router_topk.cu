// K1: router logits + top-k + gates + per-block expert histogram.
//
// Replaces agillm41.py:4398-4419 (router Linear, `.float()`, `topk` on the
// fp32 logits and `softmax` over the k chosen values cast to the activation
// dtype; top-1: `softmax` over all experts and `argmax`, agillm41.py:4401-4416).
//
// Layout: one CTA per dispatch block of 256 tokens (8 warps x 32 tokens).
// The router weight [E, d] is staged once per CTA in shared memory as fp32.
// A warp computes 4 tokens at a time: lane l owns the 16-byte chunks
// l, l+32, ... of each row (vectorised loads, fully coalesced), accumulates
// 4 x 16 partial dot products, and a transpose-reduce over the 32 lanes (16
// shuffles per token) leaves each expert's sum in two lanes. The logits are
// rounded like the reference's router output (bf16/fp16 GEMM result, then
// `.float()`), staged in shared memory, and then one thread per token does
// the selection and the softmax with the same reduction order as torch's
// warp softmax, so gates match bit for bit when the logits do.
#include "common.cuh"
#include "kernels.h"

namespace agm {

constexpr int kDispatchBlock = AGM_DISPATCH_BLOCK;  // tokens per CTA
constexpr int kRouterWarps = kDispatchBlock / 32;
constexpr int kMaxExperts = 16;
constexpr int kTokGroup = 4;

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

// Top-k selection reproducing torch.topk(sorted=True) on a CUDA device:
// the selected set is every value greater than the k-th largest plus, among
// the values equal to it, the lowest expert indices; the result is ordered by
// descending value and, among exactly-equal values, by DESCENDING expert
// index (measured on B200 with torch 2.11 for k = 2 and 3: 100% of ~120k
// tied rows). `low_first` orders exactly-equal values by ascending index
// instead.
__device__ __forceinline__ void select_topk(const float* logit, int E, int k, bool low_first, int* sel,
                                            float* val) {
  uint32_t taken = 0;
  for (int r = 0; r < k; ++r) {
    int best = -1;
    float bv = 0.f;
    for (int e = 0; e < E; ++e) {
      if (taken & (1u << e)) continue;
      const float v = logit[e];
      // NaN compares greater than everything in torch's topk ordering.
      const bool better = (best < 0) || (v > bv) || (isnan(v) && !isnan(bv));
      if (better) { best = e; bv = v; }
    }
    taken |= 1u << best;
    sel[r] = best;
    val[r] = bv;
  }
  if (!low_first) {
    // Reverse every run of exactly-equal values (ascending -> descending index).
    int r = 0;
    while (r < k) {
      int r2 = r + 1;
      while (r2 < k && val[r2] == val[r]) ++r2;
      for (int a = r, b = r2 - 1; a < b; ++a, --b) {
        const int t = sel[a]; sel[a] = sel[b]; sel[b] = t;
      }
      r = r2;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kDispatchBlock) router_topk_kernel(
    const T* __restrict__ x, const T* __restrict__ w, int64_t n_tokens, int d, int E, int k, int tie_low_first,
    const float* __restrict__ logits_in, float* __restrict__ logits_out, int32_t* __restrict__ idx_out,
    T* __restrict__ gates_out, int32_t* __restrict__ block_hist, int* err) {
  extern __shared__ __align__(16) float smem_f[];
  constexpr int CH = 16 / sizeof(T);  // elements per 16-byte chunk
  const int nchunk = d / CH;
  const bool compute = (logits_in == nullptr);
  // Dynamic smem: [E][d] fp32 router weight (only when computing logits),
  // then [8 warps][32 tokens][16] fp32 logits.
  float* w_s = smem_f;
  float* logit_s = smem_f + (compute ? E * d : 0);
  __shared__ int hist_s[kMaxExperts];

  const int warp = warp_id(), lane = lane_id();
  const int64_t blk_tok0 = static_cast<int64_t>(blockIdx.x) * kDispatchBlock;
  if (threadIdx.x < kMaxExperts) hist_s[threadIdx.x] = 0;

  if (compute) {
    // Stage W (vectorised, 16 B per thread per step), converting to fp32.
    const int total_chunks = E * nchunk;
    for (int c = threadIdx.x; c < total_chunks; c += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(w)[c];
      float f[8];
      if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
      } else {
        unpack8<T>(u, f);
      }
#pragma unroll
      for (int j = 0; j < CH; ++j) w_s[c * CH + j] = f[j];
    }
  }
  __syncthreads();

  float* my_logits = logit_s + warp * 32 * kMaxExperts;
  const int64_t warp_tok0 = blk_tok0 + warp * 32;

  if (compute) {
    for (int g = 0; g < 32; g += kTokGroup) {
      float acc[kTokGroup][kMaxExperts];
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t)
#pragma unroll
        for (int e = 0; e < kMaxExperts; ++e) acc[t][e] = 0.f;

      for (int c = lane; c < nchunk; c += 32) {
        float xf[kTokGroup][8];
#pragma unroll
        for (int t = 0; t < kTokGroup; ++t) {
          const int64_t tok = warp_tok0 + g + t;
          uint4 u = make_uint4(0, 0, 0, 0);
          if (tok < n_tokens) u = __ldg(reinterpret_cast<const uint4*>(x + tok * d) + c);
          if constexpr (sizeof(T) == 4) {
            xf[t][0] = __uint_as_float(u.x); xf[t][1] = __uint_as_float(u.y);
            xf[t][2] = __uint_as_float(u.z); xf[t][3] = __uint_as_float(u.w);
          } else {
            unpack8<T>(u, xf[t]);
          }
        }
#pragma unroll
        for (int e = 0; e < kMaxExperts; ++e) {
          if (e < E) {
            const float4* wp = reinterpret_cast<const float4*>(w_s + e * d + c * CH);
            float wf[8];
#pragma unroll
            for (int q = 0; q < CH / 4; ++q) {
              const float4 v = wp[q];
              wf[4 * q] = v.x; wf[4 * q + 1] = v.y; wf[4 * q + 2] = v.z; wf[4 * q + 3] = v.w;
            }
#pragma unroll
            for (int t = 0; t < kTokGroup; ++t)
#pragma unroll
              for (int j = 0; j < CH; ++j) acc[t][e] = fmaf(xf[t][j], wf[j], acc[t][e]);
          }
        }
      }
      // Transpose-reduce: after the xor-16/8/4/2 steps lane l holds a partial
      // sum of expert e(l) = 8*b4 + 4*b3 + 2*b2 + b1 (b = bits of l); the
      // xor-1 step completes it.
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t) {
        float v8[8], v4[4], v2[2];
        const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float send = u16 ? acc[t][i] : acc[t][i + 8];
          const float keep = u16 ? acc[t][i + 8] : acc[t][i];
          v8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float send = u8 ? v8[i] : v8[i + 4];
          const float keep = u8 ? v8[i + 4] : v8[i];
          v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float send = u4 ? v4[i] : v4[i + 2];
          const float keep = u4 ? v4[i + 2] : v4[i];
          v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        float v1;
        {
          const float send = u2 ? v2[0] : v2[1];
          const float keep = u2 ? v2[1] : v2[0];
          v1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        const float s = v1 + __shfl_xor_sync(0xffffffffu, v1, 1);
        const int e = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
        if ((lane & 1) == 0) my_logits[(g + t) * kMaxExperts + e] = round_to<T>(s);
      }
    }
  } else {
    for (int i = lane; i < 32 * E; i += 32) {
      const int t = i / E, e = i - t * E;
      const int64_t tok = warp_tok0 + t;
      my_logits[t * kMaxExperts + e] = (tok < n_tokens) ? logits_in[tok * E + e] : 0.f;
    }
  }
  __syncwarp();

  // One thread per token: selection, gates, histogram.
  const int64_t tok = warp_tok0 + lane;
  if (tok < n_tokens) {
    float lg[kMaxExperts];
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) lg[e] = (e < E) ? my_logits[lane * kMaxExperts + e] : 0.f;
    if (logits_out) {
      for (int e = 0; e < E; ++e) logits_out[tok * E + e] = lg[e];
    }
    int sel[kMaxExperts];
    float gate[kMaxExperts];
    if (k == 1) {
      // probs = softmax(scores) (warp softmax over next_pow2(E) lanes, padding
      // contributes exp(-inf) = 0), chosen = argmax(probs), first index on ties.
      float m = lg[0];
      for (int e = 1; e < E; ++e) m = fmaxf(m, lg[e]);
      float ex[kMaxExperts];
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) ex[e] = (e < E) ? expf(lg[e] - m) : 0.f;
      const float s = butterfly_sum_rt(ex, next_pow2_le32(E));
      int best = 0;
      float bp = ex[0] / s;
      for (int e = 1; e < E; ++e) {
        const float p = ex[e] / s;
        if (p > bp || (isnan(p) && !isnan(bp))) { bp = p; best = e; }
      }
      sel[0] = best;
      gate[0] = 1.f;  // straight-through gate: gate / gate.detach() == 1
    } else {
      float val[kMaxExperts];
      select_topk(lg, E, k, tie_low_first != 0, sel, val);
      // softmax over the k values (sorted descending, so val[0] is the max).
      float m = val[0];
      for (int r = 1; r < k; ++r) m = fmaxf(m, val[r]);
      float ex[kMaxExperts];
#pragma unroll
      for (int r = 0; r < kMaxExperts; ++r) ex[r] = (r < k) ? expf(val[r] - m) : 0.f;
      const float s = butterfly_sum_rt(ex, next_pow2_le32(k));
      for (int r = 0; r < k; ++r) gate[r] = ex[r] / s;
    }
    for (int r = 0; r < k; ++r) {
      const int e = sel[r];
      if (e < 0 || e >= E) {
        raise_error(err, kErrBadExpert);
        continue;
      }
      idx_out[tok * k + r] = e;
      gates_out[tok * k + r] = Traits<T>::from_f(gate[r]);
      atomicAdd(&hist_s[e], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < E) block_hist[static_cast<int64_t>(blockIdx.x) * E + threadIdx.x] = hist_s[threadIdx.x];
}

template <typename T>
static cudaError_t launch_router(const void* x, const void* w, int64_t n_tokens, int d, int E, int k, int tie_low_first,
                                 const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                                 int32_t* block_hist, int* err, cudaStream_t stream) {
  const int64_t nblk = (n_tokens + kDispatchBlock - 1) / kDispatchBlock;
  const size_t smem = (logits_in ? 0 : static_cast<size_t>(E) * d * sizeof(float)) +
                      static_cast<size_t>(kRouterWarps) * 32 * kMaxExperts * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(router_topk_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  router_topk_kernel<T><<<static_cast<unsigned>(nblk), kDispatchBlock, smem, stream>>>(
      static_cast<const T*>(x), static_cast<const T*>(w), n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx,
      static_cast<T*>(gates), block_hist, err);
  return cudaGetLastError();
}

cudaError_t router_topk(int dtype, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                        int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                        int32_t* block_hist, int* err, cudaStream_t stream) {
  if (n_tokens == 0) return cudaSuccess;
  switch (dtype) {
    case AGM_F32:
      return launch_router<float>(x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates, block_hist,
                                  err, stream);
    case AGM_BF16:
      return launch_router<__nv_bfloat16>(x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates,
                                          block_hist, err, stream);
    case AGM_F16:
      return launch_router<__half>(x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates, block_hist,
                                   err, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

size_t router_smem_bytes(int d, int E) {
  return static_cast<size_t>(E) * d * sizeof(float) + static_cast<size_t>(kRouterWarps) * 32 * kMaxExperts * 4;
}

}  // namespace agm
