// Training path of the MoE block: a forward that keeps what the backward
// needs, and the backward, as replacements for PyTorch autograd through
// MoEFFN.forward (agillm41.py:4389-4431).
//
// Two precision modes, the two the reference trains in:
//
// * same dtype (x, weights, out all fp32, bf16 or fp16): every op rounds to
//   that dtype, as the reference does without autocast;
// * autocast (x, out and the master weights fp32; compute in bf16 or fp16,
//   torch.autocast as enabled by the reference's `amp()` helper,
//   agillm41.py:3054-3066): the router and expert Linear layers run on
//   16-bit casts of their inputs and weights, the router logits are `.float()`
//   of the 16-bit GEMM output, the gates stay fp32 (`softmax(vals).to(x.dtype)`
//   with x fp32) and the combine accumulates fp32 products of the 16-bit
//   expert outputs into an fp32 `zeros_like(flat)`. In the backward the
//   16-bit weight gradients are rounded to 16 bits and returned as fp32 (the
//   cast's backward), and input gradients are summed in fp32.
//
// Forward (agm_moe_forward_train): [cast x to 16 bits] -> router (keeps the
// fp32 logits) -> plan -> permute -> FC1 -> FC2 (y in its own buffer, so the
// permuted input survives for the weight gradient) -> combine_train.
//
// Backward (agm_moe_backward), given dout = dL/dout:
//   combine_bwd:  dy[row(t,r)] = dout[t] * g[t,r]; dgate[t,r] = <dout[t], y[row]>;
//                 softmax-over-k (or top-1 straight-through) backward to the
//                 router logits dl [N, 16] (zero-fills dy's padding rows)
//   wgrad FC2:    dW2[e] = dy_e^T h_e         db2[e] = sum of dy_e's rows
//   dgrad FC2:    dh = (dy @ W2[e]) * (h > 0)
//   wgrad FC1:    dW1[e] = dh_e^T x_perm_e    db1[e] = sum of dh_e's rows
//   dgrad FC1:    dx_perm = dh @ W1[e]
//   router wgrad: dWr = dl^T x                (x rows read from x_perm)
//   dx:           dx[t] = ((dx_perm[row(t,k-1)] + ... + dx_perm[row(t,0)]) + dl[t] @ Wr)
// The order of the dx sum is the order in which autograd accumulates the
// gradients of `flat`: the index_select nodes of the last rank run first and
// the router's Linear, created first, runs last.
#include <algorithm>
#include <cstdio>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "route_math.cuh"

namespace agm {
namespace {

constexpr int kMaxE = AGM_MAX_EXPERTS;  // logits gradient rows are 16 wide
constexpr int kZeroCtas = 8;            // CTAs zero-filling one expert's padding rows of dy
constexpr int kColsumCols = 256;        // columns per segment-column-sum CTA (8 per lane)

// 8 consecutive values of T (or fp32) at p -> fp32.
template <typename T>
__device__ __forceinline__ void load8f(const T* p, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(p)), f);
  }
}

// fp32 -> 8 consecutive values of T (or fp32) at p (round to nearest even).
template <typename T>
__device__ __forceinline__ void store8f(T* p, const float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// fp32 -> 16-bit cast (autocast's input and weight casts)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) cast_f32_kernel(const float* __restrict__ in, T* __restrict__ out, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    float f[8];
    load8f<float>(in + i * 8, f);
    store8f<T>(out + i * 8, f);
  }
  for (int64_t i = n8 * 8 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = Traits<T>::from_f(in[i]);
}

// Gates of token t recomputed from the saved fp32 logits with the router's
// own arithmetic: k >= 2 -> softmax over the chosen logits (fp32, exactly the
// forward's values); k == 1 -> the straight-through value 1.
template <int K_MAX>
__device__ __forceinline__ void token_gates(const float* __restrict__ logits, const int32_t* __restrict__ idx,
                                            int64_t t, int k, int E, int (&sel)[K_MAX], float (&g)[K_MAX]) {
  float val[K_MAX];
#pragma unroll
  for (int r = 0; r < K_MAX; ++r) {
    sel[r] = (r < k) ? idx[t * k + r] : 0;
    if (sel[r] < 0 || sel[r] >= E) sel[r] = 0;  // the router never writes such ids
    val[r] = (r < k) ? logits[t * E + sel[r]] : 0.f;
  }
  if (k == 1) {
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) g[r] = (r == 0) ? 1.f : 0.f;
  } else {
    topk_gates<0, K_MAX>(val, k, g);
  }
}

// ---------------------------------------------------------------------------
// Combine for training (the saved fp32 logits give the gates):
//   G == T (same dtype): out = ((0 + r(y0*r(g0))) + r(y1*r(g1))) ..., r() = round to T;
//   G == float (autocast): out = (0 + y0*g0) + y1*g1 in fp32.
//   k == 1: out = y (the straight-through gate is exactly 1).
// Shared experts (agillm41.py:4381-4387, 4429-4430): s = s_0 + s_1 + ... in
// T, then out = out + s (rounded to G).
// ---------------------------------------------------------------------------
template <typename T, typename G, int K_MAX>
__global__ void __launch_bounds__(256) combine_train_kernel(const T* __restrict__ y, const int32_t* __restrict__ row_of,
                                                            const float* __restrict__ logits,
                                                            const int32_t* __restrict__ idx, int64_t n, int d, int k,
                                                            int E, const T* __restrict__ shared_y, int n_shared,
                                                            int64_t shared_stride, const G* __restrict__ residual,
                                                            G* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int lane = lane_id();
  const int nc8 = d / 8;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp_id(); t < n; t += warps) {
    int sel[K_MAX];
    float g[K_MAX];
    token_gates<K_MAX>(logits, idx, t, k, E, sel, g);
    int64_t row[K_MAX];
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) {
      row[r] = (r < k) ? row_of[t * k + r] : 0;
      if (sizeof(G) != 4) g[r] = round_to<T>(g[r]);  // weights.to(x.dtype)
    }
    for (int c = lane; c < nc8; c += 32) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) {
        if (r < k) {
          float v[8];
          load8f<T>(y + row[r] * d + c * 8, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (k == 1) {
              acc[i] = v[i];
            } else if (sizeof(G) == 4) {
              acc[i] = __fadd_rn(acc[i], __fmul_rn(v[i], g[r]));
            } else {
              acc[i] = round_to<T>(__fadd_rn(acc[i], round_to<T>(__fmul_rn(v[i], g[r]))));
            }
          }
        }
      }
      if (n_shared > 0) {
        float sh[8];
        load8f<T>(shared_y + t * d + c * 8, sh);
        for (int si = 1; si < n_shared; ++si) {
          float v[8];
          load8f<T>(shared_y + si * shared_stride + t * d + c * 8, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) sh[i] = round_to<T>(__fadd_rn(sh[i], v[i]));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          acc[i] = (sizeof(G) == 4) ? __fadd_rn(acc[i], sh[i]) : round_to<T>(__fadd_rn(acc[i], sh[i]));
      }
      if (residual) {  // Block: x + ff(ln2(x)), agillm41.py:4547
        float rv[8];
        load8f<G>(residual + t * d + c * 8, rv);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          acc[i] = (sizeof(G) == 4) ? __fadd_rn(rv[i], acc[i]) : round_to<T>(__fadd_rn(rv[i], acc[i]));
      }
      store8f<G>(out + t * d + c * 8, acc);
    }
  }
}

// ---------------------------------------------------------------------------
// Combine backward + routing backward.
// One warp per token. For each rank r (row p = row_of[t, r]):
//   dy[p]   = r_T(dout[t] * g'[r])          g' = r_T(g) (same dtype) or g (fp32)
//   dg[r]   = sum_c dout[t,c] * y[p,c]      (products rounded to T in same-dtype
//                                            mode, then the sum rounded to T)
// then the gradient of the router logits (agillm41.py:4401-4419):
//   k >= 2: dv = g * (dg - sum_j g_j dg_j)  (softmax over the k chosen), scattered
//           to the chosen experts;
//   k == 1: gate = r_T(p_c); dgate = dg / gate; dl_e = p_e * (dprob_e - p_c dgate)
//           with dprob = dgate at the chosen expert (straight-through gate);
// rounded to the logits' source dtype T (the `.float()` cast's backward).
// CTAs past the token CTAs zero-fill dy's padding rows.
// ---------------------------------------------------------------------------
template <typename T, typename G, int K_MAX>
__global__ void __launch_bounds__(256) combine_bwd_kernel(
    const G* __restrict__ dout, const T* __restrict__ y, const int32_t* __restrict__ row_of,
    const float* __restrict__ logits, const int32_t* __restrict__ idx, int64_t n, int d, int k, int E,
    int tok_ctas, const int32_t* __restrict__ seg_start, const int32_t* __restrict__ counts, int64_t max_rows,
    T* __restrict__ dy, T* __restrict__ dl, T* __restrict__ ds, int64_t npad, int32_t* __restrict__ dense_seg) {
  pdl_wait();
  pdl_trigger();
  const int lane = lane_id();
  const int nc8 = d / 8;
  if (static_cast<int>(blockIdx.x) >= tok_ctas) {
    const int z = blockIdx.x - tok_ctas;
    if (z == 0 && ds) {
      // shared experts: their rows past n are zero, and they form one segment
      if (threadIdx.x == 0) {
        dense_seg[0] = 0;
        dense_seg[1] = static_cast<int32_t>(npad);
      }
      const int nchunk = d * static_cast<int>(sizeof(T)) / 16;
      for (int64_t i = threadIdx.x; i < (npad - n) * nchunk; i += blockDim.x)
        reinterpret_cast<uint4*>(ds + n * d)[i] = make_uint4(0, 0, 0, 0);
    }
    const int e = z / kZeroCtas;
    const int64_t r0 = static_cast<int64_t>(seg_start[e]) + counts[e];
    const int64_t r1 = min(static_cast<int64_t>(seg_start[e + 1]), max_rows);
    const int nw = blockDim.x / 32;
    const int nchunk = d * static_cast<int>(sizeof(T)) / 16;
    for (int64_t r = r0 + (z % kZeroCtas) * nw + warp_id(); r < r1; r += kZeroCtas * nw) {
      uint4* o = reinterpret_cast<uint4*>(dy + r * d);
      for (int c = lane; c < nchunk; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int64_t warps = static_cast<int64_t>(tok_ctas) * (blockDim.x / 32);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp_id(); t < n; t += warps) {
    int sel[K_MAX];
    float g[K_MAX];
    token_gates<K_MAX>(logits, idx, t, k, E, sel, g);
    int64_t row[K_MAX];
    float gm[K_MAX], dg[K_MAX];
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) {
      row[r] = (r < k) ? row_of[t * k + r] : 0;
      gm[r] = (sizeof(G) == 4) ? g[r] : round_to<T>(g[r]);
      dg[r] = 0.f;
    }
    for (int c = lane; c < nc8; c += 32) {
      float go[8];
      load8f<G>(dout + t * d + c * 8, go);
      if (ds) store8f<T>(ds + t * d + c * 8, go);  // gradient of the shared sum: dout in T
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) {
        if (r < k) {
          float v[8], o[8];
          load8f<T>(y + row[r] * d + c * 8, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            o[i] = __fmul_rn(go[i], gm[r]);  // rounded to T by the store
            const float prod = __fmul_rn(go[i], v[i]);
            dg[r] += (sizeof(G) == 4) ? prod : round_to<T>(prod);
          }
          store8f<T>(dy + row[r] * d + c * 8, o);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) {
      dg[r] = warp_sum(dg[r]);
      if (sizeof(G) != 4) dg[r] = round_to<T>(dg[r]);
    }
    // Gradient of the logits: lane e owns expert e.
    float dle = 0.f;
    if (k == 1) {
      float lg[kMaxE], ex[kMaxE];
#pragma unroll
      for (int e = 0; e < kMaxE; ++e) lg[e] = (e < E) ? logits[t * E + e] : 0.f;
      const float s = softmax_terms(lg, E, ex);
      const int c = sel[0];
      float pc = 0.f, pe = 0.f;
#pragma unroll
      for (int e = 0; e < kMaxE; ++e) {
        const float p = ex[e] / s;
        if (e == c) pc = p;
        if (e == lane) pe = p;
      }
      const float gate_pre = (sizeof(G) == 4) ? pc : round_to<T>(pc);   // probs[..].to(x.dtype)
      const float gate = fmaxf(gate_pre, 1e-6f);                        // clamp_min(1e-6)
      float dgate = __fdiv_rn(dg[0], gate);                             // d(gate / gate.detach())
      if (sizeof(G) != 4) dgate = round_to<T>(dgate);
      if (!(gate_pre >= 1e-6f)) dgate = 0.f;                            // clamp_min backward
      const float s2 = __fmul_rn(pc, dgate);                            // sum_e p_e dprob_e
      const float dprob = (lane == c) ? dgate : 0.f;
      dle = __fmul_rn(pe, __fsub_rn(dprob, s2));
    } else {
      float prod[K_MAX];
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) prod[r] = (r < k) ? __fmul_rn(g[r], dg[r]) : 0.f;
      const float s = butterfly_sum_rt(prod, next_pow2_le32(k));
#pragma unroll
      for (int r = 0; r < K_MAX; ++r)
        if (r < k && sel[r] == lane) dle = __fmul_rn(g[r], __fsub_rn(dg[r], s));
    }
    if (lane < kMaxE) dl[t * kMaxE + lane] = Traits<T>::from_f(lane < E ? dle : 0.f);
  }
}

// ---------------------------------------------------------------------------
// Per-expert column sums (bias gradients), deterministic:
//   partial[s, g, c] = sum over rows of split s of segment g of m[row, c]
//   out[g, c] = r_T(sum_s partial[s, g, c])   (stored as OutT)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) seg_colsum_kernel(const T* __restrict__ m, int ncols,
                                                         const int32_t* __restrict__ seg_start, int groups, int splits,
                                                         float* __restrict__ partial) {
  __shared__ float red[8][kColsumCols];
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.y, s = blockIdx.z;
  const int lane = lane_id(), w = warp_id();
  const int c0 = blockIdx.x * kColsumCols + lane * 8;
  const int64_t s0 = seg_start[g], s1 = seg_start[g + 1];
  const int64_t per = (s1 - s0 + splits - 1) / splits;
  const int64_t lo = s0 + s * per, hi = min(s1, lo + per);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (c0 < ncols) {
    for (int64_t r = lo + w; r < hi; r += 8) {
      float v[8];
      if (c0 + 8 <= ncols) {
        load8f<T>(m + r * ncols + c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (c0 + i < ncols) ? Traits<T>::to_f(m[r * ncols + c0 + i]) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[w][lane * 8 + i] = acc[i];
  __syncthreads();
  const int c = threadIdx.x;
  const int col = blockIdx.x * kColsumCols + c;
  if (col < ncols) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) v += red[i][c];
    partial[(static_cast<int64_t>(s) * groups + g) * ncols + col] = v;
  }
}

// out[i] = r_T(sum_p partial[p * part_stride + i]) for i < count, p in order.
template <typename T, typename OutT>
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partial, int parts,
                                                              int64_t part_stride, int64_t count,
                                                              OutT* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v = 0.f;
    for (int p = 0; p < parts; ++p) v += partial[p * part_stride + i];
    const float r = round_to<T>(v);
    if constexpr (sizeof(OutT) == 4)
      out[i] = r;
    else
      out[i] = Traits<OutT>::from_f(r);
  }
}

// ---------------------------------------------------------------------------
// Router weight gradient partials: partial[chunk, e, c] = sum over the
// chunk's tokens of dl[t, e] * x[t, c], x[t] read from x_perm[row_of[t, 0]]
// (the permuted copy of token t's router input), or from x_perm[t] when
// row_of is null. A thread owns 4 columns for
// all 16 logit rows (64 fp32 accumulators); the chunk's logit gradients and
// row indices are staged in shared memory first, and the x values of 4 tokens
// are loaded together ahead of their multiply-adds.
// ---------------------------------------------------------------------------
constexpr int kRwMaxChunk = 256;  // tokens per router-wgrad CTA at most

template <typename T>
__global__ void __launch_bounds__(512) router_wgrad_kernel(const T* __restrict__ dl, const T* __restrict__ xperm,
                                                            const int32_t* __restrict__ row_of, int k, int64_t n,
                                                            int d, int tok_per_chunk, float* __restrict__ partial) {
  __shared__ float4 dl_s[kRwMaxChunk][kMaxE / 4];
  __shared__ int64_t row_s[kRwMaxChunk];
  pdl_wait();
  pdl_trigger();
  const int chunk = blockIdx.x;
  const int64_t t0 = static_cast<int64_t>(chunk) * tok_per_chunk;
  const int cnt = static_cast<int>(min(static_cast<int64_t>(tok_per_chunk), n - t0));
  float* dl_f = reinterpret_cast<float*>(&dl_s[0][0]);
  for (int i = threadIdx.x; i < cnt * kMaxE; i += blockDim.x) dl_f[i] = Traits<T>::to_f(dl[t0 * kMaxE + i]);
  for (int i = threadIdx.x; i < cnt; i += blockDim.x)
    row_s[i] = (row_of ? static_cast<int64_t>(row_of[(t0 + i) * k]) : t0 + i) * d;
  __syncthreads();
  const int c0 = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (c0 >= d) return;
  float acc[kMaxE][4];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[e][i] = 0.f;
  for (int j0 = 0; j0 < cnt; j0 += 4) {
    float x[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u < cnt) {
        const T* xr = xperm + row_s[j0 + u] + c0;
        if constexpr (sizeof(T) == 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(xr));
          x[u][0] = v.x; x[u][1] = v.y; x[u][2] = v.z; x[u][3] = v.w;
        } else {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(xr));
          float f[8];
          unpack8<T>(make_uint4(w.x, w.y, 0, 0), f);
          x[u][0] = f[0]; x[u][1] = f[1]; x[u][2] = f[2]; x[u][3] = f[3];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) x[u][i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j0 + u < cnt) {
#pragma unroll
        for (int e4 = 0; e4 < kMaxE / 4; ++e4) {
          const float4 g = dl_s[j0 + u][e4];  // one shared-memory read serves four logit rows
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[4 * e4 + 0][i] = fmaf(g.x, x[u][i], acc[4 * e4 + 0][i]);
            acc[4 * e4 + 1][i] = fmaf(g.y, x[u][i], acc[4 * e4 + 1][i]);
            acc[4 * e4 + 2][i] = fmaf(g.z, x[u][i], acc[4 * e4 + 2][i]);
            acc[4 * e4 + 3][i] = fmaf(g.w, x[u][i], acc[4 * e4 + 3][i]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < kMaxE; ++e)
    *reinterpret_cast<float4*>(partial + (static_cast<int64_t>(chunk) * kMaxE + e) * d + c0) =
        make_float4(acc[e][0], acc[e][1], acc[e][2], acc[e][3]);
}

// The same sum for many partials (the router weight gradient's per-chunk
// partials): a CTA owns 32 consecutive outputs; warp w adds the partials
// p = w, w + 8, w + 16, ... in order (coalesced 128-byte rows, four loads in
// flight), then warp 0 adds the 8 warp sums in warp order. The order depends
// on `parts` only: deterministic.
template <typename T, typename OutT>
__global__ void __launch_bounds__(256) reduce_partials_wide_kernel(const float* __restrict__ partial, int parts,
                                                                   int64_t part_stride, int64_t count,
                                                                   OutT* __restrict__ out) {
  __shared__ float red[8][32];
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  float v = 0.f;
  if (i < count) {
    int p = warp;
    for (; p + 24 < parts; p += 32) {
      const float a = partial[p * part_stride + i];
      const float b = partial[(p + 8) * part_stride + i];
      const float c = partial[(p + 16) * part_stride + i];
      const float d = partial[(p + 24) * part_stride + i];
      v = (((v + a) + b) + c) + d;
    }
    for (; p < parts; p += 8) v += partial[p * part_stride + i];
  }
  red[warp][lane] = v;
  __syncthreads();
  if (warp == 0 && i < count) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) t += red[w][lane];
    const float r = round_to<T>(t);
    if constexpr (sizeof(OutT) == 4)
      out[i] = r;
    else
      out[i] = Traits<OutT>::from_f(r);
  }
}

// Bias gradient from the dgrad kernel's per-quarter column sums:
// out[e, c] = r_T(sum over the 128-row tiles of expert e's segment and their
// four quarters of part[(tile * 4 + q) * n + c]), in tile order.
// CTA = (expert, 32 columns); its 8 warps each sum every 8th quarter-row of
// the expert's partials for the 32 columns (coalesced), then warp 0 adds the
// 8 warp sums in order.
template <typename T, typename OutT>
__global__ void __launch_bounds__(256) tile_parts_reduce_kernel(const float* __restrict__ part,
                                                                const int32_t* __restrict__ seg_start, int E, int n,
                                                                OutT* __restrict__ out) {
  __shared__ float red[8][32];
  pdl_wait();
  pdl_trigger();
  const int e = blockIdx.y;
  const int c = blockIdx.x * 32 + lane_id();
  const int w = warp_id();
  const int64_t q0 = static_cast<int64_t>(seg_start[e] / AGM_TILE_M) * 4;
  const int64_t q1 = static_cast<int64_t>(seg_start[e + 1] / AGM_TILE_M) * 4;
  float v = 0.f;
  if (c < n)
    for (int64_t q = q0 + w; q < q1; q += 8) v += part[q * n + c];
  red[w][lane_id()] = v;
  __syncthreads();
  if (w == 0 && c < n) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][lane_id()];
    const float r = round_to<T>(s);
    if constexpr (sizeof(OutT) == 4)
      out[static_cast<int64_t>(e) * n + c] = r;
    else
      out[static_cast<int64_t>(e) * n + c] = Traits<OutT>::from_f(r);
  }
}

// ---------------------------------------------------------------------------
// Input gradient: dx[t] = ((dx_perm[row(t,k-1)] + ... + dx_perm[row(t,0)]) + r_T(dl[t] @ Wr)),
// each add rounded to G (T in same-dtype mode, fp32 in autocast). Wr [E, d]
// (compute dtype) is staged in shared memory. A warp handles two tokens per
// iteration: their gathered rows are loaded first, and every Wr value read
// from shared memory serves both tokens' router terms.
// ---------------------------------------------------------------------------
// dx chunk of one token: the ranks' rows summed from the last rank down, then
// the router term, each add rounded to G.
template <typename T, typename G, int K_MAX>
__device__ __forceinline__ void dx_finish(const float (&a)[K_MAX][8], const float (&rt)[8], int k, G* dst,
                                          const T* __restrict__ dxs, int n_shared, int64_t shared_stride) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  bool first = true;
  // shared experts' input gradients arrive first, the last shared expert's first
  for (int si = n_shared - 1; si >= 0; --si) {
    float v[8];
    load8f<T>(dxs + si * shared_stride, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (first)
        acc[i] = v[i];
      else
        acc[i] = (sizeof(G) == 4) ? __fadd_rn(acc[i], v[i]) : round_to<T>(__fadd_rn(acc[i], v[i]));
    }
    first = false;
  }
#pragma unroll
  for (int r = K_MAX - 1; r >= 0; --r) {
    if (r < k) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (first)
          acc[i] = a[r][i];
        else
          acc[i] = (sizeof(G) == 4) ? __fadd_rn(acc[i], a[r][i]) : round_to<T>(__fadd_rn(acc[i], a[r][i]));
      }
      first = false;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float rv = round_to<T>(rt[i]);
    acc[i] = (sizeof(G) == 4) ? __fadd_rn(acc[i], rv) : round_to<T>(__fadd_rn(acc[i], rv));
  }
  store8f<G>(dst, acc);
}

template <typename T, typename G, int K_MAX>
__global__ void __launch_bounds__(256, 3) dx_kernel(const T* __restrict__ dxp, const int32_t* __restrict__ row_of,
                                                 const T* __restrict__ dl, const T* __restrict__ wr, int64_t n,
                                                 int d, int k, int E, const T* __restrict__ dxs, int n_shared,
                                                 int64_t shared_stride, G* __restrict__ dx) {
  extern __shared__ uint8_t smem_raw[];
  // [8 warps][2 tokens][16] logit gradients, then Wr [E, d]
  float* g_s = reinterpret_cast<float*>(smem_raw) + warp_id() * 2 * kMaxE;
  T* w_s = reinterpret_cast<T*>(smem_raw + 8 * 2 * kMaxE * sizeof(float));
  pdl_wait();
  pdl_trigger();
  {
    const int nchunk = E * d * static_cast<int>(sizeof(T)) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(wr);
    uint4* dst = reinterpret_cast<uint4*>(w_s);
    for (int i = threadIdx.x; i < nchunk; i += blockDim.x) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const int lane = lane_id();
  const int nc8 = d / 8;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = 2 * (static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp_id()); t < n; t += 2 * warps) {
    const bool two = t + 1 < n;
    // lane j holds the logit gradient (t + j / 16, e = j % 16)
    __syncwarp();
    g_s[lane] = (lane < kMaxE || two) ? Traits<T>::to_f(dl[t * kMaxE + lane]) : 0.f;
    __syncwarp();
    int64_t row0[K_MAX], row1[K_MAX];
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) {
      row0[r] = (r < k) ? row_of[t * k + r] : 0;
      row1[r] = (r < k && two) ? row_of[(t + 1) * k + r] : row0[r];
    }
    for (int c = lane; c < nc8; c += 32) {
      // gathered expert-path rows first (their loads overlap the router term)
      float a0[K_MAX][8], a1[K_MAX][8];
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) {
        if (r < k) {
          load8f<T>(dxp + row0[r] * d + c * 8, a0[r]);
          load8f<T>(dxp + row1[r] * d + c * 8, a1[r]);
        }
      }
      float rt0[8], rt1[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) rt0[i] = rt1[i] = 0.f;
      for (int e = 0; e < E; ++e) {
        float w[8];
        if constexpr (sizeof(T) == 4) {
          const float4* p = reinterpret_cast<const float4*>(w_s + static_cast<int64_t>(e) * d + c * 8);
          const float4 u = p[0], v = p[1];
          w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w; w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
        } else {
          unpack8<T>(*reinterpret_cast<const uint4*>(w_s + static_cast<int64_t>(e) * d + c * 8), w);
        }
        const float ge0 = g_s[e], ge1 = g_s[kMaxE + e];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          rt0[i] = fmaf(ge0, w[i], rt0[i]);
          rt1[i] = fmaf(ge1, w[i], rt1[i]);
        }
      }
      dx_finish<T, G, K_MAX>(a0, rt0, k, dx + t * d + c * 8, dxs + t * d + c * 8, n_shared, shared_stride);
      if (two)
        dx_finish<T, G, K_MAX>(a1, rt1, k, dx + (t + 1) * d + c * 8, dxs + (t + 1) * d + c * 8, n_shared,
                               shared_stride);
    }
  }
}

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------
int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}
int cuda_fail(cudaError_t e, const char* where) {
  set_last_error(std::string(where) + ": " + cudaGetErrorString(e));
  return AGM_ERR_CUDA;
}
int esize(int dtype) { return dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16) ? 2 : 0; }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int64_t rup(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename P>
  P* take(size_t bytes) {
    off = (off + 255) & ~size_t(255);
    P* p = reinterpret_cast<P*>(base ? base + off : nullptr);
    off += bytes;
    return p;
  }
};

// What the training forward keeps for the backward (plus its own temporaries).
struct Saved {
  int* err;
  float* logits;     // [n, E] fp32 (rounded like the reference's router output)
  int32_t* idx;      // [n, k]
  void* gates;       // [n, k] compute dtype (router output, unused afterwards)
  int32_t* block_hist;
  int32_t* block_off;
  int32_t* counts;   // [E]
  int32_t* seg_start;  // [E + 1]
  int32_t* num_tiles;
  int32_t* tile_expert;
  int32_t* row_of;   // [n, k]
  int32_t* token_of; // [rows]
  void* xb;          // [npad, d] compute dtype, zero rows past n (autocast: the cast input; with
                     // shared experts: their FC1 input, kept for their weight gradient)
  void* x_perm;      // [rows, d]
  void* h;           // [rows, H]
  void* y;           // [rows, d]
  uint32_t* relu_bits;  // [ceil(H / 32), rows]: h > 0 (16-bit compute dtypes)
  void* h_sh;        // [S, npad, Hs] shared experts' FC1 activations
  void* y_sh;        // [S, npad, d] shared experts' outputs
  uint32_t* bits_sh; // [S, ceil(Hs / 32), npad] (16-bit compute dtypes)
  size_t bytes;
};

int64_t npad_of(int64_t n) { return rup(std::max<int64_t>(n, 1), AGM_TILE_M); }

Saved carve_saved(void* ws, int64_t n, int d, int E, int k, int H, int eb, bool amp, int S_, int Hs) {
  Carve c(ws);
  Saved S;
  const int64_t nb = agm_dispatch_blocks(n);
  const int64_t rows = agm_max_rows(n, k, E);
  const int64_t npad = npad_of(n);
  S.err = c.take<int>(sizeof(int));
  S.logits = c.take<float>(sizeof(float) * n * E);
  S.idx = c.take<int32_t>(sizeof(int32_t) * n * k);
  S.gates = c.take<void>(static_cast<size_t>(eb) * n * k);
  S.block_hist = c.take<int32_t>(sizeof(int32_t) * nb * E);
  S.block_off = c.take<int32_t>(sizeof(int32_t) * nb * E);
  S.counts = c.take<int32_t>(sizeof(int32_t) * E);
  S.seg_start = c.take<int32_t>(sizeof(int32_t) * (E + 1));
  S.num_tiles = c.take<int32_t>(sizeof(int32_t));
  S.tile_expert = c.take<int32_t>(sizeof(int32_t) * std::max<int64_t>(rows / AGM_TILE_M, 1));
  S.row_of = c.take<int32_t>(sizeof(int32_t) * n * k);
  S.token_of = c.take<int32_t>(sizeof(int32_t) * std::max<int64_t>(rows, 1));
  S.xb = (amp || S_ > 0) ? c.take<void>(static_cast<size_t>(eb) * npad * d) : nullptr;
  S.x_perm = c.take<void>(static_cast<size_t>(eb) * rows * d);
  S.h = c.take<void>(static_cast<size_t>(eb) * rows * H);
  S.y = c.take<void>(static_cast<size_t>(eb) * rows * d);
  S.relu_bits = eb == 2 ? c.take<uint32_t>(sizeof(uint32_t) * ((H + 31) / 32) * std::max<int64_t>(rows, 1)) : nullptr;
  S.h_sh = S_ > 0 ? c.take<void>(static_cast<size_t>(eb) * S_ * npad * Hs) : nullptr;
  S.y_sh = S_ > 0 ? c.take<void>(static_cast<size_t>(eb) * S_ * npad * d) : nullptr;
  S.bits_sh = (S_ > 0 && eb == 2) ? c.take<uint32_t>(sizeof(uint32_t) * S_ * ((Hs + 31) / 32) * npad) : nullptr;
  S.bytes = (c.off + 255) & ~size_t(255);
  return S;
}

int colsum_splits(int ncols, int E) {
  const int cb = (ncols + kColsumCols - 1) / kColsumCols;
  return std::max(1, std::min(64, (4 * 148 + cb * E - 1) / (cb * E)));
}
// Tokens per router-wgrad CTA: about three CTAs per SM, at most kRwMaxChunk.
int router_tok_per_chunk(int64_t n) {
  return static_cast<int>(std::max<int64_t>(16, std::min<int64_t>(kRwMaxChunk, (n + 3 * 148 - 1) / (3 * 148))));
}
int router_chunks(int64_t n, int d) {
  (void)d;
  const int tpc = router_tok_per_chunk(n);
  return static_cast<int>(std::max<int64_t>(1, (n + tpc - 1) / tpc));
}

struct BwdWs {
  int* err;
  void* dy;     // [rows, d]; later dx_perm
  void* dh;     // [rows, H]
  void* dl;     // [n, 16]
  float* colsum;  // [splits, groups, ncols] for the largest use
  float* rpart;   // [chunks, 16, d]
  float* dh_part; // [max_tiles * 4, H]: dgrad FC2's column sums of dh (16-bit dtypes)
  void* ds;       // [npad, d] gradient of the shared experts' sum (zero rows past n)
  void* dh_sh;    // [npad, Hs] one shared expert's dh at a time
  void* dx_sh;    // [S, npad, d] shared experts' input gradients
  float* dhs_part;  // [npad / 128 * 4, Hs]
  int32_t* dense_seg;  // [2] = {0, npad}: the shared experts' one segment
  size_t bytes;
};

BwdWs carve_bwd(void* ws, int64_t n, int d, int E, int k, int H, int eb, int S_, int Hs) {
  Carve c(ws);
  BwdWs B;
  const int64_t rows = agm_max_rows(n, k, E);
  const int64_t npad = npad_of(n);
  int64_t cs = std::max<int64_t>(static_cast<int64_t>(colsum_splits(d, E)) * d * E,
                                 static_cast<int64_t>(colsum_splits(H, E)) * H * E);
  if (S_ > 0)
    cs = std::max<int64_t>(cs, std::max<int64_t>(static_cast<int64_t>(colsum_splits(d, 1)) * d,
                                                 static_cast<int64_t>(colsum_splits(Hs, 1)) * Hs));
  B.err = c.take<int>(sizeof(int));
  B.dy = c.take<void>(static_cast<size_t>(eb) * rows * d);
  B.dh = c.take<void>(static_cast<size_t>(eb) * rows * H);
  B.dl = c.take<void>(static_cast<size_t>(eb) * n * kMaxE);
  B.colsum = c.take<float>(sizeof(float) * cs);
  B.rpart = c.take<float>(sizeof(float) * router_chunks(n, d) * kMaxE * d);
  B.dh_part = eb == 2 ? c.take<float>(sizeof(float) * (rows / AGM_TILE_M) * 4 * H) : nullptr;
  B.ds = S_ > 0 ? c.take<void>(static_cast<size_t>(eb) * npad * d) : nullptr;
  B.dh_sh = S_ > 0 ? c.take<void>(static_cast<size_t>(eb) * npad * Hs) : nullptr;
  B.dx_sh = S_ > 0 ? c.take<void>(static_cast<size_t>(eb) * S_ * npad * d) : nullptr;
  B.dhs_part = (S_ > 0 && eb == 2) ? c.take<float>(sizeof(float) * (npad / AGM_TILE_M) * 4 * Hs) : nullptr;
  B.dense_seg = S_ > 0 ? c.take<int32_t>(sizeof(int32_t) * 2) : nullptr;
  B.bytes = (c.off + 255) & ~size_t(255);
  return B;
}

template <typename T>
cudaError_t launch_cast(const float* in, void* out, int64_t n, cudaStream_t s) {
  const int64_t blocks = std::min<int64_t>((n / 8 + 255) / 256 + 1, 148 * 8);
  return launch_kernel(cast_f32_kernel<T>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, in,
                       static_cast<T*>(out), n);
}

cudaError_t cast_any(int dtype, const float* in, void* out, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (dtype == AGM_BF16) return launch_cast<__nv_bfloat16>(in, out, n, s);
  if (dtype == AGM_F16) return launch_cast<__half>(in, out, n, s);
  return cudaErrorInvalidValue;
}

template <typename T, typename G>
cudaError_t launch_combine_train(const Saved& S, int64_t n, int d, int k, int E, int n_shared, const void* residual,
                                 void* out, cudaStream_t s) {
  const G* res = static_cast<const G*>(residual);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 7) / 8, 148 * 8));
  const T* y = static_cast<const T*>(S.y);
  const T* sh = static_cast<const T*>(S.y_sh);
  const int64_t stride = npad_of(n) * d;
  G* o = static_cast<G*>(out);
  if (k <= 2)
    return launch_kernel(combine_train_kernel<T, G, 2>, dim3(grid), dim3(256), 0, s, y, S.row_of, S.logits, S.idx, n,
                         d, k, E, sh, n_shared, stride, res, o);
  if (k <= 4)
    return launch_kernel(combine_train_kernel<T, G, 4>, dim3(grid), dim3(256), 0, s, y, S.row_of, S.logits, S.idx, n,
                         d, k, E, sh, n_shared, stride, res, o);
  return launch_kernel(combine_train_kernel<T, G, 16>, dim3(grid), dim3(256), 0, s, y, S.row_of, S.logits, S.idx, n,
                       d, k, E, sh, n_shared, stride, res, o);
}

template <typename T, typename G>
cudaError_t launch_combine_bwd(const void* dout, const Saved& S, const BwdWs& B, int64_t n, int d, int k, int E,
                               int64_t rows, cudaStream_t s) {
  const int tok_ctas = static_cast<int>(std::min<int64_t>((n + 7) / 8, 148 * 8));
  const unsigned grid = static_cast<unsigned>(tok_ctas + E * kZeroCtas);
  const G* go = static_cast<const G*>(dout);
  const T* y = static_cast<const T*>(S.y);
  T* dy = static_cast<T*>(B.dy);
  T* dl = static_cast<T*>(B.dl);
  T* ds = static_cast<T*>(B.ds);
  const int64_t npad = npad_of(n);
  if (k <= 2)
    return launch_kernel(combine_bwd_kernel<T, G, 2>, dim3(grid), dim3(256), 0, s, go, y, S.row_of, S.logits, S.idx,
                         n, d, k, E, tok_ctas, S.seg_start, S.counts, rows, dy, dl, ds, npad, B.dense_seg);
  if (k <= 4)
    return launch_kernel(combine_bwd_kernel<T, G, 4>, dim3(grid), dim3(256), 0, s, go, y, S.row_of, S.logits, S.idx,
                         n, d, k, E, tok_ctas, S.seg_start, S.counts, rows, dy, dl, ds, npad, B.dense_seg);
  return launch_kernel(combine_bwd_kernel<T, G, 16>, dim3(grid), dim3(256), 0, s, go, y, S.row_of, S.logits, S.idx,
                       n, d, k, E, tok_ctas, S.seg_start, S.counts, rows, dy, dl, ds, npad, B.dense_seg);
}

template <typename T, typename OutT>
cudaError_t launch_colsum(const void* m, int ncols, const int32_t* seg_start, int E, float* partial, void* out,
                          cudaStream_t s) {
  const int splits = colsum_splits(ncols, E);
  dim3 grid(static_cast<unsigned>((ncols + kColsumCols - 1) / kColsumCols), static_cast<unsigned>(E),
            static_cast<unsigned>(splits));
  cudaError_t e = launch_kernel(seg_colsum_kernel<T>, grid, dim3(256), 0, s, static_cast<const T*>(m), ncols,
                                seg_start, E, splits, partial);
  if (e != cudaSuccess) return e;
  const int64_t count = static_cast<int64_t>(E) * ncols;
  const unsigned g2 = static_cast<unsigned>(std::min<int64_t>((count + 255) / 256, 148 * 4));
  return launch_kernel(reduce_partials_kernel<T, OutT>, dim3(g2), dim3(256), 0, s,
                       static_cast<const float*>(partial), splits, count, count, static_cast<OutT*>(out));
}

template <typename T, typename OutT>
cudaError_t launch_tile_parts(const float* part, const int32_t* seg_start, int E, int ncols, void* out,
                              cudaStream_t s) {
  dim3 grid(static_cast<unsigned>((ncols + 31) / 32), static_cast<unsigned>(E));
  return launch_kernel(tile_parts_reduce_kernel<T, OutT>, grid, dim3(256), 0, s, part, seg_start, E, ncols,
                       static_cast<OutT*>(out));
}

template <typename T, typename OutT>
cudaError_t launch_router_wgrad(const BwdWs& B, const Saved& S, int64_t n, int d, int k, int E, void* dwr,
                                cudaStream_t s) {
  const int chunks = router_chunks(n, d);
  const int tpc = router_tok_per_chunk(n);
  const int threads = std::min(512, (d / 4 + 31) / 32 * 32);
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>((d / 4 + threads - 1) / threads));
  cudaError_t e = launch_kernel(router_wgrad_kernel<T>, grid, dim3(threads), 0, s, static_cast<const T*>(B.dl),
                                static_cast<const T*>(S.x_perm), S.row_of, k, n, d, tpc, B.rpart);
  if (e != cudaSuccess) return e;
  // Chunk c's partial is [16, d] at c * 16 * d; its first E rows, E * d
  // contiguous values, are the router weight's.
  const int64_t count = static_cast<int64_t>(E) * d;
  return launch_kernel(reduce_partials_wide_kernel<T, OutT>, dim3(static_cast<unsigned>((count + 31) / 32)),
                       dim3(256), 0, s, static_cast<const float*>(B.rpart), chunks,
                       static_cast<int64_t>(kMaxE) * d, count, static_cast<OutT*>(dwr));
}

template <typename T, typename G>
cudaError_t launch_dx(const BwdWs& B, const Saved& S, const void* wr, int64_t n, int d, int k, int E, int n_shared,
                      void* dx, cudaStream_t s) {
  const T* dxs = static_cast<const T*>(B.dx_sh);
  const int64_t sstride = npad_of(n) * d;
  const int smem = E * d * static_cast<int>(sizeof(T)) + 8 * 2 * kMaxE * static_cast<int>(sizeof(float));
  // As many CTAs as fit beside each other (Wr staged in each one's shared memory).
  const int per_sm = std::max(1, std::min(8, (227 * 1024) / std::max(smem + 1024, 1)));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 15) / 16, 148 * per_sm));
  const T* dxp = static_cast<const T*>(B.dy);
  const T* dl = static_cast<const T*>(B.dl);
  const T* w = static_cast<const T*>(wr);
  G* o = static_cast<G*>(dx);
  cudaError_t e;
  if (k <= 2) {
    if ((e = ensure_dynamic_smem(reinterpret_cast<const void*>(dx_kernel<T, G, 2>), smem)) != cudaSuccess) return e;
    return launch_kernel(dx_kernel<T, G, 2>, dim3(grid), dim3(256), smem, s, dxp, S.row_of, dl, w, n, d, k, E, dxs, n_shared,
                         sstride, o);
  }
  if (k <= 4) {
    if ((e = ensure_dynamic_smem(reinterpret_cast<const void*>(dx_kernel<T, G, 4>), smem)) != cudaSuccess) return e;
    return launch_kernel(dx_kernel<T, G, 4>, dim3(grid), dim3(256), smem, s, dxp, S.row_of, dl, w, n, d, k, E, dxs, n_shared,
                         sstride, o);
  }
  if ((e = ensure_dynamic_smem(reinterpret_cast<const void*>(dx_kernel<T, G, 16>), smem)) != cudaSuccess) return e;
  return launch_kernel(dx_kernel<T, G, 16>, dim3(grid), dim3(256), smem, s, dxp, S.row_of, dl, w, n, d, k, E, dxs, n_shared,
                         sstride, o);
}

// ---------------------------------------------------------------------------
// Auxiliary router losses (_collect_moe_aux, agillm41.py:4463-4492): the
// load-balance loss aux_coef * E * sum_e(load_e * importance_e) and the
// router-z loss z_coef * mean_t(logsumexp(scores_t)^2), over the router logits
// recomputed from the stashed FFN input (kept as fp32 values [N, E] in the
// saved state, each rounded to the router's dtype as F.linear rounds it).
//   importance_e = mean_t softmax(scores_t)_e
//   load_e       = #{t : argmax_e softmax(scores_t) = e} / max(1, N)   (no gradient)
// aux_stats: one CTA per token chunk, fixed-order partial sums; aux_finalize
// (one warp) adds the partials in chunk order and writes the loss and the
// backward's per-expert factors.
// ---------------------------------------------------------------------------
constexpr int kAuxThreads = 256;
constexpr int kAuxParts = kMaxE + 1;  // importance sums [16], then the sum of lse^2

int aux_tok_per_chunk(int64_t n) {
  // Chunking depends on n only, so the loss is the same on every GPU.
  const int64_t per = (n + 295) / 296;
  return static_cast<int>(std::max<int64_t>(kAuxThreads, (per + kAuxThreads - 1) / kAuxThreads * kAuxThreads));
}
int aux_chunks(int64_t n) { return n == 0 ? 0 : static_cast<int>((n + aux_tok_per_chunk(n) - 1) / aux_tok_per_chunk(n)); }

// Softmax of one token's logits (exp(l - max) / sum, the first maximum's index
// as argmax) and its logsumexp.
__device__ __forceinline__ void aux_softmax(const float* __restrict__ lrow, int E, float (&p)[kMaxE], float& lse,
                                            int& top) {
  float m = -INFINITY;
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) {
    p[e] = e < E ? lrow[e] : -INFINITY;
    m = fmaxf(m, p[e]);
  }
  float sum = 0.f;
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) {
    p[e] = e < E ? expf(p[e] - m) : 0.f;
    sum += p[e];
  }
  lse = m + logf(sum);
  top = 0;
  float best = -1.f;
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) {
    p[e] = p[e] / sum;
    if (e < E && p[e] > best) {
      best = p[e];
      top = e;
    }
  }
}

__global__ void __launch_bounds__(kAuxThreads) aux_stats_kernel(const float* __restrict__ logits, int64_t n, int E,
                                                                int tok_per_chunk, float* __restrict__ part,
                                                                int32_t* __restrict__ cnt_part) {
  __shared__ float red[kAuxThreads / 32][kAuxParts];
  __shared__ int cnt_s[kMaxE];
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x < kMaxE) cnt_s[threadIdx.x] = 0;
  __syncthreads();
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tok_per_chunk;
  const int64_t t1 = min(n, t0 + tok_per_chunk);
  float acc[kAuxParts];
#pragma unroll
  for (int i = 0; i < kAuxParts; ++i) acc[i] = 0.f;
  for (int64_t t = t0 + threadIdx.x; t < t1; t += kAuxThreads) {
    float p[kMaxE], lse;
    int top;
    aux_softmax(logits + t * E, E, p, lse, top);
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) acc[e] += p[e];
    acc[kMaxE] += lse * lse;
    atomicAdd(&cnt_s[top], 1);  // integer counts: exact in any order
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < kAuxParts; ++i) {
    const float v = warp_sum(acc[i]);
    if (lane == 0) red[warp][i] = v;
  }
  __syncthreads();
  if (threadIdx.x < kAuxParts) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kAuxThreads / 32; ++w) v += red[w][threadIdx.x];
    part[static_cast<int64_t>(blockIdx.x) * kAuxParts + threadIdx.x] = v;
  }
  if (threadIdx.x < kMaxE) cnt_part[static_cast<int64_t>(blockIdx.x) * kMaxE + threadIdx.x] = cnt_s[threadIdx.x];
}

// factors[e] = c_lb * load_e / N (the load-balance term's gradient with
// respect to probs[t, e]), factors[16] = 2 * z_coef / N (the z term's, times
// lse_t). Missing terms (coefficient <= 0) get zero factors.
__global__ void __launch_bounds__(512) aux_finalize_kernel(const float* __restrict__ part,
                                                            const int32_t* __restrict__ cnt_part, int chunks,
                                                            int64_t n, int E, float c_lb, float z_coef, int use_lb,
                                                            int use_z, float* __restrict__ loss,
                                                            float* __restrict__ factors) {
  // Warp w adds chunks w, w + 16, ... (lane < 17: the float partials, lane
  // 17..32 reads nothing); then warp 0 adds the 16 warp sums in warp order.
  __shared__ float red_s[16][32];
  __shared__ int red_c[16][32];
  __shared__ float terms[kMaxE];
  __shared__ float zsum;
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float s = 0.f;
  int c = 0;
  for (int i = warp; i < chunks; i += 16) {
    if (lane < kAuxParts) s += part[static_cast<int64_t>(i) * kAuxParts + lane];
    if (lane < kMaxE) c += cnt_part[static_cast<int64_t>(i) * kMaxE + lane];
  }
  red_s[warp][lane] = s;
  red_c[warp][lane] = c;
  __syncthreads();
  if (warp != 0) return;
  s = 0.f;
  c = 0;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    s += red_s[w][lane];
    c += red_c[w][lane];
  }
  const float nf = static_cast<float>(n);
  if (lane < kMaxE) {
    const float importance = s / nf;  // mean over tokens (NaN for no tokens, as torch's mean)
    const float load = static_cast<float>(c) / static_cast<float>(n > 0 ? n : 1);
    terms[lane] = lane < E ? load * importance : 0.f;
    factors[lane] = (use_lb && lane < E) ? c_lb * load / nf : 0.f;
  }
  if (lane == kMaxE) zsum = s;
  __syncwarp();
  if (lane == 0) {
    float dot = 0.f;
    for (int e = 0; e < E; ++e) dot += terms[e];  // the sum over experts in expert order
    const float lb = c_lb * dot;
    const float zl = z_coef * (zsum / nf);
    *loss = use_lb ? (use_z ? lb + zl : lb) : (use_z ? zl : 0.f);
    factors[kMaxE] = use_z ? 2.f * z_coef / nf : 0.f;
  }
}

// Logit gradients of the auxiliary loss for one token, written as T to
// dl[t, 0..15] (zero past E): with G the loss's upstream gradient,
//   d/dl_e = p_e * (G * f_e - sum_j p_j * G * f_j) + G * f_z * lse * p_e.
template <typename T>
__global__ void __launch_bounds__(kAuxThreads) aux_dlogit_kernel(const float* __restrict__ logits, int64_t n, int E,
                                                                 const float* __restrict__ dloss,
                                                                 const float* __restrict__ factors,
                                                                 T* __restrict__ dl) {
  pdl_wait();
  pdl_trigger();
  const float G = *dloss;
  float f[kMaxE];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) f[e] = G * factors[e];
  const float fz = G * factors[kMaxE];
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kAuxThreads + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * kAuxThreads) {
    float p[kMaxE], lse;
    int top;
    aux_softmax(logits + t * E, E, p, lse, top);
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) dot += p[e] * f[e];
    const float z = fz * lse;
    float g[kMaxE];
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) g[e] = e < E ? p[e] * (f[e] - dot) + z * p[e] : 0.f;
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = g[i];
      hi[i] = g[8 + i];
    }
    store8f<T>(dl + t * kMaxE, lo);
    store8f<T>(dl + t * kMaxE + 8, hi);
  }
}

// What the auxiliary-loss forward keeps for its backward (plus temporaries).
struct AuxSaved {
  int* err;
  float* factors;   // [17]: per-expert load-balance factors, then the z factor
  float* logits;    // [n, E] router logits (values of the router's dtype)
  int32_t* idx;     // [n] top-1 expert (the router kernel's output, unused)
  void* gates;      // [n]
  int32_t* block_hist;
  float* part;      // [chunks, 17]
  int32_t* cnt_part;  // [chunks, 16]
  size_t bytes;
};

AuxSaved carve_aux(void* ws, int64_t n, int E, int eb) {
  Carve c(ws);
  AuxSaved A;
  const int chunks = aux_chunks(n);
  A.err = c.take<int>(sizeof(int));
  A.factors = c.take<float>(sizeof(float) * (kMaxE + 1));
  A.logits = c.take<float>(sizeof(float) * n * E);
  A.idx = c.take<int32_t>(sizeof(int32_t) * n);
  A.gates = c.take<void>(static_cast<size_t>(eb) * n);
  A.block_hist = c.take<int32_t>(sizeof(int32_t) * agm_dispatch_blocks(n) * E);
  A.part = c.take<float>(sizeof(float) * chunks * kAuxParts);
  A.cnt_part = c.take<int32_t>(sizeof(int32_t) * chunks * kMaxE);
  A.bytes = c.off;
  return A;
}

struct AuxBwd {
  void* dl;      // [n, 16] logit gradients in the router's dtype
  float* rpart;  // [router chunks, 16, d] weight-gradient partials
  size_t bytes;
};

AuxBwd carve_aux_bwd(void* ws, int64_t n, int d, int eb) {
  Carve c(ws);
  AuxBwd B;
  B.dl = c.take<void>(static_cast<size_t>(eb) * n * kMaxE);
  B.rpart = c.take<float>(sizeof(float) * router_chunks(n, d) * kMaxE * d);
  B.bytes = c.off;
  return B;
}

cudaError_t launch_aux_forward(const AuxSaved& A, int64_t n, int E, float c_lb, float z_coef, int use_lb, int use_z,
                               float* loss, cudaStream_t s) {
  const int chunks = aux_chunks(n);
  cudaError_t e = cudaSuccess;
  if (chunks > 0)
    e = launch_kernel(aux_stats_kernel, dim3(static_cast<unsigned>(chunks)), dim3(kAuxThreads), 0, s,
                      static_cast<const float*>(A.logits), n, E, aux_tok_per_chunk(n), A.part, A.cnt_part);
  if (e != cudaSuccess) return e;
  return launch_kernel(aux_finalize_kernel, dim3(1), dim3(512), 0, s, static_cast<const float*>(A.part),
                       static_cast<const int32_t*>(A.cnt_part), chunks, n, E, c_lb, z_coef, use_lb, use_z, loss,
                       A.factors);
}

template <typename T>
cudaError_t launch_aux_backward(const AuxSaved& A, const AuxBwd& B, const float* dloss, const void* x, int64_t n,
                                int d, int E, void* dw, cudaStream_t s) {
  const unsigned g = static_cast<unsigned>(std::min<int64_t>((n + kAuxThreads - 1) / kAuxThreads, 148 * 8));
  cudaError_t e = launch_kernel(aux_dlogit_kernel<T>, dim3(g), dim3(kAuxThreads), 0, s,
                                static_cast<const float*>(A.logits), n, E, dloss,
                                static_cast<const float*>(A.factors), static_cast<T*>(B.dl));
  if (e != cudaSuccess) return e;
  const int chunks = router_chunks(n, d);
  const int tpc = router_tok_per_chunk(n);
  const int threads = std::min(512, (d / 4 + 31) / 32 * 32);
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>((d / 4 + threads - 1) / threads));
  e = launch_kernel(router_wgrad_kernel<T>, grid, dim3(threads), 0, s, static_cast<const T*>(B.dl),
                    static_cast<const T*>(x), static_cast<const int32_t*>(nullptr), 1, n, d, tpc, B.rpart);
  if (e != cudaSuccess) return e;
  const int64_t count = static_cast<int64_t>(E) * d;
  return launch_kernel(reduce_partials_wide_kernel<T, T>, dim3(static_cast<unsigned>((count + 31) / 32)), dim3(256),
                       0, s, static_cast<const float*>(B.rpart), chunks, static_cast<int64_t>(kMaxE) * d, count,
                       static_cast<T*>(dw));
}

}  // namespace
}  // namespace agm

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {

int check_train_args(int x_dtype, int dtype, int64_t n, int d, int E, int k, int H, int S, int Hs) {
  if (!agm::esize(dtype) || !agm::esize(x_dtype)) return agm::fail(AGM_ERR_ARG, "bad dtype code");
  if (x_dtype != dtype && !(x_dtype == AGM_F32 && dtype != AGM_F32))
    return agm::fail(AGM_ERR_ARG, "x_dtype must equal dtype, or be AGM_F32 with a 16-bit dtype (autocast)");
  const int eb = agm::esize(dtype);
  if (n < 0) return agm::fail(AGM_ERR_ARG, "n_tokens < 0");
  if (E < 1 || E > AGM_MAX_EXPERTS) return agm::fail(AGM_ERR_UNSUPPORTED, "number of experts must be in [1, 16]");
  if (k < 1 || k > E) return agm::fail(AGM_ERR_ARG, "top_k must be in [1, n_experts]");
  if (S < 0) return agm::fail(AGM_ERR_ARG, "n_shared < 0");
  if (d <= 0 || d % 8 || H <= 0 || H % 8 || (S > 0 && (Hs <= 0 || Hs % 8)))
    return agm::fail(AGM_ERR_UNSUPPORTED, "d, hidden and shared_hidden must be positive multiples of 8");
  if ((static_cast<int64_t>(d) * eb) % 16 || (static_cast<int64_t>(H) * eb) % 16 ||
      (S > 0 && (static_cast<int64_t>(Hs) * eb) % 16))
    return agm::fail(AGM_ERR_UNSUPPORTED, "d and hidden must be multiples of 16 bytes of the dtype");
  if (agm_max_rows(n, k, E) > INT32_MAX) return agm::fail(AGM_ERR_UNSUPPORTED, "too many permuted rows");
  if (dtype != AGM_F32 && !agm::router_tc_supported(d))
    return agm::fail(AGM_ERR_UNSUPPORTED, "the tensor-core router does not support this d");
  if (dtype == AGM_F32 && agm::router_smem_bytes(d, E) > 227 * 1024)
    return agm::fail(AGM_ERR_UNSUPPORTED, "router weight does not fit in shared memory for this d");
  if (static_cast<int64_t>(E) * d * eb > 200 * 1024)
    return agm::fail(AGM_ERR_UNSUPPORTED, "router weight does not fit in shared memory for the input gradient");
  return AGM_OK;
}

// One shared expert's FC1 / FC2 over all npad token rows (a single group).
agm::GemmArgs dense_args(void* c, int64_t npad, int n_out, int k_in, const void* bias, int* err) {
  agm::GemmArgs g;
  g.c = c;
  g.ldc = n_out;
  g.c_rows = npad;
  g.bias = bias;
  g.n = n_out;
  g.k = k_in;
  g.groups = 1;
  g.tile_group = nullptr;
  g.num_tiles = nullptr;
  g.max_tiles = static_cast<int>(npad / AGM_TILE_M);
  g.err = err;
  return g;
}

// Backward GEMMs: CTA pairs for 16-bit dtypes when there are enough 256 x 256
// units for the 74 clusters (dgrad also needs 256-row segments), one CTA per
// tile otherwise.
cudaError_t wgrad_any(int dtype, bool amp, const void* dc, const void* act, int64_t rows,
                      const agm::BwdGemmArgs& a, int sms, int pair_mode, cudaStream_t s) {
  // pair_mode: 0 = one CTA per tile (AGM_FLAG_NO_PAIR), 1 = pairs when they
  // fill the GPU, 2 = pairs always (AGM_FLAG_BWD_PAIR)
  const int64_t units = static_cast<int64_t>(a.groups) * (((a.m + 127) / 128 + 1) / 2) * ((a.n + 255) / 256);
  if (dtype != AGM_F32 && pair_mode > 0 && (pair_mode == 2 || units >= sms / 2))
    return agm::grouped_gemm_wgrad_pair(dtype, amp, dc, act, rows, a, sms, s);
  return agm::grouped_gemm_wgrad(dtype, amp, dc, act, rows, a, sms, s);
}
cudaError_t dgrad_any(int dtype, bool pair_rows, const void* dc, int64_t rows, const void* w,
                      const agm::BwdGemmArgs& a, bool relu_mask, int sms, int pair_mode, cudaStream_t s) {
  const int64_t units = ((static_cast<int64_t>(a.max_tiles) + 1) / 2) * ((a.n + 255) / 256);
  if (dtype != AGM_F32 && pair_rows && pair_mode > 0 && (pair_mode == 2 || units >= sms / 2))
    return agm::grouped_gemm_dgrad_pair(dtype, dc, rows, w, a, relu_mask, sms, s);
  return agm::grouped_gemm_dgrad(dtype, dc, rows, w, a, relu_mask, sms, s);
}

const uint8_t* at(const void* p, size_t bytes) { return static_cast<const uint8_t*>(p) + bytes; }
uint8_t* at(void* p, size_t bytes) { return static_cast<uint8_t*>(p) + bytes; }

}  // namespace

extern "C" {

size_t agm_moe_train_saved_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int n_shared,
                                 int shared_hidden, int x_dtype, int dtype) {
  const int eb = agm::esize(dtype);
  if (!eb || n_tokens < 0 || d <= 0 || n_experts < 1 || top_k < 1 || hidden <= 0 || n_shared < 0) return 0;
  return agm::carve_saved(nullptr, n_tokens, d, n_experts, top_k, hidden, eb, x_dtype != dtype, n_shared,
                          std::max(1, shared_hidden))
      .bytes;
}

size_t agm_moe_backward_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int n_shared,
                                        int shared_hidden, int dtype) {
  const int eb = agm::esize(dtype);
  if (!eb || n_tokens < 0 || d <= 0 || n_experts < 1 || top_k < 1 || hidden <= 0 || n_shared < 0) return 0;
  return agm::carve_bwd(nullptr, n_tokens, d, n_experts, top_k, hidden, eb, n_shared, std::max(1, shared_hidden))
      .bytes;
}

int agm_cast_f32(const float* in, void* out, int dtype, int64_t n, void* stream) {
  if (dtype != AGM_BF16 && dtype != AGM_F16) return agm::fail(AGM_ERR_ARG, "dtype must be AGM_BF16 or AGM_F16");
  if (n < 0) return agm::fail(AGM_ERR_ARG, "n < 0");
  if (n == 0) return AGM_OK;
  if (!in || !out || !agm::al16(in) || !agm::al16(out))
    return agm::fail(AGM_ERR_ARG, "in and out must be non-null and 16-byte aligned");
  cudaError_t e = agm::cast_any(dtype, in, out, n, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "cast");
}

int agm_moe_forward_train(const void* x, int x_dtype, int dtype, int64_t n_tokens, int d, int n_experts, int top_k,
                          int hidden, const void* w_router, const void* w1, const void* b1, const void* w2,
                          const void* b2, int n_shared, int shared_hidden, const void* ws1, const void* sb1,
                          const void* ws2, const void* sb2, const void* residual, void* out, void* saved,
                          size_t saved_bytes, int32_t* counts_out, int flags, void* stream_) {
  int rc = check_train_args(x_dtype, dtype, n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden);
  if (rc) return rc;
  if (!x || !w_router || !w1 || !b1 || !w2 || !b2 || !out || !saved) return agm::fail(AGM_ERR_ARG, "null pointer");
  if (n_shared > 0 && (!ws1 || !sb1 || !ws2 || !sb2)) return agm::fail(AGM_ERR_ARG, "null shared-expert pointer");
  const void* ptrs[] = {x, w_router, w1, b1, w2, b2, out, saved};
  for (const void* p : ptrs)
    if (!agm::al16(p)) return agm::fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  if (n_shared > 0 && (!agm::al16(ws1) || !agm::al16(sb1) || !agm::al16(ws2) || !agm::al16(sb2)))
    return agm::fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  if (residual && !agm::al16(residual)) return agm::fail(AGM_ERR_ARG, "residual must be 16-byte aligned");
  const int eb = agm::esize(dtype);
  const bool amp = x_dtype != dtype;
  const int Hs = std::max(1, shared_hidden);
  agm::Saved S = agm::carve_saved(saved, n_tokens, d, n_experts, top_k, hidden, eb, amp, n_shared, Hs);
  if (S.bytes > saved_bytes) return agm::fail(AGM_ERR_WORKSPACE, "saved-state buffer too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PdlScope pdl_scope(!(flags & AGM_FLAG_NO_PDL));
  cudaError_t e = cudaMemsetAsync(S.err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "memset");
  if (n_tokens == 0) {
    e = counts_out ? cudaMemsetAsync(counts_out, 0, sizeof(int32_t) * n_experts, stream) : cudaSuccess;
    return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "memset");
  }
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  const int64_t npad = agm::npad_of(n_tokens);
  const int sms = agm::sm_count();
  const void* xin = x;
  if (S.xb) {
    // [npad, d]: the compute-dtype input with zero rows past n (the shared
    // experts' weight gradient reads whole 128-row tiles of it).
    if (amp)
      e = agm::cast_any(dtype, static_cast<const float*>(x), S.xb, n_tokens * d, stream);
    else
      e = cudaMemcpyAsync(S.xb, x, static_cast<size_t>(eb) * n_tokens * d, cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess && npad > n_tokens)
      e = cudaMemsetAsync(at(S.xb, static_cast<size_t>(eb) * n_tokens * d), 0,
                          static_cast<size_t>(eb) * (npad - n_tokens) * d, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "input copy");
    xin = S.xb;
  }
  e = agm::router_topk(dtype, xin, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST, nullptr,
                       S.logits, S.idx, S.gates, S.block_hist, S.err, sms, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "router_topk");
  const bool pair = dtype != AGM_F32 && !(flags & AGM_FLAG_NO_PAIR) &&
                    static_cast<int64_t>(top_k) * n_tokens >= AGM_PAIR_MIN_ROWS;
  const int max_tiles = static_cast<int>(rows / AGM_TILE_M);
  e = agm::dispatch_plan(S.block_hist, static_cast<int>(agm_dispatch_blocks(n_tokens)), n_experts, rows, max_tiles,
                         pair ? AGM_PAIR_ROWS : AGM_TILE_M, S.block_off, S.counts, S.seg_start, S.tile_expert,
                         S.num_tiles, S.token_of, S.err, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "dispatch_plan");
  if (counts_out) {
    e = cudaMemcpyAsync(counts_out, S.counts, sizeof(int32_t) * n_experts, cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "counts copy");
  }
  e = agm::permute_rows(xin, eb, n_tokens, d, top_k, n_experts, S.idx, S.block_off, S.seg_start, S.counts, rows,
                        S.x_perm, S.row_of, S.token_of, S.err, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "permute");
  agm::GemmArgs g1;
  g1.c = S.h;
  g1.ldc = hidden;
  g1.c_rows = rows;
  g1.bias = b1;
  g1.n = hidden;
  g1.k = d;
  g1.groups = n_experts;
  g1.tile_group = S.tile_expert;
  g1.num_tiles = S.num_tiles;
  g1.max_tiles = max_tiles;
  g1.err = S.err;
  g1.relu_bits = S.relu_bits;  // the ReLU backward reads these bits instead of h
  g1.ld_bits = rows;
  // Row-tile GEMMs only (no swapped operands): the backward reads whole
  // 128-row tiles of h, so its padding rows must hold finite values.
  e = agm::grouped_gemm(dtype, S.x_perm, rows, w1, g1, true, sms, stream, pair ? AGM_GEMM_PAIR : 0);
  if (e != cudaSuccess) return agm::cuda_fail(e, "grouped_gemm fc1");
  agm::GemmArgs g2 = g1;
  g2.relu_bits = nullptr;
  g2.c = S.y;
  g2.ldc = d;
  g2.bias = b2;
  g2.n = d;
  g2.k = hidden;
  e = agm::grouped_gemm(dtype, S.h, rows, w2, g2, false, sms, stream, pair ? AGM_GEMM_PAIR : 0);
  if (e != cudaSuccess) return agm::cuda_fail(e, "grouped_gemm fc2");
  // Shared experts: one dense group, so the CTA-pair GEMM applies for large batches.
  const int shared_mode = (dtype != AGM_F32 && !(flags & AGM_FLAG_NO_PAIR) && n_tokens >= AGM_PAIR_MIN_ROWS)
                              ? AGM_GEMM_PAIR : 0;
  for (int s = 0; s < n_shared; ++s) {
    void* hs = at(S.h_sh, static_cast<size_t>(eb) * s * npad * Hs);
    agm::GemmArgs s1 = dense_args(hs, npad, Hs, d, at(sb1, static_cast<size_t>(eb) * s * Hs), S.err);
    if (S.bits_sh) {
      s1.relu_bits = S.bits_sh + static_cast<int64_t>(s) * ((Hs + 31) / 32) * npad;
      s1.ld_bits = npad;
    }
    e = agm::grouped_gemm(dtype, xin, n_tokens, at(ws1, static_cast<size_t>(eb) * s * Hs * d), s1, true, sms,
                          stream, shared_mode);
    if (e != cudaSuccess) return agm::cuda_fail(e, "grouped_gemm shared fc1");
    agm::GemmArgs s2 = dense_args(at(S.y_sh, static_cast<size_t>(eb) * s * npad * d), npad, d, Hs,
                                  at(sb2, static_cast<size_t>(eb) * s * d), S.err);
    e = agm::grouped_gemm(dtype, hs, npad, at(ws2, static_cast<size_t>(eb) * s * d * Hs), s2, false, sms, stream,
                          shared_mode);
    if (e != cudaSuccess) return agm::cuda_fail(e, "grouped_gemm shared fc2");
  }
  switch (dtype) {
    case AGM_F32:
      e = agm::launch_combine_train<float, float>(S, n_tokens, d, top_k, n_experts, n_shared, residual, out,
                                                  stream);
      break;
    case AGM_BF16:
      e = amp ? agm::launch_combine_train<__nv_bfloat16, float>(S, n_tokens, d, top_k, n_experts, n_shared, residual,
                                                                 out, stream)
              : agm::launch_combine_train<__nv_bfloat16, __nv_bfloat16>(S, n_tokens, d, top_k, n_experts, n_shared,
                                                                         residual, out, stream);
      break;
    default:
      e = amp ? agm::launch_combine_train<__half, float>(S, n_tokens, d, top_k, n_experts, n_shared, residual, out,
                                                         stream)
              : agm::launch_combine_train<__half, __half>(S, n_tokens, d, top_k, n_experts, n_shared, residual, out,
                                                          stream);
  }
  return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "combine_train");
}

int agm_moe_backward(const void* dout, int x_dtype, int dtype, int64_t n_tokens, int d, int n_experts, int top_k,
                     int hidden, const void* w_router, const void* w1, const void* w2, int n_shared,
                     int shared_hidden, const void* ws1, const void* ws2, const void* saved, size_t saved_bytes,
                     void* dx, void* dw_router, void* dw1, void* db1, void* dw2, void* db2, void* dws1, void* dsb1,
                     void* dws2, void* dsb2, void* workspace, size_t workspace_bytes, int flags, void* stream_) {
  int rc = check_train_args(x_dtype, dtype, n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden);
  if (rc) return rc;
  if (!dout || !w_router || !w1 || !w2 || !saved || !dx || !dw_router || !dw1 || !db1 || !dw2 || !db2 || !workspace)
    return agm::fail(AGM_ERR_ARG, "null pointer");
  if (n_shared > 0 && (!ws1 || !ws2 || !dws1 || !dsb1 || !dws2 || !dsb2))
    return agm::fail(AGM_ERR_ARG, "null shared-expert pointer");
  const void* ptrs[] = {dout, w_router, w1, w2, saved, dx, dw_router, dw1, db1, dw2, db2, workspace};
  for (const void* p : ptrs)
    if (!agm::al16(p)) return agm::fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  if (n_shared > 0) {
    const void* sp[] = {ws1, ws2, dws1, dsb1, dws2, dsb2};
    for (const void* p : sp)
      if (!agm::al16(p)) return agm::fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  }
  const int eb = agm::esize(dtype);
  const bool amp = x_dtype != dtype;
  const int Hs = std::max(1, shared_hidden);
  agm::Saved S = agm::carve_saved(const_cast<void*>(saved), n_tokens, d, n_experts, top_k, hidden, eb, amp, n_shared,
                                  Hs);
  if (S.bytes > saved_bytes) return agm::fail(AGM_ERR_WORKSPACE, "saved-state buffer too small");
  agm::BwdWs B = agm::carve_bwd(workspace, n_tokens, d, n_experts, top_k, hidden, eb, n_shared, Hs);
  if (B.bytes > workspace_bytes) return agm::fail(AGM_ERR_WORKSPACE, "workspace too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PdlScope pdl_scope(!(flags & AGM_FLAG_NO_PDL));
  cudaError_t e = cudaMemsetAsync(B.err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "memset");
  const int xe = agm::esize(x_dtype);
  if (n_tokens == 0) {
    // No tokens: every gradient is zero.
    const size_t sizes[] = {static_cast<size_t>(xe) * n_experts * d, static_cast<size_t>(xe) * n_experts * hidden * d,
                            static_cast<size_t>(xe) * n_experts * hidden, static_cast<size_t>(xe) * n_experts * d * hidden,
                            static_cast<size_t>(xe) * n_experts * d, static_cast<size_t>(xe) * n_shared * Hs * d,
                            static_cast<size_t>(xe) * n_shared * Hs, static_cast<size_t>(xe) * n_shared * d * Hs,
                            static_cast<size_t>(xe) * n_shared * d};
    void* outs[] = {dw_router, dw1, db1, dw2, db2, dws1, dsb1, dws2, dsb2};
    for (int i = 0; i < 9 && e == cudaSuccess; ++i)
      if (outs[i] && sizes[i]) e = cudaMemsetAsync(outs[i], 0, sizes[i], stream);
    return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "memset");
  }
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  const int64_t npad = agm::npad_of(n_tokens);
  const int sms = agm::sm_count();
  const int max_tiles = static_cast<int>(rows / AGM_TILE_M);
  // The forward padded expert segments to 256 rows exactly when this holds
  // (the caller passes the forward's AGM_FLAG_NO_PAIR here too).
  const bool pair_rows = dtype != AGM_F32 && !(flags & AGM_FLAG_NO_PAIR) &&
                         static_cast<int64_t>(top_k) * n_tokens >= AGM_PAIR_MIN_ROWS;
  const int pair_mode = (flags & AGM_FLAG_NO_PAIR) ? 0 : (flags & AGM_FLAG_BWD_PAIR) ? 2 : 1;

  // Per-segment column sums (fp32 SIMT path, and db2) into out.
  auto colsum = [&](const void* m, int ncols, const int32_t* seg, int groups, void* out) -> cudaError_t {
    switch (dtype) {
      case AGM_F32: return agm::launch_colsum<float, float>(m, ncols, seg, groups, B.colsum, out, stream);
      case AGM_BF16:
        return amp ? agm::launch_colsum<__nv_bfloat16, float>(m, ncols, seg, groups, B.colsum, out, stream)
                   : agm::launch_colsum<__nv_bfloat16, __nv_bfloat16>(m, ncols, seg, groups, B.colsum, out, stream);
      default:
        return amp ? agm::launch_colsum<__half, float>(m, ncols, seg, groups, B.colsum, out, stream)
                   : agm::launch_colsum<__half, __half>(m, ncols, seg, groups, B.colsum, out, stream);
    }
  };
  // Bias gradient from the dgrad epilogue's per-quarter partials.
  auto tile_parts = [&](const float* part, const int32_t* seg, int groups, int ncols, void* out) -> cudaError_t {
    switch (dtype) {
      case AGM_BF16:
        return amp ? agm::launch_tile_parts<__nv_bfloat16, float>(part, seg, groups, ncols, out, stream)
                   : agm::launch_tile_parts<__nv_bfloat16, __nv_bfloat16>(part, seg, groups, ncols, out, stream);
      default:
        return amp ? agm::launch_tile_parts<__half, float>(part, seg, groups, ncols, out, stream)
                   : agm::launch_tile_parts<__half, __half>(part, seg, groups, ncols, out, stream);
    }
  };

  // 1. combine + routing backward -> dy, dl (and the shared sum's gradient ds)
  switch (dtype) {
    case AGM_F32: e = agm::launch_combine_bwd<float, float>(dout, S, B, n_tokens, d, top_k, n_experts, rows, stream); break;
    case AGM_BF16:
      e = amp ? agm::launch_combine_bwd<__nv_bfloat16, float>(dout, S, B, n_tokens, d, top_k, n_experts, rows, stream)
              : agm::launch_combine_bwd<__nv_bfloat16, __nv_bfloat16>(dout, S, B, n_tokens, d, top_k, n_experts, rows,
                                                                      stream);
      break;
    default:
      e = amp ? agm::launch_combine_bwd<__half, float>(dout, S, B, n_tokens, d, top_k, n_experts, rows, stream)
              : agm::launch_combine_bwd<__half, __half>(dout, S, B, n_tokens, d, top_k, n_experts, rows, stream);
  }
  if (e != cudaSuccess) return agm::cuda_fail(e, "combine_bwd");

  // 2. FC2 weight and bias gradients: dW2[e] [d, H] = dy_e^T h_e, db2 = colsum(dy)
  agm::BwdGemmArgs w2a;
  w2a.c = dw2;
  w2a.m = d;
  w2a.n = hidden;
  w2a.groups = n_experts;
  w2a.seg_start = S.seg_start;
  w2a.err = B.err;
  e = wgrad_any(dtype, amp, B.dy, S.h, rows, w2a, sms, pair_mode, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "wgrad fc2");
  // 3. FC2 input gradient through the ReLU: dh = (dy @ W2[e]) * (h > 0)
  agm::BwdGemmArgs d2;
  d2.c = B.dh;
  d2.ldc = hidden;
  d2.c_rows = rows;
  d2.n = hidden;
  d2.k = d;
  d2.groups = n_experts;
  d2.tile_group = S.tile_expert;
  d2.num_tiles = S.num_tiles;
  d2.max_tiles = max_tiles;
  if (dtype == AGM_F32) {
    d2.aux = S.h;  // SIMT path: the ReLU mask from h, db1 from a column-sum pass
    d2.ld_aux = hidden;
  } else {
    d2.aux_bits = S.relu_bits;
    d2.ld_aux_bits = rows;
    d2.col_part = B.dh_part;  // db1 partials from the epilogue
  }
  d2.err = B.err;
  e = dgrad_any(dtype, pair_rows, B.dy, rows, w2, d2, true, sms, pair_mode, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "dgrad fc2");
  // 4. bias gradients (dy is still intact: dgrad wrote dh)
  e = colsum(B.dy, d, S.seg_start, n_experts, db2);
  if (e != cudaSuccess) return agm::cuda_fail(e, "db2");
  e = dtype == AGM_F32 ? colsum(B.dh, hidden, S.seg_start, n_experts, db1)
                       : tile_parts(B.dh_part, S.seg_start, n_experts, hidden, db1);
  if (e != cudaSuccess) return agm::cuda_fail(e, "db1");
  // 5. FC1 weight gradient: dW1[e] [H, d] = dh_e^T x_perm_e
  agm::BwdGemmArgs w1a = w2a;
  w1a.c = dw1;
  w1a.m = hidden;
  w1a.n = d;
  e = wgrad_any(dtype, amp, B.dh, S.x_perm, rows, w1a, sms, pair_mode, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "wgrad fc1");
  // 6. FC1 input gradient: dx_perm = dh @ W1[e], into dy's buffer
  agm::BwdGemmArgs d1 = d2;
  d1.c = B.dy;
  d1.ldc = d;
  d1.n = d;
  d1.k = hidden;
  d1.aux = nullptr;
  d1.aux_bits = nullptr;
  d1.col_part = nullptr;
  e = dgrad_any(dtype, pair_rows, B.dh, rows, w1, d1, false, sms, pair_mode, stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "dgrad fc1");

  // 7. shared experts: one dense segment of npad rows each, gradient ds
  //    (agillm41.py:4381-4387: s = shared[0](x) + shared[1](x) + ..., out += s)
  const int xs = agm::esize(x_dtype);
  if (n_shared > 0) {
    e = colsum(B.ds, d, B.dense_seg, 1, dsb2);  // the same for every shared expert
    for (int s = 1; s < n_shared && e == cudaSuccess; ++s)
      e = cudaMemcpyAsync(at(dsb2, static_cast<size_t>(xs) * s * d), dsb2, static_cast<size_t>(xs) * d,
                          cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared db2");
  }
  for (int s = 0; s < n_shared; ++s) {
    const void* hs = at(S.h_sh, static_cast<size_t>(eb) * s * npad * Hs);
    agm::BwdGemmArgs sw2;
    sw2.c = at(dws2, static_cast<size_t>(xs) * s * d * Hs);
    sw2.m = d;
    sw2.n = Hs;
    sw2.groups = 1;
    sw2.seg_start = B.dense_seg;
    sw2.err = B.err;
    e = wgrad_any(dtype, amp, B.ds, hs, npad, sw2, sms, pair_mode, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared wgrad fc2");
    agm::BwdGemmArgs sd2;
    sd2.c = B.dh_sh;
    sd2.ldc = Hs;
    sd2.c_rows = npad;
    sd2.n = Hs;
    sd2.k = d;
    sd2.groups = 1;
    sd2.max_tiles = static_cast<int>(npad / AGM_TILE_M);
    if (dtype == AGM_F32) {
      sd2.aux = hs;
      sd2.ld_aux = Hs;
    } else {
      sd2.aux_bits = S.bits_sh + static_cast<int64_t>(s) * ((Hs + 31) / 32) * npad;
      sd2.ld_aux_bits = npad;
      sd2.col_part = B.dhs_part;
    }
    sd2.err = B.err;
    e = dgrad_any(dtype, true, B.ds, npad, at(ws2, static_cast<size_t>(eb) * s * d * Hs), sd2, true, sms, pair_mode,
                  stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared dgrad fc2");
    void* db1s = at(dsb1, static_cast<size_t>(xs) * s * Hs);
    e = dtype == AGM_F32 ? colsum(B.dh_sh, Hs, B.dense_seg, 1, db1s) : tile_parts(B.dhs_part, B.dense_seg, 1, Hs, db1s);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared db1");
    agm::BwdGemmArgs sw1 = sw2;
    sw1.c = at(dws1, static_cast<size_t>(xs) * s * Hs * d);
    sw1.m = Hs;
    sw1.n = d;
    e = wgrad_any(dtype, amp, B.dh_sh, S.xb, npad, sw1, sms, pair_mode, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared wgrad fc1");
    agm::BwdGemmArgs sd1 = sd2;
    sd1.c = at(B.dx_sh, static_cast<size_t>(eb) * s * npad * d);
    sd1.ldc = d;
    sd1.n = d;
    sd1.k = Hs;
    sd1.aux = nullptr;
    sd1.aux_bits = nullptr;
    sd1.col_part = nullptr;
    e = dgrad_any(dtype, true, B.dh_sh, npad, at(ws1, static_cast<size_t>(eb) * s * Hs * d), sd1, false, sms,
                  pair_mode, stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "shared dgrad fc1");
  }

  // 8. router weight gradient: dWr = dl^T x
  switch (dtype) {
    case AGM_F32: e = agm::launch_router_wgrad<float, float>(B, S, n_tokens, d, top_k, n_experts, dw_router, stream); break;
    case AGM_BF16:
      e = amp ? agm::launch_router_wgrad<__nv_bfloat16, float>(B, S, n_tokens, d, top_k, n_experts, dw_router, stream)
              : agm::launch_router_wgrad<__nv_bfloat16, __nv_bfloat16>(B, S, n_tokens, d, top_k, n_experts, dw_router,
                                                                       stream);
      break;
    default:
      e = amp ? agm::launch_router_wgrad<__half, float>(B, S, n_tokens, d, top_k, n_experts, dw_router, stream)
              : agm::launch_router_wgrad<__half, __half>(B, S, n_tokens, d, top_k, n_experts, dw_router, stream);
  }
  if (e != cudaSuccess) return agm::cuda_fail(e, "router wgrad");
  // 9. input gradient
  switch (dtype) {
    case AGM_F32:
      e = agm::launch_dx<float, float>(B, S, w_router, n_tokens, d, top_k, n_experts, n_shared, dx, stream);
      break;
    case AGM_BF16:
      e = amp ? agm::launch_dx<__nv_bfloat16, float>(B, S, w_router, n_tokens, d, top_k, n_experts, n_shared, dx,
                                                     stream)
              : agm::launch_dx<__nv_bfloat16, __nv_bfloat16>(B, S, w_router, n_tokens, d, top_k, n_experts, n_shared,
                                                             dx, stream);
      break;
    default:
      e = amp ? agm::launch_dx<__half, float>(B, S, w_router, n_tokens, d, top_k, n_experts, n_shared, dx, stream)
              : agm::launch_dx<__half, __half>(B, S, w_router, n_tokens, d, top_k, n_experts, n_shared, dx, stream);
  }
  return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "dx");
}

// ---------------------------------------------------------------------------
// Auxiliary router losses (agillm41.py:4463-4492).
// ---------------------------------------------------------------------------
static int check_aux_args(int dtype, int64_t n, int d, int E) {
  if (!agm::esize(dtype)) return agm::fail(AGM_ERR_ARG, "dtype must be AGM_F32, AGM_BF16 or AGM_F16");
  if (n < 0 || n > (int64_t(1) << 31) - 1) return agm::fail(AGM_ERR_ARG, "n_tokens out of range");
  if (d <= 0 || d % 8) return agm::fail(AGM_ERR_ARG, "d must be a positive multiple of 8");
  if (E < 1 || E > AGM_MAX_EXPERTS) return agm::fail(AGM_ERR_UNSUPPORTED, "n_experts must be in [1, 16]");
  if (dtype != AGM_F32 && !agm::router_tc_supported(d))
    return agm::fail(AGM_ERR_UNSUPPORTED, "the tensor-core router does not support this d");
  if (dtype == AGM_F32 && agm::router_smem_bytes(d, E) > 227 * 1024)
    return agm::fail(AGM_ERR_UNSUPPORTED, "router weight does not fit in shared memory for this d");
  return AGM_OK;
}

size_t agm_moe_aux_saved_bytes(int64_t n_tokens, int n_experts, int dtype) {
  const int eb = agm::esize(dtype);
  if (!eb || n_tokens < 0 || n_experts < 1) return 0;
  return agm::carve_aux(nullptr, n_tokens, n_experts, eb).bytes;
}

size_t agm_moe_aux_backward_workspace_bytes(int64_t n_tokens, int d, int dtype) {
  const int eb = agm::esize(dtype);
  if (!eb || n_tokens < 0 || d <= 0) return 0;
  return agm::carve_aux_bwd(nullptr, n_tokens, d, eb).bytes;
}

int agm_moe_aux_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, const void* w_router,
                        double aux_coef, double z_coef, float* loss_out, void* saved, size_t saved_bytes, int flags,
                        void* stream_) {
  int rc = check_aux_args(dtype, n_tokens, d, n_experts);
  if (rc) return rc;
  if ((n_tokens > 0 && !x) || !w_router || !loss_out || !saved) return agm::fail(AGM_ERR_ARG, "null pointer");
  if (!agm::al16(x) || !agm::al16(w_router) || !agm::al16(saved))
    return agm::fail(AGM_ERR_ARG, "x, w_router and saved must be 16-byte aligned");
  const int eb = agm::esize(dtype);
  agm::AuxSaved A = agm::carve_aux(saved, n_tokens, n_experts, eb);
  if (A.bytes > saved_bytes) return agm::fail(AGM_ERR_WORKSPACE, "saved-state buffer too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PdlScope pdl_scope(!(flags & AGM_FLAG_NO_PDL));
  cudaError_t e = cudaMemsetAsync(A.err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return agm::cuda_fail(e, "memset");
  if (n_tokens > 0) {
    e = agm::router_topk(dtype, x, w_router, n_tokens, d, n_experts, 1, 1, nullptr, A.logits, A.idx, A.gates,
                         A.block_hist, A.err, agm::sm_count(), stream);
    if (e != cudaSuccess) return agm::cuda_fail(e, "router");
  }
  // The reference multiplies by the Python product aux_coef * num_experts.
  const float c_lb = static_cast<float>(aux_coef * n_experts);
  e = agm::launch_aux_forward(A, n_tokens, n_experts, c_lb, static_cast<float>(z_coef), aux_coef > 0, z_coef > 0,
                              loss_out, stream);
  return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "aux loss");
}

int agm_moe_aux_backward(const float* dloss, const void* x, int dtype, int64_t n_tokens, int d, int n_experts,
                         const void* saved, size_t saved_bytes, void* dw_router, void* workspace,
                         size_t workspace_bytes, int flags, void* stream_) {
  int rc = check_aux_args(dtype, n_tokens, d, n_experts);
  if (rc) return rc;
  if (!dloss || !saved || !dw_router || (n_tokens > 0 && (!x || !workspace)))
    return agm::fail(AGM_ERR_ARG, "null pointer");
  if (!agm::al16(x) || !agm::al16(saved) || !agm::al16(dw_router) || !agm::al16(workspace))
    return agm::fail(AGM_ERR_ARG, "x, saved, dw_router and workspace must be 16-byte aligned");
  const int eb = agm::esize(dtype);
  agm::AuxSaved A = agm::carve_aux(const_cast<void*>(saved), n_tokens, n_experts, eb);
  if (A.bytes > saved_bytes) return agm::fail(AGM_ERR_WORKSPACE, "saved-state buffer too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  cudaError_t e;
  if (n_tokens == 0) {
    // No tokens: the router weight's gradient is an empty sum.
    e = cudaMemsetAsync(dw_router, 0, static_cast<size_t>(eb) * n_experts * d, stream);
    return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "memset");
  }
  agm::AuxBwd B = agm::carve_aux_bwd(workspace, n_tokens, d, eb);
  if (B.bytes > workspace_bytes) return agm::fail(AGM_ERR_WORKSPACE, "workspace too small");
  agm::PdlScope pdl_scope(!(flags & AGM_FLAG_NO_PDL));
  switch (dtype) {
    case AGM_F32: e = agm::launch_aux_backward<float>(A, B, dloss, x, n_tokens, d, n_experts, dw_router, stream); break;
    case AGM_BF16:
      e = agm::launch_aux_backward<__nv_bfloat16>(A, B, dloss, x, n_tokens, d, n_experts, dw_router, stream);
      break;
    default: e = agm::launch_aux_backward<__half>(A, B, dloss, x, n_tokens, d, n_experts, dw_router, stream);
  }
  return e == cudaSuccess ? AGM_OK : agm::cuda_fail(e, "aux loss backward");
}

}  // extern "C"
