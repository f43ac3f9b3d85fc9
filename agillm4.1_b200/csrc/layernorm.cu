// LayerNorm at the Block boundary, and the Block's whole FFN half.
//
// The reference's Block computes `x + self.ff(self.ln2(x))` (agillm41.py:4547;
// with a KV cache `x + y + ff(ln2(x + y))`, 4543). torch's LayerNorm over the
// 73,728 x 1280 bf16 rows of the MoE workload runs at about a quarter of HBM
// bandwidth (measured 0.25 ms, a tenth of that FFN half). This file provides
// the LayerNorm as an HBM-bound kernel and the FFN half as one entry point:
// LayerNorm into the workspace, then agm_moe_forward with the residual added
// in its combine.
//
// Kernel: one warp per row, persistent CTAs walking the rows. A lane holds
// the row's 16-byte vectors lane + 32 j (j < VPL) packed in registers, in
// one of two buffers used in turn, so each warp keeps two rows in flight.
// The affine weight and bias sit in shared memory as fp32 float4 planes,
// staged once per CTA, so their reads are conflict-free 16-byte loads (with
// scalar loads at the lanes' 32-byte stride, an 8-way bank conflict made the
// kernel latency-bound at half of HBM bandwidth). Statistics in fp32:
// mean = sum(x) / d, then the variance as the mean of squared deviations
// from it (two passes over the registers, no cancellation),
// rstd = rsqrt(var + eps). Output y = (x - mean) * rstd * weight + bias,
// rounded once to the input dtype. torch's kernel uses a
// Welford reduction in a different order, so its mean and rstd can differ
// in the last fp32 bit and a normalised value by one unit in the last place
// of the output dtype.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace agm {

namespace {

constexpr int kLnWarps = 8;

template <typename T> struct LnVec;
template <> struct LnVec<float> {
  static constexpr int kElems = 4;
};
template <> struct LnVec<__nv_bfloat16> {
  static constexpr int kElems = 8;
};
template <> struct LnVec<__half> {
  static constexpr int kElems = 8;
};

template <typename T>
__device__ __forceinline__ void ln_unpack(const uint4& u, float (&f)[LnVec<T>::kElems]) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    unpack8<T>(u, f);
  }
}

template <typename T>
__device__ __forceinline__ uint4 ln_pack(const float (&f)[LnVec<T>::kElems]) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  } else {
    return make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row x of one warp, packed: lane holds the 16-byte vectors lane + 32 j.
template <typename T, int VPL>
__device__ __forceinline__ void ln_load_row(const T* __restrict__ x, int64_t row, int d, int lane, uint4 (&r)[VPL]) {
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * d);
  const int nvec = d / LnVec<T>::kElems;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int v = lane + 32 * j;
    r[j] = v < nvec ? __ldcs(xr + v) : make_uint4(0, 0, 0, 0);
  }
}

// Statistics and output of one row held packed in registers. The affine
// parameters are float4 planes in shared memory: plane h holds elements
// 4h .. 4h+3 of every 16-byte vector, so vector v's weights are
// w_s[h * nvec + v] (h < EV / 4) and a warp's 16-byte reads of one plane are
// contiguous (no bank conflicts).
template <typename T, int VPL>
__device__ __forceinline__ void ln_row(const uint4 (&r)[VPL], const float4* __restrict__ w_s,
                                       const float4* __restrict__ b_s, float eps, float inv_d, int d, int lane,
                                       uint4* __restrict__ orow) {
  constexpr int EV = LnVec<T>::kElems;
  const int nvec = d / EV;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    if (lane + 32 * j < nvec) {
      float f[EV];
      ln_unpack<T>(r[j], f);
#pragma unroll
      for (int e = 0; e < EV; ++e) s += f[e];
    }
  }
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    if (lane + 32 * j < nvec) {
      float f[EV];
      ln_unpack<T>(r[j], f);
#pragma unroll
      for (int e = 0; e < EV; ++e) {
        const float dv = f[e] - mean;
        q += dv * dv;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int v = lane + 32 * j;
    if (v < nvec) {
      float f[EV], y[EV], wv[EV], bv[EV];
      ln_unpack<T>(r[j], f);
#pragma unroll
      for (int h = 0; h < EV / 4; ++h) {
        const float4 w4 = w_s[h * nvec + v];
        const float4 b4 = b_s[h * nvec + v];
        wv[4 * h] = w4.x, wv[4 * h + 1] = w4.y, wv[4 * h + 2] = w4.z, wv[4 * h + 3] = w4.w;
        bv[4 * h] = b4.x, bv[4 * h + 1] = b4.y, bv[4 * h + 2] = b4.z, bv[4 * h + 3] = b4.w;
      }
#pragma unroll
      for (int e = 0; e < EV; ++e) y[e] = (f[e] - mean) * rstd * wv[e] + bv[e];
      orow[v] = ln_pack<T>(y);
    }
  }
}

template <typename T, int VPL>
__global__ void __launch_bounds__(32 * kLnWarps) layernorm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                   const T* __restrict__ b, float eps, int64_t n,
                                                                   int d, T* __restrict__ out) {
  constexpr int EV = LnVec<T>::kElems;
  extern __shared__ float4 ln_smem[];
  const int nvec = d / EV;
  float4* w_s = ln_smem;         // [EV / 4][nvec] the affine weight in fp32, in float4 planes
  float4* b_s = ln_smem + d / 4; // the bias, same layout
  const int lane = lane_id();
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const int v = i / EV, h = (i % EV) / 4, c = i % 4;
    reinterpret_cast<float*>(w_s + h * nvec + v)[c] = Traits<T>::to_f(w[i]);
    reinterpret_cast<float*>(b_s + h * nvec + v)[c] = Traits<T>::to_f(b[i]);
  }
  __syncthreads();
  const float inv_d = 1.0f / static_cast<float>(d);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLnWarps;
  int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarps + warp_id();
  // Two rows in flight per warp, in two register buffers used in turn: a
  // buffer is refilled (the row two strides on) as soon as its row is
  // written, so while the warp waits for one row the other is outstanding
  // too. (A copy from a prefetch buffer would wait for that buffer's loads
  // with nothing else outstanding.)
  uint4 ra[VPL], rb[VPL];
  if (row < n) ln_load_row<T, VPL>(x, row, d, lane, ra);
  if (row + stride < n) ln_load_row<T, VPL>(x, row + stride, d, lane, rb);
  for (; row < n; row += 2 * stride) {
    ln_row<T, VPL>(ra, w_s, b_s, eps, inv_d, d, lane, reinterpret_cast<uint4*>(out + row * d));
    if (row + 2 * stride < n) ln_load_row<T, VPL>(x, row + 2 * stride, d, lane, ra);
    if (row + stride >= n) break;
    ln_row<T, VPL>(rb, w_s, b_s, eps, inv_d, d, lane, reinterpret_cast<uint4*>(out + (row + stride) * d));
    if (row + 3 * stride < n) ln_load_row<T, VPL>(x, row + 3 * stride, d, lane, rb);
  }
}

template <typename T, int VPL>
cudaError_t launch_ln_vpl(const void* x, const void* w, const void* b, float eps, int64_t n, int d, void* out,
                          int num_sms, cudaStream_t stream) {
  const size_t smem = 2 * static_cast<size_t>(d) * sizeof(float);
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, layernorm_kernel<T, VPL>, 32 * kLnWarps,
                                                                smem);
  if (e != cudaSuccess) return e;
  // persistent: every resident CTA walks rows; no more CTAs than rows need
  const int64_t blocks_needed = (n + kLnWarps - 1) / kLnWarps;
  const int grid = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(blocks_needed, static_cast<int64_t>(std::max(per_sm, 1)) * num_sms)));
  return launch_kernel(layernorm_kernel<T, VPL>, dim3(grid), dim3(32 * kLnWarps), smem, stream,
                       static_cast<const T*>(x), static_cast<const T*>(w), static_cast<const T*>(b), eps, n, d,
                       static_cast<T*>(out));
}

template <typename T>
cudaError_t launch_ln(const void* x, const void* w, const void* b, float eps, int64_t n, int d, void* out,
                      int num_sms, cudaStream_t stream) {
  const int vpl = (d / LnVec<T>::kElems + 31) / 32;
  switch (vpl) {
    case 1: return launch_ln_vpl<T, 1>(x, w, b, eps, n, d, out, num_sms, stream);
    case 2: return launch_ln_vpl<T, 2>(x, w, b, eps, n, d, out, num_sms, stream);
    case 3: return launch_ln_vpl<T, 3>(x, w, b, eps, n, d, out, num_sms, stream);
    case 4: return launch_ln_vpl<T, 4>(x, w, b, eps, n, d, out, num_sms, stream);
    case 5: return launch_ln_vpl<T, 5>(x, w, b, eps, n, d, out, num_sms, stream);
    case 6: return launch_ln_vpl<T, 6>(x, w, b, eps, n, d, out, num_sms, stream);
    case 7: return launch_ln_vpl<T, 7>(x, w, b, eps, n, d, out, num_sms, stream);
    case 8: return launch_ln_vpl<T, 8>(x, w, b, eps, n, d, out, num_sms, stream);
    default: break;
  }
  // fp32 rows up to 1,536 elements (an fp32 residual stream of d = 1280 under autocast)
  if constexpr (sizeof(T) == 4) {
    switch (vpl) {
      case 9: return launch_ln_vpl<T, 9>(x, w, b, eps, n, d, out, num_sms, stream);
      case 10: return launch_ln_vpl<T, 10>(x, w, b, eps, n, d, out, num_sms, stream);
      case 11: return launch_ln_vpl<T, 11>(x, w, b, eps, n, d, out, num_sms, stream);
      case 12: return launch_ln_vpl<T, 12>(x, w, b, eps, n, d, out, num_sms, stream);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

int ln_fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int ln_elem_bytes(int dtype) { return dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16 ? 2 : 0); }

bool ln_aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int num_sms_cur() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

int64_t ln_round(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

cudaError_t layernorm(int dtype, const void* x, const void* w, const void* b, float eps, int64_t n, int d, void* out,
                      int num_sms, cudaStream_t stream) {
  switch (dtype) {
    case AGM_F32: return launch_ln<float>(x, w, b, eps, n, d, out, num_sms, stream);
    case AGM_BF16: return launch_ln<__nv_bfloat16>(x, w, b, eps, n, d, out, num_sms, stream);
    case AGM_F16: return launch_ln<__half>(x, w, b, eps, n, d, out, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace agm

extern "C" {

AGM_API int agm_layernorm(const void* x, const void* weight, const void* bias, float eps, int dtype, int64_t n_rows,
                          int d, void* out, void* stream) {
  const int eb = agm::ln_elem_bytes(dtype);
  if (!eb) return agm::ln_fail(AGM_ERR_ARG, "agm_layernorm: dtype must be AGM_F32, AGM_BF16 or AGM_F16");
  if (n_rows < 0) return agm::ln_fail(AGM_ERR_ARG, "agm_layernorm: n_rows < 0");
  if (d <= 0 || (static_cast<int64_t>(d) * eb) % 16 || d > (eb == 4 ? 1536 : 2048))
    return agm::ln_fail(AGM_ERR_UNSUPPORTED, "agm_layernorm: d * sizeof(dtype) must be a multiple of 16 bytes, "
                                             "d at most 2048 (16-bit) or 1536 (fp32)");
  if (n_rows == 0) return AGM_OK;
  if (!x || !weight || !bias || !out) return agm::ln_fail(AGM_ERR_ARG, "agm_layernorm: null pointer argument");
  if (!agm::ln_aligned(x) || !agm::ln_aligned(weight) || !agm::ln_aligned(bias) || !agm::ln_aligned(out))
    return agm::ln_fail(AGM_ERR_ARG, "agm_layernorm: all tensors must be 16-byte aligned");
  cudaError_t e = agm::layernorm(dtype, x, weight, bias, eps, n_rows, d, out, agm::num_sms_cur(),
                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return agm::ln_fail(AGM_ERR_CUDA, std::string("agm_layernorm: ") + cudaGetErrorString(e));
  return AGM_OK;
}

AGM_API size_t agm_moe_block_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                                             int n_shared, int shared_hidden, int dtype) {
  const int eb = agm::ln_elem_bytes(dtype);
  const size_t fwd = agm_moe_workspace_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden, dtype);
  if (!eb || !fwd) return 0;
  return static_cast<size_t>(agm::ln_round(static_cast<int64_t>(fwd), 256) +
                             agm::ln_round(static_cast<int64_t>(eb) * std::max<int64_t>(n_tokens, 1) * d, 256));
}

AGM_API int agm_moe_block_forward(const void* x, const void* ln_weight, const void* ln_bias, float ln_eps, int dtype,
                                  int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                                  const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                                  int n_shared, int shared_hidden, const void* ws1, const void* sb1, const void* ws2,
                                  const void* sb2, void* out, void* workspace, size_t workspace_bytes, int flags,
                                  void* stream) {
  const int eb = agm::ln_elem_bytes(dtype);
  if (!eb) return agm::ln_fail(AGM_ERR_ARG, "agm_moe_block_forward: bad dtype");
  if (!workspace) return agm::ln_fail(AGM_ERR_ARG, "agm_moe_block_forward: null workspace");
  const size_t need = agm_moe_block_workspace_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden,
                                                    dtype);
  if (!need || need > workspace_bytes)
    return agm::ln_fail(AGM_ERR_WORKSPACE, "agm_moe_block_forward: workspace too small");
  if (x == out) return agm::ln_fail(AGM_ERR_ARG, "agm_moe_block_forward: out may not alias x");
  const size_t fwd = static_cast<size_t>(agm::ln_round(
      static_cast<int64_t>(agm_moe_workspace_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden,
                                                   dtype)),
      256));
  void* ln_out = static_cast<uint8_t*>(workspace) + fwd;
  int rc = agm_layernorm(x, ln_weight, ln_bias, ln_eps, dtype, n_tokens, d, ln_out, stream);
  if (rc != AGM_OK) return rc;
  // the forward's error word sits at the start of the workspace, as for agm_moe_forward
  return agm_moe_forward_residual(ln_out, x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, w1, b1, w2, b2,
                                  n_shared, shared_hidden, ws1, sb1, ws2, sb2, out, workspace, fwd, flags, stream);
}

}  // extern "C"
