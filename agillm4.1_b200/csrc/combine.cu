// K4: gate-weighted combine back to token order (+ shared experts).
//
// Replaces agillm41.py:4420-4430:
//   out = zeros_like(flat)
//   for rank: out.index_add_(0, rows, expert(x[rows]) * w[rows])   (4428)
//   out = out + (shared[0](flat) + shared[1](flat) + ...)          (4429-4430)
// In bf16/fp16 mode every op rounds to the activation dtype: the product
// y*w, each index_add_ accumulation (rank 0 first, then rank 1, ...), each
// shared-expert sum and the final add. This kernel keeps exactly that chain
// (fp32 arithmetic, rounded to T after every op), so with identical expert
// outputs it reproduces the reference bit for bit.
//
// Layout: a warp per token (grid-stride); lanes stream 16-byte chunks of the
// k gathered rows of y_perm and write the token's output row once.
#include "common.cuh"
#include "kernels.h"

namespace agm {

// Rows up to kMaxChunks x 32 x 16 bytes keep every chunk of the k gathered
// rows in registers (all loads issued before any use); longer rows loop.
constexpr int kMaxChunks = 5;

template <typename T>
__device__ __forceinline__ void load8(const uint4& u, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    unpack8<T>(u, f);
  }
}

template <typename T>
__device__ __forceinline__ uint4 store8(const float (&acc)[8]) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                      __float_as_uint(acc[3]));
  } else {
    return make_uint4(pack2<T>(acc[0], acc[1]), pack2<T>(acc[2], acc[3]), pack2<T>(acc[4], acc[5]),
                      pack2<T>(acc[6], acc[7]));
  }
}

// out chunk = ((0 + round(y_0 g_0)) + round(y_1 g_1) + ...) [+ shared sum], each
// op rounded to T. __fmul_rn/__fadd_rn are never contracted into an FMA, so
// the product is rounded on its own as in the reference's `y * w` tensor.
// 16-bit types: the same chain on packed pairs. For bf16/fp16 operands a
// correctly rounded 16-bit multiply or add equals the fp32 operation followed
// by one rounding (the fp32 product is exact; an fp32 sum can only round where
// the smaller addend is below half a 16-bit ulp of the larger), and the _rn
// intrinsics are never contracted into an FMA.
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  __device__ __forceinline__ static V mul(V a, V b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static V add(V a, V b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static V splat(float g) { return __float2bfloat162_rn(g); }
  __device__ __forceinline__ static V zero() { return __float2bfloat162_rn(0.f); }
};
template <> struct Pair<__half> {
  using V = __half2;
  __device__ __forceinline__ static V mul(V a, V b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static V add(V a, V b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static V splat(float g) { return __float2half2_rn(g); }
  __device__ __forceinline__ static V zero() { return __float2half2_rn(0.f); }
};

template <typename T, int K_MAX>
__device__ __forceinline__ uint4 combine_chunk16(const uint4 (&v)[K_MAX], const float (&g)[K_MAX], int k,
                                                 const T* __restrict__ shared_y, int n_shared,
                                                 int64_t shared_stride, const T* __restrict__ residual, int64_t tok,
                                                 int d, int c) {
  using P = Pair<T>;
  using V = typename P::V;
  V acc[4] = {P::zero(), P::zero(), P::zero(), P::zero()};
#pragma unroll
  for (int r = 0; r < K_MAX; ++r) {
    if (r < k) {
      const V gg = P::splat(g[r]);  // exact: g is a T value
      const V* y = reinterpret_cast<const V*>(&v[r]);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = P::add(acc[j], P::mul(y[j], gg));
    }
  }
  if (n_shared > 0) {
    V s[4];
    for (int si = 0; si < n_shared; ++si) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(shared_y + si * shared_stride + tok * d) + c);
      const V* f = reinterpret_cast<const V*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] = (si == 0) ? f[j] : P::add(s[j], f[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = P::add(acc[j], s[j]);
  }
  if (residual) {  // Block: x + ff(ln2(x)), agillm41.py:4547
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(residual + tok * d) + c);
    const V* f = reinterpret_cast<const V*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = P::add(f[j], acc[j]);
  }
  uint4 o;
  o.x = *reinterpret_cast<uint32_t*>(&acc[0]);
  o.y = *reinterpret_cast<uint32_t*>(&acc[1]);
  o.z = *reinterpret_cast<uint32_t*>(&acc[2]);
  o.w = *reinterpret_cast<uint32_t*>(&acc[3]);
  return o;
}

template <typename T, int K_MAX>
__device__ __forceinline__ uint4 combine_chunk(const uint4 (&v)[K_MAX], const float (&g)[K_MAX], int k,
                                               const T* __restrict__ shared_y, int n_shared,
                                               int64_t shared_stride, const T* __restrict__ residual, int64_t tok,
                                               int d, int c) {
  if constexpr (sizeof(T) == 2) {
    return combine_chunk16<T, K_MAX>(v, g, k, shared_y, n_shared, shared_stride, residual, tok, d, c);
  }
  constexpr int CH = 16 / sizeof(T);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int r = 0; r < K_MAX; ++r) {
    if (r < k) {
      float f[8];
      load8<T>(v[r], f);
#pragma unroll
      for (int j = 0; j < CH; ++j) acc[j] = round_to<T>(__fadd_rn(acc[j], round_to<T>(__fmul_rn(f[j], g[r]))));
    }
  }
  if (n_shared > 0) {
    float s[8];
    for (int si = 0; si < n_shared; ++si) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(shared_y + si * shared_stride + tok * d) + c);
      float f[8];
      load8<T>(u, f);
#pragma unroll
      for (int j = 0; j < CH; ++j) s[j] = (si == 0) ? f[j] : round_to<T>(__fadd_rn(s[j], f[j]));
    }
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[j] = round_to<T>(__fadd_rn(acc[j], s[j]));
  }
  if (residual) {
    float f[8];
    load8<T>(__ldg(reinterpret_cast<const uint4*>(residual + tok * d) + c), f);
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[j] = round_to<T>(__fadd_rn(f[j], acc[j]));
  }
  return store8<T>(acc);
}

// Source of the expert output row for permuted row p: the local y_perm.
struct LocalY {
  const uint4* base;
  int nchunk;
  __device__ __forceinline__ const uint4* row(int64_t p) const { return base + p * nchunk; }
  __device__ __forceinline__ static uint4 load(const uint4* p) { return __ldg(p); }
};

template <typename T, int K_MAX, class Src>
__global__ void __launch_bounds__(256) combine_kernel(Src ysrc, const int32_t* __restrict__ row_of,
                                                      const T* __restrict__ gates, int64_t n_tokens, int d, int k,
                                                      const T* __restrict__ shared_y, int n_shared,
                                                      int64_t shared_stride, const T* __restrict__ residual,
                                                      T* __restrict__ out) {
  constexpr int CH = 16 / sizeof(T);
  const int nchunk = d / CH;
  const int lane = lane_id();
  pdl_wait();
  pdl_trigger();
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t tok = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp_id(); tok < n_tokens;
       tok += warps_total) {
    const uint4* src[K_MAX];
    float g[K_MAX];
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) {
      if (r < k) {
        src[r] = ysrc.row(row_of[tok * k + r]);
        g[r] = Traits<T>::to_f(gates[tok * k + r]);
      } else {
        src[r] = nullptr;
        g[r] = 0.f;
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + tok * d);
    bool done = false;
    if constexpr (K_MAX <= 4) {
      if (nchunk <= 32 * kMaxChunks) {
      done = true;
      uint4 v[kMaxChunks][K_MAX];
#pragma unroll
      for (int j = 0; j < kMaxChunks; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunk) {
#pragma unroll
          for (int r = 0; r < K_MAX; ++r)
            if (r < k) v[j][r] = src[r] ? Src::load(src[r] + c) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int j = 0; j < kMaxChunks; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunk)
          dst[c] = combine_chunk<T, K_MAX>(v[j], g, k, shared_y, n_shared, shared_stride, residual, tok, d, c);
      }
      }
    }
    if (!done) {
      for (int c = lane; c < nchunk; c += 32) {
        uint4 v[K_MAX];
#pragma unroll
        for (int r = 0; r < K_MAX; ++r)
          if (r < k) v[r] = src[r] ? Src::load(src[r] + c) : make_uint4(0, 0, 0, 0);
        dst[c] = combine_chunk<T, K_MAX>(v, g, k, shared_y, n_shared, shared_stride, residual, tok, d, c);
      }
    }
  }
}

template <typename T, class Src>
static cudaError_t launch_combine(Src ysrc, const int32_t* row_of, const void* gates, int64_t n, int d, int k,
                                  const void* shared_y, int n_shared, int64_t shared_stride, const void* residual,
                                  void* out, int num_sms, cudaStream_t stream) {
  const int64_t blocks = std::min<int64_t>((n + 7) / 8, static_cast<int64_t>(num_sms) * 8);
  if (blocks <= 0) return cudaSuccess;
  const T* gs = static_cast<const T*>(gates);
  const T* sh = static_cast<const T*>(shared_y);
  const T* res = static_cast<const T*>(residual);
  T* o = static_cast<T*>(out);
  const unsigned g = static_cast<unsigned>(blocks);
  if (k <= 2)
    return launch_kernel(combine_kernel<T, 2, Src>, dim3(g), dim3(256), 0, stream, ysrc, row_of, gs, n, d, k, sh,
                         n_shared, shared_stride, res, o);
  if (k <= 4)
    return launch_kernel(combine_kernel<T, 4, Src>, dim3(g), dim3(256), 0, stream, ysrc, row_of, gs, n, d, k, sh,
                         n_shared, shared_stride, res, o);
  return launch_kernel(combine_kernel<T, 16, Src>, dim3(g), dim3(256), 0, stream, ysrc, row_of, gs, n, d, k, sh,
                       n_shared, shared_stride, res, o);
}

template <typename T>
static cudaError_t combine_local(const void* y, const int32_t* row_of, const void* gates, int64_t n, int d, int k,
                                 const void* shared_y, int n_shared, int64_t shared_stride, const void* residual,
                                 void* out, int num_sms, cudaStream_t stream) {
  LocalY src{static_cast<const uint4*>(y), static_cast<int>(d * sizeof(T) / 16)};
  return launch_combine<T>(src, row_of, gates, n, d, k, shared_y, n_shared, shared_stride, residual, out, num_sms,
                           stream);
}

cudaError_t combine(int dtype, const void* y, const int32_t* row_of, const void* gates, int64_t n, int d, int k,
                    const void* shared_y, int n_shared, int64_t shared_stride, const void* residual, void* out,
                    int num_sms, cudaStream_t stream) {
  switch (dtype) {
    case AGM_F32:
      return combine_local<float>(y, row_of, gates, n, d, k, shared_y, n_shared, shared_stride, residual, out,
                                  num_sms, stream);
    case AGM_BF16:
      return combine_local<__nv_bfloat16>(y, row_of, gates, n, d, k, shared_y, n_shared, shared_stride, residual,
                                          out, num_sms, stream);
    case AGM_F16:
      return combine_local<__half>(y, row_of, gates, n, d, k, shared_y, n_shared, shared_stride, residual, out,
                                   num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
