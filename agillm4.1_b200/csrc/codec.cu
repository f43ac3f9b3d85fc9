// Tensor-state codec decode on the GPU: the payloads of the reference's
// tensor codec (agillm41.py:4858-5074, decoded by
// _agillm43_decode_tensor_state, agillm41.py:5076-5102) turned into weights
// in device memory, optionally applied to them the way the DBlock side-update
// consumer applies a decoded state (agillm41.py:6029-6046):
//
//   value  = payload                         (pack_kind "lossless" / "fp16")
//          = float(q) * scale                (pack_kind "int8_symmetric")
//          = float(q[r, c]) * float(s[r])    (pack_kind "int8_rowwise", the
//                                             row scales stored as fp16 or fp32)
//   src    = value rounded to the target's dtype   (`value.to(dtype=target.dtype)`)
//   target = src                             (copy_,  alpha >= 1)
//          = lerp(target, src, alpha)        (lerp_,  state update)
//          = target + alpha * src            (add_,   delta update)
//
// The host decompresses the payload (zstd or zlib, a CPU library) and copies
// the packed bytes to the device: 1 byte per int8 element crosses PCIe instead
// of the 4 of the reference's fp32 decode. This kernel then reads the packed
// bytes once and writes (or reads and writes) the target once: HBM-bound byte
// work, 16 elements per thread per step, grid-stride over the tensor.
#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace agm {
namespace {

constexpr int kCodecThreads = 256;
constexpr int kCodecVec = 16;  // elements per thread per step

// torch's lerp on CUDA (ATen/native/Lerp.h, opmath float): the small-weight
// form below |w| < 0.5, the end-anchored form above it.
__device__ __forceinline__ float lerp_f(float self, float end, float w) {
  return fabsf(w) < 0.5f ? self + w * (end - self) : end - (end - self) * (1.0f - w);
}

template <typename P>
__device__ __forceinline__ float packed_value(P v) {
  if constexpr (sizeof(P) == 1)
    return static_cast<float>(v);
  else
    return Traits<P>::to_f(v);
}

template <typename S>
__device__ __forceinline__ float scale_value(const S* s, int64_t row) {
  return Traits<S>::to_f(s[row]);
}

// KIND: AGM_CODEC_PLAIN (P = float / bf16 / fp16), AGM_CODEC_INT8,
// AGM_CODEC_INT8_ROWWISE (P = int8_t, S = the row-scale type).
template <int KIND, typename P, typename S, typename OutT, int MODE>
__device__ __forceinline__ void decode_one(const P* __restrict__ payload, int64_t i, int64_t cols, float scale,
                                           const S* __restrict__ row_scales, OutT* __restrict__ target, float alpha) {
  float v = packed_value<P>(payload[i]);
  if constexpr (KIND == AGM_CODEC_INT8) v = __fmul_rn(v, scale);
  if constexpr (KIND == AGM_CODEC_INT8_ROWWISE) v = __fmul_rn(v, scale_value<S>(row_scales, i / cols));
  const float src = round_to<OutT>(v);
  float t;
  if constexpr (MODE == AGM_APPLY_COPY) {
    t = src;
  } else {
    const float cur = Traits<OutT>::to_f(target[i]);
    t = MODE == AGM_APPLY_ADD ? cur + alpha * src : lerp_f(cur, src, alpha);
  }
  target[i] = Traits<OutT>::from_f(t);
}

// 16 consecutive elements of type E as raw 16-byte words (sizeof(E) words):
// loads are issued into these, the conversion to fp32 waits until the math.
template <typename E>
struct Raw16 {
  uint4 w[sizeof(E)];
};

template <typename E>
__device__ __forceinline__ void load_raw(const E* __restrict__ p, int64_t i0, Raw16<E>& r, bool nc) {
#pragma unroll
  for (int q = 0; q < static_cast<int>(sizeof(E)); ++q)
    r.w[q] = nc ? __ldg(reinterpret_cast<const uint4*>(p + i0) + q) : reinterpret_cast<const uint4*>(p + i0)[q];
}

template <typename E>
__device__ __forceinline__ void to_float(const Raw16<E>& r, float (&v)[kCodecVec]) {
  if constexpr (sizeof(E) == 1) {
    const uint32_t w[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int j = 0; j < kCodecVec; ++j)
      v[j] = static_cast<float>(static_cast<int8_t>(static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)))));
  } else if constexpr (sizeof(E) == 2) {
    float f[8];
    unpack8<E>(r.w[0], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = f[j];
    unpack8<E>(r.w[1], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 + j] = f[j];
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[4 * q] = __uint_as_float(r.w[q].x); v[4 * q + 1] = __uint_as_float(r.w[q].y);
      v[4 * q + 2] = __uint_as_float(r.w[q].z); v[4 * q + 3] = __uint_as_float(r.w[q].w);
    }
  }
}

template <typename OutT>
__device__ __forceinline__ void store_target(OutT* __restrict__ target, int64_t i0, const float (&t)[kCodecVec]) {
  if constexpr (sizeof(OutT) == 2) {
    reinterpret_cast<uint4*>(target + i0)[0] =
        make_uint4(pack2<OutT>(t[0], t[1]), pack2<OutT>(t[2], t[3]), pack2<OutT>(t[4], t[5]), pack2<OutT>(t[6], t[7]));
    reinterpret_cast<uint4*>(target + i0)[1] = make_uint4(pack2<OutT>(t[8], t[9]), pack2<OutT>(t[10], t[11]),
                                                          pack2<OutT>(t[12], t[13]), pack2<OutT>(t[14], t[15]));
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<float4*>(target + i0)[q] = make_float4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
  }
}

// The warp's 32 lanes hold the outputs of 32 consecutive groups starting at
// dst (lane l: elements [16 l, 16 l + 16)). They go through `stg` (32 x
// sizeof(OutT) 16-byte chunks, XOR-swizzled by lane so the writes spread over
// the banks) and out as sizeof(OutT) contiguous 512-byte warp stores. Written
// directly, each 16-byte store of a 64-byte-strided group output half-fills
// the 32-byte sectors it touches: on a B200 an int8 -> fp32 decode ran at
// 3.2 TB/s that way and at 5.0 TB/s through the staging. Same bytes as
// store_target.
template <typename OutT>
__device__ __forceinline__ void store_warp_staged(uint4* stg, OutT* __restrict__ dst, const float (&t)[kCodecVec],
                                                  int lane) {
  constexpr int CQ = sizeof(OutT);  // 16-byte chunks per group
  uint4 w[CQ];
  if constexpr (CQ == 2) {
    w[0] = make_uint4(pack2<OutT>(t[0], t[1]), pack2<OutT>(t[2], t[3]), pack2<OutT>(t[4], t[5]), pack2<OutT>(t[6], t[7]));
    w[1] = make_uint4(pack2<OutT>(t[8], t[9]), pack2<OutT>(t[10], t[11]), pack2<OutT>(t[12], t[13]),
                      pack2<OutT>(t[14], t[15]));
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w[q] = make_uint4(__float_as_uint(t[4 * q]), __float_as_uint(t[4 * q + 1]), __float_as_uint(t[4 * q + 2]),
                        __float_as_uint(t[4 * q + 3]));
  }
  __syncwarp();  // the previous use of stg has been read
#pragma unroll
  for (int q = 0; q < CQ; ++q) stg[lane * CQ + (q ^ (lane & (CQ - 1)))] = w[q];
  __syncwarp();
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < CQ; ++j) {
    const int c = j * 32 + lane, g = c / CQ, q = c % CQ;
    d[c] = stg[g * CQ + (q ^ (g & (CQ - 1)))];
  }
}

// Vectorised path: U groups of 16 consecutive elements per thread per step
// (U = 4 for int8 payloads: 64 B of loads in flight per thread), all loads
// (payload, row scale, and for lerp/add the target) issued before any math.
// ROW_VEC: row-wise scales with cols a multiple of 16, so one scale per group
// (found by a 32-bit division when n < 2^32).
template <int KIND, typename P, typename S, typename OutT, int MODE, bool ROW_VEC>
__device__ __forceinline__ void decode_vectors(const P* __restrict__ payload, int64_t n, int64_t cols, float scale,
                                               const S* __restrict__ row_scales, OutT* __restrict__ target,
                                               float alpha, int64_t tid, int64_t stride) {
  constexpr int U = sizeof(P) == 1 ? 4 : (sizeof(P) == 2 ? 2 : 1);
  const int64_t nvec = n / kCodecVec;
  const bool small = n < (int64_t(1) << 32);
  for (int64_t b0 = tid; b0 < nvec; b0 += stride * U) {
    Raw16<P> raw[U];
    Raw16<OutT> cur_raw[MODE == AGM_APPLY_COPY ? 1 : U];
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t b = b0 + u * stride;
      if (b < nvec) {
        const int64_t i0 = b * kCodecVec;
        load_raw<P>(payload, i0, raw[u], true);
        if constexpr (KIND == AGM_CODEC_INT8_ROWWISE && ROW_VEC) {
          const int64_t row = small ? static_cast<int64_t>(static_cast<uint32_t>(i0) / static_cast<uint32_t>(cols))
                                    : i0 / cols;
          sc[u] = scale_value<S>(row_scales, row);
        }
        if constexpr (MODE != AGM_APPLY_COPY) load_raw<OutT>(target, i0, cur_raw[u], false);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t b = b0 + u * stride;
      if (b >= nvec) continue;
      const int64_t i0 = b * kCodecVec;
      float v[kCodecVec];
      to_float<P>(raw[u], v);
      if constexpr (KIND == AGM_CODEC_INT8) {
#pragma unroll
        for (int j = 0; j < kCodecVec; ++j) v[j] = __fmul_rn(v[j], scale);
      }
      if constexpr (KIND == AGM_CODEC_INT8_ROWWISE) {
        if constexpr (ROW_VEC) {
#pragma unroll
          for (int j = 0; j < kCodecVec; ++j) v[j] = __fmul_rn(v[j], sc[u]);
        } else {
          // Rows shorter than, or not aligned to, the group: the scale
          // changes wherever a row starts inside it.
          int64_t row = i0 / cols;
          int64_t next = (row + 1) * cols;
          float s = scale_value<S>(row_scales, row);
#pragma unroll
          for (int j = 0; j < kCodecVec; ++j) {
            if (i0 + j >= next) {
              ++row;
              next += cols;
              s = scale_value<S>(row_scales, row);
            }
            v[j] = __fmul_rn(v[j], s);
          }
        }
      }
      float t[kCodecVec];
      if constexpr (MODE == AGM_APPLY_COPY) {
#pragma unroll
        for (int j = 0; j < kCodecVec; ++j) t[j] = round_to<OutT>(v[j]);
      } else {
        float cur[kCodecVec];
        to_float<OutT>(cur_raw[u], cur);
#pragma unroll
        for (int j = 0; j < kCodecVec; ++j) {
          const float src = round_to<OutT>(v[j]);
          t[j] = MODE == AGM_APPLY_ADD ? cur[j] + alpha * src : lerp_f(cur[j], src, alpha);
        }
      }
      store_target<OutT>(target, i0, t);
    }
  }
}

template <int KIND, typename P, typename S, typename OutT, int MODE>
__global__ void __launch_bounds__(kCodecThreads) codec_decode_kernel(const P* __restrict__ payload, int64_t n,
                                                                     int64_t cols, float scale,
                                                                     const S* __restrict__ row_scales,
                                                                     OutT* __restrict__ target, float alpha,
                                                                     int vec_ok) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kCodecThreads;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kCodecThreads + threadIdx.x;
  if (vec_ok) {
    if (KIND == AGM_CODEC_INT8_ROWWISE && cols % kCodecVec == 0)
      decode_vectors<KIND, P, S, OutT, MODE, true>(payload, n, cols, scale, row_scales, target, alpha, tid, stride);
    else
      decode_vectors<KIND, P, S, OutT, MODE, false>(payload, n, cols, scale, row_scales, target, alpha, tid, stride);
    for (int64_t i = n / kCodecVec * kCodecVec + tid; i < n; i += stride)
      decode_one<KIND, P, S, OutT, MODE>(payload, i, cols, scale, row_scales, target, alpha);
  } else {
    for (int64_t i = tid; i < n; i += stride)
      decode_one<KIND, P, S, OutT, MODE>(payload, i, cols, scale, row_scales, target, alpha);
  }
}

// ---------------------------------------------------------------------------
// Batched decode: up to kCodecBatch tensors of one signature (pack kind,
// payload / scale / target types, apply mode) in one launch. The tensors'
// 16-element groups are numbered one after the other (vec_begin holds the
// prefix sums); a thread finds its group's tensor by a scan of at most 16
// entries of the table, which stays in the kernel's parameter space
// (__grid_constant__). Every tensor is 16-byte aligned and, for row-wise
// scales, has rows of a multiple of 16 elements; the n % 16 tail elements of
// each tensor are decoded one per thread after the groups.
// ---------------------------------------------------------------------------
constexpr int kCodecBatch = 16;

struct CodecBatch {
  const void* payload[kCodecBatch];
  const void* scales[kCodecBatch];
  void* target[kCodecBatch];
  int64_t n[kCodecBatch];
  int64_t cols[kCodecBatch];
  int64_t vec_begin[kCodecBatch + 1];
  float scale[kCodecBatch];
  int count;
};

template <int KIND, typename P, typename S, typename OutT, int MODE>
__global__ void __launch_bounds__(kCodecThreads) codec_batch_kernel(const __grid_constant__ CodecBatch b,
                                                                    float alpha) {
  constexpr int U = sizeof(P) == 1 ? 4 : (sizeof(P) == 2 ? 2 : 1);
  __shared__ uint4 stg[kCodecThreads / 32][MODE == AGM_APPLY_COPY ? 32 * sizeof(OutT) : 1];
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kCodecThreads;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kCodecThreads + threadIdx.x;
  const int64_t total = b.vec_begin[b.count];
  // Copy mode: a warp-uniform loop (the warp's first lane decides), since the
  // staged store needs all 32 lanes; lanes past the end carry no group
  // (tt = -1).
  for (int64_t v0 = tid; (MODE == AGM_APPLY_COPY ? v0 - lane : v0) < total; v0 += stride * U) {
    Raw16<P> raw[U];
    Raw16<OutT> cur_raw[MODE == AGM_APPLY_COPY ? 1 : U];
    float sc[U];
    int tt[U];
    int64_t ii[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * stride;
      tt[u] = -1;
      if (v < total) {
        int t = 0;
        while (t + 1 < b.count && v >= b.vec_begin[t + 1]) ++t;
        const int64_t i0 = (v - b.vec_begin[t]) * kCodecVec;
        tt[u] = t;
        ii[u] = i0;
        load_raw<P>(static_cast<const P*>(b.payload[t]), i0, raw[u], true);
        if constexpr (KIND == AGM_CODEC_INT8_ROWWISE) {
          const int64_t cols = b.cols[t];
          const int64_t row = b.n[t] < (int64_t(1) << 32)
                                  ? static_cast<int64_t>(static_cast<uint32_t>(i0) / static_cast<uint32_t>(cols))
                                  : i0 / cols;
          sc[u] = scale_value<S>(static_cast<const S*>(b.scales[t]), row);
        } else {
          sc[u] = b.scale[t];
        }
        if constexpr (MODE != AGM_APPLY_COPY) load_raw<OutT>(static_cast<const OutT*>(b.target[t]), i0, cur_raw[u], false);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if constexpr (MODE != AGM_APPLY_COPY) {
        if (tt[u] < 0) continue;
      }
      float t[kCodecVec];
      if (tt[u] >= 0) {
        float v[kCodecVec];
        to_float<P>(raw[u], v);
        if constexpr (KIND != AGM_CODEC_PLAIN) {
#pragma unroll
          for (int j = 0; j < kCodecVec; ++j) v[j] = __fmul_rn(v[j], sc[u]);
        }
        if constexpr (MODE == AGM_APPLY_COPY) {
#pragma unroll
          for (int j = 0; j < kCodecVec; ++j) t[j] = round_to<OutT>(v[j]);
        } else {
          float cur[kCodecVec];
          to_float<OutT>(cur_raw[u], cur);
#pragma unroll
          for (int j = 0; j < kCodecVec; ++j) {
            const float src = round_to<OutT>(v[j]);
            t[j] = MODE == AGM_APPLY_ADD ? cur[j] + alpha * src : lerp_f(cur[j], src, alpha);
          }
        }
      }
      if constexpr (MODE == AGM_APPLY_COPY) {
        // The warp's groups are consecutive (v = v0 + u * stride, v0 = tid);
        // when all 32 belong to one tensor their outputs are one contiguous
        // run. (Copy mode only: lerp / add keep the target's old values live
        // too, and the staging would cost them half their occupancy.)
        const int t0 = __shfl_sync(0xffffffffu, tt[u], 0);
        if (__all_sync(0xffffffffu, tt[u] >= 0 && tt[u] == t0)) {
          store_warp_staged<OutT>(stg[threadIdx.x >> 5],
                                  static_cast<OutT*>(b.target[t0]) + __shfl_sync(0xffffffffu, ii[u], 0), t, lane);
          continue;
        }
      }
      if (tt[u] >= 0) store_target<OutT>(static_cast<OutT*>(b.target[tt[u]]), ii[u], t);
    }
  }
  for (int64_t j = tid; j < static_cast<int64_t>(b.count) * kCodecVec; j += stride) {
    const int t = static_cast<int>(j / kCodecVec);
    const int64_t i = b.n[t] / kCodecVec * kCodecVec + j % kCodecVec;
    if (i < b.n[t])
      decode_one<KIND, P, S, OutT, MODE>(static_cast<const P*>(b.payload[t]), i, b.cols[t], b.scale[t],
                                         static_cast<const S*>(b.scales[t]), static_cast<OutT*>(b.target[t]), alpha);
  }
}

template <int KIND, typename P, typename S, typename OutT, int MODE>
cudaError_t launch_batch(const CodecBatch& b, float alpha, int sms, cudaStream_t s) {
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, codec_batch_kernel<KIND, P, S, OutT, MODE>,
                                                                kCodecThreads, 0);
  if (e != cudaSuccess) return e;
  const int64_t want = (b.vec_begin[b.count] + kCodecThreads - 1) / kCodecThreads;
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * std::max(per_sm, 1))));
  codec_batch_kernel<KIND, P, S, OutT, MODE><<<grid, kCodecThreads, 0, s>>>(b, alpha);
  return cudaGetLastError();
}

template <int KIND, typename P, typename S, typename OutT>
cudaError_t batch_by_mode(int mode, const CodecBatch& b, float alpha, int sms, cudaStream_t s) {
  switch (mode) {
    case AGM_APPLY_COPY: return launch_batch<KIND, P, S, OutT, AGM_APPLY_COPY>(b, alpha, sms, s);
    case AGM_APPLY_LERP: return launch_batch<KIND, P, S, OutT, AGM_APPLY_LERP>(b, alpha, sms, s);
    default: return launch_batch<KIND, P, S, OutT, AGM_APPLY_ADD>(b, alpha, sms, s);
  }
}

template <int KIND, typename P, typename S>
cudaError_t batch_by_target(int target_dtype, int mode, const CodecBatch& b, float alpha, int sms, cudaStream_t s) {
  switch (target_dtype) {
    case AGM_F32: return batch_by_mode<KIND, P, S, float>(mode, b, alpha, sms, s);
    case AGM_BF16: return batch_by_mode<KIND, P, S, __nv_bfloat16>(mode, b, alpha, sms, s);
    default: return batch_by_mode<KIND, P, S, __half>(mode, b, alpha, sms, s);
  }
}

// One launch for a table of tensors sharing kind, packed / scale / target
// dtypes (checked by the caller).
cudaError_t launch_batch_any(int kind, int packed_dtype, int scales_dtype, int target_dtype, int mode,
                             const CodecBatch& b, float alpha, int sms, cudaStream_t s) {
  if (kind == AGM_CODEC_INT8) return batch_by_target<AGM_CODEC_INT8, int8_t, float>(target_dtype, mode, b, alpha, sms, s);
  if (kind == AGM_CODEC_INT8_ROWWISE)
    return scales_dtype == AGM_F16
               ? batch_by_target<AGM_CODEC_INT8_ROWWISE, int8_t, __half>(target_dtype, mode, b, alpha, sms, s)
               : batch_by_target<AGM_CODEC_INT8_ROWWISE, int8_t, float>(target_dtype, mode, b, alpha, sms, s);
  switch (packed_dtype) {
    case AGM_F32: return batch_by_target<AGM_CODEC_PLAIN, float, float>(target_dtype, mode, b, alpha, sms, s);
    case AGM_BF16: return batch_by_target<AGM_CODEC_PLAIN, __nv_bfloat16, float>(target_dtype, mode, b, alpha, sms, s);
    default: return batch_by_target<AGM_CODEC_PLAIN, __half, float>(target_dtype, mode, b, alpha, sms, s);
  }
}

template <int KIND, typename P, typename S, typename OutT, int MODE>
cudaError_t launch_decode(const void* payload, int64_t n, int64_t cols, float scale, const void* row_scales,
                          void* target, float alpha, bool vec_ok, int sms, cudaStream_t s) {
  // One wave of resident CTAs at most, each striding over the tensor.
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, codec_decode_kernel<KIND, P, S, OutT, MODE>,
                                                                kCodecThreads, 0);
  if (e != cudaSuccess) return e;
  const int64_t want = (n / (vec_ok ? kCodecVec : 1) + kCodecThreads - 1) / kCodecThreads;
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * std::max(per_sm, 1))));
  codec_decode_kernel<KIND, P, S, OutT, MODE><<<grid, kCodecThreads, 0, s>>>(
      static_cast<const P*>(payload), n, cols, scale, static_cast<const S*>(row_scales), static_cast<OutT*>(target),
      alpha, vec_ok ? 1 : 0);
  return cudaGetLastError();
}

template <int KIND, typename P, typename S, typename OutT>
cudaError_t by_mode(int mode, const void* payload, int64_t n, int64_t cols, float scale, const void* row_scales,
                    void* target, float alpha, bool vec_ok, int sms, cudaStream_t s) {
  switch (mode) {
    case AGM_APPLY_COPY:
      return launch_decode<KIND, P, S, OutT, AGM_APPLY_COPY>(payload, n, cols, scale, row_scales, target, alpha, vec_ok,
                                                             sms, s);
    case AGM_APPLY_LERP:
      return launch_decode<KIND, P, S, OutT, AGM_APPLY_LERP>(payload, n, cols, scale, row_scales, target, alpha, vec_ok,
                                                             sms, s);
    default:
      return launch_decode<KIND, P, S, OutT, AGM_APPLY_ADD>(payload, n, cols, scale, row_scales, target, alpha, vec_ok,
                                                            sms, s);
  }
}

template <int KIND, typename P, typename S>
cudaError_t by_target(int target_dtype, int mode, const void* payload, int64_t n, int64_t cols, float scale,
                      const void* row_scales, void* target, float alpha, bool vec_ok, int sms, cudaStream_t s) {
  switch (target_dtype) {
    case AGM_F32: return by_mode<KIND, P, S, float>(mode, payload, n, cols, scale, row_scales, target, alpha, vec_ok, sms, s);
    case AGM_BF16:
      return by_mode<KIND, P, S, __nv_bfloat16>(mode, payload, n, cols, scale, row_scales, target, alpha, vec_ok, sms, s);
    default: return by_mode<KIND, P, S, __half>(mode, payload, n, cols, scale, row_scales, target, alpha, vec_ok, sms, s);
  }
}

int codec_fail(int code, const char* msg) {
  set_last_error(std::string("agm_codec_decode: ") + msg);
  return code;
}

int dtype_bytes(int dtype) { return dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16) ? 2 : 0; }

// The argument checks of one tensor (AGM_OK, or the failure's code with the
// message set).
int check_tensor(const void* payload, int kind, int packed_dtype, int64_t n, int64_t cols, const void* row_scales,
                 int scales_dtype, const void* target, int target_dtype) {
  if (n < 0) return codec_fail(AGM_ERR_ARG, "n < 0");
  if (kind != AGM_CODEC_PLAIN && kind != AGM_CODEC_INT8 && kind != AGM_CODEC_INT8_ROWWISE)
    return codec_fail(AGM_ERR_ARG, "unknown pack kind");
  if (!dtype_bytes(target_dtype)) return codec_fail(AGM_ERR_ARG, "target dtype must be AGM_F32, AGM_BF16 or AGM_F16");
  if (kind == AGM_CODEC_PLAIN && !dtype_bytes(packed_dtype))
    return codec_fail(AGM_ERR_UNSUPPORTED, "lossless payloads must be fp32, bf16 or fp16");
  if (kind == AGM_CODEC_INT8_ROWWISE) {
    if (cols <= 0 || n % cols) return codec_fail(AGM_ERR_ARG, "cols must divide n for row-wise int8");
    if (scales_dtype != AGM_F32 && scales_dtype != AGM_F16)
      return codec_fail(AGM_ERR_ARG, "row scales must be AGM_F32 or AGM_F16");
    if (n > 0 && !row_scales) return codec_fail(AGM_ERR_ARG, "null row scales");
  }
  if (n == 0) return AGM_OK;
  if (!payload || !target) return codec_fail(AGM_ERR_ARG, "null pointer");
  const int pb = kind == AGM_CODEC_PLAIN ? dtype_bytes(packed_dtype) : 1;
  if (reinterpret_cast<uintptr_t>(payload) % pb || reinterpret_cast<uintptr_t>(target) % dtype_bytes(target_dtype))
    return codec_fail(AGM_ERR_ARG, "payload and target must be aligned to their element size");
  return AGM_OK;
}

}  // namespace
}  // namespace agm

extern "C" {

int agm_codec_decode(const void* payload, int kind, int packed_dtype, int64_t n, int64_t cols, float scale,
                     const void* row_scales, int scales_dtype, void* target, int target_dtype, int mode, float alpha,
                     void* stream_) {
  using namespace agm;
  if (n < 0) return codec_fail(AGM_ERR_ARG, "n < 0");
  if (kind != AGM_CODEC_PLAIN && kind != AGM_CODEC_INT8 && kind != AGM_CODEC_INT8_ROWWISE)
    return codec_fail(AGM_ERR_ARG, "unknown pack kind");
  if (mode != AGM_APPLY_COPY && mode != AGM_APPLY_LERP && mode != AGM_APPLY_ADD)
    return codec_fail(AGM_ERR_ARG, "unknown apply mode");
  if (!dtype_bytes(target_dtype)) return codec_fail(AGM_ERR_ARG, "target dtype must be AGM_F32, AGM_BF16 or AGM_F16");
  if (kind == AGM_CODEC_PLAIN && !dtype_bytes(packed_dtype))
    return codec_fail(AGM_ERR_UNSUPPORTED, "lossless payloads must be fp32, bf16 or fp16");
  if (kind == AGM_CODEC_INT8_ROWWISE) {
    if (cols <= 0 || n % cols) return codec_fail(AGM_ERR_ARG, "cols must divide n for row-wise int8");
    if (scales_dtype != AGM_F32 && scales_dtype != AGM_F16)
      return codec_fail(AGM_ERR_ARG, "row scales must be AGM_F32 or AGM_F16");
    if (n > 0 && !row_scales) return codec_fail(AGM_ERR_ARG, "null row scales");
  }
  if (n == 0) return AGM_OK;
  if (!payload || !target) return codec_fail(AGM_ERR_ARG, "null pointer");
  // Whole 16-byte vectors need 16-byte aligned payload and target.
  const uintptr_t pa = reinterpret_cast<uintptr_t>(payload), ta = reinterpret_cast<uintptr_t>(target);
  const int pb = kind == AGM_CODEC_PLAIN ? dtype_bytes(packed_dtype) : 1;
  const int tb = dtype_bytes(target_dtype);
  if (pa % pb || ta % tb) return codec_fail(AGM_ERR_ARG, "payload and target must be aligned to their element size");
  const bool vec_ok = (pa % 16 == 0) && (ta % 16 == 0);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  cudaError_t e;
  if (kind == AGM_CODEC_INT8) {
    e = by_target<AGM_CODEC_INT8, int8_t, float>(target_dtype, mode, payload, n, 1, scale, nullptr, target, alpha,
                                                 vec_ok, sms, s);
  } else if (kind == AGM_CODEC_INT8_ROWWISE) {
    e = scales_dtype == AGM_F16
            ? by_target<AGM_CODEC_INT8_ROWWISE, int8_t, __half>(target_dtype, mode, payload, n, cols, 1.f, row_scales,
                                                                target, alpha, vec_ok, sms, s)
            : by_target<AGM_CODEC_INT8_ROWWISE, int8_t, float>(target_dtype, mode, payload, n, cols, 1.f, row_scales,
                                                               target, alpha, vec_ok, sms, s);
  } else {
    switch (packed_dtype) {
      case AGM_F32:
        e = by_target<AGM_CODEC_PLAIN, float, float>(target_dtype, mode, payload, n, 1, 1.f, nullptr, target, alpha,
                                                     vec_ok, sms, s);
        break;
      case AGM_BF16:
        e = by_target<AGM_CODEC_PLAIN, __nv_bfloat16, float>(target_dtype, mode, payload, n, 1, 1.f, nullptr, target,
                                                             alpha, vec_ok, sms, s);
        break;
      default:
        e = by_target<AGM_CODEC_PLAIN, __half, float>(target_dtype, mode, payload, n, 1, 1.f, nullptr, target, alpha,
                                                      vec_ok, sms, s);
    }
  }
  if (e != cudaSuccess) {
    set_last_error(std::string("agm_codec_decode: ") + cudaGetErrorString(e));
    return AGM_ERR_CUDA;
  }
  return AGM_OK;
}

int agm_codec_decode_batch(const AgmCodecTensor* tensors, int count, int mode, float alpha, void* stream_) {
  using namespace agm;
  if (count < 0 || (count > 0 && !tensors)) return codec_fail(AGM_ERR_ARG, "bad tensor table");
  if (mode != AGM_APPLY_COPY && mode != AGM_APPLY_LERP && mode != AGM_APPLY_ADD)
    return codec_fail(AGM_ERR_ARG, "unknown apply mode");
  for (int i = 0; i < count; ++i) {
    const AgmCodecTensor& t = tensors[i];
    const int rc = check_tensor(t.payload, t.kind, t.packed_dtype, t.n, t.cols, t.row_scales, t.scales_dtype,
                                t.target, t.target_dtype);
    if (rc) return rc;
  }
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  // Tensors are applied in table order, as the reference's loop does: a
  // tensor joins an earlier tensor's launch only if its target overlaps no
  // target of that launch and none of an earlier tensor still waiting for a
  // later launch (a repeated or overlapping target in ADD / LERP mode is a
  // read-modify-write that must follow the one before it).
  auto overlap = [&](int a, int b) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(tensors[a].target);
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(tensors[b].target);
    const uintptr_t a1 = a0 + static_cast<uintptr_t>(tensors[a].n) * dtype_bytes(tensors[a].target_dtype);
    const uintptr_t b1 = b0 + static_cast<uintptr_t>(tensors[b].n) * dtype_bytes(tensors[b].target_dtype);
    return tensors[a].n > 0 && tensors[b].n > 0 && a0 < b1 && b0 < a1;
  };
  std::vector<char> done(static_cast<size_t>(count), 0);
  for (int i = 0; i < count; ++i) {
    if (done[i]) continue;
    const AgmCodecTensor& a = tensors[i];
    done[i] = 1;
    if (a.n == 0) continue;
    const bool batchable = reinterpret_cast<uintptr_t>(a.payload) % 16 == 0 &&
                           reinterpret_cast<uintptr_t>(a.target) % 16 == 0 &&
                           (a.kind != AGM_CODEC_INT8_ROWWISE || a.cols % kCodecVec == 0);
    if (!batchable) {
      const int rc = agm_codec_decode(a.payload, a.kind, a.packed_dtype, a.n, a.cols, a.scale, a.row_scales,
                                      a.scales_dtype, a.target, a.target_dtype, mode, alpha, stream_);
      if (rc) return rc;
      continue;
    }
    // Gather the later tensors of the same signature (kind, payload, scale and
    // target types), up to kCodecBatch per launch.
    CodecBatch b{};
    auto add = [&](const AgmCodecTensor& t) {
      const int k = b.count++;
      b.payload[k] = t.payload;
      b.scales[k] = t.row_scales;
      b.target[k] = t.target;
      b.n[k] = t.n;
      b.cols[k] = t.kind == AGM_CODEC_INT8_ROWWISE ? t.cols : 1;
      b.scale[k] = t.scale;
      b.vec_begin[k + 1] = b.vec_begin[k] + t.n / kCodecVec;
    };
    add(a);
    std::vector<int> members(1, i);
    for (int j = i + 1; j < count && b.count < kCodecBatch; ++j) {
      const AgmCodecTensor& t = tensors[j];
      if (done[j] || t.n == 0 || t.kind != a.kind || t.target_dtype != a.target_dtype) continue;
      if (a.kind == AGM_CODEC_PLAIN && t.packed_dtype != a.packed_dtype) continue;
      if (a.kind == AGM_CODEC_INT8_ROWWISE && (t.scales_dtype != a.scales_dtype || t.cols % kCodecVec)) continue;
      if (reinterpret_cast<uintptr_t>(t.payload) % 16 || reinterpret_cast<uintptr_t>(t.target) % 16) continue;
      bool clash = false;
      for (int m : members) clash = clash || overlap(m, j);
      for (int k = i + 1; k < j && !clash; ++k) clash = !done[k] && overlap(k, j);
      if (clash) continue;
      done[j] = 1;
      members.push_back(j);
      add(t);
    }
    const cudaError_t e = launch_batch_any(a.kind, a.packed_dtype, a.scales_dtype, a.target_dtype, mode, b, alpha,
                                           sms, s);
    if (e != cudaSuccess) {
      set_last_error(std::string("agm_codec_decode_batch: ") + cudaGetErrorString(e));
      return AGM_ERR_CUDA;
    }
  }
  return AGM_OK;
}

}  // extern "C"
