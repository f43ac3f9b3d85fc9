// K3 for small batches (AR decode): the grouped GEMM with the operands
// swapped, so the weights stream from HBM at full depth.
//
//   C[r, n] = act( sum_k A[r, k] * W[g(r), n, k] + bias[g(r), n] )
//
// computed as D[n, t] = sum_k W[e, n, k] * A[seg_start[e] + t, k] for the
// t < count[e] rows of expert segment e. In decode (64 tokens x top-2 over 14
// experts, about 9 rows per expert) the row-tile kernel spends half of every
// shared-memory stage on activation rows that are nearly all padding, and its
// ~13 MB of weight bytes in flight across the GPU cannot cover the DRAM
// latency (FC2 ran at ~3.5 TB/s). Here the weight tile is the M = 128 operand
// (16 KB per 64-deep k-block, from DRAM) and only the segment's valid rows
// form the N = 32 operand (4 KB, from L2), so a 10-stage ring keeps 160 KB of
// weights in flight per SM.
//
// Work unit: (expert e, 32-row block j of its segment, 128-column block of
// W). Units are numbered from the device-side counts, so empty experts cost
// nothing and the forward needs no host sync. One CTA per SM walks the units.
//
// Roles (320 threads): warp 0 TMA producer; warp 1 TMEM owner and
// tcgen05.mma issuer (M=128, N=32, K=16, fp32 accumulation, accumulator
// double-buffered in 2 x 32 TMEM columns); warps 2-9 epilogue: warp w reads
// TMEM lanes [32*(w%4), +32) (32 output columns n) and 16 of the 32 rows,
// adds the bias, applies ReLU, rounds and writes C[row, n] (a warp writes 64
// contiguous bytes per row). Rows past the segment's count are not written.
// Every mbarrier wait is bounded; on time-out the kernel records an error,
// drains its copies and MMAs, frees TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {

namespace {

constexpr int kBK = 64;
constexpr int kFM = 128;               // W rows (output columns n) per unit: the MMA's M
constexpr int kRows = 32;              // segment rows per unit: the MMA's N
constexpr int kStages = 10;
constexpr int kEpi = 8;
constexpr int kThreads = 64 + 32 * kEpi;
constexpr int kWBytes = kFM * kBK * 2;    // 16 KB
constexpr int kABytes = kRows * kBK * 2;  // 4 KB
constexpr int kTmemCols = 2 * kRows;
constexpr int kSmemBytes = kStages * (kWBytes + kABytes) + 256 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "swap GEMM shared memory");

struct Units {
  int n_e;                        // experts
  int blocks[AGM_MAX_EXPERTS];    // 32-row blocks of each expert
  int first[AGM_MAX_EXPERTS + 1]; // prefix sum of blocks
};

__device__ __forceinline__ void load_units(const GemmArgs& args, Units& u) {
  u.n_e = min(args.groups, AGM_MAX_EXPERTS);
  int acc = 0;
  for (int e = 0; e < u.n_e; ++e) {
    const int c = max(0, args.seg_count[e]);
    u.blocks[e] = (c + kRows - 1) / kRows;
    u.first[e] = acc;
    acc += u.blocks[e];
  }
  u.first[u.n_e] = acc;
}

// Unit t -> expert e, row block j, column block fb.
__device__ __forceinline__ void unit_coords(const Units& u, int num_fb, int t, int& e, int& j, int& fb) {
  const int b = t / num_fb;
  fb = t - b * num_fb;
  e = 0;
  while (e + 1 < u.n_e && u.first[e + 1] <= b) ++e;
  j = b - u.first[e];
}

template <typename T, bool RELU>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                             GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sA = smem + kStages * kWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kStages * kABytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  __shared__ Units u;
  const int num_fb = (args.n + kFM - 1) / kFM;
  const int num_kb = (args.k + kBK - 1) / kBK;
  if (!args.early_weights) {
    pdl_wait();
    pdl_trigger();
  }

  if (threadIdx.x == 0) {
    load_units(args, u);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpi);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = u.first[u.n_e] * num_fb;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0, armed = 0, armed_parity = 0;
    bool ok = true;
    // With early_weights, the first unit's first `ndef` stages get their
    // weight tile before the wait for the previous kernel and their rows
    // after it: the weights start streaming while the permute still runs.
    bool waited = !args.early_weights;
    const int ndef = min(kStages, num_kb);
    int deferred = 0, first_row = 0;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int e, j, fb;
      unit_coords(u, num_fb, t, e, j, fb);
      const int row0 = args.seg_start[e] + j * kRows;
      if (t == static_cast<int>(blockIdx.x)) first_row = row0;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], kWBytes + kABytes);
          if (args.w_tiled)
            tma_load_5d(sW + stage * kWBytes, &tmW, 0, 0, kb, fb, e, &full[stage]);
          else
            tma_load_3d(sW + stage * kWBytes, &tmW, kb * kBK, fb * kFM, e, &full[stage]);
          if (waited) tma_load_2d(sA + stage * kABytes, &tmA, kb * kBK, row0, &full[stage]);
        }
        if (!waited && ++deferred == ndef) {
          pdl_wait();
          pdl_trigger();
          waited = true;
          if (lane == 0)
            for (int q = 0; q < deferred; ++q) tma_load_2d(sA + q * kABytes, &tmA, q * kBK, first_row, &full[q]);
        }
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!waited) {  // no unit, or stopped early: still order after the previous kernel
      pdl_wait();
      pdl_trigger();
      if (lane == 0)
        for (int q = 0; q < deferred; ++q) tma_load_2d(sA + q * kABytes, &tmA, q * kBK, first_row, &full[q]);
    }
    __syncwarp();
    for (int s = 0; s < kStages; ++s)
      if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1, args.err, kErrTimeoutDrain);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_f16(Traits<T>::code == AGM_BF16, kFM, kRows);
    const uint32_t sW_addr = smem_u32(sW), sA_addr = smem_u32(sA);
    int stage = 0, it = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&acc_empty[acc], ((it >> 1) & 1) ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kRows;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t w_desc = smem_desc_k_sw128(sW_addr + stage * kWBytes);
          const uint64_t a_desc = smem_desc_k_sw128(sA_addr + stage * kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d_tmem, w_desc + 2 * kk, a_desc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (kb == num_kb - 1) umma_commit(&acc_full[acc]);
        }
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0, args.err, kErrTimeoutDrain);
  } else {
    // ---------------- Epilogue (warps 2..9) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;  // rows [16 * half, +16) of the unit
    const T* bias = static_cast<const T*>(args.bias);
    T* c = static_cast<T*>(args.c);
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      int e, j, fb;
      unit_coords(u, num_fb, t, e, j, fb);
      const int acc = it & 1;
      if (!mbar_wait(&acc_full[acc], (it >> 1) & 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kRows + 16 * half, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);  // the accumulator is in registers
      const int n = fb * kFM + quarter * 32 + lane;
      const int valid = min(kRows, args.seg_count[e] - j * kRows) - 16 * half;
      const int64_t row0 = static_cast<int64_t>(args.seg_start[e]) + j * kRows + 16 * half;
      if (n < args.n && valid > 0) {
        const float b = bias ? Traits<T>::to_f(bias[static_cast<int64_t>(e) * args.n + n]) : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (i < valid) {
            float v = __uint_as_float(r[i]) + b;
            if (RELU) v = fmaxf(v, 0.f);
            c[(row0 + i) * args.ldc + n] = Traits<T>::from_f(v);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <typename T, bool RELU>
cudaError_t launch_swap(const void* a, int64_t a_rows, const void* w, const GemmArgs& args, int num_sms,
                        cudaStream_t stream) {
  const CUtensorMapDataType dt = (Traits<T>::code == AGM_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tmA, tmW;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(a_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.k) * 2};
    const uint32_t box[2] = {kBK, kRows};
    if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  if (args.w_tiled) {
    // [groups][n / 128][k / 64][128 rows][64 elements]: a box is one contiguous 16 KB tile
    if (args.n % kFM || args.k % kBK) return cudaErrorInvalidValue;
    const uint64_t nkb = static_cast<uint64_t>(args.k / kBK), nfb = static_cast<uint64_t>(args.n / kFM);
    const uint64_t dims[5] = {kBK, kFM, nkb, nfb, static_cast<uint64_t>(args.groups)};
    const uint64_t tile = static_cast<uint64_t>(kFM) * kBK * 2;
    const uint64_t str[4] = {kBK * 2, tile, tile * nkb, tile * nkb * nfb};
    const uint32_t box[5] = {kBK, kFM, 1, 1, 1};
    if (!encode_tmap(&tmW, w, 5, dims, str, box, dt)) return cudaErrorInvalidValue;
  } else {
    const uint64_t dims[3] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(args.n),
                              static_cast<uint64_t>(args.groups)};
    const uint64_t str[2] = {static_cast<uint64_t>(args.k) * 2, static_cast<uint64_t>(args.k) * args.n * 2};
    const uint32_t box[3] = {kBK, kFM, 1};
    if (!encode_tmap(&tmW, w, 3, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(grouped_gemm_swap_kernel<T, RELU>), kSmemBytes);
  if (e != cudaSuccess) return e;
  // Host bound on units: every expert's rows could need one more block than
  // an even split of the max_tiles x 128 rows.
  const int num_fb = (args.n + kFM - 1) / kFM;
  const int64_t max_blocks = static_cast<int64_t>(args.max_tiles) * (AGM_TILE_M / kRows) + args.groups;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms, max_blocks * num_fb)));
  return launch_kernel(grouped_gemm_swap_kernel<T, RELU>, dim3(grid), dim3(kThreads), kSmemBytes, stream, tmA, tmW,
                       args);
}

}  // namespace

namespace {

// dst [groups][n / 128][k / 64][128][64] <- src [groups][n][k], 16 bytes per thread step.
__global__ void decode_tile_layout_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t groups,
                                          int n, int k) {
  const int64_t total = groups * static_cast<int64_t>(n) * k / 8;
  const int nkb = k / kBK, nfb = n / kFM;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = v * 8;                       // destination element
    const int c = static_cast<int>(e % kBK);
    const int r = static_cast<int>((e / kBK) % kFM);
    const int64_t t = e / (kBK * kFM);             // tile index ((g * nfb + fb) * nkb + kb)
    const int kb = static_cast<int>(t % nkb);
    const int64_t gf = t / nkb;
    const int fb = static_cast<int>(gf % nfb);
    const int64_t g = gf / nfb;
    const int64_t src_e = (g * n + static_cast<int64_t>(fb) * kFM + r) * k + static_cast<int64_t>(kb) * kBK + c;
    dst[v] = __ldcs(src + src_e / 8);
  }
}

}  // namespace

cudaError_t decode_tile_layout(const void* src, void* dst, int64_t groups, int n, int k, int num_sms,
                               cudaStream_t stream) {
  if (n % kFM || k % kBK || groups <= 0) return cudaErrorInvalidValue;
  decode_tile_layout_kernel<<<4 * num_sms, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                                             groups, n, k);
  return cudaGetLastError();
}

cudaError_t grouped_gemm_swap(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                              int num_sms, cudaStream_t stream) {
  if (!args.seg_start || !args.seg_count || args.groups > AGM_MAX_EXPERTS) return cudaErrorInvalidValue;
  switch (dtype) {
    case AGM_BF16:
      return relu ? launch_swap<__nv_bfloat16, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_swap<__nv_bfloat16, false>(a, a_rows, w, args, num_sms, stream);
    case AGM_F16:
      return relu ? launch_swap<__half, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_swap<__half, false>(a, a_rows, w, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
