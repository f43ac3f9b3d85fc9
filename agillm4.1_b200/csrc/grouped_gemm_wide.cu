// K3 on CTA pairs with 256 x 512 tiles: the grouped GEMM of
// grouped_gemm_pair.cu, each pair tile twice as wide.
//
//   C[r, n] = act( sum_k A[r, k] * W[g(r), n, k] + bias[g(r), n] )
//
// Why wider: a 256 x 256 pair tile brings 32 KB of operands per SM into
// shared memory for every 64-deep k-block, i.e. 64 bytes per tensor-core
// cycle on every SM (about 18.6 TB/s over 148 SMs at 1.965 GHz) from L2.
// A 256 x 512 tile reuses each A k-block for two 256-column accumulators:
// 48 KB per SM per k-block for twice the MMA work, 47 bytes per cycle.
//
// The two accumulators fill the SM's 512 TMEM columns, so a CTA has one
// accumulator, not a double buffer. The epilogue therefore never stages a
// whole tile: each warp reads 32 accumulator columns at a time, adds the
// bias, applies ReLU, rounds to the activation dtype and stores them straight
// to global memory (16-byte stores, one row per thread), and releases the
// accumulator as soon as its last columns are in registers. The 4-stage ring
// (48 KB per stage) meanwhile holds the next tile's first k-blocks, so the
// MMAs resume at once.
//
// Work unit: row tiles 2p and 2p+1 (same weight group: expert segments are
// padded to 256 rows) x one 512-column tile. Every output element sums its
// k-blocks in the same order with the same MMA shape (M=256, K=16) as the
// 256 x 256 kernel, so the two give identical bits.
//
// Roles (320 threads per CTA, both CTAs):
//   warp 0   TMA producer: A rows (16 KB) and the CTA's halves of the two
//            weight sub-tiles (2 x 16 KB) per stage, counted on rank 0's
//            `full` barrier.
//   warp 1   rank 0: tcgen05.mma M=256 N=256 (or the ragged width) K=16 into
//            TMEM columns [0, 256) and [256, 512); both ranks allocate and
//            free the pair's tensor memory.
//   warps 2-5 drain columns [0, 256), warps 6-9 columns [256, 512) of the
//            CTA's 128 rows (warp w reads TMEM lanes 32 * (w % 4) ...).
// Every mbarrier wait is bounded; both CTAs always reach the final cluster
// barrier, after which tensor memory is freed.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {

namespace {

constexpr int kBM = AGM_TILE_M;        // 128 rows per CTA, 256 per pair
constexpr int kBK = 64;
constexpr int kSubN = 256;             // columns per accumulator
constexpr int kWideN = 2 * kSubN;      // columns per pair tile
constexpr int kStages = 4;
constexpr int kGroupPairs = 8;         // rasterisation: 8 pairs (16 row tiles) per group
constexpr int kEpi = 8;
constexpr int kThreads = 64 + 32 * kEpi;
constexpr int kABytes = kBM * kBK * 2;              // 16 KB
constexpr int kBHalfBytes = (kSubN / 2) * kBK * 2;  // 16 KB: one CTA's half of one sub-tile
constexpr int kStageBytes = kABytes + 2 * kBHalfBytes;
constexpr int kTmemCols = 512;
constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "wide pair GEMM shared memory");

// Columns one pair MMA computes for n_valid columns of a sub-tile: a multiple
// of 32 (each CTA then holds a multiple of 16 weight rows), 0 if none.
__device__ __forceinline__ int wide_n_mma(int n_valid) {
  return n_valid <= 0 ? 0 : min(kSubN, (n_valid + 31) / 32 * 32);
}

__device__ __forceinline__ void wide_coords(int t, int num_p, int num_n, int& p, int& n_blk) {
  const int span = kGroupPairs * num_n;
  const int grp = t / span;
  const int first = grp * kGroupPairs;
  const int gp = min(num_p - first, kGroupPairs);
  const int r = t - grp * span;
  p = first + r % gp;
  n_blk = r / gp;
}

template <typename T, bool RELU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sStage = smem;  // stage s: A [16 KB] | B sub 0 half [16 KB] | B sub 1 half [16 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                    // rank 0's are used
  uint64_t* empty = bars + kStages;         // both ranks
  uint64_t* acc_full = bars + 2 * kStages;  // both ranks
  uint64_t* acc_empty = acc_full + 1;       // rank 0's is used
  uint64_t* drain = acc_empty + 1;          // rank 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(cluster_count_x());
  if (!args.early_weights) {
    pdl_wait();
    pdl_trigger();
  }

  int num_m = args.max_tiles;
  if (args.num_tiles) {
    const int nt = *args.num_tiles;
    if (nt > args.max_tiles) {
      if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(args.err, kErrTileOverflow);
    } else {
      num_m = nt;
    }
  }
  const int num_p = (num_m + 1) / 2;
  const int num_n = (args.n + kWideN - 1) / kWideN;
  const int total = num_p * num_n;
  const int num_kb = (args.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * kEpi);
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or copy
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    const uint32_t full0 = cluster_map(smem_u32(full), 0);
    int stage = 0;
    uint32_t phase = 0, armed = 0, armed_parity = 0;
    bool ok = true;
    // With early_weights, the first unit's first `ndef` stages get their
    // weight halves before the wait for the previous kernel and their A rows
    // after it.
    bool waited = !args.early_weights;
    const int ndef = min(kStages, num_kb);
    int deferred = 0, first_m = 0;
    for (int t = cluster; t < total && ok; t += nclusters) {
      int p, n_blk;
      wide_coords(t, num_p, num_n, p, n_blk);
      const int m0 = 2 * p;
      const int my_m = (!leader && m0 + 1 < num_m) ? m0 + 1 : m0;
      if (t == cluster) first_m = my_m;
      int g = args.tile_group ? args.tile_group[m0] : 0;
      if (g < 0 || g >= args.groups) g = 0;
      const int n0 = n_blk * kWideN;
      const int nm0 = wide_n_mma(args.n - n0), nm1 = wide_n_mma(args.n - n0 - kSubN);
      // Rank r holds weight rows [n0 + s * 256 + r * nm_s / 2, + nm_s / 2) of
      // sub-tile s (its 128-row box may run past them; the MMA reads only nm_s / 2).
      const int b_row0 = n0 + static_cast<int>(rank) * (nm0 / 2);
      const int b_row1 = n0 + kSubN + static_cast<int>(rank) * (nm1 / 2);
      const uint32_t bytes = 2 * (kABytes + (nm1 > 0 ? 2 : 1) * kBHalfBytes);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = sStage + stage * kStageBytes;
          if (leader) mbar_arrive_expect_tx(&full[stage], bytes);
          const uint32_t fb = full0 + stage * 8;
          tma_load_3d_pair(st + kABytes, &tmB, kb * kBK, b_row0, g, fb);
          if (nm1 > 0) tma_load_3d_pair(st + kABytes + kBHalfBytes, &tmB, kb * kBK, b_row1, g, fb);
          if (waited) tma_load_2d_pair(st, &tmA, kb * kBK, my_m * kBM, fb);
        }
        if (!waited && ++deferred == ndef) {
          pdl_wait();
          pdl_trigger();
          waited = true;
          if (lane == 0)
            for (int j = 0; j < deferred; ++j)
              tma_load_2d_pair(sStage + j * kStageBytes, &tmA, j * kBK, first_m * kBM, full0 + j * 8);
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
        for (int j = 0; j < deferred; ++j)
          tma_load_2d_pair(sStage + j * kStageBytes, &tmA, j * kBK, first_m * kBM, full0 + j * 8);
    }
    __syncwarp();
    // Drain: the pair MMAs that read this CTA's stages have completed (their
    // commit released `empty`), so no copy or read of this shared memory is
    // still in flight when the CTA leaves.
    bool drained = true;
    for (int s = 0; s < kStages && drained; ++s)
      if (armed & (1u << s)) drained = mbar_wait(&empty[s], (armed_parity >> s) & 1, args.err, kErrTimeoutDrain);
  } else if (warp == 1) {
    if (leader) {
      // ---------------- MMA issuer (rank 0) ----------------
      const uint32_t s_addr = smem_u32(sStage);
      int stage = 0, it = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < total && ok; t += nclusters, ++it) {
        int p, n_blk;
        wide_coords(t, num_p, num_n, p, n_blk);
        const int n0 = n_blk * kWideN;
        const int nm0 = wide_n_mma(args.n - n0), nm1 = wide_n_mma(args.n - n0 - kSubN);
        const bool bf = Traits<T>::code == AGM_BF16;
        const uint32_t idesc0 = idesc_f16(bf, 2 * kBM, nm0);
        const uint32_t idesc1 = idesc_f16(bf, 2 * kBM, nm1 > 0 ? nm1 : 32);
        if (!mbar_wait(acc_empty, (it & 1) ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
          *abort_s = 1;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
            *abort_s = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t st = s_addr + stage * kStageBytes;
            const uint64_t a_desc = smem_desc_k_sw128(st);
            const uint64_t b0_desc = smem_desc_k_sw128(st + kABytes);
            const uint64_t b1_desc = smem_desc_k_sw128(st + kABytes + kBHalfBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16_pair(tmem_base, a_desc + 2 * kk, b0_desc + 2 * kk, idesc0, (kb > 0 || kk > 0) ? 1u : 0u);
            if (nm1 > 0) {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk)
                umma_f16_pair(tmem_base + kSubN, a_desc + 2 * kk, b1_desc + 2 * kk, idesc1,
                              (kb > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit_pair(&empty[stage], 0x3);
            if (kb == num_kb - 1) umma_commit_pair(acc_full, 0x3);
          }
          __syncwarp();
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (lane == 0) umma_commit_pair(drain, 0x1);
      __syncwarp();
      mbar_wait(drain, 0, args.err, kErrTimeoutDrain);
    }
  } else {
    // ---------------- Epilogue (warps 2..9, both CTAs) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int sub = ew >> 2;              // accumulator: columns [256 * sub, +256) of the tile
    const uint32_t acc_empty0 = cluster_map(smem_u32(acc_empty), 0);
    const T* bias = static_cast<const T*>(args.bias);
    T* c = static_cast<T*>(args.c);
    int it = 0;
    for (int t = cluster; t < total; t += nclusters, ++it) {
      int p, n_blk;
      wide_coords(t, num_p, num_n, p, n_blk);
      const int m0 = 2 * p;
      const bool has2 = m0 + 1 < num_m;
      const int my_m = leader ? m0 : m0 + 1;
      const bool store = leader || has2;
      int g = args.tile_group ? args.tile_group[m0] : 0;
      if (g < 0 || g >= args.groups) g = 0;
      if (leader && ew == 0 && lane == 0 && has2 && args.tile_group && args.tile_group[m0 + 1] != args.tile_group[m0])
        raise_error(args.err, kErrPairGroup);
      if (!mbar_wait(acc_full, it & 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const int n0 = n_blk * kWideN + sub * kSubN;
      const int n_valid = min(kSubN, args.n - n0);   // <= 0: this accumulator is unused
      const int n_chunks = n_valid > 0 ? (n_valid + 31) / 32 : 0;
      const T* brow = bias ? bias + static_cast<int64_t>(g) * args.n + n0 : nullptr;
      const int64_t row = static_cast<int64_t>(my_m) * kBM + quarter * 32 + lane;
      T* crow = c + row * args.ldc + n0;
      const bool row_ok = store && row < args.c_rows;
      for (int c32 = 0; c32 < n_chunks; ++c32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + sub * kSubN + c32 * 32, r);
        tmem_ld_wait();
        if (c32 == n_chunks - 1) {
          // the whole accumulator of this warp is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive(acc_empty);
            else
              mbar_arrive_remote(acc_empty0);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int col = c32 * 32 + q * 8;
          if (col >= n_valid) continue;
          float bv[8];
          if (brow) {
            const uint4 bu = __ldg(reinterpret_cast<const uint4*>(brow + col));
            unpack8<T>(bu, bv);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) bv[j] = 0.f;
          }
          float v[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[j] = __uint_as_float(r[q * 8 + j]) + bv[j];
            if (RELU) v[j] = fmaxf(v[j], 0.f);
          }
          const uint4 o = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]),
                                     pack2<T>(v[6], v[7]));
          if (row_ok) *reinterpret_cast<uint4*>(crow + col) = o;
        }
      }
      if (n_chunks == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(acc_empty);
          else
            mbar_arrive_remote(acc_empty0);
        }
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs are done with the pair's tensor memory and shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <typename T, bool RELU>
cudaError_t launch_wide(const void* a, int64_t a_rows, const void* w, const GemmArgs& args, int num_sms,
                        cudaStream_t stream) {
  const CUtensorMapDataType dt = (Traits<T>::code == AGM_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tmA, tmB;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(a_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.k) * 2};
    const uint32_t box[2] = {kBK, kBM};
    if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(args.n),
                              static_cast<uint64_t>(args.groups)};
    const uint64_t str[2] = {static_cast<uint64_t>(args.k) * 2, static_cast<uint64_t>(args.k) * args.n * 2};
    const uint32_t box[3] = {kBK, kSubN / 2, 1};
    if (!encode_tmap(&tmB, w, 3, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(grouped_gemm_wide_kernel<T, RELU>), kSmemBytes);
  if (e != cudaSuccess) return e;
  const int num_n = (args.n + kWideN - 1) / kWideN;
  const int64_t max_units = static_cast<int64_t>((args.max_tiles + 1) / 2) * num_n;
  int ctas = args.max_ctas > 0 ? std::min(args.max_ctas, num_sms) : num_sms;
  ctas = static_cast<int>(std::min<int64_t>(ctas, 2 * std::max<int64_t>(1, max_units)));
  ctas = std::max(2, ctas & ~1);
  return launch_kernel(grouped_gemm_wide_kernel<T, RELU>, dim3(ctas), dim3(kThreads), kSmemBytes, stream, tmA, tmB,
                       args);
}

}  // namespace

cudaError_t grouped_gemm_wide(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                              int num_sms, cudaStream_t stream) {
  // 16-byte row stores: the output row stride and width must be multiples of 8 elements.
  if (args.relu_bits || args.tile_dst || args.groups2 > 0 || (args.ldc % 8) || (args.n % 8))
    return cudaErrorInvalidValue;
  switch (dtype) {
    case AGM_BF16:
      return relu ? launch_wide<__nv_bfloat16, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_wide<__nv_bfloat16, false>(a, a_rows, w, args, num_sms, stream);
    case AGM_F16:
      return relu ? launch_wide<__half, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_wide<__half, false>(a, a_rows, w, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
