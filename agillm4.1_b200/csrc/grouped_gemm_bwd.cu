// K3 backward: the expert projections' input and weight gradients.
//
// Autograd of the expert FFN `Linear(d,H) -> ReLU -> Linear(H,d)`
// (agillm41.py:4332-4336, called per (rank, expert) at 4428) computes, per
// expert segment of permuted rows:
//
//   dgrad   dA[r, n] = sum_k dC[r, k] * W[g(r), k, n]      (W in nn.Linear layout [out, in])
//           FC2: dh = (dy @ W2) masked by h > 0  (ReLU backward on the saved output)
//           FC1: dx_perm = dh @ W1
//   wgrad   dW[g, m, n] = sum_{rows r of segment g} dC[r, m] * A[r, n]
//           FC2: dW2 = dy^T h,  FC1: dW1 = dh^T x_perm
//
// Both run on the 5th-generation tensor cores with fp32 accumulation in TMEM
// and read every operand in its natural row-major layout: the weight in dgrad
// and both activations in wgrad are "MN-major" operands (the M or N index is
// the contiguous one), which tcgen05 reads directly from a 128-byte-swizzled
// shared-memory tile when the instruction descriptor's transpose bits are set.
// No transposed copy of any tensor is made.
//
// Shared-memory tiles: a K-major operand is a 128 x 64 TMA box (rows of 64
// elements = 128 B, 8-row groups 1024 B apart). An MN-major operand of extent
// X (128 or 256) along M/N is X/64 TMA boxes of 64 (MN, contiguous) x 64 (K)
// elements, 8 KB each: inside a box K-row j sits at j * 128 B, so the 8-row K
// groups are 1024 B apart (the descriptor's stride byte offset) and the 64-wide
// MN chunks 8 KB apart (its leading byte offset). One MMA (K = 16) consumes
// two K groups, so consecutive MMAs of a stage advance the start by 2 KB.
//
// Kernel structure (as the forward grouped GEMM): persistent CTAs, one per SM,
// 320 threads; warp 0 issues TMA loads into a ring of stages, warp 1 owns
// TMEM and issues tcgen05.mma (M = 128, N = BN, fp32 accumulate, double-
// buffered accumulator), warps 2-9 drain TMEM, round to the output type and
// write 32-row x 128-byte chunks with TMA stores through swizzled staging
// buffers. Every mbarrier wait is bounded; on time-out the kernel records an
// error bit, drains its copies and MMAs, frees TMEM and returns.
//
// fp32 (the reference's fp32 mode): a SIMT kernel with the same two modes.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {
namespace {

constexpr int BM = AGM_TILE_M;  // 128
constexpr int BK = 64;
constexpr int kGroupM = 16;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStgBytes = 32 * 128;  // one 32-row x 128-byte output chunk
constexpr int kBox = 64 * BK * 2;    // one 64 x 64 MN-major box (8 KB)

template <int BN>
struct BwdCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STG_BYTES = kEpiWarps * kStgBytes;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STG_BYTES + 256 + 1024;
};

__device__ __forceinline__ void dgrad_coords(int t, int num_m, int num_n, int& m_blk, int& n_blk) {
  const int span = kGroupM * num_n;
  const int g = t / span;
  const int first_m = g * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = t - g * span;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

// Work of one output tile.
struct TileJob {
  int g;       // expert
  int m_blk;   // row tile (dgrad: of the permuted rows; wgrad: of dW's rows)
  int n_blk;
  int k0;      // first K index (wgrad: first permuted row of the segment)
  int num_kb;  // K blocks of 64
};

template <int MODE, int BN>
__device__ __forceinline__ TileJob tile_job(int t, const BwdGemmArgs& a, int num_m, int num_n) {
  TileJob j;
  if (MODE == 0) {
    dgrad_coords(t, num_m, num_n, j.m_blk, j.n_blk);
    int g = a.tile_group ? a.tile_group[j.m_blk] : 0;
    j.g = (g < 0 || g >= a.groups) ? 0 : g;
    j.k0 = 0;
    j.num_kb = (a.k + BK - 1) / BK;
  } else {
    const int per = num_m * num_n;
    j.g = t / per;
    const int r = t - j.g * per;
    j.m_blk = r % num_m;
    j.n_blk = r / num_m;
    // Segments are whole multiples of 128 rows (zero-filled padding rows),
    // so K blocks of 64 never reach into the next segment.
    const int s0 = a.seg_start[j.g], s1 = a.seg_start[j.g + 1];
    j.k0 = s0;
    j.num_kb = max(0, s1 - s0) / BK;
  }
  return j;
}

// MODE 0 (dgrad): A = dC [rows, K] K-major (2-D map), B = W [G, K, N]
//                 MN-major (3-D map, N innermost), C = [rows, N].
//                 RELU_MASK: C = round(acc) where the forward's ReLU bit
//                 (aux_bits) is set, else 0. col_part (nullable): per-quarter
//                 column sums of C (the next layer's bias gradient).
// MODE 1 (wgrad): A = dC [rows, M] MN-major, B = act [rows, N] MN-major
//                 (2-D maps, K = permuted rows), C = [G, M, N] (3-D map).
template <typename T, typename OutT, int BN, int MODE, bool RELU_MASK>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_bwd_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, BwdGemmArgs args) {
  using Cfg = BwdCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool A_MN = (MODE == 1);
  constexpr int OUT_COLS = 128 / sizeof(OutT);  // columns per 128-byte staging row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sStg = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + Cfg::STG_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  pdl_wait();
  pdl_trigger();
  int num_m, total;
  const int num_n = (args.n + BN - 1) / BN;
  if (MODE == 0) {
    num_m = args.max_tiles;
    if (args.num_tiles) {
      const int nt = *args.num_tiles;
      if (nt > args.max_tiles) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(args.err, kErrTileOverflow);
      } else {
        num_m = nt;
      }
    }
    total = num_m * num_n;
  } else {
    num_m = (args.m + BM - 1) / BM;
    total = args.groups * num_m * num_n;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const TileJob j = tile_job<MODE, BN>(t, args, num_m, num_n);
      const int n0 = j.n_blk * BN;
      const int n_valid = min(BN, args.n - n0);
      const int nbox = (n_valid + 63) / 64;
      const uint32_t bytes = Cfg::A_BYTES + nbox * kBox;
      for (int kb = 0; kb < j.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], bytes);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int kc = j.k0 + kb * BK;
          if (A_MN) {
            tma_load_2d(a_dst, &tmA, j.m_blk * BM, kc, &full[stage]);
            tma_load_2d(a_dst + kBox, &tmA, j.m_blk * BM + 64, kc, &full[stage]);
          } else {
            tma_load_2d(a_dst, &tmA, kc, j.m_blk * BM, &full[stage]);
          }
          for (int b = 0; b < nbox; ++b) {
            if (MODE == 0)
              tma_load_3d(b_dst + b * kBox, &tmB, n0 + b * 64, kc, j.g, &full[stage]);
            else
              tma_load_2d(b_dst + b * kBox, &tmB, n0 + b * 64, kc, &full[stage]);
          }
        }
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    __syncwarp();
    for (int s = 0; s < STAGES; ++s)
      if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1, args.err, kErrTimeoutDrain);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const TileJob j = tile_job<MODE, BN>(t, args, num_m, num_n);
      const int n_valid = min(BN, args.n - j.n_blk * BN);
      const int n_mma = (n_valid + 15) / 16 * 16;
      const uint32_t idesc = idesc_f16(Traits<T>::code == AGM_BF16, BM, n_mma) | (A_MN ? (1u << 15) : 0u) | (1u << 16);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < j.num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = sA_addr + stage * Cfg::A_BYTES;
          const uint64_t a_desc = A_MN ? smem_desc_mn_sw128(a_addr, kBox) : smem_desc_k_sw128(a_addr);
          const uint64_t b_desc = smem_desc_mn_sw128(sB_addr + stage * Cfg::B_BYTES, kBox);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: 16 elements = 32 B along the row; MN-major: 16 K rows = 2 KB.
            const uint64_t a_step = A_MN ? static_cast<uint64_t>(kk) * (2048 >> 4) : static_cast<uint64_t>(2 * kk);
            const uint64_t b_step = static_cast<uint64_t>(kk) * (2048 >> 4);
            umma_f16(d_tmem, a_desc + a_step, b_desc + b_step, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      // An empty K range (an expert with no rows) issues no MMA: the commit
      // arrives at once and the epilogue writes zeros.
      if (lane == 0) umma_commit(&acc_full[acc]);
      __syncwarp();
    }
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0, args.err, kErrTimeoutDrain);
  } else {
    // ---------------- Epilogue (warps 2..9) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    uint8_t* stg = sStg + ew * kStgBytes;
    const uint32_t stg_row = lane * 128;
    constexpr int kChunks = BN / 128;  // 64-column chunks per warp per tile
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const TileJob j = tile_job<MODE, BN>(t, args, num_m, num_n);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int n0 = j.n_blk * BN;
      const int n_valid = min(BN, args.n - n0);
      const int row0 = j.m_blk * BM + quarter * 32;
      // ReLU mask words of this warp's chunks, fetched while the MMAs run.
      uint32_t mbits[kChunks][2];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        mbits[c][0] = mbits[c][1] = 0u;
        const int col = (half + 2 * c) * 64;
        if (RELU_MASK && col < n_valid) {
          const int64_t w0 = (n0 + col) >> 5;
          const uint32_t* b = args.aux_bits + row0 + lane;
          mbits[c][0] = __ldg(b + w0 * args.ld_aux_bits);
          if (col + 32 < n_valid) mbits[c][1] = __ldg(b + (w0 + 1) * args.ld_aux_bits);
        }
      }
      if (!mbar_wait(&acc_full[acc], acc_phase, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const bool zero = (j.num_kb == 0);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int c64 = half + 2 * c;
        if (c64 * 64 >= n_valid) break;
        const int col = c64 * 64;
        uint32_t r[64];
        if (!zero) {
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + col;
          tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) r[i] = 0u;
        }
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = round_to<T>(__uint_as_float(r[i]));
        if (RELU_MASK) {
          // ReLU backward: keep where the forward's activation was > 0.
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (!((mbits[c][0] >> i) & 1u)) v[i] = 0.f;
            if (!((mbits[c][1] >> i) & 1u)) v[32 + i] = 0.f;
          }
        }
        if (MODE == 0 && args.col_part) {
          // Bias gradient of the layer this gradient feeds: column sums of
          // the rounded values, one fp32 partial per 32-row quarter.
          float s0, s1;
          warp_colsum64(v, lane, s0, s1);
          if (col + 2 * lane < n_valid)
            *reinterpret_cast<float2*>(args.col_part + (static_cast<int64_t>(j.m_blk) * 4 + quarter) * args.n + n0 +
                                       col + 2 * lane) = make_float2(s0, s1);
        }
#pragma unroll
        for (int sub = 0; sub < 64 / OUT_COLS; ++sub) {
          if (col + sub * OUT_COLS >= n_valid) break;
          if (lane == 0) bulk_wait_group_read0();
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint4 o;
            if constexpr (sizeof(OutT) == 4) {
              const float* f = &v[sub * 32 + q * 4];
              o = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                             __float_as_uint(f[3]));
            } else {
              const float* f = &v[q * 8];
              o = make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
            }
            *reinterpret_cast<uint4*>(stg + stg_row + ((q ^ (lane & 7)) << 4)) = o;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (MODE == 0)
              tma_store_2d(&tmC, stg, n0 + col + sub * OUT_COLS, row0);
            else
              tma_store_3d(&tmC, stg, n0 + col + sub * OUT_COLS, row0, j.g);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// fp32 SIMT kernel (reference fp32 mode): 64 x 64 tiles, 4 x 4 per thread.
// ---------------------------------------------------------------------------
template <int MODE, bool RELU_MASK>
__global__ void __launch_bounds__(256) grouped_gemm_bwd_f32_kernel(const float* __restrict__ A,
                                                                   const float* __restrict__ B, BwdGemmArgs args) {
  constexpr int TM = 64, TN = 64, TK = 16;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  pdl_wait();
  pdl_trigger();
  const int N = args.n;
  int g, kbeg, kend;
  int64_t m0;
  if (MODE == 0) {
    int num_m = args.max_tiles;
    if (args.num_tiles) num_m = min(*args.num_tiles, args.max_tiles);
    const int tile = blockIdx.x / (BM / TM);
    if (tile >= num_m) return;
    g = args.tile_group ? args.tile_group[tile] : 0;
    if (g < 0 || g >= args.groups) g = 0;
    m0 = static_cast<int64_t>(tile) * BM + (blockIdx.x % (BM / TM)) * TM;
    kbeg = 0;
    kend = args.k;
  } else {
    const int per = (args.m + TM - 1) / TM;
    g = blockIdx.x / per;
    m0 = static_cast<int64_t>(blockIdx.x % per) * TM;
    kbeg = args.seg_start[g];
    kend = args.seg_start[g + 1];
  }
  const int n0 = blockIdx.y * TN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = kbeg; k0 < kend; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      if (MODE == 0) {
        const int r = i / TK, kk = i % TK;  // A [rows, K]
        As[kk][r] = (k0 + kk < kend) ? A[(m0 + r) * args.k + k0 + kk] : 0.f;
        const int kk2 = i / TN, n = i % TN;  // W [G, K, N]
        Bs[kk2][n] = (k0 + kk2 < kend && n0 + n < N)
                         ? B[(static_cast<int64_t>(g) * args.k + k0 + kk2) * N + n0 + n]
                         : 0.f;
      } else {
        const int kk = i / TM, m = i % TM;  // A [rows, M]
        As[kk][m] = (k0 + kk < kend && m0 + m < args.m) ? A[static_cast<int64_t>(k0 + kk) * args.m + m0 + m] : 0.f;
        const int n = i % TN;  // B [rows, N]
        Bs[kk][n] = (k0 + kk < kend && n0 + n < N) ? B[static_cast<int64_t>(k0 + kk) * N + n0 + n] : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
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
  float* C = static_cast<float*>(args.c);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (MODE == 0 ? (r >= args.c_rows) : (r >= args.m)) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (RELU_MASK && !(static_cast<const float*>(args.aux)[r * args.ld_aux + n] > 0.f)) v = 0.f;
      if (MODE == 0)
        C[r * args.ldc + n] = v;
      else
        C[(static_cast<int64_t>(g) * args.m + r) * N + n] = v;
    }
  }
}

CUtensorMapDataType tmap_type(int code) {
  switch (code) {
    case AGM_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case AGM_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

template <typename T, typename OutT, int BN, int MODE, bool RELU_MASK>
cudaError_t launch_bwd_tc(const void* a, const void* b, int64_t a_rows, const BwdGemmArgs& args, int num_sms,
                          cudaStream_t stream) {
  using Cfg = BwdCfg<BN>;
  const CUtensorMapDataType dt = tmap_type(Traits<T>::code);
  const CUtensorMapDataType dto = tmap_type(sizeof(OutT) == 4 ? AGM_F32 : Traits<T>::code);
  CUtensorMap tmA, tmB, tmC;
  if (MODE == 0) {
    {  // A: [a_rows, K] K-major
      const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(a_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.k) * 2};
      const uint32_t box[2] = {BK, BM};
      if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // B: W [G, K, N], N innermost
      const uint64_t dims[3] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.k),
                                static_cast<uint64_t>(args.groups)};
      const uint64_t str[2] = {static_cast<uint64_t>(args.n) * 2, static_cast<uint64_t>(args.n) * args.k * 2};
      const uint32_t box[3] = {64, BK, 1};
      if (!encode_tmap(&tmB, b, 3, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // C: [c_rows, N]
      const uint64_t dims[2] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.c_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.ldc) * sizeof(OutT)};
      const uint32_t box[2] = {static_cast<uint32_t>(128 / sizeof(OutT)), 32};
      if (!encode_tmap(&tmC, args.c, 2, dims, str, box, dto)) return cudaErrorInvalidValue;
    }
  } else {
    {  // A: dC [a_rows, M], M innermost
      const uint64_t dims[2] = {static_cast<uint64_t>(args.m), static_cast<uint64_t>(a_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.m) * 2};
      const uint32_t box[2] = {64, BK};
      if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // B: act [a_rows, N], N innermost
      const uint64_t dims[2] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(a_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.n) * 2};
      const uint32_t box[2] = {64, BK};
      if (!encode_tmap(&tmB, b, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // C: [G, M, N]
      const uint64_t dims[3] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.m),
                                static_cast<uint64_t>(args.groups)};
      const uint64_t str[2] = {static_cast<uint64_t>(args.n) * sizeof(OutT),
                               static_cast<uint64_t>(args.n) * args.m * sizeof(OutT)};
      const uint32_t box[3] = {static_cast<uint32_t>(128 / sizeof(OutT)), 32, 1};
      if (!encode_tmap(&tmC, args.c, 3, dims, str, box, dto)) return cudaErrorInvalidValue;
    }
  }
  auto kern = grouped_gemm_bwd_kernel<T, OutT, BN, MODE, RELU_MASK>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), Cfg::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int num_n = (args.n + BN - 1) / BN;
  const int64_t max_total = MODE == 0 ? static_cast<int64_t>(args.max_tiles) * num_n
                                      : static_cast<int64_t>(args.groups) * ((args.m + BM - 1) / BM) * num_n;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms, max_total)));
  return launch_kernel(kern, dim3(grid), dim3(kThreads), Cfg::SMEM_BYTES, stream, tmA, tmB, tmC, args);
}

template <typename T, typename OutT, int MODE, bool RELU_MASK>
cudaError_t dispatch_bwd_bn(const void* a, const void* b, int64_t a_rows, const BwdGemmArgs& args, int num_sms,
                            cudaStream_t stream) {
  const int64_t m_tiles = MODE == 0 ? args.max_tiles : static_cast<int64_t>(args.groups) * ((args.m + BM - 1) / BM);
  const int64_t tiles256 = m_tiles * ((args.n + 255) / 256);
  if (tiles256 >= 2 * num_sms) return launch_bwd_tc<T, OutT, 256, MODE, RELU_MASK>(a, b, a_rows, args, num_sms, stream);
  return launch_bwd_tc<T, OutT, 128, MODE, RELU_MASK>(a, b, a_rows, args, num_sms, stream);
}

}  // namespace

cudaError_t grouped_gemm_dgrad(int dtype, const void* dc, int64_t rows, const void* w, const BwdGemmArgs& args,
                               bool relu_mask, int num_sms, cudaStream_t stream) {
  if (args.max_tiles <= 0 || args.n <= 0) return cudaSuccess;
  switch (dtype) {
    case AGM_F32: {
      dim3 grid(static_cast<unsigned>(args.max_tiles * (BM / 64)), static_cast<unsigned>((args.n + 63) / 64));
      const float* A = static_cast<const float*>(dc);
      const float* B = static_cast<const float*>(w);
      return relu_mask ? launch_kernel(grouped_gemm_bwd_f32_kernel<0, true>, grid, dim3(256), 0, stream, A, B, args)
                       : launch_kernel(grouped_gemm_bwd_f32_kernel<0, false>, grid, dim3(256), 0, stream, A, B, args);
    }
    case AGM_BF16:
      return relu_mask ? dispatch_bwd_bn<__nv_bfloat16, __nv_bfloat16, 0, true>(dc, w, rows, args, num_sms, stream)
                       : dispatch_bwd_bn<__nv_bfloat16, __nv_bfloat16, 0, false>(dc, w, rows, args, num_sms, stream);
    case AGM_F16:
      return relu_mask ? dispatch_bwd_bn<__half, __half, 0, true>(dc, w, rows, args, num_sms, stream)
                       : dispatch_bwd_bn<__half, __half, 0, false>(dc, w, rows, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t grouped_gemm_wgrad(int dtype, bool out_f32, const void* dc, const void* act, int64_t rows,
                               const BwdGemmArgs& args, int num_sms, cudaStream_t stream) {
  if (args.groups <= 0 || args.m <= 0 || args.n <= 0) return cudaSuccess;
  switch (dtype) {
    case AGM_F32: {
      dim3 grid(static_cast<unsigned>(args.groups * ((args.m + 63) / 64)), static_cast<unsigned>((args.n + 63) / 64));
      return launch_kernel(grouped_gemm_bwd_f32_kernel<1, false>, grid, dim3(256), 0, stream,
                           static_cast<const float*>(dc), static_cast<const float*>(act), args);
    }
    case AGM_BF16:
      return out_f32 ? dispatch_bwd_bn<__nv_bfloat16, float, 1, false>(dc, act, rows, args, num_sms, stream)
                     : dispatch_bwd_bn<__nv_bfloat16, __nv_bfloat16, 1, false>(dc, act, rows, args, num_sms, stream);
    case AGM_F16:
      return out_f32 ? dispatch_bwd_bn<__half, float, 1, false>(dc, act, rows, args, num_sms, stream)
                     : dispatch_bwd_bn<__half, __half, 1, false>(dc, act, rows, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
