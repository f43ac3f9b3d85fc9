// K3 backward on CTA pairs: the dgrad and wgrad GEMMs of grouped_gemm_bwd.cu
// with 256 x 256 tiles computed by a cluster of two CTAs (one TPC) through
// tcgen05.mma with cta_group::2.
//
//   dgrad   C[r, n]    = sum_k dC[r, k] * W[g(r), k, n]             (MODE 0)
//   wgrad   C[g, m, n] = sum_{r in segment g} dC[r, m] * act[r, n]   (MODE 1)
//
// Why pairs: a one-CTA 128 x 256 tile streams 48 KB of operands per 64-deep
// k-block from L2 for 4 MFLOP of tensor work; the pair computes 256 x 256
// with each CTA loading 32 KB (its 128 rows of A, half of B), so the
// L2-to-SM traffic per FLOP drops by a third and the ring holds 6 stages.
//
// Operands (128-byte swizzle): B is MN-major in both modes (the weight
// [G, K, N] in dgrad, the activation [rows, N] in wgrad); each CTA holds
// n_mma / 2 of the tile's columns as 64-column TMA boxes (8 KB, K rows 128 B
// apart), the pair MMA reading both halves at the same shared-memory offsets.
// A is K-major (dgrad, 128 x 64 box) or MN-major (wgrad, two 64 x 64 boxes).
// n_mma is the valid column count rounded up to 128, so each half is whole
// 64-column boxes.
//
// Work units: dgrad - row tiles 2p and 2p+1 (same group: the plan pads expert
// segments to 256 rows in this mode) x one 256-column tile; wgrad - (expert,
// 256-row block of C, 256-column tile), K = the expert's rows. A pair whose
// second row tile does not exist has the peer CTA repeat the first tile's rows
// (dgrad) or read zero rows (wgrad), storing nothing.
//
// Roles as grouped_gemm_pair.cu: warp 0 of both CTAs loads (counting bytes on
// rank 0's `full` barrier), warp 1 of rank 0 issues the MMAs and commits to
// both CTAs, warps 2-9 of each CTA drain its 128 accumulator rows with the
// epilogue of grouped_gemm_bwd.cu (rounding, ReLU mask bits, bias column-sum
// partials, TMA stores). Every mbarrier wait is bounded; both CTAs always
// reach the final cluster barrier, after which tensor memory is freed.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {
namespace {

constexpr int kBM = AGM_TILE_M;  // 128 rows per CTA, 256 per pair
constexpr int kBK = 64;
constexpr int kPairN = 256;
constexpr int kStages = 6;
constexpr int kGroupPairs = 8;
constexpr int kEpi = 8;
constexpr int kThreads = 64 + 32 * kEpi;
constexpr int kBox = 64 * kBK * 2;          // one 64 x 64 box (8 KB)
constexpr int kABytes = kBM * kBK * 2;      // 16 KB
constexpr int kBBytes = (kPairN / 2) * kBK * 2;  // 16 KB: this CTA's half of B
constexpr int kStgBytes = 32 * 128;
constexpr int kTmemCols = 2 * kPairN;
constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + kEpi * kStgBytes + 256 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "pair backward GEMM shared memory");

__device__ __forceinline__ int pair_n_mma(int n_valid) { return min(kPairN, (n_valid + 127) / 128 * 128); }

struct PairJob {
  int g;
  int m0;      // first row tile of the pair
  int my_m;    // this CTA's row tile
  bool store;  // this CTA's rows exist
  int n_blk;
  int k0;
  int num_kb;
};

template <int MODE>
__device__ __forceinline__ PairJob pair_job(int t, const BwdGemmArgs& a, int num_m, int num_p, int num_n,
                                            uint32_t rank) {
  PairJob j;
  int p;
  if (MODE == 0) {
    const int span = kGroupPairs * num_n;
    const int grp = t / span;
    const int first = grp * kGroupPairs;
    const int gp = min(num_p - first, kGroupPairs);
    const int r = t - grp * span;
    p = first + r % gp;
    j.n_blk = r / gp;
    j.m0 = 2 * p;
    int g = a.tile_group ? a.tile_group[j.m0] : 0;
    j.g = (g < 0 || g >= a.groups) ? 0 : g;
    const bool has2 = j.m0 + 1 < num_m;
    j.my_m = (rank == 1 && has2) ? j.m0 + 1 : j.m0;
    j.store = rank == 0 || has2;
    j.k0 = 0;
    j.num_kb = (a.k + kBK - 1) / kBK;
  } else {
    const int per = num_p * num_n;
    j.g = t / per;
    const int r = t - j.g * per;
    p = r % num_p;
    j.n_blk = r / num_p;
    j.m0 = 2 * p;
    j.my_m = j.m0 + static_cast<int>(rank);
    j.store = j.my_m < num_m;
    const int s0 = a.seg_start[j.g], s1 = a.seg_start[j.g + 1];
    j.k0 = s0;
    j.num_kb = max(0, s1 - s0) / kBK;
  }
  return j;
}

template <typename T, typename OutT, int MODE, bool RELU_MASK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_bwd_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                 const __grid_constant__ CUtensorMap tmC, BwdGemmArgs args) {
  constexpr bool A_MN = (MODE == 1);
  constexpr int OUT_COLS = 128 / sizeof(OutT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint8_t* sStg = smem + kStages * (kABytes + kBBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + kEpi * kStgBytes);
  uint64_t* full = bars;                    // rank 0's are used
  uint64_t* empty = bars + kStages;         // both ranks
  uint64_t* acc_full = bars + 2 * kStages;  // both ranks
  uint64_t* acc_empty = acc_full + 2;       // rank 0's are used
  uint64_t* drain = acc_empty + 2;          // rank 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(cluster_count_x());
  pdl_wait();
  pdl_trigger();

  int num_m;
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
  } else {
    num_m = (args.m + kBM - 1) / kBM;
  }
  const int num_p = (num_m + 1) / 2;
  const int num_n = (args.n + kPairN - 1) / kPairN;
  const int total = (MODE == 0 ? 1 : args.groups) * num_p * num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpi);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
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
    for (int t = cluster; t < total && ok; t += nclusters) {
      const PairJob j = pair_job<MODE>(t, args, num_m, num_p, num_n, rank);
      const int n0 = j.n_blk * kPairN;
      const int half = pair_n_mma(args.n - n0) / 2;  // this CTA's columns: [n0 + rank * half, + half)
      const int nbox = half / 64;
      const int bcol = n0 + static_cast<int>(rank) * half;
      const uint32_t bytes = 2 * (kABytes + nbox * kBox);  // both CTAs' bytes, armed by rank 0
      for (int kb = 0; kb < j.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(&full[stage], bytes);
          const uint32_t fb = full0 + stage * 8;
          uint8_t* a_dst = sA + stage * kABytes;
          uint8_t* b_dst = sB + stage * kBBytes;
          const int kc = j.k0 + kb * kBK;
          if (A_MN) {
            tma_load_2d_pair(a_dst, &tmA, j.my_m * kBM, kc, fb);
            tma_load_2d_pair(a_dst + kBox, &tmA, j.my_m * kBM + 64, kc, fb);
          } else {
            tma_load_2d_pair(a_dst, &tmA, kc, j.my_m * kBM, fb);
          }
          for (int b = 0; b < nbox; ++b) {
            if (MODE == 0)
              tma_load_3d_pair(b_dst + b * kBox, &tmB, bcol + b * 64, kc, j.g, fb);
            else
              tma_load_2d_pair(b_dst + b * kBox, &tmB, bcol + b * 64, kc, fb);
          }
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
    __syncwarp();
    // Drain: the pair MMAs that read this CTA's stages have completed (their
    // commit released `empty`), so nothing reads this shared memory later.
    bool drained = true;
    for (int s = 0; s < kStages && drained; ++s)
      if (armed & (1u << s)) drained = mbar_wait(&empty[s], (armed_parity >> s) & 1, args.err, kErrTimeoutDrain);
  } else if (warp == 1) {
    if (leader) {
      // ---------------- MMA issuer (rank 0) ----------------
      const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
      int stage = 0, it = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < total && ok; t += nclusters, ++it) {
        const PairJob j = pair_job<MODE>(t, args, num_m, num_p, num_n, rank);
        const int n_mma = pair_n_mma(args.n - j.n_blk * kPairN);
        const uint32_t idesc =
            idesc_f16(Traits<T>::code == AGM_BF16, 2 * kBM, n_mma) | (A_MN ? (1u << 15) : 0u) | (1u << 16);
        const int acc = it & 1;
        if (!mbar_wait(&acc_empty[acc], ((it >> 1) & 1) ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
          *abort_s = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairN;
        for (int kb = 0; kb < j.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
            *abort_s = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = sA_addr + stage * kABytes;
            const uint64_t a_desc = A_MN ? smem_desc_mn_sw128(a_addr, kBox) : smem_desc_k_sw128(a_addr);
            const uint64_t b_desc = smem_desc_mn_sw128(sB_addr + stage * kBBytes, kBox);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t a_step = A_MN ? static_cast<uint64_t>(kk) * (2048 >> 4) : static_cast<uint64_t>(2 * kk);
              const uint64_t b_step = static_cast<uint64_t>(kk) * (2048 >> 4);
              umma_f16_pair(d_tmem, a_desc + a_step, b_desc + b_step, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        // An empty K range (an expert with no rows) issues no MMA: the commit
        // arrives at once and the epilogues write zeros.
        if (lane == 0) umma_commit_pair(&acc_full[acc], 0x3);
        __syncwarp();
      }
      if (lane == 0) umma_commit_pair(drain, 0x1);
      __syncwarp();
      mbar_wait(drain, 0, args.err, kErrTimeoutDrain);
    }
  } else {
    // ---------------- Epilogue (warps 2..9, both CTAs) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    uint8_t* stg = sStg + ew * kStgBytes;
    const uint32_t stg_row = lane * 128;
    const uint32_t acc_empty0 = cluster_map(smem_u32(acc_empty), 0);
    constexpr int kChunks = kPairN / 128;
    int it = 0;
    for (int t = cluster; t < total; t += nclusters, ++it) {
      const PairJob j = pair_job<MODE>(t, args, num_m, num_p, num_n, rank);
      const int acc = it & 1;
      const int n0 = j.n_blk * kPairN;
      const int n_valid = min(kPairN, args.n - n0);
      const int row0 = j.my_m * kBM + quarter * 32;
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
      if (MODE == 0 && leader && ew == 0 && lane == 0 && j.m0 + 1 < num_m && args.tile_group &&
          args.tile_group[j.m0 + 1] != args.tile_group[j.m0])
        raise_error(args.err, kErrPairGroup);  // segments not padded to 256 rows
      if (!mbar_wait(&acc_full[acc], (it >> 1) & 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const bool zero = (j.num_kb == 0);
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const int c64 = half + 2 * c;
        if (!j.store || c64 * 64 >= n_valid) break;
        const int col = c64 * 64;
        uint32_t r[64];
        if (!zero) {
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kPairN + col;
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
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (!((mbits[c][0] >> i) & 1u)) v[i] = 0.f;
            if (!((mbits[c][1] >> i) & 1u)) v[32 + i] = 0.f;
          }
        }
        if (MODE == 0 && args.col_part) {
          float s0, s1;
          warp_colsum64(v, lane, s0, s1);
          if (col + 2 * lane < n_valid)
            *reinterpret_cast<float2*>(args.col_part + (static_cast<int64_t>(j.my_m) * 4 + quarter) * args.n + n0 +
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
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&acc_empty[acc]);
        else
          mbar_arrive_remote(acc_empty0 + acc * 8);
      }
    }
    if (lane == 0) bulk_wait_group0();
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

CUtensorMapDataType tmap_dt(int code) {
  switch (code) {
    case AGM_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case AGM_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

template <typename T, typename OutT, int MODE, bool RELU_MASK>
cudaError_t launch_bwd_pair(const void* a, const void* b, int64_t a_rows, const BwdGemmArgs& args, int num_sms,
                            cudaStream_t stream) {
  const CUtensorMapDataType dt = tmap_dt(Traits<T>::code);
  const CUtensorMapDataType dto = tmap_dt(sizeof(OutT) == 4 ? AGM_F32 : Traits<T>::code);
  CUtensorMap tmA, tmB, tmC;
  if (MODE == 0) {
    {  // A: [a_rows, K] K-major
      const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(a_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.k) * 2};
      const uint32_t box[2] = {kBK, kBM};
      if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // B: W [G, K, N], N innermost
      const uint64_t dims[3] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.k),
                                static_cast<uint64_t>(args.groups)};
      const uint64_t str[2] = {static_cast<uint64_t>(args.n) * 2, static_cast<uint64_t>(args.n) * args.k * 2};
      const uint32_t box[3] = {64, kBK, 1};
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
      const uint32_t box[2] = {64, kBK};
      if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
    }
    {  // B: act [a_rows, N], N innermost
      const uint64_t dims[2] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(a_rows)};
      const uint64_t str[1] = {static_cast<uint64_t>(args.n) * 2};
      const uint32_t box[2] = {64, kBK};
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
  auto kern = grouped_gemm_bwd_pair_kernel<T, OutT, MODE, RELU_MASK>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmemBytes);
  if (e != cudaSuccess) return e;
  const int num_n = (args.n + kPairN - 1) / kPairN;
  const int64_t m_tiles = MODE == 0 ? args.max_tiles : (args.m + kBM - 1) / kBM;
  const int64_t units = (MODE == 0 ? 1 : args.groups) * ((m_tiles + 1) / 2) * num_n;
  int ctas = static_cast<int>(std::min<int64_t>(num_sms, 2 * std::max<int64_t>(1, units)));
  ctas = std::max(2, ctas & ~1);
  return launch_kernel(kern, dim3(ctas), dim3(kThreads), kSmemBytes, stream, tmA, tmB, tmC, args);
}

}  // namespace

cudaError_t grouped_gemm_dgrad_pair(int dtype, const void* dc, int64_t rows, const void* w, const BwdGemmArgs& args,
                                    bool relu_mask, int num_sms, cudaStream_t stream) {
  if (args.max_tiles <= 0 || args.n <= 0) return cudaSuccess;
  switch (dtype) {
    case AGM_BF16:
      return relu_mask ? launch_bwd_pair<__nv_bfloat16, __nv_bfloat16, 0, true>(dc, w, rows, args, num_sms, stream)
                       : launch_bwd_pair<__nv_bfloat16, __nv_bfloat16, 0, false>(dc, w, rows, args, num_sms, stream);
    case AGM_F16:
      return relu_mask ? launch_bwd_pair<__half, __half, 0, true>(dc, w, rows, args, num_sms, stream)
                       : launch_bwd_pair<__half, __half, 0, false>(dc, w, rows, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t grouped_gemm_wgrad_pair(int dtype, bool out_f32, const void* dc, const void* act, int64_t rows,
                                    const BwdGemmArgs& args, int num_sms, cudaStream_t stream) {
  if (args.groups <= 0 || args.m <= 0 || args.n <= 0) return cudaSuccess;
  switch (dtype) {
    case AGM_BF16:
      return out_f32 ? launch_bwd_pair<__nv_bfloat16, float, 1, false>(dc, act, rows, args, num_sms, stream)
                     : launch_bwd_pair<__nv_bfloat16, __nv_bfloat16, 1, false>(dc, act, rows, args, num_sms, stream);
    case AGM_F16:
      return out_f32 ? launch_bwd_pair<__half, float, 1, false>(dc, act, rows, args, num_sms, stream)
                     : launch_bwd_pair<__half, __half, 1, false>(dc, act, rows, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
