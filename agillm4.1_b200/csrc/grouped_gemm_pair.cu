// K3 on CTA pairs: the grouped GEMM of grouped_gemm.cu with 256 x 256 tiles
// computed by a cluster of two CTAs (one TPC) through tcgen05.mma with
// cta_group::2.
//
//   C[r, n] = act( sum_k A[r, k] * W[g(r), n, k] + bias[g(r), n] )
//
// Why pairs: a 128 x 256 tile on one SM streams 48 KB of operands into shared
// memory per 64-deep k-block; its 4-stage ring then holds too few bytes in
// flight to cover the L2 latency (ncu: tensor pipe 66-74% busy while shared
// memory, L2 and DRAM are all below 60%). A pair computes a 256 x 256 tile:
// each CTA loads its own 128 rows of A and one half (128 columns) of the
// weight tile, i.e. 32 KB per k-block instead of 48 KB for the same tensor
// work per SM, and the freed shared memory gives a 6-stage ring.
//
// Work unit: row tiles 2p and 2p+1 (128 rows each, from the device tile
// table) x one 256-column tile. Both row tiles must use the same weight
// group: the dispatch plan pads every expert segment to 256 rows for this
// kernel (a pair whose groups differ raises kErrPairGroup and is computed
// with the first tile's group). When the tile count is odd the last pair has
// no second tile: the peer CTA then repeats the first tile's rows and stores
// nothing.
//
// A second, dense problem may share the launch (GemmArgs::groups2 > 0: the
// shared experts of a MoE block, every token through each of them): its
// units follow the first problem's, with their own tensor maps, N, K, bias
// and per-group row offsets, so the block's routed and shared projections
// take one launch each and the shared units fill the routed tail.
//
// Roles (320 threads per CTA, both CTAs):
//   warp 0   TMA producer: waits for a free stage (its own `empty` barrier,
//            released by the pair MMA's commit), loads its A rows and B half
//            and counts the bytes on rank 0's `full` barrier (rank 0 arms it
//            with the bytes of both CTAs).
//   warp 1   rank 0: issues tcgen05.mma (M=256, K=16, N=256 or, on a ragged
//            last column tile, its columns rounded up to 32) and commits to
//            both CTAs' `empty` / `acc_full` barriers; both ranks: allocate
//            and free the pair's tensor memory (2 x 256 accumulator columns).
//   warps 2-9  epilogue of this CTA's 128 rows (same code as the one-CTA
//            kernel: tcgen05.ld, bias, ReLU, round, swizzled staging, TMA
//            store), then one arrive per warp on rank 0's `acc_empty`.
// Every mbarrier wait is bounded; both CTAs always reach the final cluster
// barrier, after which tensor memory is freed.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {

namespace {

constexpr int kBM = AGM_TILE_M;        // 128 rows per CTA, 256 per pair
constexpr int kBK = 64;
constexpr int kPairN = 256;            // columns per pair tile (128 of B per CTA)
constexpr int kHalfN = kPairN / 2;
constexpr int kStages = 6;
constexpr int kGroupPairs = 8;         // rasterisation: 8 pairs (16 row tiles) per group
constexpr int kEpi = 8;                // epilogue warps
constexpr int kThreads = 64 + 32 * kEpi;
constexpr int kABytes = kBM * kBK * 2;      // 16 KB
constexpr int kBBytes = kHalfN * kBK * 2;   // 16 KB
constexpr int kStgBytes = 32 * 64 * 2;      // one 32 x 64 output chunk per epilogue warp
constexpr int kTmemCols = 2 * kPairN;       // double-buffered accumulator
constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + kEpi * kStgBytes + 256 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "pair GEMM shared memory");

// Columns one pair MMA computes for a column tile with n_valid columns: a
// multiple of 32 (each CTA then holds a multiple of 16 weight rows), so the
// ragged last tile (FC1: 3200 = 12 x 256 + 128) does only the work it needs.
__device__ __forceinline__ int pair_n_mma(int n_valid) { return min(kPairN, (n_valid + 31) / 32 * 32); }

__device__ __forceinline__ void pair_coords(int t, int num_p, int num_n, int& p, int& n_blk) {
  const int span = kGroupPairs * num_n;
  const int grp = t / span;
  const int first = grp * kGroupPairs;
  const int gp = min(num_p - first, kGroupPairs);
  const int r = t - grp * span;
  p = first + r % gp;
  n_blk = r / gp;
}

// One work unit: a pair of row tiles x one 256-column tile, of the first
// (grouped, tile-table) problem or of the optional second (dense) problem.
struct PairUnit {
  int prob;     // 0 or 1
  int m0;       // first row tile of the pair (problem 0: tile-table index; problem 1: tile within its group)
  int n_blk;    // column tile
  int g;        // weight group
  int row0;     // A / C row of tile m0 (problem 1: includes the group's offsets via a_off / c_off)
  int a_off;    // problem 1: the group's A row offset
  int c_off;    // problem 1: the group's C row offset
  bool has2;    // tile m0 + 1 exists
  int n;        // columns of the problem
  int k;        // inner dimension of the problem
};

__device__ __forceinline__ PairUnit pair_unit(int t, int total0, int num_p, int num_m, int num_n, int num_p2,
                                              int num_n2, const GemmArgs& args) {
  PairUnit u;
  if (t < total0) {
    int p, n_blk;
    pair_coords(t, num_p, num_n, p, n_blk);
    u.prob = 0;
    u.m0 = 2 * p;
    u.n_blk = n_blk;
    int g = args.tile_group ? args.tile_group[u.m0] : 0;
    u.g = (g < 0 || g >= args.groups) ? 0 : g;
    u.row0 = u.m0 * kBM;
    u.a_off = u.c_off = 0;
    u.has2 = u.m0 + 1 < num_m;
    u.n = args.n;
    u.k = args.k;
  } else {
    const int t2 = t - total0;
    const int per_group = num_p2 * num_n2;
    const int g = t2 / per_group;
    int p, n_blk;
    pair_coords(t2 - g * per_group, num_p2, num_n2, p, n_blk);
    u.prob = 1;
    u.m0 = 2 * p;
    u.n_blk = n_blk;
    u.g = g;
    u.row0 = u.m0 * kBM;
    u.a_off = static_cast<int>(g * args.a2_group_rows);
    u.c_off = static_cast<int>(g * args.c2_group_rows);
    u.has2 = u.m0 + 1 < args.tiles2;
    u.n = args.n2;
    u.k = args.k2;
  }
  return u;
}

template <typename T, bool RELU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmA2,
                             const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmC2,
                             GemmArgs args) {
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
  const int num_n = (args.n + kPairN - 1) / kPairN;
  const int total0 = num_p * num_n;
  const int num_p2 = args.groups2 > 0 ? (args.tiles2 + 1) / 2 : 0;
  const int num_n2 = args.groups2 > 0 ? (args.n2 + kPairN - 1) / kPairN : 0;
  const int total = total0 + args.groups2 * num_p2 * num_n2;

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
    if (args.groups2 > 0) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
      tma_prefetch_desc(&tmC2);
    }
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
    // weight half-tile before the wait for the previous kernel and their A
    // rows after it.
    bool waited = !args.early_weights;
    int deferred = 0, ndef = 0, first_row = 0;
    const CUtensorMap* first_a = &tmA;
    uint32_t src_ready = 0;  // sources whose rows are known to have arrived (tile_src)
    for (int t = cluster; t < total && ok; t += nclusters) {
      const PairUnit u = pair_unit(t, total0, num_p, num_m, num_n, num_p2, num_n2, args);
      if (u.prob == 0 && args.tile_src) {
        // Expert parallelism: wait (bounded) for the source's "rows
        // delivered" release before the first load of one of its tiles; the
        // proxy fence orders the TMA reads after that acquire.
        const int src = args.tile_src[u.m0];
        if (src >= 0 && src < 32 && !((src_ready >> src) & 1u)) {
          if (lane == 0 && ld_acquire_sys(args.src_signal + src) < args.src_epoch) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys(args.src_signal + src) < args.src_epoch) {
              if (globaltimer_ns() - t0 > AGM_WAIT_LIMIT_NS) {
                raise_error(args.err, kErrTimeoutFull);
                *abort_s = 1;
                break;
              }
              __nanosleep(128);
            }
          }
          if (lane == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
          __syncwarp();
          if (*abort_s) {
            ok = false;
            break;
          }
          src_ready |= 1u << src;
        }
      }
      const CUtensorMap* mA = u.prob ? &tmA2 : &tmA;
      const CUtensorMap* mB = u.prob ? &tmB2 : &tmB;
      // Rank 1 loads the pair's second row tile (or repeats the first when there is none).
      const int a_row = u.a_off + (u.m0 + ((!leader && u.has2) ? 1 : 0)) * kBM;
      const int num_kb = (u.k + kBK - 1) / kBK;
      if (t == cluster) {
        first_row = a_row;
        first_a = mA;
        ndef = min(kStages, num_kb);
      }
      // Rank r holds weight rows [n0 + r * n_mma / 2, +n_mma / 2) of the tile
      // (its 128-row box may run past them; the MMA reads only n_mma / 2).
      const int b_row = u.n_blk * kPairN + static_cast<int>(rank) * (pair_n_mma(u.n - u.n_blk * kPairN) / 2);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (kABytes + kBBytes));
          const uint32_t fb = full0 + stage * 8;
          tma_load_3d_pair(sB + stage * kBBytes, mB, kb * kBK, b_row, u.g, fb);
          if (waited) tma_load_2d_pair(sA + stage * kABytes, mA, kb * kBK, a_row, fb);
        }
        if (!waited && ++deferred == ndef) {
          pdl_wait();
          pdl_trigger();
          waited = true;
          if (lane == 0)
            for (int j = 0; j < deferred; ++j)
              tma_load_2d_pair(sA + j * kABytes, first_a, j * kBK, first_row, full0 + j * 8);
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
          tma_load_2d_pair(sA + j * kABytes, first_a, j * kBK, first_row, full0 + j * 8);
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
      const uint32_t sA_addr = smem_u32(sA), sB_addr = smem_u32(sB);
      int stage = 0, it = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < total && ok; t += nclusters, ++it) {
        const PairUnit u = pair_unit(t, total0, num_p, num_m, num_n, num_p2, num_n2, args);
        const int num_kb = (u.k + kBK - 1) / kBK;
        const uint32_t idesc = idesc_f16(Traits<T>::code == AGM_BF16, 2 * kBM, pair_n_mma(u.n - u.n_blk * kPairN));
        const int acc = it & 1;
        if (!mbar_wait(&acc_empty[acc], ((it >> 1) & 1) ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
          *abort_s = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
            *abort_s = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t a_desc = smem_desc_k_sw128(sA_addr + stage * kABytes);
            const uint64_t b_desc = smem_desc_k_sw128(sB_addr + stage * kBBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16_pair(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(&empty[stage], 0x3);
            if (kb == num_kb - 1) umma_commit_pair(&acc_full[acc], 0x3);
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
    const int half = ew >> 2;
    uint8_t* stg = sStg + ew * kStgBytes;
    const uint32_t stg_row = lane * 128;
    const uint32_t acc_empty0 = cluster_map(smem_u32(acc_empty), 0);
    int it = 0;
    for (int t = cluster; t < total; t += nclusters, ++it) {
      const PairUnit u = pair_unit(t, total0, num_p, num_m, num_n, num_p2, num_n2, args);
      const int my_m = leader ? u.m0 : u.m0 + 1;
      const bool store = leader || u.has2;
      const T* bias = static_cast<const T*>(u.prob ? args.bias2 : args.bias);
      const CUtensorMap* mC = u.prob ? &tmC2 : &tmC;
      // training (first problem only): keep the ReLU mask
      const bool want_bits = RELU && u.prob == 0 && args.relu_bits != nullptr;
      const bool to_tiles = u.prob == 0 && args.tile_dst != nullptr;
      if (u.prob == 0 && leader && ew == 0 && lane == 0 && u.has2 && args.tile_group &&
          args.tile_group[u.m0 + 1] != args.tile_group[u.m0])
        raise_error(args.err, kErrPairGroup);
      const int acc = it & 1;
      if (!mbar_wait(&acc_full[acc], (it >> 1) & 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const int n0 = u.n_blk * kPairN;
      const int n_valid = min(kPairN, u.n - n0);
      const T* brow = bias ? bias + static_cast<int64_t>(u.g) * u.n + n0 : nullptr;
      const int c_row = u.c_off + my_m * kBM + quarter * 32;
      for (int c64 = half; store && c64 * 64 < n_valid; c64 += 2) {
        const int col = c64 * 64;
        uint32_t r[64];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kPairN + col;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
        uint64_t bits = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float bv[8];
          if (brow && col + q * 8 < n_valid) {
            const uint4 bu = __ldg(reinterpret_cast<const uint4*>(brow + col + q * 8));
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
            if (RELU && want_bits && round_to<T>(v[j]) > 0.f) bits |= 1ull << (q * 8 + j);
          }
          const uint4 o = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]),
                                     pack2<T>(v[6], v[7]));
          *reinterpret_cast<uint4*>(stg + stg_row + ((q ^ (lane & 7)) << 4)) = o;
        }
        if (RELU && want_bits) {
          // lanes are consecutive rows: each word row is one coalesced store
          const int64_t row = my_m * kBM + quarter * 32 + lane;
          const int w0 = (n0 + col) >> 5;
          args.relu_bits[static_cast<int64_t>(w0) * args.ld_bits + row] = static_cast<uint32_t>(bits);
          if (col + 32 < n_valid)
            args.relu_bits[static_cast<int64_t>(w0 + 1) * args.ld_bits + row] = static_cast<uint32_t>(bits >> 32);
        }
        if (to_tiles) {
          // This tile's rows go to their own buffer (expert parallelism: the
          // token owner's home rows, possibly in a peer GPU's memory): read
          // the staged chunk back unswizzled, 4 rows of 128 B per store.
          __syncwarp();
          uint8_t* dst = reinterpret_cast<uint8_t*>(args.tile_dst[my_m]) +
                         (static_cast<int64_t>(quarter * 32) * args.ldc + n0 + col) * sizeof(T);
          const int sub = lane >> 3, q = lane & 7;
          const bool col_ok = col + q * 8 < n_valid;
#pragma unroll
          for (int itr = 0; itr < 8; ++itr) {
            const int rr = itr * 4 + sub;
            const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((q ^ (rr & 7)) << 4));
            if (col_ok) *reinterpret_cast<uint4*>(dst + (static_cast<int64_t>(rr) * args.ldc + q * 8) * sizeof(T)) = v;
          }
          __syncwarp();
        } else {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(mC, stg, n0 + col, c_row);
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
    if (lane == 0) {
      bulk_wait_group0();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
    }
    if (args.tile_dst) __threadfence_system();  // every lane stored rows, some into peers' memory
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

template <typename T>
bool encode_pair_maps(const void* a, int64_t a_rows, const void* w, void* c, int64_t c_rows, int64_t ldc, int n,
                      int k, int groups, CUtensorMap* tmA, CUtensorMap* tmB, CUtensorMap* tmC) {
  const CUtensorMapDataType dt = (Traits<T>::code == AGM_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(a_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(k) * 2};
    const uint32_t box[2] = {kBK, kBM};
    if (!encode_tmap(tmA, a, 2, dims, str, box, dt)) return false;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n), static_cast<uint64_t>(groups)};
    const uint64_t str[2] = {static_cast<uint64_t>(k) * 2, static_cast<uint64_t>(k) * n * 2};
    const uint32_t box[3] = {kBK, kHalfN, 1};
    if (!encode_tmap(tmB, w, 3, dims, str, box, dt)) return false;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(n), static_cast<uint64_t>(c_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(ldc) * 2};
    const uint32_t box[2] = {64, 32};
    if (!encode_tmap(tmC, c, 2, dims, str, box, dt)) return false;
  }
  return true;
}

template <typename T, bool RELU>
cudaError_t launch_pair(const void* a, int64_t a_rows, const void* w, const GemmArgs& args, int num_sms,
                        cudaStream_t stream) {
  CUtensorMap tmA, tmB, tmC, tmA2, tmB2, tmC2;
  if (!encode_pair_maps<T>(a, a_rows, w, args.c, args.c_rows, args.ldc, args.n, args.k, args.groups, &tmA, &tmB,
                           &tmC))
    return cudaErrorInvalidValue;
  if (args.groups2 > 0) {
    if (args.tiles2 <= 0 || !args.a2 || !args.w2 || !args.c2 || args.n2 <= 0 || args.k2 <= 0)
      return cudaErrorInvalidValue;
    if (!encode_pair_maps<T>(args.a2, args.a2_rows, args.w2, args.c2, args.c2_rows, args.ldc2, args.n2, args.k2,
                             args.groups2, &tmA2, &tmB2, &tmC2))
      return cudaErrorInvalidValue;
  } else {
    tmA2 = tmA;
    tmB2 = tmB;
    tmC2 = tmC;
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(grouped_gemm_pair_kernel<T, RELU>), kSmemBytes);
  if (e != cudaSuccess) return e;
  const int num_n = (args.n + kPairN - 1) / kPairN;
  int64_t max_units = static_cast<int64_t>((args.max_tiles + 1) / 2) * num_n;
  if (args.groups2 > 0)
    max_units += static_cast<int64_t>(args.groups2) * ((args.tiles2 + 1) / 2) * ((args.n2 + kPairN - 1) / kPairN);
  int ctas = args.max_ctas > 0 ? std::min(args.max_ctas, num_sms) : num_sms;
  ctas = static_cast<int>(std::min<int64_t>(ctas, 2 * std::max<int64_t>(1, max_units)));
  ctas = std::max(2, ctas & ~1);
  return launch_kernel(grouped_gemm_pair_kernel<T, RELU>, dim3(ctas), dim3(kThreads), kSmemBytes, stream, tmA, tmB,
                       tmC, tmA2, tmB2, tmC2, args);
}

}  // namespace

cudaError_t grouped_gemm_pair(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                              int num_sms, cudaStream_t stream) {
  switch (dtype) {
    case AGM_BF16:
      return relu ? launch_pair<__nv_bfloat16, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_pair<__nv_bfloat16, false>(a, a_rows, w, args, num_sms, stream);
    case AGM_F16:
      return relu ? launch_pair<__half, true>(a, a_rows, w, args, num_sms, stream)
                  : launch_pair<__half, false>(a, a_rows, w, args, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace agm
