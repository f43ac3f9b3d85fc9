// K3: grouped GEMM over expert segments (the expert FFN projections).
//
// Replaces the per-expert `nn.Linear` calls of agillm41.py:4428 (expert =
// Linear(d,H) -> ReLU -> Linear(H,d), agillm41.py:4332-4336, run through
// `_run_expert`, 4367-4379): 2*E small cuBLAS GEMMs per rank in the reference
// become two launches of one persistent kernel here, FC1 (+b1, ReLU) and
// FC2 (+b2), each covering every expert segment.
//
//   C[r, n] = act( sum_k A[r, k] * W[g(r), n, k] + bias[g(r), n] )
//
// A: [rows, K] row-major (the permuted activations, segments padded to 128
// rows), W: [G, N, K] (nn.Linear weight layout, K contiguous), C: [rows, N].
// The group g(r) of a 128-row tile comes from a tile table that the dispatch
// kernel writes on the device, together with the number of valid tiles, so
// the forward needs no host sync.
//
// bf16/fp16 path (tcgen05, sm_100a): persistent CTAs (one per SM), 320
// threads: warp 0 issues TMA loads (128x64 A tile + BNx64 W tile per stage,
// 128-byte swizzle, one CTA per copy), warp 1 owns the TMEM allocation and issues
// tcgen05.mma (M=128, N=BN, K=16, fp32 accumulation in TMEM), warps 2-9 drain
// the accumulator (tcgen05.ld; two warps per TMEM lane quarter, alternate
// 64-column chunks), add the bias, apply ReLU, round to the activation dtype,
// stage each 32x64 chunk in shared memory (128-byte swizzle) and write it with
// a TMA store. The accumulator is double-buffered in TMEM (2 x BN columns) so
// the epilogue of one tile overlaps the MMAs of the next.
// Every mbarrier wait is bounded; on time-out the kernel records an error
// code, drains its in-flight copies and MMAs, frees TMEM and returns.
//
// fp32 path: a SIMT kernel (64x64 tiles, 4x4 outputs per thread, fp32 FMA),
// used for the reference's fp32 mode where tensor-core tf32 rounding would
// exceed the 1e-4 parity tolerance.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {

constexpr int BM = AGM_TILE_M;  // 128 rows per tile
constexpr int BK = 64;          // 64 x 16-bit = 128 B: one swizzle atom row
constexpr int kGroupM = 16;     // tile rasterisation: 16 row tiles per group
constexpr int kEpiWarps = 8;     // two epilogue warps per TMEM lane quarter
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kStgBytes = 32 * 64 * 2;  // one 32-row x 64-column output chunk (TMA store source)


template <int BN>
struct TcCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STG_BYTES = kEpiWarps * kStgBytes;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + 1024;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_blk, int& n_blk) {
  const int span = kGroupM * num_n;
  const int g = t / span;
  const int first_m = g * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = t - g * span;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

template <typename T, int BN, bool RELU>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmC, GemmArgs args) {
  using Cfg = TcCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sStg = smem + STAGES * Cfg::STAGE_BYTES;  // [8 warps][32 rows][128 B], 128-byte swizzled
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + Cfg::STG_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
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
  const int num_n = (args.n + BN - 1) / BN;
  const int total = num_m * num_n;
  const int num_kb = (args.k + BK - 1) / BK;

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
    uint32_t armed = 0;             // stages armed at least once
    uint32_t armed_parity = 0;      // parity of the last arming of each stage
    bool ok = true;
    // With early_weights, the first tile's first `ndef` stages get their
    // weight tile before the wait for the previous kernel and their A tile
    // after it.
    bool waited = !args.early_weights;
    const int ndef = min(STAGES, num_kb);
    int deferred = 0, first_m = 0;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int m_blk, n_blk;
      tile_coords(t, num_m, num_n, m_blk, n_blk);
      if (t == static_cast<int>(blockIdx.x)) first_m = m_blk;
      int g = args.tile_group ? args.tile_group[m_blk] : 0;
      if (g < 0 || g >= args.groups) g = 0;  // cannot happen: the plan kernel writes ids < groups
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_3d(sB + stage * Cfg::B_BYTES, &tmB, kb * BK, n_blk * BN, g, &full[stage]);
          if (waited) tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, kb * BK, m_blk * BM, &full[stage]);
        }
        if (!waited && ++deferred == ndef) {
          pdl_wait();
          pdl_trigger();
          waited = true;
          if (lane == 0)
            for (int j = 0; j < deferred; ++j) tma_load_2d(sA + j * Cfg::A_BYTES, &tmA, j * BK, first_m * BM, &full[j]);
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
    if (!waited) {  // no tile, or stopped early: still order after the previous kernel
      pdl_wait();
      pdl_trigger();
      if (lane == 0)
        for (int j = 0; j < deferred; ++j) tma_load_2d(sA + j * Cfg::A_BYTES, &tmA, j * BK, first_m * BM, &full[j]);
    }
    __syncwarp();
    // Drain: every armed stage's last load must have landed before exit.
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
      int m_blk, n_blk;
      tile_coords(t, num_m, num_n, m_blk, n_blk);
      const int n_valid = min(BN, args.n - n_blk * BN);
      const int n_mma = (n_valid + 15) / 16 * 16;
      const uint32_t idesc = idesc_f16(Traits<T>::code == AGM_BF16, BM, n_mma);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t a_desc = smem_desc_k_sw128(sA_addr + stage * Cfg::A_BYTES);
          const uint64_t b_desc = smem_desc_k_sw128(sB_addr + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // advance 16 elements (32 B) along K inside the swizzle atom
            umma_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (kb == num_kb - 1) umma_commit(&acc_full[acc]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Drain: wait for every MMA this thread issued before TMEM is freed.
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0, args.err, kErrTimeoutDrain);
  } else {
    // ---------------- Epilogue (warps 2..9) ----------------
    // Warp w reads TMEM lanes [32*(w%4), +32) (its quarter of the 128 rows);
    // warps 2-5 take the even 64-column chunks of the tile, warps 6-9 the odd
    // ones. A chunk (32 rows x 64 columns) is biased, activated, rounded,
    // written to this warp's staging buffer in the 128-byte swizzled layout
    // (conflict-free 16-byte stores) and sent to global memory with one TMA
    // store, which also clips rows/columns outside C.
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    uint8_t* stg = sStg + ew * kStgBytes;
    const uint32_t stg_row = lane * 128;
    int it = 0;
    const T* bias = static_cast<const T*>(args.bias);
    const bool want_bits = RELU && args.relu_bits != nullptr;  // training: keep the ReLU mask
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      int m_blk, n_blk;
      tile_coords(t, num_m, num_n, m_blk, n_blk);
      int g = args.tile_group ? args.tile_group[m_blk] : 0;
      if (g < 0 || g >= args.groups) g = 0;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase, args.err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const int n0 = n_blk * BN;
      const int n_valid = min(BN, args.n - n0);
      const T* brow = bias ? bias + static_cast<int64_t>(g) * args.n + n0 : nullptr;
      for (int c64 = half; c64 * 64 < n_valid; c64 += 2) {
        const int col = c64 * 64;
        uint32_t r[64];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + col;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        // The staging buffer is free once the previous chunk's TMA store has read it.
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
          // 128-byte swizzle: 16-byte chunk q of row `lane` lives at chunk q ^ (lane % 8).
          *reinterpret_cast<uint4*>(stg + stg_row + ((q ^ (lane & 7)) << 4)) = o;
        }
        if (RELU && want_bits) {
          // lanes are consecutive rows: each word row is one coalesced store
          const int64_t row = m_blk * BM + quarter * 32 + lane;
          const int w0 = (n0 + col) >> 5;
          args.relu_bits[static_cast<int64_t>(w0) * args.ld_bits + row] = static_cast<uint32_t>(bits);
          if (col + 32 < n_valid)
            args.relu_bits[static_cast<int64_t>(w0 + 1) * args.ld_bits + row] = static_cast<uint32_t>(bits >> 32);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, stg, n0 + col, m_blk * BM + quarter * 32);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
    if (lane == 0) {
      bulk_wait_group0();
      // The output may be read by other GPUs after a flag barrier: make the
      // async-proxy stores visible to generic and system-scope readers.
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
    }
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
// fp32 SIMT grouped GEMM (reference fp32 mode)
// ---------------------------------------------------------------------------
template <bool RELU>
__global__ void __launch_bounds__(256) grouped_gemm_f32_kernel(const float* __restrict__ A, int64_t a_rows,
                                                               const float* __restrict__ W, GemmArgs args) {
  constexpr int TM = 64, TN = 64, TK = 16;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  pdl_wait();
  pdl_trigger();
  int num_m = args.max_tiles;
  if (args.num_tiles) num_m = min(*args.num_tiles, args.max_tiles);
  const int tile = blockIdx.x / (BM / TM);
  if (tile >= num_m) return;
  const int sub = blockIdx.x % (BM / TM);
  int g = args.tile_group ? args.tile_group[tile] : 0;
  if (g < 0 || g >= args.groups) g = 0;
  const int64_t m0 = static_cast<int64_t>(tile) * BM + sub * TM;
  const int n0 = blockIdx.y * TN;
  const int N = args.n, K = args.k;
  const float* Wg = W + static_cast<int64_t>(g) * N * K;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int r = i / TK, kk = i % TK;
      const int64_t gr = m0 + r;
      As[kk][r] = (gr < a_rows && k0 + kk < K) ? A[gr * K + k0 + kk] : 0.f;
      const int n = n0 + r;
      Bs[kk][r] = (n < N && k0 + kk < K) ? Wg[static_cast<int64_t>(n) * K + k0 + kk] : 0.f;
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
  const float* bias = static_cast<const float*>(args.bias);
  float* C = static_cast<float*>(args.c);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (r >= args.c_rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j] + (bias ? bias[static_cast<int64_t>(g) * N + n] : 0.f);
      if (RELU) v = fmaxf(v, 0.f);
      C[r * args.ldc + n] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D/3-D row-major tensor of 16-bit elements: dims innermost first.
bool encode_tmap(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                        const uint32_t* box, CUtensorMapDataType dt) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn || rank < 1 || rank > 5) return false;
  cuuint64_t gdim[5], gstr[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  CUresult r = fn(m, dt, rank, const_cast<void*>(base), gdim, gstr, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int BN, bool RELU>
static cudaError_t launch_tc(const void* a, int64_t a_rows, const void* w, const GemmArgs& args, int num_sms,
                             cudaStream_t stream) {
  using Cfg = TcCfg<BN>;
  const CUtensorMapDataType dt = (Traits<T>::code == AGM_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tmA, tmB;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(a_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.k) * 2};
    const uint32_t box[2] = {BK, BM};
    if (!encode_tmap(&tmA, a, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(args.n),
                              static_cast<uint64_t>(args.groups)};
    const uint64_t str[2] = {static_cast<uint64_t>(args.k) * 2, static_cast<uint64_t>(args.k) * args.n * 2};
    const uint32_t box[3] = {BK, static_cast<uint32_t>(BN), 1};
    if (!encode_tmap(&tmB, w, 3, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  CUtensorMap tmC;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.c_rows)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.ldc) * 2};
    const uint32_t box[2] = {64, 32};
    if (!encode_tmap(&tmC, args.c, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(grouped_gemm_tc_kernel<T, BN, RELU>),
                                      Cfg::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int num_n = (args.n + BN - 1) / BN;
  const int64_t max_total = static_cast<int64_t>(args.max_tiles) * num_n;
  const int ctas = args.max_ctas > 0 ? std::min(args.max_ctas, num_sms) : num_sms;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas, max_total)));
  return launch_kernel(grouped_gemm_tc_kernel<T, BN, RELU>, dim3(grid), dim3(kGemmThreads), Cfg::SMEM_BYTES, stream,
                       tmA, tmB, tmC, args);
}

template <typename T, bool RELU>
static cudaError_t dispatch_bn(const void* a, int64_t a_rows, const void* w, const GemmArgs& args, int num_sms,
                               cudaStream_t stream, int force_bn) {
  // Few tiles (decode-sized problems): narrower tiles keep more SMs busy.
  const int64_t tiles256 = static_cast<int64_t>(args.max_tiles) * ((args.n + 255) / 256);
  const int bn = force_bn ? force_bn : (tiles256 >= 2 * num_sms ? 256 : 128);
  if (bn == 256) return launch_tc<T, 256, RELU>(a, a_rows, w, args, num_sms, stream);
  return launch_tc<T, 128, RELU>(a, a_rows, w, args, num_sms, stream);
}

cudaError_t grouped_gemm(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                         int num_sms, cudaStream_t stream, int force_bn) {
  if (args.max_tiles <= 0 || args.n <= 0) return cudaSuccess;
  if (force_bn == -1 && dtype != AGM_F32) return grouped_gemm_pair(dtype, a, a_rows, w, args, relu, num_sms, stream);
  if (force_bn == -2 && dtype != AGM_F32) return grouped_gemm_swap(dtype, a, a_rows, w, args, relu, num_sms, stream);
  if (force_bn < 0) force_bn = 0;
  if (dtype == AGM_F32) {
    dim3 grid(static_cast<unsigned>(args.max_tiles * (BM / 64)), static_cast<unsigned>((args.n + 63) / 64));
    const float* A = static_cast<const float*>(a);
    const float* W = static_cast<const float*>(w);
    return relu ? launch_kernel(grouped_gemm_f32_kernel<true>, grid, dim3(256), 0, stream, A, a_rows, W, args)
                : launch_kernel(grouped_gemm_f32_kernel<false>, grid, dim3(256), 0, stream, A, a_rows, W, args);
  }
  if (dtype == AGM_BF16) {
    return relu ? dispatch_bn<__nv_bfloat16, true>(a, a_rows, w, args, num_sms, stream, force_bn)
                : dispatch_bn<__nv_bfloat16, false>(a, a_rows, w, args, num_sms, stream, force_bn);
  }
  if (dtype == AGM_F16) {
    return relu ? dispatch_bn<__half, true>(a, a_rows, w, args, num_sms, stream, force_bn)
                : dispatch_bn<__half, false>(a, a_rows, w, args, num_sms, stream, force_bn);
  }
  return cudaErrorInvalidValue;
}

}  // namespace agm
