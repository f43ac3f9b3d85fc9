// K1: router logits + top-k + gates + per-block expert histogram.
//
// Replaces agillm41.py:4398-4419 (router Linear, `.float()`, `topk` on the
// fp32 logits and `softmax` over the k chosen values cast to the activation
// dtype; top-1: `softmax` over all experts and `argmax`, agillm41.py:4401-4416).
//
// bf16 / fp16 (router_tc_kernel): the logits are a [N, d] x [d, E] product, so
// they run on the 5th-generation tensor cores while x streams from HBM once:
// persistent CTAs (two per SM) walk 128-token tiles; warp 0 streams 128x64
// tiles of x through a 4-stage TMA ring, the router weight [E <= 16, d]
// stays resident in shared memory (TMA zero-fills rows E..15), warp 1 issues
// tcgen05.mma M=128 N=16 K=16 with fp32 accumulation into TMEM (two 16-column
// buffers), and each of the 128 epilogue threads reads the 16 logits of its
// token (its TMEM lane) with one tcgen05.ld, rounds them like the reference's
// bf16/fp16 GEMM output and selects top-k in registers.
//
// fp32, or logits supplied by the caller (router_topk_kernel): a SIMT kernel,
// one CTA per 128 tokens, 4 tokens per warp iteration, 16-byte vector loads
// and a transpose-reduce over the lanes.
//
// Both kernels share the per-token selection (route_warp): it follows
// torch.topk and torch's warp softmax so gates match bit for bit when the
// logits do, and writes one histogram row per 128-token dispatch block.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "route_math.cuh"

namespace agm {

constexpr int kDispatchBlock = AGM_DISPATCH_BLOCK;  // 128 tokens
constexpr int kRouterWarps = kDispatchBlock / 32;
constexpr int kMaxExperts = AGM_MAX_EXPERTS;       // 16
constexpr int kTokGroup = 4;


// Per-token selection state: top_k = KC in 1..4 is a compile-time constant
// (arrays of pow2_ceil(KC)); KC = 0 takes top_k at run time (arrays of 16).
// Every loop is fully unrolled with predicates so the arrays stay in registers.
template <int KC>
struct RouteK {
  static constexpr int S = KC > 0 ? pow2_ceil(KC) : kMaxExperts;
};
constexpr int kFastTopK = 4;

// Selection and gates of one token from its fp32 logits lg[0..E) (already
// rounded like the reference's router output).
//
// top-k (k >= 2) reproduces torch.topk(sorted=True) on a CUDA device: the
// selected set is every value greater than the k-th largest plus, among the
// values equal to it, the lowest expert indices; the result is ordered by
// descending value and, among exactly-equal values, by DESCENDING expert
// index (measured on B200 with torch 2.11 for k = 2 and 3: 100% of ~120k tied
// rows). `low_first` orders exactly-equal values by ascending index instead.
// The gates are softmax over the k chosen values (agillm41.py:4417-4419).
//
// top-1: probs = softmax(scores) (torch's warp softmax over next_pow2(E)
// lanes, padding contributes exp(-inf) = 0), chosen = argmax(probs), first
// index on ties, straight-through gate 1 (agillm41.py:4401-4416).
template <int KC>
__device__ __forceinline__ void select_route(const float (&lg)[kMaxExperts], int E, int k, bool low_first,
                                             int (&sel)[RouteK<KC>::S], float (&gate)[RouteK<KC>::S]) {
  constexpr int S = RouteK<KC>::S;
  if (KC > 0) k = KC;
#pragma unroll
  for (int r = 0; r < S; ++r) {
    sel[r] = -1;
    gate[r] = 0.f;
  }
  if (k == 1) {
    float ex[kMaxExperts];
    const float s = softmax_terms(lg, E, ex);
    int best = 0;
    float bp = ex[0] / s;
#pragma unroll
    for (int e = 1; e < kMaxExperts; ++e) {
      if (e < E) {
        const float p = ex[e] / s;
        if (p > bp || (isnan(p) && !isnan(bp))) {
          bp = p;
          best = e;
        }
      }
    }
    sel[0] = best;
    gate[0] = 1.f;  // gate / gate.detach() == 1
    return;
  }
  float val[S];
  uint32_t taken = 0;
#pragma unroll
  for (int r = 0; r < S; ++r) {
    val[r] = 0.f;
    if (r < k) {
      int best = -1;
      float bv = 0.f;
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) {
        if (e < E && !((taken >> e) & 1u)) {
          const float v = lg[e];
          // NaN compares greater than everything in torch's topk ordering.
          if (best < 0 || v > bv || (isnan(v) && !isnan(bv))) {
            best = e;
            bv = v;
          }
        }
      }
      if (best >= 0) taken |= 1u << best;
      sel[r] = best;
      val[r] = bv;
    }
  }
  if (!low_first) {
    // Runs of exactly-equal values come out in ascending index order; an
    // odd-even pass sort that only swaps equal neighbours reverses each run.
#pragma unroll
    for (int pass = 0; pass < S; ++pass) {
#pragma unroll
      for (int j = pass & 1; j + 1 < S; j += 2) {
        if (j + 1 < k && val[j] == val[j + 1] && sel[j] < sel[j + 1]) {
          const int t = sel[j];
          sel[j] = sel[j + 1];
          sel[j + 1] = t;
        }
      }
    }
  }
  // softmax over the k values (sorted descending, so val[0] is the max).
  topk_gates<KC, S>(val, k, gate);
}

// One warp's 32 tokens (one per lane; `valid` false past the end): writes the
// logits (optional), expert indices and gates, and the warp's expert counts
// into hist_row[0..16) from ballots, without shared-memory atomics.
template <typename T, int KC>
__device__ __forceinline__ void route_warp(const float (&lg)[kMaxExperts], bool valid, int E, int k, bool low_first,
                                           int64_t tok, float* __restrict__ logits_out,
                                           int32_t* __restrict__ idx_out, T* __restrict__ gates_out, int* hist_row,
                                           int* err) {
  constexpr int S = RouteK<KC>::S;
  if (KC > 0) k = KC;
  int sel[S];
  float gate[S];
  if (valid) {
    if (logits_out) {
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e)
        if (e < E) logits_out[tok * E + e] = lg[e];
    }
    select_route<KC>(lg, E, k, low_first, sel, gate);
#pragma unroll
    for (int r = 0; r < S; ++r) {
      if (r < k) {
        const int e = sel[r];
        if (e < 0 || e >= E) {
          raise_error(err, kErrBadExpert);
          sel[r] = -1;
        } else {
          idx_out[tok * k + r] = e;
          gates_out[tok * k + r] = Traits<T>::from_f(gate[r]);
        }
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < S; ++r) sel[r] = -1;
  }
  const int lane = lane_id();
  int c = 0;
#pragma unroll
  for (int r = 0; r < S; ++r) {
    if (r < k) {  // k is uniform over the warp
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e) {
        const uint32_t b = __ballot_sync(0xffffffffu, sel[r] == e);
        if (lane == e) c += __popc(b);
      }
    }
  }
  if (lane < kMaxExperts) hist_row[lane] = c;
}

// ---------------------------------------------------------------------------
// SIMT router (fp32, or caller-supplied logits)
// ---------------------------------------------------------------------------
template <typename T, int KC>
__global__ void __launch_bounds__(kDispatchBlock) router_topk_kernel(
    const T* __restrict__ x, const T* __restrict__ w, int64_t n_tokens, int d, int E, int k, int tie_low_first,
    const float* __restrict__ logits_in, float* __restrict__ logits_out, int32_t* __restrict__ idx_out,
    T* __restrict__ gates_out, int32_t* __restrict__ block_hist, int* err) {
  extern __shared__ __align__(16) float smem_f[];
  constexpr int CH = 16 / sizeof(T);  // elements per 16-byte chunk
  const int nchunk = d / CH;
  const bool compute = (logits_in == nullptr);
  pdl_wait();
  pdl_trigger();
  // Dynamic smem: [E][d] fp32 router weight (only when computing logits),
  // then [warps][32 tokens][16] fp32 logits.
  float* w_s = smem_f;
  float* logit_s = smem_f + (compute ? E * d : 0);
  __shared__ int hist_w[kRouterWarps][kMaxExperts];

  const int warp = warp_id(), lane = lane_id();

  if (compute) {
    // Stage W (vectorised, 16 B per thread per step), converting to fp32.
    const int total_chunks = E * nchunk;
    for (int c = threadIdx.x; c < total_chunks; c += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(w)[c];
      float f[8];
      if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
      } else {
        unpack8<T>(u, f);
      }
#pragma unroll
      for (int j = 0; j < CH; ++j) w_s[c * CH + j] = f[j];
    }
  }
  __syncthreads();

  // Persistent over 128-token blocks: W is staged once per CTA.
  float* my_logits = logit_s + warp * 32 * kMaxExperts;
  const int64_t nblk = (n_tokens + kDispatchBlock - 1) / kDispatchBlock;
  for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
  const int64_t warp_tok0 = blk * kDispatchBlock + warp * 32;

  if (compute) {
    for (int g = 0; g < 32; g += kTokGroup) {
      float acc[kTokGroup][kMaxExperts];
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t)
#pragma unroll
        for (int e = 0; e < kMaxExperts; ++e) acc[t][e] = 0.f;

      // The next chunk's x vectors are loaded before this chunk's FMAs (two
      // chunks of loads in flight per lane).
      uint4 u_next[kTokGroup];
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t) {
        const int64_t tok = warp_tok0 + g + t;
        u_next[t] = (lane < nchunk && tok < n_tokens) ? __ldg(reinterpret_cast<const uint4*>(x + tok * d) + lane)
                                                      : make_uint4(0, 0, 0, 0);
      }
      for (int c = lane; c < nchunk; c += 32) {
        float xf[kTokGroup][8];
        uint4 u_cur[kTokGroup];
#pragma unroll
        for (int t = 0; t < kTokGroup; ++t) u_cur[t] = u_next[t];
        const int cn = c + 32;
#pragma unroll
        for (int t = 0; t < kTokGroup; ++t) {
          const int64_t tok = warp_tok0 + g + t;
          u_next[t] = (cn < nchunk && tok < n_tokens) ? __ldg(reinterpret_cast<const uint4*>(x + tok * d) + cn)
                                                       : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int t = 0; t < kTokGroup; ++t) {
          const uint4 u = u_cur[t];
          if constexpr (sizeof(T) == 4) {
            xf[t][0] = __uint_as_float(u.x); xf[t][1] = __uint_as_float(u.y);
            xf[t][2] = __uint_as_float(u.z); xf[t][3] = __uint_as_float(u.w);
          } else {
            unpack8<T>(u, xf[t]);
          }
        }
#pragma unroll
        for (int e = 0; e < kMaxExperts; ++e) {
          if (e < E) {
            const float4* wp = reinterpret_cast<const float4*>(w_s + e * d + c * CH);
            float wf[8];
#pragma unroll
            for (int q = 0; q < CH / 4; ++q) {
              const float4 v = wp[q];
              wf[4 * q] = v.x; wf[4 * q + 1] = v.y; wf[4 * q + 2] = v.z; wf[4 * q + 3] = v.w;
            }
#pragma unroll
            for (int t = 0; t < kTokGroup; ++t)
#pragma unroll
              for (int j = 0; j < CH; ++j) acc[t][e] = fmaf(xf[t][j], wf[j], acc[t][e]);
          }
        }
      }
      // Transpose-reduce: after the xor-16/8/4/2 steps lane l holds a partial
      // sum of expert e(l) = 8*b4 + 4*b3 + 2*b2 + b1 (b = bits of l); the
      // xor-1 step completes it.
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t) {
        float v8[8], v4[4], v2[2];
        const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float send = u16 ? acc[t][i] : acc[t][i + 8];
          const float keep = u16 ? acc[t][i + 8] : acc[t][i];
          v8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float send = u8 ? v8[i] : v8[i + 4];
          const float keep = u8 ? v8[i + 4] : v8[i];
          v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float send = u4 ? v4[i] : v4[i + 2];
          const float keep = u4 ? v4[i + 2] : v4[i];
          v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        float v1;
        {
          const float send = u2 ? v2[0] : v2[1];
          const float keep = u2 ? v2[1] : v2[0];
          v1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        const float s = v1 + __shfl_xor_sync(0xffffffffu, v1, 1);
        const int e = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
        if ((lane & 1) == 0) my_logits[(g + t) * kMaxExperts + e] = round_to<T>(s);
      }
    }
  } else {
    for (int i = lane; i < 32 * E; i += 32) {
      const int t = i / E, e = i - t * E;
      const int64_t tok = warp_tok0 + t;
      my_logits[t * kMaxExperts + e] = (tok < n_tokens) ? logits_in[tok * E + e] : 0.f;
    }
  }
  __syncwarp();

  // One thread per token: selection, gates, histogram.
  const int64_t tok = warp_tok0 + lane;
  float lg[kMaxExperts];
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) lg[e] = (e < E) ? my_logits[lane * kMaxExperts + e] : 0.f;
  route_warp<T, KC>(lg, tok < n_tokens, E, k, tie_low_first != 0, tok, logits_out, idx_out, gates_out, hist_w[warp],
                    err);
  __syncthreads();
  if (threadIdx.x < E) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < kRouterWarps; ++w) c += hist_w[w][threadIdx.x];
    block_hist[blk * E + threadIdx.x] = c;
  }
  __syncthreads();  // logit_s and hist_w are reused by the next block
  }
}

// ---------------------------------------------------------------------------
// Tensor-core router (bf16 / fp16): TMA-fed tcgen05, thread-per-token epilogue
// ---------------------------------------------------------------------------
// Stages of the x ring: 4 with two CTAs per SM (8 x 16 KB of x in flight per
// SM) when CTAs walk several tiles; 10 with one CTA per SM when every CTA has
// at most one tile (small batches), so most of a tile's k-blocks are in
// flight at once instead of arriving in 5 serial round trips.
constexpr int kRtStages = 4;
constexpr int kRtStagesDeep = 10;
constexpr int kRtThreads = 192;
constexpr int kRtABytes = 128 * 64 * 2;   // one 128-token x 64-feature tile
constexpr int kRtWBytes = 16 * 64 * 2;    // one 16-expert x 64-feature tile of the router weight

__host__ __device__ constexpr int rt_smem_bytes(int nkb, int stages = kRtStages) {
  return stages * kRtABytes + nkb * kRtWBytes + 1024 + 1024;
}

template <typename T, int KC, int STAGES>
__global__ void __launch_bounds__(kRtThreads, STAGES == kRtStages ? 2 : 1) router_tc_kernel(
    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, int64_t n_tokens, int d,
    int E, int k, int tie_low_first, float* __restrict__ logits_out, int32_t* __restrict__ idx_out,
    T* __restrict__ gates_out, int32_t* __restrict__ block_hist, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nkb = (d + 63) / 64;
  uint8_t* sA = smem;
  uint8_t* sW = smem + STAGES * kRtABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + nkb * kRtWBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* w_full = acc_empty + 2;
  uint64_t* drain = w_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Per-warp expert counts, one set per accumulator buffer: [2][4 warps][16],
  // then one "an epilogue warp gave up" flag per buffer.
  int* hist_w = reinterpret_cast<int*>(bars + 32);  // past up to 26 barriers and the two words after them
  volatile int* epi_fail = hist_w + 2 * 4 * kMaxExperts;

  const int warp = warp_id(), lane = lane_id();
  const int num_tiles = static_cast<int>((n_tokens + 127) / 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(w_full, 1);
    mbar_init(drain, 1);
    *abort_s = 0;
    epi_fail[0] = epi_fail[1] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Setup above overlaps the previous kernel; x, the router weight and the
  // outputs are touched only after it has completed.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(w_full, nkb * kRtWBytes);
      for (int kb = 0; kb < nkb; ++kb) tma_load_2d(sW + kb * kRtWBytes, &tmW, kb * 64, 0, w_full);
    }
    int stage = 0;
    uint32_t phase = 0, armed = 0, armed_parity = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrTimeoutEmpty) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], kRtABytes);
          tma_load_2d(sA + stage * kRtABytes, &tmX, kb * 64, t * 128, &full[stage]);
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
    for (int s = 0; s < STAGES; ++s)
      if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1, err, kErrTimeoutDrain);
    mbar_wait(w_full, 0, err, kErrTimeoutDrain);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_f16(Traits<T>::code == AGM_BF16, 128, 16);
    const uint32_t sA_addr = smem_u32(sA), sW_addr = smem_u32(sW);
    int stage = 0, it = 0;
    uint32_t phase = 0;
    bool ok = mbar_wait(w_full, 0, err, kErrTimeoutFull);
    if (!ok) *abort_s = 1;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&acc_empty[acc], ((it >> 1) & 1) ^ 1, err, kErrTimeoutAcc) || *abort_s) {
        *abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * 16;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&full[stage], phase, err, kErrTimeoutFull) || *abort_s) {
          *abort_s = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t a_desc = smem_desc_k_sw128(sA_addr + stage * kRtABytes);
          const uint64_t w_desc = smem_desc_k_sw128(sW_addr + kb * kRtWBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(d_tmem, a_desc + 2 * kk, w_desc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (kb == nkb - 1) umma_commit(&acc_full[acc]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (lane == 0) umma_commit(drain);
    __syncwarp();
    mbar_wait(drain, 0, err, kErrTimeoutDrain);
  } else {
    // ---------------- Epilogue: one thread per token ----------------
    const int quarter = warp & 3;
    int it = 0;
    // One named barrier per tile: the four warps' counts of tile `it` sit in
    // hist_w[acc], which is written again only by tile it + 2, after every
    // warp has passed tile it + 1's barrier (so after the reads below). A
    // warp that gives up still reaches the barrier and raises epi_fail[acc],
    // so all four warps leave the loop together and none waits on the
    // barrier for a warp that has left.
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (it >> 1) & 1, err, kErrTimeoutAcc) &&
                                                  !*abort_s);
      if (ok) {
        tc_fence_after();
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 16, r);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);  // the accumulator is in registers: release it
        const int64_t tok = static_cast<int64_t>(t) * 128 + quarter * 32 + lane;
        float lg[kMaxExperts];
#pragma unroll
        for (int e = 0; e < kMaxExperts; ++e) lg[e] = round_to<T>(__uint_as_float(r[e]));
        route_warp<T, KC>(lg, tok < n_tokens, E, k, tie_low_first != 0, tok, logits_out, idx_out, gates_out,
                          hist_w + (acc * 4 + quarter) * kMaxExperts, err);
      } else if (lane == 0) {
        *abort_s = 1;
        epi_fail[acc] = 1;
      }
      named_bar_sync(1, 128);
      if (epi_fail[acc]) break;
      const int et = threadIdx.x - 64;  // epilogue thread index 0..127
      if (et < E) {
        const int* h = hist_w + acc * 4 * kMaxExperts + et;
        block_hist[static_cast<int64_t>(t) * E + et] = h[0] + h[kMaxExperts] + h[2 * kMaxExperts] + h[3 * kMaxExperts];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

template <typename T, int KC>
static cudaError_t launch_router_tc(const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                                    int tie_low_first, float* logits_out, int32_t* idx, void* gates,
                                    int32_t* block_hist, int* err, int num_sms, cudaStream_t stream) {
  const CUtensorMapDataType dt = (Traits<T>::code == AGM_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tmX, tmW;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(n_tokens)};
    const uint64_t str[1] = {static_cast<uint64_t>(d) * 2};
    const uint32_t box[2] = {64, 128};
    if (!encode_tmap(&tmX, x, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(E)};
    const uint64_t str[1] = {static_cast<uint64_t>(d) * 2};
    const uint32_t box[2] = {64, 16};
    if (!encode_tmap(&tmW, w, 2, dims, str, box, dt)) return cudaErrorInvalidValue;
  }
  const int nkb = (d + 63) / 64;
  const int64_t tiles = (n_tokens + 127) / 128;
  if (tiles <= num_sms && rt_smem_bytes(nkb, kRtStagesDeep) <= 227 * 1024) {
    const int smem = rt_smem_bytes(nkb, kRtStagesDeep);
    cudaError_t e =
        ensure_dynamic_smem(reinterpret_cast<const void*>(router_tc_kernel<T, KC, kRtStagesDeep>), smem);
    if (e != cudaSuccess) return e;
    return launch_kernel(router_tc_kernel<T, KC, kRtStagesDeep>, dim3(static_cast<unsigned>(tiles)), dim3(kRtThreads),
                         smem, stream, tmX, tmW, n_tokens, d, E, k, tie_low_first, logits_out, idx,
                         static_cast<T*>(gates), block_hist, err);
  }
  const int smem = rt_smem_bytes(nkb);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(router_tc_kernel<T, KC, kRtStages>), smem);
  if (e != cudaSuccess) return e;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, 2 * num_sms));
  return launch_kernel(router_tc_kernel<T, KC, kRtStages>, dim3(grid), dim3(kRtThreads), smem, stream, tmX, tmW,
                       n_tokens, d, E, k, tie_low_first, logits_out, idx, static_cast<T*>(gates), block_hist, err);
}

template <typename T, int KC>
static cudaError_t launch_router(const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                                 int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx,
                                 void* gates, int32_t* block_hist, int* err, int num_sms, cudaStream_t stream) {
  const int64_t nblk = (n_tokens + kDispatchBlock - 1) / kDispatchBlock;
  const size_t smem = (logits_in ? 0 : static_cast<size_t>(E) * d * sizeof(float)) +
                      static_cast<size_t>(kRouterWarps) * 32 * kMaxExperts * sizeof(float);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(router_topk_kernel<T, KC>), static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // As many CTAs as are resident at once, each looping over token blocks.
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, router_topk_kernel<T, KC>, kDispatchBlock, smem);
  if (e != cudaSuccess) return e;
  const int64_t grid = std::min<int64_t>(nblk, static_cast<int64_t>(std::max(per_sm, 1)) * std::max(num_sms, 1));
  return launch_kernel(router_topk_kernel<T, KC>, dim3(static_cast<unsigned>(grid)), dim3(kDispatchBlock), smem, stream,
                       static_cast<const T*>(x), static_cast<const T*>(w), n_tokens, d, E, k, tie_low_first, logits_in,
                       logits_out, idx, static_cast<T*>(gates), block_hist, err);
}

// The tensor-core router keeps the whole router weight resident next to its
// 8-stage x ring: d up to 4096 (64 k-blocks of 2 KB) fits in shared memory.
bool router_tc_supported(int d) { return d > 0 && d % 8 == 0 && rt_smem_bytes((d + 63) / 64) <= 227 * 1024; }

// One kernel per (dtype, top_k <= 4); larger top_k takes it at run time.
template <typename T, int KC>
static cudaError_t launch_any(bool tc, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                              int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                              int32_t* block_hist, int* err, int num_sms, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    if (tc)
      return launch_router_tc<T, KC>(x, w, n_tokens, d, E, k, tie_low_first, logits_out, idx, gates, block_hist, err,
                                     num_sms, stream);
  }
  return launch_router<T, KC>(x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates, block_hist,
                              err, num_sms, stream);
}

template <typename T>
static cudaError_t launch_k(bool tc, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                            int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                            int32_t* block_hist, int* err, int num_sms, cudaStream_t stream) {
#define AGM_ROUTER_K(KC)                                                                                       \
  return launch_any<T, KC>(tc, x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates, \
                           block_hist, err, num_sms, stream)
  static_assert(kFastTopK == 4, "one case per compiled top_k");
  switch (k) {
    case 1: AGM_ROUTER_K(1);
    case 2: AGM_ROUTER_K(2);
    case 3: AGM_ROUTER_K(3);
    case 4: AGM_ROUTER_K(4);
    default: AGM_ROUTER_K(0);
  }
#undef AGM_ROUTER_K
}

cudaError_t router_topk(int dtype, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                        int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                        int32_t* block_hist, int* err, int num_sms, cudaStream_t stream) {
  if (n_tokens == 0) return cudaSuccess;
  const bool tc = !logits_in && router_tc_supported(d);
  switch (dtype) {
    case AGM_F32:
      return launch_k<float>(false, x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates,
                             block_hist, err, num_sms, stream);
    case AGM_BF16:
      return launch_k<__nv_bfloat16>(tc, x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates,
                                     block_hist, err, num_sms, stream);
    case AGM_F16:
      return launch_k<__half>(tc, x, w, n_tokens, d, E, k, tie_low_first, logits_in, logits_out, idx, gates,
                              block_hist, err, num_sms, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Decode front: router + dispatch plan + permute of one dispatch block
// ---------------------------------------------------------------------------
// At decode batch sizes (<= 128 tokens, one dispatch block) the three kernels
// above cost about 19 us per layer in a CUDA graph, mostly latency: the
// tensor-core router is one CTA whose 20 x tiles pass through one SM, then
// two more launches follow. Here one cluster of 8 CTAs does all three: CTA r
// takes tokens [16 r, 16 r + 16), two per warp, with its token rows and the
// router weight (fp32) staged in shared memory; the logits are fp32 FMAs over
// the lane's 16-byte chunks lane + 32 j then
// a transpose-reduce across lanes (the SIMT router's order), rounded once to
// the dtype; warp 0 selects top-k for the CTA's 16
// tokens (select_route, as in the other routers) and ballots per-expert
// token masks. After a cluster barrier every CTA reads the 8 CTAs' per-expert
// counts through distributed shared memory: the totals give the block
// histogram, counts and padded segment starts (as dispatch_plan_kernel
// computes them for one block), the counts of lower-ranked CTAs give each
// token's rank within its expert (ascending token order, as permute_kernel),
// and each warp copies its two tokens' rows to their destination rows. Code is kept loop-based (not unrolled over chunks): a
// launch runs it once, and cold instruction-cache misses were its largest
// stall. A last cluster barrier keeps every CTA's shared memory
// alive until the others have read it.
constexpr int kFrontCtas = 8;
constexpr int kFrontWarps = 8;
constexpr int kFrontTokCta = kDispatchBlock / kFrontCtas;  // 16
constexpr int kFrontTokWarp = kFrontTokCta / kFrontWarps;  // 2
constexpr int kFrontChunks = 8;  // d <= 32 x 8 chunks = 2048: 16 rows x 2d + E x 4d bytes of shared memory

template <typename T, int KC>
__global__ void __launch_bounds__(32 * kFrontWarps) decode_front_kernel(
    const T* __restrict__ x, const T* __restrict__ w, int n_tokens, int d, int E, int k, int tie_low_first,
    float* __restrict__ logits_out, int32_t* __restrict__ idx_out, T* __restrict__ gates_out, FrontOut o, int* err) {
  constexpr int S = RouteK<KC>::S;
  if (KC > 0) k = KC;
  __shared__ float logit_s[kFrontTokCta][kMaxExperts];
  __shared__ int cnt_s[kMaxExperts];          // this CTA's tokens per expert (read by the whole cluster)
  __shared__ uint32_t mask_s[kMaxExperts];    // bit t: local token t picked expert e
  __shared__ uint32_t pm_s[kFrontWarps][kMaxExperts];  // the same, per warp (bits 0-1: its two tokens)
  __shared__ int tot_s[kMaxExperts], pre_s[kMaxExperts], seg_s[kMaxExperts + 1];
  const int warp = warp_id(), lane = lane_id();
  const int rank = static_cast<int>(cluster_ctarank());
  const int nchunk = d / 8;  // 16-byte chunks per row (16-bit dtypes)
  pdl_wait();
  pdl_trigger();

  // 1. Logits of this warp's two tokens. The CTA stages its 16 token rows
  // (packed, as loaded) and the router weight (fp32, in two float4 planes:
  // plane h holds elements 4h..4h+3 of every 16-byte chunk,
  // w_s[h][e * nchunk + c]) in shared memory, every load in flight at once;
  // the FMA loop then reads both with conflict-free 16-byte loads. Loops over
  // chunks are not unrolled: the kernel runs once per launch, so its code has
  // to stay small enough not to wait on instruction-cache misses.
  extern __shared__ float4 front_smem[];
  const int wchunks = E * nchunk;
  float4* w_s = front_smem;                                          // [2][E * nchunk]
  uint4* x_s = reinterpret_cast<uint4*>(front_smem + 2 * wchunks);   // [16][nchunk]
  {
    const uint4* w4 = reinterpret_cast<const uint4*>(w);
    const uint4* x4 = reinterpret_cast<const uint4*>(x) + static_cast<int64_t>(rank) * kFrontTokCta * nchunk;
    const int valid_rows = max(0, min(kFrontTokCta, n_tokens - rank * kFrontTokCta));
    const int xchunks = valid_rows * nchunk;
    constexpr int kBatch = 4;
#pragma unroll 1
    for (int i0 = threadIdx.x; i0 < xchunks; i0 += kBatch * blockDim.x) {
      uint4 u[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int i = i0 + b * blockDim.x;
        u[b] = i < xchunks ? __ldg(x4 + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int i = i0 + b * blockDim.x;
        if (i < xchunks) x_s[i] = u[b];
      }
    }
#pragma unroll 1
    for (int i0 = threadIdx.x; i0 < wchunks; i0 += kBatch * blockDim.x) {
      uint4 u[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int i = i0 + b * blockDim.x;
        u[b] = i < wchunks ? __ldg(w4 + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int i = i0 + b * blockDim.x;
        if (i < wchunks) {
          float f[8];
          unpack8<T>(u[b], f);
          w_s[i] = make_float4(f[0], f[1], f[2], f[3]);
          w_s[wchunks + i] = make_float4(f[4], f[5], f[6], f[7]);
        }
      }
    }
  }
  __syncthreads();
  const int ltok0 = warp * kFrontTokWarp;  // local token index
  const bool live[kFrontTokWarp] = {rank * kFrontTokCta + ltok0 < n_tokens, rank * kFrontTokCta + ltok0 + 1 < n_tokens};
  float acc[kFrontTokWarp][kMaxExperts];
#pragma unroll
  for (int t = 0; t < kFrontTokWarp; ++t)
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) acc[t][e] = 0.f;
#pragma unroll 1
  for (int c = lane; c < nchunk; c += 32) {
    float xf[kFrontTokWarp][8];
#pragma unroll
    for (int t = 0; t < kFrontTokWarp; ++t)
      unpack8<T>(live[t] ? x_s[(ltok0 + t) * nchunk + c] : make_uint4(0, 0, 0, 0), xf[t]);
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) {
      if (e < E) {
        const float4 lo = w_s[e * nchunk + c], hi = w_s[wchunks + e * nchunk + c];
        const float wf[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int t = 0; t < kFrontTokWarp; ++t)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[t][e] = fmaf(xf[t][i], wf[i], acc[t][e]);
      }
    }
  }
  // Transpose-reduce (as the SIMT router): after the xor-16/8/4/2 steps lane l
  // holds a partial sum of expert 8*b4 + 4*b3 + 2*b2 + b1 (b = bits of l).
#pragma unroll
  for (int t = 0; t < kFrontTokWarp; ++t) {
    float v8[8], v4[4], v2[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = u16 ? acc[t][i] : acc[t][i + 8];
      const float keep = u16 ? acc[t][i + 8] : acc[t][i];
      v8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = u8 ? v8[i] : v8[i + 4];
      const float keep = u8 ? v8[i + 4] : v8[i];
      v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = u4 ? v4[i] : v4[i + 2];
      const float keep = u4 ? v4[i + 2] : v4[i];
      v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    float v1;
    {
      const float send = u2 ? v2[0] : v2[1];
      const float keep = u2 ? v2[1] : v2[0];
      v1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    const float sum = v1 + __shfl_xor_sync(0xffffffffu, v1, 1);
    const int e = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
    if ((lane & 1) == 0) logit_s[ltok0 + t][e] = round_to<T>(sum);
  }
  __syncwarp();

  // 2. Selection: lanes 0 and 1 of each warp take its two tokens.
  int sel[S];
#pragma unroll
  for (int r = 0; r < S; ++r) sel[r] = -1;
  const int my_ltok = ltok0 + (lane & 1);
  const int64_t my_tok = static_cast<int64_t>(rank) * kFrontTokCta + my_ltok;
  const bool my_valid = lane < kFrontTokWarp && my_tok < n_tokens;
  if (my_valid) {
    float lg[kMaxExperts];
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e) lg[e] = (e < E) ? logit_s[my_ltok][e] : 0.f;
    if (logits_out) {
#pragma unroll
      for (int e = 0; e < kMaxExperts; ++e)
        if (e < E) logits_out[my_tok * E + e] = lg[e];
    }
    float gate[S];
    select_route<KC>(lg, E, k, tie_low_first != 0, sel, gate);
#pragma unroll
    for (int r = 0; r < S; ++r) {
      if (r < k) {
        const int e = sel[r];
        if (e < 0 || e >= E) {
          raise_error(err, kErrBadExpert);
          sel[r] = -1;
        } else {
          idx_out[my_tok * k + r] = e;
          gates_out[my_tok * k + r] = Traits<T>::from_f(gate[r]);
        }
      }
    }
  }
#pragma unroll 1
  for (int e = 0; e < E; ++e) {
    bool hit = false;
#pragma unroll
    for (int r = 0; r < S; ++r) hit |= (r < k && sel[r] == e);
    const uint32_t m = __ballot_sync(0xffffffffu, hit) & 3u;
    if (lane == 0) pm_s[warp][e] = m;
  }
  __syncthreads();
  if (threadIdx.x < E) {
    uint32_t m = 0;
#pragma unroll
    for (int q = 0; q < kFrontWarps; ++q) m |= pm_s[q][threadIdx.x] << (kFrontTokWarp * q);
    mask_s[threadIdx.x] = m;
    cnt_s[threadIdx.x] = __popc(m);
  }
  cluster_sync();  // every CTA's cnt_s is written

  // 3. Plan of the block: totals over the cluster, this CTA's offsets, padded segment starts.
  if (warp == 0) {
    int tot = 0, pre = 0;
    if (lane < E) {
      const uint32_t a = smem_u32(&cnt_s[lane]);
      for (int q = 0; q < kFrontCtas; ++q) {
        const int v = ld_shared_cluster_s32(cluster_map(a, q));
        tot += v;
        if (q < rank) pre += v;
      }
    }
    const int padded = lane < E ? (tot + o.seg_align - 1) / o.seg_align * o.seg_align : 0;
    int incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane < E) {
      tot_s[lane] = tot;
      pre_s[lane] = pre;
      seg_s[lane] = incl - padded;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      seg_s[E] = total;
      if (rank == 0 && (total > o.max_rows || total / AGM_TILE_M > o.max_tiles)) raise_error(err, kErrRowOverflow);
    }
  }
  __syncthreads();
  const int total_rows = static_cast<int>(min(static_cast<int64_t>(seg_s[E]), o.max_rows));
  const int ntiles = total_rows / AGM_TILE_M;
  if (rank == 0) {
    if (threadIdx.x < E) {
      o.block_hist[threadIdx.x] = tot_s[threadIdx.x];
      o.block_off[threadIdx.x] = 0;
      o.counts[threadIdx.x] = tot_s[threadIdx.x];
    }
    if (threadIdx.x <= E) o.seg_start[threadIdx.x] = seg_s[threadIdx.x];
    if (threadIdx.x == 0) *o.num_tiles = ntiles;
    for (int m = threadIdx.x; m < ntiles; m += blockDim.x) {
      const int row = m * AGM_TILE_M;
      int e = 0;
      while (e + 1 < E && seg_s[e + 1] <= row) ++e;
      o.tile_expert[m] = e;
    }
  }
  // Padding rows of x_perm are zeroed when the GEMMs read them (row tiles),
  // spread over the cluster's threads. token_of keeps the source token of
  // every valid row; its padding entries are not written (nothing reads them).
  if (o.zero_pad) {
    const int gt = rank * blockDim.x + threadIdx.x, gn = kFrontCtas * blockDim.x;
    uint4* xp = static_cast<uint4*>(o.x_perm);
#pragma unroll 1
    for (int e = 0; e < E; ++e) {
      const int p0 = seg_s[e] + tot_s[e], p1 = min(seg_s[e + 1], total_rows);
      const int64_t q1 = static_cast<int64_t>(max(p1 - p0, 0)) * nchunk;
      for (int64_t q = gt; q < q1; q += gn)
        xp[(p0 + q / nchunk) * static_cast<int64_t>(nchunk) + q % nchunk] = make_uint4(0, 0, 0, 0);
    }
  }

  // 4. Destination rows of lanes 0-1's tokens, then 5. the warp copies both tokens' rows.
  int dest[S];
#pragma unroll
  for (int r = 0; r < S; ++r) dest[r] = -1;
  if (my_valid) {
    const uint32_t lt_mask = (1u << my_ltok) - 1u;
#pragma unroll
    for (int r = 0; r < S; ++r) {
      const int e = sel[r];
      if (r < k && e >= 0 && e < E) {
        const int64_t row = static_cast<int64_t>(seg_s[e]) + pre_s[e] + __popc(mask_s[e] & lt_mask);
        if (row < o.max_rows) {
          dest[r] = static_cast<int>(row);
          o.row_of[my_tok * k + r] = static_cast<int32_t>(row);
          o.token_of[row] = static_cast<int32_t>(my_tok);
        } else {
          raise_error(err, kErrRowOverflow);
        }
      }
    }
  }
  uint4* xp = static_cast<uint4*>(o.x_perm);
#pragma unroll
  for (int t = 0; t < kFrontTokWarp; ++t) {
#pragma unroll
    for (int r = 0; r < S; ++r) {
      const int row = __shfl_sync(0xffffffffu, dest[r], t);
      if (r < k && row >= 0) {
        uint4* dst = xp + static_cast<int64_t>(row) * nchunk;
        const uint4* src = x_s + (ltok0 + t) * nchunk;
#pragma unroll 4
        for (int c = lane; c < nchunk; c += 32) dst[c] = src[c];
      }
    }
  }
  cluster_sync();  // no CTA leaves while another may still read its cnt_s
}

bool decode_front_supported(int dtype, int64_t n_tokens, int d, int E, int k) {
  return (dtype == AGM_BF16 || dtype == AGM_F16) && n_tokens > 0 && n_tokens <= kDispatchBlock && d > 0 &&
         d % 8 == 0 && d / 8 <= 32 * kFrontChunks && E >= 1 && E <= kMaxExperts && k >= 1 && k <= E;
}

template <typename T>
static cudaError_t launch_front(const void* x, const void* w, int64_t n_tokens, int d, int E, int k, int tie_low_first,
                                float* logits_out, int32_t* idx, void* gates, const FrontOut& o, int* err,
                                cudaStream_t stream) {
  const dim3 grid(kFrontCtas), block(32 * kFrontWarps);
  const int n = static_cast<int>(n_tokens);
  // the router weight in fp32 and the CTA's 16 token rows
  const int smem = E * d * static_cast<int>(sizeof(float)) + kFrontTokCta * d * 2;
  cudaError_t e = cudaSuccess;
  switch (k) {
    case 1: e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel<T, 1>), smem); break;
    case 2: e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel<T, 2>), smem); break;
    case 3: e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel<T, 3>), smem); break;
    case 4: e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel<T, 4>), smem); break;
    default: e = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel<T, 0>), smem); break;
  }
  if (e != cudaSuccess) return e;
  T* g = static_cast<T*>(gates);
  const T* xs = static_cast<const T*>(x);
  const T* ws = static_cast<const T*>(w);
  switch (k) {
    case 1: return launch_cluster_kernel(decode_front_kernel<T, 1>, grid, block, kFrontCtas, smem, stream, xs, ws, n, d, E, k,
                                         tie_low_first, logits_out, idx, g, o, err);
    case 2: return launch_cluster_kernel(decode_front_kernel<T, 2>, grid, block, kFrontCtas, smem, stream, xs, ws, n, d, E, k,
                                         tie_low_first, logits_out, idx, g, o, err);
    case 3: return launch_cluster_kernel(decode_front_kernel<T, 3>, grid, block, kFrontCtas, smem, stream, xs, ws, n, d, E, k,
                                         tie_low_first, logits_out, idx, g, o, err);
    case 4: return launch_cluster_kernel(decode_front_kernel<T, 4>, grid, block, kFrontCtas, smem, stream, xs, ws, n, d, E, k,
                                         tie_low_first, logits_out, idx, g, o, err);
    default: return launch_cluster_kernel(decode_front_kernel<T, 0>, grid, block, kFrontCtas, smem, stream, xs, ws, n, d, E,
                                          k, tie_low_first, logits_out, idx, g, o, err);
  }
}

cudaError_t decode_front(int dtype, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                         int tie_low_first, float* logits_out, int32_t* idx, void* gates, const FrontOut& o, int* err,
                         cudaStream_t stream) {
  if (!decode_front_supported(dtype, n_tokens, d, E, k)) return cudaErrorInvalidValue;
  if (o.seg_align != AGM_TILE_M && o.seg_align != 2 * AGM_TILE_M) return cudaErrorInvalidValue;
  if (dtype == AGM_BF16)
    return launch_front<__nv_bfloat16>(x, w, n_tokens, d, E, k, tie_low_first, logits_out, idx, gates, o, err, stream);
  return launch_front<__half>(x, w, n_tokens, d, E, k, tie_low_first, logits_out, idx, gates, o, err, stream);
}

size_t router_smem_bytes(int d, int E) {
  return static_cast<size_t>(E) * d * sizeof(float) + static_cast<size_t>(kRouterWarps) * 32 * kMaxExperts * 4;
}

}  // namespace agm
