// K2: expert histogram -> prefix sums -> stable scatter permutation.
//
// Replaces the reference's dispatch loop (agillm41.py:4421-4428): for every
// (rank, expert) it runs `nonzero` (a device->host sync) and `index_select`.
// Here the whole dispatch is two kernels and no host sync:
//
// * dispatch_plan_kernel (one CTA): per expert, an exclusive scan of the
//   per-block histograms written by the router kernel gives each dispatch
//   block its base offset inside the expert's segment; per-expert counts;
//   segment starts padded to the GEMM row tile (128 rows, or 256 when the
//   expert GEMMs run on CTA pairs); the row-tile -> expert table
//   and the number of row tiles (read by the persistent GEMM on the device).
// * permute_kernel (one CTA per dispatch block of 128 tokens, plus 8 CTAs per
//   expert that zero-fill the segment's padding rows, except for the
//   swapped-operand GEMMs, which never use them): warp ballots give each
//   (token, rank) its rank among the block's tokens routed to the same expert,
//   in ascending token order, so the permutation is deterministic and equals
//   the reference's ascending `nonzero` order. Rows of x are copied with
//   16-byte vector loads/stores to every destination row of the token.
//
// Output layout in HBM: x_perm [max_rows, d] (expert segments back to back,
// each padded to a multiple of 128 or 256 rows), row_of [N, k] (destination row of
// each (token, rank)), token_of [max_rows] (source token of each row, -1 for
// padding rows).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace agm {

constexpr int kTile = AGM_TILE_M;
constexpr int kBlk = AGM_DISPATCH_BLOCK;
constexpr int kPlanThreads = 512;
constexpr int kPlanUnroll = 8;
constexpr int kMaxChunks = 8;  // 16-byte chunks per lane held in registers (rows up to 4 KB)
// CTAs that zero-fill one expert segment's padding rows (up to 255 rows; one
// CTA per expert made this fill the longest part of a small-batch permute).
constexpr int kZeroCtas = 8;

__global__ void __launch_bounds__(kPlanThreads) dispatch_plan_kernel(
    const int32_t* __restrict__ block_hist, int n_blocks, int E, int64_t max_rows, int max_tiles, int seg_align,
    int32_t* __restrict__ block_off, int32_t* __restrict__ counts, int32_t* __restrict__ seg_start,
    int32_t* __restrict__ tile_expert, int32_t* __restrict__ num_tiles, int32_t* __restrict__ token_of, int* err) {
  __shared__ int tot_s[32];
  __shared__ int seg_s[33];
  const int warp = warp_id(), lane = lane_id();
  pdl_wait();
  pdl_trigger();
  const int nwarps = blockDim.x / 32;
  // 1. Per-expert exclusive scan over blocks (one warp per expert). The
  //    loads of kPlanUnroll x 32 blocks are issued together before the scan
  //    so a long histogram costs a few memory round trips, not one per 32.
  for (int e = warp; e < E; e += nwarps) {
    int carry = 0;
    for (int b0 = 0; b0 < n_blocks; b0 += 32 * kPlanUnroll) {
      int v[kPlanUnroll];
#pragma unroll
      for (int j = 0; j < kPlanUnroll; ++j) {
        const int b = b0 + 32 * j + lane;
        v[j] = (b < n_blocks) ? block_hist[static_cast<int64_t>(b) * E + e] : 0;
      }
#pragma unroll
      for (int j = 0; j < kPlanUnroll; ++j) {
        const int b = b0 + 32 * j + lane;
        int incl = v[j];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += n;
        }
        if (b < n_blocks) block_off[static_cast<int64_t>(b) * E + e] = carry + incl - v[j];
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    if (lane == 0) tot_s[e] = carry;
  }
  __syncthreads();
  // 2. Padded segment starts.
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      seg_s[e] = acc;
      acc += (tot_s[e] + seg_align - 1) / seg_align * seg_align;
    }
    seg_s[E] = acc;
    if (acc > max_rows || acc / kTile > max_tiles) raise_error(err, kErrRowOverflow);
  }
  __syncthreads();
  const int total_rows = min(static_cast<int64_t>(seg_s[E]), max_rows);
  const int ntiles = total_rows / kTile;
  if (threadIdx.x < E) counts[threadIdx.x] = tot_s[threadIdx.x];
  if (threadIdx.x <= E) seg_start[threadIdx.x] = seg_s[threadIdx.x];
  if (threadIdx.x == 0) *num_tiles = ntiles;
  // 3. Tile table and padding rows of token_of.
  for (int m = threadIdx.x; m < ntiles; m += blockDim.x) {
    const int row = m * kTile;
    int e = 0;
    while (e + 1 < E && seg_s[e + 1] <= row) ++e;
    tile_expert[m] = e;
  }
  for (int e = 0; e < E; ++e) {
    const int p0 = seg_s[e] + tot_s[e], p1 = min(seg_s[e + 1], total_rows);
    for (int r = p0 + threadIdx.x; r < p1; r += blockDim.x) token_of[r] = -1;
  }
}

// Destination of permuted row p: the local x_perm buffer.
struct LocalRows {
  static constexpr bool kSystemFence = false;
  uint4* base;
  int nchunk;
  __device__ __forceinline__ uint4* row(int64_t p) const { return base + p * nchunk; }
};

template <int K_MAX, class Dst>
__global__ void __launch_bounds__(kBlk) permute_kernel(
    const uint4* __restrict__ x, int64_t n_tokens, int nchunk /* 16-byte chunks per row */, int k, int E,
    int n_blocks, int split, const int32_t* __restrict__ idx, const int32_t* __restrict__ block_off,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ counts, int64_t max_rows, Dst dst,
    int32_t* __restrict__ row_of, int32_t* __restrict__ token_of, int* err) {
  const int warp = warp_id(), lane = lane_id();
  pdl_wait();
  pdl_trigger();
  if (static_cast<int>(blockIdx.x) >= n_blocks * split) {
    // Zero-fill the padding rows of one expert segment: kZeroCtas CTAs per
    // expert, one row per warp at a time.
    const int z = blockIdx.x - n_blocks * split;
    const int e = z / kZeroCtas;
    const int64_t r0 = seg_start[e] + counts[e];
    const int64_t r1 = min(static_cast<int64_t>(seg_start[e + 1]), max_rows);
    const int nw = blockDim.x / 32;
    for (int64_t r = r0 + (z % kZeroCtas) * nw + warp; r < r1; r += kZeroCtas * nw) {
      uint4* o = dst.row(r);
      if (o)
        for (int c = lane; c < nchunk; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    }
    if constexpr (Dst::kSystemFence) __threadfence_system();
    return;
  }
  // `split` CTAs share one dispatch block (small batches): each computes the
  // block's destination rows and copies every split-th pair of its tokens.
  const int blk = blockIdx.x / split, part = blockIdx.x % split;
  __shared__ uint32_t mask_s[kBlk / 32][32];
  __shared__ int cnt_s[kBlk / 32][32];
  __shared__ int off_s[kBlk / 32][32];
  const int64_t tok = static_cast<int64_t>(blk) * kBlk + threadIdx.x;
  const bool valid = tok < n_tokens;
  int my_e[K_MAX];
#pragma unroll
  for (int r = 0; r < K_MAX; ++r) my_e[r] = (valid && r < k) ? idx[tok * k + r] : -1;
  // Per-warp masks: lanes whose token picked expert e (at any rank).
  for (int e = 0; e < E; ++e) {
    bool hit = false;
#pragma unroll
    for (int r = 0; r < K_MAX; ++r) hit |= (my_e[r] == e);
    const uint32_t m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) {
      mask_s[warp][e] = m;
      cnt_s[warp][e] = __popc(m);
    }
  }
  __syncthreads();
  if (threadIdx.x < E) {
    const int e = threadIdx.x;
    int acc = 0;
    for (int w = 0; w < kBlk / 32; ++w) {
      off_s[w][e] = acc;
      acc += cnt_s[w][e];
    }
  }
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
  int dest[K_MAX];
#pragma unroll
  for (int r = 0; r < K_MAX; ++r) {
    dest[r] = -1;
    const int e = my_e[r];
    if (e >= 0 && e < E) {
      const int64_t row = static_cast<int64_t>(seg_start[e]) + block_off[static_cast<int64_t>(blk) * E + e] +
                          off_s[warp][e] + __popc(mask_s[warp][e] & lt);
      if (row >= 0 && row < max_rows) {
        dest[r] = static_cast<int>(row);
        if (part == 0) {
          row_of[tok * k + r] = static_cast<int32_t>(row);
          if (token_of) token_of[row] = static_cast<int32_t>(tok);
        }
      } else if (part == 0) {
        raise_error(err, kErrRowOverflow);
      }
    } else if (e >= E && part == 0) {
      raise_error(err, kErrBadExpert);
    }
  }
  // Copy rows: the warp walks its 32 tokens two at a time; every lane loads
  // all of its 16-byte chunks of both rows before storing them to the k
  // destination rows, so up to 2 x kMaxChunks loads per lane are in flight.
  const int64_t warp_tok0 = static_cast<int64_t>(blk) * kBlk + warp * 32;
  if (nchunk <= 32 * kMaxChunks) {
    for (int i = 2 * part; i < 32; i += 2 * split) {
      const int64_t t0 = warp_tok0 + i, t1 = t0 + 1;
      if (t0 >= n_tokens) break;
      const bool has1 = t1 < n_tokens;
      int d0[K_MAX], d1[K_MAX];
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) {
        d0[r] = __shfl_sync(0xffffffffu, dest[r], i);
        d1[r] = __shfl_sync(0xffffffffu, dest[r], i + 1);
      }
      const uint4* s0 = x + t0 * nchunk;
      const uint4* s1 = x + t1 * nchunk;
      uint4 v0[kMaxChunks], v1[kMaxChunks];
#pragma unroll
      for (int j = 0; j < kMaxChunks; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunk) {
          v0[j] = __ldg(s0 + c);
          if (has1) v1[j] = __ldg(s1 + c);
        }
      }
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) {
        if (r >= k) break;
        uint4* o0 = d0[r] >= 0 ? dst.row(d0[r]) : nullptr;
        uint4* o1 = (has1 && d1[r] >= 0) ? dst.row(d1[r]) : nullptr;
#pragma unroll
        for (int j = 0; j < kMaxChunks; ++j) {
          const int c = lane + 32 * j;
          if (c < nchunk) {
            if (o0) o0[c] = v0[j];
            if (o1) o1[c] = v1[j];
          }
        }
      }
    }
  } else {
    for (int i = part; i < 32; i += split) {
      const int64_t t = warp_tok0 + i;
      if (t >= n_tokens) break;
      int drow[K_MAX];
#pragma unroll
      for (int r = 0; r < K_MAX; ++r) drow[r] = __shfl_sync(0xffffffffu, dest[r], i);
      const uint4* src = x + t * nchunk;
      for (int c = lane; c < nchunk; c += 32) {
        const uint4 v = __ldg(src + c);
        for (int r = 0; r < k && r < K_MAX; ++r)
          if (drow[r] >= 0) {
            uint4* o = dst.row(drow[r]);
            if (o) o[c] = v;
          }
      }
    }
  }
  if constexpr (Dst::kSystemFence) __threadfence_system();
}

cudaError_t dispatch_plan(const int32_t* block_hist, int n_blocks, int E, int64_t max_rows, int max_tiles,
                          int seg_align, int32_t* block_off, int32_t* counts, int32_t* seg_start,
                          int32_t* tile_expert, int32_t* num_tiles, int32_t* token_of, int* err, cudaStream_t stream) {
  if (seg_align != kTile && seg_align != 2 * kTile) return cudaErrorInvalidValue;
  return launch_kernel(dispatch_plan_kernel, dim3(1), dim3(kPlanThreads), 0, stream, block_hist, n_blocks, E, max_rows,
                       max_tiles, seg_align, block_off, counts, seg_start, tile_expert, num_tiles, token_of, err);
}

template <class Dst>
static cudaError_t launch_permute(const void* x, int elem_bytes, int64_t n_tokens, int d, int k, int E,
                                  const int32_t* idx, const int32_t* block_off, const int32_t* seg_start,
                                  const int32_t* counts, int64_t max_rows, Dst dst, int32_t* row_of,
                                  int32_t* token_of, int* err, cudaStream_t stream, bool zero_pad = true) {
  const int n_blocks = static_cast<int>((n_tokens + kBlk - 1) / kBlk);
  const int nchunk = d * elem_bytes / 16;
  // Small batches: up to 16 CTAs per dispatch block, so the row copies of a
  // few hundred tokens are not serialised in one or two warps.
  const int split = n_blocks >= 64 ? 1 : std::min(16, 64 / n_blocks);
  const unsigned grid = static_cast<unsigned>(n_blocks * split + (zero_pad ? E * kZeroCtas : 0));
  if (n_tokens <= 0) return cudaSuccess;
  const uint4* xs = static_cast<const uint4*>(x);
  if (k <= 2)
    return launch_kernel(permute_kernel<2, Dst>, dim3(grid), dim3(kBlk), 0, stream, xs, n_tokens, nchunk, k, E,
                         n_blocks, split, idx, block_off, seg_start, counts, max_rows, dst, row_of, token_of, err);
  if (k <= 4)
    return launch_kernel(permute_kernel<4, Dst>, dim3(grid), dim3(kBlk), 0, stream, xs, n_tokens, nchunk, k, E,
                         n_blocks, split, idx, block_off, seg_start, counts, max_rows, dst, row_of, token_of, err);
  return launch_kernel(permute_kernel<16, Dst>, dim3(grid), dim3(kBlk), 0, stream, xs, n_tokens, nchunk, k, E,
                       n_blocks, split, idx, block_off, seg_start, counts, max_rows, dst, row_of, token_of, err);
}

cudaError_t permute_rows(const void* x, int elem_bytes, int64_t n_tokens, int d, int k, int E, const int32_t* idx,
                         const int32_t* block_off, const int32_t* seg_start, const int32_t* counts, int64_t max_rows,
                         void* x_perm, int32_t* row_of, int32_t* token_of, int* err, cudaStream_t stream,
                         bool zero_pad) {
  LocalRows dst{static_cast<uint4*>(x_perm), d * elem_bytes / 16};
  return launch_permute(x, elem_bytes, n_tokens, d, k, E, idx, block_off, seg_start, counts, max_rows, dst, row_of,
                        token_of, err, stream, zero_pad);
}

cudaError_t permute_rows_ep(const void* x, int elem_bytes, int64_t n_tokens, int d, int k, int E, const int32_t* idx,
                            const int32_t* block_off, const int32_t* seg_start, const int32_t* counts,
                            int64_t max_rows, const EpRoute* route, int32_t* row_of, int* err, cudaStream_t stream) {
  EpRows dst{route, d * elem_bytes / 16};
  return launch_permute(x, elem_bytes, n_tokens, d, k, E, idx, block_off, seg_start, counts, max_rows, dst, row_of,
                        nullptr, err, stream);
}

}  // namespace agm
