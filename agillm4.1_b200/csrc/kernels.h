// Internal launch interface shared by the kernel files and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <utility>

namespace agm {

// Whether launches use programmatic dependent launch (see pdl_wait in
// common.cuh): on unless the environment sets AGM_NO_PDL=1 or the calling
// thread is inside a forward called with AGM_FLAG_NO_PDL.
bool pdl_enabled();
// Scope of one forward call: sets this thread's PDL choice, restores it after.
struct PdlScope {
  explicit PdlScope(bool on);
  ~PdlScope();
  bool prev;
};

// Kernel launch on `stream` with the programmatic-serialization attribute
// (when enabled): the kernel may begin before the previous kernel on the
// stream completes, and must call pdl_wait() before touching its outputs.
template <typename... Exp, typename... Act>
inline cudaError_t launch_kernel(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// launch_kernel with a cluster of `cluster` CTAs along x (grid a multiple of it).
template <typename... Exp, typename... Act>
inline cudaError_t launch_cluster_kernel(void (*kernel)(Exp...), dim3 grid, dim3 block, int cluster, size_t smem,
                                         cudaStream_t stream, Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// Arguments of the grouped GEMM  c[r, :] = act(a[r, :] @ w[g]^T + bias[g]).
struct GemmArgs {
  void* c;
  int64_t ldc;
  int64_t c_rows;             // rows of c that exist (rows beyond are not stored)
  const void* bias;           // [groups, n] or nullptr
  int n;
  int k;
  int groups;
  const int32_t* tile_group;  // [max_tiles] or nullptr (all tiles -> group 0)
  const int32_t* num_tiles;   // device count of valid row tiles, or nullptr
  int max_tiles;              // host bound (and the count when num_tiles is null)
  int* err;
  int max_ctas = 0;           // cap on persistent CTAs (0 = one per SM), leaves SMs to concurrent kernels
  // Swapped-operand kernel (small batches) only: expert e's rows are
  // [seg_start[e], seg_start[e] + seg_count[e]) (device arrays, groups entries).
  const int32_t* seg_start = nullptr;
  const int32_t* seg_count = nullptr;
  // Swapped-operand kernel only: the weight is in the decode tile layout
  // [groups][n / 128][k / 64][128][64] (each 128 x 64 tile one contiguous
  // 16 KB block) instead of [groups][n][k]; n % 128 == 0, k % 64 == 0.
  bool w_tiled = false;
  // The caller guarantees that the tile table / segment counts and the
  // weights were written at least two kernels before this launch (true
  // inside agm_moe_forward): the kernel then reads them and streams its first
  // weight tiles before waiting for the previous kernel (programmatic
  // dependent launch). Otherwise it waits before reading anything.
  bool early_weights = false;
  // ReLU epilogue only, nullable: bit j of relu_bits[w * ld_bits + r] is set
  // when the stored c[r, 32 w + j] > 0 (training keeps this [ceil(n/32), rows]
  // mask for the ReLU backward instead of re-reading c).
  uint32_t* relu_bits = nullptr;
  int64_t ld_bits = 0;
  // CTA-pair kernel only, nullable: row tile t's 128 output rows go to the
  // 16-bit row-major buffer at address tile_dst[t] (row stride ldc elements)
  // instead of c, e.g. the token owner's buffer on a peer GPU (expert
  // parallelism); stored with 16-byte vector stores.
  const uint64_t* tile_dst = nullptr;
  // CTA-pair kernel only, nullable: row tile t came from source rank
  // tile_src[t] (expert parallelism); before loading the first tile of a
  // source the producer waits (bounded) until src_signal[source] >= src_epoch,
  // the source's release of "rows delivered".
  const int32_t* tile_src = nullptr;
  const uint64_t* src_signal = nullptr;
  uint64_t src_epoch = 0;
  // CTA-pair kernel only: a second, dense problem computed in the same launch
  // after this one's tiles (the shared experts of a MoE block): groups2
  // groups of tiles2 row tiles each; group g reads A rows from
  // g * a2_group_rows (a2: a2_rows x k2), weight [g] of w2 ([groups2, n2, k2]),
  // bias2 [groups2, n2], and writes C rows from g * c2_group_rows of c2
  // (c2_rows x n2, row stride ldc2). groups2 = 0: no second problem.
  int groups2 = 0;
  const void* a2 = nullptr;
  int64_t a2_rows = 0;
  const void* w2 = nullptr;
  const void* bias2 = nullptr;
  void* c2 = nullptr;
  int64_t c2_rows = 0;
  int64_t ldc2 = 0;
  int n2 = 0;
  int k2 = 0;
  int tiles2 = 0;
  int64_t a2_group_rows = 0;
  int64_t c2_group_rows = 0;
};

// Expert-parallel routing of one rank's permuted rows (see ep_p2p.cu): a list
// of segments of its x_perm tiles; segment s sends tiles [seg_lo, seg_hi) to
// rank seg_rank, landing at tile seg_base of that rank's receive buffer
// (at most seg_limit tiles fit). peer_recv holds the device addresses of
// every rank's receive buffer as mapped into this process.
constexpr int kEpMaxRanks = 16;
constexpr int kEpMaxSegs = 64;
struct EpRoute {
  int world;
  int rank;
  int n_seg;
  int seg_rank[kEpMaxSegs];
  int64_t seg_lo[kEpMaxSegs];
  int64_t seg_hi[kEpMaxSegs];
  int64_t seg_base[kEpMaxSegs];
  int64_t seg_limit[kEpMaxSegs];
  uint64_t peer_recv[kEpMaxRanks];
};

// Row index of permuted row p in the receive buffer of the rank that
// computes it (that rank in *dest_rank); -1 if the row is not sent (or would
// overflow).
__device__ __forceinline__ int64_t ep_dest_row(const EpRoute* route, int64_t p, int* dest_rank) {
  const int64_t t = p >> 7;
  const int n = route->n_seg;
  for (int s = 0; s < n; ++s) {
    const int64_t lo = route->seg_lo[s], hi = route->seg_hi[s];
    if (t >= lo && t < hi) {
      if (t - lo >= route->seg_limit[s]) return -1;
      *dest_rank = route->seg_rank[s];
      return (route->seg_base[s] + (t - lo)) * 128 + (p & 127);
    }
  }
  return -1;
}

// Destination row of permuted row p on its receiving rank (nullptr if p is
// not sent). Rows are 16-byte chunked (nchunk chunks per row).
struct EpRows {
  static constexpr bool kSystemFence = true;  // rows land in other GPUs' memory
  const EpRoute* route;
  int nchunk;
  __device__ __forceinline__ uint4* row(int64_t p) const {
    int r = 0;
    const int64_t drow = ep_dest_row(route, p, &r);
    return drow < 0 ? nullptr : reinterpret_cast<uint4*>(route->peer_recv[r]) + drow * nchunk;
  }
};

// Tiled TMA descriptor (128-byte swizzle, zero OOB fill) for a row-major
// tensor of rank 1 to 5; dims and box innermost first, strides in bytes.
bool encode_tmap(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                 const uint32_t* box, CUtensorMapDataType dt);

// Set the message returned by agm_last_error() (thread-local).
void set_last_error(const std::string& msg);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device)
// and size: later calls that need no more shared memory make no CUDA call, so
// a forward issued inside a stream capture only enqueues work.
cudaError_t ensure_dynamic_smem(const void* func, int bytes);

cudaError_t router_topk(int dtype, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                        int tie_low_first, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                        int32_t* block_hist, int* err, int num_sms, cudaStream_t stream);
// Decode front (router_topk.cu): router, dispatch plan and permute of at most
// one 128-token dispatch block in one launch (a cluster of 8 CTAs), with the
// outputs of router_topk + dispatch_plan + permute_rows; the logits are fp32
// dot products (CUDA cores) rounded once to the dtype.
struct FrontOut {
  int32_t* block_hist;
  int32_t* block_off;
  int32_t* counts;
  int32_t* seg_start;
  int32_t* tile_expert;
  int32_t* num_tiles;
  int32_t* token_of;
  int32_t* row_of;
  void* x_perm;
  int64_t max_rows;
  int max_tiles;
  int seg_align;
  int zero_pad;
};
bool decode_front_supported(int dtype, int64_t n_tokens, int d, int E, int k);
cudaError_t decode_front(int dtype, const void* x, const void* w, int64_t n_tokens, int d, int E, int k,
                         int tie_low_first, float* logits_out, int32_t* idx, void* gates, const FrontOut& o, int* err,
                         cudaStream_t stream);
// Shared memory of the SIMT router (fp32, or caller-supplied logits).
size_t router_smem_bytes(int d, int E);
// Whether the tensor-core router (bf16/fp16) handles this d.
bool router_tc_supported(int d);
// seg_align: expert segments start at multiples of this many rows (128, or
// 256 for the CTA-pair GEMM).
cudaError_t dispatch_plan(const int32_t* block_hist, int n_blocks, int E, int64_t max_rows, int max_tiles,
                          int seg_align, int32_t* block_off, int32_t* counts, int32_t* seg_start,
                          int32_t* tile_expert, int32_t* num_tiles, int32_t* token_of, int* err, cudaStream_t stream);
// zero_pad: zero-fill each segment's padding rows of x_perm (false only where
// nothing reads them: the swapped-operand GEMMs, whose output columns of a
// padding row are computed from that row alone and never written).
cudaError_t permute_rows(const void* x, int elem_bytes, int64_t n_tokens, int d, int k, int E, const int32_t* idx,
                         const int32_t* block_off, const int32_t* seg_start, const int32_t* counts, int64_t max_rows,
                         void* x_perm, int32_t* row_of, int32_t* token_of, int* err, cudaStream_t stream,
                         bool zero_pad = true);
cudaError_t permute_rows_ep(const void* x, int elem_bytes, int64_t n_tokens, int d, int k, int E, const int32_t* idx,
                            const int32_t* block_off, const int32_t* seg_start, const int32_t* counts,
                            int64_t max_rows, const EpRoute* route, int32_t* row_of, int* err, cudaStream_t stream);
// force_bn: 0 = auto, 128 / 256 = one-CTA tile width, -1 = CTA pairs,
// -2 = swapped operands over expert segments (args.seg_start / seg_count).
cudaError_t grouped_gemm(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                         int num_sms, cudaStream_t stream, int force_bn);
cudaError_t grouped_gemm_pair(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                              int num_sms, cudaStream_t stream);
// 16-bit weight [groups][n][k] -> the decode tile layout [groups][n/128][k/64][128][64].
cudaError_t decode_tile_layout(const void* src, void* dst, int64_t groups, int n, int k, int num_sms,
                               cudaStream_t stream);
cudaError_t grouped_gemm_swap(int dtype, const void* a, int64_t a_rows, const void* w, const GemmArgs& args, bool relu,
                              int num_sms, cudaStream_t stream);
// Backward grouped GEMMs (grouped_gemm_bwd.cu).
//   dgrad: c[r, n] = sum_k dc[r, k] * w[g(r), k, n]  (w [groups, k, n]; g from
//          the tile table, row tiles of 128), masked by aux[r, n] > 0 when
//          relu_mask (ReLU backward on the saved activation aux [rows, ld_aux]).
//   wgrad: c[g, m, n] = sum_{r in segment g} dc[r, m] * act[r, n], the
//          segment rows [seg_start[g], seg_start[g+1]) (whole 128-row tiles,
//          zero padding rows); c is fp32 (out_f32, the value rounded to the
//          compute dtype first) or the compute dtype.
struct BwdGemmArgs {
  void* c = nullptr;
  int64_t ldc = 0;
  int64_t c_rows = 0;          // dgrad: rows of c that exist
  int m = 0;                   // wgrad: rows of each group's c
  int n = 0;
  int k = 0;                   // dgrad: inner dimension
  int groups = 1;
  const int32_t* tile_group = nullptr;  // dgrad
  const int32_t* num_tiles = nullptr;   // dgrad
  int max_tiles = 0;                    // dgrad
  const int32_t* seg_start = nullptr;   // wgrad: [groups + 1]
  const void* aux = nullptr;            // dgrad relu_mask, fp32: the activation [rows, ld_aux]
  int64_t ld_aux = 0;
  const uint32_t* aux_bits = nullptr;   // dgrad relu_mask, 16-bit: GemmArgs::relu_bits of the forward
  int64_t ld_aux_bits = 0;
  // dgrad, nullable: fp32 column sums of c per 32-row quarter of each row
  // tile, [max_tiles * 4, n] (the bias gradient of the layer c feeds).
  float* col_part = nullptr;
  int* err = nullptr;
};
cudaError_t grouped_gemm_dgrad(int dtype, const void* dc, int64_t rows, const void* w, const BwdGemmArgs& args,
                               bool relu_mask, int num_sms, cudaStream_t stream);
cudaError_t grouped_gemm_wgrad(int dtype, bool out_f32, const void* dc, const void* act, int64_t rows,
                               const BwdGemmArgs& args, int num_sms, cudaStream_t stream);
// The same on CTA pairs (grouped_gemm_bwd_pair.cu, 16-bit dtypes): 256 x 256
// tiles; dgrad needs row tiles 2i and 2i+1 in one group (256-row segments).
cudaError_t grouped_gemm_dgrad_pair(int dtype, const void* dc, int64_t rows, const void* w, const BwdGemmArgs& args,
                                    bool relu_mask, int num_sms, cudaStream_t stream);
cudaError_t grouped_gemm_wgrad_pair(int dtype, bool out_f32, const void* dc, const void* act, int64_t rows,
                                    const BwdGemmArgs& args, int num_sms, cudaStream_t stream);
// residual (nullable, [n, d]): added last, out = residual + (routed + shared).
cudaError_t combine(int dtype, const void* y, const int32_t* row_of, const void* gates, int64_t n, int d, int k,
                    const void* shared_y, int n_shared, int64_t shared_stride, const void* residual, void* out,
                    int num_sms, cudaStream_t stream);

}  // namespace agm
