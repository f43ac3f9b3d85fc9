// C ABI of the MoE block forward: argument checks, workspace layout and the
// launch sequence that replaces MoEFFN.forward (agillm41.py:4389-4431).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "common.cuh"
#include "kernels.h"


namespace {

thread_local std::string g_err;


int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_err = std::string(where) + ": " + cudaGetErrorString(e);
  return AGM_ERR_CUDA;
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case AGM_F32: return 4;
    case AGM_BF16: return 2;
    case AGM_F16: return 2;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms_current() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }


int check_common(int dtype, int d, int n_experts, int top_k) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(AGM_ERR_ARG, "dtype must be AGM_F32, AGM_BF16 or AGM_F16");
  if (d <= 0 || (d * eb) % 16 != 0)
    return fail(AGM_ERR_UNSUPPORTED, "d * sizeof(dtype) must be a positive multiple of 16 bytes");
  if (n_experts < 1 || n_experts > AGM_MAX_EXPERTS)
    return fail(AGM_ERR_UNSUPPORTED, "number of experts must be in [1, 16]");
  if (top_k < 1 || top_k > n_experts) return fail(AGM_ERR_ARG, "top_k must be in [1, n_experts]");
  return AGM_OK;
}

// The router keeps its weight in shared memory: the tensor-core router (bf16,
// fp16) holds it as 16-bit tiles, the SIMT router (fp32, or routing from
// caller-supplied logits) as fp32.
bool router_fits(int dtype, int d, int n_experts, bool logits_in) {
  if (logits_in) return agm::router_smem_bytes(0, n_experts) <= 227 * 1024;
  if (dtype != AGM_F32 && agm::router_tc_supported(d)) return true;
  return agm::router_smem_bytes(d, n_experts) <= 227 * 1024;
}

struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename P>
  P* take(size_t bytes) {
    off = (off + 255) & ~size_t(255);
    P* p = reinterpret_cast<P*>(base ? base + off : nullptr);
    off += bytes;
    return p;
  }
};

struct FwdLayout {
  int* err;
  int32_t* idx;
  void* gates;
  int32_t* block_hist;
  int32_t* block_off;
  int32_t* counts;
  int32_t* seg_start;
  int32_t* num_tiles;
  int32_t* tile_expert;
  int32_t* row_of;
  int32_t* token_of;
  void* x_perm;  // also holds y (FC2 output) once FC1 has consumed x_perm
  void* h;
  void* h_sh;
  void* y_sh;
  size_t bytes;
};

FwdLayout carve(void* ws, int64_t n, int d, int E, int k, int H, int S, int Hs, int eb) {
  Carver c(ws);
  FwdLayout L;
  const int64_t nb = agm_dispatch_blocks(n);
  const int64_t rows = agm_max_rows(n, k, E);
  const int64_t npad = round_up(std::max<int64_t>(n, 1), AGM_TILE_M);
  L.err = c.take<int>(sizeof(int));
  L.idx = c.take<int32_t>(sizeof(int32_t) * n * k);
  L.gates = c.take<void>(static_cast<size_t>(eb) * n * k);
  L.block_hist = c.take<int32_t>(sizeof(int32_t) * nb * E);
  L.block_off = c.take<int32_t>(sizeof(int32_t) * nb * E);
  L.counts = c.take<int32_t>(sizeof(int32_t) * E);
  L.seg_start = c.take<int32_t>(sizeof(int32_t) * (E + 1));
  L.num_tiles = c.take<int32_t>(sizeof(int32_t));
  L.tile_expert = c.take<int32_t>(sizeof(int32_t) * (rows / AGM_TILE_M));
  L.row_of = c.take<int32_t>(sizeof(int32_t) * n * k);
  L.token_of = c.take<int32_t>(sizeof(int32_t) * rows);
  L.x_perm = c.take<void>(static_cast<size_t>(eb) * rows * d);
  L.h = c.take<void>(static_cast<size_t>(eb) * rows * H);
  L.h_sh = S > 0 ? c.take<void>(static_cast<size_t>(eb) * S * npad * Hs) : nullptr;  // [S, npad, Hs]
  L.y_sh = S > 0 ? c.take<void>(static_cast<size_t>(eb) * S * npad * d) : nullptr;
  L.bytes = (c.off + 255) & ~size_t(255);
  return L;
}

}  // namespace

namespace agm {
void set_last_error(const std::string& msg) { g_err = msg; }

namespace {
thread_local int tl_pdl = -1;  // -1: no forward scope on this thread
}

bool pdl_enabled() {
  static const bool env_off = [] {
    const char* v = std::getenv("AGM_NO_PDL");
    return v && v[0] == '1';
  }();
  if (env_off) return false;
  return tl_pdl != 0;
}

PdlScope::PdlScope(bool on) : prev(tl_pdl != 0) { tl_pdl = on ? 1 : 0; }
PdlScope::~PdlScope() { tl_pdl = prev ? 1 : 0; }

cudaError_t ensure_dynamic_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{func, dev}];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}
}  // namespace agm

extern "C" {

const char* agm_last_error(void) { return g_err.c_str(); }

int agm_abi_version(void) { return AGM_ABI_VERSION; }

int64_t agm_dispatch_blocks(int64_t n_tokens) {
  return n_tokens <= 0 ? 0 : (n_tokens + AGM_DISPATCH_BLOCK - 1) / AGM_DISPATCH_BLOCK;
}

int64_t agm_max_rows(int64_t n_tokens, int top_k, int n_experts) {
  if (n_tokens <= 0) return 0;
  const int64_t kn = static_cast<int64_t>(top_k) * n_tokens;
  const int64_t align = kn >= AGM_PAIR_MIN_ROWS ? AGM_PAIR_ROWS : AGM_TILE_M;
  return round_up(kn + static_cast<int64_t>(n_experts) * (align - 1), align);
}

int agm_router_topk(const void* x, const void* w_router, int dtype, int64_t n_tokens, int d, int n_experts,
                    int top_k, int flags, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                    int32_t* block_hist, int* err, void* stream) {
  int rc = check_common(dtype, d, n_experts, top_k);
  if (rc) return rc;
  if (n_tokens < 0) return fail(AGM_ERR_ARG, "n_tokens < 0");
  if (n_tokens == 0) return AGM_OK;
  if (!idx || !gates || !block_hist || (!logits_in && (!x || !w_router)))
    return fail(AGM_ERR_ARG, "null pointer argument");
  if (!logits_in && (!aligned16(x) || !aligned16(w_router)))
    return fail(AGM_ERR_ARG, "x and w_router must be 16-byte aligned");
  if (!router_fits(dtype, d, n_experts, logits_in != nullptr))
    return fail(AGM_ERR_UNSUPPORTED, "router weight does not fit in shared memory for this d and dtype");
  cudaError_t e = agm::router_topk(dtype, x, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST,
                                   logits_in, logits_out, idx, gates, block_hist, err, num_sms_current(),
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "router_topk");
}

int agm_dispatch_plan(const int32_t* block_hist, int64_t n_tokens, int n_experts, int top_k, int32_t* block_off,
                      int32_t* counts, int32_t* seg_start, int32_t* tile_expert, int32_t* num_tiles,
                      int32_t* token_of, int* err, void* stream) {
  if (n_experts < 1 || n_experts > AGM_MAX_EXPERTS) return fail(AGM_ERR_UNSUPPORTED, "experts must be in [1, 16]");
  if (n_tokens < 0 || top_k < 1 || top_k > n_experts) return fail(AGM_ERR_ARG, "bad n_tokens or top_k");
  if (!block_off || !counts || !seg_start || !tile_expert || !num_tiles || !token_of || (n_tokens > 0 && !block_hist))
    return fail(AGM_ERR_ARG, "null pointer argument");
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  if (rows > INT32_MAX) return fail(AGM_ERR_UNSUPPORTED, "too many permuted rows for int32 indices");
  cudaError_t e = agm::dispatch_plan(block_hist, static_cast<int>(agm_dispatch_blocks(n_tokens)), n_experts, rows,
                                     static_cast<int>(rows / AGM_TILE_M), AGM_TILE_M, block_off, counts, seg_start,
                                     tile_expert, num_tiles, token_of, err, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "dispatch_plan");
}

int agm_permute(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, const int32_t* idx,
                const int32_t* block_off, const int32_t* seg_start, const int32_t* counts, void* x_perm,
                int32_t* row_of, int32_t* token_of, int* err, void* stream) {
  int rc = check_common(dtype, d, n_experts, top_k);
  if (rc) return rc;
  if (n_tokens <= 0) return n_tokens < 0 ? fail(AGM_ERR_ARG, "n_tokens < 0") : AGM_OK;
  if (!x || !idx || !block_off || !seg_start || !counts || !x_perm || !row_of || !token_of)
    return fail(AGM_ERR_ARG, "null pointer argument");
  if (!aligned16(x) || !aligned16(x_perm)) return fail(AGM_ERR_ARG, "x and x_perm must be 16-byte aligned");
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  cudaError_t e = agm::permute_rows(x, elem_bytes(dtype), n_tokens, d, top_k, n_experts, idx, block_off, seg_start,
                                    counts, rows, x_perm, row_of, token_of, err, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "permute");
}

int agm_grouped_gemm(const void* a, int64_t a_rows, const void* w, const void* bias, int dtype, int groups,
                     int n_out, int k_in, const int32_t* tile_group, const int32_t* num_tiles, int64_t max_tiles,
                     int relu, int force_bn, void* c, int64_t c_rows, int* err, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(AGM_ERR_ARG, "bad dtype");
  if (max_tiles <= 0 || n_out <= 0 || c_rows <= 0) return AGM_OK;
  if (!a || !w || !c) return fail(AGM_ERR_ARG, "null pointer argument");
  if (groups < 1 || k_in <= 0 || a_rows <= 0) return fail(AGM_ERR_ARG, "bad groups / k_in / a_rows");
  if ((static_cast<int64_t>(k_in) * eb) % 16 || (static_cast<int64_t>(n_out) * eb) % 16)
    return fail(AGM_ERR_UNSUPPORTED, "k_in and n_out must be multiples of 16 bytes of dtype");
  if (!aligned16(a) || !aligned16(w) || !aligned16(c) || (bias && !aligned16(bias)))
    return fail(AGM_ERR_ARG, "a, w, bias and c must be 16-byte aligned");
  if (max_tiles > INT32_MAX / 2) return fail(AGM_ERR_UNSUPPORTED, "too many tiles");
  if (force_bn != 0 && force_bn != 128 && force_bn != 256 && force_bn != AGM_GEMM_PAIR)
    return fail(AGM_ERR_ARG, "force_bn must be 0, 128, 256 or AGM_GEMM_PAIR");
  agm::GemmArgs ga;
  ga.c = c;
  ga.ldc = n_out;
  ga.c_rows = c_rows;
  ga.bias = bias;
  ga.n = n_out;
  ga.k = k_in;
  ga.groups = groups;
  ga.tile_group = tile_group;
  ga.num_tiles = num_tiles;
  ga.max_tiles = static_cast<int>(max_tiles);
  ga.err = err;
  cudaError_t e = agm::grouped_gemm(dtype, a, a_rows, w, ga, relu != 0, num_sms_current(),
                                    static_cast<cudaStream_t>(stream), force_bn);
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "grouped_gemm");
}

int agm_combine(const void* y_perm, const int32_t* row_of, const void* gates, int dtype, int64_t n_tokens, int d,
                int top_k, const void* shared_y, int n_shared, int64_t shared_stride_rows, void* out, void* stream) {
  const int eb = elem_bytes(dtype);
  if (!eb) return fail(AGM_ERR_ARG, "bad dtype");
  if (n_tokens <= 0) return n_tokens < 0 ? fail(AGM_ERR_ARG, "n_tokens < 0") : AGM_OK;
  if (d <= 0 || (d * eb) % 16) return fail(AGM_ERR_UNSUPPORTED, "d * sizeof(dtype) must be a multiple of 16");
  if (top_k < 1 || top_k > AGM_MAX_EXPERTS) return fail(AGM_ERR_ARG, "bad top_k");
  if (!y_perm || !row_of || !gates || !out || (n_shared > 0 && !shared_y))
    return fail(AGM_ERR_ARG, "null pointer argument");
  if (!aligned16(y_perm) || !aligned16(out) || (shared_y && !aligned16(shared_y)))
    return fail(AGM_ERR_ARG, "y_perm, shared_y and out must be 16-byte aligned");
  cudaError_t e = agm::combine(dtype, y_perm, row_of, gates, n_tokens, d, top_k, shared_y, n_shared,
                               shared_stride_rows * d, nullptr, out, num_sms_current(),
                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "combine");
}

size_t agm_moe_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int n_shared,
                               int shared_hidden, int dtype) {
  const int eb = elem_bytes(dtype);
  if (!eb || n_tokens < 0 || d <= 0 || n_experts < 1 || top_k < 1 || hidden <= 0) return 0;
  return carve(nullptr, n_tokens, d, n_experts, top_k, hidden, std::max(0, n_shared), std::max(1, shared_hidden), eb)
      .bytes;
}

}  // extern "C"

namespace {

// agm_moe_forward with an optional residual added in the combine.
int moe_forward_impl(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                     const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                     int n_shared, int shared_hidden, const void* ws1, const void* sb1, const void* ws2,
                     const void* sb2, const void* residual, void* out, void* workspace, size_t workspace_bytes,
                     int flags, int32_t* idx_out, void* gates_out, int32_t* counts_out, float* logits_out,
                     const float* logits_in, void* const* stage_events, void* stream_) {
  if (residual && !aligned16(residual)) return fail(AGM_ERR_ARG, "residual must be 16-byte aligned");
  int rc = check_common(dtype, d, n_experts, top_k);
  if (rc) return rc;
  const int eb = elem_bytes(dtype);
  if (n_tokens < 0) return fail(AGM_ERR_ARG, "n_tokens < 0");
  if (hidden <= 0 || (static_cast<int64_t>(hidden) * eb) % 16)
    return fail(AGM_ERR_UNSUPPORTED, "hidden * sizeof(dtype) must be a positive multiple of 16 bytes");
  if (n_shared < 0) return fail(AGM_ERR_ARG, "n_shared < 0");
  if (n_shared > 0 && (shared_hidden <= 0 || (static_cast<int64_t>(shared_hidden) * eb) % 16))
    return fail(AGM_ERR_UNSUPPORTED, "shared_hidden * sizeof(dtype) must be a positive multiple of 16 bytes");
  if (!x || !w_router || !w1 || !b1 || !w2 || !b2 || !out || !workspace)
    return fail(AGM_ERR_ARG, "null pointer argument");
  if (n_shared > 0 && (!ws1 || !sb1 || !ws2 || !sb2)) return fail(AGM_ERR_ARG, "null shared-expert pointer");
  const void* ptrs[] = {x, w_router, w1, b1, w2, b2, out, workspace};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  if (n_shared > 0 && (!aligned16(ws1) || !aligned16(sb1) || !aligned16(ws2) || !aligned16(sb2)))
    return fail(AGM_ERR_ARG, "all tensors must be 16-byte aligned");
  if (!router_fits(dtype, d, n_experts, logits_in != nullptr))
    return fail(AGM_ERR_UNSUPPORTED, "router weight does not fit in shared memory for this d and dtype");
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  if (rows > INT32_MAX) return fail(AGM_ERR_UNSUPPORTED, "too many permuted rows for int32 indices");
  FwdLayout L = carve(workspace, n_tokens, d, n_experts, top_k, hidden, n_shared, std::max(1, shared_hidden), eb);
  if (L.bytes > workspace_bytes) return fail(AGM_ERR_WORKSPACE, "workspace too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  auto mark = [&](int i) -> cudaError_t {
    return stage_events ? cudaEventRecord(static_cast<cudaEvent_t>(stage_events[i]), stream) : cudaSuccess;
  };
  agm::PdlScope pdl_scope(!(flags & AGM_FLAG_NO_PDL));
  cudaError_t e = cudaSuccess;
  if (!(flags & AGM_FLAG_KEEP_ERROR)) {
    e = cudaMemsetAsync(L.err, 0, sizeof(int), stream);
    if (e != cudaSuccess) return cuda_fail(e, "memset");
  }
  if (n_tokens == 0) {
    for (int i = 0; i < AGM_STAGE_EVENTS && e == cudaSuccess; ++i) e = mark(i);
    return e == cudaSuccess ? AGM_OK : cuda_fail(e, "event record");
  }
  int32_t* idx = idx_out ? idx_out : L.idx;
  void* gates = gates_out ? gates_out : L.gates;
  const int sms = num_sms_current();
  const int64_t max_tiles = rows / AGM_TILE_M;
  // Expert GEMMs on CTA pairs (256 x 256 tiles; expert segments padded to
  // 256 rows) once there are enough rows that the extra padding is small:
  // about E x 64 more rows on average, under 6% of k x n from the threshold up.
  const bool pair = dtype != AGM_F32 && !(flags & AGM_FLAG_NO_PAIR) &&
                    static_cast<int64_t>(top_k) * n_tokens >= AGM_PAIR_MIN_ROWS;
  // Decode-sized batches: swapped operands, so the weights stream at full
  // depth and only the valid rows of each segment enter the MMA.
  const bool swap = dtype != AGM_F32 && !(flags & AGM_FLAG_NO_SWAP) &&
                    static_cast<int64_t>(top_k) * n_tokens <= static_cast<int64_t>(AGM_SWAP_ROWS_PER_EXPERT) * n_experts;
  const bool tiled = (flags & AGM_FLAG_DECODE_TILES) != 0;
  if (tiled && (!swap || hidden % 128 || d % 128))
    return fail(AGM_ERR_UNSUPPORTED, "decode tile layout: decode-sized batches (top_k * n_tokens <= 32 * n_experts), "
                                     "16-bit dtypes, d and hidden multiples of 128");
  const int seg_align = pair ? AGM_PAIR_ROWS : AGM_TILE_M;
  const int gemm_mode = pair ? AGM_GEMM_PAIR : (swap ? -2 : 0);

  if ((e = mark(0)) != cudaSuccess) return cuda_fail(e, "event record");
  // The swapped-operand GEMMs read no padding row of x_perm into a written
  // output: its zero-fill (E x up to 127 rows) is skipped.
  const bool zero_pad = gemm_mode != -2;
  // At most one dispatch block (decode): router, plan and permute in one
  // cluster launch, with the same outputs.
  const bool front = !(flags & AGM_FLAG_NO_FRONT) && !logits_in &&
                     agm::decode_front_supported(dtype, n_tokens, d, n_experts, top_k);
  if (front) {
    agm::FrontOut fo{L.block_hist, L.block_off,  L.counts, L.seg_start,          L.tile_expert,
                     L.num_tiles,  L.token_of,   L.row_of, L.x_perm,             rows,
                     static_cast<int>(max_tiles), seg_align, zero_pad ? 1 : 0};
    e = agm::decode_front(dtype, x, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST,
                          logits_out, idx, gates, fo, L.err, stream);
    if (e != cudaSuccess) return cuda_fail(e, "decode_front");
    for (int i = 1; i <= 3 && e == cudaSuccess; ++i) e = mark(i);
    if (e != cudaSuccess) return cuda_fail(e, "event record");
  } else {
    e = agm::router_topk(dtype, x, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST,
                         logits_in, logits_out, idx, gates, L.block_hist, L.err, sms, stream);
    if (e != cudaSuccess) return cuda_fail(e, "router_topk");
    if ((e = mark(1)) != cudaSuccess) return cuda_fail(e, "event record");
    e = agm::dispatch_plan(L.block_hist, static_cast<int>(agm_dispatch_blocks(n_tokens)), n_experts, rows,
                           static_cast<int>(max_tiles), seg_align, L.block_off, L.counts, L.seg_start, L.tile_expert,
                           L.num_tiles, L.token_of, L.err, stream);
    if (e != cudaSuccess) return cuda_fail(e, "dispatch_plan");
    if ((e = mark(2)) != cudaSuccess) return cuda_fail(e, "event record");
    e = agm::permute_rows(x, eb, n_tokens, d, top_k, n_experts, idx, L.block_off, L.seg_start, L.counts, rows,
                          L.x_perm, L.row_of, L.token_of, L.err, stream, zero_pad);
    if (e != cudaSuccess) return cuda_fail(e, "permute");
    if ((e = mark(3)) != cudaSuccess) return cuda_fail(e, "event record");
  }
  agm::GemmArgs g1;
  g1.c = L.h;
  g1.ldc = hidden;
  g1.c_rows = rows;
  g1.bias = b1;
  g1.n = hidden;
  g1.k = d;
  g1.groups = n_experts;
  g1.tile_group = L.tile_expert;
  g1.num_tiles = L.num_tiles;
  g1.max_tiles = static_cast<int>(max_tiles);
  g1.err = L.err;
  g1.seg_start = L.seg_start;
  g1.seg_count = L.counts;
  // The tile table and counts come from the plan, two or more launches back,
  // and the weights from before this forward: the GEMMs stream their first
  // weight tiles while the kernel before them finishes. Behind the decode
  // front the tables come from the kernel just before, so the GEMMs wait for
  // it before reading anything.
  g1.early_weights = !front;
  g1.w_tiled = tiled;
  const int64_t npad = round_up(n_tokens, AGM_TILE_M);
  // Shared experts: one dense group over all tokens, so any two row tiles
  // share their weights and the CTA-pair GEMM applies without padding.
  const int shared_mode = (dtype != AGM_F32 && !(flags & AGM_FLAG_NO_PAIR) && n_tokens >= AGM_PAIR_MIN_ROWS)
                              ? AGM_GEMM_PAIR : 0;
  // Both on CTA pairs: the shared experts ride in the routed launches as a
  // second, dense problem (one FC1 and one FC2 launch for the whole block;
  // every tile computed exactly as by its own launch).
  const bool fold = n_shared > 0 && pair && shared_mode == AGM_GEMM_PAIR && !(flags & AGM_FLAG_NO_FOLD);
  if (fold) {
    g1.groups2 = n_shared;
    g1.a2 = x;
    g1.a2_rows = n_tokens;
    g1.w2 = ws1;
    g1.bias2 = sb1;
    g1.c2 = L.h_sh;
    g1.c2_rows = n_shared * npad;
    g1.ldc2 = shared_hidden;
    g1.n2 = shared_hidden;
    g1.k2 = d;
    g1.tiles2 = static_cast<int>(npad / AGM_TILE_M);
    g1.a2_group_rows = 0;
    g1.c2_group_rows = npad;
  }
  e = agm::grouped_gemm(dtype, L.x_perm, rows, w1, g1, true, sms, stream, gemm_mode);
  if (e != cudaSuccess) return cuda_fail(e, "grouped_gemm fc1");
  if ((e = mark(4)) != cudaSuccess) return cuda_fail(e, "event record");
  agm::GemmArgs g2 = g1;
  g2.early_weights = true;  // the tables are two launches back here in both cases
  g2.c = L.x_perm;  // y reuses the x_perm buffer
  g2.ldc = d;
  g2.bias = b2;
  g2.n = d;
  g2.k = hidden;
  if (fold) {
    g2.a2 = L.h_sh;
    g2.a2_rows = n_shared * npad;
    g2.w2 = ws2;
    g2.bias2 = sb2;
    g2.c2 = L.y_sh;
    g2.c2_rows = n_shared * npad;
    g2.ldc2 = d;
    g2.n2 = d;
    g2.k2 = shared_hidden;
    g2.a2_group_rows = npad;
    g2.c2_group_rows = npad;
  }
  e = agm::grouped_gemm(dtype, L.h, rows, w2, g2, false, sms, stream, gemm_mode);
  if (e != cudaSuccess) return cuda_fail(e, "grouped_gemm fc2");
  if ((e = mark(5)) != cudaSuccess) return cuda_fail(e, "event record");

  for (int s = 0; s < (fold ? 0 : n_shared); ++s) {
    agm::GemmArgs s1;
    s1.c = L.h_sh;
    s1.ldc = shared_hidden;
    s1.c_rows = npad;
    s1.bias = static_cast<const uint8_t*>(sb1) + static_cast<size_t>(eb) * s * shared_hidden;
    s1.n = shared_hidden;
    s1.k = d;
    s1.groups = 1;
    s1.tile_group = nullptr;
    s1.num_tiles = nullptr;
    s1.max_tiles = static_cast<int>(npad / AGM_TILE_M);
    s1.err = L.err;
    s1.early_weights = true;
    e = agm::grouped_gemm(dtype, x, n_tokens, static_cast<const uint8_t*>(ws1) + static_cast<size_t>(eb) * s * shared_hidden * d,
                          s1, true, sms, stream, shared_mode);
    if (e != cudaSuccess) return cuda_fail(e, "grouped_gemm shared fc1");
    agm::GemmArgs s2 = s1;
    s2.c = static_cast<uint8_t*>(L.y_sh) + static_cast<size_t>(eb) * s * npad * d;
    s2.ldc = d;
    s2.bias = static_cast<const uint8_t*>(sb2) + static_cast<size_t>(eb) * s * d;
    s2.n = d;
    s2.k = shared_hidden;
    e = agm::grouped_gemm(dtype, L.h_sh, npad, static_cast<const uint8_t*>(ws2) + static_cast<size_t>(eb) * s * d * shared_hidden,
                          s2, false, sms, stream, shared_mode);
    if (e != cudaSuccess) return cuda_fail(e, "grouped_gemm shared fc2");
  }
  if ((e = mark(6)) != cudaSuccess) return cuda_fail(e, "event record");

  e = agm::combine(dtype, L.x_perm, L.row_of, gates, n_tokens, d, top_k, L.y_sh, n_shared, npad * d, residual, out,
                   sms, stream);
  if (e != cudaSuccess) return cuda_fail(e, "combine");
  if ((e = mark(7)) != cudaSuccess) return cuda_fail(e, "event record");
  if (counts_out) {
    e = cudaMemcpyAsync(counts_out, L.counts, sizeof(int32_t) * n_experts, cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "counts copy");
  }
  return AGM_OK;
}

}  // namespace

extern "C" {

int agm_moe_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                    const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2, int n_shared,
                    int shared_hidden, const void* ws1, const void* sb1, const void* ws2, const void* sb2, void* out,
                    void* workspace, size_t workspace_bytes, int flags, int32_t* idx_out, void* gates_out,
                    int32_t* counts_out, float* logits_out, const float* logits_in, void* const* stage_events,
                    void* stream) {
  return moe_forward_impl(x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, w1, b1, w2, b2, n_shared,
                          shared_hidden, ws1, sb1, ws2, sb2, nullptr, out, workspace, workspace_bytes, flags, idx_out,
                          gates_out, counts_out, logits_out, logits_in, stage_events, stream);
}

int agm_moe_forward_residual(const void* x, const void* residual, int dtype, int64_t n_tokens, int d, int n_experts,
                             int top_k, int hidden, const void* w_router, const void* w1, const void* b1,
                             const void* w2, const void* b2, int n_shared, int shared_hidden, const void* ws1,
                             const void* sb1, const void* ws2, const void* sb2, void* out, void* workspace,
                             size_t workspace_bytes, int flags, void* stream) {
  if (!residual) return fail(AGM_ERR_ARG, "null residual");
  return moe_forward_impl(x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, w1, b1, w2, b2, n_shared,
                          shared_hidden, ws1, sb1, ws2, sb2, residual, out, workspace, workspace_bytes, flags, nullptr,
                          nullptr, nullptr, nullptr, nullptr, nullptr, stream);
}

int agm_decode_tile_layout(const void* w, void* out, int dtype, int64_t groups, int n, int k, void* stream) {
  if (dtype != AGM_BF16 && dtype != AGM_F16)
    return fail(AGM_ERR_UNSUPPORTED, "agm_decode_tile_layout: 16-bit weights only");
  if (groups <= 0 || n <= 0 || k <= 0 || n % 128 || k % 64)
    return fail(AGM_ERR_ARG, "agm_decode_tile_layout: n must be a multiple of 128 and k of 64");
  if (!w || !out || !aligned16(w) || !aligned16(out) || w == out)
    return fail(AGM_ERR_ARG, "agm_decode_tile_layout: 16-byte aligned, distinct source and destination");
  cudaError_t e = agm::decode_tile_layout(w, out, groups, n, k, num_sms_current(), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? AGM_OK : cuda_fail(e, "agm_decode_tile_layout");
}

int agm_read_device_error(int* err, int* code, void* stream) {
  if (!err || !code) return fail(AGM_ERR_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "read device error");
  *code = host;
  if (host != 0) {
    e = cudaMemsetAsync(err, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "reset device error");
    char buf[96];
    std::snprintf(buf, sizeof(buf), "device error word 0x%x", host);
    g_err = buf;
    return AGM_ERR_DEVICE;
  }
  return AGM_OK;
}

}  // extern "C"
