// MoE block forward on HOST buffers, pipelined over token chunks.
//
// The reference's inference moves activations between host and device around
// the block when layers are paged (agillm41.py:7656-7668, block-stream) and a
// host-side caller of this library hands it host memory. Copying the whole
// batch in, running the block and copying the result out leaves the GPU idle
// during both copies. Tokens are independent in the MoE block, so this entry
// point splits the batch into chunks and overlaps, on three streams,
//   H2D of chunk c+1   |   forward of chunk c   |   D2H of chunk c-1
// with two device slots for inputs and two for outputs. The result is
// bit-identical to agm_moe_forward on the whole batch (every kernel computes a
// token from that token's row only).
//
// Streams/events: the forward runs on the caller's stream; the copies run on
// two non-blocking streams per device that the library creates on first use
// and keeps. When the call returns, all work is enqueued and the caller's
// stream waits for the last device->host copy, so synchronising that stream
// means the host output is ready. Host buffers should be page-locked for the
// copies to overlap (pageable memory still gives correct results). Calls on
// one device are serialised on an internal lock while they enqueue.
#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr int kMaxDevices = 64;

struct CopyCtx {
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_h2d[2] = {}, ev_fwd[2] = {}, ev_d2h[2] = {};
};

std::mutex g_mu;
CopyCtx g_ctx[kMaxDevices];

int cuda_err(cudaError_t e, const char* what) {
  agm::set_last_error(std::string("agm_moe_forward_host: ") + what + ": " + cudaGetErrorString(e));
  return AGM_ERR_CUDA;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

extern "C" {

AGM_API size_t agm_moe_host_workspace_bytes(int64_t chunk_tokens, int d, int n_experts, int top_k, int hidden,
                                            int n_shared, int shared_hidden, int dtype) {
  const int eb = dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16 ? 2 : 0);
  if (!eb || chunk_tokens <= 0) return 0;
  const size_t fwd = agm_moe_workspace_bytes(chunk_tokens, d, n_experts, top_k, hidden, n_shared,
                                             shared_hidden > 0 ? shared_hidden : 1, dtype);
  if (!fwd) return 0;
  const size_t slot = static_cast<size_t>(round_up(static_cast<int64_t>(eb) * chunk_tokens * d, 256));
  return static_cast<size_t>(round_up(static_cast<int64_t>(fwd), 256)) + 4 * slot;
}

AGM_API int agm_moe_forward_host(const void* x_host, int dtype, int64_t n_tokens, int d, int n_experts, int top_k,
                                 int hidden, const void* w_router, const void* w1, const void* b1, const void* w2,
                                 const void* b2, int n_shared, int shared_hidden, const void* ws1, const void* sb1,
                                 const void* ws2, const void* sb2, void* out_host, void* workspace,
                                 size_t workspace_bytes, int64_t chunk_tokens, int flags, void* stream_) {
  const int eb = dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16 ? 2 : 0);
  if (!eb) {
    agm::set_last_error("agm_moe_forward_host: bad dtype");
    return AGM_ERR_ARG;
  }
  if (n_tokens < 0 || chunk_tokens <= 0) {
    agm::set_last_error("agm_moe_forward_host: n_tokens < 0 or chunk_tokens <= 0");
    return AGM_ERR_ARG;
  }
  if (n_tokens == 0) return AGM_OK;
  if (!x_host || !out_host || !workspace) {
    agm::set_last_error("agm_moe_forward_host: null pointer argument");
    return AGM_ERR_ARG;
  }
  chunk_tokens = std::min(chunk_tokens, n_tokens);
  const size_t need = agm_moe_host_workspace_bytes(chunk_tokens, d, n_experts, top_k, hidden, n_shared,
                                                   shared_hidden, dtype);
  if (!need || need > workspace_bytes) {
    agm::set_last_error("agm_moe_forward_host: workspace too small (need " + std::to_string(need) + " bytes)");
    return AGM_ERR_WORKSPACE;
  }
  const size_t fwd_bytes = static_cast<size_t>(
      round_up(static_cast<int64_t>(agm_moe_workspace_bytes(chunk_tokens, d, n_experts, top_k, hidden, n_shared,
                                                             shared_hidden > 0 ? shared_hidden : 1, dtype)),
               256));
  const size_t slot_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(eb) * chunk_tokens * d, 256));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* fwd_ws = ws;
  uint8_t* xs[2] = {ws + fwd_bytes, ws + fwd_bytes + slot_bytes};
  uint8_t* os[2] = {ws + fwd_bytes + 2 * slot_bytes, ws + fwd_bytes + 3 * slot_bytes};

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    agm::set_last_error("agm_moe_forward_host: device ordinal beyond 63");
    return AGM_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  CopyCtx& C = g_ctx[dev];
  if (!C.ready) {
    if ((e = cudaStreamCreateWithFlags(&C.h2d, cudaStreamNonBlocking)) != cudaSuccess) return cuda_err(e, "stream");
    if ((e = cudaStreamCreateWithFlags(&C.d2h, cudaStreamNonBlocking)) != cudaSuccess) return cuda_err(e, "stream");
    for (int i = 0; i < 2; ++i) {
      if ((e = cudaEventCreateWithFlags(&C.ev_h2d[i], cudaEventDisableTiming)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&C.ev_fwd[i], cudaEventDisableTiming)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&C.ev_d2h[i], cudaEventDisableTiming)) != cudaSuccess)
        return cuda_err(e, "event");
    }
    C.ready = true;
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream_);
  // The copy streams must not start before work the caller already queued
  // (e.g. producing the weights) has finished: order them after `cs`.
  if ((e = cudaEventRecord(C.ev_fwd[0], cs)) != cudaSuccess) return cuda_err(e, "record");
  if ((e = cudaStreamWaitEvent(C.h2d, C.ev_fwd[0], 0)) != cudaSuccess) return cuda_err(e, "wait");
  if ((e = cudaStreamWaitEvent(C.d2h, C.ev_fwd[0], 0)) != cudaSuccess) return cuda_err(e, "wait");

  // One clear of the error word; every chunk's forward then accumulates into it.
  if ((e = cudaMemsetAsync(fwd_ws, 0, sizeof(int), cs)) != cudaSuccess) return cuda_err(e, "memset");
  const uint8_t* xh = static_cast<const uint8_t*>(x_host);
  uint8_t* oh = static_cast<uint8_t*>(out_host);
  const int64_t n_chunks = (n_tokens + chunk_tokens - 1) / chunk_tokens;
  const size_t row_bytes = static_cast<size_t>(eb) * d;
  for (int64_t c = 0; c < n_chunks; ++c) {
    const int s = static_cast<int>(c & 1);
    const int64_t t0 = c * chunk_tokens;
    const int64_t nt = std::min(chunk_tokens, n_tokens - t0);
    const size_t bytes = row_bytes * nt;
    // H2D of this chunk once the forward that last read slot s is done.
    if (c >= 2 && (e = cudaStreamWaitEvent(C.h2d, C.ev_fwd[s], 0)) != cudaSuccess) return cuda_err(e, "wait");
    if ((e = cudaMemcpyAsync(xs[s], xh + row_bytes * t0, bytes, cudaMemcpyHostToDevice, C.h2d)) != cudaSuccess)
      return cuda_err(e, "H2D copy");
    if ((e = cudaEventRecord(C.ev_h2d[s], C.h2d)) != cudaSuccess) return cuda_err(e, "record");
    // Forward once the input is in and the D2H that last read out slot s is done.
    if ((e = cudaStreamWaitEvent(cs, C.ev_h2d[s], 0)) != cudaSuccess) return cuda_err(e, "wait");
    if (c >= 2 && (e = cudaStreamWaitEvent(cs, C.ev_d2h[s], 0)) != cudaSuccess) return cuda_err(e, "wait");
    const int rc = agm_moe_forward(xs[s], dtype, nt, d, n_experts, top_k, hidden, w_router, w1, b1, w2, b2, n_shared,
                                   shared_hidden, ws1, sb1, ws2, sb2, os[s], fwd_ws, fwd_bytes,
                                   flags | AGM_FLAG_KEEP_ERROR, nullptr,
                                   nullptr, nullptr, nullptr, nullptr, nullptr, cs);
    if (rc != AGM_OK) return rc;
    if ((e = cudaEventRecord(C.ev_fwd[s], cs)) != cudaSuccess) return cuda_err(e, "record");
    // D2H of this chunk's output.
    if ((e = cudaStreamWaitEvent(C.d2h, C.ev_fwd[s], 0)) != cudaSuccess) return cuda_err(e, "wait");
    if ((e = cudaMemcpyAsync(oh + row_bytes * t0, os[s], bytes, cudaMemcpyDeviceToHost, C.d2h)) != cudaSuccess)
      return cuda_err(e, "D2H copy");
    if ((e = cudaEventRecord(C.ev_d2h[s], C.d2h)) != cudaSuccess) return cuda_err(e, "record");
  }
  // The caller's stream completes after the last copy out.
  const int last = static_cast<int>((n_chunks - 1) & 1);
  if ((e = cudaStreamWaitEvent(cs, C.ev_d2h[last], 0)) != cudaSuccess) return cuda_err(e, "wait");
  if (n_chunks > 1 && (e = cudaStreamWaitEvent(cs, C.ev_d2h[last ^ 1], 0)) != cudaSuccess)
    return cuda_err(e, "wait");
  return AGM_OK;
}

}  // extern "C"
