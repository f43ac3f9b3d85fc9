// MoE block forward that allocates nothing: its scratch is a static device array.
//
// Who needs this: hosts that own every byte of device memory through their
// own pool and hand a plugin nothing but its input and output buffers, and
// processes that must not grow their GPU footprint (or pay the implicit
// device synchronisation of cudaMalloc) once they are running. Such callers
// cannot provide the workspace that agm_moe_forward takes, so this entry point
// uses a fixed scratch area compiled into the library instead.
//
// The scratch is one file-scope __device__ array of AGM_NOALLOC_SCRATCH_BYTES.
// Every GPU that loads this part of the library keeps it until the process
// exits. Its device address is looked up once per device (cudaGetSymbolAddress,
// on the first call made while that device is current) and then reused.
// All calls share the array and it keeps the last call's contents; the only
// state that must start at zero (the device error word, the array's first int)
// is cleared by every call, AGM_FLAG_KEEP_ERROR or not, so the word reports
// the latest call alone. agm_moe_noalloc_error_word hands its device address
// to the caller, who reads it with agm_read_device_error. Calls that overlap
// on the GPU (different streams, or different host threads on one device)
// race on the array.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[AGM_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    agm::set_last_error(std::string("agm_moe_forward_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    return AGM_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    agm::set_last_error("agm_moe_forward_noalloc: device ordinal beyond 63");
    return AGM_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      agm::set_last_error(std::string("agm_moe_forward_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      return AGM_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return AGM_OK;
}

}  // namespace

extern "C" AGM_API int agm_moe_forward_noalloc(const void* x, int dtype, int64_t n_tokens, int d, int n_experts,
                                               int top_k, int hidden, const void* w_router, const void* w1,
                                               const void* b1, const void* w2, const void* b2, int n_shared,
                                               int shared_hidden, const void* ws1, const void* sb1, const void* ws2,
                                               const void* sb2, void* out, int flags, void* stream) {
  const size_t need = agm_moe_workspace_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared,
                                              shared_hidden > 0 ? shared_hidden : 1, dtype);
  if (need > static_cast<size_t>(AGM_NOALLOC_SCRATCH_BYTES)) {
    agm::set_last_error("agm_moe_forward_noalloc: this problem needs " + std::to_string(need) +
                        " bytes of scratch but the built-in scratch holds " +
                        std::to_string(static_cast<size_t>(AGM_NOALLOC_SCRATCH_BYTES)) +
                        " bytes (AGM_NOALLOC_SCRATCH_BYTES); use fewer tokens per call or agm_moe_forward "
                        "with a caller-provided workspace");
    return AGM_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != AGM_OK) return rc;
  // Argument checks (shapes, alignment, dtype) happen in agm_moe_forward.
  // The shared error word is always cleared first: an error left by an
  // earlier, unrelated call must not be reported as this call's.
  return agm_moe_forward(x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, w1, b1, w2, b2, n_shared,
                         shared_hidden, ws1, sb1, ws2, sb2, out, scratch, AGM_NOALLOC_SCRATCH_BYTES,
                         flags & ~AGM_FLAG_KEEP_ERROR, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, stream);
}

extern "C" AGM_API int agm_moe_noalloc_error_word(int** err) {
  if (!err) {
    agm::set_last_error("agm_moe_noalloc_error_word: null pointer argument");
    return AGM_ERR_ARG;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != AGM_OK) return rc;
  *err = static_cast<int*>(scratch);
  return AGM_OK;
}
