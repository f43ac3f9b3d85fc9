// Expert-parallel MoE block forward over NVLink peer memory (one process per
// GPU), with the all-to-all fused into the kernels around the expert GEMM.
//
// The reference runs the block on one device (agillm41.py:4389-4431). Here P
// ranks each route their own tokens and share the expert FFN work; instead of
// two collective all-to-all passes, the data moves inside the kernels:
//
//   router -> local dispatch plan -> [counts to every peer + flag barrier]
//   -> device plan (global tile sequence, this rank's share)
//   -> permute: every (token, rank) row is written straight into the
//      receive buffer of the rank that computes it (NVLink stores)
//   -> [flag barrier] -> grouped FC1/FC2 on the received tiles, FC2 writes
//      into this rank's result buffer -> [flag barrier]
//   -> combine: each token's k expert rows are read straight from the result
//      buffers of the ranks that computed them (NVLink loads).
//
// No host synchronisation and no library collective: the counts exchange and
// the three barriers are flag writes/reads in peer memory with bounded waits.
//
// Every rank owns one "comm" buffer allocated with cudaMalloc (IPC-shareable),
// laid out identically on all ranks:
//   [0, 256)            signals: uint64 per source rank, monotonically raised
//                       epochs (rank r writes signal[r] on every peer)
//   [256, ...)          counts inbox: int32 [kEpMaxRanks][E] (row i from rank i)
//   off_recv            receive buffer [cap_rows, d] (rows to compute)
//   off_y               result buffer  [cap_rows, d] (their FFN outputs)
// Peers' comm buffers are mapped into this process with CUDA IPC.
//
// Placement (the global tile sequence is ordered by (expert, source, tile);
// rank r computes the contiguous range [bounds[r], bounds[r+1])):
//   0 static   - bounds at expert boundaries of contiguous ownership ranges
//                (first E mod P ranks own one more expert);
//   1 balanced - P near-equal ranges (every rank holds all expert weights);
//   2 local    - every rank holds all expert weights; each rank computes its
//                own tiles up to an equal share and only the excess moves.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace agm {

constexpr int kSigBytes = 256;

__host__ __device__ inline int64_t ep_round(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
__host__ __device__ inline int64_t ep_off_inbox() { return kSigBytes; }
__host__ __device__ inline int64_t ep_off_recv(int E) {
  return ep_round(ep_off_inbox() + static_cast<int64_t>(kEpMaxRanks) * E * 4, 4096);
}
__host__ __device__ inline int64_t ep_off_y(int E, int64_t cap_rows, int d, int eb) {
  return ep_off_recv(E) + ep_round(cap_rows * d * eb, 4096);
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct PeerComm {
  uint64_t base[kEpMaxRanks];  // every rank's comm buffer as mapped in this process
};

// Signal `epoch` to every rank and wait (bounded) until every rank signalled
// at least `epoch` here. Called by one warp; lane r < world handles rank r.
__device__ __forceinline__ void ep_barrier_warp(const PeerComm& pc, int world, int rank, uint64_t epoch, int* err) {
  const int lane = lane_id();
  __threadfence_system();
  __syncwarp();
  if (lane < world) st_release_sys(reinterpret_cast<uint64_t*>(pc.base[lane]) + rank, epoch);
  if (lane < world) {
    const uint64_t* sig = reinterpret_cast<const uint64_t*>(pc.base[rank]) + lane;
    if (ld_acquire_sys(sig) < epoch) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(sig) < epoch) {
        if (globaltimer_ns() - t0 > AGM_WAIT_LIMIT_NS) {
          raise_error(err, kErrTimeoutFull);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncwarp();
  __threadfence_system();
}

__global__ void ep_counts_exchange_kernel(PeerComm pc, int world, int rank, int E, const int32_t* __restrict__ counts,
                                          uint64_t epoch, int* err) {
  // Write this rank's counts into row `rank` of every peer's inbox, then barrier.
  for (int i = threadIdx.x; i < world * E; i += blockDim.x) {
    const int r = i / E, e = i - r * E;
    int32_t* inbox = reinterpret_cast<int32_t*>(pc.base[r] + ep_off_inbox());
    inbox[rank * E + e] = counts[e];
  }
  __syncthreads();
  if (threadIdx.x < 32) ep_barrier_warp(pc, world, rank, epoch, err);
}

__global__ void ep_barrier_kernel(PeerComm pc, int world, int rank, uint64_t epoch, int* err) {
  ep_barrier_warp(pc, world, rank, epoch, err);
}

// One CTA: the global plan from the counts inbox (identical on every rank),
// this rank's send segments and its receive-side tile table.
//
// The plan is one contiguous piece of every source's tiles (in its x_perm
// order) per destination rank, piece(i, r) = [lo, hi):
//   static / balanced: the global tile sequence is ordered by (expert, source,
//     tile) and rank r computes the range [bounds[r], bounds[r+1]); since a
//     source's tiles appear in that sequence in x_perm order, the tiles it
//     sends to r are contiguous;
//   local (every rank holds every expert): rank r's quota is an equal share of
//     all tiles; each source keeps its first min(own, quota) tiles and sends
//     the rest, in order, to the ranks below quota (lowest rank first).
// A destination lays its pieces out by source rank.
__global__ void ep_plan_kernel(PeerComm pc, int world, int rank, int E, int placement, int first_local_expert,
                               int n_local_experts, int64_t cap_rows, int d, int eb, EpRoute* route,
                               int32_t* __restrict__ recv_tile_expert, int32_t* __restrict__ recv_num_tiles,
                               int* err) {
  __shared__ int64_t tiles[kEpMaxRanks][AGM_MAX_EXPERTS];
  __shared__ int64_t plo[kEpMaxRanks][kEpMaxRanks];  // piece(i, r) = [plo, phi) of source i's tiles
  __shared__ int64_t phi[kEpMaxRanks][kEpMaxRanks];
  const int32_t* inbox = reinterpret_cast<const int32_t*>(pc.base[rank] + ep_off_inbox());
  if (threadIdx.x == 0) {
    int64_t T[kEpMaxRanks];
    int64_t total = 0;
    for (int i = 0; i < world; ++i) {
      T[i] = 0;
      for (int e = 0; e < E; ++e) {
        tiles[i][e] = (static_cast<int64_t>(inbox[i * E + e]) + 127) / 128;
        T[i] += tiles[i][e];
      }
      total += T[i];
      for (int r = 0; r < world; ++r) plo[i][r] = phi[i][r] = 0;
    }
    if (placement == 2) {
      int64_t quota[kEpMaxRanks], keep[kEpMaxRanks], deficit[kEpMaxRanks];
      for (int r = 0; r < world; ++r) {
        quota[r] = total / world + (r < total % world ? 1 : 0);
        keep[r] = min(T[r], quota[r]);
        deficit[r] = quota[r] - keep[r];
        plo[r][r] = 0;
        phi[r][r] = keep[r];
      }
      int r = 0;
      for (int i = 0; i < world; ++i) {
        int64_t pos = keep[i];
        while (pos < T[i]) {
          while (r < world && deficit[r] == 0) ++r;
          if (r >= world) break;  // cannot happen: quotas sum to the total
          const int64_t n = min(T[i] - pos, deficit[r]);
          plo[i][r] = pos;
          phi[i][r] = pos + n;
          pos += n;
          deficit[r] -= n;
        }
      }
    } else {
      // Global sequence (expert, source, tile) and the ranks' ranges in it.
      int64_t g0[kEpMaxRanks][AGM_MAX_EXPERTS];
      int64_t e_start[AGM_MAX_EXPERTS + 1];
      int64_t bounds[kEpMaxRanks + 1];
      int64_t pos = 0;
      for (int e = 0; e < E; ++e) {
        e_start[e] = pos;
        for (int i = 0; i < world; ++i) {
          g0[i][e] = pos;
          pos += tiles[i][e];
        }
      }
      e_start[E] = pos;
      if (placement == 0) {
        const int base = E / world, extra = E % world;
        int e = 0;
        for (int q = 0; q < world; ++q) {
          bounds[q] = e_start[min(e, E)];
          e += base + (q < extra ? 1 : 0);
        }
      } else {
        for (int q = 0; q < world; ++q) bounds[q] = (static_cast<int64_t>(q) * total) / world;
      }
      bounds[world] = total;
      for (int i = 0; i < world; ++i) {
        int64_t start = 0;
        for (int q = 0; q < world; ++q) {
          int64_t n = 0;
          for (int e = 0; e < E; ++e) {
            const int64_t lo = max(g0[i][e], bounds[q]), hi = min(g0[i][e] + tiles[i][e], bounds[q + 1]);
            n += hi > lo ? hi - lo : 0;
          }
          plo[i][q] = start;
          phi[i][q] = start + n;
          start += n;
        }
      }
    }
    // Send segments of this rank.
    route->world = world;
    route->rank = rank;
    int ns = 0;
    const int64_t cap_tiles = cap_rows / 128;
    for (int q = 0; q < world; ++q) {
      route->peer_recv[q] = pc.base[q] + ep_off_recv(E);
      route->peer_y[q] = pc.base[q] + ep_off_y(E, cap_rows, d, eb);
      if (phi[rank][q] <= plo[rank][q]) continue;
      int64_t base = 0;
      for (int i = 0; i < rank; ++i) base += phi[i][q] - plo[i][q];
      route->seg_rank[ns] = q;
      route->seg_lo[ns] = plo[rank][q];
      route->seg_hi[ns] = phi[rank][q];
      route->seg_base[ns] = base;
      route->seg_limit[ns] = max(static_cast<int64_t>(0), cap_tiles - base);  // never write past q's buffer
      ++ns;
    }
    route->n_seg = ns;
    int64_t n_recv = 0;
    for (int i = 0; i < world; ++i) n_recv += phi[i][rank] - plo[i][rank];
    if (n_recv > cap_tiles) raise_error(err, kErrRowOverflow);
    *recv_num_tiles = static_cast<int32_t>(min(n_recv, cap_tiles));
  }
  __syncthreads();
  // Receive-side tile table: source i's tiles [plo, phi) in order; the expert
  // of source i's tile t follows from its per-expert tile counts.
  int64_t off = 0;
  for (int i = 0; i < world; ++i) {
    const int64_t lo = plo[i][rank], n = phi[i][rank] - lo;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
      const int64_t t = lo + j;
      int64_t acc = 0;
      int e = 0;
      while (e < E - 1 && acc + tiles[i][e] <= t) acc += tiles[i][e++];
      int le = e - first_local_expert;
      if (le < 0 || le >= n_local_experts) {
        raise_error(err, kErrBadExpert);
        le = 0;
      }
      const int64_t slot = off + j;
      if (slot * 128 < cap_rows) recv_tile_expert[slot] = le;
    }
    off += n;
  }
}

}  // namespace agm

namespace {

int ep_fail(int code, const std::string& msg) {
  agm::set_last_error(msg);
  return code;
}

int ep_cuda(cudaError_t e, const char* what) {
  return ep_fail(AGM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int eb_of(int dtype) { return dtype == AGM_F32 ? 4 : (dtype == AGM_BF16 || dtype == AGM_F16 ? 2 : 0); }

struct EpLayout {
  int* err;
  int32_t* idx;
  void* gates;
  int32_t* block_hist;
  int32_t* block_off;
  int32_t* counts;
  int32_t* seg_start;
  int32_t* num_tiles_local;
  int32_t* tile_expert_local;
  int32_t* token_of;
  int32_t* row_of;
  agm::EpRoute* route;
  int32_t* recv_tile_expert;
  int32_t* recv_num_tiles;
  void* h;
  size_t bytes;
};

EpLayout ep_carve(void* ws, int64_t n, int d, int E, int k, int H, int64_t cap_rows, int eb) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = (off + 255) & ~size_t(255);
    void* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  };
  const int64_t nb = agm_dispatch_blocks(n);
  const int64_t rows = agm_max_rows(n, k, E);
  EpLayout L;
  L.err = static_cast<int*>(take(sizeof(int)));
  L.idx = static_cast<int32_t*>(take(sizeof(int32_t) * n * k));
  L.gates = take(static_cast<size_t>(eb) * n * k);
  L.block_hist = static_cast<int32_t*>(take(sizeof(int32_t) * nb * E));
  L.block_off = static_cast<int32_t*>(take(sizeof(int32_t) * nb * E));
  L.counts = static_cast<int32_t*>(take(sizeof(int32_t) * E));
  L.seg_start = static_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
  L.num_tiles_local = static_cast<int32_t*>(take(sizeof(int32_t)));
  L.tile_expert_local = static_cast<int32_t*>(take(sizeof(int32_t) * (rows / 128 + 1)));
  L.token_of = static_cast<int32_t*>(take(sizeof(int32_t) * (rows + 1)));
  L.row_of = static_cast<int32_t*>(take(sizeof(int32_t) * n * k));
  L.route = static_cast<agm::EpRoute*>(take(sizeof(agm::EpRoute)));
  L.recv_tile_expert = static_cast<int32_t*>(take(sizeof(int32_t) * (cap_rows / 128 + 1)));
  L.recv_num_tiles = static_cast<int32_t*>(take(sizeof(int32_t)));
  L.h = take(static_cast<size_t>(eb) * cap_rows * H);
  L.bytes = (off + 255) & ~size_t(255);
  return L;
}

int num_sms_dev() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace

extern "C" {

AGM_API size_t agm_ep_comm_bytes(int n_experts, int64_t cap_rows, int d, int dtype) {
  const int eb = eb_of(dtype);
  if (!eb || n_experts < 1 || n_experts > AGM_MAX_EXPERTS || cap_rows <= 0 || d <= 0) return 0;
  return static_cast<size_t>(agm::ep_off_y(n_experts, cap_rows, d, eb) + agm::ep_round(cap_rows * d * eb, 4096));
}

AGM_API int agm_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr || !bytes) return ep_fail(AGM_ERR_ARG, "agm_ep_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return ep_cuda(e, "agm_ep_alloc: cudaMalloc");
  e = cudaMemset(*ptr, 0, std::min<size_t>(bytes, agm::ep_off_recv(AGM_MAX_EXPERTS)));
  if (e != cudaSuccess) return ep_cuda(e, "agm_ep_alloc: cudaMemset");
  return AGM_OK;
}

AGM_API int agm_ep_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? AGM_OK : ep_cuda(e, "agm_ep_free");
}

AGM_API int agm_ep_ipc_handle(void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return ep_fail(AGM_ERR_ARG, "agm_ep_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return ep_cuda(e, "agm_ep_ipc_handle");
  memcpy(handle_out, &h, sizeof(h));
  return AGM_OK;
}

AGM_API int agm_ep_ipc_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return ep_fail(AGM_ERR_ARG, "agm_ep_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? AGM_OK : ep_cuda(e, "agm_ep_ipc_open");
}

AGM_API int agm_ep_ipc_close(void* peer_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? AGM_OK : ep_cuda(e, "agm_ep_ipc_close");
}

AGM_API size_t agm_ep_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int64_t cap_rows,
                                      int dtype) {
  const int eb = eb_of(dtype);
  if (!eb || n_tokens < 0 || cap_rows <= 0) return 0;
  return ep_carve(nullptr, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb).bytes;
}

// Phase 1 (comm stream): route and permute this rank's tokens into the
// receive buffers of the ranks that compute them; ends with the barrier after
// which every rank's received rows are complete.
AGM_API int agm_ep_dispatch(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                            const void* w_router, int n_local_experts, int first_local_expert, int placement,
                            int world, int rank, const uint64_t* peer_comm, int64_t cap_rows, uint64_t epoch,
                            void* workspace, size_t workspace_bytes, int flags, void* const* stage_events,
                            void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: bad dtype");
  if (world < 1 || world > agm::kEpMaxRanks || rank < 0 || rank >= world)
    return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_dispatch: world must be in [1, 16] and rank in [0, world)");
  if (n_experts < 1 || n_experts > AGM_MAX_EXPERTS || top_k < 1 || top_k > n_experts)
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: bad n_experts / top_k");
  if (placement < 0 || placement > 2) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: placement must be 0, 1 or 2");
  if (cap_rows <= 0 || cap_rows % 128)
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: cap_rows must be a multiple of 128");
  if (!peer_comm || !w_router || !workspace || (n_tokens > 0 && !x))
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: null pointer");
  if (epoch == 0) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: epoch must start at 1");
  if (n_tokens < 0) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: n_tokens < 0");
  EpLayout L = ep_carve(workspace, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb);
  if (L.bytes > workspace_bytes) return ep_fail(AGM_ERR_WORKSPACE, "agm_ep_dispatch: workspace too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PeerComm pc;
  for (int r = 0; r < agm::kEpMaxRanks; ++r) pc.base[r] = r < world ? peer_comm[r] : 0;
  const int sms = num_sms_dev();
  const int64_t rows = agm_max_rows(n_tokens, top_k, n_experts);
  auto mark = [&](int i) -> cudaError_t {
    return stage_events ? cudaEventRecord(static_cast<cudaEvent_t>(stage_events[i]), stream) : cudaSuccess;
  };
  cudaError_t e = cudaMemsetAsync(L.err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return ep_cuda(e, "memset");
  if ((e = mark(0)) != cudaSuccess) return ep_cuda(e, "event");
  e = cudaMemsetAsync(L.counts, 0, sizeof(int32_t) * n_experts, stream);
  if (e != cudaSuccess) return ep_cuda(e, "memset");
  if (n_tokens > 0) {
    e = agm::router_topk(dtype, x, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST, nullptr,
                         nullptr, L.idx, L.gates, L.block_hist, L.err, sms, stream);
    if (e != cudaSuccess) return ep_cuda(e, "router_topk");
    e = agm::dispatch_plan(L.block_hist, static_cast<int>(agm_dispatch_blocks(n_tokens)), n_experts, rows,
                           static_cast<int>(rows / 128), AGM_TILE_M, L.block_off, L.counts, L.seg_start,
                           L.tile_expert_local,
                           L.num_tiles_local, L.token_of, L.err, stream);
    if (e != cudaSuccess) return ep_cuda(e, "dispatch_plan");
  }
  if ((e = mark(1)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_counts_exchange_kernel<<<1, 256, 0, stream>>>(pc, world, rank, n_experts, L.counts, epoch, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "counts exchange");
  agm::ep_plan_kernel<<<1, 512, 0, stream>>>(pc, world, rank, n_experts, placement, first_local_expert,
                                             n_local_experts, cap_rows, d, eb, L.route, L.recv_tile_expert,
                                             L.recv_num_tiles, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "ep plan");
  if ((e = mark(2)) != cudaSuccess) return ep_cuda(e, "event");
  if (n_tokens > 0) {
    e = agm::permute_rows_ep(x, eb, n_tokens, d, top_k, n_experts, L.idx, L.block_off, L.seg_start, L.counts, rows,
                             L.route, L.row_of, L.err, stream);
    if (e != cudaSuccess) return ep_cuda(e, "dispatch");
  }
  if ((e = mark(3)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_barrier_kernel<<<1, 32, 0, stream>>>(pc, world, rank, epoch + 1, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "barrier");
  if ((e = mark(4)) != cudaSuccess) return ep_cuda(e, "event");
  return AGM_OK;
}

// Phase 2 (compute stream): FC1/FC2 over the received tiles into this rank's
// result buffer, then the barrier after which every rank's results are
// complete. gemm_ctas > 0 caps the GEMM's persistent CTAs (leaving SMs to
// the other phases of another chunk running concurrently).
AGM_API int agm_ep_expert(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden, const void* w1,
                          const void* b1, const void* w2, const void* b2, int n_local_experts, int world, int rank,
                          const uint64_t* peer_comm, int64_t cap_rows, uint64_t epoch, void* workspace,
                          size_t workspace_bytes, int gemm_ctas, void* const* stage_events, void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_ARG, "agm_ep_expert: bad dtype");
  if (world < 1 || world > agm::kEpMaxRanks || rank < 0 || rank >= world)
    return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_expert: bad world / rank");
  if (!peer_comm || !w1 || !b1 || !w2 || !b2 || !workspace) return ep_fail(AGM_ERR_ARG, "agm_ep_expert: null pointer");
  if (cap_rows <= 0 || cap_rows % 128) return ep_fail(AGM_ERR_ARG, "agm_ep_expert: bad cap_rows");
  EpLayout L = ep_carve(workspace, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb);
  if (L.bytes > workspace_bytes) return ep_fail(AGM_ERR_WORKSPACE, "agm_ep_expert: workspace too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PeerComm pc;
  for (int r = 0; r < agm::kEpMaxRanks; ++r) pc.base[r] = r < world ? peer_comm[r] : 0;
  const int sms = num_sms_dev();
  auto mark = [&](int i) -> cudaError_t {
    return stage_events ? cudaEventRecord(static_cast<cudaEvent_t>(stage_events[i]), stream) : cudaSuccess;
  };
  cudaError_t e;
  void* recv = reinterpret_cast<void*>(peer_comm[rank] + agm::ep_off_recv(n_experts));
  void* y = reinterpret_cast<void*>(peer_comm[rank] + agm::ep_off_y(n_experts, cap_rows, d, eb));
  agm::GemmArgs g1;
  g1.c = L.h;
  g1.ldc = hidden;
  g1.c_rows = cap_rows;
  g1.bias = b1;
  g1.n = hidden;
  g1.k = d;
  g1.groups = n_local_experts;
  g1.tile_group = L.recv_tile_expert;
  g1.num_tiles = L.recv_num_tiles;
  g1.max_tiles = static_cast<int>(cap_rows / 128);
  g1.err = L.err;
  g1.max_ctas = gemm_ctas;
  e = agm::grouped_gemm(dtype, recv, cap_rows, w1, g1, true, sms, stream, 0);
  if (e != cudaSuccess) return ep_cuda(e, "grouped_gemm fc1");
  if ((e = mark(0)) != cudaSuccess) return ep_cuda(e, "event");
  agm::GemmArgs g2 = g1;
  g2.c = y;
  g2.ldc = d;
  g2.bias = b2;
  g2.n = d;
  g2.k = hidden;
  e = agm::grouped_gemm(dtype, L.h, cap_rows, w2, g2, false, sms, stream, 0);
  if (e != cudaSuccess) return ep_cuda(e, "grouped_gemm fc2");
  if ((e = mark(1)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_barrier_kernel<<<1, 32, 0, stream>>>(pc, world, rank, epoch + 2, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "barrier");
  if ((e = mark(2)) != cudaSuccess) return ep_cuda(e, "event");
  return AGM_OK;
}

// Phase 3 (comm stream): each token's k expert rows, read from the ranks that
// computed them, gate-weighted into out [n, d].
AGM_API int agm_ep_combine(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           int64_t cap_rows, void* out, void* workspace, size_t workspace_bytes, void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_ARG, "agm_ep_combine: bad dtype");
  if (!workspace || (n_tokens > 0 && !out)) return ep_fail(AGM_ERR_ARG, "agm_ep_combine: null pointer");
  EpLayout L = ep_carve(workspace, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb);
  if (L.bytes > workspace_bytes) return ep_fail(AGM_ERR_WORKSPACE, "agm_ep_combine: workspace too small");
  if (n_tokens <= 0) return AGM_OK;
  cudaError_t e = agm::combine_ep(dtype, L.route, L.row_of, L.gates, n_tokens, d, top_k, out, num_sms_dev(),
                                  static_cast<cudaStream_t>(stream_));
  return e == cudaSuccess ? AGM_OK : ep_cuda(e, "combine");
}

AGM_API int agm_ep_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                           int n_local_experts, int first_local_expert, int placement, int world, int rank,
                           const uint64_t* peer_comm, int64_t cap_rows, uint64_t epoch, void* out, void* workspace,
                           size_t workspace_bytes, int flags, void* const* stage_events, void* stream) {
  if (!w1 || !b1 || !w2 || !b2 || (n_tokens > 0 && !out))
    return ep_fail(AGM_ERR_ARG, "agm_ep_forward: null pointer argument");
  int rc = agm_ep_dispatch(x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, n_local_experts,
                           first_local_expert, placement, world, rank, peer_comm, cap_rows, epoch, workspace,
                           workspace_bytes, flags, stage_events, stream);
  if (rc != AGM_OK) return rc;
  rc = agm_ep_expert(dtype, n_tokens, d, n_experts, top_k, hidden, w1, b1, w2, b2, n_local_experts, world, rank,
                     peer_comm, cap_rows, epoch, workspace, workspace_bytes, 0,
                     stage_events ? stage_events + 5 : nullptr, stream);
  if (rc != AGM_OK) return rc;
  rc = agm_ep_combine(dtype, n_tokens, d, n_experts, top_k, hidden, cap_rows, out, workspace, workspace_bytes, stream);
  if (rc != AGM_OK) return rc;
  if (stage_events) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(stage_events[8]), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ep_cuda(e, "event");
  }
  return AGM_OK;
}

}  // extern "C"
