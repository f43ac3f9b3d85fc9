// Expert-parallel MoE block forward over NVLink peer memory (one process per
// GPU), with the all-to-all fused into the kernels around the expert GEMM.
//
// The reference runs the block on one device (agillm41.py:4389-4431). Here P
// ranks each route their own tokens and share the expert FFN work; instead of
// two collective all-to-all passes, the data moves inside the kernels:
//
//   router -> local dispatch plan -> [counts to every peer + flag barrier]
//   -> device plan (every rank computes the same one from the counts)
//   -> permute: every (token, rank) row is written straight into the
//      receive buffer of the rank that computes it (NVLink stores)
//   -> [signal to every rank] -> grouped FC1/FC2 (CTA pairs) on the received
//      tiles, own rows first; FC1 waits for a source's signal only before its
//      first tile from that source, so it starts while peers' rows arrive;
//      FC2's epilogue writes each output row straight into the home buffer
//      of the rank that owns the token, at the row's x_perm position
//      (NVLink stores, overlapped with the GEMM) -> [flag barrier]
//   -> combine: each token's k expert rows, read from this rank's own home
//      buffer (the single-GPU combine kernel).
//
// No host synchronisation and no library collective: the counts exchange, the
// delivery signals and the barrier after FC2 are flag writes/reads in peer
// memory with bounded waits.
//
// Every rank owns one "comm" buffer allocated with cudaMalloc (IPC-shareable),
// laid out identically on all ranks:
//   [0, 256)            signals: uint64 per source rank, monotonically raised
//                       epochs (rank r writes signal[r] on every peer)
//   [256, ...)          counts inbox: int32 [kEpMaxRanks][E] (row i from rank i)
//   off_recv            receive buffer [cap_rows, d] (rows this rank computes)
//   off_home            home buffer [home_rows, d] (FFN outputs of this rank's
//                       own permuted rows, written by whoever computed them)
// Peers' comm buffers are mapped into this process with CUDA IPC.
//
// Work is planned in 256-row units (see ep_plan_kernel). Placements:
//   AGM_EP_HOLDERS  - each expert's weights live on the ranks of a bitmask:
//                     the static contiguous ownership (7/7, 4/4/3/3, ...),
//                     optionally with replicas of the hottest experts; an
//                     expert held by several ranks is split among them;
//   AGM_EP_BALANCED - every rank holds every expert; P near-equal ranges of
//                     the global (expert, source, unit) sequence;
//   AGM_EP_LOCAL    - every rank holds every expert; each rank computes its
//                     own units up to an equal share, only the excess moves.
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
// This rank's home buffer: the FFN outputs of its own permuted rows, written
// by the ranks that computed them, at the rows' x_perm positions.
__host__ __device__ inline int64_t ep_off_home(int E, int64_t cap_rows, int d, int eb) {
  return ep_off_recv(E) + ep_round(cap_rows * d * eb, 4096);
}

constexpr int kEpUnitRows = AGM_PAIR_ROWS;              // work unit: two 128-row GEMM tiles
constexpr int kEpUnitTiles = AGM_PAIR_ROWS / 128;
constexpr int kEpBalanced = AGM_EP_BALANCED, kEpLocal = AGM_EP_LOCAL;

struct EpPlacement {
  int code;                           // AGM_EP_HOLDERS / AGM_EP_BALANCED / AGM_EP_LOCAL
  uint32_t holders[AGM_MAX_EXPERTS];  // bit r: rank r holds expert e's weights
};


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

// The release half of a barrier: after the permute has written this rank's
// rows into the computing ranks' receive buffers, tell every rank so
// (signal[rank] = epoch on each). The waits happen where the rows are
// consumed: the expert GEMM's producer waits, per source, before loading the
// first tile that source sent (GemmArgs::tile_src).
__global__ void ep_signal_kernel(PeerComm pc, int world, int rank, uint64_t epoch) {
  const int lane = lane_id();
  __threadfence_system();
  __syncwarp();
  if (lane < world) st_release_sys(reinterpret_cast<uint64_t*>(pc.base[lane]) + rank, epoch);
}

// One CTA: the global plan from the counts inbox (identical on every rank),
// this rank's send segments and its receive-side tile tables.
//
// Work is counted in units of 256 rows: every (source, expert) segment of a
// source's x_perm is padded to 256 rows (two GEMM row tiles), so every piece
// of work is whole row-tile pairs of one expert and the CTA-pair GEMM can
// compute it. The plan cuts each source's expert segments into pieces, one
// per computing rank, cut[i][e][r] = [lo, hi) in source i's x_perm units:
//   holders (static ownership, optionally with replicas of hot experts):
//     every expert's units, taken source by source in order, are split into
//     consecutive chunks, one per rank holding the expert (ranks ascending).
//     An expert held by one rank goes to it whole; the experts held by
//     several ranks are then spread, largest first, by water-filling: each
//     raises its holders' loads toward a common level, lowest-loaded holder
//     (then lowest rank) first;
//   balanced (every rank holds every expert): the global sequence (expert,
//     source, unit) is cut into P near-equal ranges;
//   local (every rank holds every expert): rank r's quota is an equal share
//     of all units; each source keeps its first min(own, quota) units and
//     sends the rest, in order, to the ranks below quota (lowest rank first).
// A destination lays its pieces out by (source, expert), its own source
// first. For every received tile the tables give the local weight index of
// its expert, the source rank, and the address, in the source rank's home
// buffer, where the tile's FFN output goes.
__global__ void __launch_bounds__(256) ep_plan_kernel(PeerComm pc, int world, int rank, int E, EpPlacement pl,
                                                      int64_t cap_rows, int64_t home_rows, int d, int eb,
                                                      EpRoute* route, int32_t* __restrict__ recv_tile_expert,
                                                      int32_t* __restrict__ recv_tile_src,
                                                      uint64_t* __restrict__ recv_tile_dst,
                                                      int32_t* __restrict__ recv_num_tiles, int* err) {
  __shared__ int units[kEpMaxRanks][AGM_MAX_EXPERTS];
  __shared__ int xoff[kEpMaxRanks][AGM_MAX_EXPERTS];   // unit offset of expert e's segment in source i
  __shared__ int gofs[kEpMaxRanks][AGM_MAX_EXPERTS];   // offset of source i's units in expert e's sequence
  __shared__ int chunk0[AGM_MAX_EXPERTS][kEpMaxRanks];  // rank r's chunk of expert e's sequence
  __shared__ int chunk1[AGM_MAX_EXPERTS][kEpMaxRanks];
  __shared__ int plo[kEpMaxRanks][kEpMaxRanks];         // local placement: piece (i, r) of source i's units
  __shared__ int phi[kEpMaxRanks][kEpMaxRanks];
  __shared__ int cut_lo[kEpMaxRanks][AGM_MAX_EXPERTS][kEpMaxRanks];
  __shared__ int cut_hi[kEpMaxRanks][AGM_MAX_EXPERTS][kEpMaxRanks];
  __shared__ int base_send[AGM_MAX_EXPERTS][kEpMaxRanks];  // destination unit offset of piece (rank, e, r)
  __shared__ int base_recv[kEpMaxRanks][AGM_MAX_EXPERTS];  // destination unit offset of piece (i, e, rank)
  __shared__ int total_recv;
  const int32_t* inbox = reinterpret_cast<const int32_t*>(pc.base[rank] + ep_off_inbox());
  const int tid = threadIdx.x;
  const int pairs = world * E;
  for (int t = tid; t < pairs; t += blockDim.x) {
    const int i = t / E, e = t - i * E;
    const int c = inbox[i * E + e];
    units[i][e] = c > 0 ? (c + kEpUnitRows - 1) / kEpUnitRows : 0;
  }
  __syncthreads();
  if (tid == 0) {
    int T[kEpMaxRanks];
    int U[AGM_MAX_EXPERTS];
    int total = 0;
    for (int e = 0; e < E; ++e) U[e] = 0;
    for (int i = 0; i < world; ++i) {
      T[i] = 0;
      for (int e = 0; e < E; ++e) {
        xoff[i][e] = T[i];
        gofs[i][e] = U[e];
        T[i] += units[i][e];
        U[e] += units[i][e];
      }
      total += T[i];
      for (int r = 0; r < world; ++r) plo[i][r] = phi[i][r] = 0;
    }
    for (int e = 0; e < E; ++e)
      for (int r = 0; r < world; ++r) chunk0[e][r] = chunk1[e][r] = 0;
    if (pl.code == kEpLocal) {
      int quota[kEpMaxRanks], keep[kEpMaxRanks], deficit[kEpMaxRanks];
      for (int r = 0; r < world; ++r) {
        quota[r] = total / world + (r < total % world ? 1 : 0);
        keep[r] = min(T[r], quota[r]);
        deficit[r] = quota[r] - keep[r];
        plo[r][r] = 0;
        phi[r][r] = keep[r];
      }
      int r = 0;
      for (int i = 0; i < world; ++i) {
        int pos = keep[i];
        while (pos < T[i]) {
          while (r < world && deficit[r] == 0) ++r;
          if (r >= world) break;  // cannot happen: quotas sum to the total
          const int n = min(T[i] - pos, deficit[r]);
          plo[i][r] = pos;
          phi[i][r] = pos + n;
          pos += n;
          deficit[r] -= n;
        }
      }
    } else if (pl.code == kEpBalanced) {
      int e_start = 0;
      for (int e = 0; e < E; ++e) {
        for (int r = 0; r < world; ++r) {
          const int lo = static_cast<int>((static_cast<int64_t>(r) * total) / world);
          const int hi = static_cast<int>((static_cast<int64_t>(r + 1) * total) / world);
          const int a = max(lo, e_start), b = min(hi, e_start + U[e]);
          chunk0[e][r] = b > a ? a - e_start : 0;
          chunk1[e][r] = b > a ? b - e_start : 0;
        }
        e_start += U[e];
      }
    } else {
      // Holders: single-holder experts first, then water-filling of the
      // replicated ones, largest first (ties: lower expert index first).
      int load[kEpMaxRanks];
      int alloc[AGM_MAX_EXPERTS][kEpMaxRanks];
      const uint32_t wmask = (1u << world) - 1u;
      for (int r = 0; r < world; ++r) load[r] = 0;
      int order[AGM_MAX_EXPERTS];
      int n_rep = 0;
      for (int e = 0; e < E; ++e) {
        for (int r = 0; r < world; ++r) alloc[e][r] = 0;
        const uint32_t h = pl.holders[e] & wmask;
        if (h == 0) {
          raise_error(err, kErrBadExpert);
          continue;
        }
        if ((h & (h - 1)) == 0) {
          const int owner = __ffs(h) - 1;
          alloc[e][owner] = U[e];
          load[owner] += U[e];
        } else {
          int j = n_rep++;
          while (j > 0 && U[order[j - 1]] < U[e]) {  // stable: equal sizes keep index order
            order[j] = order[j - 1];
            --j;
          }
          order[j] = e;
        }
      }
      for (int q = 0; q < n_rep; ++q) {
        const int e = order[q];
        const uint32_t h = pl.holders[e] & wmask;
        int hs[kEpMaxRanks];
        int m = 0;
        for (int r = 0; r < world; ++r) {
          if (!((h >> r) & 1u)) continue;
          int j = m++;
          while (j > 0 && load[hs[j - 1]] > load[r]) {  // by load, then rank
            hs[j] = hs[j - 1];
            --j;
          }
          hs[j] = r;
        }
        int remaining = U[e], cnt = 1, level = load[hs[0]];
        while (cnt < m && remaining >= (load[hs[cnt]] - level) * cnt) {
          remaining -= (load[hs[cnt]] - level) * cnt;
          level = load[hs[cnt]];
          ++cnt;
        }
        const int qn = remaining / cnt, rem = remaining - qn * cnt;
        for (int t = 0; t < cnt; ++t) {
          const int target = level + qn + (t < rem ? 1 : 0);
          alloc[e][hs[t]] = target - load[hs[t]];
          load[hs[t]] = target;
        }
      }
      for (int e = 0; e < E; ++e) {
        int c = 0;
        for (int r = 0; r < world; ++r) {
          chunk0[e][r] = c;
          c += alloc[e][r];
          chunk1[e][r] = c;
        }
      }
    }
  }
  __syncthreads();
  // Pieces: one thread per (source, expert).
  for (int t = tid; t < pairs; t += blockDim.x) {
    const int i = t / E, e = t - i * E;
    const int u = units[i][e], x0 = xoff[i][e], g0 = gofs[i][e];
    for (int r = 0; r < world; ++r) {
      int a, b;
      if (pl.code == kEpLocal) {
        a = max(plo[i][r], x0);
        b = min(phi[i][r], x0 + u);
      } else {
        a = x0 + max(chunk0[e][r], g0) - g0;
        b = x0 + min(chunk1[e][r], g0 + u) - g0;
      }
      cut_lo[i][e][r] = a;
      cut_hi[i][e][r] = b > a ? b : a;
    }
  }
  __syncthreads();
  // Destination offsets: one thread per destination rank.
  // A destination lays its pieces out source by source starting with its
  // own rows (sources r, r+1, ... mod P), so its GEMM can begin on rows that
  // never crossed NVLink while the peers' rows are still arriving.
  if (tid < world) {
    const int r = tid;
    int acc = 0;
    for (int j = 0; j < world; ++j) {
      const int i = (r + j) % world;
      for (int e = 0; e < E; ++e) {
        if (i == rank) base_send[e][r] = acc;
        if (r == rank) base_recv[i][e] = acc;
        acc += cut_hi[i][e][r] - cut_lo[i][e][r];
      }
    }
    if (r == rank) total_recv = acc;
  }
  __syncthreads();
  const int64_t cap_tiles = cap_rows / 128;
  if (tid == 0) {
    route->world = world;
    route->rank = rank;
    int ns = 0;
    for (int q = 0; q < world; ++q) route->peer_recv[q] = pc.base[q] + ep_off_recv(E);
    for (int e = 0; e < E; ++e)
      for (int q = 0; q < world; ++q) {
        const int lo = cut_lo[rank][e][q], hi = cut_hi[rank][e][q];
        if (hi <= lo) continue;
        if (ns == kEpMaxSegs) {
          raise_error(err, kErrRowOverflow);
          continue;
        }
        const int64_t base = static_cast<int64_t>(base_send[e][q]) * kEpUnitTiles;
        route->seg_rank[ns] = q;
        route->seg_lo[ns] = static_cast<int64_t>(lo) * kEpUnitTiles;
        route->seg_hi[ns] = static_cast<int64_t>(hi) * kEpUnitTiles;
        route->seg_base[ns] = base;
        route->seg_limit[ns] = max(static_cast<int64_t>(0), cap_tiles - base);  // never write past q's buffer
        ++ns;
      }
    route->n_seg = ns;
    const int64_t n_recv = static_cast<int64_t>(total_recv) * kEpUnitTiles;
    if (n_recv > cap_tiles) raise_error(err, kErrRowOverflow);
    *recv_num_tiles = static_cast<int32_t>(min(n_recv, cap_tiles));
  }
  // Receive-side tables, one (source, expert) piece after another.
  const int64_t row_bytes = static_cast<int64_t>(d) * eb;
  const int64_t home_tiles = home_rows / 128;
  for (int p = 0; p < pairs; ++p) {
    const int i = p / E, e = p - i * E;
    const int lo = cut_lo[i][e][rank], n = (cut_hi[i][e][rank] - lo) * kEpUnitTiles;
    if (n <= 0) continue;
    const bool held = (pl.holders[e] >> rank) & 1u;
    int le = 0;
    for (int e2 = 0; e2 < e; ++e2) le += (pl.holders[e2] >> rank) & 1u;
    if (!held) {
      if (tid == 0) raise_error(err, kErrBadExpert);
      le = 0;
    }
    const int64_t slot0 = static_cast<int64_t>(base_recv[i][e]) * kEpUnitTiles;
    const uint64_t home = pc.base[i] + ep_off_home(E, cap_rows, d, eb);
    for (int j = tid; j < n; j += blockDim.x) {
      const int64_t slot = slot0 + j;
      const int64_t src_tile = static_cast<int64_t>(lo) * kEpUnitTiles + j;
      if (slot >= cap_tiles) continue;
      if (src_tile >= home_tiles) {
        raise_error(err, kErrRowOverflow);
        continue;
      }
      recv_tile_expert[slot] = le;
      recv_tile_src[slot] = i;
      recv_tile_dst[slot] = home + static_cast<uint64_t>(src_tile * 128 * row_bytes);
    }
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

// The expert-parallel path runs the CTA-pair GEMM: 16-bit activations only.
int eb_of(int dtype) { return (dtype == AGM_BF16 || dtype == AGM_F16) ? 2 : 0; }

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
  int32_t* recv_tile_src;
  uint64_t* recv_tile_dst;
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
  const int64_t rows = agm_ep_max_rows(n, k, E);
  const int64_t cap_tiles = cap_rows / 128;
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
  L.recv_tile_expert = static_cast<int32_t*>(take(sizeof(int32_t) * (cap_tiles + 1)));
  L.recv_tile_src = static_cast<int32_t*>(take(sizeof(int32_t) * (cap_tiles + 1)));
  L.recv_tile_dst = static_cast<uint64_t*>(take(sizeof(uint64_t) * (cap_tiles + 1)));
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

int check_rows(int64_t cap_rows, int64_t home_rows, const char* who) {
  if (cap_rows <= 0 || cap_rows % AGM_PAIR_ROWS || home_rows <= 0 || home_rows % AGM_PAIR_ROWS)
    return ep_fail(AGM_ERR_ARG, std::string(who) + ": cap_rows and home_rows must be positive multiples of 256");
  return AGM_OK;
}

}  // namespace

extern "C" {

AGM_API int64_t agm_ep_max_rows(int64_t n_tokens, int top_k, int n_experts) {
  if (n_tokens <= 0) return 0;
  const int64_t kn = static_cast<int64_t>(top_k) * n_tokens;
  const int64_t a = AGM_PAIR_ROWS;
  return (kn + static_cast<int64_t>(n_experts) * (a - 1) + a - 1) / a * a;
}

AGM_API size_t agm_ep_comm_bytes(int n_experts, int64_t cap_rows, int64_t home_rows, int d, int dtype) {
  const int eb = eb_of(dtype);
  if (!eb || n_experts < 1 || n_experts > AGM_MAX_EXPERTS || cap_rows <= 0 || home_rows <= 0 || d <= 0) return 0;
  return static_cast<size_t>(agm::ep_off_home(n_experts, cap_rows, d, eb) + agm::ep_round(home_rows * d * eb, 4096));
}

AGM_API int64_t agm_ep_home_offset(int n_experts, int64_t cap_rows, int d, int dtype) {
  const int eb = eb_of(dtype);
  if (!eb || n_experts < 1 || n_experts > AGM_MAX_EXPERTS || cap_rows <= 0 || d <= 0) return -1;
  return agm::ep_off_home(n_experts, cap_rows, d, eb);
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
// receive buffers of the ranks that compute them; ends by signalling every
// rank that this rank's rows are delivered.
AGM_API int agm_ep_dispatch(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                            const void* w_router, int placement, const uint32_t* expert_holders, int world, int rank,
                            const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch,
                            void* workspace, size_t workspace_bytes, int flags, void* const* stage_events,
                            void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_dispatch: dtype must be AGM_BF16 or AGM_F16");
  if (world < 1 || world > agm::kEpMaxRanks || rank < 0 || rank >= world)
    return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_dispatch: world must be in [1, 16] and rank in [0, world)");
  if (n_experts < 1 || n_experts > AGM_MAX_EXPERTS || top_k < 1 || top_k > n_experts)
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: bad n_experts / top_k");
  if (placement != AGM_EP_HOLDERS && placement != AGM_EP_BALANCED && placement != AGM_EP_LOCAL)
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: placement must be AGM_EP_HOLDERS, AGM_EP_BALANCED or AGM_EP_LOCAL");
  int rc = check_rows(cap_rows, home_rows, "agm_ep_dispatch");
  if (rc) return rc;
  if (!peer_comm || !w_router || !workspace || !expert_holders || (n_tokens > 0 && !x))
    return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: null pointer");
  if (epoch == 0) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: epoch must start at 1");
  if (n_tokens < 0) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: n_tokens < 0");
  const int64_t rows = agm_ep_max_rows(n_tokens, top_k, n_experts);
  if (rows > home_rows) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: more permuted rows than home_rows holds");
  agm::EpPlacement pl{};
  pl.code = placement;
  const uint32_t wmask = (1u << world) - 1u;
  for (int e = 0; e < n_experts; ++e) {
    pl.holders[e] = expert_holders[e] & wmask;
    if (!pl.holders[e]) return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: an expert has no holder");
    if (placement != AGM_EP_HOLDERS && pl.holders[e] != wmask)
      return ep_fail(AGM_ERR_ARG, "agm_ep_dispatch: balanced and local placements need every expert on every rank");
  }
  EpLayout L = ep_carve(workspace, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb);
  if (L.bytes > workspace_bytes) return ep_fail(AGM_ERR_WORKSPACE, "agm_ep_dispatch: workspace too small");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  agm::PeerComm pc;
  for (int r = 0; r < agm::kEpMaxRanks; ++r) pc.base[r] = r < world ? peer_comm[r] : 0;
  const int sms = num_sms_dev();
  auto mark = [&](int i) -> cudaError_t {
    return stage_events ? cudaEventRecord(static_cast<cudaEvent_t>(stage_events[i]), stream) : cudaSuccess;
  };
  cudaError_t e = cudaMemsetAsync(L.err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return ep_cuda(e, "memset");
  if ((e = mark(0)) != cudaSuccess) return ep_cuda(e, "event");
  e = cudaMemsetAsync(L.counts, 0, sizeof(int32_t) * n_experts, stream);
  if (e != cudaSuccess) return ep_cuda(e, "memset");
  // Router, plan and permute may each start while the previous kernel
  // finishes (each waits before reading its inputs); the flag kernels are
  // plain launches, ordered after everything before them.
  agm::PdlScope pdl(!(flags & AGM_FLAG_NO_PDL));
  if (n_tokens > 0) {
    e = agm::router_topk(dtype, x, w_router, n_tokens, d, n_experts, top_k, flags & AGM_FLAG_TIE_LOW_FIRST, nullptr,
                         nullptr, L.idx, L.gates, L.block_hist, L.err, sms, stream);
    if (e != cudaSuccess) return ep_cuda(e, "router_topk");
    e = agm::dispatch_plan(L.block_hist, static_cast<int>(agm_dispatch_blocks(n_tokens)), n_experts, rows,
                           static_cast<int>(rows / 128), AGM_PAIR_ROWS, L.block_off, L.counts, L.seg_start,
                           L.tile_expert_local, L.num_tiles_local, L.token_of, L.err, stream);
    if (e != cudaSuccess) return ep_cuda(e, "dispatch_plan");
  }
  if ((e = mark(1)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_counts_exchange_kernel<<<1, 256, 0, stream>>>(pc, world, rank, n_experts, L.counts, epoch, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "counts exchange");
  agm::ep_plan_kernel<<<1, 256, 0, stream>>>(pc, world, rank, n_experts, pl, cap_rows, home_rows, d, eb, L.route,
                                             L.recv_tile_expert, L.recv_tile_src, L.recv_tile_dst,
                                             L.recv_num_tiles, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "ep plan");
  if ((e = mark(2)) != cudaSuccess) return ep_cuda(e, "event");
  if (n_tokens > 0) {
    e = agm::permute_rows_ep(x, eb, n_tokens, d, top_k, n_experts, L.idx, L.block_off, L.seg_start, L.counts, rows,
                             L.route, L.row_of, L.err, stream);
    if (e != cudaSuccess) return ep_cuda(e, "dispatch");
  }
  if ((e = mark(3)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_signal_kernel<<<1, 32, 0, stream>>>(pc, world, rank, epoch + 1);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "signal");
  if ((e = mark(4)) != cudaSuccess) return ep_cuda(e, "event");
  return AGM_OK;
}

// Phase 2 (compute stream): FC1 over the received tiles into h (its producer
// waits, per source, for that source's signal before loading its first
// tile; own rows come first), FC2 from h
// straight into the home buffers of the ranks whose tokens they are (NVLink
// stores for peers), then the barrier after which every rank's results are
// complete. gemm_ctas > 0 caps the GEMM's persistent CTAs (leaving SMs to
// the other phases of another chunk running concurrently).
AGM_API int agm_ep_expert(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden, const void* w1,
                          const void* b1, const void* w2, const void* b2, int n_local_experts, int world, int rank,
                          const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch,
                          void* workspace, size_t workspace_bytes, int gemm_ctas, void* const* stage_events,
                          void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_expert: dtype must be AGM_BF16 or AGM_F16");
  if (world < 1 || world > agm::kEpMaxRanks || rank < 0 || rank >= world)
    return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_expert: bad world / rank");
  if (!peer_comm || !w1 || !b1 || !w2 || !b2 || !workspace) return ep_fail(AGM_ERR_ARG, "agm_ep_expert: null pointer");
  if (n_local_experts < 1 || n_local_experts > n_experts)
    return ep_fail(AGM_ERR_ARG, "agm_ep_expert: n_local_experts must be in [1, n_experts]");
  int rc = check_rows(cap_rows, home_rows, "agm_ep_expert");
  if (rc) return rc;
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
  // Rows of source i are complete once i signalled epoch + 1 here.
  g1.tile_src = L.recv_tile_src;
  g1.src_signal = reinterpret_cast<const uint64_t*>(peer_comm[rank]);
  g1.src_epoch = epoch + 1;
  // The tables come from the plan, three launches back, and the weights from
  // before the forward: FC1 streams its first weight tiles while the kernel
  // before it finishes, and FC2 while FC1 finishes.
  g1.early_weights = true;
  agm::PdlScope pdl(true);
  e = agm::grouped_gemm(dtype, recv, cap_rows, w1, g1, true, sms, stream, AGM_GEMM_PAIR);
  if (e != cudaSuccess) return ep_cuda(e, "grouped_gemm fc1");
  if ((e = mark(0)) != cudaSuccess) return ep_cuda(e, "event");
  agm::GemmArgs g2 = g1;
  g2.c = L.h;             // not stored to: every tile's rows go to tile_dst
  g2.ldc = d;
  g2.bias = b2;
  g2.n = d;
  g2.k = hidden;
  g2.tile_dst = L.recv_tile_dst;
  g2.tile_src = nullptr;  // h is this rank's own
  g2.early_weights = true;
  e = agm::grouped_gemm(dtype, L.h, cap_rows, w2, g2, false, sms, stream, AGM_GEMM_PAIR);
  if (e != cudaSuccess) return ep_cuda(e, "grouped_gemm fc2");
  if ((e = mark(1)) != cudaSuccess) return ep_cuda(e, "event");
  agm::ep_barrier_kernel<<<1, 32, 0, stream>>>(pc, world, rank, epoch + 2, L.err);
  if ((e = cudaGetLastError()) != cudaSuccess) return ep_cuda(e, "barrier");
  if ((e = mark(2)) != cudaSuccess) return ep_cuda(e, "event");
  return AGM_OK;
}

// Phase 3 (comm stream): each token's k expert rows, gate-weighted, from this
// rank's home buffer (where the computing ranks wrote them).
AGM_API int agm_ep_combine(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           int64_t cap_rows, const void* home, void* out, void* workspace, size_t workspace_bytes,
                           void* stream_) {
  const int eb = eb_of(dtype);
  if (!eb) return ep_fail(AGM_ERR_UNSUPPORTED, "agm_ep_combine: dtype must be AGM_BF16 or AGM_F16");
  if (!workspace || (n_tokens > 0 && (!out || !home))) return ep_fail(AGM_ERR_ARG, "agm_ep_combine: null pointer");
  EpLayout L = ep_carve(workspace, n_tokens, d, n_experts, top_k, hidden, cap_rows, eb);
  if (L.bytes > workspace_bytes) return ep_fail(AGM_ERR_WORKSPACE, "agm_ep_combine: workspace too small");
  if (n_tokens <= 0) return AGM_OK;
  cudaError_t e = agm::combine(dtype, home, L.row_of, L.gates, n_tokens, d, top_k, nullptr, 0, 0, nullptr, out,
                               num_sms_dev(), static_cast<cudaStream_t>(stream_));
  return e == cudaSuccess ? AGM_OK : ep_cuda(e, "combine");
}

AGM_API int agm_ep_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                           int placement, const uint32_t* expert_holders, int world, int rank,
                           const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch, void* out,
                           void* workspace, size_t workspace_bytes, int flags, void* const* stage_events,
                           void* stream) {
  if (!w1 || !b1 || !w2 || !b2 || !expert_holders || !peer_comm || (n_tokens > 0 && !out))
    return ep_fail(AGM_ERR_ARG, "agm_ep_forward: null pointer argument");
  if (rank < 0 || rank >= agm::kEpMaxRanks || n_experts < 1 || n_experts > AGM_MAX_EXPERTS)
    return ep_fail(AGM_ERR_ARG, "agm_ep_forward: bad rank / n_experts");
  int n_local = 0;
  for (int e = 0; e < n_experts; ++e) n_local += (expert_holders[e] >> rank) & 1u;
  int rc = agm_ep_dispatch(x, dtype, n_tokens, d, n_experts, top_k, hidden, w_router, placement, expert_holders,
                           world, rank, peer_comm, cap_rows, home_rows, epoch, workspace, workspace_bytes, flags,
                           stage_events, stream);
  if (rc != AGM_OK) return rc;
  rc = agm_ep_expert(dtype, n_tokens, d, n_experts, top_k, hidden, w1, b1, w2, b2, n_local, world, rank, peer_comm,
                     cap_rows, home_rows, epoch, workspace, workspace_bytes, 0,
                     stage_events ? stage_events + 5 : nullptr, stream);
  if (rc != AGM_OK) return rc;
  const int eb = eb_of(dtype);
  const void* home = reinterpret_cast<const void*>(peer_comm[rank] + agm::ep_off_home(n_experts, cap_rows, d, eb));
  rc = agm_ep_combine(dtype, n_tokens, d, n_experts, top_k, hidden, cap_rows, home, out, workspace, workspace_bytes,
                      stream);
  if (rc != AGM_OK) return rc;
  if (stage_events) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(stage_events[8]), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ep_cuda(e, "event");
  }
  return AGM_OK;
}

}  // extern "C"
