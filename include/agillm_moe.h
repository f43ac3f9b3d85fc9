/*
 * agillm_moe.h - C ABI of the B200 (sm_100a) MoE block forward for AGILLM4.1.
 *
 * Drop-in boundary for the reference's `MoEFFN.forward` (agillm41.py:4389-4431).
 * The reference is a Python/PyTorch module, so its "FFI" is the module's
 * forward; each entry point below replaces the part of that forward cited in
 * its comment. All pointers are DEVICE pointers (unless stated), all tensors
 * are dense row-major, and every call is asynchronous on the CUDA stream
 * passed as `stream` (a cudaStream_t; NULL = legacy default stream).
 *
 * Return value: AGM_OK (0) or a negative AGM_ERR_* code; agm_last_error()
 * then describes the failure (thread-local). Kernels never trap: device-side
 * problems (impossible routing, a wait that timed out) are OR-ed into a device
 * error word that the caller reads with agm_read_device_error().
 *
 * dtype: AGM_F32, AGM_BF16 or AGM_F16 for activations, weights, biases and
 * gates alike (the reference runs the block in one dtype: bf16 when the model
 * is converted with --infer_dtype, fp32 otherwise).
 */
#ifndef AGILLM_MOE_H_
#define AGILLM_MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AGM_API __attribute__((visibility("default")))
#else
#define AGM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AGM_ABI_VERSION 1

enum { AGM_F32 = 0, AGM_BF16 = 1, AGM_F16 = 2 };

enum {
  AGM_OK = 0,
  AGM_ERR_ARG = -1,         /* invalid argument (shape, dtype, alignment, null) */
  AGM_ERR_UNSUPPORTED = -2, /* valid for the reference, not supported here     */
  AGM_ERR_CUDA = -3,        /* CUDA runtime error                              */
  AGM_ERR_DEVICE = -4,      /* device error word was non-zero                  */
  AGM_ERR_WORKSPACE = -5    /* workspace too small                             */
};

/* Rows per GEMM row tile. Every expert segment of the permuted activations is
 * padded to a multiple of this (of AGM_PAIR_ROWS inside agm_moe_forward when
 * its expert GEMMs run on CTA pairs). */
#define AGM_TILE_M 128
/* Rows of one CTA-pair GEMM tile (two row tiles sharing one weight group). */
#define AGM_PAIR_ROWS 256
/* agm_moe_forward runs its expert GEMMs on CTA pairs (and pads expert
 * segments to AGM_PAIR_ROWS) when top_k * n_tokens reaches this. */
#define AGM_PAIR_MIN_ROWS 16384
/* agm_moe_forward runs its expert GEMMs with swapped operands (weights as the
 * 128-row MMA operand, each expert's rows as N = 32) when top_k * n_tokens is
 * at most this many rows per expert on average (decode batches). */
#define AGM_SWAP_ROWS_PER_EXPERT 32
/* agm_grouped_gemm force_bn value: 256 x 256 tiles on CTA pairs (tcgen05
 * cta_group::2); row tiles 2i and 2i+1 must share a group. */
#define AGM_GEMM_PAIR (-1)
/* Tokens handled by one CTA of the router and permute kernels. */
#define AGM_DISPATCH_BLOCK 128
/* Largest supported number of experts (router kernel keeps 16 logits/token). */
#define AGM_MAX_EXPERTS 16

/* Number of events agm_moe_forward records when stage_events is given. */
#define AGM_STAGE_EVENTS 8

/* forward flags */
#define AGM_FLAG_TIE_LOW_FIRST 0x1 /* order exactly-equal top-k values by ascending expert index
                                      (default: descending, as torch.topk does on CUDA) */
#define AGM_FLAG_KEEP_ERROR 0x2    /* agm_moe_forward: do not clear the device error word first */
#define AGM_FLAG_NO_PAIR 0x4       /* agm_moe_forward: one-CTA GEMM tiles even where CTA pairs apply */
#define AGM_FLAG_NO_SWAP 0x8       /* agm_moe_forward: row-tile GEMMs even for small batches */
#define AGM_FLAG_NO_PDL 0x10       /* agm_moe_forward: launch each kernel after the previous one
                                      completes (default: programmatic dependent launch) */
#define AGM_FLAG_BWD_PAIR 0x20     /* agm_moe_backward: CTA-pair GEMMs wherever they apply, also for
                                      problems too small to fill the GPU with pair tiles */
#define AGM_FLAG_NO_FOLD 0x40     /* agm_moe_forward: shared experts in their own GEMM launches
                                      (default: inside the routed FC1 / FC2 launches on CTA pairs) */
#define AGM_FLAG_DECODE_TILES 0x80 /* agm_moe_forward: w1 and w2 are in the decode tile layout
                                      [E][n/128][k/64][128][64] (agm_decode_tile_layout), each
                                      128 x 64 weight tile one contiguous 16 KB block; only for
                                      decode-sized batches (top_k * n_tokens <= 32 * n_experts,
                                      16-bit dtypes, d and hidden multiples of 128) */
#define AGM_FLAG_NO_FRONT 0x100    /* agm_moe_forward: router, dispatch plan and permute as three
                                      kernels even for n_tokens <= 128 (default there: one cluster
                                      kernel of 8 CTAs doing all three; 16-bit dtypes, d <= 2048,
                                      logits computed by the library) */

AGM_API const char* agm_last_error(void);
AGM_API int agm_abi_version(void);

/* Number of dispatch blocks for n_tokens tokens: ceil(n / AGM_DISPATCH_BLOCK). */
AGM_API int64_t agm_dispatch_blocks(int64_t n_tokens);
/* Upper bound on permuted rows: round_up(k*n + E*(P-1), P) with P =
 * AGM_PAIR_ROWS when k*n >= AGM_PAIR_MIN_ROWS, else AGM_TILE_M. */
AGM_API int64_t agm_max_rows(int64_t n_tokens, int top_k, int n_experts);

/* Router + top-k. Replaces agillm41.py:4398-4419 (scores = router(x).float();
 * top-k: vals, idx = topk(scores, k); w = softmax(vals).to(dtype);
 * top-1 (4401-4416): idx = argmax(softmax(scores)), gate 1.0).
 *   x [n, d], w_router [E, d]      -> idx int32 [n, k], gates [n, k] (dtype),
 *                                     block_hist int32 [agm_dispatch_blocks(n), E]
 *   logits_in  (nullable) fp32 [n, E]: select from these logits instead of
 *                                     computing them (bit-exactness checks)
 *   logits_out (nullable) fp32 [n, E]: the logits (rounded like the reference)
 *   flags: AGM_FLAG_TIE_LOW_FIRST
 *   err: device int (nullable)                                                */
AGM_API int agm_router_topk(const void* x, const void* w_router, int dtype, int64_t n_tokens, int d, int n_experts,
                    int top_k, int flags, const float* logits_in, float* logits_out, int32_t* idx, void* gates,
                    int32_t* block_hist, int* err, void* stream);

/* Dispatch plan (expert histogram prefix sums). Replaces the `nonzero` calls
 * of the reference dispatch loop (agillm41.py:4421-4426).
 *   block_hist [nb, E] -> block_off [nb, E], counts [E], seg_start [E+1]
 *   (segments padded to AGM_TILE_M), tile_expert [max_rows/AGM_TILE_M],
 *   num_tiles [1], token_of [max_rows] (padding rows set to -1).          */
AGM_API int agm_dispatch_plan(const int32_t* block_hist, int64_t n_tokens, int n_experts, int top_k, int32_t* block_off,
                      int32_t* counts, int32_t* seg_start, int32_t* tile_expert, int32_t* num_tiles,
                      int32_t* token_of, int* err, void* stream);

/* Stable scatter permutation. Replaces `flat.index_select(0, rows)` of
 * agillm41.py:4428: x [n, d] -> x_perm [max_rows, d] (expert segments in
 * ascending token order, padding rows zeroed), row_of [n, k], token_of.  */
AGM_API int agm_permute(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, const int32_t* idx,
                const int32_t* block_off, const int32_t* seg_start, const int32_t* counts, void* x_perm,
                int32_t* row_of, int32_t* token_of, int* err, void* stream);

/* Grouped GEMM over row tiles. Replaces the expert Linear layers
 * (agillm41.py:4332-4336 via `_run_expert`, 4367-4379):
 *   c[r, :] = act(a[r, :] @ w[g]^T + bias[g])   g = tile_group[r / AGM_TILE_M]
 *   a [a_rows, k_in], w [groups, n_out, k_in], bias [groups, n_out] (nullable),
 *   c [c_rows, n_out]; tile_group (nullable: all tiles use group 0);
 *   num_tiles (nullable device int: valid tiles; else max_tiles are valid).
 *   relu: 1 = ReLU epilogue (FC1), 0 = none (FC2).  force_bn: 0 = auto,
 *   128 or 256 = GEMM tile width, AGM_GEMM_PAIR = 256 x 256 tiles on CTA
 *   pairs (tile_group[2i] == tile_group[2i+1]; a mismatch sets a device
 *   error bit) (bf16/fp16 only).                                          */
AGM_API int agm_grouped_gemm(const void* a, int64_t a_rows, const void* w, const void* bias, int dtype, int groups,
                     int n_out, int k_in, const int32_t* tile_group, const int32_t* num_tiles, int64_t max_tiles,
                     int relu, int force_bn, void* c, int64_t c_rows, int* err, void* stream);

/* Gate-weighted combine. Replaces `out.index_add_(0, rows, y * w[rows])`
 * (agillm41.py:4420-4428) and `out = out + shared(flat)` (4429-4430):
 *   out[t] = sum_r y_perm[row_of[t, r]] * gates[t, r]  (+ sum_s shared_y[s, t])
 *   with every op rounded to dtype in the reference's order.
 *   shared_y (nullable) [n_shared, shared_stride_rows, d].                  */
AGM_API int agm_combine(const void* y_perm, const int32_t* row_of, const void* gates, int dtype, int64_t n_tokens, int d,
                int top_k, const void* shared_y, int n_shared, int64_t shared_stride_rows, void* out, void* stream);

/* Workspace needed by agm_moe_forward (bytes). */
AGM_API size_t agm_moe_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int n_shared,
                               int shared_hidden, int dtype);

/* Whole MoE block forward. Replaces MoEFFN.forward (agillm41.py:4389-4431)
 * in eval mode:
 *   x [n, d]; w_router [E, d]; w1 [E, H, d]; b1 [E, H]; w2 [E, d, H]; b2 [E, d];
 *   shared experts (n_shared may be 0): ws1 [S, Hs, d]; sb1 [S, Hs];
 *   ws2 [S, d, Hs]; sb2 [S, d];  out [n, d].
 *   Optional outputs (nullable): idx_out int32 [n, k], gates_out [n, k],
 *   counts_out int32 [E], logits_out fp32 [n, E].
 *   logits_in (nullable) fp32 [n, E]: route with these router logits instead
 *   of computing them (e.g. the logits of the library GEMM the reference
 *   calls, for routing that is bit-exact with it on the same GPU).
 *   The device error word is the first int of the workspace.
 *   stage_events (nullable): AGM_STAGE_EVENTS cudaEvent_t handles recorded on
 *   `stream` before the router and after the router, dispatch plan, permute,
 *   FC1, FC2, shared experts and combine (for per-kernel timing).
 * No host synchronisation; every kernel runs on `stream`.                  */
AGM_API int agm_moe_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                    const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2, int n_shared,
                    int shared_hidden, const void* ws1, const void* sb1, const void* ws2, const void* sb2, void* out,
                    void* workspace, size_t workspace_bytes, int flags, int32_t* idx_out, void* gates_out,
                    int32_t* counts_out, float* logits_out, const float* logits_in, void* const* stage_events,
                    void* stream);

/* agm_moe_forward plus the residual add that follows it in Block.forward
 * (agillm41.py:4547, `x + self.ff(self.ln2(x))`; 4543 with a KV cache): the
 * combine adds residual [n, d] (dtype) last, out = residual + MoEFFN(x), with
 * the reference's rounding (the sum rounded once). x is the LayerNorm output,
 * residual the block input; out may alias neither. Flags as agm_moe_forward. */
AGM_API int agm_moe_forward_residual(const void* x, const void* residual, int dtype, int64_t n_tokens, int d,
                                     int n_experts, int top_k, int hidden, const void* w_router, const void* w1,
                                     const void* b1, const void* w2, const void* b2, int n_shared, int shared_hidden,
                                     const void* ws1, const void* sb1, const void* ws2, const void* sb2, void* out,
                                     void* workspace, size_t workspace_bytes, int flags, void* stream);

/* LayerNorm over the last dimension with an affine weight and bias, as the
 * Block's nn.LayerNorm(d) computes it (agillm41.py:4518; applied as ln2 at
 * 4543 and 4547): x [n, d] -> out [n, d] in dtype. Statistics in fp32 (mean,
 * then the mean squared deviation from it, rstd = rsqrt(var + eps)); y =
 * (x - mean) * rstd * weight + bias rounded once to dtype. torch reduces in
 * another order, so a value can differ from torch's by one unit in the last
 * place of dtype. d * sizeof(dtype) a multiple of 16 bytes; d <= 2048 for
 * 16-bit dtypes, <= 1536 for fp32. One warp per row, HBM-bound.            */
AGM_API int agm_layernorm(const void* x, const void* weight, const void* bias, float eps, int dtype, int64_t n_rows,
                          int d, void* out, void* stream);

/* The FFN half of Block.forward (agillm41.py:4547, `x + self.ff(self.ln2(x))`;
 * with a KV cache 4543, pass x + y): out = x + MoEFFN(LayerNorm(x)) with the
 * LayerNorm of agm_layernorm written into the workspace and the residual
 * added in the combine (agm_moe_forward_residual). workspace >=
 * agm_moe_block_workspace_bytes(...); its first int is the device error
 * word. out may not alias x.                                                 */
AGM_API size_t agm_moe_block_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                                             int n_shared, int shared_hidden, int dtype);
AGM_API int agm_moe_block_forward(const void* x, const void* ln_weight, const void* ln_bias, float ln_eps, int dtype,
                                  int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                                  const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                                  int n_shared, int shared_hidden, const void* ws1, const void* sb1, const void* ws2,
                                  const void* sb2, void* out, void* workspace, size_t workspace_bytes, int flags,
                                  void* stream);

/* Size of the scratch area compiled into the library for
 * agm_moe_forward_noalloc (32 MiB; e.g. up to 967 tokens at d=1280, H=3200,
 * 14 experts, top-2, bf16 without shared experts, or 647 tokens with one
 * shared expert of hidden 2560). */
#define AGM_NOALLOC_SCRATCH_BYTES (32u << 20)

/* agm_moe_forward for callers that cannot allocate device memory (no
 * counterpart in the reference): a host that owns all GPU memory through its
 * own pool and passes only input/output buffers, or a process that must not
 * grow its GPU footprint at run time. Same arguments and results as
 * agm_moe_forward without the workspace; the scratch is a fixed array of
 * AGM_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU that loads
 * it until the process exits. A problem needing more scratch is rejected with
 * AGM_ERR_WORKSPACE. The first call on each device looks up the array's device
 * address (with that device current); make that first call before any stream
 * capture. All calls share the array: calls that overlap on the GPU race. The
 * device error word is the array's first int, cleared by every call (the
 * AGM_FLAG_KEEP_ERROR flag is ignored here), so it reports the latest call
 * alone; agm_moe_noalloc_error_word gives its address.                     */
AGM_API int agm_moe_forward_noalloc(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k,
                                    int hidden, const void* w_router, const void* w1, const void* b1, const void* w2,
                                    const void* b2, int n_shared, int shared_hidden, const void* ws1, const void* sb1,
                                    const void* ws2, const void* sb2, void* out, int flags, void* stream);

/* Device address of agm_moe_forward_noalloc's error word on the current
 * device (the first int of its built-in scratch), for agm_read_device_error.
 * Like agm_moe_forward_noalloc it allocates nothing; the first call on a
 * device looks the address up with that device current. */
AGM_API int agm_moe_noalloc_error_word(int** err);

/* Device workspace for agm_moe_forward_host with chunks of chunk_tokens. */
AGM_API size_t agm_moe_host_workspace_bytes(int64_t chunk_tokens, int d, int n_experts, int top_k, int hidden,
                                            int n_shared, int shared_hidden, int dtype);

/* MoEFFN.forward (agillm41.py:4389-4431) on HOST buffers x_host [n, d] ->
 * out_host [n, d] (page-locked for overlap), for callers whose activations
 * live in host memory (the reference pages layers between host and device,
 * agillm41.py:7656-7668). The batch is split into chunks of chunk_tokens;
 * the host->device copy of one chunk, the forward of the previous one and
 * the device->host copy of the one before run concurrently (two copy streams
 * owned by the library, the forward on `stream`). Bit-identical to
 * agm_moe_forward on the whole batch. Weights are device pointers as for
 * agm_moe_forward; workspace >= agm_moe_host_workspace_bytes(chunk_tokens,...).
 * On return `stream` is ordered after the last copy out. The device error
 * word (first int of the workspace) accumulates over all chunks.            */
AGM_API int agm_moe_forward_host(const void* x_host, int dtype, int64_t n_tokens, int d, int n_experts, int top_k,
                                 int hidden, const void* w_router, const void* w1, const void* b1, const void* w2,
                                 const void* b2, int n_shared, int shared_hidden, const void* ws1, const void* sb1,
                                 const void* ws2, const void* sb2, void* out_host, void* workspace,
                                 size_t workspace_bytes, int64_t chunk_tokens, int flags, void* stream);

/* ---- Expert parallelism across the GPUs of one node (NVLink peer memory) ----
 * The reference runs MoEFFN.forward (agillm41.py:4389-4431) on one device; the
 * entry points below spread its expert FFN work (the loop over experts,
 * agillm41.py:4421-4428) over P ranks (one process per GPU) and move rows
 * inside the kernels instead of through a collective. Each rank allocates one
 * communication buffer (agm_ep_alloc, IPC-shareable), shares its handle
 * (agm_ep_ipc_handle) with the other ranks, which map it (agm_ep_ipc_open);
 * every rank then calls agm_ep_forward with the same sequence of epochs
 * (1, 4, 7, ...: each call uses epoch, epoch+1, epoch+2). 16-bit dtypes
 * (AGM_BF16, AGM_F16) only: the expert GEMMs run on CTA pairs, and every
 * (rank, expert) segment is padded to AGM_PAIR_ROWS rows.                   */

/* Placements (where each expert's weights live and who computes its rows). */
#define AGM_EP_HOLDERS 0   /* expert e on the ranks of bitmask holders[e]: the static
                              contiguous ownership, optionally plus replicas of hot experts */
#define AGM_EP_BALANCED 1  /* every rank holds every expert; equal shares of the global work */
#define AGM_EP_LOCAL 2     /* every rank holds every expert; each keeps its own rows up to
                              an equal share, only the excess moves */

/* Rows of one rank's permuted buffer for n_tokens (segments padded to 256). */
AGM_API int64_t agm_ep_max_rows(int64_t n_tokens, int top_k, int n_experts);
/* Bytes of one rank's communication buffer: signals, counts inbox, receive
 * rows (cap_rows: rows this rank may compute) and home rows (home_rows =
 * agm_ep_max_rows of the most tokens a rank routes per call: the FFN outputs
 * of its own rows, written by the computing ranks). Both multiples of 256. */
AGM_API size_t agm_ep_comm_bytes(int n_experts, int64_t cap_rows, int64_t home_rows, int d, int dtype);
/* Byte offset of the home rows in a communication buffer (for agm_ep_combine). */
AGM_API int64_t agm_ep_home_offset(int n_experts, int64_t cap_rows, int d, int dtype);
/* cudaMalloc a communication buffer (signals and inbox zeroed). */
AGM_API int agm_ep_alloc(size_t bytes, void** ptr);
AGM_API int agm_ep_free(void* ptr);
/* 64-byte CUDA IPC handle of a buffer from agm_ep_alloc. */
AGM_API int agm_ep_ipc_handle(void* ptr, void* handle_out);
/* Map a peer's buffer into this process (device pointer) / unmap it. */
AGM_API int agm_ep_ipc_open(const void* handle, void** peer_ptr);
AGM_API int agm_ep_ipc_close(void* peer_ptr);
/* Local (non-shared) device workspace of agm_ep_forward. */
AGM_API size_t agm_ep_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int64_t cap_rows,
                                      int dtype);
/* Expert-parallel MoEFFN.forward of this rank's tokens x [n, d] -> out [n, d].
 * w_router [E, d] (all experts). expert_holders: HOST array of E bitmasks,
 * bit r set when rank r holds expert e (every rank passes the same array);
 * w1/b1/w2/b2 hold this rank's experts in ascending expert order. placement
 * AGM_EP_HOLDERS: an expert with one holder is computed there; an expert with
 * several is split among them each call, largest first, by water-filling the
 * holders' loads. AGM_EP_BALANCED / AGM_EP_LOCAL need every bit set.
 * peer_comm: HOST array of `world` device addresses of every rank's
 * communication buffer as mapped here (own buffer at [rank]). The counts
 * exchange, the delivery signals and the barrier after FC2 are flag writes
 * in peer memory, bounded waits (a time-out sets the device error word, the
 * first int of the workspace). A rank's receive buffer holds its own rows
 * first; FC1 waits for a source's delivery signal only before that source's
 * first tile, so it starts while the peers' rows still arrive.
 * stage_events (nullable): AGM_EP_STAGE_EVENTS cudaEvent_t handles recorded
 * before the router and after: local plan, counts exchange + global plan,
 * dispatch (permute into peers), delivery signal, FC1, FC2 (which writes
 * every output row into its owner's home buffer), barrier, combine.
 * No host synchronisation; outputs are bit-identical to agm_moe_forward on
 * the same tokens.                                                           */
#define AGM_EP_STAGE_EVENTS 9

/* agm_ep_forward in three phases, so that the phases of consecutive token
 * chunks can overlap on two streams (chunk j's expert GEMMs on a compute
 * stream while chunk j+1 is dispatched and chunk j-1 combined on a comm
 * stream). Each chunk in flight needs its own communication buffer, workspace
 * and epoch sequence; a chunk's phases must run in order (dispatch, expert,
 * combine) with the caller ordering them across streams (events).
 * agm_ep_dispatch: router, local plan, counts exchange, device plan, rows into
 *   the computing ranks' receive buffers, delivery signal to every rank
 *   (stage_events: 5 events).
 * agm_ep_expert: FC1/FC2 on the received tiles (n_local_experts weights),
 *   results into the owners' home buffers, barrier; gemm_ctas > 0 caps the
 *   GEMM's persistent CTAs (stage_events: 3 events).
 * agm_ep_combine: gate-weighted combine from `home` (this rank's buffer +
 *   agm_ep_home_offset).                                                      */
AGM_API int agm_ep_dispatch(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                            const void* w_router, int placement, const uint32_t* expert_holders, int world, int rank,
                            const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch,
                            void* workspace, size_t workspace_bytes, int flags, void* const* stage_events,
                            void* stream);
AGM_API int agm_ep_expert(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden, const void* w1,
                          const void* b1, const void* w2, const void* b2, int n_local_experts, int world, int rank,
                          const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch,
                          void* workspace, size_t workspace_bytes, int gemm_ctas, void* const* stage_events,
                          void* stream);
AGM_API int agm_ep_combine(int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           int64_t cap_rows, const void* home, void* out, void* workspace, size_t workspace_bytes,
                           void* stream);
AGM_API int agm_ep_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                           const void* w_router, const void* w1, const void* b1, const void* w2, const void* b2,
                           int placement, const uint32_t* expert_holders, int world, int rank,
                           const uint64_t* peer_comm, int64_t cap_rows, int64_t home_rows, uint64_t epoch, void* out,
                           void* workspace, size_t workspace_bytes, int flags, void* const* stage_events,
                           void* stream);

/* ---- Training: forward that keeps its intermediates, and the backward ----
 * Together these replace PyTorch autograd through MoEFFN.forward
 * (agillm41.py:4389-4431) as the reference trains it (`_train_phase`,
 * agillm41.py:6790-6840: loss.backward() through every Block's MoE FFN).
 * Precision modes:
 *   x_dtype == dtype: x, weights, out, dout, dx and every gradient in one
 *     dtype (fp32, or bf16/fp16 for a model converted to 16 bits);
 *   x_dtype == AGM_F32, dtype AGM_BF16/AGM_F16: torch.autocast over fp32
 *     master weights (the reference's `amp()`, agillm41.py:3054-3066). x, out,
 *     dout, dx and every weight/bias gradient are fp32; the weights passed are
 *     their 16-bit casts (agm_cast_f32); the gradients are the 16-bit values
 *     autograd computes for those casts, returned as fp32.
 * Shared experts (n_shared >= 0, hidden shared_hidden; agillm41.py:4381-4387,
 * 4429-4430) have the layouts of agm_moe_forward: ws1 [S, Hs, d], sb1 [S, Hs],
 * ws2 [S, d, Hs], sb2 [S, d]; their gradients have the same shapes. */

/* Bytes of the state agm_moe_forward_train keeps for agm_moe_backward. */
AGM_API size_t agm_moe_train_saved_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden, int n_shared,
                                         int shared_hidden, int x_dtype, int dtype);
/* Bytes of agm_moe_backward's scratch workspace. */
AGM_API size_t agm_moe_backward_workspace_bytes(int64_t n_tokens, int d, int n_experts, int top_k, int hidden,
                                                int n_shared, int shared_hidden, int dtype);
/* fp32 -> bf16/fp16 cast of n values (autocast's casts of the input and of
 * the weights, agillm41.py:4399 and 4332-4336 under torch.autocast). */
AGM_API int agm_cast_f32(const float* in, void* out, int dtype, int64_t n, void* stream);
/* MoEFFN.forward in training mode (agillm41.py:4389-4431): the same result
 * as agm_moe_forward (x_dtype == dtype) or as the reference under autocast
 * (x_dtype == AGM_F32), keeping the router logits, routing, plan, permuted
 * input, FC1 activations (and their ReLU masks) and expert outputs in `saved`
 * (agm_moe_train_saved_bytes) for agm_moe_backward. counts_out (nullable)
 * int32 [E]: rows routed to each expert (an expert with none gets no
 * gradient at all in the reference, which never calls it). residual
 * (nullable, [n, d], x_dtype): added last as in agm_moe_forward_residual
 * (its gradient is dout itself; agm_moe_backward is unchanged). The device error
 * word is the first int of `saved`. Weight layouts as agm_moe_forward.
 * flags: AGM_FLAG_TIE_LOW_FIRST, AGM_FLAG_NO_PAIR, AGM_FLAG_NO_PDL. */
AGM_API int agm_moe_forward_train(const void* x, int x_dtype, int dtype, int64_t n_tokens, int d, int n_experts,
                                  int top_k, int hidden, const void* w_router, const void* w1, const void* b1,
                                  const void* w2, const void* b2, int n_shared, int shared_hidden, const void* ws1,
                                  const void* sb1, const void* ws2, const void* sb2, const void* residual, void* out,
                                  void* saved, size_t saved_bytes, int32_t* counts_out, int flags, void* stream);
/* Backward of agm_moe_forward_train. Replaces autograd through
 * agillm41.py:4398-4430 (router Linear, top-k/softmax gates or the top-1
 * straight-through gate, index_select, expert Linear/ReLU/Linear, `* weight`,
 * index_add_, shared experts): dout [n, d] (x_dtype) -> dx [n, d] (x_dtype),
 * dw_router [E, d], dw1 [E, H, d], db1 [E, H], dw2 [E, d, H], db2 [E, d] and
 * the shared experts' dws1, dsb1, dws2, dsb2 (x_dtype; written, not
 * accumulated). w_router/w1/w2/ws1/ws2 are the compute-dtype weights the
 * forward used; `saved` is unchanged. The device error word is the first int
 * of `workspace`. */
AGM_API int agm_moe_backward(const void* dout, int x_dtype, int dtype, int64_t n_tokens, int d, int n_experts,
                             int top_k, int hidden, const void* w_router, const void* w1, const void* w2, int n_shared,
                             int shared_hidden, const void* ws1, const void* ws2, const void* saved,
                             size_t saved_bytes, void* dx, void* dw_router, void* dw1, void* db1, void* dw2, void* db2,
                             void* dws1, void* dsb1, void* dws2, void* dsb2, void* workspace, size_t workspace_bytes,
                             int flags, void* stream);

/* ---- Tensor-state codec decode ------------------------------------------
 * Decodes one tensor of the reference's tensor codec
 * (_agillm43_encode_tensor_state / _agillm43_decode_tensor_state,
 * agillm41.py:4858-5102) from its packed payload, already decompressed and in
 * device memory, and writes or applies it to a device tensor of n elements,
 * as the DBlock side-update consumer applies a decoded state
 * (agillm41.py:6029-6046):
 *   kind AGM_CODEC_PLAIN         value = payload (packed_dtype: "lossless" or
 *                                "fp16" pack kinds)
 *   kind AGM_CODEC_INT8          value = float(q) * scale ("int8_symmetric")
 *   kind AGM_CODEC_INT8_ROWWISE  value = float(q[r, c]) * float(row_scales[r])
 *                                with cols elements per row, row scales in
 *                                scales_dtype (AGM_F16 or AGM_F32) ("int8_rowwise")
 * then src = value rounded to target_dtype and
 *   mode AGM_APPLY_COPY  target = src                  (copy_)
 *   mode AGM_APPLY_LERP  target = lerp(target, src, alpha)   (lerp_, torch's formula)
 *   mode AGM_APPLY_ADD   target = target + alpha * src (add_, delta updates)
 * Payload and target need their element alignment; 16-byte alignment takes
 * the vectorised path. */
enum { AGM_CODEC_PLAIN = 0, AGM_CODEC_INT8 = 1, AGM_CODEC_INT8_ROWWISE = 2 };
enum { AGM_APPLY_COPY = 0, AGM_APPLY_LERP = 1, AGM_APPLY_ADD = 2 };
AGM_API int agm_codec_decode(const void* payload, int kind, int packed_dtype, int64_t n, int64_t cols, float scale,
                             const void* row_scales, int scales_dtype, void* target, int target_dtype, int mode,
                             float alpha, void* stream);

/* Several tensors in as few launches as possible (the side-update consumer's
 * loop over a decoded state, agillm41.py:6029-6046, applies every tensor of
 * the state with the same alpha and mode): tensors that share pack kind and
 * payload / scale / target dtypes, are 16-byte aligned and (row-wise int8)
 * have rows of a multiple of 16 elements go up to 16 per launch; any other
 * tensor takes agm_codec_decode. Each entry's fields mean what the arguments
 * of agm_codec_decode mean; every entry is checked before anything launches.
 * The result is that of applying the entries one after another in table
 * order: an entry whose target overlaps the target of an earlier entry (the
 * same tensor twice, say, in ADD or LERP mode) is decoded in a later launch. */
typedef struct AgmCodecTensor {
  const void* payload;
  const void* row_scales;
  void* target;
  int64_t n;
  int64_t cols;
  float scale;
  int kind;
  int packed_dtype;
  int scales_dtype;
  int target_dtype;
} AgmCodecTensor;
AGM_API int agm_codec_decode_batch(const AgmCodecTensor* tensors, int count, int mode, float alpha, void* stream);

/* ---- Auxiliary router losses --------------------------------------------
 * Replaces the per-module body of _collect_moe_aux (agillm41.py:4463-4492):
 * recompute the router logits from the stashed FFN input x [n_tokens, d]
 * (dtype = the router weight's dtype, as `inp.to(router.weight.dtype)`), then
 *   loss = aux_coef * E * sum_e(load_e * importance_e)      if aux_coef > 0
 *        + z_coef * mean_t(logsumexp(logits_t)^2)           if z_coef > 0
 * with importance = mean over tokens of softmax(logits), load_e = the
 * fraction of tokens whose softmax argmax is e (no gradient). loss_out is one
 * device float; 0 when both coefficients are <= 0, NaN for no tokens (as
 * torch's mean of nothing). Sums run in a fixed order: the loss is
 * deterministic. The backward reads the upstream gradient of the loss from
 * device memory (dloss, one float) and writes the router weight's gradient
 * dw_router [E, d] in dtype (the input x is not differentiated: the reference
 * detaches it). */
AGM_API size_t agm_moe_aux_saved_bytes(int64_t n_tokens, int n_experts, int dtype);
AGM_API size_t agm_moe_aux_backward_workspace_bytes(int64_t n_tokens, int d, int dtype);
AGM_API int agm_moe_aux_forward(const void* x, int dtype, int64_t n_tokens, int d, int n_experts,
                                const void* w_router, double aux_coef, double z_coef, float* loss_out, void* saved,
                                size_t saved_bytes, int flags, void* stream);
AGM_API int agm_moe_aux_backward(const float* dloss, const void* x, int dtype, int64_t n_tokens, int d,
                                 int n_experts, const void* saved, size_t saved_bytes, void* dw_router,
                                 void* workspace, size_t workspace_bytes, int flags, void* stream);

/* Decode tile layout of an expert weight stack for AGM_FLAG_DECODE_TILES:
 * w [groups][n][k] (nn.Linear layout, 16-bit) -> out [groups][n/128][k/64]
 * [128][64], every 128 x 64 tile one contiguous 16 KB block, so the
 * decode-regime GEMM streams each weight tile from HBM as one run instead of
 * 128 pieces of 128 bytes. n % 128 == 0, k % 64 == 0; out has w's size. */
AGM_API int agm_decode_tile_layout(const void* w, void* out, int dtype, int64_t groups, int n, int k, void* stream);

/* Synchronise `stream`, read the device error word at `err` (e.g. the first
 * int of a forward workspace) into *code and reset it to 0. Returns AGM_OK if
 * the word was 0, AGM_ERR_DEVICE otherwise.                                */
AGM_API int agm_read_device_error(int* err, int* code, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AGILLM_MOE_H_ */
