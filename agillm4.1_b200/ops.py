"""Python entry points over the C ABI, one per kernel stage plus the fused forward.

Each function takes torch CUDA tensors, allocates its outputs with torch's
caching allocator and launches on the current stream. They mirror the stages
of the reference forward (agillm41.py:4389-4431):

* :func:`router_topk`      router logits, top-k / top-1, gates (4398-4419)
* :func:`dispatch_plan`    expert counts and segment layout (replaces `nonzero`, 4425)
* :func:`permute`          stable scatter of token rows (replaces `index_select`, 4428)
* :func:`grouped_gemm`     expert Linear layers over all segments (4428, 4332-4336)
* :func:`combine`          gate-weighted `index_add_` + shared experts (4420-4430)
* :func:`moe_forward`      all of the above in one call, no host sync
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch

from . import _lib
from ._lib import AGM_FLAG_TIE_LOW_FIRST, AGM_TILE_M, check, dtype_code, load, ptr, stream_handle

# Order of exactly-equal top-k values. The default follows torch.topk on a
# CUDA device (descending expert index among equal values); `tie_low_first`
# orders them by ascending index instead.
def _flags(tie_low_first: bool) -> int:
    return AGM_FLAG_TIE_LOW_FIRST if tie_low_first else 0


def dispatch_blocks(n_tokens: int) -> int:
    return int(load().agm_dispatch_blocks(n_tokens))


def max_rows(n_tokens: int, top_k: int, n_experts: int) -> int:
    return int(load().agm_max_rows(n_tokens, top_k, n_experts))


def router_topk(x: torch.Tensor, w_router: torch.Tensor, top_k: int, *, logits_in: Optional[torch.Tensor] = None,
                want_logits: bool = False, tie_low_first: bool = False, err: Optional[torch.Tensor] = None):
    """Returns (idx int32 [N,k], gates [N,k], block_hist int32 [nb,E], logits fp32 [N,E] or None)."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    dev = x.device
    idx = torch.empty(n, top_k, dtype=torch.int32, device=dev)
    gates = torch.empty(n, top_k, dtype=x.dtype, device=dev)
    hist = torch.empty(dispatch_blocks(n), E, dtype=torch.int32, device=dev)
    logits = torch.empty(n, E, dtype=torch.float32, device=dev) if want_logits else None
    if logits_in is not None:
        logits_in = logits_in.to(dtype=torch.float32).contiguous()
    rc = lib.agm_router_topk(ptr(x), ptr(w_router), dtype_code(x.dtype), n, d, E, top_k, _flags(tie_low_first),
                             ptr(logits_in), ptr(logits), ptr(idx), ptr(gates), ptr(hist), ptr(err),
                             stream_handle(dev))
    check(rc, "agm_router_topk")
    return idx, gates, hist, logits


def dispatch_plan(block_hist: torch.Tensor, n_tokens: int, top_k: int, err: Optional[torch.Tensor] = None
                  ) -> Dict[str, torch.Tensor]:
    lib = load()
    E = block_hist.shape[1]
    dev = block_hist.device
    rows = max_rows(n_tokens, top_k, E)
    out = dict(
        block_off=torch.empty_like(block_hist),
        counts=torch.empty(E, dtype=torch.int32, device=dev),
        seg_start=torch.empty(E + 1, dtype=torch.int32, device=dev),
        tile_expert=torch.empty(max(rows // AGM_TILE_M, 1), dtype=torch.int32, device=dev),
        num_tiles=torch.empty(1, dtype=torch.int32, device=dev),
        token_of=torch.empty(max(rows, 1), dtype=torch.int32, device=dev),
    )
    rc = lib.agm_dispatch_plan(ptr(block_hist), n_tokens, E, top_k, ptr(out["block_off"]), ptr(out["counts"]),
                               ptr(out["seg_start"]), ptr(out["tile_expert"]), ptr(out["num_tiles"]),
                               ptr(out["token_of"]), ptr(err), stream_handle(dev))
    check(rc, "agm_dispatch_plan")
    return out


def permute(x: torch.Tensor, idx: torch.Tensor, plan: Dict[str, torch.Tensor], n_experts: int,
            err: Optional[torch.Tensor] = None):
    """Returns (x_perm [max_rows, d], row_of int32 [N,k]); fills plan['token_of']."""
    lib = load()
    n, d = x.shape
    k = idx.shape[1]
    rows = max_rows(n, k, n_experts)
    x_perm = torch.empty(max(rows, 1), d, dtype=x.dtype, device=x.device)
    row_of = torch.empty(n, k, dtype=torch.int32, device=x.device)
    rc = lib.agm_permute(ptr(x), dtype_code(x.dtype), n, d, n_experts, k, ptr(idx), ptr(plan["block_off"]),
                         ptr(plan["seg_start"]), ptr(plan["counts"]), ptr(x_perm), ptr(row_of),
                         ptr(plan["token_of"]), ptr(err), stream_handle(x.device))
    check(rc, "agm_permute")
    return x_perm, row_of


def grouped_gemm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], *, relu: bool,
                 tile_group: Optional[torch.Tensor] = None, num_tiles: Optional[torch.Tensor] = None,
                 max_tiles: Optional[int] = None, c_rows: Optional[int] = None, force_bn: int = 0,
                 err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """c = act(a @ w[g]^T + bias[g]) per 128-row tile; w is [G, N, K] (nn.Linear layout)."""
    lib = load()
    a_rows, k_in = a.shape
    if w.dim() == 2:
        w = w.unsqueeze(0)
        bias = None if bias is None else bias.unsqueeze(0)
    G, n_out, k_w = w.shape
    if k_w != k_in:
        raise ValueError(f"a has {k_in} features, w expects {k_w}")
    if max_tiles is None:
        max_tiles = (a_rows + AGM_TILE_M - 1) // AGM_TILE_M
    if c_rows is None:
        c_rows = a_rows
    c = torch.empty(c_rows, n_out, dtype=a.dtype, device=a.device)
    rc = lib.agm_grouped_gemm(ptr(a), a_rows, ptr(w), ptr(bias), dtype_code(a.dtype), G, n_out, k_in,
                              ptr(tile_group), ptr(num_tiles), max_tiles, int(relu), force_bn, ptr(c), c_rows,
                              ptr(err), stream_handle(a.device))
    check(rc, "agm_grouped_gemm")
    return c


def combine(y_perm: torch.Tensor, row_of: torch.Tensor, gates: torch.Tensor,
            shared_y: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_r y_perm[row_of[t,r]] * gates[t,r] (+ sum_s shared_y[s, t]), reference rounding order."""
    lib = load()
    n, k = row_of.shape
    d = y_perm.shape[1]
    out = torch.empty(n, d, dtype=y_perm.dtype, device=y_perm.device)
    n_shared = 0 if shared_y is None else shared_y.shape[0]
    stride = 0 if shared_y is None else shared_y.shape[1]
    rc = lib.agm_combine(ptr(y_perm), ptr(row_of), ptr(gates), dtype_code(y_perm.dtype), n, d, k, ptr(shared_y),
                         n_shared, stride, ptr(out), stream_handle(y_perm.device))
    check(rc, "agm_combine")
    return out


def _event_array(events):
    if events is None:
        return None
    if len(events) != _lib.AGM_STAGE_EVENTS:
        raise ValueError(f"stage_events needs {_lib.AGM_STAGE_EVENTS} events")
    for ev in events:
        if not ev.cuda_event:
            ev.record()  # torch creates the CUDA event lazily, on its first record
    return (ctypes.c_void_p * len(events))(*[ev.cuda_event for ev in events])


class Workspace:
    """Device scratch for :func:`moe_forward`, grown on demand and reused.

    One workspace per (device, stream): forwards on the same stream run one
    after another, so they can share it.
    """

    _cache: Dict[tuple, torch.Tensor] = {}

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = cls._cache.get(key)
        if buf is None or buf.numel() < nbytes:
            cls._cache.pop(key, None)
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            cls._cache[key] = buf
        return buf

    @classmethod
    def clear(cls) -> None:
        cls._cache.clear()


def workspace_bytes(n_tokens: int, d: int, n_experts: int, top_k: int, hidden: int, n_shared: int,
                    shared_hidden: int, dtype: torch.dtype) -> int:
    return int(load().agm_moe_workspace_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared, shared_hidden,
                                              dtype_code(dtype)))


def moe_forward_residual(x: torch.Tensor, residual: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor,
                         b1: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor, top_k: int, *,
                         shared: Optional[tuple] = None, check_errors: bool = False) -> torch.Tensor:
    """residual + MoE(x) in one launch sequence (Block's `x + ff(ln2(x))`,
    agillm41.py:4547): x [N, d] is the LayerNorm output, residual [N, d] the
    block input; the combine adds the residual last."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    H = w1.shape[1]
    dev = x.device
    if residual.shape != x.shape or residual.dtype != x.dtype:
        raise _lib.MoEKernelError("residual must have x's shape and dtype")
    ws1, sb1, ws2, sb2, S, Hs = _shared_parts(shared)
    out = torch.empty_like(x)
    nbytes = workspace_bytes(n, d, E, top_k, H, S, Hs, x.dtype)
    workspace = Workspace.get(dev, nbytes)
    rc = lib.agm_moe_forward_residual(ptr(x), ptr(residual.contiguous()), dtype_code(x.dtype), n, d, E, top_k, H,
                                      ptr(w_router), ptr(w1), ptr(b1), ptr(w2), ptr(b2), S, Hs, ptr(ws1), ptr(sb1),
                                      ptr(ws2), ptr(sb2), ptr(out), ptr(workspace), workspace.numel(), 0,
                                      stream_handle(dev))
    check(rc, "agm_moe_forward_residual")
    if check_errors:
        code = _lib.read_device_error(workspace[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_forward_residual")
    return out


def decode_tile_layout(w: torch.Tensor) -> torch.Tensor:
    """[E, n, k] 16-bit weight stack -> the decode tile layout [E, n/128, k/64, 128, 64]
    (agm_decode_tile_layout), for moe_forward(..., decode_tiles=True)."""
    lib = load()
    E, n, k = w.shape
    out = torch.empty(E, n // 128, k // 64, 128, 64, dtype=w.dtype, device=w.device)
    rc = lib.agm_decode_tile_layout(ptr(w.contiguous()), ptr(out), dtype_code(w.dtype), E, n, k,
                                    stream_handle(w.device))
    check(rc, "agm_decode_tile_layout")
    return out


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm over the last dimension of x [N, d] (agm_layernorm)."""
    lib = load()
    n, d = x.shape
    out = torch.empty_like(x) if out is None else out
    rc = lib.agm_layernorm(ptr(x), ptr(weight), ptr(bias), float(eps), dtype_code(x.dtype), n, d, ptr(out),
                           stream_handle(x.device))
    check(rc, "agm_layernorm")
    return out


def moe_block_forward(x: torch.Tensor, ln_weight: torch.Tensor, ln_bias: torch.Tensor, ln_eps: float,
                      w_router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor,
                      top_k: int, *, shared: Optional[tuple] = None, check_errors: bool = False) -> torch.Tensor:
    """x + MoEFFN(LayerNorm(x)): the FFN half of Block.forward (agillm41.py:4547) in one call."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    H = w1.shape[1]
    if shared is not None:
        ws1, sb1, ws2, sb2 = shared
        S, Hs = ws1.shape[0], ws1.shape[1]
    else:
        ws1 = sb1 = ws2 = sb2 = None
        S, Hs = 0, 1
    nbytes = int(lib.agm_moe_block_workspace_bytes(n, d, E, top_k, H, S, Hs, dtype_code(x.dtype)))
    if nbytes == 0:
        raise _lib.MoEKernelError("agm_moe_block_workspace_bytes: unsupported shape or dtype")
    ws = Workspace.get(x.device, nbytes)
    out = torch.empty_like(x)
    rc = lib.agm_moe_block_forward(ptr(x), ptr(ln_weight), ptr(ln_bias), float(ln_eps), dtype_code(x.dtype), n, d, E,
                                   top_k, H, ptr(w_router), ptr(w1), ptr(b1), ptr(w2), ptr(b2), S, Hs, ptr(ws1),
                                   ptr(sb1), ptr(ws2), ptr(sb2), ptr(out), ptr(ws), ws.numel(), 0,
                                   stream_handle(x.device))
    check(rc, "agm_moe_block_forward")
    if check_errors:
        code = _lib.read_device_error(ws[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_block_forward")
    return out


def moe_forward(x: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
                b2: torch.Tensor, top_k: int, *, shared: Optional[tuple] = None, out: Optional[torch.Tensor] = None,
                want: tuple = (), tie_low_first: bool = False, workspace: Optional[torch.Tensor] = None,
                check_errors: bool = False, stage_events=None, logits_in: Optional[torch.Tensor] = None,
                pair: bool = True, swap: bool = True, pdl: bool = True, fold: bool = True,
                decode_tiles: bool = False, front: bool = True):
    """Fused forward: x [N, d] -> out [N, d]. ``want`` may hold 'idx', 'gates', 'counts', 'logits'.

    Weights: w_router [E, d]; w1 [E, H, d]; b1 [E, H]; w2 [E, d, H]; b2 [E, d];
    shared = (ws1 [S,Hs,d], sb1 [S,Hs], ws2 [S,d,Hs], sb2 [S,d]) or None.
    ``logits_in``: optional fp32 [N, E] router logits to route with instead
    of computing them in the router kernel.
    ``stage_events``: optional list of AGM_STAGE_EVENTS torch.cuda.Event
    (timing enabled) recorded around each kernel stage on the current stream.
    ``pair``: let large batches run the expert GEMMs on CTA pairs (False:
    one-CTA tiles throughout). ``swap``: let decode-sized batches run them
    with swapped operands (False: row tiles throughout). ``pdl``: launch each
    kernel so it may start while the previous one finishes (False: each
    waits for the previous kernel to complete before it launches). ``fold``:
    on CTA pairs, run the shared experts inside the routed FC1/FC2 launches
    (False: their own launches; the result is the same bit for bit).
    ``decode_tiles``: w1 and w2 are in the decode tile layout
    (:func:`decode_tile_layout`); decode-sized batches only. ``front``: let
    batches of at most 128 tokens run router, dispatch plan and permute as
    one cluster kernel (False: three kernels; the logits then come from the
    tensor-core router, whose fp32 summation order differs).
    Returns out, or (out, extras dict) when ``want`` is not empty.
    """
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    H = b1.shape[-1]                      # w1 is [E, H, d], or [E, H/128, d/64, 128, 64] in decode tiles
    if decode_tiles and (w1.dim() != 5 or w2.dim() != 5):
        raise ValueError("decode_tiles=True expects w1 and w2 from decode_tile_layout()")
    dev = x.device
    if shared is not None:
        ws1, sb1, ws2, sb2 = shared
        S, Hs = ws1.shape[0], ws1.shape[1]
    else:
        ws1 = sb1 = ws2 = sb2 = None
        S, Hs = 0, 0
    if out is None:
        out = torch.empty_like(x)
    nbytes = workspace_bytes(n, d, E, top_k, H, S, max(Hs, 1), x.dtype)
    if workspace is None:
        workspace = Workspace.get(dev, nbytes)
    extras = {}
    if "idx" in want:
        extras["idx"] = torch.empty(n, top_k, dtype=torch.int32, device=dev)
    if "gates" in want:
        extras["gates"] = torch.empty(n, top_k, dtype=x.dtype, device=dev)
    if "counts" in want:
        extras["counts"] = torch.empty(E, dtype=torch.int32, device=dev)
    if "logits" in want:
        extras["logits"] = torch.empty(n, E, dtype=torch.float32, device=dev)
    ev_arr = _event_array(stage_events)  # kept alive across the call
    rc = lib.agm_moe_forward(
        ptr(x), dtype_code(x.dtype), n, d, E, top_k, H, ptr(w_router), ptr(w1), ptr(b1), ptr(w2), ptr(b2), S,
        max(Hs, 1), ptr(ws1), ptr(sb1), ptr(ws2), ptr(sb2), ptr(out), ptr(workspace), workspace.numel(),
        _flags(tie_low_first) | (0 if pair else _lib.AGM_FLAG_NO_PAIR) | (0 if swap else _lib.AGM_FLAG_NO_SWAP)
        | (0 if pdl else _lib.AGM_FLAG_NO_PDL) | (0 if fold else _lib.AGM_FLAG_NO_FOLD)
        | (_lib.AGM_FLAG_DECODE_TILES if decode_tiles else 0) | (0 if front else _lib.AGM_FLAG_NO_FRONT),
        ptr(extras.get("idx")), ptr(extras.get("gates")), ptr(extras.get("counts")),
        ptr(extras.get("logits")), ptr(logits_in), None if ev_arr is None else ctypes.addressof(ev_arr),
        stream_handle(dev))
    check(rc, "agm_moe_forward")
    if check_errors:
        code = _lib.read_device_error(workspace[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_forward")
    return (out, extras) if want else out


class HostWorkspace:
    """Device scratch for :func:`moe_forward_host`, one per (device, stream)."""

    _cache: Dict[tuple, torch.Tensor] = {}

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = cls._cache.get(key)
        if buf is None or buf.numel() < nbytes:
            cls._cache.pop(key, None)
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            cls._cache[key] = buf
        return buf


DEFAULT_CHUNK_TOKENS = 6144


def moe_forward_host(x_host: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor,
                     w2: torch.Tensor, b2: torch.Tensor, top_k: int, *, shared: Optional[tuple] = None,
                     out_host: Optional[torch.Tensor] = None, chunk_tokens: int = DEFAULT_CHUNK_TOKENS,
                     tie_low_first: bool = False, check_errors: bool = False) -> torch.Tensor:
    """MoE forward on host tensors: x_host [N, d] (CPU, ideally pinned) -> out_host [N, d] (CPU).

    Weights are on the GPU (the current device). Copies in, the forward and
    copies out overlap chunk by chunk; on return the current stream is ordered
    after the last copy, so ``torch.cuda.current_stream().synchronize()``
    makes ``out_host`` ready.
    """
    lib = load()
    if x_host.is_cuda:
        raise _lib.MoEKernelError("moe_forward_host takes host (CPU) tensors; use moe_forward for device tensors")
    if not x_host.is_contiguous():
        raise _lib.MoEKernelError("x_host must be contiguous")
    n, d = x_host.shape
    E = w_router.shape[0]
    H = w1.shape[1]
    dev = w1.device
    if shared is not None:
        ws1, sb1, ws2, sb2 = shared
        S, Hs = ws1.shape[0], ws1.shape[1]
    else:
        ws1 = sb1 = ws2 = sb2 = None
        S, Hs = 0, 0
    if out_host is None:
        out_host = torch.empty(n, d, dtype=x_host.dtype, pin_memory=True)
    chunk = max(1, min(int(chunk_tokens), n)) if n else 1
    nbytes = int(lib.agm_moe_host_workspace_bytes(chunk, d, E, top_k, H, S, max(Hs, 1), dtype_code(x_host.dtype)))
    ws = HostWorkspace.get(dev, nbytes)
    rc = lib.agm_moe_forward_host(
        x_host.data_ptr(), dtype_code(x_host.dtype), n, d, E, top_k, H, ptr(w_router), ptr(w1), ptr(b1), ptr(w2),
        ptr(b2), S, max(Hs, 1), ptr(ws1), ptr(sb1), ptr(ws2), ptr(sb2), out_host.data_ptr(), ptr(ws), ws.numel(),
        chunk, _flags(tie_low_first), stream_handle(dev))
    check(rc, "agm_moe_forward_host")
    if check_errors:
        code = _lib.read_device_error(ws[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_forward_host")
    return out_host


# ---------------------------------------------------------------------------
# Training: forward that keeps its intermediates, and the backward
# ---------------------------------------------------------------------------
def cast_f32(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 CUDA tensor -> contiguous copy in bf16/fp16 (round to nearest even)."""
    if x.dtype != torch.float32:
        raise _lib.MoEKernelError(f"cast_f32 takes an fp32 tensor, not {x.dtype}")
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    rc = load().agm_cast_f32(ptr(x), ptr(out), dtype_code(dtype), x.numel(), stream_handle(x.device))
    check(rc, "agm_cast_f32")
    return out


def train_saved_bytes(n_tokens: int, d: int, n_experts: int, top_k: int, hidden: int, x_dtype: torch.dtype,
                      dtype: torch.dtype, n_shared: int = 0, shared_hidden: int = 1) -> int:
    return int(load().agm_moe_train_saved_bytes(n_tokens, d, n_experts, top_k, hidden, n_shared,
                                                max(shared_hidden, 1), dtype_code(x_dtype), dtype_code(dtype)))


def _shared_parts(shared):
    if shared is None:
        return None, None, None, None, 0, 1
    ws1, sb1, ws2, sb2 = shared
    return ws1, sb1, ws2, sb2, ws1.shape[0], ws1.shape[1]


def moe_forward_train(x: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor,
                      w2: torch.Tensor, b2: torch.Tensor, top_k: int, *, shared: Optional[tuple] = None,
                      residual: Optional[torch.Tensor] = None, tie_low_first: bool = False, pair: bool = True,
                      pdl: bool = True, check_errors: bool = False, want_counts: bool = False):
    """Training forward: x [N, d] -> (out [N, d] in x's dtype, saved uint8 buffer).

    The weights are in the compute dtype: x's dtype, or bf16/fp16 with x fp32
    (autocast: the weights are the 16-bit casts of fp32 master weights).
    ``shared`` = (ws1 [S,Hs,d], sb1 [S,Hs], ws2 [S,d,Hs], sb2 [S,d]) or None.
    ``saved`` holds what :func:`moe_backward` needs; its first int is the
    device error word. With ``want_counts`` the result also carries the rows
    routed to each expert (int32 [E]): (out, saved, counts)."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    H = w1.shape[1]
    dev = x.device
    dtype = w1.dtype
    ws1, sb1, ws2, sb2, S, Hs = _shared_parts(shared)
    nbytes = train_saved_bytes(n, d, E, top_k, H, x.dtype, dtype, S, Hs)
    saved = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    out = torch.empty(n, d, dtype=x.dtype, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev) if want_counts else None
    flags = _flags(tie_low_first) | (0 if pair else _lib.AGM_FLAG_NO_PAIR) | (0 if pdl else _lib.AGM_FLAG_NO_PDL)
    rc = lib.agm_moe_forward_train(ptr(x), dtype_code(x.dtype), dtype_code(dtype), n, d, E, top_k, H, ptr(w_router),
                                   ptr(w1), ptr(b1), ptr(w2), ptr(b2), S, Hs, ptr(ws1), ptr(sb1), ptr(ws2), ptr(sb2),
                                   ptr(None if residual is None else residual.contiguous()), ptr(out), ptr(saved),
                                   saved.numel(), ptr(counts), flags, stream_handle(dev))
    check(rc, "agm_moe_forward_train")
    if check_errors:
        code = _lib.read_device_error(saved[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_forward_train")
    return (out, saved, counts) if want_counts else (out, saved)


def moe_backward(dout: torch.Tensor, saved: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor,
                 w2: torch.Tensor, top_k: int, *, shared: Optional[tuple] = None, pair: bool = True,
                 pair_always: bool = False, pdl: bool = True, check_errors: bool = False):
    """Backward of :func:`moe_forward_train`: dout [N, d] (x's dtype) ->
    (dx, dw_router [E, d], dw1 [E, H, d], db1 [E, H], dw2 [E, d, H], db2 [E, d])
    plus, with ``shared`` (the forward's (ws1, sb1, ws2, sb2)), a seventh item
    (dws1, dsb1, dws2, dsb2); all in x's dtype (fp32 under autocast).
    ``pair`` must be the value the forward was called with; ``pair_always``
    runs the GEMMs on CTA pairs wherever they apply, whatever the size."""
    lib = load()
    n, d = dout.shape
    E = w_router.shape[0]
    H = w1.shape[1]
    dev = dout.device
    dtype = w1.dtype
    gdt = dout.dtype
    ws1, _, ws2, _, S, Hs = _shared_parts(shared)
    dout = dout.contiguous()
    dx = torch.empty(n, d, dtype=gdt, device=dev)
    dwr = torch.empty(E, d, dtype=gdt, device=dev)
    dw1 = torch.empty(E, H, d, dtype=gdt, device=dev)
    db1 = torch.empty(E, H, dtype=gdt, device=dev)
    dw2 = torch.empty(E, d, H, dtype=gdt, device=dev)
    db2 = torch.empty(E, d, dtype=gdt, device=dev)
    sg = None
    if S:
        sg = (torch.empty(S, Hs, d, dtype=gdt, device=dev), torch.empty(S, Hs, dtype=gdt, device=dev),
              torch.empty(S, d, Hs, dtype=gdt, device=dev), torch.empty(S, d, dtype=gdt, device=dev))
    nbytes = int(lib.agm_moe_backward_workspace_bytes(n, d, E, top_k, H, S, Hs, dtype_code(dtype)))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    rc = lib.agm_moe_backward(ptr(dout), dtype_code(gdt), dtype_code(dtype), n, d, E, top_k, H, ptr(w_router),
                              ptr(w1), ptr(w2), S, Hs, ptr(ws1), ptr(ws2), ptr(saved), saved.numel(), ptr(dx),
                              ptr(dwr), ptr(dw1), ptr(db1), ptr(dw2), ptr(db2),
                              *(ptr(t) for t in (sg or (None, None, None, None))), ptr(ws), ws.numel(),
                              (0 if pdl else _lib.AGM_FLAG_NO_PDL) | (0 if pair else _lib.AGM_FLAG_NO_PAIR)
                              | (_lib.AGM_FLAG_BWD_PAIR if pair_always else 0), stream_handle(dev))
    check(rc, "agm_moe_backward")
    if check_errors:
        code = _lib.read_device_error(ws[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_backward")
    if S:
        return dx, dwr, dw1, db1, dw2, db2, sg
    return dx, dwr, dw1, db1, dw2, db2


def moe_aux_forward(x: torch.Tensor, w_router: torch.Tensor, aux_coef: float, z_coef: float, *,
                    check_errors: bool = False):
    """Load-balance + router-z loss of one MoE module (agillm41.py:4477-4491):
    x [N, d] in the router weight's dtype -> (loss, a 0-d fp32 CUDA tensor;
    saved uint8 buffer for :func:`moe_aux_backward`)."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    dev = x.device
    dt = dtype_code(w_router.dtype)
    x = x.contiguous()
    saved = torch.empty(max(int(lib.agm_moe_aux_saved_bytes(n, E, dt)), 256), dtype=torch.uint8, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    rc = lib.agm_moe_aux_forward(ptr(x), dt, n, d, E, ptr(w_router.contiguous()), float(aux_coef), float(z_coef),
                                 ptr(loss), ptr(saved), saved.numel(), 0, stream_handle(dev))
    check(rc, "agm_moe_aux_forward")
    if check_errors:
        code = _lib.read_device_error(saved[:4].view(torch.int32))
        if code:
            raise _lib.MoEKernelError(f"device error word 0x{code:x} after agm_moe_aux_forward")
    return loss, saved


def moe_aux_backward(dloss: torch.Tensor, x: torch.Tensor, w_router: torch.Tensor, saved: torch.Tensor
                     ) -> torch.Tensor:
    """Router weight gradient [E, d] (the weight's dtype) of the loss of
    :func:`moe_aux_forward`, given its upstream gradient ``dloss`` (0-d)."""
    lib = load()
    n, d = x.shape
    E = w_router.shape[0]
    dev = x.device
    dt = dtype_code(w_router.dtype)
    g = dloss.to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    dw = torch.empty(E, d, dtype=w_router.dtype, device=dev)
    ws = torch.empty(max(int(lib.agm_moe_aux_backward_workspace_bytes(n, d, dt)), 256), dtype=torch.uint8,
                     device=dev)
    rc = lib.agm_moe_aux_backward(ptr(g), ptr(x.contiguous()), dt, n, d, E, ptr(saved), saved.numel(), ptr(dw),
                                  ptr(ws), ws.numel(), 0, stream_handle(dev))
    check(rc, "agm_moe_aux_backward")
    return dw
