"""The library's stages as torch operators (namespace ``agillm_moe``).

The ctypes functions in :mod:`.ops` are invisible to torch's dispatcher:
FX tracing and ``torch.compile`` cannot see through them and fake tensors
cannot propagate shapes across them. This module registers the same C-ABI
entry points as custom operators with fake (meta) implementations, so a
graph that contains the MoE block can be traced, shape-checked and compiled
with the B200 kernels as opaque nodes:

=====================================  ==========================================================
``agillm_moe::router_topk``            router logits + top-k + gates + block histogram
                                       (agillm41.py:4398-4419)
``agillm_moe::dispatch_plan``          per-expert counts, padded segments, tile table (4421-4426)
``agillm_moe::permute``                expert-sorted rows (``index_select`` of 4428)
``agillm_moe::grouped_gemm``           one expert Linear (+ ReLU) over the row tiles (4367-4379)
``agillm_moe::combine``                gate-weighted ``index_add_`` of 4428 (+ shared experts)
``agillm_moe::moe_forward``            the whole block, ``MoEFFN.forward`` (4389-4431)
=====================================  ==========================================================

Every operator launches on the current CUDA stream and allocates its outputs
through torch's caching allocator. CPU tensors raise ``MoEKernelError`` (no
CPU path). Registration happens on import; ``torch.ops.agillm_moe.<name>``
then works wherever ``agillm41_b200`` was imported.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import ops
from ._lib import AGM_TILE_M, MoEKernelError

_NS = "agillm_moe"


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise MoEKernelError("agillm_moe operators run on CUDA tensors only (there is no CPU path)")


@torch.library.custom_op(f"{_NS}::router_topk", mutates_args=())
def router_topk(x: torch.Tensor, w_router: torch.Tensor, top_k: int) -> Tuple[torch.Tensor, torch.Tensor,
                                                                              torch.Tensor, torch.Tensor]:
    """(idx int32 [N, k], gates [N, k] in x's dtype, block_hist int32 [ceil(N/128), E], logits fp32 [N, E])."""
    _cuda(x, w_router)
    idx, gates, hist, logits = ops.router_topk(x.contiguous(), w_router.contiguous(), top_k, want_logits=True)
    return idx, gates, hist, logits


@router_topk.register_fake
def _(x, w_router, top_k):
    n, E = x.shape[0], w_router.shape[0]
    return (x.new_empty(n, top_k, dtype=torch.int32), x.new_empty(n, top_k),
            x.new_empty(ops.dispatch_blocks(n), E, dtype=torch.int32), x.new_empty(n, E, dtype=torch.float32))


@torch.library.custom_op(f"{_NS}::dispatch_plan", mutates_args=())
def dispatch_plan(block_hist: torch.Tensor, n_tokens: int, top_k: int) -> List[torch.Tensor]:
    """[block_off, counts [E], seg_start [E+1], tile_expert, num_tiles [1], token_of] (int32)."""
    _cuda(block_hist)
    p = ops.dispatch_plan(block_hist.contiguous(), n_tokens, top_k)
    return [p["block_off"], p["counts"], p["seg_start"], p["tile_expert"], p["num_tiles"], p["token_of"]]


@dispatch_plan.register_fake
def _(block_hist, n_tokens, top_k):
    E = block_hist.shape[1]
    rows = ops.max_rows(n_tokens, top_k, E)
    i32 = torch.int32
    return [block_hist.new_empty(block_hist.shape, dtype=i32), block_hist.new_empty(E, dtype=i32),
            block_hist.new_empty(E + 1, dtype=i32), block_hist.new_empty(max(rows // AGM_TILE_M, 1), dtype=i32),
            block_hist.new_empty(1, dtype=i32), block_hist.new_empty(max(rows, 1), dtype=i32)]


@torch.library.custom_op(f"{_NS}::permute", mutates_args=())
def permute(x: torch.Tensor, idx: torch.Tensor, block_off: torch.Tensor, counts: torch.Tensor,
            seg_start: torch.Tensor, token_of: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(x_perm [max_rows, d], row_of int32 [N, k], token_of int32 [max_rows]: source token of each row)."""
    _cuda(x, idx, block_off, counts, seg_start, token_of)
    plan = dict(block_off=block_off, counts=counts, seg_start=seg_start, token_of=token_of.clone())
    x_perm, row_of = ops.permute(x.contiguous(), idx.contiguous(), plan, counts.shape[0])
    return x_perm, row_of, plan["token_of"]


@permute.register_fake
def _(x, idx, block_off, counts, seg_start, token_of):
    n, d = x.shape
    rows = ops.max_rows(n, idx.shape[1], counts.shape[0])
    return x.new_empty(max(rows, 1), d), idx.new_empty(idx.shape, dtype=torch.int32), torch.empty_like(token_of)


@torch.library.custom_op(f"{_NS}::grouped_gemm", mutates_args=())
def grouped_gemm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], tile_group: Optional[torch.Tensor],
                 num_tiles: Optional[torch.Tensor], relu: bool) -> torch.Tensor:
    """c [rows, N] = act(a @ w[g]^T + bias[g]) per 128-row tile, w [G, N, K] (nn.Linear layout)."""
    _cuda(a, w, bias, tile_group, num_tiles)
    return ops.grouped_gemm(a.contiguous(), w.contiguous(), None if bias is None else bias.contiguous(), relu=relu,
                            tile_group=tile_group, num_tiles=num_tiles)


@grouped_gemm.register_fake
def _(a, w, bias, tile_group, num_tiles, relu):
    n_out = w.shape[-2]
    return a.new_empty(a.shape[0], n_out)


@torch.library.custom_op(f"{_NS}::combine", mutates_args=())
def combine(y_perm: torch.Tensor, row_of: torch.Tensor, gates: torch.Tensor,
            shared_y: Optional[torch.Tensor]) -> torch.Tensor:
    """out [N, d] = sum_r y_perm[row_of[t, r]] * gates[t, r] (+ sum_s shared_y[s, t]), the reference's rounding."""
    _cuda(y_perm, row_of, gates, shared_y)
    return ops.combine(y_perm.contiguous(), row_of.contiguous(), gates.contiguous(),
                       None if shared_y is None else shared_y.contiguous())


@combine.register_fake
def _(y_perm, row_of, gates, shared_y):
    return y_perm.new_empty(row_of.shape[0], y_perm.shape[1])


@torch.library.custom_op(f"{_NS}::moe_forward", mutates_args=())
def moe_forward(x: torch.Tensor, w_router: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
                b2: torch.Tensor, top_k: int, ws1: Optional[torch.Tensor] = None, sb1: Optional[torch.Tensor] = None,
                ws2: Optional[torch.Tensor] = None, sb2: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MoEFFN.forward on flattened tokens: x [N, d] -> [N, d]; optional shared experts ws1 [S, Hs, d] ..."""
    _cuda(x, w_router, w1, b1, w2, b2, ws1, sb1, ws2, sb2)
    shared = None if ws1 is None else (ws1.contiguous(), sb1.contiguous(), ws2.contiguous(), sb2.contiguous())
    return ops.moe_forward(x.contiguous(), w_router.contiguous(), w1, b1, w2, b2, top_k, shared=shared)


@moe_forward.register_fake
def _(x, w_router, w1, b1, w2, b2, top_k, ws1=None, sb1=None, ws2=None, sb2=None):
    return torch.empty_like(x)


__all__ = ["router_topk", "dispatch_plan", "permute", "grouped_gemm", "combine", "moe_forward"]
