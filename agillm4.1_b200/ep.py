"""Expert-parallel MoE block forward across the GPUs of one node.

The reference runs the whole MoE block on one device (agillm41.py:4389-4431);
this module spreads the expert FFN work of a block over P ranks (one process
per GPU, `torch.distributed` over NCCL) while every rank keeps its own tokens:

1. each rank routes and permutes its tokens (router, dispatch plan, permute
   kernels): x_perm holds its rows expert-major, each (rank, expert) segment
   padded to 128-row GEMM tiles;
2. the ranks all-gather their per-expert counts (E int32 per rank; one
   device->host read per forward for the all-to-all split sizes);
3. every rank computes the same plan (:func:`plan_dispatch`) over the global
   tile sequence ordered by (expert, source rank, tile); rank r computes a
   contiguous range of it. Along any source's x_perm the destination rank is
   non-decreasing, so x_perm itself is the all-to-all send buffer;
4. all-to-all of the rows (NCCL, NVLink/NVSwitch), the grouped FC1/FC2 GEMM
   on the received tiles (the tile -> expert table comes from the plan), and
   the reverse all-to-all, which returns y rows to their x_perm positions;
5. each rank combines its tokens' k rows (the unchanged combine kernel).

Placement:
* ``"static"``: expert ownership in contiguous ranges (14 experts over 2/4/8
  ranks: 7/7, 4/4/3/3, 2x6+1x2); a rank holds the weights of its experts only.
* ``"balanced"``: every rank holds all expert weights and the global tile
  sequence is cut into P near-equal ranges, so a hot expert's tiles are spread
  over several ranks (skewed routing stays balanced; results are unchanged
  because rows are independent).
* ``"local"`` (peer-memory forward only): every rank holds all expert weights
  and computes its own tiles up to an equal share of the total; only the
  excess moves (to the ranks below their share), so the exchange carries just
  the imbalance between the ranks' token counts.
* ``"replicated"`` (peer-memory forward only): the static ownership plus
  replicas of the hottest experts, at most ``budget`` extra experts per rank
  (:func:`choose_replicas`, from a profile of per-expert counts); each call
  splits a replicated expert's rows among its holders by water-filling their
  loads (:func:`plan_cuts`).

Rows are independent in the MoE block, so the output of every token is
bit-identical to the single-GPU forward of the same token.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist

TILE = 128


def static_owner_ranges(n_experts: int, world: int) -> List[range]:
    """Contiguous expert ranges: the first (E mod P) ranks get one more."""
    base, extra = divmod(n_experts, world)
    out, e = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append(range(e, e + n))
        e += n
    return out


UNIT = 256   # peer-memory path: work unit of 256 rows (a CTA-pair GEMM row tile pair)


def holder_masks(n_experts: int, world: int, placement: str, replicas=None) -> List[int]:
    """Bitmask of the ranks holding each expert's weights (bit r = rank r).

    "static": the contiguous ownership ranges; "replicated": the same plus
    ``replicas[r]`` (expert ids rank r also holds); "balanced"/"local": all.
    """
    if placement in ("balanced", "local"):
        return [(1 << world) - 1] * n_experts
    masks = [0] * n_experts
    for r, rng in enumerate(static_owner_ranges(n_experts, world)):
        for e in rng:
            masks[e] |= 1 << r
    if placement == "replicated":
        for r, extra in enumerate(replicas or []):
            for e in extra:
                masks[int(e)] |= 1 << r
    elif placement != "static":
        raise ValueError(f"unknown placement {placement!r}")
    return masks


def held_experts(masks: Sequence[int], rank: int) -> List[int]:
    """Experts whose weights rank ``rank`` holds, ascending (its weight stack order)."""
    return [e for e, m in enumerate(masks) if (m >> rank) & 1]


def _waterfill_alloc(U: np.ndarray, masks: Sequence[int], world: int) -> np.ndarray:
    """alloc[e, r]: units of expert e computed by rank r under holder masks
    (the device plan's rule, ep_p2p.cu ep_plan_kernel): single-holder experts
    whole, then the replicated ones, largest first (ties: lower index), each
    water-filled over its holders from the lowest load (ties: lower rank)."""
    E = len(masks)
    alloc = np.zeros((E, world), dtype=np.int64)
    load = np.zeros(world, dtype=np.int64)
    rep = []
    for e in range(E):
        h = [r for r in range(world) if (masks[e] >> r) & 1]
        if len(h) == 1:
            alloc[e, h[0]] = U[e]
            load[h[0]] += U[e]
        else:
            rep.append(e)
    rep.sort(key=lambda e: (-int(U[e]), e))
    for e in rep:
        hs = sorted((r for r in range(world) if (masks[e] >> r) & 1), key=lambda r: (int(load[r]), r))
        remaining, cnt, level = int(U[e]), 1, int(load[hs[0]])
        while cnt < len(hs) and remaining >= (int(load[hs[cnt]]) - level) * cnt:
            remaining -= (int(load[hs[cnt]]) - level) * cnt
            level = int(load[hs[cnt]])
            cnt += 1
        q, rem = divmod(remaining, cnt)
        for t in range(cnt):
            target = level + q + (1 if t < rem else 0)
            alloc[e, hs[t]] = target - load[hs[t]]
            load[hs[t]] = target
    return alloc


def plan_cuts(counts_all: np.ndarray, placement: str, masks: Optional[Sequence[int]] = None,
              unit: int = UNIT) -> np.ndarray:
    """Host mirror of the peer-memory device plan (ep_p2p.cu ep_plan_kernel).

    Returns cut [P, E, P, 2]: source i's rows of expert e in its x_perm units
    [lo, hi) (units of ``unit`` rows, counted from the start of its x_perm,
    every (source, expert) segment padded to whole units) computed by rank r.
    """
    counts_all = np.asarray(counts_all, dtype=np.int64)
    P, E = counts_all.shape
    units = (counts_all + unit - 1) // unit
    T = units.sum(axis=1)
    U = units.sum(axis=0)
    total = int(T.sum())
    xoff = np.zeros((P, E), dtype=np.int64)
    xoff[:, 1:] = np.cumsum(units, axis=1)[:, :-1]
    gofs = np.zeros((P, E), dtype=np.int64)
    gofs[1:, :] = np.cumsum(units, axis=0)[:-1, :]
    cut = np.zeros((P, E, P, 2), dtype=np.int64)
    if placement == "local":
        pieces = np.zeros((P, P, 2), dtype=np.int64)
        quota = np.array([total // P + (1 if r < total % P else 0) for r in range(P)], dtype=np.int64)
        keep = np.minimum(T, quota)
        deficit = quota - keep
        for r in range(P):
            pieces[r, r] = (0, keep[r])
        r = 0
        for i in range(P):
            pos = int(keep[i])
            while pos < T[i]:
                while r < P and deficit[r] == 0:
                    r += 1
                n = int(min(T[i] - pos, deficit[r]))
                pieces[i, r] = (pos, pos + n)
                pos += n
                deficit[r] -= n
        for i in range(P):
            for e in range(E):
                for r in range(P):
                    a = max(pieces[i, r, 0], xoff[i, e])
                    b = min(pieces[i, r, 1], xoff[i, e] + units[i, e])
                    cut[i, e, r] = (a, max(a, b))
        return cut
    chunk = np.zeros((E, P, 2), dtype=np.int64)
    if placement == "balanced":
        e_start = 0
        for e in range(E):
            for r in range(P):
                lo, hi = (r * total) // P, ((r + 1) * total) // P
                a, b = max(lo, e_start), min(hi, e_start + U[e])
                chunk[e, r] = (a - e_start, b - e_start) if b > a else (0, 0)
            e_start += U[e]
    else:
        if masks is None:
            masks = holder_masks(E, P, placement)
        alloc = _waterfill_alloc(U, masks, P)
        for e in range(E):
            c = 0
            for r in range(P):
                chunk[e, r] = (c, c + alloc[e, r])
                c += alloc[e, r]
    for i in range(P):
        for e in range(E):
            u, x0, g0 = units[i, e], xoff[i, e], gofs[i, e]
            for r in range(P):
                a = x0 + max(chunk[e, r, 0], g0) - g0
                b = x0 + min(chunk[e, r, 1], g0 + u) - g0
                cut[i, e, r] = (a, max(a, b))
    return cut


def rank_loads(counts_all: np.ndarray, placement: str, masks: Optional[Sequence[int]] = None,
               unit: int = UNIT) -> np.ndarray:
    """Units each rank computes under a placement (sum of its pieces)."""
    cut = plan_cuts(counts_all, placement, masks, unit)
    return (cut[..., 1] - cut[..., 0]).sum(axis=(0, 1))


def choose_replicas(counts_all: np.ndarray, budget: int = 2, target: float = 1.02,
                    unit: int = UNIT) -> List[List[int]]:
    """Replicas of hot experts on top of the static ownership, at most
    ``budget`` extra experts per rank, chosen from a profile of per-expert row
    counts (e.g. the all-gathered counts of a calibration forward).

    Greedy: while the busiest rank's planned load (:func:`rank_loads`, the
    same water-filling the device runs) exceeds ``target`` x the mean, give
    the expert it computes most of a replica on the least-loaded rank with
    budget left that does not hold it yet; a move is kept only if it lowers
    (the busiest load, the number of ranks at it), so ties among several
    busiest ranks are worked off one by one. Returns ``replicas[r]`` = expert
    ids rank r adds.
    """
    counts_all = np.asarray(counts_all, dtype=np.int64)
    P, E = counts_all.shape
    replicas: List[List[int]] = [[] for _ in range(P)]
    if P == 1:
        return replicas
    while True:
        masks = holder_masks(E, P, "replicated", replicas)
        loads = rank_loads(counts_all, "holders", masks, unit)
        mean = loads.sum() / P
        if mean == 0 or loads.max() <= target * mean:
            return replicas
        cut = plan_cuts(counts_all, "holders", masks, unit)
        per_e = (cut[..., 1] - cut[..., 0]).sum(axis=0)        # [E, P] units of e computed by r
        busiest = int(np.argmax(loads))
        improved = False
        for e in sorted(range(E), key=lambda e: -int(per_e[e, busiest])):
            if per_e[e, busiest] == 0:
                break
            cands = [r for r in range(P) if len(replicas[r]) < budget and not (masks[e] >> r) & 1]
            for dest in sorted(cands, key=lambda r: (int(loads[r]), r)):
                trial = [list(x) for x in replicas]
                trial[dest].append(e)
                tl = rank_loads(counts_all, "holders", holder_masks(E, P, "replicated", trial), unit)
                if (tl.max(), int((tl == tl.max()).sum())) < (loads.max(), int((loads == loads.max()).sum())):
                    replicas = trial
                    improved = True
                    break
            if improved:
                break
        if not improved:
            return replicas


@dataclass
class DispatchPlan:
    """Per-rank view of one expert-parallel dispatch.

    send_rows[r]    rows of this rank's x_perm sent to rank r (in order)
    recv_rows[i]    rows received from source rank i (in order)
    recv_tile_expert  expert of every received 128-row tile (receive order)
    tile_ranges     [P+1] boundaries of the ranks' ranges in the global tile sequence
    """

    send_rows: List[int]
    recv_rows: List[int]
    recv_tile_expert: np.ndarray
    tile_ranges: np.ndarray
    local_rows: int


def plan_pieces(counts_all: np.ndarray, placement: str) -> np.ndarray:
    """Pieces [P, P, 2]: source i sends its x_perm tiles [lo, hi) to rank r.

    The same plan the device computes for the peer-memory forward:
    "static"/"balanced" cut the global (expert, source, tile) sequence into
    contiguous rank ranges; "local" gives every rank an equal share of all
    tiles, lets each source keep its first min(own, share) tiles and sends the
    rest, in order, to the ranks below their share (lowest rank first).
    """
    counts_all = np.asarray(counts_all, dtype=np.int64)
    P, E = counts_all.shape
    tiles = (counts_all + TILE - 1) // TILE
    T = tiles.sum(axis=1)
    total = int(T.sum())
    pieces = np.zeros((P, P, 2), dtype=np.int64)
    if placement == "local":
        quota = np.array([total // P + (1 if r < total % P else 0) for r in range(P)], dtype=np.int64)
        keep = np.minimum(T, quota)
        deficit = quota - keep
        for r in range(P):
            pieces[r, r] = (0, keep[r])
        r = 0
        for i in range(P):
            pos = int(keep[i])
            while pos < T[i]:
                while r < P and deficit[r] == 0:
                    r += 1
                n = int(min(T[i] - pos, deficit[r]))
                pieces[i, r] = (pos, pos + n)
                pos += n
                deficit[r] -= n
        return pieces
    for i in range(P):
        plan = plan_dispatch(counts_all, i, placement)
        start = 0
        for r in range(P):
            n = plan.send_rows[r] // TILE
            pieces[i, r] = (start, start + n)
            start += n
    return pieces


def plan_dispatch(counts_all: np.ndarray, rank: int, placement: str = "static") -> DispatchPlan:
    """Plan one forward from the all-gathered counts [P, E] (rows per rank per expert)."""
    counts_all = np.asarray(counts_all, dtype=np.int64)
    P, E = counts_all.shape
    tiles = (counts_all + TILE - 1) // TILE                      # [P, E]
    # Global tile sequence ordered by (expert, source rank, tile).
    per_e = tiles.sum(axis=0)                                     # [E]
    e_start = np.concatenate([[0], np.cumsum(per_e)])             # [E+1]
    total = int(e_start[-1])
    if placement == "static":
        owners = static_owner_ranges(E, P)
        bounds = np.array([e_start[o.start] for o in owners] + [total], dtype=np.int64)
    elif placement == "balanced":
        bounds = np.array([(r * total) // P for r in range(P)] + [total], dtype=np.int64)
    else:
        raise ValueError(f"placement must be 'static' or 'balanced', not {placement!r}")
    # Global position of source i's tiles for expert e: e_start[e] + sum_{i'<i} tiles[i', e].
    src_off = np.zeros((P, E), dtype=np.int64)
    src_off[1:] = np.cumsum(tiles, axis=0)[:-1]
    g0 = e_start[:-1][None, :] + src_off                          # [P, E] first global tile
    g1 = g0 + tiles                                               # [P, E] one past last

    def overlap(i, r):
        lo, hi = bounds[r], bounds[r + 1]
        return np.clip(np.minimum(g1[i], hi) - np.maximum(g0[i], lo), 0, None)  # [E] tiles

    send_rows = [int(overlap(rank, r).sum()) * TILE for r in range(P)]
    recv_rows = [int(overlap(i, rank).sum()) * TILE for i in range(P)]
    te = []
    for i in range(P):
        ov = overlap(i, rank)
        for e in range(E):
            te.extend([e] * int(ov[e]))
    return DispatchPlan(send_rows, recv_rows, np.asarray(te, dtype=np.int32), bounds,
                        int(tiles[rank].sum()) * TILE)


class LocalOps:
    """The single-GPU kernel stages used by the expert-parallel forward."""

    def route(self, x, w_router, top_k):
        """-> (idx, gates, x_perm, row_of, counts[E] int32 on device)."""
        from . import ops
        idx, gates, hist, _ = ops.router_topk(x, w_router, top_k)
        plan = ops.dispatch_plan(hist, x.shape[0], top_k)
        x_perm, row_of = ops.permute(x, idx, plan, w_router.shape[0])
        return idx, gates, x_perm, row_of, plan["counts"]

    def ffn(self, rows, w1, b1, w2, b2, tile_expert):
        from . import ops
        n_tiles = tile_expert.numel()
        h = ops.grouped_gemm(rows, w1, b1, relu=True, tile_group=tile_expert, max_tiles=n_tiles)
        return ops.grouped_gemm(h, w2, b2, relu=False, tile_group=tile_expert, max_tiles=n_tiles)

    def combine(self, y_perm, row_of, gates):
        from . import ops
        return ops.combine(y_perm, row_of, gates)


class ExpertParallelMoE:
    """Expert-parallel forward of one MoE block (no autograd).

    ``weights``: (w_router [E, d], w1 [E_w, H, d], b1 [E_w, H], w2 [E_w, d, H],
    b2 [E_w, d]) on this rank's device, where E_w = E for "balanced" and the
    rank's owned experts (``static_owner_ranges``) for "static".
    """

    def __init__(self, weights: Sequence[torch.Tensor], top_k: int, n_experts: int, group=None,
                 placement: str = "static", local_ops: Optional[LocalOps] = None):
        self.w_router, self.w1, self.b1, self.w2, self.b2 = weights
        self.top_k = int(top_k)
        self.E = int(n_experts)
        self.group = group
        self.placement = placement
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ops = local_ops or LocalOps()
        self.first_local_expert = static_owner_ranges(self.E, self.world)[self.rank].start \
            if placement == "static" else 0
        self.last_plan: Optional[DispatchPlan] = None

    @staticmethod
    def shard_weights(w1, b1, w2, b2, rank: int, world: int, placement: str, replicas=None):
        """The expert weights a rank keeps for a placement (held experts in
        ascending order; "replicated" adds ``replicas[rank]`` to the static
        ownership)."""
        if placement in ("balanced", "local"):
            return w1, b1, w2, b2
        keep = held_experts(holder_masks(w1.shape[0], world, placement, replicas), rank)
        idx = torch.tensor(keep, dtype=torch.long, device=w1.device)
        return tuple(t.index_select(0, idx).contiguous() for t in (w1, b1, w2, b2))

    def forward(self, x: torch.Tensor, events: Optional[Sequence] = None) -> torch.Tensor:
        """``events``: optional 7 CUDA events recorded on the current stream at
        the boundaries route | count exchange + plan | dispatch all-to-all |
        expert FFN | return all-to-all | combine (for timing)."""
        n, d = x.shape

        def mark(i):
            if events is not None:
                events[i].record()

        mark(0)
        idx, gates, x_perm, row_of, counts = self.ops.route(x, self.w_router, self.top_k)
        mark(1)
        # (2) counts of every rank; one device->host read for the split sizes.
        counts_all = torch.empty(self.world * self.E, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(counts_all, counts.contiguous(), group=self.group)
        plan = plan_dispatch(counts_all.cpu().numpy().reshape(self.world, self.E), self.rank, self.placement)
        self.last_plan = plan
        # (4) dispatch rows, expert FFN on the received tiles, return rows.
        send = x_perm[:plan.local_rows]
        recv = torch.empty(sum(plan.recv_rows), d, dtype=x.dtype, device=x.device)
        tile_expert = torch.from_numpy(plan.recv_tile_expert - self.first_local_expert).to(x.device,
                                                                                           non_blocking=True)
        mark(2)
        dist.all_to_all_single(recv, send, output_split_sizes=plan.recv_rows, input_split_sizes=plan.send_rows,
                               group=self.group)
        mark(3)
        if recv.shape[0] > 0:
            y_recv = self.ops.ffn(recv, self.w1, self.b1, self.w2, self.b2, tile_expert)
        else:
            y_recv = recv
        mark(4)
        y_perm = torch.empty_like(x_perm)
        dist.all_to_all_single(y_perm[:plan.local_rows], y_recv.contiguous(), output_split_sizes=plan.send_rows,
                               input_split_sizes=plan.recv_rows, group=self.group)
        mark(5)
        # (5) combine this rank's tokens.
        out = self.ops.combine(y_perm, row_of, gates)
        mark(6)
        return out


class _CommSlot:
    """One communication buffer (mapped on every rank) plus its workspace and
    epoch sequence: the resources of one token chunk in flight."""

    def __init__(self, lib, _lib, group, world, rank, n_experts, cap_rows, home_rows, d, hidden, top_k, max_tokens,
                 dtype, device):
        import ctypes

        self.lib, self._lib, self.group = lib, _lib, group
        code = _lib.dtype_code(dtype)
        nbytes = int(lib.agm_ep_comm_bytes(n_experts, cap_rows, home_rows, d, code))
        if nbytes == 0:
            raise ValueError("expert-parallel communication buffer: unsupported dtype or sizes")
        ptr = ctypes.c_void_p()
        _lib.check(lib.agm_ep_alloc(nbytes, ctypes.byref(ptr)), "agm_ep_alloc")
        self.own = ptr.value
        handle = (ctypes.c_uint8 * 64)()
        _lib.check(lib.agm_ep_ipc_handle(self.own, handle), "agm_ep_ipc_handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened, ptrs = [], []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(self.own)
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            pp = ctypes.c_void_p()
            _lib.check(lib.agm_ep_ipc_open(hb, ctypes.byref(pp)), "agm_ep_ipc_open")
            self.opened.append(pp.value)
            ptrs.append(pp.value)
        self.peer_comm = (ctypes.c_uint64 * world)(*ptrs)
        self.home = self.own + int(lib.agm_ep_home_offset(n_experts, cap_rows, d, code))
        self.ws = torch.empty(int(lib.agm_ep_workspace_bytes(max_tokens, d, n_experts, top_k, hidden, cap_rows,
                                                              code)), dtype=torch.uint8, device=device)
        self.epoch = 1

    def close(self):
        for p in self.opened:
            self.lib.agm_ep_ipc_close(p)
        self.opened = []

    def free(self):
        if self.own is not None:
            self.lib.agm_ep_free(self.own)
            self.own = None


class P2PExpertParallelMoE:
    """Expert-parallel forward with the all-to-all fused into the kernels.

    Every rank allocates a communication buffer (receive rows, home rows,
    signal flags, counts inbox) and maps every peer's buffer through CUDA IPC.
    ``forward`` runs with no host sync: the permute kernel writes each row
    straight into the receive buffer of the rank that computes it (NVLink
    stores), flag barriers in peer memory order the phases, the FC2 epilogue
    writes every output row straight into the home buffer of the rank that
    owns the token (NVLink stores, overlapped with the GEMM), and the combine
    reads this rank's own home buffer. See the C ABI ``agm_ep_forward``.

    ``weights``: (w_router [E, d], w1, b1, w2, b2) where the expert stacks
    hold this rank's experts in ascending order (:meth:`ExpertParallelMoE.
    shard_weights` with the same placement and ``replicas``). Placements:
    "static" (contiguous ownership 7/7, 4/4/3/3, 2x6+1x2 for 14 experts),
    "replicated" (static plus ``replicas[r]``, see :func:`choose_replicas`),
    "balanced" and "local" (every rank holds every expert).

    ``chunks > 1`` splits this rank's tokens into chunks and overlaps them on
    two streams: chunk j's expert GEMMs (capped at ``num_SMs - reserve_sms``
    CTAs) run while chunk j+1 is dispatched and chunk j-1 combined on the
    caller's stream; two communication slots alternate between chunks.
    Results are bit-identical for any chunking and placement (tokens are
    independent). All ranks must call ``forward`` the same number of times
    with the same ``chunks`` (every call is a collective).
    """

    def __init__(self, weights: Sequence[torch.Tensor], top_k: int, n_experts: int, max_tokens: int, group=None,
                 placement: str = "balanced", cap_rows: Optional[int] = None, chunks: int = 1,
                 reserve_sms: int = 20, replicas=None):
        from . import _lib, ops

        self._lib = _lib
        self._ops = ops
        self.lib = _lib.load()
        self.w_router, self.w1, self.b1, self.w2, self.b2 = weights
        self.top_k, self.E = int(top_k), int(n_experts)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.placement = placement
        self.replicas = [list(map(int, r)) for r in (replicas or [[] for _ in range(self.world)])]
        self.masks = holder_masks(self.E, self.world, placement, self.replicas)
        self.pl_code = {"static": _lib.AGM_EP_HOLDERS, "replicated": _lib.AGM_EP_HOLDERS,
                        "balanced": _lib.AGM_EP_BALANCED, "local": _lib.AGM_EP_LOCAL}[placement]
        import ctypes
        self.holders = (ctypes.c_uint32 * self.E)(*self.masks)
        self.n_local = len(held_experts(self.masks, self.rank))
        if self.w1.shape[0] != self.n_local:
            raise ValueError(f"rank holds {self.w1.shape[0]} experts, placement {placement} needs {self.n_local}")
        self.device = self.w1.device
        self.d = int(self.w_router.shape[1])
        self.H = int(self.w1.shape[1])
        self.dtype = self.w1.dtype
        self.max_tokens = int(max_tokens)
        self.chunks = max(1, int(chunks))
        self.chunk_tokens = (self.max_tokens + self.chunks - 1) // self.chunks
        rows = int(self.lib.agm_ep_max_rows(self.chunk_tokens, self.top_k, self.E))
        self.home_rows = max(UNIT, rows)
        if cap_rows is None:
            cap_rows = self.world * self.home_rows if placement in ("static", "replicated") else 2 * self.home_rows
        self.cap_rows = (int(cap_rows) + UNIT - 1) // UNIT * UNIT
        n_slots = 1 if self.chunks == 1 else 2
        self.slots = [_CommSlot(self.lib, _lib, group, self.world, self.rank, self.E, self.cap_rows, self.home_rows,
                                self.d, self.H, self.top_k, self.chunk_tokens, self.dtype, self.device)
                      for _ in range(n_slots)]
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.gemm_ctas = 0 if self.chunks == 1 else max(2, (sms - int(reserve_sms)) & ~1)
        self.compute_stream = torch.cuda.Stream(self.device) if self.chunks > 1 else None
        dist.barrier(group=group)

    # -- phases ------------------------------------------------------------
    def _dispatch(self, slot, x, events=None):
        import ctypes
        _lib = self._lib
        ev = self._event_array(events)
        rc = self.lib.agm_ep_dispatch(
            _lib.ptr(x), _lib.dtype_code(x.dtype), x.shape[0], self.d, self.E, self.top_k, self.H,
            _lib.ptr(self.w_router), self.pl_code, ctypes.addressof(self.holders), self.world, self.rank,
            ctypes.addressof(slot.peer_comm), self.cap_rows, self.home_rows, slot.epoch, _lib.ptr(slot.ws),
            slot.ws.numel(), 0, None if ev is None else ctypes.addressof(ev), _lib.stream_handle(x.device))
        _lib.check(rc, "agm_ep_dispatch")

    def _expert(self, slot, n, events=None):
        import ctypes
        _lib = self._lib
        ev = self._event_array(events)
        rc = self.lib.agm_ep_expert(
            _lib.dtype_code(self.dtype), n, self.d, self.E, self.top_k, self.H, _lib.ptr(self.w1),
            _lib.ptr(self.b1), _lib.ptr(self.w2), _lib.ptr(self.b2), self.n_local, self.world, self.rank,
            ctypes.addressof(slot.peer_comm), self.cap_rows, self.home_rows, slot.epoch, _lib.ptr(slot.ws),
            slot.ws.numel(), self.gemm_ctas, None if ev is None else ctypes.addressof(ev),
            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "agm_ep_expert")

    def _combine(self, slot, n, out):
        _lib = self._lib
        rc = self.lib.agm_ep_combine(_lib.dtype_code(self.dtype), n, self.d, self.E, self.top_k, self.H,
                                     self.cap_rows, slot.home, _lib.ptr(out), _lib.ptr(slot.ws), slot.ws.numel(),
                                     torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "agm_ep_combine")
        slot.epoch += 3

    @staticmethod
    def _event_array(events):
        import ctypes
        if events is None:
            return None
        for e in events:
            if not e.cuda_event:
                e.record()
        return (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])

    # -- forward -----------------------------------------------------------
    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, events=None) -> torch.Tensor:
        """``events`` (chunks == 1 only): 9 CUDA events recorded at the stage
        boundaries listed for ``agm_ep_forward``."""
        n = x.shape[0]
        if n > self.max_tokens:
            raise ValueError(f"{n} tokens > max_tokens={self.max_tokens}")
        out = torch.empty_like(x) if out is None else out
        if self.chunks == 1:
            slot = self.slots[0]
            self._dispatch(slot, x, None if events is None else events[:5])
            self._expert(slot, n, None if events is None else events[5:8])
            self._combine(slot, n, out)
            if events is not None:
                events[8].record()
            return out
        comm = torch.cuda.current_stream(self.device)
        comp = self.compute_stream
        bounds = [min(n, j * self.chunk_tokens) for j in range(self.chunks + 1)]
        ev_disp = [torch.cuda.Event() for _ in range(self.chunks)]
        ev_ffn = [torch.cuda.Event() for _ in range(self.chunks)]
        comp.wait_stream(comm)

        def combine(j):
            comm.wait_event(ev_ffn[j])
            self._combine(self.slots[j % 2], bounds[j + 1] - bounds[j], out[bounds[j]:bounds[j + 1]])

        for j in range(self.chunks):
            slot = self.slots[j % 2]
            self._dispatch(slot, x[bounds[j]:bounds[j + 1]])
            ev_disp[j].record(comm)
            with torch.cuda.stream(comp):
                comp.wait_event(ev_disp[j])
                self._expert(slot, bounds[j + 1] - bounds[j])
                ev_ffn[j].record(comp)
            if j >= 1:
                combine(j - 1)
        combine(self.chunks - 1)
        return out

    def device_error(self) -> int:
        code = 0
        for slot in self.slots:
            code |= self._lib.read_device_error(slot.ws[:4].view(torch.int32))
        return code

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's buffers."""
        if not self.slots:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for slot in self.slots:
            slot.close()
        dist.barrier(group=self.group)
        for slot in self.slots:
            slot.free()
        self.slots = []
