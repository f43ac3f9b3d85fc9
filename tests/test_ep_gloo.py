"""Expert-parallel host logic on CPU ranks (gloo, world size 2-4): planning,
count exchange, row all-to-all and tile tables, with the kernel stages
replaced by oracle stand-ins. Every rank's output must equal the
single-process reference forward of its own tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from agillm41_b200 import ep
from oracle import reference_moe


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, placement, skew, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ep_cpu_ops import OracleLocalOps
        d, H, E, k, n = 64, 96, 14, 2, 300 + 37 * rank
        bias = reference_moe.zipf_logit_bias(E, 3, scale=2.0) if skew else None
        sd = reference_moe.make_state(d, H, E, 7, bias_std=0.05, router_logit_bias=bias)
        x = reference_moe.make_input(n, d, 100 + rank, pin_feature0=skew)
        w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)])
        b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)])
        w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)])
        b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)])
        mine = ep.ExpertParallelMoE.shard_weights(w1, b1, w2, b2, rank, world, placement)
        moe = ep.ExpertParallelMoE((sd["router.weight"],) + tuple(mine), k, E, placement=placement,
                                   local_ops=OracleLocalOps())
        out = moe.forward(x)
        ref = reference_moe.moe_forward(x, sd, k)
        err = (out - ref).abs().max().item()
        result_q.put((rank, err, moe.last_plan.recv_rows, moe.last_plan.send_rows))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,placement,skew", [(2, "static", False), (2, "balanced", True),
                                                  (4, "static", True), (3, "balanced", False)])
def test_ep_matches_single_process(world, placement, skew):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, placement, skew, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    results = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, recv_rows, send_rows in results:
        assert err < 1e-5, f"rank {rank}: max |ep - reference| = {err}"
    # Rows sent by i to j are rows received by j from i.
    send = np.array([r[3] for r in results])
    recv = np.array([r[2] for r in results])
    assert (send == recv.T).all()


def test_plan_static_ownership_and_balance():
    rng = np.random.default_rng(0)
    P, E = 8, 14
    counts = rng.integers(0, 5000, size=(P, E))
    counts[:, 3] *= 6                                       # a hot expert
    owners = ep.static_owner_ranges(E, P)
    assert [len(o) for o in owners] == [2, 2, 2, 2, 2, 2, 1, 1]
    assert [len(o) for o in ep.static_owner_ranges(14, 4)] == [4, 4, 3, 3]
    tiles = (counts + 127) // 128
    for placement in ("static", "balanced"):
        plans = [ep.plan_dispatch(counts, r, placement) for r in range(P)]
        for i in range(P):
            assert sum(plans[i].send_rows) == plans[i].local_rows == tiles[i].sum() * 128
            for j in range(P):
                assert plans[i].send_rows[j] == plans[j].recv_rows[i]
        work = np.array([p.recv_tile_expert.size for p in plans])
        assert work.sum() == tiles.sum()
        if placement == "balanced":
            assert work.max() - work.min() <= 1
        else:
            for r in range(P):
                assert set(plans[r].recv_tile_expert.tolist()) <= set(owners[r])


def test_local_plan_pieces():
    """Locality-first plan: pieces partition each source's tiles, every rank
    gets an equal share, and only the excess over a rank's share moves."""
    rng = np.random.default_rng(1)
    for P in (2, 3, 8):
        counts = rng.integers(0, 4000, size=(P, 14))
        counts[0] *= 3                                    # one rank with many more tokens
        tiles = ((counts + 127) // 128).sum(axis=1)
        pieces = ep.plan_pieces(counts, "local")
        total = tiles.sum()
        for i in range(P):
            spans = sorted((lo, hi) for lo, hi in pieces[i] if hi > lo)
            assert spans[0][0] == 0 and spans[-1][1] == tiles[i]
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        load = (pieces[:, :, 1] - pieces[:, :, 0]).sum(axis=0)
        assert load.max() - load.min() <= 1 and load.sum() == total
        moved = sum(pieces[i, r, 1] - pieces[i, r, 0] for i in range(P) for r in range(P) if r != i)
        share = total // P
        assert moved <= np.maximum(tiles - share, 0).sum()
        same = ep.plan_pieces(np.tile(counts[1], (P, 1)), "local")
        assert all(same[i, r, 1] == same[i, r, 0] for i in range(P) for r in range(P) if r != i)


def _check_cuts(counts, cut, unit=ep.UNIT):
    """Pieces of every source tile its expert segments exactly, in order."""
    P, E = counts.shape
    units = (counts + unit - 1) // unit
    for i in range(P):
        start = 0
        for e in range(E):
            spans = sorted((int(lo), int(hi)) for lo, hi in cut[i, e] if hi > lo)
            if units[i, e] == 0:
                assert not spans
                continue
            assert spans[0][0] == start and spans[-1][1] == start + units[i, e]
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            start += units[i, e]


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_peer_plan_cuts_cover_every_unit(P):
    """The host mirror of the device plan (ep_plan_kernel): for every
    placement the pieces partition each (source, expert) segment, experts go
    only to ranks that hold them, and balanced/local loads are even."""
    rng = np.random.default_rng(10 + P)
    E = 14
    counts = rng.integers(0, 20000, size=(P, E))
    counts[:, 5] *= 5
    counts[0, 2] = 0
    for placement in ("static", "balanced", "local"):
        masks = ep.holder_masks(E, P, placement)
        cut = ep.plan_cuts(counts, placement, masks)
        _check_cuts(counts, cut)
        per_e = (cut[..., 1] - cut[..., 0]).sum(axis=0)          # [E, P]
        for e in range(E):
            for r in range(P):
                if per_e[e, r]:
                    assert (masks[e] >> r) & 1
        load = per_e.sum(axis=0)
        if placement != "static":
            assert load.max() - load.min() <= 1
    # replicated: random replica sets within a budget of 2
    reps = [sorted(rng.choice(E, size=min(2, E), replace=False).tolist()) for _ in range(P)]
    masks = ep.holder_masks(E, P, "replicated", reps)
    cut = ep.plan_cuts(counts, "replicated", masks)
    _check_cuts(counts, cut)
    per_e = (cut[..., 1] - cut[..., 0]).sum(axis=0)
    assert all((masks[e] >> r) & 1 for e in range(E) for r in range(P) if per_e[e, r])
    # water-filling never loads a rank more than static ownership does
    assert per_e.sum(axis=0).max() <= ep.rank_loads(counts, "static").max()


def _zipf_profile(P, n_tok=73728, seed=3):
    """Per-rank expert counts of the skewed expert-parallel workload's
    routing: the Zipf(1.2) logit bias on top of N(0, 1) x against the seeded
    router (computed in fp32 on a token sample, scaled to n_tok)."""
    E, d = 14, 1280
    bias = reference_moe.zipf_logit_bias(E, seed, s=1.2, scale=0.63)
    sd = reference_moe.make_state(d, 64, E, seed, router_logit_bias=bias)
    counts = np.zeros((P, E), dtype=np.int64)
    for r in range(P):
        x = reference_moe.make_input(2048, d, seed + 1000 * r, pin_feature0=True)
        idx = torch.topk(x @ sd["router.weight"].t(), 2, dim=-1).indices
        counts[r] = np.bincount(idx.flatten().numpy(), minlength=E) * (n_tok // 2048)
    return counts


@pytest.mark.parametrize("P", [2, 4, 8])
def test_choose_replicas_balances_skew(P):
    """Hot-expert replication on top of static ownership (at most 2 extra
    experts per rank) brings the skewed workload's busiest rank to within 15%
    of the mean, where static ownership alone is far above it."""
    counts = _zipf_profile(P)
    static = ep.rank_loads(counts, "static")
    reps = ep.choose_replicas(counts, budget=2)
    assert all(len(r) <= 2 for r in reps)
    masks = ep.holder_masks(14, P, "replicated", reps)
    for r in range(P):
        assert not set(reps[r]) & set(ep.static_owner_ranges(14, P)[r])
    load = ep.rank_loads(counts, "replicated", masks)
    mean = load.sum() / P
    assert load.sum() == static.sum()
    assert load.max() <= 1.15 * mean, (load.max() / mean, static.max() / mean, reps)
    if P == 8:
        assert static.max() / mean > 2.0


def test_choose_replicas_uniform_profile():
    """Uniform routing: 14 experts over 8 ranks (2x6 + 1x2) leaves the
    two-expert ranks 14% above the mean; replicas level it."""
    P, E = 8, 14
    counts = np.full((P, E), 73728 * 2 // E, dtype=np.int64)
    static = ep.rank_loads(counts, "static")
    reps = ep.choose_replicas(counts, budget=2)
    load = ep.rank_loads(counts, "replicated", ep.holder_masks(E, P, "replicated", reps))
    assert static.max() / (static.sum() / P) > 1.1
    assert load.max() / (load.sum() / P) <= 1.03
