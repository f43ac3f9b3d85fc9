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
