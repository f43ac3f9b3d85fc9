"""Expert-parallel forward on 2 GPUs: every rank's output equals the
single-GPU forward of its own tokens, bit for bit, for every placement
(static, replicated hot experts, balanced, local; NCCL all-to-all and
peer-memory paths) under skewed routing. Skipped on a host with fewer than
two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from agillm41_b200 import ep, ops, synthetic

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        d, H, E, k, n = 1280, 3200, 14, 2, 3000 + 500 * rank
        bias = synthetic.zipf_logit_bias(E, 3, scale=0.63)
        sd = synthetic.make_state(d, H, E, 3, dtype=torch.bfloat16, device=dev, bias_std=0.02,
                                  router_logit_bias=bias)
        x = synthetic.make_input(n, d, 50 + rank, dtype=torch.bfloat16, device=dev, pin_feature0=True)
        w = [torch.stack([sd[f"experts.{e}.{i}.{p}"] for e in range(E)]).contiguous()
             for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias"))]
        wr = sd["router.weight"].contiguous()
        ref = ops.moe_forward(x, wr, *w, k)
        res = {}
        for placement in ("static", "balanced"):
            mine = ep.ExpertParallelMoE.shard_weights(*w, rank, world, placement)
            moe = ep.ExpertParallelMoE((wr,) + tuple(mine), k, E, placement=placement)
            out = moe.forward(x)
            out2 = moe.forward(x)
            torch.cuda.synchronize()
            res[placement] = (bool(torch.equal(out, ref)), bool(torch.equal(out, out2)))
        # replicas of the hot experts from the all-gathered counts of this batch
        counts = ops.moe_forward(x, wr, *w, k, want=("counts",))[1]["counts"].to(torch.int32)
        counts_all = torch.empty(world * E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(counts_all, counts)
        replicas = ep.choose_replicas(counts_all.cpu().numpy().reshape(world, E), budget=2)
        for placement, chunks in (("static", 1), ("balanced", 1), ("local", 1), ("replicated", 1), ("balanced", 2),
                                  ("static", 3), ("local", 2), ("replicated", 2)):
            reps = replicas if placement == "replicated" else None
            mine = ep.ExpertParallelMoE.shard_weights(*w, rank, world, placement, replicas=reps)
            moe = ep.P2PExpertParallelMoE((wr,) + tuple(mine), k, E, max_tokens=4000, placement=placement,
                                          chunks=chunks, replicas=reps)
            outs = [moe.forward(x).clone() for _ in range(3)]
            torch.cuda.synchronize()
            err = moe.device_error()
            res[f"p2p_{placement}_chunks{chunks}"] = (all(bool(torch.equal(o, ref)) for o in outs), err == 0)
            moe.close()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_bit_identical():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        assert p.exitcode == 0
    for _ in range(2):
        rank, res = q.get(timeout=5)
        for placement, (same_as_single, ok) in res.items():
            assert same_as_single, f"rank {rank} {placement}: differs from the single-GPU forward"
            assert ok, f"rank {rank} {placement}: not deterministic or device error"


def test_p2p_path_single_rank():
    """The peer-memory expert-parallel path with one rank (no peers): device
    plan, row mapping, flag barriers and the mapped combine on one GPU."""
    import datetime

    import torch.distributed as dist

    from agillm41_b200 import ep, ops, synthetic

    dev = torch.device("cuda", 0)
    store = dist.HashStore()
    dist.init_process_group("gloo", store=store, rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    try:
        d, H, E, k = 1280, 3200, 14, 2
        sd = synthetic.make_state(d, H, E, 9, dtype=torch.bfloat16, device=dev, bias_std=0.02)
        w = [torch.stack([sd[f"experts.{e}.{i}.{p}"] for e in range(E)]).contiguous()
             for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias"))]
        wr = sd["router.weight"].contiguous()
        for placement, chunks in (("static", 1), ("balanced", 1), ("local", 1), ("replicated", 1), ("balanced", 3)):
            moe = ep.P2PExpertParallelMoE((wr,) + tuple(w), k, E, max_tokens=5000, placement=placement,
                                          chunks=chunks, replicas=[[]] if placement == "replicated" else None)
            for n in (4096, 1, 777, 5000):
                x = synthetic.make_input(n, d, n, dtype=torch.bfloat16, device=dev)
                out = moe.forward(x)
                ref = ops.moe_forward(x, wr, *w, k)
                torch.cuda.synchronize()
                assert torch.equal(out, ref), (placement, chunks, n)
            assert moe.device_error() == 0
            moe.close()
    finally:
        dist.destroy_process_group()
