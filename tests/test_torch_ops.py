"""The stage entry points registered as torch operators (agillm_moe::*):
registration, fake-tensor shape propagation (what FX tracing and
torch.compile see) and the refusal of CPU tensors. CPU only; the GPU
results of the same operators are checked in tests/test_gpu_kernels.py."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import agillm41_b200  # noqa: F401  (registers the operators)
from agillm41_b200 import MoEKernelError, ops

D, H, E, K, N = 1280, 3200, 14, 2, 1000


def test_operators_registered():
    for name in ("router_topk", "dispatch_plan", "permute", "grouped_gemm", "combine", "moe_forward"):
        assert hasattr(torch.ops.agillm_moe, name), name


def test_fake_shapes_follow_the_kernels_buffers():
    with FakeTensorMode():
        x = torch.empty(N, D, dtype=torch.bfloat16, device="cuda")
        wr = torch.empty(E, D, dtype=torch.bfloat16, device="cuda")
        idx, gates, hist, logits = torch.ops.agillm_moe.router_topk(x, wr, K)
        assert idx.shape == (N, K) and idx.dtype == torch.int32
        assert gates.shape == (N, K) and gates.dtype == torch.bfloat16
        assert hist.shape == (ops.dispatch_blocks(N), E) and logits.shape == (N, E)
        plan = torch.ops.agillm_moe.dispatch_plan(hist, N, K)
        rows = ops.max_rows(N, K, E)
        assert plan[1].shape == (E,) and plan[2].shape == (E + 1,) and plan[5].shape == (rows,)
        x_perm, row_of, token_of = torch.ops.agillm_moe.permute(x, idx, plan[0], plan[1], plan[2], plan[5])
        assert x_perm.shape == (rows, D) and row_of.shape == (N, K)
        w1 = torch.empty(E, H, D, dtype=torch.bfloat16, device="cuda")
        b1 = torch.empty(E, H, dtype=torch.bfloat16, device="cuda")
        h = torch.ops.agillm_moe.grouped_gemm(x_perm, w1, b1, plan[3], plan[4], True)
        assert h.shape == (rows, H)
        w2 = torch.empty(E, D, H, dtype=torch.bfloat16, device="cuda")
        b2 = torch.empty(E, D, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.agillm_moe.grouped_gemm(h, w2, b2, plan[3], plan[4], False)
        out = torch.ops.agillm_moe.combine(y, row_of, gates, None)
        assert out.shape == (N, D) and out.dtype == torch.bfloat16
        full = torch.ops.agillm_moe.moe_forward(x, wr, w1, b1, w2, b2, K)
        assert full.shape == x.shape and full.dtype == x.dtype


def test_cpu_tensors_refused():
    x = torch.zeros(4, D, dtype=torch.bfloat16)
    wr = torch.zeros(E, D, dtype=torch.bfloat16)
    with pytest.raises(MoEKernelError):
        torch.ops.agillm_moe.router_topk(x, wr, K)


@pytest.mark.gpu
def test_operators_on_the_gpu_match_the_fused_forward():
    """The stage operators chained by hand give the fused forward's bits."""
    from agillm41_b200 import synthetic

    dev = torch.device("cuda")
    n = 3000
    sd = synthetic.make_state(D, H, E, 70, dtype=torch.bfloat16, device=dev, bias_std=0.02)
    w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).contiguous()
    b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).contiguous()
    w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).contiguous()
    b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).contiguous()
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(n, D, 71, dtype=torch.bfloat16, device=dev)
    ref = ops.moe_forward(x, wr, w1, b1, w2, b2, K, pair=False, swap=False)
    full = torch.ops.agillm_moe.moe_forward(x, wr, w1, b1, w2, b2, K)
    idx, gates, hist, logits = torch.ops.agillm_moe.router_topk(x, wr, K)
    block_off, counts, seg_start, tile_expert, num_tiles, token_of = torch.ops.agillm_moe.dispatch_plan(hist, n, K)
    x_perm, row_of, _ = torch.ops.agillm_moe.permute(x, idx, block_off, counts, seg_start, token_of)
    h = torch.ops.agillm_moe.grouped_gemm(x_perm, w1, b1, tile_expert, num_tiles, True)
    y = torch.ops.agillm_moe.grouped_gemm(h, w2, b2, tile_expert, num_tiles, False)
    out = torch.ops.agillm_moe.combine(y, row_of, gates, None)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.equal(full, ops.moe_forward(x, wr, w1, b1, w2, b2, K))
    assert int(counts.sum()) == K * n
