"""End-to-end parity of the MoE block forward on the GPU.

Two router-logit sources are tested:

* ``reference_gemm`` - the logits come from the reference's own call
  (``router(x).float()``, a library GEMM) and the selection, dispatch,
  expert FFNs and combine run on our kernels: indices, gates and per-expert
  counts are bit-exact with the oracle (the reference's torch op sequence)
  on the same GPU, and every output row is within the bf16 tolerance
  (2e-2 rel / 1e-2 abs) or the fp32 tolerance (1e-4);
* ``kernel`` (default) - the router kernel computes the logits with fp32
  accumulation and one rounding. The reference's library GEMM may round its
  partial sums, so a few tokens whose top-k gap is within one rounding step
  pick a different expert; every such row must coincide with a logit that
  differs from the reference's or with an exact tie, and all other rows are
  within tolerance.

Also: the golden vectors (reference run on CPU) and size-independent
properties at the full 73,728-token workload.
"""
import pytest
import torch
import torch.nn.functional as F

import agillm41_b200
from agillm41_b200 import ops, synthetic
from gpu_helpers import assert_close_rows, explained_index_mismatches, gate_slack, packed
from golden_io import Golden, names
from oracle import reference_moe

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def run_ours(x, sd, k, E, reference_logits=False, want=("idx", "gates", "counts", "logits")):
    w1, b1, w2, b2, shared = packed(sd, E, DEV)
    wr = sd["router.weight"].to(DEV).contiguous()
    x = x.to(DEV).contiguous()
    logits_in = F.linear(x, wr).float() if reference_logits else None
    out, extra = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=shared, want=want, check_errors=True,
                                 logits_in=logits_in)
    return out, extra


def tie_rows(logits, k):
    E = logits.shape[1]
    top = torch.topk(logits, min(k + 1, E), -1).values
    return (top[:, 1:] == top[:, :-1]).any(1)


def check_against_oracle(x, sd, k, E, dtype, max_flip_frac):
    aux = {}
    with torch.no_grad():
        ref = reference_moe.moe_forward(x, sd, k, aux=aux)
    # Reference logits: bit-exact routing everywhere.
    out, ex = run_ours(x, sd, k, E, reference_logits=True)
    assert torch.equal(ex["idx"].long(), aux["idx"])
    assert torch.equal(ex["counts"].long(), aux["counts"])
    assert torch.equal(ex["gates"], aux["gates"])
    n = x.shape[0]
    assert_close_rows(out, ref, torch.ones(n, dtype=torch.bool, device=DEV), dtype, aux["term_scale"])
    # Kernel logits: explained flips only.
    out2, ex2 = run_ours(x, sd, k, E)
    rows, unexplained = explained_index_mismatches(ex2["idx"], aux["idx"], ex2["logits"], aux["logits"], k)
    assert not unexplained, f"unexplained index mismatches at rows {unexplained[:10]}"
    assert rows.numel() <= max(2, int(max_flip_frac * n)), rows.numel()
    ok = torch.ones(n, dtype=torch.bool, device=DEV)
    ok[rows] = False
    # Where a logit differs without flipping the choice, the gates differ too.
    assert_close_rows(out2, ref, ok, dtype, aux["term_scale"],
                      slack=gate_slack(ex2["gates"], aux["gates"], aux["term_scale"]))
    same_logits = (ex2["logits"] == aux["logits"]).all(1)
    assert torch.equal(ex2["gates"][same_logits], aux["gates"][same_logits])
    return rows.numel()


@pytest.mark.parametrize("name", names())
def test_against_golden(name):
    """Golden vectors = the reference module run on CPU (fp32 exactly, bf16 via
    its CPU GEMM). CPU and CUDA topk order exact ties differently, so rows
    with a tie among the top k+1 logits are excluded from the index check."""
    g = Golden(name)
    assert g.inputs_match()
    out, ex = run_ours(g.x, g.sd, g.top_k, g.E)
    out = out.cpu()
    idx = ex["idx"].cpu().long()
    ties = tie_rows(g.logits, g.top_k)
    same = (idx == g.idx).all(1)
    E = g.logits.shape[1]
    if g.dtype == torch.float32:
        assert bool(same[~ties].all()), f"index mismatch outside tie rows: {(~same & ~ties).nonzero().flatten()[:8]}"
        torch.testing.assert_close(ex["logits"].cpu(), g.logits, rtol=1e-5, atol=1e-5)
        # Per-expert counts over the rows without a tie (CPU and CUDA order
        # exact ties differently; every other row must route identically).
        ours_c = torch.bincount(idx[~ties].flatten(), minlength=E)
        ref_c = torch.bincount(g.idx[~ties].flatten(), minlength=E)
        assert torch.equal(ours_c, ref_c)
        if not ties.any():
            assert torch.equal(ex["counts"].cpu().long(), g.counts)
    else:
        # Every index mismatch must be explained: the kernel's logit differs
        # from the reference's (the CPU library GEMM's bf16 rounding of its
        # partial sums) or the reference's top k+1 logits hold an exact tie.
        rows, unexplained = explained_index_mismatches(idx, g.idx, ex["logits"].cpu(), g.logits, g.top_k)
        assert not unexplained, f"unexplained index mismatches at rows {unexplained[:10]}"
        assert int(rows.numel()) == int((~same).sum())
    assert_close_rows(out, g.out, same, g.dtype)


CASES = [
    # d, H, E, k, N, dtype, shared, seed
    (1280, 3200, 14, 2, 4096, torch.bfloat16, 0, 1),
    (1280, 3200, 14, 2, 999, torch.float16, 0, 5),
    (1280, 5120, 14, 2, 2048, torch.bfloat16, 0, 6),
    (1280, 5120, 2, 1, 1500, torch.bfloat16, 1, 7),     # production shape: E=2, top-1, 1 shared 2d
    (256, 512, 8, 3, 3000, torch.bfloat16, 2, 8),
    (1280, 3200, 14, 2, 64, torch.bfloat16, 0, 2),       # decode batch
    (1280, 3200, 14, 2, 1, torch.bfloat16, 0, 9),
    (1280, 3200, 14, 2, 300, torch.float32, 0, 10),
]


@pytest.mark.parametrize("d,H,E,k,N,dtype,S,seed", CASES)
def test_against_oracle_same_gpu(d, H, E, k, N, dtype, S, seed):
    sd = reference_moe.make_state(d, H, E, seed, dtype=dtype, device=DEV, bias_std=0.02, shared=S,
                                  shared_hidden=2 * d if S else None)
    x = reference_moe.make_input(N, d, seed, dtype=dtype, device=DEV)
    check_against_oracle(x, sd, k, E, dtype, max_flip_frac=0.02)


def test_full_workload_parity_and_properties():
    """The bench workload (B=48, L=1536, d=1280, H=3200, E=14, top-2, bf16, seed 1)."""
    d, H, E, k, N = 1280, 3200, 14, 2, 48 * 1536
    sd = reference_moe.make_state(d, H, E, 1, dtype=torch.bfloat16, device=DEV)
    x = reference_moe.make_input(N, d, 1, dtype=torch.bfloat16, device=DEV)
    flips = check_against_oracle(x, sd, k, E, torch.bfloat16, max_flip_frac=0.02)
    print(f"full workload: {flips} of {N} tokens routed differently with kernel logits")
    out, ex = run_ours(x, sd, k, E)
    assert int(ex["counts"].sum()) == k * N
    # Determinism: a second run is bit-identical.
    out2, ex2 = run_ours(x, sd, k, E)
    assert torch.equal(out, out2) and torch.equal(ex["idx"], ex2["idx"])


def test_decode_chain_28_layers():
    """AR decode shape: 28 independent layers on 64 tokens; each layer's input
    is the previous layer's reference output plus N(0,1) (seed 2)."""
    d, H, E, k, B, L = 1280, 3200, 14, 2, 64, 28
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(B, d, generator=g).to(torch.bfloat16).to(DEV)
    for layer in range(L):
        sd = reference_moe.make_state(d, H, E, 1000 + layer, dtype=torch.bfloat16, device=DEV)
        check_against_oracle(x, sd, k, E, torch.bfloat16, max_flip_frac=0.05)
        with torch.no_grad():
            ref = reference_moe.moe_forward(x, sd, k)
        x = (ref.float() + torch.randn(B, d, generator=g).to(DEV)).to(torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_module_forward(dtype):
    """The drop-in module (constructor, load_state_dict, forward) on the GPU,
    with the reference's router GEMM so every row is comparable."""
    d, H, E, k, N = 1280, 3200, 14, 2, 1000
    sd = reference_moe.make_state(d, H, E, 3, dtype=dtype, bias_std=0.02)
    m = agillm41_b200.MoEFFN(d, mlp_mult=4, experts=E, top_k=k)
    m.experts = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(d, H), torch.nn.ReLU(),
                                                         torch.nn.Linear(H, d)) for _ in range(E)])
    m.load_state_dict(sd)
    m = m.to(device=DEV, dtype=dtype).eval()
    m.check_device_errors = True
    m.router_logits = "reference_gemm"
    x = reference_moe.make_input(N, d, 3, dtype=dtype, device=DEV).reshape(2, N // 2, d)
    with torch.no_grad():
        y = m(x)
        ref = reference_moe.moe_forward(x, {kk: v.to(DEV) for kk, v in sd.items()}, k)
        # After a state reload the packed weights follow the parameters.
        sd2 = reference_moe.make_state(d, H, E, 4, dtype=dtype, bias_std=0.02)
        m.load_state_dict(sd2)
        y2 = m(x)
        ref2 = reference_moe.moe_forward(x, {kk: v.to(DEV) for kk, v in sd2.items()}, k)
    assert y.shape == x.shape and y.dtype == dtype
    every = torch.ones(N // 2, dtype=torch.bool, device=DEV)
    for a, b in ((y, ref), (y2, ref2)):
        for r in range(2):
            assert_close_rows(a[r], b[r], every, dtype)
    m.train()
    m.requires_grad_(True)
    with pytest.raises(agillm41_b200.MoEKernelError):
        m(x)
    assert m.last_router_input is not None


def test_module_production_shape_top1_shared():
    """E=2, top-1, one shared expert of hidden 2d (the production flag set)."""
    d = 1280
    m = agillm41_b200.MoEFFN(d, mlp_mult=4, experts=2, top_k=1, shared_experts=1, shared_mlp_mult=2)
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    m = m.to(device=DEV, dtype=torch.bfloat16).eval()
    m.router_logits = "reference_gemm"
    x = torch.randn(3, 100, d, generator=g).to(torch.bfloat16).to(DEV)
    sd = {k: v for k, v in m.state_dict().items()}
    with torch.no_grad():
        y = m(x)
        ref = reference_moe.moe_forward(x, sd, 1)
    assert_close_rows(y.reshape(-1, d), ref.reshape(-1, d), torch.ones(300, dtype=torch.bool, device=DEV),
                      torch.bfloat16)


@pytest.mark.parametrize("n,chunk", [(5000, 1024), (4096, 4096), (3000, 8192), (777, 100), (40000, 8192)])
def test_host_pipeline_bit_identical(n, chunk):
    """agm_moe_forward_host (host buffers, chunked, copies overlapped with the
    forward) gives exactly the device forward's result."""
    d, H, E, k = 1280, 3200, 14, 2
    sd = reference_moe.make_state(d, H, E, 21, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = reference_moe.make_input(n, d, 21, dtype=torch.bfloat16)
    ref = ops.moe_forward(x.to(DEV), wr, w1, b1, w2, b2, k)
    x_host = x.pin_memory()
    out = ops.moe_forward_host(x_host, wr, w1, b1, w2, b2, k, chunk_tokens=chunk, check_errors=True)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, ref.cpu())


def test_module_forward_host_matches_device():
    d, H, E, k = 1280, 3200, 14, 2
    m = agillm41_b200.MoEFFN(d, mlp_mult=4, experts=E, top_k=k)
    m.experts = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(d, H), torch.nn.ReLU(),
                                                         torch.nn.Linear(H, d)) for _ in range(E)])
    m.load_state_dict(reference_moe.make_state(d, H, E, 22, bias_std=0.02))
    m = m.to(device=DEV, dtype=torch.bfloat16).eval()
    x = reference_moe.make_input(2 * 700, d, 22, dtype=torch.bfloat16).reshape(2, 700, d)
    with torch.no_grad():
        y_dev = m(x.to(DEV)).cpu()
        y_host = m.forward_host(x.pin_memory(), chunk_tokens=512)
    assert y_host.shape == x.shape and not y_host.is_cuda
    assert torch.equal(y_host, y_dev)


@pytest.mark.parametrize("n,k", [(1000, 2), (64, 2), (300, 1)])
def test_cuda_graph_capture_replay(n, k):
    """The forward makes no host synchronisation, so it captures into a CUDA
    graph; replays on new inputs give exactly the eager forward's result."""
    d, H, E = 1280, 3200, 14
    sd = reference_moe.make_state(d, H, E, 23, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    xs = [reference_moe.make_input(n, d, 23 + i, dtype=torch.bfloat16, device=DEV) for i in range(3)]
    eager = [ops.moe_forward(x, wr, w1, b1, w2, b2, k).clone() for x in xs]
    x_static = xs[0].clone()
    out_static = torch.empty_like(x_static)
    ws = torch.empty(ops.workspace_bytes(n, d, E, k, H, 0, 1, torch.bfloat16), dtype=torch.uint8, device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.moe_forward(x_static, wr, w1, b1, w2, b2, k, out=out_static, workspace=ws)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.moe_forward(x_static, wr, w1, b1, w2, b2, k, out=out_static, workspace=ws)
    for x, ref in zip(reversed(xs), reversed(eager)):
        x_static.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_static, ref)
    assert _lib_error(ws) == 0
    del graph


def _lib_error(ws):
    from agillm41_b200 import _lib
    return _lib.read_device_error(ws[:4].view(torch.int32))


def test_pair_gemm_forward_matches_single_cta():
    """Above the pair threshold the forward pads expert segments to 256 rows and
    runs the expert GEMMs on CTA pairs; the result equals the one-CTA path."""
    d, H, E, k, n = 1280, 3200, 14, 2, 12000
    sd = reference_moe.make_state(d, H, E, 24, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = reference_moe.make_input(n, d, 24, dtype=torch.bfloat16, device=DEV)
    out_p, ex_p = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "counts"), check_errors=True)
    out_1, ex_1 = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "counts"), check_errors=True, pair=False)
    assert torch.equal(ex_p["idx"], ex_1["idx"]) and torch.equal(ex_p["counts"], ex_1["counts"])
    assert torch.equal(out_p, out_1)


def test_pair_gemm_shared_expert_matches_single_cta():
    """The production MoE (2 experts, top-1, one shared expert of 2d) above the
    pair threshold: the shared expert's dense GEMMs run on CTA pairs over 129
    row tiles (the last pair holds one) and match the one-CTA path bit for bit."""
    d, E, k, n = 1280, 2, 1, 16500
    sd = synthetic.make_state(d, 4 * d, E, 26, dtype=torch.bfloat16, device=DEV, bias_std=0.02, shared=1,
                              shared_hidden=2 * d)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    sh = tuple(sd[f"shared.0.{i}.{p}"].unsqueeze(0).contiguous()
               for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")))
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(n, d, 26, dtype=torch.bfloat16, device=DEV)
    out_p = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    out_1 = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True, pair=False)
    assert torch.equal(out_p, out_1)
    res = torch.randn(n, d, generator=torch.Generator().manual_seed(27)).to(DEV, torch.bfloat16)
    out_r = ops.moe_forward_residual(x, res, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    assert torch.equal(out_r, out_p + res)


@pytest.mark.parametrize("E,k,H,S,n", [(2, 1, 5120, 1, 33792), (2, 1, 5120, 1, 16500), (14, 2, 3200, 2, 16400),
                                       (8, 3, 2048, 1, 20000)])
def test_shared_experts_folded_into_routed_launches(E, k, H, S, n):
    """Above the pair threshold the shared experts' dense GEMMs ride in the
    routed FC1/FC2 launches as a second problem (agillm41.py:4381-4387,
    4429-4430). The production shape (2 experts, top-1, H = 4d, one shared
    expert of 2d, 22 x 1536 tokens, agillm41.py:8590-8594), an odd number of
    shared row tiles (16,500 tokens: 129), two shared experts with top-2, and
    top-3: bit-identical to the shared experts in their own launches and to
    the one-CTA path; the fused residual add on top of the folded forward."""
    d = 1280
    sd = synthetic.make_state(d, H, E, 40 + S, dtype=torch.bfloat16, device=DEV, bias_std=0.02, shared=S,
                              shared_hidden=2 * d)
    w1, b1, w2, b2, sh = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(n, d, 41 + S, dtype=torch.bfloat16, device=DEV)
    out_f = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    out_s = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True, fold=False)
    assert torch.equal(out_f, out_s)
    out_1 = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True, pair=False)
    assert torch.equal(out_f, out_1)
    res = torch.randn(n, d, generator=torch.Generator().manual_seed(43)).to(DEV, torch.bfloat16)
    out_r = ops.moe_forward_residual(x, res, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    assert torch.equal(out_r, out_f + res)


@pytest.mark.parametrize("n,k,E,S", [(64, 2, 14, 0), (200, 2, 14, 0), (37, 1, 4, 0), (64, 1, 2, 1)])
def test_decode_tile_layout_forward(n, k, E, S):
    """Decode-regime forward with w1/w2 in the decode tile layout
    (AGM_FLAG_DECODE_TILES): each 128 x 64 weight tile is one contiguous 16 KB
    block, loaded by a 5-D TMA box into the same shared-memory image, so the
    result equals the nn.Linear-layout forward bit for bit (shared experts,
    when present, keep their own layout)."""
    d, H = 1280, 3200 if E != 2 else 5120
    sd = synthetic.make_state(d, H, E, 95 + n, dtype=torch.bfloat16, device=DEV, bias_std=0.02, shared=S,
                              shared_hidden=2 * d if S else None)
    w1, b1, w2, b2, sh = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    t1, t2 = ops.decode_tile_layout(w1), ops.decode_tile_layout(w2)
    assert torch.equal(t1, w1.view(E, H // 128, 128, d // 64, 64).permute(0, 1, 3, 2, 4))
    assert torch.equal(t2, w2.view(E, d // 128, 128, H // 64, 64).permute(0, 1, 3, 2, 4))
    x = synthetic.make_input(n, d, 96 + n, dtype=torch.bfloat16, device=DEV)
    ref = ops.moe_forward(x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    out = ops.moe_forward(x, wr, t1, b1, t2, b2, k, shared=sh, check_errors=True, decode_tiles=True)
    assert torch.equal(out, ref)


def test_decode_tile_layout_refused_outside_decode():
    d, H, E, k, n = 1280, 3200, 14, 2, 4096
    sd = synthetic.make_state(d, H, E, 97, dtype=torch.bfloat16, device=DEV)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    x = synthetic.make_input(n, d, 98, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(agillm41_b200.MoEKernelError):
        ops.moe_forward(x, sd["router.weight"].contiguous(), ops.decode_tile_layout(w1), b1,
                        ops.decode_tile_layout(w2), b2, k, decode_tiles=True)


@pytest.mark.parametrize("n,k,E", [(64, 2, 14), (200, 2, 14), (37, 1, 4), (96, 3, 16)])
def test_swap_gemm_forward_matches_row_tiles(n, k, E):
    """Decode-sized batches run the expert GEMMs with swapped operands (weights
    as the MMA's M side, each expert's rows as N); the result equals the
    row-tile path. (200, 2, 14) puts more than 32 rows on some experts, so
    their segments span several 32-row blocks; (37, 1, 4) leaves experts empty."""
    d, H = 1280, 3200
    sd = reference_moe.make_state(d, H, E, 25 + n, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = reference_moe.make_input(n, d, 25 + n, dtype=torch.bfloat16, device=DEV)
    out_s, ex_s = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "counts"), check_errors=True)
    out_t, ex_t = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "counts"), check_errors=True, swap=False)
    assert torch.equal(ex_s["idx"], ex_t["idx"]) and torch.equal(ex_s["counts"], ex_t["counts"])
    assert torch.equal(out_s, out_t)


@pytest.mark.parametrize("n", [64, 3000, 12000])
def test_programmatic_launch_matches_serialised(n):
    """Kernels launched to overlap the previous kernel's tail (each waits for
    it before touching its outputs) give exactly the serialised result, on the
    swapped-operand (64), one-CTA (3000) and CTA-pair (12000) GEMM paths."""
    d, H, E, k = 1280, 3200, 14, 2
    sd = reference_moe.make_state(d, H, E, 26, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    xs = [reference_moe.make_input(n, d, 26 + i, dtype=torch.bfloat16, device=DEV) for i in range(3)]
    serial = [ops.moe_forward(x, wr, w1, b1, w2, b2, k, pdl=False, check_errors=True) for x in xs]
    # back to back on one stream, so every kernel overlaps the one before it
    outs = [ops.moe_forward(x, wr, w1, b1, w2, b2, k) for x in xs]
    torch.cuda.synchronize()
    for a, b in zip(outs, serial):
        assert torch.equal(a, b)


@pytest.mark.parametrize("k,E,S", [(2, 14, 0), (1, 2, 1)])
def test_expert_stream_matches_resident(k, E, S):
    """set_expert_stream(True) with the routed experts on the host, as the
    reference's block streaming leaves them (agillm41.py:7656-7668): the
    output equals the device-resident forward bit for bit, and the load and
    token counters follow the reference (one load per (rank, expert) call
    with rows)."""
    d, H, n = 256, 512, 300
    m = agillm41_b200.MoEFFN(d, mlp_mult=2, experts=E, top_k=k, shared_experts=S, shared_mlp_mult=2 if S else 0)
    m.load_state_dict(reference_moe.make_state(d, H, E, 27, bias_std=0.02, shared=S, shared_hidden=2 * d if S else None))
    m = m.to(device=DEV, dtype=torch.bfloat16).eval()
    x = reference_moe.make_input(n, d, 27, dtype=torch.bfloat16, device=DEV).reshape(3, 100, d)
    with torch.no_grad():
        ref = m(x)
        idx, _, _, _ = ops.router_topk(x.reshape(n, d), m.router.weight.detach().contiguous(), k)
    for ex in m.experts:
        ex.to("cpu")
    m.set_expert_stream(True)
    m.expert_stream_stats = {"loads": 0, "tokens": 0}
    with torch.no_grad():
        out = m(x)
        out2 = m(x)
    assert torch.equal(out, ref) and torch.equal(out2, ref)
    loads = sum(int((torch.bincount(idx[:, r].long(), minlength=E) > 0).sum()) for r in range(k))
    assert m.expert_stream_stats == {"loads": 2 * loads, "tokens": 2 * k * n}
    assert all(p.device.type == "cpu" for ex in m.experts for p in ex.parameters())
    with pytest.raises(agillm41_b200.MoEKernelError):
        m.train()
        m(x.requires_grad_(True))


@pytest.mark.parametrize("S", [0, 1])
def test_forward_residual_equals_separate_add(S):
    """forward_residual(h, x) (the residual added by the combine kernel, as
    Block's `x + ff(ln2(x))`) equals x + forward(h) bit for bit."""
    d, H, E, k, n = 1280, 3200, 14, 2, 3000
    m = agillm41_b200.MoEFFN(d, mlp_mult=4, experts=E, top_k=k, shared_experts=S, shared_mlp_mult=2 if S else 0)
    m.experts = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(d, H), torch.nn.ReLU(),
                                                         torch.nn.Linear(H, d)) for _ in range(E)])
    m.load_state_dict(reference_moe.make_state(d, H, E, 28, bias_std=0.02, shared=S, shared_hidden=2 * d if S else None))
    m = m.to(device=DEV, dtype=torch.bfloat16).eval()
    h = reference_moe.make_input(n, d, 28, dtype=torch.bfloat16, device=DEV)
    x = reference_moe.make_input(n, d, 29, dtype=torch.bfloat16, device=DEV)
    with torch.no_grad():
        assert torch.equal(m.forward_residual(h, x), x + m(h))
        m.router_logits = "reference_gemm"
        assert torch.equal(m.forward_residual(h, x), x + m(h))
