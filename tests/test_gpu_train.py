"""Training parity: the MoE block's autograd node (agm_moe_forward_train +
agm_moe_backward) against autograd through the reference's op sequence.

The comparator is the oracle (oracle/reference_moe.py, pinned bit for bit to
the reference's forward and backward by tests/test_oracle_grads.py) run with
torch autograd on the same GPU, in the same precision mode:

* one dtype throughout (bf16, fp16, fp32), as a model converted to that dtype;
* torch.autocast(bf16) over fp32 master weights with an fp32 input, as the
  reference trains with --amp (agillm41.py:3054-3066, 6793).

Routing: the router kernel accumulates its logits in fp32 and rounds once,
the library GEMM may round partial sums, so a token whose top-k gap is one
rounding step can pick another expert. The oracle therefore routes with the
kernel's logit values (``logits_override``), while its gradients still flow
through the reference's router Linear; the index lists are then identical
and every gradient is comparable.

Tolerances (written per comparison below): fp32 mode 1e-4 relative plus 1e-4
of the tensor's largest magnitude; bf16/fp16 2e-2 relative plus 1e-2 of the
tensor's largest magnitude, and a whole-tensor relative error under 1e-2.
Gradients are sums over many rows whose accumulation order differs between
any two implementations, and in 16-bit modes the reference rounds partial
results (per rank, per expert call) that the fused kernels keep in fp32.
"""
import pytest
import torch
import torch.nn as nn
import torch.utils.checkpoint as ckpt

import agillm41_b200
from agillm41_b200 import ops, synthetic
from golden_io import GoldenGrad, grad_names
from gpu_helpers import packed
from oracle import reference_moe

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def assert_grad_close(ours, ref, dtype, name):
    assert ours is not None, f"{name}: no gradient"
    assert ours.shape == ref.shape and ours.dtype == ref.dtype, (name, ours.shape, ref.shape, ours.dtype, ref.dtype)
    a, b = ours.float(), ref.float()
    scale = float(b.abs().max().clamp_min(1e-30))
    if dtype == torch.float32:
        rtol, atol, rel_max = 1e-4, 1e-4 * scale, 1e-5
    else:
        rtol, atol, rel_max = 2e-2, 1e-2 * scale, 1e-2
    diff = (a - b).abs()
    bad = diff > atol + rtol * b.abs()
    assert not bool(bad.any()), (f"{name}: {int(bad.sum())} of {b.numel()} elements beyond tolerance "
                                 f"(max diff {diff.max().item():.4g}, scale {scale:.4g})")
    rel = float((a - b).norm() / b.norm().clamp_min(1e-30))
    assert rel < rel_max, f"{name}: relative error {rel:.3g}"


def make_module(sd, d, H, E, k, dtype):
    S = reference_moe.num_shared_in(sd)
    Hs = sd["shared.0.0.weight"].shape[0] if S else 0
    m = agillm41_b200.MoEFFN(d, mlp_mult=max(1, H // d), experts=E, top_k=k, shared_experts=S,
                             shared_mlp_mult=max(1, Hs // d) if S else 0)
    if H != m.mlp_mult * d:
        m.experts = nn.ModuleList([nn.Sequential(nn.Linear(d, H), nn.ReLU(), nn.Linear(H, d)) for _ in range(E)])
    if S and m.shared[0][0].weight.shape[0] != Hs:
        m.shared = nn.ModuleList([nn.Sequential(nn.Linear(d, Hs), nn.ReLU(), nn.Linear(Hs, d)) for _ in range(S)])
    m.load_state_dict({kk: v.float() for kk, v in sd.items()})
    m = m.to(device=DEV, dtype=dtype).train()
    m.check_device_errors = True
    return m


def kernel_logits(x, sd, k, compute_dtype):
    """The router kernel's fp32 logits for x (cast to the compute dtype)."""
    E = sd["router.weight"].shape[0]
    sdc = {kk: v.to(DEV, compute_dtype) for kk, v in sd.items()}
    w1, b1, w2, b2, _ = packed(sdc, E, DEV)
    with torch.no_grad():
        _, ex = ops.moe_forward(x.to(DEV, compute_dtype).contiguous(), sdc["router.weight"].contiguous(), w1, b1,
                                w2, b2, k, want=("logits", "counts"), check_errors=True)
    return ex["logits"], ex["counts"]


def run_pair(sd, x, dout, k, dtype, amp=None):
    """(ours, oracle): each a dict with 'out', 'dx' and the state-dict gradients."""
    E = sd["router.weight"].shape[0]
    d = x.shape[1]
    H = sd["experts.0.0.weight"].shape[0]
    master = torch.float32 if amp else dtype
    compute = amp or dtype
    logits, counts = kernel_logits(x, sd, k, compute)

    m = make_module(sd, d, H, E, k, master)
    xo = x.to(DEV, master).clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=amp, enabled=amp is not None):
        y = m(xo.reshape(2, -1, d))
    y.reshape(-1, d).backward(dout.to(DEV, master))
    ours = {"out": y.detach().reshape(-1, d), "dx": xo.grad}
    ours.update({kk: p.grad for kk, p in m.named_parameters()})

    sdl = {kk: v.to(DEV, master).clone().requires_grad_(True) for kk, v in sd.items()}
    xr = x.to(DEV, master).clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=amp, enabled=amp is not None):
        yr = reference_moe.moe_forward(xr, sdl, k, logits_override=logits)
    yr.backward(dout.to(DEV, master))
    ref = {"out": yr.detach(), "dx": xr.grad}
    ref.update({kk: v.grad for kk, v in sdl.items()})
    return ours, ref, counts


def compare(ours, ref, dtype, counts=None):
    for key, r in ref.items():
        o = ours[key]
        if r is None:
            # The reference never called this expert: no gradient at all.
            assert o is None, f"{key}: expected no gradient"
            e = int(key.split(".")[1])
            assert counts is not None and int(counts[e]) == 0
            continue
        assert_grad_close(o, r, dtype, key)


def case(d, H, E, k, n, seed, bias_std=0.02, shared=0, shared_hidden=None):
    sd = synthetic.make_state(d, H, E, seed, dtype=torch.float32, bias_std=bias_std, shared=shared,
                              shared_hidden=shared_hidden)
    x = synthetic.make_input(n, d, seed)
    g = torch.Generator().manual_seed(seed + 7)
    dout = torch.randn(n, d, generator=g)
    return sd, x, dout


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [1, 2])
def test_same_dtype_matches_reference_autograd(dtype, k):
    sd, x, dout = case(256, 512, 14, k, 512, 51 + k)
    ours, ref, counts = run_pair(sd, x, dout, k, dtype)
    compare(ours, ref, dtype, counts)


@pytest.mark.parametrize("k", [1, 2])
def test_autocast_over_fp32_weights_matches_reference_autograd(k):
    sd, x, dout = case(256, 512, 14, k, 512, 61 + k)
    ours, ref, counts = run_pair(sd, x, dout, k, torch.float32, amp=torch.bfloat16)
    assert ours["out"].dtype == torch.float32 and ours["dx"].dtype == torch.float32
    compare(ours, ref, torch.bfloat16, counts)


def test_top3_four_experts():
    sd, x, dout = case(128, 256, 4, 3, 300, 71, bias_std=0.1)
    ours, ref, counts = run_pair(sd, x, dout, 3, torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


@pytest.mark.parametrize("empty_grad", ["none", "zero"])
def test_experts_without_rows(empty_grad):
    """Experts 1 and 4 receive no token: no gradient (or zeros on request)."""
    d, H, E, k, n = 128, 256, 6, 2, 200
    sd = synthetic.make_state(d, H, E, 81, dtype=torch.float32, bias_std=0.05)
    w = sd["router.weight"]
    for e in range(E):
        w[e] = -w[e].abs() - 0.05 if e in (1, 4) else w[e].abs() + 0.01
    x = synthetic.make_input(n, d, 81).abs() + 0.01
    dout = torch.randn(n, d, generator=torch.Generator().manual_seed(82))
    if empty_grad == "none":
        ours, ref, counts = run_pair(sd, x, dout, k, torch.bfloat16)
        assert int(counts[1]) == 0 and int(counts[4]) == 0
        compare(ours, ref, torch.bfloat16, counts)
        return
    m = make_module(sd, d, H, E, k, torch.bfloat16)
    m.empty_expert_grad = "zero"
    xo = x.to(DEV, torch.bfloat16).requires_grad_(True)
    m(xo).backward(dout.to(DEV, torch.bfloat16))
    for e in (1, 4):
        for p in m.experts[e].parameters():
            assert p.grad is not None and int(torch.count_nonzero(p.grad)) == 0
    assert int(torch.count_nonzero(m.experts[0][0].weight.grad)) > 0


def test_full_width_autocast():
    """d=1280, H=3200, 14 experts, top-2 (the block's production shape)."""
    sd, x, dout = case(1280, 3200, 14, 2, 1024, 91)
    ours, ref, counts = run_pair(sd, x, dout, 2, torch.float32, amp=torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


def test_cta_pair_segments_autocast():
    """k*N >= 16,384: the forward's GEMMs run on CTA pairs and expert segments
    are padded to 256 rows; the backward reads that layout."""
    sd, x, dout = case(1280, 3200, 14, 2, 8192, 93)
    ours, ref, counts = run_pair(sd, x, dout, 2, torch.float32, amp=torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


@pytest.mark.parametrize("name", [n for n in grad_names() if "fp32" in n])
def test_fp32_gradients_match_reference_golden(name):
    """fp32 mode against the reference's own CPU gradients (no oracle)."""
    g = GoldenGrad(name)
    m = make_module(g.sd, g.d, g.H, g.E, g.top_k, torch.float32)
    logits, counts = kernel_logits(g.x, g.sd, g.top_k, torch.float32)
    ref_idx = g.idx
    our_idx = logits.topk(g.top_k, dim=-1).indices.cpu() if g.top_k > 1 else logits.argmax(-1, keepdim=True).cpu()
    assert torch.equal(our_idx, ref_idx), "routing differs from the reference's"
    x = g.x.to(DEV).clone().requires_grad_(True)
    y = m(x)
    y.backward(g.dout.to(DEV))
    torch.testing.assert_close(y.detach().cpu(), g.out, rtol=1e-4, atol=1e-4)
    assert_grad_close(x.grad.cpu(), g.dx, torch.float32, "dx")
    ref = g.grads()
    for key, p in m.named_parameters():
        e = int(key.split(".")[1]) if key.startswith("experts.") else None
        if e is not None and not g.expert_has_grad[e]:
            assert p.grad is None, key
            continue
        assert_grad_close(p.grad.cpu(), ref[key], torch.float32, key)


def _ops_grads(sd, x, dout, k, amp, fwd_pair, bwd_pair, bwd_always):
    E = sd["router.weight"].shape[0]
    compute = torch.bfloat16
    sdc = {kk: v.to(DEV, compute) for kk, v in sd.items()}
    w1, b1, w2, b2, shared = packed(sdc, E, DEV)
    wr = sdc["router.weight"].contiguous()
    xin = x.to(DEV, torch.float32 if amp else compute).contiguous()
    gout = dout.to(DEV, xin.dtype).contiguous()
    out, saved = ops.moe_forward_train(xin, wr, w1, b1, w2, b2, k, shared=shared, pair=fwd_pair, check_errors=True)
    res = ops.moe_backward(gout, saved, wr, w1, w2, k, shared=shared, pair=bwd_pair, pair_always=bwd_always,
                           check_errors=True)
    flat = [out] + list(res[:6]) + (list(res[6]) if shared is not None else [])
    return flat


@pytest.mark.parametrize("shape", ["full_width_8192", "ragged_shared", "production_16500"])
@pytest.mark.parametrize("amp", [False, True])
def test_cta_pair_backward_matches_one_cta(shape, amp):
    """The CTA-pair backward GEMMs (256 x 256 tiles on two SMs) give the same
    bits as the one-CTA kernels: odd row-tile counts, a ragged last column
    tile, experts without rows and a shared expert included."""
    if shape == "full_width_8192":
        sd, x, dout = case(1280, 3200, 14, 2, 8192, 161)
        k = 2
    elif shape == "production_16500":
        # Above the pair threshold the shared expert's dense GEMMs run on CTA
        # pairs too: 129 row tiles, so the last pair holds one tile.
        sd, x, dout = case(1280, 5120, 2, 1, 16500, 164, shared=1, shared_hidden=2560)
        k = 1
    else:
        d, H, E, k, n = 256, 320, 6, 2, 300
        sd = synthetic.make_state(d, H, E, 162, dtype=torch.float32, bias_std=0.05, shared=1, shared_hidden=192)
        w = sd["router.weight"]
        for e in range(E):
            w[e] = -w[e].abs() - 0.05 if e in (1, 4) else w[e].abs() + 0.01
        x = synthetic.make_input(n, d, 162).abs() + 0.01
        dout = torch.randn(n, d, generator=torch.Generator().manual_seed(163))
    one_cta = _ops_grads(sd, x, dout, k, amp, fwd_pair=False, bwd_pair=False, bwd_always=False)
    pairs = _ops_grads(sd, x, dout, k, amp, fwd_pair=True, bwd_pair=True, bwd_always=True)
    for i, (a, b) in enumerate(zip(one_cta, pairs)):
        assert torch.equal(a, b), f"output {i} differs"


def test_backward_is_deterministic():
    sd, x, dout = case(256, 512, 14, 2, 700, 101)
    grads = []
    for _ in range(2):
        m = make_module(sd, 256, 512, 14, 2, torch.bfloat16)
        xo = x.to(DEV, torch.bfloat16).requires_grad_(True)
        m(xo).backward(dout.to(DEV, torch.bfloat16))
        grads.append([xo.grad] + [p.grad for p in m.parameters()])
    for a, b in zip(*grads):
        assert torch.equal(a, b)


def test_activation_checkpointing_gives_identical_gradients():
    """Non-reentrant checkpointing (agillm41.py:1202, 4662) drops the saved
    state and recomputes the forward in the backward: same gradients."""
    sd, x, dout = case(256, 512, 14, 2, 400, 111)
    res = []
    for use_ckpt in (False, True):
        m = make_module(sd, 256, 512, 14, 2, torch.float32)
        xo = x.to(DEV).requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = ckpt.checkpoint(m, xo, use_reentrant=False) if use_ckpt else m(xo)
        y.backward(dout.to(DEV))
        res.append([xo.grad] + [p.grad for p in m.parameters()])
    for a, b in zip(*res):
        assert torch.equal(a, b)


def test_optimizer_step_reaches_the_kernels():
    """After an optimiser step on the module's parameters the next forward
    uses the updated weights (the packed weights and their 16-bit casts
    follow the parameters): its output equals that of a fresh module loaded
    with the updated state dict."""
    sd, x, dout = case(256, 512, 14, 2, 512, 121)
    m = make_module(sd, 256, 512, 14, 2, torch.float32)
    opt = torch.optim.SGD(m.parameters(), lr=0.5)
    xo = x.to(DEV)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y0 = m(xo)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(xo)
    y.backward(dout.to(DEV))
    opt.step()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y1 = m(xo)
    fresh = make_module({kk: v.detach().cpu() for kk, v in m.state_dict().items()}, 256, 512, 14, 2, torch.float32)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = fresh(xo)
    assert not torch.equal(y0, y1)
    assert torch.equal(y1, y2)


def test_inference_under_autocast_matches_reference():
    sd, x, _ = case(256, 512, 14, 2, 256, 131)
    m = make_module(sd, 256, 512, 14, 2, torch.float32).eval()
    logits, _ = kernel_logits(x, sd, 2, torch.bfloat16)
    sdd = {kk: v.to(DEV) for kk, v in sd.items()}
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x.to(DEV))
        yr = reference_moe.moe_forward(x.to(DEV), sdd, 2, logits_override=logits)
    assert y.dtype == torch.float32
    assert_grad_close(y, yr, torch.bfloat16, "out")


def test_shared_expert_production_shape_autocast():
    """The production MoE of AGILLM4.1: 2 experts, top-1, one shared expert of
    hidden 2d (agillm41.py:8590-8591), under autocast over fp32 weights."""
    sd, x, dout = case(256, 1024, 2, 1, 512, 141, shared=1, shared_hidden=512)
    ours, ref, counts = run_pair(sd, x, dout, 1, torch.float32, amp=torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_two_shared_experts_top2(dtype):
    sd, x, dout = case(256, 512, 6, 2, 400, 151, shared=2, shared_hidden=256)
    ours, ref, counts = run_pair(sd, x, dout, 2, dtype)
    compare(ours, ref, dtype, counts)


def test_cpu_input_is_refused():
    m2 = agillm41_b200.MoEFFN(64, mlp_mult=2, experts=4, top_k=2).train()
    with pytest.raises(agillm41_b200.MoEKernelError):
        m2(torch.randn(8, 64, requires_grad=True))


def test_top5_generic_width():
    """top_k above 4 takes the kernels' generic (16-wide) variant."""
    sd, x, dout = case(128, 256, 8, 5, 160, 171, bias_std=0.1)
    ours, ref, counts = run_pair(sd, x, dout, 5, torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


def test_autocast_fp16():
    sd, x, dout = case(256, 512, 14, 2, 512, 181)
    ours, ref, counts = run_pair(sd, x, dout, 2, torch.float32, amp=torch.float16)
    compare(ours, ref, torch.float16, counts)


def test_full_size_bench_workload_autocast():
    """The bench's 73,728-token workload (B=48 x L=1536, d=1280, H=3200,
    14 experts, top-2) under autocast: CTA-pair GEMMs forward and backward."""
    sd, x, dout = case(1280, 3200, 14, 2, 73728, 191)
    ours, ref, counts = run_pair(sd, x, dout, 2, torch.float32, amp=torch.bfloat16)
    compare(ours, ref, torch.bfloat16, counts)


@pytest.mark.parametrize("amp", [None, torch.bfloat16])
def test_forward_residual_training_equals_separate_add(amp):
    """The fused residual (Block's `x + ff(ln2(x))`) gives the same output and
    gradients, bit for bit, as the MoE block followed by a separate add."""
    sd, x, dout = case(256, 512, 14, 2, 512, 201, shared=1, shared_hidden=256)
    master = torch.float32 if amp else torch.bfloat16
    res_in = synthetic.make_input(512, 256, 202)
    outs = []
    for fused in (False, True):
        m = make_module(sd, 256, 512, 14, 2, master)
        h = x.to(DEV, master).clone().requires_grad_(True)
        r = res_in.to(DEV, master).clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=amp or torch.bfloat16, enabled=amp is not None):
            y = m.forward_residual(h, r) if fused else r + m(h)
        y.backward(dout.to(DEV, master))
        outs.append([y.detach(), h.grad, r.grad] + [p.grad for p in m.parameters()])
    for a, b in zip(*outs):
        assert torch.equal(a, b)
