"""Auxiliary router losses on the GPU: agm_moe_aux_forward/backward (through
``collect_moe_aux`` and the ops wrappers) against the reference's golden
vectors and against autograd through the oracle's restatement of
``_collect_moe_aux`` (agillm41.py:4463-4492) on the same GPU.

The kernels recompute the router logits with the router kernel (fp32
accumulation, one rounding to the router's dtype); a library GEMM may round
differently, so where argmax could flip on a one-rounding-step gap the oracle
takes the kernel's logit values (``scores_override``; its gradient still flows
through the reference's router Linear).

Tolerances: loss 1e-5 relative (fp32) / 1e-3 relative (16-bit logits);
router gradients 1e-4 relative plus 1e-4 of the largest magnitude (fp32),
2e-2 relative plus 1e-2 of the largest magnitude (16-bit). The sums over
tokens run in a different order than torch's.
"""
import math

import pytest
import torch

import agillm41_b200
from agillm41_b200 import ops, synthetic
from golden_io import GoldenAux, aux_names
from oracle import reference_moe

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _exact_fp32_matmul():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def assert_close(ours, ref, dtype, name):
    a, b = ours.float().cpu(), ref.float().cpu()
    assert a.shape == b.shape, (name, a.shape, b.shape)
    scale = float(b.abs().max().clamp_min(1e-30))
    rtol, atol = (1e-4, 1e-4 * scale) if dtype == torch.float32 else (2e-2, 1e-2 * scale)
    diff = (a - b).abs()
    bad = diff > atol + rtol * b.abs()
    assert not bool(bad.any()), f"{name}: {int(bad.sum())} of {b.numel()} beyond tolerance (max {diff.max():.3g})"


def assert_loss_close(ours, ref, dtype, name="loss"):
    a, b = float(ours.detach() if torch.is_tensor(ours) else ours), float(ref.detach() if torch.is_tensor(ref) else ref)
    tol = (1e-5 if dtype == torch.float32 else 1e-3) * abs(b) + 1e-8
    assert abs(a - b) <= tol, f"{name}: {a!r} vs {b!r}"


def kernel_scores(x, w):
    return ops.router_topk(x.contiguous(), w.contiguous(), 1, want_logits=True, tie_low_first=True)[3]


def ours(xs, ws, aux_coef, z_coef, upstream=1.0):
    """Loss and router gradients through the fused kernels (module order)."""
    total, leaves = None, []
    for x, w in zip(xs, ws):
        wl = w.detach().clone().requires_grad_(True)
        leaves.append(wl)
        loss = agillm41_b200.moe._MoEAuxNode.apply(wl, x, aux_coef, z_coef, None, True)
        total = loss if total is None else total + loss
    total.backward(torch.tensor(upstream, device=DEV))
    return total.detach(), [w.grad for w in leaves]


def oracle(xs, ws, aux_coef, z_coef, upstream=1.0, override=True):
    leaves = [w.detach().clone().requires_grad_(True) for w in ws]
    ov = [kernel_scores(x, w) for x, w in zip(xs, ws)] if override else None
    loss = reference_moe.collect_moe_aux(xs, leaves, aux_coef, z_coef, scores_override=ov)
    loss.backward(torch.tensor(upstream, device=DEV))
    return loss.detach(), [w.grad for w in leaves]


@pytest.mark.parametrize("name", aux_names())
def test_golden_vectors(name):
    """Against the reference's own CPU loss and gradients."""
    g = GoldenAux(name)
    xs = [x.to(DEV) for x in g.xs]
    ws = [w.to(DEV) for w in g.ws]
    loss, grads = ours(xs, ws, g.aux_coef, g.z_coef, g.upstream)
    assert loss.dtype == torch.float32
    assert_loss_close(loss, g.loss, g.dtype)
    for i, (a, b) in enumerate(zip(grads, g.d_router)):
        assert a.dtype == g.dtype
        assert_close(a, b, g.dtype, f"d_router{i}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("E,n,aux_coef,z_coef", [(14, 4096, 0.01, 0.001), (2, 3001, 0.01, 0.001),
                                                 (16, 777, 0.0, 0.01), (8, 1500, 0.05, 0.0)])
def test_against_oracle(dtype, E, n, aux_coef, z_coef):
    d = 1280
    w = synthetic.make_state(d, d, E, 70 + E, dtype=dtype, device=DEV)["router.weight"]
    x = synthetic.make_input(n, d, 70 + n, dtype=dtype, device=DEV)
    loss, grads = ours([x], [w], aux_coef, z_coef, upstream=3.0)
    ref_loss, ref_grads = oracle([x], [w], aux_coef, z_coef, upstream=3.0)
    assert_loss_close(loss, ref_loss, dtype)
    assert_close(grads[0], ref_grads[0], dtype, "d_router")


def test_full_size_fp32():
    """The 73,728-token, d = 1280, 14-expert workload with fp32 stashes (the
    autocast trainer's LayerNorm output and fp32 router weight)."""
    n, d, E = 73728, 1280, 14
    w = synthetic.make_state(d, d, E, 81, dtype=torch.float32, device=DEV)["router.weight"]
    x = synthetic.make_input(n, d, 81, dtype=torch.float32, device=DEV)
    loss, grads = ours([x], [w], 0.01, 0.001, upstream=65536.0)
    ref_loss, ref_grads = oracle([x], [w], 0.01, 0.001, upstream=65536.0)
    assert_loss_close(loss, ref_loss, torch.float32)
    assert_close(grads[0], ref_grads[0], torch.float32, "d_router")


def test_deterministic():
    n, d, E = 20000, 1280, 14
    w = synthetic.make_state(d, d, E, 82, dtype=torch.bfloat16, device=DEV)["router.weight"]
    x = synthetic.make_input(n, d, 82, dtype=torch.bfloat16, device=DEV)
    a = ours([x], [w], 0.01, 0.001)
    b = ours([x], [w], 0.01, 0.001)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1][0], b[1][0])


def test_no_tokens():
    """No stashed rows: NaN loss (torch's mean of nothing) and a zero gradient."""
    w = synthetic.make_state(64, 64, 4, 83, dtype=torch.float32, device=DEV)["router.weight"]
    x = torch.empty(0, 64, device=DEV)
    loss, grads = ours([x], [w], 0.01, 0.001)
    ref_loss = reference_moe.collect_moe_aux([x], [w], 0.01, 0.001)
    assert math.isnan(float(loss)) and math.isnan(float(ref_loss))
    assert torch.count_nonzero(grads[0]) == 0


def _two_module_model(dtype):
    torch.manual_seed(84)
    model = torch.nn.ModuleList([
        agillm41_b200.MoEFFN(256, mlp_mult=2, experts=14, top_k=2),
        agillm41_b200.MoEFFN(256, mlp_mult=4, experts=2, top_k=1, shared_experts=1, shared_mlp_mult=2),
    ]).to(DEV, dtype).train()
    return model


@pytest.mark.parametrize("amp", [False, True])
def test_collect_moe_aux_on_modules(amp):
    """The trainer's sequence: training forward (stashes the router input),
    then collect_moe_aux outside autocast (agillm41.py:6793-6798), the loss's
    router gradients against the oracle on the same stashes; every stash is
    cleared."""
    model = _two_module_model(torch.float32 if amp else torch.bfloat16)
    x = synthetic.make_input(3 * 700, 256, 85, dtype=torch.float32 if amp else torch.bfloat16,
                             device=DEV).reshape(3, 700, 256)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
        for m in model:
            m(x)
    stashes = [m.last_router_input.clone() for m in model]
    ws = [m.router.weight.detach() for m in model]
    loss = agillm41_b200.collect_moe_aux(model, 0.01, 0.001)
    assert all(m.last_router_input is None for m in model)
    assert torch.is_tensor(loss) and loss.dtype == torch.float32
    loss.backward()
    ref_loss, ref_grads = oracle(stashes, ws, 0.01, 0.001)
    dt = model[0].router.weight.dtype
    assert_loss_close(loss, ref_loss, dt)
    for m, g in zip(model, ref_grads):
        assert_close(m.router.weight.grad, g, dt, "router.weight.grad")


def test_collect_moe_aux_under_autocast():
    """Called inside torch.autocast, the router Linear runs in bf16 on casts
    of the fp32 stash and weight; the gradient comes back in fp32."""
    model = _two_module_model(torch.float32)
    x = synthetic.make_input(1000, 256, 86, dtype=torch.float32, device=DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        for m in model:
            m(x)
        stashes = [m.last_router_input.clone() for m in model]
        loss = agillm41_b200.collect_moe_aux(model, 0.01, 0.001)
        leaves = [m.router.weight.detach().clone().requires_grad_(True) for m in model]
        ov = [kernel_scores(s.to(torch.bfloat16), w.detach().to(torch.bfloat16)) for s, w in zip(stashes, leaves)]
        ref = reference_moe.collect_moe_aux(stashes, leaves, 0.01, 0.001, scores_override=ov)
    loss.backward()
    ref.backward()
    assert_loss_close(loss, ref, torch.bfloat16)
    for m, w in zip(model, leaves):
        assert m.router.weight.grad.dtype == torch.float32
        assert_close(m.router.weight.grad, w.grad, torch.bfloat16, "router.weight.grad")
