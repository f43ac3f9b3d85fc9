"""The oracle's backward is pinned to the reference's: autograd through the
torch restatement (oracle/reference_moe.py) on CPU reproduces the gradients
that the reference MoEFFN gave in training mode (tests/golden/grad_*.npz,
written by tests/golden/make_golden_grads.py from the reference itself)."""
import pytest
import torch

from golden_io import GoldenGrad, grad_names
from oracle import reference_moe


def oracle_grads(g, sd=None, detach_gates=False):
    sd = {k: v.clone().requires_grad_(True) for k, v in (sd or g.sd).items()}
    x = g.x.clone().requires_grad_(True)
    out = reference_moe.moe_forward(x, sd, g.top_k)
    out.backward(g.dout)
    return out.detach(), x.grad, {k: v.grad for k, v in sd.items()}


def test_grad_cases_exist():
    names = grad_names()
    assert len(names) >= 6
    dts = {GoldenGrad(n).dtype for n in names}
    assert torch.float32 in dts and torch.bfloat16 in dts
    ks = {GoldenGrad(n).top_k for n in names}
    assert {1, 2, 3} <= ks


@pytest.mark.parametrize("name", grad_names())
def test_grad_inputs_regenerate(name):
    assert GoldenGrad(name).inputs_match()


@pytest.mark.parametrize("name", grad_names())
def test_oracle_backward_reproduces_reference(name):
    g = GoldenGrad(name)
    out, dx, grads = oracle_grads(g)
    assert torch.equal(out, g.out)
    # Same torch ops on the same CPU kernels as when the vectors were made.
    tol = dict(rtol=1e-6, atol=1e-6) if g.dtype == torch.float32 else dict(rtol=0, atol=0)
    torch.testing.assert_close(dx, g.dx, **tol)
    ref = g.grads()
    for key, gr in grads.items():
        e = int(key.split(".")[1]) if key.startswith("experts.") else None
        if e is not None and not g.expert_has_grad[e]:
            assert gr is None, key          # never called: no gradient at all
            continue
        torch.testing.assert_close(gr, ref[key], **tol, msg=key)


def test_empty_experts_have_no_gradient():
    g = GoldenGrad("grad_empty_fp32_n16")
    assert g.expert_has_grad.count(False) == 2
    assert [int(c) for c in g.counts if int(c) == 0] == [0, 0]


@pytest.mark.parametrize("name", ["grad_top2_fp32_n24", "grad_top3_fp32_n16"])
def test_planted_oracle_mistake_is_caught(name):
    """An oracle whose gates carry no gradient (a detached softmax, a common
    slip) must not reproduce the reference's router-weight gradient."""
    g = GoldenGrad(name)
    sd = {k: v.clone().requires_grad_(True) for k, v in g.sd.items()}
    flat = g.x.clone().requires_grad_(True)
    scores = torch.nn.functional.linear(flat, sd["router.weight"]).float()
    vals, idx = torch.topk(scores, g.top_k, dim=-1)
    w = vals.softmax(-1).detach().to(flat.dtype)                     # planted mistake
    out = torch.zeros_like(flat)
    for r in range(g.top_k):
        for e in range(g.E):
            rows = (idx[:, r] == e).nonzero().flatten()
            if rows.numel():
                y = reference_moe._expert(sd, f"experts.{e}.", flat.index_select(0, rows))
                out.index_add_(0, rows, y * w[rows, r:r + 1])
    out.backward(g.dout)
    assert sd["router.weight"].grad is None or not torch.allclose(sd["router.weight"].grad, g.d_router)
    assert not torch.allclose(flat.grad, g.dx, rtol=1e-4, atol=1e-5)
