"""LayerNorm at the Block boundary (agm_layernorm) and the Block's FFN half
in one call (agm_moe_block_forward: x + MoEFFN(LayerNorm(x)), agillm41.py:4547).

The LayerNorm is compared with the float64 LayerNorm of the same 16-bit
inputs: every output within one unit in the last place of the dtype, plus
the fp32 rounding of the terms (where the normalised value and the bias
nearly cancel) and the worst-case error of the fp32 mean, and at most 1e-3 of
them not the correctly rounded value; with torch's F.layer_norm on the same
GPU, at most 1e-2 of the elements differ (fp32: within 1e-5, relative +
absolute). The FFN half equals
the separate LayerNorm + agm_moe_forward_residual bit for bit, and against
the reference formula with torch's LayerNorm it is within the bf16 parity
tolerance on every row whose routing matches; rows routed differently must
have a LayerNorm output that differs from torch's.
"""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import agillm41_b200
from agillm41_b200 import ops, synthetic
from gpu_helpers import assert_close_rows, packed

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _ulp(v, dtype):
    bits = 7 if dtype == torch.bfloat16 else 10
    e = torch.floor(torch.log2(v.float().abs().clamp_min(2.0 ** -60)))
    return torch.pow(2.0, e - bits)


def _ln_params(d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    w = (1.0 + 0.2 * torch.randn(d, generator=g)).to(DEV, dtype)
    b = (0.2 * torch.randn(d, generator=g)).to(DEV, dtype)
    return w, b


@pytest.mark.parametrize("dtype,d,n", [(torch.bfloat16, 1280, 73728), (torch.bfloat16, 1280, 7),
                                       (torch.float16, 2048, 1000), (torch.bfloat16, 256, 333),
                                       (torch.float32, 1280, 4096), (torch.float32, 1536, 17)])
def test_layernorm_matches_torch(dtype, d, n):
    g = torch.Generator().manual_seed(n + d)
    x = (torch.randn(n, d, generator=g) * 3.0 + 0.5).to(DEV, dtype)
    w, b = _ln_params(d, dtype, d)
    ours = ops.layernorm(x, w, b, 1e-5)
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    torch.cuda.synchronize()
    if dtype == torch.float32:
        torch.testing.assert_close(ours, ref, rtol=1e-5, atol=1e-5)
        return
    # the LayerNorm of the same 16-bit values in float64, rounded once to the dtype
    xd = x.double()
    mean = xd.mean(dim=-1, keepdim=True)
    var = ((xd - mean) ** 2).mean(dim=-1, keepdim=True)
    std = torch.sqrt(var + 1e-5)
    scaled = (xd - mean) / std * w.double()
    exact64 = scaled + b.double()
    exact = exact64.to(dtype)
    d_ours = (ours.double() - exact64).abs()
    # One unit in the last place of the result, plus the fp32 rounding of the
    # terms (relative, where the normalised value and the bias nearly cancel),
    # plus the error of the fp32 mean, which is absolute: each lane sums d/32
    # values, then 5 butterfly adds and the multiply by 1/d, so |mean error| <=
    # (d/32 + 7) u mean|x| (u = 2^-24) and it reaches y scaled by |w| / std.
    mean_err = (d / 32 + 7) * 2.0 ** -24 * xd.abs().mean(dim=-1, keepdim=True)
    bound = (_ulp(exact64, dtype).double() * 1.001 + 4e-6 * (scaled.abs() + b.double().abs())
             + mean_err / std * w.double().abs())
    assert bool((d_ours <= bound).all()), float((d_ours - bound).max())
    assert float((ours != exact).float().mean()) <= 1e-3          # correctly rounded almost everywhere
    # agreement with torch's kernel (which reduces in another order)
    assert float((ours != ref).float().mean()) <= 1e-2


def test_layernorm_rejects_unsupported_width():
    x = torch.zeros(4, 4096, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(4096, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(agillm41_b200.MoEKernelError):
        ops.layernorm(x, w, w, 1e-5)


@pytest.mark.parametrize("E,k,S,n", [(14, 2, 0, 73728), (14, 2, 0, 3000), (2, 1, 1, 20000), (8, 3, 0, 64)])
def test_block_ffn_half(E, k, S, n):
    d, H = 1280, 3200 if E != 2 else 5120
    sd = synthetic.make_state(d, H, E, 80 + E, dtype=torch.bfloat16, device=DEV, bias_std=0.02, shared=S,
                              shared_hidden=2 * d if S else None)
    w1, b1, w2, b2, sh = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = (synthetic.make_input(n, d, 81 + E, dtype=torch.float32, device=DEV) * 2.0 + 0.3).to(torch.bfloat16)
    lw, lb = _ln_params(d, torch.bfloat16, 82)
    out = ops.moe_block_forward(x, lw, lb, 1e-5, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    # the same kernels in two calls: identical
    ln = ops.layernorm(x, lw, lb, 1e-5)
    sep = ops.moe_forward_residual(ln, x, wr, w1, b1, w2, b2, k, shared=sh, check_errors=True)
    assert torch.equal(out, sep)
    # against torch's LayerNorm: parity on the rows routed alike
    ln_ref = F.layer_norm(x, (d,), lw, lb, 1e-5)
    ref = ops.moe_forward_residual(ln_ref, x, wr, w1, b1, w2, b2, k, shared=sh)
    _, ex_o = ops.moe_forward(ln, wr, w1, b1, w2, b2, k, shared=sh, want=("idx",))
    _, ex_r = ops.moe_forward(ln_ref, wr, w1, b1, w2, b2, k, shared=sh, want=("idx",))
    same = (ex_o["idx"] == ex_r["idx"]).all(dim=1)
    ln_differs = (ln != ln_ref).any(dim=1)
    assert bool((same | ln_differs).all()), "a routing difference without a LayerNorm difference"
    assert_close_rows(out, ref, same, torch.bfloat16)


def test_module_forward_block_inference_and_training():
    d, H, E, k, n = 1280, 3200, 14, 2, 2048
    sd = synthetic.make_state(d, H, E, 90, dtype=torch.bfloat16, bias_std=0.02)
    m = agillm41_b200.MoEFFN(d, mlp_mult=4, experts=E, top_k=k)
    m.experts = nn.ModuleList([nn.Sequential(nn.Linear(d, H), nn.ReLU(), nn.Linear(H, d)) for _ in range(E)])
    m.load_state_dict(sd)
    m = m.to(device=DEV, dtype=torch.bfloat16).eval()
    ln = nn.LayerNorm(d).to(device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        ln.weight.copy_(_ln_params(d, torch.bfloat16, 91)[0])
        ln.bias.copy_(_ln_params(d, torch.bfloat16, 91)[1])
    x = synthetic.make_input(n, d, 92, dtype=torch.bfloat16, device=DEV).reshape(2, n // 2, d)
    with torch.no_grad():
        fused = m.forward_block(x, ln)
        sep = m.forward_residual(ops.layernorm(x.reshape(n, d), ln.weight, ln.bias, ln.eps).reshape(x.shape), x)
    assert torch.equal(fused, sep)
    # with gradients the module keeps torch's LayerNorm (training path)
    m.train()
    xg = x.clone().requires_grad_(True)
    y = m.forward_block(xg, ln)
    y2 = m.forward_residual(ln(xg), xg)
    assert torch.equal(y, y2)
