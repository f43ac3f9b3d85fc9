"""The decode front: router, dispatch plan and permute of at most one 128-token
dispatch block as one cluster kernel (agm_moe_forward's default for
decode-sized batches; AGM_FLAG_NO_FRONT gives the three separate kernels).

Its router logits are fp32 dot products summed on the CUDA cores and rounded
once to the activation dtype (the reference's `router(x).float()`,
agillm41.py:4398-4399), checked against float64 dot products with the same
bound as the other router tests. Given those logits, everything else must
equal the three-kernel path fed the same logits through logits_in bit for
bit: expert indices, gates, counts and the forward output (same selection,
plan, permutation, expert GEMMs and combine), with the swapped-operand GEMMs
(padding rows not zero-filled) and with the row-tile GEMMs (padding rows
zero-filled), with either tie order.
"""
import pytest
import torch

from agillm41_b200 import ops, synthetic
from gpu_helpers import packed

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _ulp(v, dtype):
    bits = 7 if dtype == torch.bfloat16 else 10
    e = torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -60)))
    return torch.pow(2.0, e - bits)


CASES = [
    # dtype, n, d, H, E, k
    (torch.bfloat16, 64, 1280, 3200, 14, 2),    # the decode workload
    (torch.bfloat16, 1, 1280, 3200, 14, 2),
    (torch.bfloat16, 128, 1280, 3200, 14, 2),   # one full dispatch block
    (torch.float16, 37, 256, 512, 6, 3),
    (torch.bfloat16, 100, 2048, 512, 16, 4),    # widest supported row, 16 experts
    (torch.bfloat16, 20, 1280, 5120, 2, 1),     # production expert count, top-1
    (torch.bfloat16, 50, 512, 512, 8, 6),       # top-k beyond the specialised kernels
]


@pytest.mark.parametrize("dtype,n,d,H,E,k", CASES)
@pytest.mark.parametrize("swap", [True, False])
def test_front_matches_three_kernels_on_its_logits(dtype, n, d, H, E, k, swap):
    sd = synthetic.make_state(d, H, E, 500 + n + E, dtype=dtype, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(n, d, 600 + n, dtype=dtype, device=DEV)
    want = ("idx", "gates", "counts", "logits")
    out, ex = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=want, swap=swap, check_errors=True)
    # logits: fp32 accumulation, one rounding
    exact = x.double() @ wr.double().T
    rounded = exact.to(dtype).double()
    mag = x.double().abs() @ wr.double().abs().T
    lg = ex["logits"].double()
    assert bool(((lg - rounded).abs() <= _ulp(rounded, dtype) + 1e-6 * mag).all())
    assert int((lg != rounded).sum()) <= max(2, lg.numel() // 100)
    # the three-kernel path on the same logits
    out_r, ex_r = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=want, swap=swap, front=False,
                                  logits_in=ex["logits"], check_errors=True)
    for key in ("idx", "gates", "counts"):
        assert torch.equal(ex[key], ex_r[key]), key
    assert torch.equal(out, out_r)
    assert int(ex["counts"].sum()) == n * k


def test_front_tie_order_and_repeatability():
    dtype, n, d, H, E, k = torch.bfloat16, 64, 256, 256, 8, 2
    sd = synthetic.make_state(d, H, E, 77, dtype=dtype, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    # duplicated router rows: every token sees exactly tied logits between experts 2 and 5
    wr = sd["router.weight"].clone()
    wr[5] = wr[2]
    x = synthetic.make_input(n, d, 78, dtype=dtype, device=DEV)
    for low_first in (False, True):
        out, ex = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "logits"), tie_low_first=low_first,
                                  check_errors=True)
        out2, ex2 = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx", "logits"), tie_low_first=low_first)
        assert torch.equal(out, out2) and torch.equal(ex["idx"], ex2["idx"])
        out_r, ex_r = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("idx",), tie_low_first=low_first, front=False,
                                      logits_in=ex["logits"])
        assert torch.equal(ex["idx"], ex_r["idx"]) and torch.equal(out, out_r)


def test_front_residual_and_caller_logits():
    """The residual entry point takes the front too; caller-supplied logits keep the three kernels."""
    dtype, n, d, H, E, k = torch.bfloat16, 64, 1280, 3200, 14, 2
    sd = synthetic.make_state(d, H, E, 88, dtype=dtype, device=DEV, bias_std=0.02)
    w1, b1, w2, b2, _ = packed(sd, E, DEV)
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(n, d, 89, dtype=dtype, device=DEV)
    res = synthetic.make_input(n, d, 90, dtype=dtype, device=DEV)
    out = ops.moe_forward(x, wr, w1, b1, w2, b2, k)
    fused = ops.moe_forward_residual(x, res, wr, w1, b1, w2, b2, k, check_errors=True)
    assert torch.equal(fused, out + res)
    # caller-supplied logits route through the three kernels: the same result on the front's own logits
    _, ex = ops.moe_forward(x, wr, w1, b1, w2, b2, k, want=("logits",))
    assert torch.equal(ops.moe_forward(x, wr, w1, b1, w2, b2, k, logits_in=ex["logits"]), out)
