"""agm_moe_forward_noalloc: the forward for callers that cannot allocate.

Some hosts own all of the GPU's memory through their own pool and give a
plugin only its input and output buffers, or forbid any growth of the GPU
footprint once running; they cannot hand agm_moe_forward a workspace. The
no-allocation entry point uses scratch compiled into the library instead.
This test calls it through the C ABI twice in a row (the calls share that
scratch) and checks each result against the workspace-taking entry point on
the same inputs, with the bf16 parity check the other GPU tests use. It also
checks that a problem too large for the scratch is refused with a clear error.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from agillm41_b200 import _lib, ops, synthetic
from gpu_helpers import assert_close_rows

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
D, H, E, K = 1280, 3200, 14, 2


def _weights(seed):
    sd = synthetic.make_state(D, H, E, seed, dtype=torch.bfloat16, device=DEV, bias_std=0.02)
    w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).contiguous()
    b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).contiguous()
    w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).contiguous()
    b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).contiguous()
    return sd["router.weight"].contiguous(), w1, b1, w2, b2


def _noalloc(lib, x, wr, w1, b1, w2, b2, out):
    n = x.shape[0]
    return lib.agm_moe_forward_noalloc(x.data_ptr(), _lib.AGM_BF16, n, D, E, K, H, wr.data_ptr(), w1.data_ptr(),
                                       b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), 0, 1, None, None, None, None,
                                       out.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_forward_twice():
    lib = _lib.load()
    wr, w1, b1, w2, b2 = _weights(31)
    for call, n in enumerate((64, 700)):          # decode batch, then a larger one in the same scratch
        x = synthetic.make_input(n, D, 40 + call, dtype=torch.bfloat16, device=DEV)
        ref = ops.moe_forward(x, wr, w1, b1, w2, b2, K)
        out = torch.full_like(x, float("nan"))
        rc = _noalloc(lib, x, wr, w1, b1, w2, b2, out)
        assert rc == 0, lib.agm_last_error().decode()
        torch.cuda.synchronize()
        assert_close_rows(out, ref, torch.ones(n, dtype=torch.bool, device=DEV), torch.bfloat16)
        assert torch.equal(out, ref)  # same kernels on the same inputs: identical


def test_noalloc_rejects_oversize_problem():
    lib = _lib.load()
    wr, w1, b1, w2, b2 = _weights(32)
    n = 20000                                     # needs far more than AGM_NOALLOC_SCRATCH_BYTES
    need = lib.agm_moe_workspace_bytes(n, D, E, K, H, 0, 1, _lib.AGM_BF16)
    assert need > (32 << 20)
    x = torch.zeros(n, D, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros_like(x)
    rc = _noalloc(lib, x, wr, w1, b1, w2, b2, out)
    assert rc == -5
    msg = lib.agm_last_error().decode()
    assert "AGM_NOALLOC_SCRATCH_BYTES" in msg and str(need) in msg
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(out)) == 0    # nothing was launched
