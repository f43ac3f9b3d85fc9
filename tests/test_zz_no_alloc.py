"""agm_moe_forward_noalloc: the forward for callers that cannot allocate.

Some hosts own all of the GPU's memory through their own pool and give a
plugin only its input and output buffers, or forbid any growth of the GPU
footprint once running; they cannot hand agm_moe_forward a workspace. The
no-allocation entry point uses scratch compiled into the library instead.
This test calls it through the C ABI twice in a row (the calls share that
scratch) and checks each result against the workspace-taking entry point on
the same inputs, with the bf16 parity check the other GPU tests use, and
reads the device error word through agm_moe_noalloc_error_word after each
call. It also covers a call with a shared expert (more scratch per token),
the largest token count that fits the scratch exactly, and the refusal of
one token more.

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
HS = 2 * D                     # hidden of the shared expert in the shared-expert case
SCRATCH = 32 << 20             # AGM_NOALLOC_SCRATCH_BYTES


def _weights(seed, shared=0):
    sd = synthetic.make_state(D, H, E, seed, dtype=torch.bfloat16, device=DEV, bias_std=0.02, shared=shared,
                              shared_hidden=HS if shared else None)
    w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).contiguous()
    b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).contiguous()
    w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).contiguous()
    b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).contiguous()
    sh = None
    if shared:
        sh = tuple(torch.stack([sd[f"shared.{s}.{i}.{p}"] for s in range(shared)]).contiguous()
                   for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")))
    return sd["router.weight"].contiguous(), w1, b1, w2, b2, sh


def _noalloc(lib, x, wr, w1, b1, w2, b2, out, sh=None, flags=0):
    n = x.shape[0]
    n_sh, hs = (0, 1) if sh is None else (sh[0].shape[0], sh[0].shape[1])
    sp = [None] * 4 if sh is None else [t.data_ptr() for t in sh]
    return lib.agm_moe_forward_noalloc(x.data_ptr(), _lib.AGM_BF16, n, D, E, K, H, wr.data_ptr(), w1.data_ptr(),
                                       b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), n_sh, hs, *sp, out.data_ptr(),
                                       flags, torch.cuda.current_stream().cuda_stream)


def _error_word(lib):
    """Read (and reset) the no-allocation forward's device error word."""
    err = ctypes.c_void_p()
    rc = lib.agm_moe_noalloc_error_word(ctypes.byref(err))
    assert rc == 0, lib.agm_last_error().decode()
    assert err.value
    code = ctypes.c_int(-1)
    rc = lib.agm_read_device_error(err, ctypes.byref(code), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code.value >= 0
    assert (rc == 0) == (code.value == 0), lib.agm_last_error().decode()
    return code.value


def _check(lib, n, seed, sh_count=0, flags=0):
    wr, w1, b1, w2, b2, sh = _weights(seed, sh_count)
    x = synthetic.make_input(n, D, seed + 9, dtype=torch.bfloat16, device=DEV)
    ref = ops.moe_forward(x, wr, w1, b1, w2, b2, K, shared=sh)
    out = torch.full_like(x, float("nan"))
    rc = _noalloc(lib, x, wr, w1, b1, w2, b2, out, sh, flags)
    assert rc == 0, lib.agm_last_error().decode()
    assert _error_word(lib) == 0
    torch.cuda.synchronize()
    assert_close_rows(out, ref, torch.ones(n, dtype=torch.bool, device=DEV), torch.bfloat16)
    assert torch.equal(out, ref)  # same kernels on the same inputs: identical


def test_noalloc_matches_workspace_forward_twice():
    lib = _lib.load()
    for call, n in enumerate((64, 700)):          # decode batch, then a larger one in the same scratch
        _check(lib, n, 31 + call)


def test_noalloc_shared_expert_and_keep_error_flag():
    # One shared expert of hidden 2d (the production shape's): the scratch
    # holds its hidden rows too. AGM_FLAG_KEEP_ERROR is ignored by this entry
    # point (the shared error word is always cleared first).
    lib = _lib.load()
    _check(lib, 300, 41, sh_count=1, flags=_lib.AGM_FLAG_KEEP_ERROR)


def _largest_fitting(lib, n_shared, hs):
    best = 0
    for n in range(1, 4096):
        if lib.agm_moe_workspace_bytes(n, D, E, K, H, n_shared, hs, _lib.AGM_BF16) <= SCRATCH:
            best = n
    return best


def test_noalloc_at_the_scratch_limit():
    lib = _lib.load()
    n = _largest_fitting(lib, 0, 1)
    assert lib.agm_moe_workspace_bytes(n, D, E, K, H, 0, 1, _lib.AGM_BF16) <= SCRATCH
    assert lib.agm_moe_workspace_bytes(n + 1, D, E, K, H, 0, 1, _lib.AGM_BF16) > SCRATCH
    _check(lib, n, 51)
    # one token more: refused with AGM_ERR_WORKSPACE, nothing launched
    wr, w1, b1, w2, b2, _ = _weights(52)
    x = torch.zeros(n + 1, D, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros_like(x)
    rc = _noalloc(lib, x, wr, w1, b1, w2, b2, out)
    assert rc == -5
    assert "AGM_NOALLOC_SCRATCH_BYTES" in lib.agm_last_error().decode()
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(out)) == 0


def test_noalloc_rejects_oversize_problem():
    lib = _lib.load()
    wr, w1, b1, w2, b2, _ = _weights(32)
    n = 20000                                     # needs far more than AGM_NOALLOC_SCRATCH_BYTES
    need = lib.agm_moe_workspace_bytes(n, D, E, K, H, 0, 1, _lib.AGM_BF16)
    assert need > SCRATCH
    x = torch.zeros(n, D, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros_like(x)
    rc = _noalloc(lib, x, wr, w1, b1, w2, b2, out)
    assert rc == -5
    msg = lib.agm_last_error().decode()
    assert "AGM_NOALLOC_SCRATCH_BYTES" in msg and str(need) in msg
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(out)) == 0    # nothing was launched
