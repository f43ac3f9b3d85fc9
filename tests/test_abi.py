"""The C-ABI library loads on a host without a GPU and exports exactly the
entry points that include/agillm_moe.h declares; argument errors are reported
without touching a device."""
import ctypes
import os
import re

import pytest

import agillm41_b200
from agillm41_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "agillm_moe.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"AGM_API\s+[\w\s\*]+?\b(agm_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "agm_moe_forward" in syms and "agm_router_topk" in syms
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert lib.agm_abi_version() == 1


def test_library_has_no_driver_link_dependency():
    # The driver is resolved at run time; the .so must load where no libcuda exists.
    ctypes.CDLL(_lib.LIB_PATH)


def test_size_helpers():
    lib = _lib.load()
    assert lib.agm_dispatch_blocks(0) == 0
    B = _lib.AGM_DISPATCH_BLOCK
    assert lib.agm_dispatch_blocks(1) == 1
    assert lib.agm_dispatch_blocks(B) == 1
    assert lib.agm_dispatch_blocks(B + 1) == 2
    assert lib.agm_max_rows(73728, 2, 14) == ((2 * 73728 + 14 * 255 + 255) // 256) * 256
    assert lib.agm_max_rows(64, 2, 14) == ((2 * 64 + 14 * 127 + 127) // 128) * 128
    assert lib.agm_max_rows(8192, 2, 14) == ((2 * 8192 + 14 * 255 + 255) // 256) * 256
    assert lib.agm_max_rows(0, 2, 14) == 0
    ws = lib.agm_moe_workspace_bytes(73728, 1280, 14, 2, 3200, 0, 1, _lib.AGM_BF16)
    rows = lib.agm_max_rows(73728, 2, 14)
    # x_perm/y and h dominate: rows * (d + H) * 2 bytes.
    assert ws >= rows * (1280 + 3200) * 2
    assert ws < rows * (1280 + 3200) * 2 + 64 * 1024 * 1024


@pytest.mark.parametrize("call,code", [
    ("bad_dtype", _lib.AGM_OK - 1),
    ("bad_topk", _lib.AGM_OK - 1),
    ("too_many_experts", _lib.AGM_OK - 2),
    ("odd_d", _lib.AGM_OK - 2),
    ("null_ptrs", _lib.AGM_OK - 1),
])
def test_argument_errors_are_reported(call, code):
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)  # never dereferenced: validation fails first
    args = dict(x=fake, w=fake, dtype=_lib.AGM_BF16, n=16, d=64, E=14, k=2)
    if call == "bad_dtype":
        args["dtype"] = 7
    elif call == "bad_topk":
        args["k"] = 15
    elif call == "too_many_experts":
        args["E"] = 17
    elif call == "odd_d":
        args["d"] = 60
    if call == "null_ptrs":
        rc = lib.agm_router_topk(fake, fake, args["dtype"], 16, 64, 14, 2, 0, None, None, None, None, None, None,
                                 None)
    else:
        rc = lib.agm_router_topk(args["x"], args["w"], args["dtype"], args["n"], args["d"], args["E"], args["k"], 0,
                                 None, None, fake, fake, fake, None, None)
    assert rc == code
    assert lib.agm_last_error().decode()


def test_forward_rejects_small_workspace():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    rc = lib.agm_moe_forward(fake, _lib.AGM_BF16, 1024, 64, 14, 2, 128, fake, fake, fake, fake, fake, 0, 1, None,
                             None, None, None, fake, fake, 1024, 0, None, None, None, None, None, None, None)
    assert rc == -5
    assert "workspace" in lib.agm_last_error().decode()


def test_package_exports():
    assert agillm41_b200.MoEFFN is not None
    assert os.path.exists(agillm41_b200.LIB_PATH)


def test_training_entry_points_validate_without_a_device():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    n, d, E, k, H = 1024, 64, 14, 2, 128
    need = lib.agm_moe_train_saved_bytes(n, d, E, k, H, 0, 1, _lib.AGM_BF16, _lib.AGM_BF16)
    rows = lib.agm_max_rows(n, k, E)
    assert need >= rows * (2 * d + H) * 2            # x_perm, y and h are kept
    amp = lib.agm_moe_train_saved_bytes(n, d, E, k, H, 0, 1, _lib.AGM_F32, _lib.AGM_BF16)
    assert amp >= need + n * d * 2                   # plus the 16-bit cast of x
    shared = lib.agm_moe_train_saved_bytes(n, d, E, k, H, 1, 2 * d, _lib.AGM_BF16, _lib.AGM_BF16)
    assert shared >= need + n * (d + 2 * d + d) * 2  # x copy, shared FC1 activation and output
    assert lib.agm_moe_backward_workspace_bytes(n, d, E, k, H, 0, 1, _lib.AGM_BF16) >= rows * (d + H) * 2
    fwd = [fake, _lib.AGM_BF16, _lib.AGM_BF16, n, d, E, k, H, fake, fake, fake, fake, fake, 0, 1, None, None, None,
           None, None, fake, fake]
    # saved buffer too small
    assert lib.agm_moe_forward_train(*fwd, 1024, None, 0, None) == -5
    assert "saved" in lib.agm_last_error().decode()
    # fp16 input with bf16 weights is neither mode
    bad = list(fwd)
    bad[1] = _lib.AGM_F16
    assert lib.agm_moe_forward_train(*bad, need, None, 0, None) == -1
    assert "x_dtype" in lib.agm_last_error().decode()
    # shared experts without their weights
    sh = list(fwd)
    sh[13], sh[14] = 1, 2 * d
    assert lib.agm_moe_forward_train(*sh, shared, None, 0, None) == -1
    # misaligned residual
    mis = list(fwd)
    mis[19] = ctypes.c_void_p(4096 + 8)
    assert lib.agm_moe_forward_train(*mis, need, None, 0, None) == -1
    assert lib.agm_moe_forward_residual(fake, None, _lib.AGM_BF16, n, d, E, k, H, fake, fake, fake, fake, fake, 0, 1,
                                        None, None, None, None, fake, fake, 1 << 30, 0, None) == -1
    # backward: workspace too small
    rc = lib.agm_moe_backward(fake, _lib.AGM_BF16, _lib.AGM_BF16, n, d, E, k, H, fake, fake, fake, 0, 1, None, None,
                              fake, need, fake, fake, fake, fake, fake, fake, None, None, None, None, fake, 1024, 0,
                              None)
    assert rc == -5 and "workspace" in lib.agm_last_error().decode()
    assert lib.agm_cast_f32(fake, fake, _lib.AGM_F32, 16, None) == -1


def test_aux_entry_points_validate_without_a_device():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    n, d, E = 1000, 64, 14
    need = lib.agm_moe_aux_saved_bytes(n, E, _lib.AGM_F32)
    assert need >= n * E * 4                          # the fp32 logits are kept
    assert lib.agm_moe_aux_saved_bytes(-1, E, _lib.AGM_F32) == 0
    assert lib.agm_moe_aux_backward_workspace_bytes(n, d, _lib.AGM_BF16) >= n * 16 * 2
    fwd = [fake, _lib.AGM_F32, n, d, E, fake, 0.01, 0.001, fake, fake]
    assert lib.agm_moe_aux_forward(*fwd, 1024, 0, None) == -5
    assert "saved" in lib.agm_last_error().decode()
    bad = list(fwd)
    bad[4] = 17
    assert lib.agm_moe_aux_forward(*bad, need, 0, None) == -2
    bad = list(fwd)
    bad[3] = 12
    assert lib.agm_moe_aux_forward(*bad, need, 0, None) == -1
    bad = list(fwd)
    bad[8] = None
    assert lib.agm_moe_aux_forward(*bad, need, 0, None) == -1
    bad = list(fwd)
    bad[0] = ctypes.c_void_p(4096 + 4)
    assert lib.agm_moe_aux_forward(*bad, need, 0, None) == -1
    rc = lib.agm_moe_aux_backward(fake, fake, _lib.AGM_F32, n, d, E, fake, need, fake, fake, 1024, 0, None)
    assert rc == -5 and "workspace" in lib.agm_last_error().decode()


def test_codec_decode_validates_without_a_device():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    args = dict(payload=fake, kind=_lib.AGM_CODEC_INT8, packed=0, n=1000, cols=1, scale=0.5, scales=None,
                scales_dtype=0, target=fake, target_dtype=_lib.AGM_F32, mode=_lib.AGM_APPLY_COPY, alpha=1.0)

    def call(**kw):
        a = dict(args, **kw)
        return lib.agm_codec_decode(a["payload"], a["kind"], a["packed"], a["n"], a["cols"], a["scale"], a["scales"],
                                    a["scales_dtype"], a["target"], a["target_dtype"], a["mode"], a["alpha"], None)

    assert call(kind=7) == -1
    assert call(mode=9) == -1
    assert call(target_dtype=5) == -1
    assert call(kind=_lib.AGM_CODEC_PLAIN, packed=5) == -2
    assert call(kind=_lib.AGM_CODEC_INT8_ROWWISE, cols=7, scales=fake, scales_dtype=_lib.AGM_F16) == -1
    assert call(kind=_lib.AGM_CODEC_INT8_ROWWISE, cols=10, scales=fake, scales_dtype=_lib.AGM_BF16) == -1
    assert call(kind=_lib.AGM_CODEC_INT8_ROWWISE, cols=10, scales=None, scales_dtype=_lib.AGM_F16) == -1
    assert call(payload=None) == -1
    assert call(target=ctypes.c_void_p(4096 + 2)) == -1          # fp32 target off its 4-byte alignment
    assert call(n=-1) == -1
    assert call(n=0, payload=None, target=None) == 0              # nothing to do


def test_codec_batch_validates_every_entry_first():
    lib = _lib.load()
    fake = 4096
    good = _lib.AgmCodecTensor(payload=fake, row_scales=None, target=fake, n=64, cols=1, scale=0.5,
                               kind=_lib.AGM_CODEC_INT8, packed_dtype=0, scales_dtype=0, target_dtype=_lib.AGM_F32)
    bad = _lib.AgmCodecTensor(payload=fake, row_scales=None, target=fake, n=64, cols=7, scale=1.0,
                              kind=_lib.AGM_CODEC_INT8_ROWWISE, packed_dtype=0, scales_dtype=_lib.AGM_F16,
                              target_dtype=_lib.AGM_F32)
    table = (_lib.AgmCodecTensor * 2)(good, bad)
    # the second entry is rejected before the first one launches (no device here)
    assert lib.agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), 2, _lib.AGM_APPLY_COPY, 1.0, None) == -1
    assert "cols" in lib.agm_last_error().decode()
    assert lib.agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), 1, 9, 1.0, None) == -1
    assert lib.agm_codec_decode_batch(None, -1, _lib.AGM_APPLY_COPY, 1.0, None) == -1
    assert lib.agm_codec_decode_batch(None, 0, _lib.AGM_APPLY_COPY, 1.0, None) == 0
    assert ctypes.sizeof(_lib.AgmCodecTensor) == 64


def test_training_forward_refuses_cpu_tensors():
    import torch

    m = agillm41_b200.MoEFFN(64, mlp_mult=2, experts=4, top_k=2).train()
    with pytest.raises(agillm41_b200.MoEKernelError):
        m(torch.randn(8, 64, requires_grad=True)).sum().backward()
