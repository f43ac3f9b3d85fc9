"""ctypes binding of ``lib/libagillm_moe.so`` (the C ABI in ``include/agillm_moe.h``).

The library is the only compute path: there is no CPU or PyTorch fallback.
If it cannot be loaded, or a tensor is not a CUDA tensor, the call raises.
Torch tensors cross the boundary as raw device pointers; every launch goes on
the current torch CUDA stream.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libagillm_moe.so")

AGM_F32, AGM_BF16, AGM_F16 = 0, 1, 2
AGM_OK = 0
AGM_TILE_M = 128
AGM_PAIR_ROWS = 256
AGM_PAIR_MIN_ROWS = 16384
AGM_GEMM_PAIR = -1
AGM_DISPATCH_BLOCK = 128
AGM_MAX_EXPERTS = 16
AGM_FLAG_TIE_LOW_FIRST = 0x1
AGM_FLAG_KEEP_ERROR = 0x2
AGM_FLAG_NO_PAIR = 0x4
AGM_FLAG_NO_SWAP = 0x8
AGM_FLAG_NO_PDL = 0x10
AGM_EP_HOLDERS, AGM_EP_BALANCED, AGM_EP_LOCAL = 0, 1, 2
AGM_FLAG_BWD_PAIR = 0x20
AGM_FLAG_NO_FOLD = 0x40
AGM_FLAG_DECODE_TILES = 0x80
AGM_FLAG_NO_FRONT = 0x100
AGM_CODEC_PLAIN, AGM_CODEC_INT8, AGM_CODEC_INT8_ROWWISE = 0, 1, 2
AGM_APPLY_COPY, AGM_APPLY_LERP, AGM_APPLY_ADD = 0, 1, 2


class AgmCodecTensor(ctypes.Structure):
    """One entry of agm_codec_decode_batch's table (include/agillm_moe.h)."""
    _fields_ = [("payload", ctypes.c_void_p), ("row_scales", ctypes.c_void_p), ("target", ctypes.c_void_p),
                ("n", ctypes.c_int64), ("cols", ctypes.c_int64), ("scale", ctypes.c_float), ("kind", ctypes.c_int),
                ("packed_dtype", ctypes.c_int), ("scales_dtype", ctypes.c_int), ("target_dtype", ctypes.c_int)]
AGM_SWAP_ROWS_PER_EXPERT = 32
AGM_STAGE_EVENTS = 8
AGM_EP_STAGE_EVENTS = 9

_DTYPE_CODE = {torch.float32: AGM_F32, torch.bfloat16: AGM_BF16, torch.float16: AGM_F16}

# Exported entry points and their C signatures (must match include/agillm_moe.h).
_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "agm_last_error": (ctypes.c_char_p, []),
    "agm_abi_version": (_I, []),
    "agm_dispatch_blocks": (_I64, [_I64]),
    "agm_max_rows": (_I64, [_I64, _I, _I]),
    "agm_router_topk": (_I, [_P, _P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "agm_dispatch_plan": (_I, [_P, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "agm_permute": (_I, [_P, _I, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "agm_grouped_gemm": (_I, [_P, _I64, _P, _P, _I, _I, _I, _I, _P, _P, _I64, _I, _I, _P, _I64, _P, _P]),
    "agm_combine": (_I, [_P, _P, _P, _I, _I64, _I, _I, _P, _I, _I64, _P, _P]),
    "agm_moe_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I, _I, _I]),
    "agm_moe_forward": (_I, [_P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                             _P, _SZ, _I, _P, _P, _P, _P, _P, _P, _P]),
    "agm_read_device_error": (_I, [_P, _P, _P]),
    "agm_moe_host_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I, _I, _I]),
    "agm_moe_forward_host": (_I, [_P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _P,
                                  _SZ, _I64, _I, _P]),
    "agm_ep_max_rows": (_I64, [_I64, _I, _I]),
    "agm_ep_comm_bytes": (_SZ, [_I, _I64, _I64, _I, _I]),
    "agm_ep_home_offset": (_I64, [_I, _I64, _I, _I]),
    "agm_ep_alloc": (_I, [_SZ, _P]),
    "agm_ep_free": (_I, [_P]),
    "agm_ep_ipc_handle": (_I, [_P, _P]),
    "agm_ep_ipc_open": (_I, [_P, _P]),
    "agm_ep_ipc_close": (_I, [_P]),
    "agm_ep_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I64, _I]),
    "agm_ep_forward": (_I, [_P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _I, _I, _P, _I64, _I64,
                            ctypes.c_uint64, _P, _P, _SZ, _I, _P, _P]),
    "agm_ep_dispatch": (_I, [_P, _I, _I64, _I, _I, _I, _I, _P, _I, _P, _I, _I, _P, _I64, _I64, ctypes.c_uint64, _P,
                             _SZ, _I, _P, _P]),
    "agm_ep_expert": (_I, [_I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _P, _I64, _I64, ctypes.c_uint64, _P,
                           _SZ, _I, _P, _P]),
    "agm_ep_combine": (_I, [_I, _I64, _I, _I, _I, _I, _I64, _P, _P, _P, _SZ, _P]),
    "agm_moe_forward_noalloc": (_I, [_P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                     _I, _P]),
    "agm_moe_noalloc_error_word": (_I, [_P]),
    "agm_layernorm": (_I, [_P, _P, _P, ctypes.c_float, _I, _I64, _I, _P, _P]),
    "agm_decode_tile_layout": (_I, [_P, _P, _I, _I64, _I, _I, _P]),
    "agm_moe_block_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I, _I, _I]),
    "agm_moe_block_forward": (_I, [_P, _P, _P, ctypes.c_float, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I,
                                   _P, _P, _P, _P, _P, _P, _SZ, _I, _P]),
    "agm_moe_train_saved_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I, _I, _I, _I]),
    "agm_moe_backward_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I, _I, _I]),
    "agm_cast_f32": (_I, [_P, _P, _I, _I64, _P]),
    "agm_moe_forward_train": (_I, [_P, _I, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P,
                                   _P, _P, _P, _SZ, _P, _I, _P]),
    "agm_moe_forward_residual": (_I, [_P, _P, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P,
                                      _P, _P, _SZ, _I, _P]),
    "agm_moe_backward": (_I, [_P, _I, _I, _I64, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P, _P, _P, _SZ,
                              _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _I, _P]),
    "agm_codec_decode": (_I, [_P, _I, _I, _I64, _I64, ctypes.c_float, _P, _I, _P, _I, _I, ctypes.c_float, _P]),
    "agm_codec_decode_batch": (_I, [_P, _I, _I, ctypes.c_float, _P]),
    "agm_moe_aux_saved_bytes": (_SZ, [_I64, _I, _I]),
    "agm_moe_aux_backward_workspace_bytes": (_SZ, [_I64, _I, _I]),
    "agm_moe_aux_forward": (_I, [_P, _I, _I64, _I, _I, _P, ctypes.c_double, ctypes.c_double, _P, _P, _SZ, _I, _P]),
    "agm_moe_aux_backward": (_I, [_P, _P, _I, _I64, _I, _I, _P, _SZ, _P, _P, _SZ, _I, _P]),
}


class MoEKernelError(RuntimeError):
    """A C-ABI call returned an error (bad argument, CUDA error, device error word)."""


_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load the shared library (once). Raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MoEKernelError(
                f"{LIB_PATH} is missing: build it with `python agillm4.1_b200/build.py` "
                "(nvcc, sm_100a). There is no fallback path.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.agm_abi_version() != 1:
            raise MoEKernelError("libagillm_moe.so ABI version mismatch")
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != AGM_OK:
        msg = load().agm_last_error().decode(errors="replace")
        raise MoEKernelError(f"{what} failed ({rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise MoEKernelError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise MoEKernelError("CUDA tensors only: the MoE kernels have no CPU path")
    if not t.is_contiguous():
        raise MoEKernelError("tensors passed to the MoE kernels must be contiguous")
    return t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def read_device_error(err: torch.Tensor) -> int:
    """Synchronise the current stream and return (and clear) a device error word."""
    code = ctypes.c_int(0)
    lib = load()
    rc = lib.agm_read_device_error(ptr(err), ctypes.byref(code), stream_handle(err.device))
    if rc != AGM_OK and code.value == 0:
        check(rc, "agm_read_device_error")
    return int(code.value)
