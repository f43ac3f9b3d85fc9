"""Tensor-state codec decode on the GPU (agillm41.py:4858-5102, 6029-6046).

The reference ships DBlock lease and update payloads (expert weights
included) through a tensor codec: per tensor an int8 payload with one scale
("int8_symmetric"), an int8 payload with fp16 row scales ("int8_rowwise"),
an fp16 payload or the lossless bytes, each zstd-compressed (zlib behind a
"ZLIB" tag where zstandard is missing). ``_agillm43_decode_tensor_state``
turns every tensor back into fp32 on the host, and the side-update consumer
then copies each fp32 value to the GPU and applies it to the parameter
(``copy_``, ``lerp_`` or, for delta updates, ``add_``).

Here the host only decompresses (threads in parallel; zlib and zstandard
release the GIL), the packed bytes cross PCIe (1 byte per int8 element
instead of 4), and ``agm_codec_decode_batch`` dequantises and applies them on
the GPU in one pass over each parameter, the tensors of one kind in one
launch:

* :func:`decode_tensor_state` - drop-in for ``_agillm43_decode_tensor_state``
  that returns device tensors (fp32 for the int8 kinds, the packed dtype
  otherwise, as the reference's values);
* :func:`apply_tensor_state` - the decode fused with the consumer's update
  into existing device tensors (the expert weights of a ``MoEFFN`` among
  them), with the reference's key and shape checks.
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes
import os
import zlib
from typing import Dict, Mapping, Optional

import numpy as np
import torch

from . import _lib
from ._lib import MoEKernelError, load, ptr, stream_handle

MAGIC = "__agillm43_tensor_state_codec__"
_KINDS = {"int8_symmetric": _lib.AGM_CODEC_INT8, "int8_rowwise": _lib.AGM_CODEC_INT8_ROWWISE}
_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16, "int8": torch.int8}


def is_encoded(state) -> bool:
    """True for a codec state (agillm41.py:5077)."""
    return isinstance(state, dict) and str(state.get(MAGIC, "")).startswith("agillm43_tensor_state_v")


def _bytes(data) -> bytes:
    if torch.is_tensor(data):
        return data.detach().cpu().contiguous().numpy().tobytes()
    return bytes(data)


def _decompress(data, codec) -> bytes:
    """A payload's packed bytes (agillm41.py:4806-4812): zlib behind a "ZLIB"
    tag, else zstd, or the raw bytes when the codec is not "zstd"."""
    raw = _bytes(data)
    if codec != "zstd":
        return raw
    if raw.startswith(b"ZLIB"):
        return zlib.decompress(raw[4:])
    try:
        import zstandard
    except ImportError as exc:  # pragma: no cover - depends on the host
        raise MoEKernelError("zstd-compressed codec payload, but the zstandard module is not installed") from exc
    return zstandard.ZstdDecompressor().decompress(raw)


def _dtype(name) -> torch.dtype:
    key = str(name).replace("torch.", "")
    if key not in _DTYPES:
        raise MoEKernelError(f"codec payload dtype {name!r} is not supported on the GPU path")
    return _DTYPES[key]


class _Payload:
    """One tensor's packed bytes (and row scales) staged in pinned memory."""

    def __init__(self, key, item):
        self.key = key
        self.kind_name = item.get("pack_kind")
        self.shape = tuple(int(x) for x in item.get("shape"))
        self.packed_dtype = _dtype(item.get("packed_dtype"))
        raw = _decompress(item.get("data", b""), item.get("codec"))
        self.packed = _pinned(raw)
        self.n = int(np.prod(self.shape)) if self.shape else 1
        if self.packed.numel() != self.n * torch.empty((), dtype=self.packed_dtype).element_size():
            raise MoEKernelError(f"{key}: payload holds {self.packed.numel()} bytes, shape {self.shape} "
                                 f"of {self.packed_dtype} needs more or less")
        self.scale = 1.0
        self.rows = 0
        self.scales = None
        self.scales_dtype = None
        if self.kind_name == "int8_symmetric":
            self.scale = float(item.get("scale") or 1.0)
        elif self.kind_name == "int8_rowwise":
            rows = int(item.get("rows") or 0)
            if item.get("scales_data") is not None:
                rows = rows or int(item.get("scale_rows") or 0)
                sraw = _decompress(item["scales_data"], item.get("scales_codec"))
                self.scales_dtype = _dtype(item.get("scales_dtype") or "float16")
                self.scales = _pinned(sraw)
            else:
                s = item.get("scales")
                if not torch.is_tensor(s):
                    raise ValueError(f"rowwise tensor codec missing scales for {key}")
                self.scales_dtype = torch.float32
                self.scales = s.detach().float().cpu().contiguous().view(torch.uint8).pin_memory()
                rows = rows or int(s.numel())
            self.rows = rows
            if rows <= 0 or self.n % rows:
                raise MoEKernelError(f"{key}: {rows} row scales do not divide {self.n} elements")

    def value_dtype(self):
        """The dtype of the reference's decoded value."""
        return torch.float32 if self.kind_name in _KINDS else self.packed_dtype

    def upload(self, dev):
        """Asynchronous copies of the packed bytes (and row scales) to ``dev``."""
        q = self.packed.to(dev, non_blocking=True)
        s = self.scales.to(dev, non_blocking=True) if self.scales is not None else None
        return q, s

    def entry(self, q, s, target: torch.Tensor) -> "_lib.AgmCodecTensor":
        """This tensor's row of agm_codec_decode_batch's table."""
        kind = _KINDS.get(self.kind_name, _lib.AGM_CODEC_PLAIN)
        return _lib.AgmCodecTensor(
            payload=ptr(q), row_scales=ptr(s), target=ptr(target), n=self.n,
            cols=self.n // self.rows if kind == _lib.AGM_CODEC_INT8_ROWWISE else 1, scale=self.scale, kind=kind,
            packed_dtype=_lib.dtype_code(self.packed_dtype) if kind == _lib.AGM_CODEC_PLAIN else 0,
            scales_dtype=_lib.dtype_code(self.scales_dtype) if s is not None else 0,
            target_dtype=_lib.dtype_code(target.dtype))


def _decode_into(jobs, mode: int, alpha: float) -> None:
    """Decode every (payload, target) pair of ``jobs`` (an iterable): the
    packed bytes are copied to the target's device as each payload is staged
    (while later ones still decompress), then one agm_codec_decode_batch
    call per device decodes the lot (tensors of one signature share a
    launch)."""
    per_dev = {}
    for p, target in jobs:
        q, s = p.upload(target.device)
        per_dev.setdefault(target.device, []).append((p.entry(q, s, target), q, s))
    for dev, rows in per_dev.items():
        table = (_lib.AgmCodecTensor * len(rows))(*[r[0] for r in rows])
        rc = load().agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), len(rows), mode, float(alpha),
                                           stream_handle(dev))
        _lib.check(rc, "agm_codec_decode_batch")


def _pinned(raw: bytes) -> torch.Tensor:
    t = torch.empty(len(raw), dtype=torch.uint8, pin_memory=True)
    if raw:
        t.numpy()[:] = np.frombuffer(raw, dtype=np.uint8)
    return t


def _staged(state, threads: Optional[int]):
    items = list((state.get("tensors") or {}).items())
    workers = max(1, min(len(items), threads or min(16, os.cpu_count() or 1)))
    with cf.ThreadPoolExecutor(workers) as pool:
        for p in pool.map(lambda kv: _Payload(*kv), items):
            yield p


def decode_tensor_state(state, device="cuda", *, threads: Optional[int] = None) -> Dict[str, object]:
    """``_agillm43_decode_tensor_state`` (agillm41.py:5076-5102) with the
    dequantisation on the GPU: returns the plain entries and one device
    tensor per encoded tensor, with the reference's values (fp32 for the
    int8 kinds, the packed dtype otherwise). A state that is not a codec
    state is returned unchanged, as by the reference."""
    if not is_encoded(state):
        return state
    dev = torch.device(device)
    if dev.type != "cuda":
        raise MoEKernelError("decode_tensor_state decodes on a CUDA device (there is no CPU path)")
    out = dict(state.get("plain") or {})

    def jobs():
        for p in _staged(state, threads):
            out[p.key] = torch.empty(p.shape, dtype=p.value_dtype(), device=dev)
            yield p, out[p.key]

    _decode_into(jobs(), _lib.AGM_APPLY_COPY, 1.0)
    return out


def apply_tensor_state(state, targets: Mapping[str, torch.Tensor], *, alpha: float = 1.0, delta: bool = False,
                       threads: Optional[int] = None) -> int:
    """Decode ``state`` straight into ``targets`` (device tensors keyed like
    the state: a module's ``named_parameters()``/``named_buffers()``), as the
    side-update consumer applies a decoded state (agillm41.py:6029-6046):
    ``copy_`` when alpha >= 1, ``lerp_(value, alpha)`` otherwise, or
    ``add_(value, alpha=alpha)`` for a delta update; the value is rounded to
    the target's dtype first. Raises KeyError for an unknown key and
    ValueError for a shape mismatch or a delta to a non-floating target, as the
    reference does. Returns the number of tensors applied."""
    if not is_encoded(state):
        raise MoEKernelError("apply_tensor_state takes a codec state (see is_encoded)")
    mode = _lib.AGM_APPLY_ADD if delta else (_lib.AGM_APPLY_COPY if alpha >= 1.0 else _lib.AGM_APPLY_LERP)
    for key, item in (state.get("tensors") or {}).items():  # checks before any byte moves
        target = targets.get(key)
        if target is None:
            raise KeyError(f"unknown core key {key}")
        if tuple(int(x) for x in item.get("shape")) != tuple(target.shape):
            raise ValueError(f"{key} shape mismatch update={tuple(item.get('shape'))} target={tuple(target.shape)}")
        if delta and not target.is_floating_point():
            raise ValueError(f"{key} delta update targets non-floating tensor")
    for key in state.get("tensors") or {}:
        if not targets[key].is_cuda or not targets[key].is_contiguous():
            raise MoEKernelError(f"{key}: targets must be contiguous CUDA tensors (there is no CPU path)")
    done = []

    def jobs():
        for p in _staged(state, threads):
            done.append(targets[p.key])
            yield p, targets[p.key]

    with torch.no_grad():
        _decode_into(jobs(), mode, alpha)
    for target in done:
        # An in-place update: bump the version counter as torch's own
        # in-place ops do, so caches keyed on it (the MoE block's packed
        # weights) see the new values.
        torch.autograd.graph.increment_version(target)
    return len(done)
