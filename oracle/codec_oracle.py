"""Restatement of the reference's tensor-state codec (oracle; test infrastructure).

Follows ``agillm41.py``:

* payload bytes / zstd-or-zlib decompression   4784-4812 (``_agillm43_zstd_compress``,
  ``_agillm43_payload_bytes``, ``_agillm43_zstd_decompress``)
* bytes -> tensor                                4815-4826 (``_agillm43_tensor_bytes``,
  ``_agillm43_tensor_from_bytes``)
* scales payloads                                4845-4855 (``_agillm43_pack_aux_tensor``,
  ``_agillm43_unpack_aux_tensor``)
* encoder quantisers                             4893-4946 (int8 symmetric, row-wise int8
  with fp16-stored row scales), the fp16 and lossless kinds 5008-5016
* decoder                                        5076-5102 (``_agillm43_decode_tensor_state``)
* how the side-update consumer applies a decoded state: ``value.to(target
  dtype)`` then ``copy_`` (alpha >= 1), ``lerp_`` or ``add_(alpha=...)``
  (delta updates)                                6029-6046

The same torch calls in the same order as the reference, so on the same
device it reproduces the reference's values bit for bit
(``tests/golden/make_golden_codec.py`` asserts this against the imported
reference). Only ``tests/`` and ``bench.py``'s CPU-baseline leg use it.
"""
from __future__ import annotations

import warnings
import zlib

import torch

MAGIC = "__agillm43_tensor_state_codec__"
VERSION = "agillm43_tensor_state_v3_rowq8c"


def payload_bytes(data) -> bytes:                                      # 4796-4799
    if torch.is_tensor(data):
        return data.detach().cpu().contiguous().numpy().tobytes()
    return bytes(data)


def compress(raw: bytes, level: int = 1) -> bytes:
    """The reference's compressor with zstandard absent: zlib behind a
    "ZLIB" tag (4784-4791)."""
    return b"ZLIB" + zlib.compress(raw, max(1, min(9, int(level))))


def decompress(data) -> bytes:                                         # 4806-4812
    data = payload_bytes(data)
    if data.startswith(b"ZLIB"):
        return zlib.decompress(data[4:])
    import zstandard as zstd  # only payloads written with zstandard present
    return zstd.ZstdDecompressor().decompress(data)


def dtype_from_name(name):                                             # 4780-4781
    return getattr(torch, str(name).replace("torch.", ""))


def dtype_name(dtype) -> str:                                          # 4776-4777
    return str(dtype).replace("torch.", "")


def tensor_bytes(t: torch.Tensor) -> bytes:                            # 4815-4817
    return t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()


def tensor_from_bytes(raw: bytes, name, shape) -> torch.Tensor:        # 4820-4825
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        return torch.frombuffer(memoryview(raw), dtype=dtype_from_name(name)).clone().reshape(
            tuple(int(x) for x in shape))


def byte_tensor(data: bytes) -> torch.Tensor:                          # 4800-4804
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)
        return torch.frombuffer(memoryview(data), dtype=torch.uint8).clone()


def pack_bytes(raw: bytes, level: int = 1):
    """Compressed when that is smaller, else raw (4845-4850, 5021-5027)."""
    c = compress(raw, level)
    return (byte_tensor(c), "zstd") if len(c) < len(raw) else (byte_tensor(raw), "raw")


def unpack_bytes(data, codec: str) -> bytes:
    return decompress(data) if codec == "zstd" else payload_bytes(data)


def int8_symmetric(src: torch.Tensor):                                 # 4893-4896
    f = src.float()
    maxabs = float(f.abs().max().item()) if f.numel() else 0.0
    scale = max(maxabs / 127.0, 1.0e-12)
    q = torch.clamp(torch.round(f / scale), -127, 127).to(torch.int8).contiguous()
    return q, scale


def int8_rowwise(src: torch.Tensor):                                   # 4916-4923
    f = src.float()
    cols = int(f.shape[-1])
    rows = int(f.numel() // cols)
    flat = f.reshape(rows, cols)
    scales = flat.abs().amax(dim=1).div(127.0).clamp_min(1.0e-12).to(torch.float32).contiguous()
    q = torch.clamp(torch.round(flat / scales[:, None]), -127, 127).to(torch.int8).contiguous()
    return q.reshape(tuple(src.shape)), scales, rows, cols


def encode_item(src: torch.Tensor, pack_kind: str, level: int = 1) -> dict:
    """One tensor in the reference's item layout (5031-5048) with the given
    pack kind ("int8_symmetric", "int8_rowwise" with fp16 row scales, "fp16"
    or "lossless")."""
    src = src.detach().cpu().contiguous()
    item = {"shape": list(src.shape), "orig_dtype": dtype_name(src.dtype), "pack_kind": pack_kind, "scale": None,
            "scales": None, "scales_data": None, "scales_codec": None, "scales_dtype": None, "rows": None,
            "cols": None, "scale_nbytes": 0}
    if pack_kind == "int8_symmetric":
        packed, item["scale"] = int8_symmetric(src)
    elif pack_kind == "int8_rowwise":
        packed, scales, item["rows"], item["cols"] = int8_rowwise(src)
        stored = scales.to(torch.float16).contiguous()                 # 4940-4950
        item["scales_data"], item["scales_codec"] = pack_bytes(tensor_bytes(stored), level)
        item["scales_dtype"] = dtype_name(stored.dtype)
        item["scale_nbytes"] = int(item["scales_data"].numel())
    elif pack_kind == "fp16":
        packed = src.to(torch.float16).contiguous()
    else:
        packed = src
    raw = tensor_bytes(packed)
    item["data"], item["codec"] = pack_bytes(raw, level)
    item["packed_dtype"] = dtype_name(packed.dtype)
    item["raw_nbytes"] = len(raw)
    item["packed_nbytes"] = int(item["data"].numel())
    return item


def encode_state(state, kinds) -> dict:
    """A codec state (5050-5068) holding ``state``'s tensors, each with the
    pack kind ``kinds[key]``."""
    tensors = {k: encode_item(v, kinds[k]) for k, v in state.items()}
    return {MAGIC: VERSION, "mode": "explicit", "zstd_level": 1, "tensor_count": len(tensors), "plain": {},
            "tensors": tensors}


def decode_tensor_state(state):                                        # 5076-5102
    if not (isinstance(state, dict) and str(state.get(MAGIC, "")).startswith("agillm43_tensor_state_v")):
        return state
    out = dict(state.get("plain") or {})
    for key, item in (state.get("tensors") or {}).items():
        data = item.get("data", b"")
        raw = decompress(data) if item.get("codec") == "zstd" else payload_bytes(data)
        packed = tensor_from_bytes(raw, item.get("packed_dtype"), item.get("shape"))
        if item.get("pack_kind") == "int8_symmetric":
            scale = float(item.get("scale") or 1.0)
            value = packed.float().mul_(scale)
        elif item.get("pack_kind") == "int8_rowwise":
            rows = int(item.get("rows") or 0)
            scales_data = item.get("scales_data")
            if scales_data is not None:
                rows = rows or int(item.get("scale_rows") or 0)
                raw_s = unpack_bytes(scales_data, item.get("scales_codec"))
                scales = tensor_from_bytes(raw_s, item.get("scales_dtype") or "float16", [rows]).float()
            else:
                scales = item.get("scales")
                if not torch.is_tensor(scales):
                    raise ValueError(f"rowwise tensor codec missing scales for {key}")
                scales = scales.float()
                rows = rows or int(scales.numel())
            value = packed.float().reshape(rows, -1).mul_(scales.reshape(rows, 1)).reshape(
                tuple(int(x) for x in item.get("shape")))
        else:
            value = packed
        out[key] = value
    return out


def apply_value(target: torch.Tensor, value: torch.Tensor, alpha: float = 1.0, delta: bool = False) -> None:
    """The side-update consumer's per-key update (6035-6045), in place."""
    if tuple(value.shape) != tuple(target.shape):
        raise ValueError(f"shape mismatch update={tuple(value.shape)} target={tuple(target.shape)}")
    src = value.to(device=target.device, dtype=target.dtype, non_blocking=True)
    if delta:
        if not target.is_floating_point():
            raise ValueError("delta update targets non-floating tensor")
        target.add_(src, alpha=alpha)
    elif alpha >= 1.0:
        target.copy_(src)
    else:
        target.lerp_(src, alpha)

