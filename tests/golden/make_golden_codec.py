"""Generate the tensor-codec golden vectors from the reference itself.

Run from the repository root, in a container that has the reference checkout:

    python tests/golden/make_golden_codec.py [--ref /root/reference/agillm41.py]

For every encoder mode in ``MODES`` it encodes a seeded MoE-layer state
(experts' FC1/FC2 weights and biases, one expert with an outlier row, the
router and a bf16 shared-expert weight) with the reference's
``_agillm43_encode_tensor_state`` (agillm41.py:4858-5074; without zstandard
the reference compresses with zlib behind a "ZLIB" tag), decodes it with
``_agillm43_decode_tensor_state`` (5076-5102) and applies the decoded values
to seeded fp32 and bf16 targets the way the side-update consumer does
(6035-6045: copy, lerp with alpha 0.3 and 0.75, delta add with alpha 0.5). It
asserts that ``oracle/codec_oracle.py`` decodes to the same bits and that its
encoder reproduces the reference's payload bytes for the pack kinds the
reference chose, then writes ``tests/golden/codec_<mode>.npz``: the item
metadata as JSON, each payload's bytes, the decoded values and the applied
targets.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from make_golden import load_reference, to_np  # noqa: E402
from oracle import codec_oracle as orc  # noqa: E402
from oracle.golden_cases import CODEC_APPLY, CODEC_APPLY_KEYS, CODEC_MODES, codec_state, codec_target  # noqa: E402


def run_mode(ref, mode, outdir):
    state = codec_state()
    enc = ref._agillm43_encode_tensor_state(dict(state), mode=mode, zstd_level=1)
    dec = ref._agillm43_decode_tensor_state(enc)
    dec_o = orc.decode_tensor_state(enc)
    rec = {"mode": np.array(mode)}
    meta = {}
    for key, item in enc["tensors"].items():
        assert torch.equal(dec[key], dec_o[key]) and dec[key].dtype == dec_o[key].dtype, (mode, key)
        if item["pack_kind"] in ("int8_symmetric", "int8_rowwise", "fp16", "lossless"):
            mine = orc.encode_item(state[key], item["pack_kind"])
            assert torch.equal(mine["data"], item["data"]), (mode, key, "payload bytes")
            if item["pack_kind"] == "int8_rowwise":
                assert torch.equal(mine["scales_data"], item["scales_data"]), (mode, key, "scale bytes")
        m = {k: v for k, v in item.items() if k not in ("data", "scales_data", "scales")}
        meta[key] = m
        rec[f"data/{key}"] = item["data"].numpy()
        if item.get("scales_data") is not None:
            rec[f"scales_data/{key}"] = item["scales_data"].numpy()
        rec[f"decoded/{key}"] = to_np(dec[key])
        if key not in CODEC_APPLY_KEYS:
            continue
        for tdt in (torch.float32, torch.bfloat16):
            for name, alpha, delta in CODEC_APPLY:
                t = codec_target(key, state[key].shape, tdt)
                orc.apply_value(t, dec[key], alpha, delta)
                # the reference's lines, run here on the reference's decoded value
                t2 = codec_target(key, state[key].shape, tdt)
                src = dec[key].to(dtype=tdt)
                if delta:
                    t2.add_(src, alpha=alpha)
                elif alpha >= 1.0:
                    t2.copy_(src)
                else:
                    t2.lerp_(src, alpha)
                assert torch.equal(t, t2), (mode, key, name)
                rec[f"applied/{name}/{str(tdt)[6:]}/{key}"] = to_np(t)
    rec["meta"] = np.array(json.dumps(meta, sort_keys=True))
    rec["header"] = np.array(json.dumps({k: v for k, v in enc.items() if k != "tensors"}, sort_keys=True,
                                        default=str))
    path = os.path.join(outdir, "codec_" + mode.replace("-", "_") + ".npz")
    np.savez_compressed(path, **rec)
    kinds = {k: v["pack_kind"] for k, v in meta.items()}
    print(f"{mode}: {kinds} -> {os.path.relpath(path, ROOT)} ({os.path.getsize(path) // 1024} KB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("AGILLM41_REFERENCE", "/root/reference/agillm41.py"),
                    help="the reference's agillm41.py (default: $AGILLM41_REFERENCE, else /root/reference/agillm41.py)")
    args = ap.parse_args()
    ref = load_reference(args.ref)
    for mode in CODEC_MODES:
        run_mode(ref, mode, HERE)


if __name__ == "__main__":
    main()
