"""Generate the golden vectors for the MoE block forward from the reference itself.

Run from the repository root, in a container that has the reference checkout:

    python tests/golden/make_golden.py [--ref /root/reference/agillm41.py]

It imports the reference's ``agillm41.py`` (synthetic tokenizer, module
registered in ``sys.modules`` before execution), builds ``MoEFFN`` modules
(agillm41.py:4323-4360), loads seeded weights (``oracle.reference_moe.make_state``),
runs the reference ``forward`` (agillm41.py:4389-4431) on CPU, and writes one
``.npz`` per case next to this script. For every case it also runs the torch
restatement in ``oracle/reference_moe.py`` and asserts that it reproduces the
reference bit for bit, so the oracle is pinned to the reference.

Cases store seeds, shapes, SHA-256 hashes of the weights and input (which the
tests regenerate with ``oracle.reference_moe.make_state``/``make_input`` and
check against the hashes) and the reference outputs; one tiny case also stores
its weights and input outright. bf16 tensors are stored as their uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import reference_moe as orc  # noqa: E402
from oracle.golden_cases import CASES, case_inputs  # noqa: E402


def load_reference(path: str):
    os.environ.setdefault("AGILLM_SYNTHETIC_TOKENIZER", "1")
    os.environ.setdefault("AGILLM_SYNTHETIC_VOCAB", "32000")
    spec = importlib.util.spec_from_file_location("agillm41", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["agillm41"] = mod
    spec.loader.exec_module(mod)
    return mod


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def tensor_hash(t: torch.Tensor) -> str:
    return hashlib.sha256(to_np(t.contiguous()).tobytes()).hexdigest()


def state_hash(sd) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(to_np(sd[k].contiguous()).tobytes())
    return h.hexdigest()


def build_module(ref, d, hidden, experts, top_k, shared, shared_hidden, sd, dtype):
    nn = torch.nn
    mult = hidden // d if hidden % d == 0 else 1
    m = ref.MoEFFN(d, mlp_mult=mult, experts=experts, top_k=top_k,
                   shared_experts=shared, shared_mlp_mult=(shared_hidden // d if shared and shared_hidden % d == 0 else 1))
    if hidden != m.mlp_mult * d:
        # Expert hidden sizes that the constructor cannot express (it truncates
        # mlp_mult to an int): swap the experts for same-keyed Sequentials.
        m.experts = nn.ModuleList([nn.Sequential(nn.Linear(d, hidden), nn.ReLU(), nn.Linear(hidden, d))
                                   for _ in range(experts)])
    if shared and m.shared[0][0].weight.shape[0] != shared_hidden:
        m.shared = nn.ModuleList([nn.Sequential(nn.Linear(d, shared_hidden), nn.ReLU(), nn.Linear(shared_hidden, d))
                                  for _ in range(shared)])
    m.load_state_dict(sd)
    return m.to(dtype).eval()


def run_case(ref, case, outdir):
    (name, d, H, E, k, N, seed, dtype, shared, shared_H, bias_std, special, store_w) = case
    sd32, x32 = case_inputs(case)
    sd = {kk: v.to(dtype) for kk, v in sd32.items()}
    x = x32.to(dtype)
    m = build_module(ref, d, H, E, k, shared, shared_H, sd32, dtype)
    # The module's own state must equal the restatement's input state.
    msd = m.state_dict()
    assert set(msd) == set(sd), (sorted(msd), sorted(sd))
    for kk in sd:
        assert torch.equal(msd[kk], sd[kk]), kk
    with torch.no_grad():
        y_ref = m(x.reshape(1, N, d)).reshape(N, d)
        aux = {}
        y_orc = orc.moe_forward(x, sd, k, aux=aux)
    assert y_ref.dtype == dtype
    assert torch.equal(y_ref, y_orc), f"{name}: restatement differs from the reference"
    rec = dict(
        name=np.array(name), d=d, hidden=H, experts=E, top_k=k, n_tokens=N, seed=seed,
        dtype=np.array(str(dtype).replace("torch.", "")), shared=shared, shared_hidden=shared_H,
        bias_std=bias_std, special=np.array(special or ""),
        out=to_np(y_ref), logits=to_np(aux["logits"]), idx=to_np(aux["idx"]),
        gates=to_np(aux["gates"]), counts=to_np(aux["counts"]),
        x_sha256=np.array(tensor_hash(x)), state_sha256=np.array(state_hash(sd)),
        torch_version=np.array(torch.__version__),
    )
    if store_w:
        rec["x"] = to_np(x)
        for kk, v in sd.items():
            rec["w:" + kk] = to_np(v)
    path = os.path.join(outdir, name + ".npz")
    np.savez_compressed(path, **rec)
    ties = int((aux["logits"].topk(min(k + 1, E), dim=-1).values.diff(dim=-1) == 0).any(dim=-1).sum())
    print(f"{name}: N={N} d={d} H={H} E={E} k={k} {dtype} counts={aux['counts'].tolist()} "
          f"rows_with_ties={ties} -> {os.path.relpath(path, ROOT)} ({os.path.getsize(path)//1024} KB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("AGILLM41_REFERENCE", "/root/reference/agillm41.py"),
                    help="the reference's agillm41.py (default: $AGILLM41_REFERENCE, else /root/reference/agillm41.py)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    ref = load_reference(args.ref)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for case in CASES:
        if args.only and args.only not in case[0]:
            continue
        run_case(ref, case, HERE)


if __name__ == "__main__":
    main()
