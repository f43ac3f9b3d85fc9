"""Generate the auxiliary-loss golden vectors from the reference itself.

Run from the repository root, in a container that has the reference checkout:

    python tests/golden/make_golden_aux.py [--ref /root/reference/agillm41.py]

For every case of ``oracle.golden_cases.AUX_CASES`` it builds reference
``MoEFFN`` modules (agillm41.py:4323-4360) with the case's router weights,
runs their training forward (which stashes the detached router input,
agillm41.py:4392-4397), calls the reference's ``_collect_moe_aux``
(agillm41.py:4463-4492) on CPU and back-propagates the case's upstream
gradient. It asserts that ``oracle.reference_moe.collect_moe_aux`` gives the
same loss and router gradients bit for bit, then writes
``tests/golden/<name>.npz`` with the inputs, router weights, loss and router
weight gradients (bf16 as uint16 bit patterns).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from make_golden import load_reference, to_np  # noqa: E402
from oracle import reference_moe as orc  # noqa: E402
from oracle.golden_cases import AUX_CASES, aux_case_inputs  # noqa: E402


def run_case(ref, case, outdir):
    (name, d, E, N, seed, dtype, aux_coef, z_coef, modules, gscale, special) = case
    pairs = [(x.to(dtype), w.to(dtype)) for x, w in aux_case_inputs(case)]
    mods = []
    for x, w in pairs:
        m = ref.MoEFFN(d, mlp_mult=1, experts=E, top_k=1).to(dtype).train()
        with torch.no_grad():
            m.router.weight.copy_(w)
        m(x.reshape(1, N, d))  # the training forward stashes the router input
        assert torch.equal(m.last_router_input, x)
        mods.append(m)
    model = torch.nn.ModuleList(mods)
    loss = ref._collect_moe_aux(model, aux_coef, z_coef)
    assert all(m.last_router_input is None for m in mods)
    upstream = torch.tensor(gscale, dtype=loss.dtype)
    loss.backward(upstream)
    d_ref = [m.router.weight.grad for m in mods]

    w_leaf = [w.clone().requires_grad_(True) for _, w in pairs]
    loss_o = orc.collect_moe_aux([x for x, _ in pairs], w_leaf, aux_coef, z_coef)
    loss_o.backward(upstream)
    assert loss.dtype == torch.float32 and torch.equal(loss.detach(), loss_o.detach()), f"{name}: loss differs"
    for i, (a, b) in enumerate(zip(d_ref, w_leaf)):
        assert torch.equal(a, b.grad), f"{name}: router gradient {i} differs"
    rec = dict(name=np.array(name), d=d, experts=E, n_tokens=N, seed=seed,
               dtype=np.array(str(dtype).replace("torch.", "")), aux_coef=aux_coef, z_coef=z_coef,
               modules=modules, upstream=gscale, special=np.array(special or ""),
               loss=np.float32(loss.item()), torch_version=np.array(torch.__version__))
    for i, ((x, w), g) in enumerate(zip(pairs, d_ref)):
        rec[f"x{i}"] = to_np(x)
        rec[f"w{i}"] = to_np(w)
        rec[f"d_router{i}"] = to_np(g)
    path = os.path.join(outdir, name + ".npz")
    np.savez_compressed(path, **rec)
    print(f"{name}: N={N} d={d} E={E} {dtype} modules={modules} loss={loss.item():.8g} "
          f"-> {os.path.relpath(path, ROOT)} ({os.path.getsize(path) // 1024} KB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("AGILLM41_REFERENCE", "/root/reference/agillm41.py"),
                    help="the reference's agillm41.py (default: $AGILLM41_REFERENCE, else /root/reference/agillm41.py)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    ref = load_reference(args.ref)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for case in AUX_CASES:
        if args.only and args.only not in case[0]:
            continue
        run_case(ref, case, HERE)


if __name__ == "__main__":
    main()
