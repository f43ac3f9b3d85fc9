"""Golden-vector case table for the MoE block forward (oracle; test infrastructure).

Each case names the shapes, seed, dtype and special construction used by
``tests/golden/make_golden.py`` to run the reference ``MoEFFN`` and by the
tests to regenerate identical weights and inputs (checked against the SHA-256
hashes stored in each ``tests/golden/<name>.npz``).

Specials:
* ``ties``  - duplicated router rows give bit-identical logits, i.e. exact ties
  at the top-1, top-2 and 2nd/3rd positions (the reference resolves them with
  ``torch.topk``, agillm41.py:4418).
* ``empty`` - an all-positive input with all-negative router rows for experts 5
  and 9, so those experts receive no tokens (the reference skips them through
  ``rows.numel() == 0``, agillm41.py:4426).
"""
from __future__ import annotations

import torch

from . import reference_moe as orc

CASES = [
    # name, d, H, E, k, N, seed, dtype, shared, shared_H, bias_std, special, store_weights
    ("cfg1_fp32", 1280, 3200, 14, 2, 256, 0, torch.float32, 0, 0, 0.0, None, False),
    ("cfg1_bf16", 1280, 3200, 14, 2, 256, 0, torch.bfloat16, 0, 0, 0.0, None, False),
    ("small_top2_fp32_n17", 64, 128, 14, 2, 17, 11, torch.float32, 0, 0, 0.1, None, False),
    ("small_top2_bf16_n64", 64, 128, 14, 2, 64, 12, torch.bfloat16, 0, 0, 0.1, None, False),
    ("small_top1_bf16_n33", 64, 128, 14, 1, 33, 13, torch.bfloat16, 0, 0, 0.1, None, False),
    ("small_top1_fp32_n9", 64, 192, 6, 1, 9, 14, torch.float32, 0, 0, 0.1, None, False),
    ("small_top3_e4_fp32_n5", 64, 128, 4, 3, 5, 15, torch.float32, 0, 0, 0.1, None, True),
    ("small_shared_bf16_n40", 64, 128, 14, 2, 40, 16, torch.bfloat16, 2, 96, 0.1, None, False),
    ("small_shared_top1_fp32_n24", 64, 256, 2, 1, 24, 17, torch.float32, 1, 128, 0.1, None, False),
    ("small_ties_bf16_n64", 64, 128, 14, 2, 64, 18, torch.bfloat16, 0, 0, 0.1, "ties", False),
    ("small_ties_fp32_n48", 64, 128, 14, 2, 48, 19, torch.float32, 0, 0, 0.1, "ties", False),
    ("small_empty_fp32_n32", 64, 128, 14, 2, 32, 20, torch.float32, 0, 0, 0.1, "empty", False),
    ("edge_n1_bf16", 128, 320, 14, 2, 1, 21, torch.bfloat16, 0, 0, 0.1, None, False),
    ("edge_n2_fp32", 128, 320, 14, 2, 2, 22, torch.float32, 0, 0, 0.1, None, False),
    ("edge_n3_bf16", 128, 320, 14, 2, 3, 23, torch.bfloat16, 0, 0, 0.1, None, False),
    ("edge_n200_d1280_bf16", 1280, 320, 14, 2, 200, 24, torch.bfloat16, 0, 0, 0.05, None, False),
]


# Gradient golden cases (training backward through the reference MoEFFN):
# the same tuple layout as CASES (no shared experts, no stored weights).
GRAD_CASES = [
    ("grad_top2_fp32_n24", 64, 64, 4, 2, 24, 41, torch.float32, 0, 0, 0.1, None, False),
    ("grad_top2_bf16_n24", 64, 64, 4, 2, 24, 42, torch.bfloat16, 0, 0, 0.1, None, False),
    ("grad_top1_fp32_n20", 64, 64, 4, 1, 20, 43, torch.float32, 0, 0, 0.1, None, False),
    ("grad_top1_bf16_n20", 64, 64, 4, 1, 20, 44, torch.bfloat16, 0, 0, 0.1, None, False),
    ("grad_top3_fp32_n16", 64, 96, 5, 3, 16, 45, torch.float32, 0, 0, 0.1, None, False),
    ("grad_empty_fp32_n16", 64, 64, 6, 2, 16, 46, torch.float32, 0, 0, 0.1, "empty", False),
    ("grad_shared_top1_fp32_n20", 64, 64, 2, 1, 20, 47, torch.float32, 1, 128, 0.1, None, False),
    ("grad_shared2_top2_bf16_n24", 64, 64, 4, 2, 24, 48, torch.bfloat16, 2, 64, 0.1, None, False),
]


def grad_output(case):
    """Seeded upstream gradient dL/dout [N, d] (fp32) of a gradient case."""
    (name, d, H, E, k, N, seed, dtype, shared, shared_H, bias_std, special, store_w) = case
    g = torch.Generator().manual_seed(seed + 1000)
    return torch.randn(N, d, generator=g, dtype=torch.float32)


def special_state(sd, special, experts):
    """Apply a case's special construction to an fp32 state dict in place."""
    if special == "ties":
        # Identical router rows give bit-identical logits: exact ties in the
        # top-1, top-2 and 2nd/3rd positions.
        w = sd["router.weight"]
        w[7] = w[3]
        w[2] = w[1]
        w[11] = w[10]
        w[12] = w[10]
    elif special == "empty":
        # With an all-positive input, all-negative router rows never win.
        w = sd["router.weight"]
        empty = (5, 9) if experts == 14 else (1, experts - 2)
        for e in empty:
            w[e] = -w[e].abs() - 0.05
        for e in range(experts):
            if e not in empty:
                w[e] = w[e].abs() + 0.01
    return sd


def case_by_name(name: str):
    for c in CASES + GRAD_CASES:
        if c[0] == name:
            return c
    raise KeyError(name)


def case_inputs(case):
    """Return (fp32 state dict, fp32 input [N, d]) for a case tuple."""
    (name, d, H, E, k, N, seed, dtype, shared, shared_H, bias_std, special, store_w) = case
    sd32 = orc.make_state(d, H, E, seed, dtype=torch.float32, bias_std=bias_std,
                          shared=shared, shared_hidden=shared_H or None)
    sd32 = special_state(sd32, special, E)
    x32 = orc.make_input(N, d, seed)
    if special == "empty":
        x32 = x32.abs() + 0.01
    return sd32, x32
