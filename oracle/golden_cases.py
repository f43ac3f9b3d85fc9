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


# Auxiliary-loss golden cases (_collect_moe_aux, agillm41.py:4463-4492):
# (name, d, experts, n_tokens, seed, dtype, aux_coef, z_coef, modules,
#  upstream gradient, special). "zero_rows" zeroes every 7th input row, so
# those tokens' probabilities tie and argmax takes the first expert.
AUX_CASES = [
    ("aux_lb_z_fp32_e14_n300", 64, 14, 300, 61, torch.float32, 0.01, 0.001, 1, 1.0, None),
    ("aux_lb_z_bf16_e2_n257", 64, 2, 257, 62, torch.bfloat16, 0.01, 0.001, 1, 1.0, None),
    ("aux_lb_only_fp32_e8_n128", 64, 8, 128, 63, torch.float32, 0.05, 0.0, 1, 1.0, None),
    ("aux_z_only_fp32_e16_n96", 64, 16, 96, 64, torch.float32, 0.0, 0.01, 1, 1.0, None),
    ("aux_two_modules_fp32_e4_n200", 64, 4, 200, 65, torch.float32, 0.01, 0.001, 2, 1024.0, None),
    ("aux_ties_fp32_e6_n140", 64, 6, 140, 66, torch.float32, 0.02, 0.002, 1, 1.0, "zero_rows"),
]


def aux_case_inputs(case):
    """Return [(fp32 stashed input [N, d], fp32 router weight [E, d])] per module."""
    (name, d, E, N, seed, dtype, aux_coef, z_coef, modules, gscale, special) = case
    out = []
    for i in range(modules):
        w = orc.make_state(d, d, E, seed + 100 * i, dtype=torch.float32)["router.weight"]
        x = orc.make_input(N, d, seed + 100 * i)
        if special == "zero_rows":
            x[::7] = 0
        out.append((x, w))
    return out


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
    for c in CASES + GRAD_CASES + AUX_CASES:
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


# Tensor-codec golden cases (agillm41.py:4858-5102): the encoder modes, and
# the side-update applications (name, alpha, delta) of agillm41.py:6035-6045.
CODEC_MODES = ["int8-zstd", "rowq8-zstd", "fp16-zstd", "zstd", "adaptive-zstd"]
CODEC_APPLY = [("copy", 1.0, False), ("lerp03", 0.3, False), ("lerp075", 0.75, False), ("add05", 0.5, True)]
CODEC_APPLY_KEYS = ["experts.0.0.weight", "experts.1.0.weight", "experts.1.2.bias", "shared.0.0.weight"]


def codec_state():
    """A small seeded MoE-layer state: two experts (expert 1's FC1 weight has
    an outlier row), the router, and a bf16 shared-expert weight. Weights are
    drawn at the scale of trained block weights (std 0.02), so the adaptive
    mode's error budget picks int8 for some tensors and row-wise int8 or fp16
    for others."""
    g = torch.Generator().manual_seed(91)
    d, H, E = 64, 96, 2
    sd = {}
    for e in range(E):
        sd[f"experts.{e}.0.weight"] = torch.randn(H, d, generator=g) * 0.02
        sd[f"experts.{e}.0.bias"] = torch.randn(H, generator=g) * 0.01
        sd[f"experts.{e}.2.weight"] = torch.randn(d, H, generator=g) * 0.02
        sd[f"experts.{e}.2.bias"] = torch.randn(d, generator=g) * 0.01
    sd["experts.1.0.weight"][7] = torch.linspace(-4.0, 4.0, d)   # one outlier row: row-wise int8
    sd["experts.1.2.bias"] *= 200.0                               # large 1-D values: fp16
    sd["router.weight"] = torch.randn(E, d, generator=g) * 0.05
    sd["shared.0.0.weight"] = (torch.randn(2 * d, d, generator=g) * 0.02).to(torch.bfloat16)
    return sd


def codec_target(key, shape, dtype):
    """Seeded target tensor that a decoded value is applied to."""
    g = torch.Generator().manual_seed(92 + sum(map(ord, key)))
    return (torch.randn(tuple(shape), generator=g) * 0.02).to(dtype)
