"""Seeded synthetic workloads for the MoE block (benchmarks and tests).

Weights and inputs are drawn from CPU ``torch.Generator`` streams, so a seed
gives the same tensors on every host; weights carry the reference module's
state-dict keys (agillm41.py:4331-4351) so they load into either module.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch


def make_state(d: int, hidden: int, experts: int, seed: int, *, dtype=torch.float32,
               device="cpu", w_std: float = 0.02, bias_std: float = 0.0,
               shared: int = 0, shared_hidden: Optional[int] = None,
               router_logit_bias: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
    """Seeded synthetic weights with the reference's state-dict keys.

    Draw order (one CPU ``torch.Generator`` seeded with ``seed``): router
    ``[E,d]``, then for e = 0..E-1 ``W1 [H,d]`` and ``W2 [d,H]``, then (only if
    ``bias_std > 0``) for e = 0..E-1 ``b1 [H]`` and ``b2 [d]``, then shared
    experts the same way. Weights ~ N(0, w_std^2); biases zero unless
    ``bias_std > 0``. Values are drawn in fp32 and then cast, so the bf16 state
    is the rounding of the fp32 one.
    """
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    sd: Dict[str, torch.Tensor] = {}
    sd["router.weight"] = torch.randn(experts, d, generator=g) * w_std
    for e in range(experts):
        sd[f"experts.{e}.0.weight"] = torch.randn(hidden, d, generator=g) * w_std
        sd[f"experts.{e}.2.weight"] = torch.randn(d, hidden, generator=g) * w_std
    for e in range(experts):
        if bias_std > 0:
            sd[f"experts.{e}.0.bias"] = torch.randn(hidden, generator=g) * bias_std
            sd[f"experts.{e}.2.bias"] = torch.randn(d, generator=g) * bias_std
        else:
            sd[f"experts.{e}.0.bias"] = torch.zeros(hidden)
            sd[f"experts.{e}.2.bias"] = torch.zeros(d)
    sh = int(shared_hidden or hidden)
    for s in range(int(shared)):
        sd[f"shared.{s}.0.weight"] = torch.randn(sh, d, generator=g) * w_std
        sd[f"shared.{s}.2.weight"] = torch.randn(d, sh, generator=g) * w_std
        if bias_std > 0:
            sd[f"shared.{s}.0.bias"] = torch.randn(sh, generator=g) * bias_std
            sd[f"shared.{s}.2.bias"] = torch.randn(d, generator=g) * bias_std
        else:
            sd[f"shared.{s}.0.bias"] = torch.zeros(sh)
            sd[f"shared.{s}.2.bias"] = torch.zeros(d)
    if router_logit_bias is not None:
        # A router has no bias term (agillm41.py:4331). A per-expert logit
        # offset b_e is carried by the weights instead: every row gets
        # b_e / ALPHA on input feature 0, and ``make_input`` pins feature 0
        # to ALPHA, so logit_e = W_e[1:] . x[1:] + b_e (up to the rounding of b_e / ALPHA).
        sd["router.weight"][:, 0] = router_logit_bias.float() / BIAS_ALPHA
    return {k: v.to(dtype=dtype, device=device) for k, v in sd.items()}


BIAS_ALPHA = 4.0


def make_input(n_tokens: int, d: int, seed: int, *, dtype=torch.float32, device="cpu",
               batch: Optional[int] = None, pin_feature0: bool = False) -> torch.Tensor:
    """x ~ N(0,1), drawn after the weights from its own generator (seed+1000003).

    With ``pin_feature0`` the first feature is set to the constant used by
    ``make_state(router_logit_bias=...)``.
    """
    g = torch.Generator(device="cpu").manual_seed(int(seed) + 1000003)
    x = torch.randn(n_tokens, d, generator=g)
    if pin_feature0:
        x[:, 0] = BIAS_ALPHA
    if batch is not None:
        x = x.reshape(batch, n_tokens // batch, d)
    return x.to(dtype=dtype, device=device)


def zipf_logit_bias(experts: int, seed: int, s: float = 1.2, scale: float = 1.0) -> torch.Tensor:
    """Per-expert logit offsets log(p_e) * scale with p ∝ Zipf(s) over a
    seeded permutation of the experts (the skewed-routing workload)."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    perm = torch.randperm(experts, generator=g)
    ranks = torch.empty(experts)
    ranks[perm] = torch.arange(1, experts + 1, dtype=torch.float32)
    p = ranks.pow(-s)
    p = p / p.sum()
    return torch.log(p) * float(scale)
