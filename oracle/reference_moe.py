"""Torch restatement of the reference MoE block forward (oracle; test infrastructure).

Follows ``MoEFFN`` in the reference's ``agillm41.py``:

* constructor / parameter structure  agillm41.py:4324-4360
* expert = Linear(d,H) -> ReLU -> Linear(H,d)  agillm41.py:4332-4336
* forward                            agillm41.py:4389-4431
    - flatten                        4390-4391
    - router logits in weight dtype, then ``.float()``   4398-4399
    - top-1 branch (softmax, argmax, straight-through gate)  4401-4416
    - top-k branch: ``topk`` on the fp32 logits, softmax over the k
      values, cast to the activation dtype                 4418-4419
    - per (rank, expert) ``nonzero`` / ``index_select`` / expert /
      ``* weight`` / ``index_add_`` into ``zeros_like(flat)``  4420-4428
    - shared experts: ``s = shared[0](flat); s = s + shared[i](flat)``,
      ``out = out + s``                                     4381-4387, 4429-4430
* ``_collect_moe_aux`` (load-balance and router-z losses)  agillm41.py:4463-4492

The restatement uses exactly the same torch calls in the same order as the
reference, so on the same device and dtype it reproduces the reference bit for
bit (``tests/golden/make_golden.py`` asserts this against the imported
reference module). Weights are passed as a state-dict mapping with the
reference's keys (``router.weight``, ``experts.{e}.{0,2}.{weight,bias}``,
``shared.{s}.{0,2}.{weight,bias}``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this module.
"""
from __future__ import annotations

from typing import Dict, Mapping, Optional

import torch
import torch.nn.functional as F


def _expert(sd: Mapping[str, torch.Tensor], prefix: str, rows: torch.Tensor) -> torch.Tensor:
    # nn.Sequential(nn.Linear(d, H), nn.ReLU(), nn.Linear(H, d)): agillm41.py:4332-4336
    h = F.linear(rows, sd[prefix + "0.weight"], sd[prefix + "0.bias"])
    h = torch.relu(h)
    return F.linear(h, sd[prefix + "2.weight"], sd[prefix + "2.bias"])


def num_experts_in(sd: Mapping[str, torch.Tensor]) -> int:
    return int(sd["router.weight"].shape[0])


def num_shared_in(sd: Mapping[str, torch.Tensor]) -> int:
    n = 0
    while f"shared.{n}.0.weight" in sd:
        n += 1
    return n


class _ValueOf(torch.autograd.Function):
    """Forward: `value` (a constant); backward: the gradient goes to `t`
    unchanged. Used by ``logits_override`` so that routing follows given
    logits while autograd still runs through the reference's router Linear."""

    @staticmethod
    def forward(ctx, t, value):
        return value.to(device=t.device, dtype=t.dtype).clone()

    @staticmethod
    def backward(ctx, g):
        return g, None


def moe_forward(x: torch.Tensor, sd: Mapping[str, torch.Tensor], top_k: int,
                aux: Optional[Dict[str, torch.Tensor]] = None,
                logits_override: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reference MoE forward (agillm41.py:4389-4431).

    Autograd runs through it as through the reference (the same torch ops),
    so with ``requires_grad`` inputs or weights ``.backward()`` gives the
    reference's gradients, under torch.autocast too.

    ``logits_override`` (optional fp32 [N, E], test plumbing): route with these
    logit values instead of the router GEMM's; gradients still flow through the
    router Linear. Kernels whose router logits differ from the library GEMM's
    by a rounding step can so be compared on identical routing.

    ``aux`` (optional dict) receives ``logits`` (fp32 [N,E]), ``idx`` (int64
    [N,k]), ``gates`` ([N,k], activation dtype), ``counts`` (int64 [E]) and
    ``term_scale`` (fp32 [N,d]): the sum of the magnitudes of the terms added
    into each output element (|y_r * w_r| over ranks, |shared_s| over shared
    experts), which sets the size of the rounding error the result carries.
    Computing it does not change the output.
    """
    E = num_experts_in(sd)
    k = min(max(1, int(top_k)), E)                                  # 4329
    orig_shape = x.shape
    flat = x.reshape(-1, orig_shape[-1])                             # 4391
    wr = sd["router.weight"]
    router_in = flat.to(wr.dtype) if flat.dtype != wr.dtype else flat  # 4398
    scores = F.linear(router_in, wr).float()                         # 4399
    if logits_override is not None:
        scores = _ValueOf.apply(scores, logits_override)
    n_shared = num_shared_in(sd)

    scale = torch.zeros(flat.shape, dtype=torch.float32, device=flat.device) if aux is not None else None
    if k == 1:                                                       # 4401-4416
        probs = scores.softmax(dim=-1)
        chosen = probs.argmax(dim=-1)
        out = torch.zeros_like(flat)
        for e in range(E):
            mask = chosen == e
            if not bool(mask.any()):
                continue
            gate = probs[mask, e].to(flat.dtype).clamp_min(1e-6)
            gate_st = (gate / gate.detach()).unsqueeze(-1)
            out[mask] = _expert(sd, f"experts.{e}.", flat[mask]) * gate_st
            if aux is not None:
                scale[mask] = out[mask].float().abs()
        idx = chosen.unsqueeze(-1)
        gates = torch.ones_like(idx, dtype=flat.dtype)
    else:
        vals, idx = torch.topk(scores, k=k, dim=-1)                  # 4418
        weights = vals.softmax(dim=-1).to(flat.dtype)                # 4419
        out = torch.zeros_like(flat)                                 # 4420
        for rank in range(k):                                        # 4421
            chosen = idx[:, rank]
            weight = weights[:, rank].unsqueeze(-1)
            for e in range(E):                                       # 4424
                rows = (chosen == e).nonzero(as_tuple=False).flatten()
                if rows.numel() == 0:
                    continue
                term = _expert(sd, f"experts.{e}.", flat.index_select(0, rows)) * weight.index_select(0, rows)
                out.index_add_(0, rows, term)                        # 4428
                if aux is not None:
                    scale.index_add_(0, rows, term.float().abs())
        gates = weights
    if n_shared > 0:                                                 # 4429-4430, 4381-4387
        s = _expert(sd, "shared.0.", flat)
        if aux is not None:
            scale += s.float().abs()
        for i in range(1, n_shared):
            si = _expert(sd, f"shared.{i}.", flat)
            s = s + si
            if aux is not None:
                scale += si.float().abs()
        out = out + s
    if aux is not None:
        aux["logits"] = scores
        aux["idx"] = idx
        aux["gates"] = gates
        aux["counts"] = torch.bincount(idx.reshape(-1), minlength=E)
        aux["term_scale"] = scale.reshape(orig_shape)
    return out.reshape(orig_shape)


def collect_moe_aux(router_inputs, router_weights, aux_coef: float = 0.0, z_coef: float = 0.0,
                    scores_override=None):
    """Restatement of ``_collect_moe_aux`` (agillm41.py:4463-4492) over the
    (stashed router input, router weight) pairs of the MoE modules in module
    order: the load-balance loss ``aux_coef * E * sum(load * importance)`` and
    the router-z loss ``z_coef * mean(logsumexp(scores) ** 2)`` with the same
    torch calls in the same order (the router is the bias-free Linear of
    agillm41.py:4332), so autograd through it gives the reference's gradients.
    An input of None (nothing stashed) is skipped. Returns a scalar tensor or
    0.0.

    ``scores_override`` (test-only, one entry per module or None): the given
    fp32 logit values replace the router's in the forward while the gradient
    still flows through the reference's router Linear, so that a kernel
    whose logits round differently can be compared on identical argmax."""
    total = None
    overrides = scores_override if scores_override is not None else [None] * len(router_inputs)
    for inp, w, ov in zip(router_inputs, router_weights, overrides):
        if inp is None or (aux_coef <= 0 and z_coef <= 0):                 # 4478
            continue
        router_in = inp.to(w.dtype) if inp.dtype != w.dtype else inp        # 4481
        scores = F.linear(router_in, w).float()                             # 4482
        if ov is not None:
            scores = _ValueOf.apply(scores, ov)
        probs = scores.softmax(dim=-1)                                      # 4483
        importance = probs.mean(dim=0)                                      # 4484
        top1 = probs.argmax(dim=-1)                                         # 4485
        n_exp = w.shape[0]
        load = torch.bincount(top1, minlength=n_exp).to(importance.dtype) / max(1, top1.numel())  # 4486
        if aux_coef > 0:
            lb = aux_coef * n_exp * (load.detach() * importance).sum()     # 4487-4489
            total = lb if total is None else total + lb
        if z_coef > 0:
            zl = z_coef * (torch.logsumexp(scores, dim=-1) ** 2).mean()     # 4490-4491
            total = zl if total is None else total + zl
    return total if total is not None else 0.0


# Seeded synthetic weights and inputs (the workload definitions) live in the
# package so that the benchmark can build its workload without the oracle.
from agillm41_b200.synthetic import BIAS_ALPHA, make_input, make_state, zipf_logit_bias  # noqa: E402,F401
