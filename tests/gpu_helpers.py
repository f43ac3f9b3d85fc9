"""Shared helpers for the GPU parity tests."""
import torch

from oracle import reference_moe

BF16_RTOL, BF16_ATOL = 2e-2, 1e-2   # bf16 output tolerance (reference parity rule)
F32_TOL = 1e-4                      # fp32 mode tolerance


def packed(sd, E, device):
    """Stack the reference state dict into the kernel's [E, ...] layout."""
    w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).to(device).contiguous()
    b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).to(device).contiguous()
    w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).to(device).contiguous()
    b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).to(device).contiguous()
    S = reference_moe.num_shared_in(sd)
    shared = None
    if S:
        shared = tuple(torch.stack([sd[f"shared.{s}.{i}.{p}"] for s in range(S)]).to(device).contiguous()
                       for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")))
    return w1, b1, w2, b2, shared


def explained_index_mismatches(our_idx, ref_idx, our_logits, ref_logits, k):
    """Rows whose top-k indices differ; each must coincide with a logit that
    differs from the reference's (fp32 summation order can flip a bf16
    rounding) or with an exact tie among the reference's top k+1 logits."""
    diff = (our_idx.long() != ref_idx.long()).any(dim=1)
    rows = diff.nonzero().flatten()
    unexplained = []
    E = ref_logits.shape[1]
    kk = min(k + 1, E)
    for t in rows.tolist():
        if not torch.equal(our_logits[t], ref_logits[t]):
            continue
        top = torch.topk(ref_logits[t], kk).values
        if (top[1:] == top[:-1]).any():
            continue
        unexplained.append(t)
    return rows, unexplained


def bf16_ulp(v):
    e = torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -100)))
    return torch.pow(2.0, e - 7)


def assert_close_rows(ours, ref, rows_ok, dtype, term_scale=None, slack=None):
    """Output parity on the rows whose routing matches.

    fp32: every element within 1e-4 (abs and rel).
    bf16/fp16: every element within 1e-2 abs + 2e-2 rel, or (at most 1e-3 of
    the elements) - where the gated
    expert outputs nearly cancel - within two bf16 ulps of the magnitude of
    the summed terms (`term_scale` from the oracle): any two implementations
    whose fp32 accumulation orders differ can round an expert output to
    neighbouring bf16 values, and that step survives the cancellation.
    Without `term_scale`, at most one element in 10^5 may use a 0.0625 bound.
    `slack` (per element, optional) widens the envelope where the gates
    themselves differ from the reference's (see `gate_slack`).
    """
    if dtype == torch.float32:
        torch.testing.assert_close(ours[rows_ok], ref[rows_ok], rtol=F32_TOL, atol=F32_TOL)
        return
    a, b = ours[rows_ok].float(), ref[rows_ok].float()
    diff = (a - b).abs()
    nominal = BF16_ATOL + BF16_RTOL * b.abs()
    outside = diff > nominal
    if term_scale is not None:
        env = torch.maximum(nominal, 2 * bf16_ulp(term_scale[rows_ok].float()))
        if slack is not None:
            env = env + slack[rows_ok]
        bad = diff > env
        assert not bool(bad.any()), (
            f"{int(bad.sum())} elements beyond the rounding envelope (max diff {diff.max().item():.4g})")
        assert int(outside.sum()) <= max(1, int(1e-3 * b.numel())), int(outside.sum())
        return
    n_out = int(outside.sum())
    assert n_out <= max(1, int(1e-5 * b.numel())), (
        f"{n_out} of {b.numel()} elements outside 1e-2 abs / 2e-2 rel (max diff {diff.max().item():.4g})")
    assert bool((diff <= 0.0625 + BF16_RTOL * b.abs()).all()), f"max diff {diff.max().item():.4g}"


def gate_slack(our_gates, ref_gates, term_scale):
    """Output difference a change of gates explains, per element:
    sum_r |dg_r| |y_r| <= max_r(|dg_r| / g_r) * sum_r g_r |y_r| = rel * term_scale."""
    g = ref_gates.float()
    rel = ((our_gates.float() - g).abs() / g.abs().clamp_min(1e-6)).max(dim=1).values
    return rel[:, None] * term_scale.float()
