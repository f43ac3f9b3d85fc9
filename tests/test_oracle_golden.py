"""The oracle is pinned to the reference: regenerated inputs hash-match the
golden vectors, and the torch restatement reproduces the reference outputs."""
import numpy as np
import pytest
import torch

from golden_io import Golden, names
from oracle import permute_oracle, reference_moe


@pytest.mark.parametrize("name", names())
def test_inputs_regenerate(name):
    g = Golden(name)
    assert g.inputs_match(), f"{name}: regenerated weights/input differ from the ones the golden vector was made with"


@pytest.mark.parametrize("name", names())
def test_oracle_reproduces_reference(name):
    g = Golden(name)
    aux = {}
    with torch.no_grad():
        out = reference_moe.moe_forward(g.x, g.sd, g.top_k, aux=aux)
    assert torch.equal(aux["counts"], g.counts)
    assert torch.equal(aux["idx"], g.idx)
    if g.dtype == torch.float32:
        # Same torch ops on the same CPU kernels: equal up to BLAS blocking.
        torch.testing.assert_close(out, g.out, rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(aux["logits"], g.logits, rtol=1e-6, atol=1e-6)
    else:
        torch.testing.assert_close(out.float(), g.out.float(), rtol=1e-2, atol=1e-2)
        assert torch.equal(aux["logits"], g.logits)


@pytest.mark.parametrize("name", ["cfg1_fp32", "small_top2_fp32_n17", "small_ties_fp32_n48"])
def test_planted_oracle_mistake_is_caught(name):
    """A wrong oracle (renormalisation over all experts instead of the k
    chosen, a common MoE variant) must not pass the golden check."""
    g = Golden(name)
    sd = g.sd
    flat = g.x.reshape(-1, g.d)
    scores = torch.nn.functional.linear(flat, sd["router.weight"]).float()
    vals, idx = torch.topk(scores, g.top_k, dim=-1)
    wrong = scores.softmax(-1).gather(1, idx).to(flat.dtype)   # planted mistake
    out = torch.zeros_like(flat)
    for r in range(g.top_k):
        for e in range(g.E):
            rows = (idx[:, r] == e).nonzero().flatten()
            if rows.numel():
                y = reference_moe._expert(sd, f"experts.{e}.", flat.index_select(0, rows))
                out.index_add_(0, rows, y * wrong[rows, r:r + 1])
    assert not torch.allclose(out, g.out, rtol=1e-4, atol=1e-4)


def test_dispatch_layout_fast_matches_loop():
    rng = np.random.default_rng(0)
    for n, k, E in [(1, 1, 1), (5, 2, 14), (257, 2, 14), (300, 3, 7), (1000, 1, 2)]:
        idx = np.stack([rng.permutation(E)[:k] for _ in range(n)])
        a = permute_oracle.dispatch_layout(idx, E)
        b = permute_oracle.dispatch_layout_fast(idx, E)
        for u, v in zip(a, b):
            np.testing.assert_array_equal(u, v)


@pytest.mark.parametrize("name", names())
def test_dispatch_layout_on_golden(name):
    g = Golden(name)
    counts, seg, row_of, token_of, tile_expert = permute_oracle.dispatch_layout(g.idx.numpy(), g.E)
    np.testing.assert_array_equal(counts, g.counts.numpy())
    # Every (token, rank) has a distinct row; rows within a segment ascend by token.
    assert len(set(row_of.reshape(-1).tolist())) == row_of.size
    for e in range(g.E):
        toks = token_of[seg[e]:seg[e] + counts[e]]
        assert (np.diff(toks) > 0).all()
        assert (token_of[seg[e] + counts[e]:seg[e + 1]] == -1).all()
        # The reference's rows for expert e are its nonzero() over ranks: the same set.
        ref_rows = sorted(np.nonzero((g.idx.numpy() == e).any(axis=1))[0].tolist())
        assert toks.tolist() == ref_rows
    assert len(tile_expert) * 128 == seg[-1]


def test_make_state_draw_order_is_stable():
    a = reference_moe.make_state(16, 32, 3, 5)
    b = reference_moe.make_state(16, 32, 3, 5)
    for k in a:
        assert torch.equal(a[k], b[k])
    assert list(a)[:3] == ["router.weight", "experts.0.0.weight", "experts.0.2.weight"]
