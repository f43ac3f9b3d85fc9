"""Kernel-level parity on the GPU: each stage against the oracle / torch."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from agillm41_b200 import _lib, ops
from agillm41_b200._lib import read_device_error
from oracle import permute_oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _err():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


def _ref_grouped(a, w, bias, tile_group, relu):
    """Per-tile fp32 (or fp64) reference of the grouped GEMM."""
    acc = torch.float64 if a.dtype == torch.float64 else torch.float32
    ref = torch.zeros(a.shape[0], w.shape[1], dtype=acc, device=a.device)
    for m, gi in enumerate(tile_group.tolist()):
        r = slice(m * 128, (m + 1) * 128)
        ref[r] = a[r].to(acc) @ w[gi].to(acc).T + (0 if bias is None else bias[gi].to(acc))
    return ref.relu() if relu else ref


def _tie_logits(n, E, seed, grid=0.25):
    g = torch.Generator(device="cpu").manual_seed(seed)
    # Coarse values force many exact ties at every top-k position.
    return (torch.randint(-8, 9, (n, E), generator=g).float() * grid).to(DEV)


@pytest.mark.parametrize("k", [2, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_topk_bit_exact_from_reference_logits(k, dtype):
    """Given the reference's fp32 logits, indices and gates match torch.topk +
    softmax on this GPU bit for bit, ties included (agillm41.py:4418-4419)."""
    n, E, d = 5000, 14, 64
    logits = _tie_logits(n, E, seed=k)
    ref_vals, ref_idx = torch.topk(logits, k, dim=-1)
    ref_gates = ref_vals.softmax(dim=-1).to(dtype)
    x = torch.zeros(n, d, dtype=dtype, device=DEV)
    w = torch.zeros(E, d, dtype=dtype, device=DEV)
    err = _err()
    idx, gates, hist, _ = ops.router_topk(x, w, k, logits_in=logits, err=err)
    assert read_device_error(err) == 0
    bad = (idx.long() != ref_idx).any(1)
    assert int(bad.sum()) == 0, (
        f"{int(bad.sum())} rows differ; first: ours {idx[bad][:3].tolist()} ref {ref_idx[bad][:3].tolist()} "
        f"logits {logits[bad][:3].tolist()}")
    assert torch.equal(gates, ref_gates)
    counts = torch.bincount(ref_idx.flatten(), minlength=E)
    assert torch.equal(hist.sum(0).long(), counts)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_top1_bit_exact_from_reference_logits(dtype):
    """Top-1 branch: chosen = argmax(softmax(scores)) (agillm41.py:4402-4403)."""
    n, E, d = 3000, 14, 64
    logits = _tie_logits(n, E, seed=7)
    ref = logits.softmax(-1).argmax(-1)
    x = torch.zeros(n, d, dtype=dtype, device=DEV)
    w = torch.zeros(E, d, dtype=dtype, device=DEV)
    idx, gates, hist, _ = ops.router_topk(x, w, 1, logits_in=logits)
    assert torch.equal(idx[:, 0].long(), ref)
    assert torch.equal(gates, torch.ones_like(gates))


def _ulp(v, dtype):
    """Spacing of the floating-point grid of `dtype` at |v| (as fp32)."""
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    e = torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -60)))
    if dtype == torch.float16:
        e = e.clamp_min(-14)
    return torch.pow(2.0, e - mant)


@pytest.mark.parametrize("dtype,n,d,E,k", [
    (torch.bfloat16, 4096, 1280, 14, 2),
    (torch.bfloat16, 777, 64, 14, 2),
    (torch.float32, 1000, 1280, 14, 2),
    (torch.float16, 513, 256, 6, 3),
    (torch.bfloat16, 300, 128, 2, 1),
])
def test_router_logits_and_selection(dtype, n, d, E, k):
    """The router kernel's logits are the exact dot products rounded once to
    the activation dtype (checked against fp64), and every index difference
    from the reference's `router(x).float()` + topk is explained by a logit
    the reference's library GEMM rounded differently or by an exact tie."""
    g = torch.Generator(device="cpu").manual_seed(n + d)
    x = torch.randn(n, d, generator=g).to(dtype).to(DEV)
    w = (torch.randn(E, d, generator=g) * 0.02).to(dtype).to(DEV)
    ref_logits = F.linear(x, w).float()
    exact = (x.double() @ w.double().T)
    err = _err()
    idx, gates, hist, logits = ops.router_topk(x, w, k, want_logits=True, err=err)
    assert read_device_error(err) == 0
    rounded = exact.to(dtype).float()
    if dtype == torch.float32:
        torch.testing.assert_close(logits, exact.float(), rtol=2e-6, atol=2e-6)
    else:
        # fp32 accumulation then one rounding: equal to the correctly rounded
        # dot product except where the fp32 sum straddles a rounding boundary
        # (for a near-zero logit the fp32 error, ~1e-6 of sum |x w|, can exceed
        # one ulp of the tiny result).
        mag = (x.double().abs() @ w.double().abs().T).float()
        assert ((logits - rounded).abs() <= _ulp(rounded, dtype) + 1e-6 * mag).all()
        assert (logits == rounded).float().mean().item() > 0.995
    if k == 1:
        ref_idx = ref_logits.softmax(-1).argmax(-1, keepdim=True)
    else:
        ref_idx = torch.topk(ref_logits, k, -1).indices
    from gpu_helpers import explained_index_mismatches
    rows, unexplained = explained_index_mismatches(idx, ref_idx, logits, ref_logits, k)
    assert not unexplained, f"unexplained index mismatches at rows {unexplained[:10]}"
    assert rows.numel() <= max(3, n // 50)
    print(f"router {dtype} n={n} d={d}: logits differing from the library GEMM "
          f"{(logits != ref_logits).float().mean().item():.3%}, index rows differing {rows.numel()}")


@pytest.mark.parametrize("n,E,k", [(1, 14, 2), (3, 14, 2), (257, 14, 2), (4099, 14, 2), (1000, 7, 3), (513, 2, 1),
                                   (20000, 14, 2)])
def test_dispatch_plan_and_permute_exact(n, E, k):
    d = 256
    g = torch.Generator(device="cpu").manual_seed(n)
    # Skewed routing: expert 0 hot, expert E-1 never chosen (when E > k + 1).
    p = torch.ones(E)
    p[0] = 5.0
    if E > k + 1:
        p[E - 1] = 0.0
    idx_np = torch.multinomial(p.expand(n, E), k, replacement=False, generator=g).numpy()
    idx = torch.from_numpy(idx_np.astype(np.int32)).to(DEV)
    x = torch.randn(n, d, generator=g).to(torch.bfloat16).to(DEV)
    # Build block histograms the way the router kernel does.
    nb = ops.dispatch_blocks(n)
    hist = torch.zeros(nb, E, dtype=torch.int32)
    for b in range(nb):
        seg = idx_np[b * _lib.AGM_DISPATCH_BLOCK:(b + 1) * _lib.AGM_DISPATCH_BLOCK].reshape(-1)
        hist[b] = torch.from_numpy(np.bincount(seg, minlength=E).astype(np.int32))
    hist = hist.to(DEV)
    err = _err()
    plan = ops.dispatch_plan(hist, n, k, err=err)
    x_perm, row_of = ops.permute(x, idx, plan, E, err=err)
    assert read_device_error(err) == 0
    counts, seg, row_of_ref, token_of_ref, tile_expert = permute_oracle.dispatch_layout_fast(idx_np, E)
    np.testing.assert_array_equal(plan["counts"].cpu().numpy(), counts)
    np.testing.assert_array_equal(plan["seg_start"].cpu().numpy(), seg)
    assert int(plan["num_tiles"].item()) == len(tile_expert)
    np.testing.assert_array_equal(plan["tile_expert"][:len(tile_expert)].cpu().numpy(), tile_expert)
    np.testing.assert_array_equal(row_of.cpu().numpy(), row_of_ref)
    total = int(seg[-1])
    np.testing.assert_array_equal(plan["token_of"][:total].cpu().numpy(), token_of_ref)
    tok = torch.from_numpy(token_of_ref).to(DEV)
    filled = tok >= 0
    assert torch.equal(x_perm[:total][filled], x[tok[filled]])
    assert torch.count_nonzero(x_perm[:total][~filled]) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows_per_group,N,K,relu,bn", [
    ([128, 256, 0, 384], 3200, 1280, True, 0),
    ([128, 256, 0, 384], 1280, 3200, False, 0),
    ([128, 128], 200, 96, True, 128),
    ([256], 256, 64, False, 256),
    ([128, 0, 0, 128], 320, 1280, True, 256),
    ([384, 128, 256], 1280, 320, False, 128),
])
def test_grouped_gemm_tc(dtype, rows_per_group, N, K, relu, bn):
    """tcgen05 grouped GEMM vs an fp32 torch matmul of the same bf16/fp16 operands."""
    G = len(rows_per_group)
    g = torch.Generator(device="cpu").manual_seed(N + K)
    rows = sum(rows_per_group)
    a = torch.randn(rows, K, generator=g).to(dtype).to(DEV)
    w = (torch.randn(G, N, K, generator=g) * 0.05).to(dtype).to(DEV)
    bias = (torch.randn(G, N, generator=g) * 0.1).to(dtype).to(DEV)
    tile_group = torch.tensor(sum([[gi] * (r // 128) for gi, r in enumerate(rows_per_group)], []),
                              dtype=torch.int32, device=DEV)
    num_tiles = torch.tensor([tile_group.numel()], dtype=torch.int32, device=DEV)
    err = _err()
    c = ops.grouped_gemm(a, w, bias, relu=relu, tile_group=tile_group, num_tiles=num_tiles,
                         max_tiles=tile_group.numel() + 2, force_bn=bn, err=err)
    assert read_device_error(err) == 0
    ref = _ref_grouped(a, w, bias, tile_group, relu)
    torch.testing.assert_close(c.float(), ref.to(dtype).float(), rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows_per_group,N,K,relu", [
    ([256, 512, 0, 768], 3200, 1280, True),    # FC1 shape, partial last column tile
    ([256, 512, 0, 768], 1280, 3200, False),   # FC2 shape
    ([256, 384], 1280, 1280, True),            # odd tile count: the last pair has one tile
    ([256], 192, 64, False),                   # one column tile narrower than 256
    ([0, 256, 256], 320, 320, True),
])
def test_grouped_gemm_pair(dtype, rows_per_group, N, K, relu):
    """CTA-pair (cta_group::2, 256 x 256 tiles) grouped GEMM vs an fp32 torch matmul."""
    G = len(rows_per_group)
    g = torch.Generator(device="cpu").manual_seed(N + K + 7)
    rows = sum(rows_per_group)
    a = torch.randn(rows, K, generator=g).to(dtype).to(DEV)
    w = (torch.randn(G, N, K, generator=g) * 0.05).to(dtype).to(DEV)
    bias = (torch.randn(G, N, generator=g) * 0.1).to(dtype).to(DEV)
    tile_group = torch.tensor(sum([[gi] * (r // 128) for gi, r in enumerate(rows_per_group)], []),
                              dtype=torch.int32, device=DEV)
    num_tiles = torch.tensor([tile_group.numel()], dtype=torch.int32, device=DEV)
    err = _err()
    c = ops.grouped_gemm(a, w, bias, relu=relu, tile_group=tile_group, num_tiles=num_tiles,
                         max_tiles=tile_group.numel(), force_bn=_lib.AGM_GEMM_PAIR, err=err)
    assert read_device_error(err) == 0
    ref = _ref_grouped(a, w, bias, tile_group, relu)
    torch.testing.assert_close(c.float(), ref.to(dtype).float(), rtol=1e-2, atol=2e-2)
    # Same products as the one-CTA kernel: both accumulate in fp32 over K in the same order.
    c1 = ops.grouped_gemm(a, w, bias, relu=relu, tile_group=tile_group, num_tiles=num_tiles,
                          max_tiles=tile_group.numel(), force_bn=256, err=err)
    assert torch.equal(c, c1)


def test_grouped_gemm_pair_group_mismatch_flagged():
    """Row tiles 0 and 1 in different groups cannot share a pair: the kernel
    sets the device error bit (and still terminates normally)."""
    a = torch.randn(256, 128, device=DEV).to(torch.bfloat16)
    w = (torch.randn(2, 256, 128, device=DEV) * 0.05).to(torch.bfloat16)
    tile_group = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    err = _err()
    ops.grouped_gemm(a, w, None, relu=False, tile_group=tile_group, max_tiles=2, force_bn=_lib.AGM_GEMM_PAIR,
                     err=err)
    assert read_device_error(err) & (1 << 7)


def test_grouped_gemm_tc_device_tile_count():
    """Tiles beyond the device-side count are not computed (decode-sized case)."""
    dtype = torch.bfloat16
    a = torch.randn(512, 1280, device=DEV).to(dtype)
    w = (torch.randn(2, 1280, 1280, device=DEV) * 0.02).to(dtype)
    tile_group = torch.tensor([0, 1, 1, 0], dtype=torch.int32, device=DEV)
    num_tiles = torch.tensor([2], dtype=torch.int32, device=DEV)
    c = ops.grouped_gemm(a, w, None, relu=False, tile_group=tile_group, num_tiles=num_tiles, max_tiles=4)
    c.zero_()
    c = ops.grouped_gemm(a, w, None, relu=False, tile_group=tile_group, num_tiles=num_tiles, max_tiles=4)
    ref0 = a[:128].float() @ w[0].float().T
    ref1 = a[128:256].float() @ w[1].float().T
    torch.testing.assert_close(c[:128].float(), ref0, rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(c[128:256].float(), ref1, rtol=1e-2, atol=2e-2)


def test_grouped_gemm_f32():
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(384, 320, device=DEV)
    w = torch.randn(2, 200, 320, device=DEV) * 0.05
    bias = torch.randn(2, 200, device=DEV)
    tile_group = torch.tensor([1, 0, 1], dtype=torch.int32, device=DEV)
    c = ops.grouped_gemm(a, w, bias, relu=True, tile_group=tile_group, max_tiles=3)
    ref = _ref_grouped(a.double(), w.double(), bias.double(), tile_group, True).float()
    torch.testing.assert_close(c, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("k,S", [(2, 0), (1, 0), (3, 2), (2, 1)])
def test_combine_reference_rounding(dtype, k, S):
    """Bit-exact against the reference's op sequence: zeros, index_add_ of
    y*w per rank, then + (shared sum)."""
    n, d, rows = 1000, 1280, 4000
    g = torch.Generator(device="cpu").manual_seed(k * 10 + S)
    y = torch.randn(rows, d, generator=g).to(dtype).to(DEV)
    row_of = torch.stack([torch.randperm(rows, generator=g)[:n] for _ in range(k)], 1).to(torch.int32).to(DEV)
    gates = torch.rand(n, k, generator=g).to(dtype).to(DEV)
    shared_y = torch.randn(S, n, d, generator=g).to(dtype).to(DEV) if S else None
    out = ops.combine(y, row_of, gates, shared_y)
    ref = torch.zeros(n, d, dtype=dtype, device=DEV)
    ar = torch.arange(n, device=DEV)
    for r in range(k):
        ref.index_add_(0, ar, y[row_of[:, r].long()] * gates[:, r:r + 1])
    if S:
        s = shared_y[0]
        for i in range(1, S):
            s = s + shared_y[i]
        ref = ref + s
    assert torch.equal(out, ref)
