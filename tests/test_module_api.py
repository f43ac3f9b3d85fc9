"""The B200 module keeps the reference MoEFFN interface (CPU-only checks).

Where the reference checkout is present (the build container), the tests also
load it and check drop-in compatibility against the real class; elsewhere
those cases are skipped.
"""
import importlib.util
import os
import sys

import pytest
import torch

import agillm41_b200
from agillm41_b200 import MoEFFN, MoEKernelError

from conftest import REFERENCE_PY as REF


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF):
        pytest.skip("reference checkout not present")
    os.environ.setdefault("AGILLM_SYNTHETIC_TOKENIZER", "1")
    os.environ.setdefault("AGILLM_SYNTHETIC_VOCAB", "32000")
    if "agillm41" in sys.modules:
        return sys.modules["agillm41"]
    spec = importlib.util.spec_from_file_location("agillm41", REF)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["agillm41"] = mod
    spec.loader.exec_module(mod)
    return mod


def expected_keys(E, S):
    keys = ["router.weight"]
    for e in range(E):
        keys += [f"experts.{e}.0.weight", f"experts.{e}.0.bias", f"experts.{e}.2.weight", f"experts.{e}.2.bias"]
    for s in range(S):
        keys += [f"shared.{s}.0.weight", f"shared.{s}.0.bias", f"shared.{s}.2.weight", f"shared.{s}.2.bias"]
    return keys


@pytest.mark.parametrize("kw", [dict(experts=14, top_k=2, mlp_mult=4), dict(experts=2, top_k=1, mlp_mult=4,
                                                                          shared_experts=1, shared_mlp_mult=2),
                                dict(experts=1, top_k=3), dict(experts=4, top_k=0)])
def test_constructor_and_keys(kw):
    m = MoEFFN(64, **kw)
    E = max(1, kw.get("experts", 4))
    assert m.num_experts == E
    assert m.top_k == min(max(1, kw.get("top_k", 1)), E)
    assert list(m.state_dict()) == expected_keys(E, kw.get("shared_experts", 0))
    assert m.experts[0][0].weight.shape == (m.mlp_mult * 64, 64)
    if kw.get("shared_experts"):
        assert m.shared[0][0].weight.shape == (2 * 64, 64)
        assert torch.count_nonzero(m.shared[0][2].weight) == 0
    for attr in ("d", "mlp_mult", "num_experts", "top_k", "num_shared", "last_router_input", "expert_stream",
                 "expert_stream_empty_cache", "expert_stream_stats"):
        assert hasattr(m, attr)
    assert m.set_expert_stream(True, empty_cache=False) is m and m.expert_stream and not m.expert_stream_empty_cache


def test_matches_reference_class(ref):
    for kw in (dict(experts=14, top_k=2, mlp_mult=4), dict(experts=2, top_k=1, mlp_mult=4, shared_experts=1,
                                                           shared_mlp_mult=2)):
        a = MoEFFN(64, **kw)
        b = ref.MoEFFN(64, **kw)
        sa, sb = a.state_dict(), b.state_dict()
        assert list(sa) == list(sb)
        for k in sa:
            assert sa[k].shape == sb[k].shape and sa[k].dtype == sb[k].dtype
        assert set(vars(b)) - set(vars(a)) == set()
        # A reference checkpoint loads into the B200 module and back, strictly.
        a.load_state_dict(sb)
        b.load_state_dict(a.state_dict())


def test_legacy_dense_ffn_seeding_matches_reference(ref):
    torch.manual_seed(0)
    dense = torch.nn.Sequential(torch.nn.Linear(64, 256), torch.nn.ReLU(), torch.nn.Linear(256, 64))
    legacy = {k: v.clone() for k, v in dense.state_dict().items()}
    a = MoEFFN(64, experts=3, top_k=1)
    b = ref.MoEFFN(64, experts=3, top_k=1)
    a.load_state_dict(dict(legacy), strict=False)
    b.load_state_dict(dict(legacy), strict=False)
    for e in range(3):
        assert torch.equal(a.experts[e][0].weight, dense[0].weight)
        assert torch.equal(b.experts[e][2].bias, dense[2].bias)


def test_install_into_reference(ref):
    cls = agillm41_b200.install(ref)
    try:
        assert ref.MoEFFN is cls and issubclass(cls, cls._reference_class)
        blk = ref.Block(64, 4, 16, moe_ffn=True, moe_experts=14, moe_top_k=2, moe_mlp_mult=2)
        assert isinstance(blk.ff, cls) and isinstance(blk.ff, cls._reference_class)
        assert list(blk.ff.state_dict()) == expected_keys(14, 0)
        # _collect_moe_aux sees the module through the reference's global name.
        blk.train()
        with pytest.raises(MoEKernelError):
            blk.ff(torch.randn(2, 3, 64))     # CPU tensor: no fallback
        assert blk.ff.last_router_input is not None
        assert agillm41_b200.install(ref) is cls  # idempotent
    finally:
        agillm41_b200.uninstall(ref)
    assert not getattr(ref.MoEFFN, "_is_b200", False)


def test_install_rebinds_collect_moe_aux(ref):
    """install() rebinds _collect_moe_aux to the fused version (the training
    steps call it through the module global, agillm41.py:1378, 6798); its
    host-side contract is the reference's: stashes are cleared, 0.0 when
    nothing is stashed or both coefficients are <= 0, CPU tensors refused."""
    orig = ref._collect_moe_aux
    agillm41_b200.install(ref)
    try:
        assert ref._collect_moe_aux is not orig and ref._collect_moe_aux._is_b200
        model = torch.nn.ModuleList([ref.MoEFFN(64, experts=4, top_k=1), ref.MoEFFN(64, experts=4, top_k=1)])
        assert ref._collect_moe_aux(model, 0.01, 0.001) == 0.0
        model[0].last_router_input = torch.randn(8, 64)
        assert ref._collect_moe_aux(model, 0.0, 0.0) == 0.0
        assert model[0].last_router_input is None
        model[1].last_router_input = torch.randn(8, 64)
        with pytest.raises(MoEKernelError):
            ref._collect_moe_aux(model, 0.01, 0.0)   # CPU tensor: no fallback
        assert model[1].last_router_input is None
    finally:
        agillm41_b200.uninstall(ref)
    assert ref._collect_moe_aux is orig
    agillm41_b200.install(ref, fuse_aux=False)
    try:
        assert ref._collect_moe_aux is orig
    finally:
        agillm41_b200.uninstall(ref)


def test_fused_residual_block(ref):
    """install(fuse_residual=True) rebinds Block to a subclass whose MoE
    residual add runs in the combine kernel; other FFNs keep the reference's
    own forward (checked numerically here on CPU with a dense FFN)."""
    orig_block = ref.Block
    agillm41_b200.install(ref, fuse_residual=True)
    try:
        assert ref.Block is not orig_block and issubclass(ref.Block, orig_block)
        torch.manual_seed(0)
        dense = ref.Block(64, 4, 16, moe_ffn=False).eval()
        plain = orig_block(64, 4, 16, moe_ffn=False).eval()
        plain.load_state_dict(dense.state_dict())
        x = torch.randn(2, 5, 64)
        with torch.no_grad():
            assert torch.equal(dense(x, None), plain(x, None))
        moe = ref.Block(64, 4, 16, moe_ffn=True, moe_experts=14, moe_top_k=2, moe_mlp_mult=2).eval()
        with torch.no_grad(), pytest.raises(MoEKernelError):
            moe(x, None)                         # CPU tensors: no fallback
    finally:
        agillm41_b200.uninstall(ref)
    assert ref.Block is orig_block and not getattr(ref.MoEFFN, "_is_b200", False)


def test_fused_layernorm_block(ref):
    """install(fuse_layernorm=True) rebinds Block to the fused subclass with
    ln2 on the library's LayerNorm in inference; a dense FFN keeps the
    reference's forward, and a MoE block on CPU still refuses (no CPU path)."""
    orig_block = ref.Block
    agillm41_b200.install(ref, fuse_layernorm=True)
    try:
        assert issubclass(ref.Block, orig_block) and ref.Block._fuse_layernorm
        torch.manual_seed(0)
        dense = ref.Block(64, 4, 16, moe_ffn=False).eval()
        plain = orig_block(64, 4, 16, moe_ffn=False).eval()
        plain.load_state_dict(dense.state_dict())
        x = torch.randn(2, 5, 64)
        with torch.no_grad():
            assert torch.equal(dense(x, None), plain(x, None))
        moe = ref.Block(64, 4, 16, moe_ffn=True, moe_experts=14, moe_top_k=2, moe_mlp_mult=2).eval()
        assert set(moe.state_dict()) == set(orig_block(64, 4, 16, moe_ffn=True, moe_experts=14, moe_top_k=2,
                                                       moe_mlp_mult=2).state_dict())
        with torch.no_grad(), pytest.raises(MoEKernelError):
            moe(x, None)
    finally:
        agillm41_b200.uninstall(ref)
    assert ref.Block is orig_block


def test_cpu_input_raises():
    m = MoEFFN(64, experts=14, top_k=2).eval()
    with torch.no_grad(), pytest.raises(MoEKernelError, match="CUDA"):
        m(torch.randn(1, 4, 64))
