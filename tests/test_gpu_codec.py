"""Tensor-codec decode on the GPU (agm_codec_decode through
agillm41_b200.codec) against the reference's golden vectors and against the
oracle's restatement (oracle/codec_oracle.py) run with the same torch calls
on the same GPU.

Decoding is one fp32 multiply per element (or none) and one rounding to the
target's dtype, so every comparison of decoded values and of copied targets
is bit-exact. The lerp and add applications are compared bit-exactly with
torch's own CUDA lerp_/add_ on the same GPU (the reference applies updates to
device parameters); against the CPU golden vectors (torch's CPU kernels may
round the multiply-add differently) they are held to one unit in the last
place of the target dtype.
"""
import pytest
import torch

import agillm41_b200
from agillm41_b200 import codec
from golden_io import GoldenCodec, codec_names
from oracle import codec_oracle
from oracle.golden_cases import CODEC_APPLY, codec_target

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def within_one_ulp(a, b):
    a, b = a.cpu(), b.cpu()
    if a.dtype == torch.bfloat16:
        ia, ib = a.view(torch.int16).int(), b.view(torch.int16).int()
    else:
        ia, ib = a.view(torch.int32).long(), b.view(torch.int32).long()
    return bool(((ia - ib).abs() <= 1).all())


@pytest.mark.parametrize("name", codec_names())
def test_decode_matches_reference(name):
    g = GoldenCodec(name)
    dec = codec.decode_tensor_state(g.state, DEV)
    for key in g.meta:
        ref = g.decoded(key)
        assert dec[key].is_cuda and dec[key].dtype == ref.dtype, key
        assert torch.equal(dec[key].cpu(), ref), key


@pytest.mark.parametrize("name", codec_names())
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_apply_matches_reference(name, dtype):
    g = GoldenCodec(name)
    keys = g.applied_keys()
    dec_cpu = codec_oracle.decode_tensor_state(g.state)
    for app, alpha, delta in CODEC_APPLY:
        state = dict(g.state)
        state["tensors"] = {k: g.state["tensors"][k] for k in keys}
        targets = {k: codec_target(k, g.meta[k]["shape"], dtype).to(DEV) for k in keys}
        assert codec.apply_tensor_state(state, targets, alpha=alpha, delta=delta) == len(keys)
        for k in keys:
            ref_gpu = codec_target(k, g.meta[k]["shape"], dtype).to(DEV)
            codec_oracle.apply_value(ref_gpu, dec_cpu[k].to(DEV), alpha, delta)
            assert torch.equal(targets[k], ref_gpu), (k, app)
            golden = g.applied(app, dtype, k)
            if app == "copy":
                assert torch.equal(targets[k].cpu(), golden), (k, app)
            else:
                assert within_one_ulp(targets[k], golden), (k, app)


@pytest.mark.parametrize("kind", ["int8_rowwise", "int8_symmetric", "fp16", "lossless"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_production_expert_shapes(kind, dtype):
    """The production MoE's expert tensors (d = 1280, H = 4d, 2 experts)
    decoded into dtype targets, against the oracle's CPU decode."""
    g = torch.Generator().manual_seed(93)
    d, H = 1280, 5120
    state = {"experts.0.0.weight": torch.randn(H, d, generator=g) * 0.02,
             "experts.0.0.bias": torch.randn(H, generator=g) * 0.01,
             "experts.1.2.weight": torch.randn(d, H, generator=g) * 0.02,
             "experts.1.2.bias": torch.randn(d, generator=g) * 0.01}
    kinds = {k: (kind if (kind != "int8_rowwise" or v.ndim == 2) else "int8_symmetric") for k, v in state.items()}
    enc = codec_oracle.encode_state(state, kinds)
    ref = codec_oracle.decode_tensor_state(enc)
    targets = {k: torch.empty(v.shape, dtype=dtype, device=DEV) for k, v in state.items()}
    codec.apply_tensor_state(enc, targets)
    for k in state:
        assert torch.equal(targets[k].cpu(), ref[k].to(dtype)), k


@pytest.mark.parametrize("shape", [(37, 8), (3, 1000), (1001,), (5, 33)])
@pytest.mark.parametrize("mode", ["copy", "lerp", "add"])
def test_ragged_shapes_and_rows(shape, mode):
    """Element counts off the 16-element vector (tail path), rows shorter
    than a vector (several row scales in one vector), a target that is not
    16-byte aligned (scalar path)."""
    g = torch.Generator().manual_seed(94)
    src = torch.randn(shape, generator=g)
    kind = "int8_rowwise" if len(shape) == 2 else "int8_symmetric"
    enc = codec_oracle.encode_state({"w": src}, {"w": kind})
    dec = codec_oracle.decode_tensor_state(enc)["w"]
    alpha, delta = {"copy": (1.0, False), "lerp": (0.4, False), "add": (0.5, True)}[mode]
    for offset in (0, 1):
        base = torch.randn(src.numel() + 1, generator=g).to(DEV, torch.bfloat16)
        target = base[offset:offset + src.numel()].view(shape)
        ref = target.clone()
        codec_oracle.apply_value(ref, dec.to(DEV), alpha, delta)
        codec.apply_tensor_state(enc, {"w": target}, alpha=alpha, delta=delta)
        assert torch.equal(target, ref), offset


def test_update_reaches_the_moe_forward():
    """Applying a codec state to a B200 MoEFFN's parameters (as the side-update
    consumer does to the core's parameters) changes its forward exactly as
    loading the oracle-decoded values would."""
    torch.manual_seed(95)
    m = agillm41_b200.MoEFFN(256, mlp_mult=2, experts=4, top_k=2).to(DEV, torch.bfloat16).eval()
    x = torch.randn(3, 40, 256, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        y0 = m(x)
    new = {k: (v.float().cpu() + 0.01 * torch.randn(v.shape)) for k, v in m.state_dict().items()}
    kinds = {k: ("int8_rowwise" if v.ndim == 2 else "fp16") for k, v in new.items()}
    enc = codec_oracle.encode_state(new, kinds)
    params = dict(m.named_parameters())
    assert codec.apply_tensor_state(enc, params) == len(new)
    fresh = agillm41_b200.MoEFFN(256, mlp_mult=2, experts=4, top_k=2).to(DEV, torch.bfloat16).eval()
    fresh.load_state_dict({k: v.to(torch.bfloat16) for k, v in codec_oracle.decode_tensor_state(enc).items()})
    with torch.no_grad():
        y1, y2 = m(x), fresh(x)
    assert not torch.equal(y0, y1)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("mode", ["lerp", "copy"])
def test_batch_matches_single_tensor_calls(mode):
    """agm_codec_decode_batch (the path of decode/apply_tensor_state) against
    one agm_codec_decode call per tensor: 23 tensors of mixed pack kinds and
    target dtypes, 18 of one kind (two launches), rows of 8 elements (not
    batchable), an unaligned target view (t5); bit for bit, in lerp and copy
    mode. In copy mode a warp whose 32 groups lie in one tensor stores through
    shared memory and a warp that straddles two tensors stores directly; the
    1000 + i element tensors give both kinds of warp."""
    import ctypes

    from agillm41_b200 import _lib

    apply_mode, alpha = {"lerp": (_lib.AGM_APPLY_LERP, 0.4), "copy": (_lib.AGM_APPLY_COPY, 1.0)}[mode]

    g = torch.Generator().manual_seed(96)
    specs = [(f"t{i}", "int8_symmetric", (1000 + i,), torch.float32) for i in range(18)]  # two launches of a kind
    specs += [("t18", "int8_rowwise", (64, 64), torch.bfloat16), ("t19", "int8_rowwise", (37, 8), torch.float32),
              ("t20", "fp16", (333,), torch.bfloat16), ("t21", "lossless", (515,), torch.float32),
              ("t22", "int8_rowwise", (12, 8), torch.bfloat16)]
    state = {k: torch.randn(shape, generator=g) for k, _, shape, _ in specs}
    enc = codec_oracle.encode_state(state, {k: kind for k, kind, _, _ in specs})
    staged = [codec._Payload(k, enc["tensors"][k]) for k, _, _, _ in specs]
    base = {k: torch.randn(int(torch.tensor(shape).prod()) + 1, generator=g).to(DEV, dt) for k, _, shape, dt in specs}
    view = {k: (base[k][1:] if k == "t5" else base[k][:-1]).view(shape) for k, _, shape, dt in specs}
    single = {k: v.clone() for k, v in view.items()}
    lib = _lib.load()
    stream = _lib.stream_handle(DEV)
    keep = []
    rows = []
    for p in staged:
        q, s = p.upload(DEV)
        keep += [q, s]
        e = p.entry(q, s, single[p.key])
        rc = lib.agm_codec_decode(e.payload, e.kind, e.packed_dtype, e.n, e.cols, e.scale, e.row_scales,
                                  e.scales_dtype, e.target, e.target_dtype, apply_mode, alpha, stream)
        _lib.check(rc, "agm_codec_decode")
        rows.append(p.entry(q, s, view[p.key]))
    table = (_lib.AgmCodecTensor * len(rows))(*rows)
    _lib.check(lib.agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), len(rows), apply_mode, alpha,
                                          stream), "agm_codec_decode_batch")
    torch.cuda.synchronize()
    for k in view:
        assert torch.equal(view[k], single[k]), k


def test_batch_overlapping_targets_apply_in_order():
    """Entries whose targets overlap (the same tensor three times, and a view
    overlapping half of it) are applied one after another in table order, as
    the reference's loop over keys does: in ADD mode each update must see the
    previous one. Compared bit for bit with one agm_codec_decode call per
    entry, in order."""
    import ctypes

    from agillm41_b200 import _lib

    g = torch.Generator().manual_seed(97)
    specs = [(f"u{i}", "int8_symmetric", (2048,)) for i in range(4)]
    state = {k: torch.randn(shape, generator=g) for k, _, shape in specs}
    enc = codec_oracle.encode_state(state, {k: kind for k, kind, _ in specs})
    staged = [codec._Payload(k, enc["tensors"][k]) for k, _, _ in specs]
    base = torch.randn(4096, generator=g).to(DEV)
    # u0, u1, u2 -> base[0:2048]; u3 -> base[1024:3072] (overlaps the upper half)
    tgt = {"u0": (0, 2048), "u1": (0, 2048), "u2": (0, 2048), "u3": (1024, 3072)}
    lib = _lib.load()
    stream = _lib.stream_handle(DEV)
    single, batched = base.clone(), base.clone()
    keep, rows = [], []
    for p in staged:
        q, s = p.upload(DEV)
        keep += [q, s]
        lo, hi = tgt[p.key]
        e = p.entry(q, s, single[lo:hi])
        _lib.check(lib.agm_codec_decode(e.payload, e.kind, e.packed_dtype, e.n, e.cols, e.scale, e.row_scales,
                                        e.scales_dtype, e.target, e.target_dtype, _lib.AGM_APPLY_ADD, 0.5, stream),
                   "agm_codec_decode")
        rows.append(p.entry(q, s, batched[lo:hi]))
    table = (_lib.AgmCodecTensor * len(rows))(*rows)
    _lib.check(lib.agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), len(rows), _lib.AGM_APPLY_ADD, 0.5,
                                          stream), "agm_codec_decode_batch")
    torch.cuda.synchronize()
    assert torch.equal(batched, single)
    assert not torch.equal(batched, base)
