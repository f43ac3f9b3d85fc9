"""The tensor-codec oracle against the reference's golden vectors, and the
host-side checks of the GPU codec path (CPU).

tests/golden/make_golden_codec.py ran the reference's encoder and decoder
(agillm41.py:4858-5102) and its side-update application (6035-6045) and
asserted the restatement bit-identical; these tests re-check the
restatement against the stored vectors.
"""
import pytest
import torch

from agillm41_b200 import MoEKernelError, codec
from golden_io import GoldenCodec, codec_names
from oracle import codec_oracle
from oracle.golden_cases import CODEC_APPLY, codec_state, codec_target


def test_codec_cases_exist():
    assert len(codec_names()) == 5


@pytest.mark.parametrize("name", codec_names())
def test_oracle_decodes_reference_payloads(name):
    g = GoldenCodec(name)
    dec = codec_oracle.decode_tensor_state(g.state)
    for key in g.meta:
        ref = g.decoded(key)
        assert dec[key].dtype == ref.dtype and torch.equal(dec[key], ref), key


@pytest.mark.parametrize("name", codec_names())
def test_oracle_encoder_reproduces_payload_bytes(name):
    g = GoldenCodec(name)
    state = codec_state()
    for key, m in g.meta.items():
        mine = codec_oracle.encode_item(state[key], m["pack_kind"])
        assert torch.equal(mine["data"], g.state["tensors"][key]["data"]), key
        if m["pack_kind"] == "int8_symmetric":
            assert mine["scale"] == m["scale"]


@pytest.mark.parametrize("name", codec_names())
def test_oracle_apply_matches_reference(name):
    g = GoldenCodec(name)
    dec = codec_oracle.decode_tensor_state(g.state)
    for key in g.applied_keys():
        for dt in (torch.float32, torch.bfloat16):
            for app, alpha, delta in CODEC_APPLY:
                t = codec_target(key, dec[key].shape, dt)
                codec_oracle.apply_value(t, dec[key], alpha, delta)
                assert torch.equal(t, g.applied(app, dt, key)), (key, dt, app)


def test_adaptive_mode_covers_every_pack_kind():
    kinds = {m["pack_kind"] for m in GoldenCodec("codec_adaptive_zstd").meta.values()}
    assert kinds == {"int8_symmetric", "int8_rowwise", "fp16"}


def test_host_checks_before_any_device_work():
    g = GoldenCodec("codec_rowq8_zstd")
    assert codec.is_encoded(g.state) and not codec.is_encoded({"a": torch.zeros(1)})
    plain = {"a": torch.zeros(2)}
    assert codec.decode_tensor_state(plain) is plain          # not a codec state: unchanged
    with pytest.raises(MoEKernelError):
        codec.decode_tensor_state(g.state, device="cpu")       # no CPU path
    targets = {k: torch.zeros(tuple(m["shape"])) for k, m in g.meta.items()}
    with pytest.raises(KeyError):
        codec.apply_tensor_state(g.state, {k: v for k, v in targets.items() if k != "router.weight"})
    bad = dict(targets)
    bad["router.weight"] = torch.zeros(3, 3)
    with pytest.raises(ValueError):
        codec.apply_tensor_state(g.state, bad)
    ints = dict(targets)
    ints["router.weight"] = torch.zeros(tuple(g.meta["router.weight"]["shape"]), dtype=torch.int32)
    with pytest.raises(ValueError):
        codec.apply_tensor_state(g.state, ints, delta=True)
    with pytest.raises(MoEKernelError):
        codec.apply_tensor_state(g.state, targets)             # CPU targets


def test_payload_decompression_matches_the_reference_framing():
    raw = bytes(range(256)) * 8
    assert codec._decompress(codec_oracle.compress(raw), "zstd") == raw
    assert codec._decompress(raw, "raw") == raw
    assert codec._decompress(torch.frombuffer(bytearray(codec_oracle.compress(raw)), dtype=torch.uint8),
                             "zstd") == raw
