"""Host-side logic of the lfm2opt mirror that needs no GPU: env-driven granularity, buffers, weight quantizer."""

import pytest
import torch

from lfm2opt import int8 as L
from lfm2opt.quant import quantize_int8
import oracle
from conftest import golden, to_t


def test_quantize_int8_is_the_reference_expression():
    d = golden("quantize_int8")
    for i in range(4):
        q, s = quantize_int8(to_t(d[f"w{i}"], bf16=True))
        assert torch.equal(q, to_t(d[f"q{i}"])) and torch.equal(s, to_t(d[f"s{i}"]))


def test_act_group_env(monkeypatch):
    monkeypatch.delenv("LFM2_INT8_GROUP", raising=False)
    monkeypatch.delenv("LFM2_INT8_GROUP_KINDS", raising=False)
    assert L.act_group("qkv", 1152) == 64  # reference default: grouped
    monkeypatch.setenv("LFM2_INT8_GROUP", "0")
    assert L.act_group("qkv", 1152) == 0
    assert L.act_group("w2", 8192) == 64  # wide inputs stay grouped, as in the reference
    monkeypatch.setenv("LFM2_INT8_GROUP", "64")
    monkeypatch.setenv("LFM2_INT8_GROUP_KINDS", "fc2,w2")
    assert L.act_group("fc2", 1152) == 64 and L.act_group("qkv", 1152) == 0
    monkeypatch.setenv("LFM2_INT8_GROUP", "32")
    with pytest.raises(ValueError):
        L.act_group("qkv", 1152)


def test_a16_kinds(monkeypatch):
    monkeypatch.setenv("LFM2_INT8_A16", "fc2,w2")
    assert L.a16_kinds() == {"fc2", "w2"}
    monkeypatch.delenv("LFM2_INT8_A16")
    assert L.a16_kinds() == set()


def test_qbuf_shapes():
    q, s = L.qbuf(10, 256, 64, "cpu")
    assert q.shape == (10, 256) and q.dtype == torch.int8 and s.shape == (4, 10)
    q, s = L.qbuf(10, 256, 0, "cpu")
    assert s.shape == (10,)


def test_int8linear_pads_and_quantizes_on_cpu_without_kernels():
    w = torch.randn(4304, 64, dtype=torch.bfloat16)
    b = torch.randn(4304, dtype=torch.bfloat16)
    lin = L.Int8Linear(w, b, pad_n=48, kind="fc1")
    assert lin.N == 4352 and lin.K == 64 and lin.bias.shape == (4352,)
    q, s = oracle.quantize_int8_ref(torch.nn.functional.pad(w, (0, 0, 0, 48)))
    assert torch.equal(lin.q, q) and torch.equal(lin.s, s)
    assert lin.bias[4304:].abs().sum().item() == 0
    lin0 = L.Int8Linear(w, None, group=0)
    assert lin0.group == 0
    with pytest.raises(ValueError):
        L.Int8Linear(w, None, group=32)


def test_quantize_int4_matches_reference_golden():
    """lfm2opt.quant.quantize_int4 / dequantize_int4 (load-time torch ops) give the reference's bytes and scales."""
    from lfm2opt.quant import dequantize_int4, quantize_int4
    d = golden("quantize_int4")
    for i in range(4):
        N, K, group, clip = (int(v) for v in d[f"meta{i}"])
        p, s = quantize_int4(to_t(d[f"w{i}"], bf16=True), group, clip_search=bool(clip))
        assert torch.equal(p, to_t(d[f"p{i}"])) and torch.equal(s, to_t(d[f"s{i}"])), i
        assert torch.equal(dequantize_int4(p, s), to_t(d[f"d{i}"])), i
