"""The decode-attention oracle on CPU, pinned to the reference's own check expression.

The reference tests its split attention kernel against F.scaled_dot_product_attention over the cache prefix with
grouped-query heads (tests/test_kernels.py:94-115). The fp64 oracle must agree with that expression evaluated in fp32
on the same inputs, and its per-split partials must merge (the reference's combine, kernels/lfm2_decode.cu:389-416)
into the same values."""

import math

import pytest
import torch

from oracle.attention import decode_attention_f64, decode_attention_sdpa, split_partials_f64

BF = torch.bfloat16


def case(B, NKV, max_len, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, 4 * NKV, 64, generator=g).to(BF)
    kc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF)
    vc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF)
    return q, kc, vc


@pytest.mark.parametrize("B,NKV,max_len,pos", [(2, 8, 3072, 2300), (1, 2, 300, 0), (3, 1, 129, 128)])
def test_oracle_matches_sdpa(B, NKV, max_len, pos):
    q, kc, vc = case(B, NKV, max_len, pos + 7)
    scale = 64 ** -0.5
    o = decode_attention_f64(q, kc, vc, pos, scale)
    r = decode_attention_sdpa(q.float(), kc.float(), vc.float(), pos, scale).double()
    assert (o - r).abs().max().item() < 1e-5


@pytest.mark.parametrize("S", [16, 4, 1, 40])
def test_split_partials_merge_to_the_oracle(S):
    B, NKV, max_len, pos = 2, 2, 1000, 700
    q, kc, vc = case(B, NKV, max_len, S)
    scale = 0.125
    ws = split_partials_f64(q, kc, vc, pos, scale, S)
    M = ws[..., 0].max(dim=-1).values
    L = torch.zeros(B, 4 * NKV, dtype=torch.float64)
    o = torch.zeros(B, 4 * NKV, 64, dtype=torch.float64)
    for s in range(S):
        ls = ws[:, :, s, 1]
        if (ls == 0).all():
            assert math.isinf(ws[0, 0, s, 0].item())  # empty split: m = -inf, l = 0
            continue
        c = torch.exp(ws[:, :, s, 0] - M)
        L += ls * c
        o += ws[:, :, s, 2:] * c[..., None]
    assert (o / L[..., None] - decode_attention_f64(q, kc, vc, pos, scale)).abs().max().item() < 1e-12


def test_length_one_is_v0():
    q, kc, vc = case(2, 8, 64, 3)
    o = decode_attention_f64(q, kc, vc, 0, 0.125)
    assert torch.equal(o, vc[:, :, :1].double().repeat_interleave(4, 1).squeeze(2))
