"""The decode-step and attention oracles against golden vectors made by the reference's own test code.

tests/golden/decode_kernels.npz and attention.npz hold the inputs and the reference values that the reference's
tests/test_kernels.py computes (test_add_rmsnorm, test_shortconv, test_qk_rope_kv with transformers'
apply_rotary_pos_emb, test_attention with F.scaled_dot_product_attention), executed on CPU by
tests/golden/make_golden.py. oracle/decode.py restates those expressions, so it must reproduce them bit for bit;
oracle/attention.py computes in fp64 and must meet the reference test's bar against its bf16 SDPA."""

import torch

from conftest import golden, to_t
from oracle.attention import decode_attention_f64
from oracle.decode import add_rmsnorm_ref, qk_norm_rope_kv_ref, rms, shortconv_step_ref

BF = torch.bfloat16
EPS = 1e-5


def bf(d, k):
    return to_t(d[k], bf16=True)


def test_add_rmsnorm_oracle_equals_the_reference_expressions():
    d = golden("decode_kernels")
    h, y, w = bf(d, "norm_h"), bf(d, "norm_y"), bf(d, "norm_w")
    rh, rx = add_rmsnorm_ref(h, y, w, EPS)
    assert torch.equal(rh, bf(d, "norm_ref_h")) and torch.equal(rx, bf(d, "norm_ref_x"))
    assert torch.equal(rms(h, w, EPS), bf(d, "norm_ref_x_noadd"))


def test_shortconv_oracle_equals_the_reference_expressions():
    d = golden("decode_kernels")
    y, st = shortconv_step_ref(bf(d, "conv_bcx"), bf(d, "conv_state"), bf(d, "conv_w"))
    assert torch.equal(st, bf(d, "conv_ref_state"))
    assert torch.equal(y, bf(d, "conv_ref_y"))


def test_qk_norm_rope_oracle_equals_transformers_rope():
    d = golden("decode_kernels")
    B, max_len, pos = (int(v) for v in d["qk_meta"])
    q, k, v = qk_norm_rope_kv_ref(bf(d, "qk_qkv"), bf(d, "qk_qw"), bf(d, "qk_kw"), to_t(d["qk_inv_freq"]), 1.0, pos,
                                  32, 8, EPS)
    assert torch.equal(q, bf(d, "qk_ref_q")) and torch.equal(k, bf(d, "qk_ref_k")) and torch.equal(v, bf(d, "qk_ref_v"))


def test_attention_oracle_meets_the_reference_bar_against_its_sdpa():
    d = golden("attention")
    q, kc, vc = bf(d, "q"), bf(d, "kc"), bf(d, "vc")
    _, _, pos = (int(v) for v in d["meta"])
    scale = float(d["scale"])
    for p, ref in ((pos, bf(d, "ref")), (0, bf(d, "ref_len1"))):
        o = decode_attention_f64(q, kc, vc, p, scale)
        err = (o - ref.double()).abs().max().item()
        assert err <= 2e-2 * max(ref.double().abs().max().item(), 1.0)
        assert err <= 2 ** -7 * max(ref.double().abs().max().item(), 1.0)  # bf16 rounding of either side
