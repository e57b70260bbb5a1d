"""The oracle against the golden vectors made by the reference's own code (tests/golden/make_golden.py)."""

import numpy as np
import torch

import oracle
from oracle.gemm import gemm_i8_grouped_ref
from conftest import golden, to_t


def test_quantize_int8_matches_reference():
    d = golden("quantize_int8")
    for i in range(4):
        q, s = oracle.quantize_int8_ref(to_t(d[f"w{i}"], bf16=True))
        assert torch.equal(q, to_t(d[f"q{i}"])), i
        assert torch.equal(s, to_t(d[f"s{i}"])), i


def test_quant_rows_matches_reference():
    d = golden("quant_rows")
    for i in range(3):
        q, s = oracle.quant_rows_ref(to_t(d[f"x{i}"], bf16=True))
        assert torch.equal(q, to_t(d[f"q{i}"])) and torch.equal(s, to_t(d[f"s{i}"])), i
        q, s = oracle.quant_groups_ref(to_t(d[f"gx{i}"], bf16=True))
        assert torch.equal(q, to_t(d[f"gq{i}"])) and torch.equal(s, to_t(d[f"gs{i}"])), i


def _gemm_case(d, i):
    M, K, N, bias, gelu = (int(v) for v in d[f"meta{i}"])
    b = to_t(d[f"b{i}"], bf16=True) if bias else None
    return (to_t(d[f"xq{i}"]), to_t(d[f"sx{i}"]), to_t(d[f"wq{i}"]), to_t(d[f"sw{i}"]), b, bool(gelu))


def test_gemm_i8_matches_reference():
    d = golden("gemm_i8")
    for i in range(4):
        xq, sx, wq, sw, b, gelu = _gemm_case(d, i)
        y = oracle.gemm_i8_ref(xq, sx, wq, sw, b, gelu)
        assert torch.equal(y.view(torch.int16), to_t(d[f"y{i}"])), i


def test_gemm_i8_grouped_matches_reference():
    d = golden("gemm_i8_grouped")
    for i in range(3):
        xq, sxT, wq, sw, b, gelu = _gemm_case(d, i)
        r = to_t(d[f"r{i}"])
        assert torch.equal(oracle.gemm_i8_grouped_f64(xq, sxT, wq, sw, b, gelu), r), i
        # the fp32-fold oracle meets the reference's own acceptance bound (tests/test_int8_gemm.py:101-103)
        y = gemm_i8_grouped_ref(xq, sxT, wq, sw, b, gelu).double()
        e_ours = ((y - r).norm() / r.norm()).item()
        e_round = ((r.to(torch.bfloat16).double() - r).norm() / r.norm()).item()
        assert e_ours <= 1.05 * e_round + 1e-6, (i, e_ours, e_round)


def test_gemv_matches_reference():
    d = golden("gemv")
    n = len([k for k in d.files if k.startswith("name")])
    assert n >= 20
    for i in range(n):
        W = to_t(d[f"W{i}"], bf16="bf16" in str(d[f"name{i}"]))
        s = to_t(d[f"s{i}"]) if d[f"s{i}"].size else None
        x = to_t(d[f"x{i}"], bf16=True)
        y = oracle.gemv_ref(W, s, x)
        assert torch.equal(y.view(torch.int16), to_t(d[f"y{i}"])), str(d[f"name{i}"])


def test_int_mm_exact_against_fp64():
    g = torch.Generator().manual_seed(5)
    xq = torch.randint(-127, 128, (33, 8192), generator=g, dtype=torch.int8)
    wq = torch.randint(-127, 128, (40, 8192), generator=g, dtype=torch.int8)
    e = (xq.double() @ wq.double().t())
    assert torch.equal(oracle.int_mm_exact(xq, wq).double(), e)


def test_quant_edge_cases():
    # all-zero rows take the 1e-8 floor; ties round half to even; codes saturate at +-127
    x = torch.zeros(3, 64, dtype=torch.bfloat16)
    x[1, 0] = 127.0
    x[1, 1] = 0.5
    x[1, 2] = 1.5
    x[2, :] = -3.0
    q, s = oracle.quant_rows_ref(x)
    assert s[0].item() == np.float32(1e-8) / np.float32(127)
    assert q[0].abs().max().item() == 0
    assert q[1, :3].tolist() == [127, 0, 2]
    assert (q[2] == -127).all()
