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


def _f32(v):
    return np.float32(v)


def _butterfly_scalar(lanes):
    v = [_f32(x) for x in lanes]
    for o in (16, 8, 4, 2, 1):
        v = [_f32(v[l] + v[l ^ o]) for l in range(32)]
    assert all(x == v[0] for x in v)  # every lane ends with the same total
    return v[0]


def _fmaf(a, b, c):
    from oracle import _c
    return _c.fmaf(np.array([a], np.float32), np.array([b], np.float32), np.array([c], np.float32))[0]


def test_layernorm_order_matches_lane_loop():
    """The vectorised layernorm statistics equal a literal per-lane loop over the reference's warp layout
    (kernels/int8_gemm.cu:541-570): chunk c*32+l belongs to lane l, ((v0+v1)+v2)+v3 per chunk, xor butterfly."""
    from oracle.producers import layernorm_stats

    g = torch.Generator().manual_seed(11)
    for D in (1152, 200, 2048):
        X = (torch.randn(3, D, generator=g) * 3 + 0.5).to(torch.bfloat16).float().numpy()
        mean, rstd = layernorm_stats(X, 1e-6)
        for r in range(3):
            x = X[r]
            lanes = [_f32(0)] * 32
            for ci in range(D // 4):
                v = x[4 * ci:4 * ci + 4]
                lanes[ci % 32] = _f32(lanes[ci % 32] + _f32(_f32(_f32(v[0] + v[1]) + v[2]) + v[3]))
            m = _f32(_butterfly_scalar(lanes) / _f32(D))
            assert m == mean[r], (D, r)
            lanes = [_f32(0)] * 32
            for ci in range(D // 4):
                for j in range(4):
                    d = _f32(x[4 * ci + j] - m)
                    lanes[ci % 32] = _fmaf(d, d, lanes[ci % 32])
            var = _f32(_butterfly_scalar(lanes) / _f32(D))
            assert _f32(1.0 / np.sqrt(np.float64(_f32(var + _f32(1e-6))))) == rstd[r], (D, r)


def test_rmsnorm_order_matches_thread_loop():
    """The vectorised RMSNorm statistic equals a literal loop over the reference's block layout
    (kernels/int8_gemm.cu:600-614 with block_sum, kernels/lfm2_decode.cu:79-90)."""
    from oracle.producers import rmsnorm_rs

    g = torch.Generator().manual_seed(12)
    for H in (2048, 1024, 320):
        X = (torch.randn(2, H, generator=g) * 2).to(torch.bfloat16).float().numpy()
        rs = rmsnorm_rs(X, 1e-5)
        for r in range(2):
            part = [_f32(0)] * 256
            for i in range(H):
                part[i % 256] = _fmaf(X[r, i], X[r, i], part[i % 256])
            warps = [_butterfly_scalar(part[32 * w:32 * w + 32]) for w in range(8)]
            ss = _butterfly_scalar(warps + [_f32(0)] * 24)
            v = _f32(_f32(ss / _f32(H)) + _f32(1e-5))
            assert _f32(1.0 / np.sqrt(np.float64(v))) == rs[r], (H, r)


def test_quantize_int4_matches_reference():
    d = golden("quantize_int4")
    for i in range(4):
        N, K, group, clip = (int(v) for v in d[f"meta{i}"])
        p, s = oracle.quantize_int4_ref(to_t(d[f"w{i}"], bf16=True), group, bool(clip))
        assert torch.equal(p, to_t(d[f"p{i}"])) and torch.equal(s, to_t(d[f"s{i}"])), i
        assert torch.equal(oracle.dequantize_int4_ref(p, s), to_t(d[f"d{i}"])), i


def test_gemv_w4_matches_reference():
    d = golden("gemv_w4")
    n = len([k for k in d.files if k.startswith("name")])
    assert n >= 2
    for i in range(n):
        y = oracle.gemv_w4_ref(to_t(d[f"p{i}"]), to_t(d[f"s{i}"]), to_t(d[f"x{i}"], bf16=True))
        assert torch.equal(y.view(torch.int16), to_t(d[f"y{i}"])), str(d[f"name{i}"])
