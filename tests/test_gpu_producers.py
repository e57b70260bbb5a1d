"""Fused producers on the B200 against the CPU oracle, which restates the reference's reductions
(kernels/int8_gemm.cu:529-682; oracle/producers.py).

The residual update h += y is bit-exact. The normalisation statistic goes through rsqrtf on the GPU (the reference's
intrinsic), whose result is within 2 fp32 ulps of the correctly rounded 1/sqrt (CUDA's documented bound); the oracle's
is correctly rounded. So every row must equal, code for code and scale for scale, the oracle's row computed with one
of the five fp32 values within 2 ulps of the correctly rounded statistic: an exact check per row, which fails on any
difference in summation order or rounding point. The bit-for-bit pin against the reference's own kernels on the same
GPU is in tests/test_gpu_reference_kernels.py.

silu_mul_q has no reduction; its only inexact step is __expf (the reference's intrinsic) against the CPU's exp, so
against this oracle an int8 code may differ by one on rare elements (the bit-exact check is again the reference's
kernel, and the reference's unfused silu_mul followed by this oracle's quantizer)."""

import pytest
import torch

from oracle import producers as P
from lfm2opt.int8 import qbuf
from lfm2opt.kernels import int8_ext

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def rows_match_some_shift(q, s, grouped, ref_fn):
    """Every row of (q, s) equals the oracle's row for one rstd shift k in [-2, 2] fp32 ulps."""
    q, s = q.cpu(), s.cpu()
    rows = q.shape[0]
    matched = torch.zeros(rows, dtype=torch.bool)
    used = {}
    for k in (0, -1, 1, -2, 2):
        rq, rs = ref_fn(k)
        eq = (q == rq).all(dim=1) & ((s == rs).all(dim=0) if grouped else (s == rs))
        used[k] = int((eq & ~matched).sum())
        matched |= eq
        if matched.all():
            break
    bad = (~matched).nonzero().flatten().tolist()
    assert not bad, f"rows {bad[:8]} match no rstd within 2 ulps (rows matched per shift: {used})"
    return used


LN_CASES = [(300, 1152), (257, 2048), (1, 1152), (37, 768), (9, 200), (5, 16384)]


@pytest.mark.parametrize("grouped", [0, 64])
@pytest.mark.parametrize("with_y", [True, False])
@pytest.mark.parametrize("rows,D", LN_CASES)
def test_add_layernorm_q(cuda_dev, grouped, with_y, rows, D):
    if grouped and D % 64:
        pytest.skip("grouped scales need D % 64 == 0")
    g = torch.Generator().manual_seed(1 + grouped + D)
    h0 = (torch.randn(rows, D, generator=g) + 0.3).to(BF)
    y = torch.randn(rows, D, generator=g).to(BF) if with_y else None
    w = (torch.rand(D, generator=g) + 0.5).to(BF)
    b = torch.randn(D, generator=g).to(BF)
    h = h0.clone().to(cuda_dev)
    q, s = qbuf(rows, D, grouped, cuda_dev)
    int8_ext().add_layernorm_q(h, None if y is None else y.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev), q, s, 1e-6)
    rh, _, _ = P.add_layernorm_q_ref(h0, y, w, b, 1e-6, grouped)
    assert torch.equal(h.cpu(), rh)
    rows_match_some_shift(q, s, grouped, lambda k: P.add_layernorm_q_ref(h0, y, w, b, 1e-6, grouped, k)[1:])


RMS_CASES = [(257, 2048), (1, 2048), (64, 1024), (3, 8192), (17, 320)]


@pytest.mark.parametrize("grouped", [0, 64])
@pytest.mark.parametrize("with_y", [True, False])
@pytest.mark.parametrize("rows,H", RMS_CASES)
def test_add_rmsnorm_q(cuda_dev, grouped, with_y, rows, H):
    g = torch.Generator().manual_seed(2 + grouped + H)
    h0 = torch.randn(rows, H, generator=g).to(BF)
    y = torch.randn(rows, H, generator=g).to(BF) if with_y else None
    w = (torch.rand(H, generator=g) + 0.5).to(BF)
    h = h0.clone().to(cuda_dev)
    q, s = qbuf(rows, H, grouped, cuda_dev)
    int8_ext().add_rmsnorm_q(h, None if y is None else y.to(cuda_dev), w.to(cuda_dev), q, s, 1e-5)
    rh, _, _ = P.add_rmsnorm_q_ref(h0, y, w, 1e-5, grouped)
    assert torch.equal(h.cpu(), rh)
    rows_match_some_shift(q, s, grouped, lambda k: P.add_rmsnorm_q_ref(h0, y, w, 1e-5, grouped, k)[1:])


@pytest.mark.parametrize("grouped", [0, 64])
def test_silu_mul_q(cuda_dev, grouped):
    g = torch.Generator().manual_seed(3 + grouped)
    rows, I = 257, 8192
    gg = (torch.randn(rows, 2 * I, generator=g) * 2).to(BF)
    q, s = qbuf(rows, I, grouped, cuda_dev)
    int8_ext().silu_mul_q(gg.to(cuda_dev), q, s)
    rq, rs = P.silu_mul_q_ref(gg, grouped)
    dq = (q.cpu().int() - rq.int()).abs()
    assert dq.max().item() <= 1
    assert (dq > 0).float().mean().item() < 2e-3
    assert ((s.cpu() - rs).abs() <= rs.abs() * 2 ** -7).all()
