"""Fused producers on the B200 against the oracle: the residual update h += y is bit-exact; the quantized outputs
match except where rsqrtf / __expf (GPU intrinsics) and the CPU's 1/sqrt / exp round a bf16 value differently
(<= 1 int8 code on a tiny fraction of elements; scales within one part in 2^7)."""

import pytest
import torch

from oracle import producers as P
from lfm2opt.int8 import qbuf
from lfm2opt.kernels import int8_ext

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def close_q(q, s, rq, rs):
    dq = (q.int() - rq.int()).abs()
    assert dq.max().item() <= 1
    assert (dq > 0).float().mean().item() < 2e-3
    assert ((s - rs).abs() <= rs.abs() * 2 ** -7).all()


@pytest.mark.parametrize("grouped", [0, 64])
@pytest.mark.parametrize("with_y", [True, False])
def test_add_layernorm_q(cuda_dev, grouped, with_y):
    g = torch.Generator().manual_seed(1 + grouped)
    rows, D = 300, 1152
    h0 = torch.randn(rows, D, generator=g).to(BF)
    y = torch.randn(rows, D, generator=g).to(BF) if with_y else None
    w = (torch.rand(D, generator=g) + 0.5).to(BF)
    b = torch.randn(D, generator=g).to(BF)
    h = h0.clone().to(cuda_dev)
    q, s = qbuf(rows, D, grouped, cuda_dev)
    int8_ext().add_layernorm_q(h, None if y is None else y.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev), q, s, 1e-6)
    rh, rq, rs = P.add_layernorm_q_ref(h0, y, w, b, 1e-6, grouped)
    assert torch.equal(h.cpu(), rh)
    close_q(q.cpu(), s.cpu(), rq, rs)


@pytest.mark.parametrize("grouped", [0, 64])
@pytest.mark.parametrize("with_y", [True, False])
def test_add_rmsnorm_q(cuda_dev, grouped, with_y):
    g = torch.Generator().manual_seed(2 + grouped)
    rows, H = 257, 2048
    h0 = torch.randn(rows, H, generator=g).to(BF)
    y = torch.randn(rows, H, generator=g).to(BF) if with_y else None
    w = (torch.rand(H, generator=g) + 0.5).to(BF)
    h = h0.clone().to(cuda_dev)
    q, s = qbuf(rows, H, grouped, cuda_dev)
    int8_ext().add_rmsnorm_q(h, None if y is None else y.to(cuda_dev), w.to(cuda_dev), q, s, 1e-5)
    rh, rq, rs = P.add_rmsnorm_q_ref(h0, y, w, 1e-5, grouped)
    assert torch.equal(h.cpu(), rh)
    close_q(q.cpu(), s.cpu(), rq, rs)


@pytest.mark.parametrize("grouped", [0, 64])
def test_silu_mul_q(cuda_dev, grouped):
    g = torch.Generator().manual_seed(3 + grouped)
    rows, I = 257, 8192
    gg = (torch.randn(rows, 2 * I, generator=g) * 2).to(BF)
    q, s = qbuf(rows, I, grouped, cuda_dev)
    int8_ext().silu_mul_q(gg.to(cuda_dev), q, s)
    rq, rs = P.silu_mul_q_ref(gg, grouped)
    close_q(q.cpu(), s.cpu(), rq, rs)
