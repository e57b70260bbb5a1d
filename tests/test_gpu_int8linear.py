"""The reference-facing API (lfm2opt.int8.Int8Linear) end to end on the B200 against the oracle pipeline."""

import pytest
import torch

import oracle
from lfm2opt.int8 import Int8Linear, quantize_rows

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.mark.parametrize("group", [0, 64])
@pytest.mark.parametrize("gelu", [False, True])
def test_int8linear_a8(cuda_dev, group, gelu):
    g = torch.Generator().manual_seed(group + gelu)
    w = (torch.randn(4304, 1152, generator=g) * 0.02).to(BF)
    b = (torch.randn(4304, generator=g) * 0.02).to(BF)
    x = torch.randn(2, 300, 1152, generator=g).to(BF)
    lin = Int8Linear(w.to(cuda_dev), b.to(cuda_dev), group=group)
    y = lin(x.to(cuda_dev), gelu=gelu)
    assert y.shape == (2, 300, 4304)
    x2 = x.reshape(-1, 1152)
    if group:
        xq, sx = oracle.quant_groups_ref(x2)
        r = oracle.gemm_i8_grouped_ref(xq, sx, lin.q.cpu(), lin.s.cpu(), b, gelu)
    else:
        xq, sx = oracle.quant_rows_ref(x2)
        r = oracle.gemm_i8_ref(xq, sx, lin.q.cpu(), lin.s.cpu(), b, gelu)
    from test_gpu_gemm import assert_close_bf16
    assert_close_bf16(y.reshape(-1, 4304).cpu(), r, gelu)


def test_int8linear_quant_out_chain(cuda_dev):
    """vision MLP: fc1 (GELU) writes fc2's int8 input inside its epilogue; fc2 consumes the tuple."""
    g = torch.Generator().manual_seed(7)
    w1 = (torch.randn(4304, 1152, generator=g) * 0.02).to(BF)
    b1 = (torch.randn(4304, generator=g) * 0.02).to(BF)
    w2 = (torch.randn(1152, 4304, generator=g) * 0.02).to(BF)
    x = torch.randn(1024, 1152, generator=g).to(BF)
    fc1 = Int8Linear(w1.to(cuda_dev), b1.to(cuda_dev), pad_n=48, kind="fc1", group=64)
    fc2 = Int8Linear(w2.to(cuda_dev), None, pad_k=48, kind="fc2", group=64)
    hq = fc1(x.to(cuda_dev), gelu=True, quant_out=True)
    assert hq[0].shape == (1024, 4352) and hq[1].shape == (68, 1024)
    y = fc2(hq)
    assert y.shape == (1024, 1152)
    # oracle chain from the same int8 hand-off
    r = oracle.gemm_i8_grouped_ref(hq[0].cpu(), hq[1].cpu(), fc2.q.cpu(), fc2.s.cpu())
    assert oracle.bf16_ulps(y.cpu(), r) == 0
    xq, sx = quantize_rows(x.to(cuda_dev), 64)
    oq, os_ = oracle.gemm_i8_q_ref(xq.cpu(), sx.cpu(), fc1.q.cpu(), fc1.s.cpu(), fc1.bias.cpu(), True)
    assert (hq[0].cpu().int() - oq.int()).abs().max().item() <= 1


def test_int8linear_silu_gate(cuda_dev):
    g = torch.Generator().manual_seed(8)
    w13 = (torch.randn(2 * 8192, 2048, generator=g) * 0.02).to(BF)
    x = torch.randn(512, 2048, generator=g).to(BF)
    lin = Int8Linear(w13.to(cuda_dev), None, group=0, kind="w13")
    y = lin(x.to(cuda_dev), silu_gate=True)
    assert y.shape == (512, 8192)
    xq, sx = oracle.quant_rows_ref(x)
    r = oracle.gemm_i8_silu_ref(xq, sx, lin.q.cpu(), lin.s.cpu())
    ok, detail = oracle.silu_chain_close(y.cpu(), r)
    assert ok, detail
