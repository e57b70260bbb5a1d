"""quant_rows / quant_groups on the B200 against the oracle: bit-exact codes and scales."""

import pytest
import torch

import oracle
from conftest import golden, to_t
from lfm2opt.int8 import quantize_rows

pytestmark = pytest.mark.gpu


def _x(M, K, seed, outlier=True):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=g) * torch.rand(M, 1, generator=g) * 4).to(torch.bfloat16)
    if outlier:
        x[0, min(3, K - 1)] = 37.0
    return x


@pytest.mark.parametrize("M,K", [(1, 2048), (37, 1152), (2327, 2048), (9216, 1152), (5, 4304), (64, 8192),
                                 (3, 16384), (300, 8), (17, 136), (1000, 2048), (5001, 1280), (4097, 1296),
                                 (65536, 1152), (700, 8)])
def test_quant_rows(cuda_dev, M, K):
    x = _x(M, K, M * 7 + K)
    q, s = quantize_rows(x.to(cuda_dev))
    rq, rs = oracle.quant_rows_ref(x)
    assert torch.equal(q.cpu(), rq), (q.cpu() != rq).sum().item()
    assert torch.equal(s.cpu(), rs)


@pytest.mark.parametrize("M,K", [(1, 2048), (37, 1152), (2327, 8192), (9216, 4352), (5, 64), (33, 16384),
                                 (7, 192)])
def test_quant_groups(cuda_dev, M, K):
    x = _x(M, K, M * 11 + K)
    q, s = quantize_rows(x.to(cuda_dev), 64)
    rq, rs = oracle.quant_groups_ref(x)
    assert torch.equal(q.cpu(), rq), (q.cpu() != rq).sum().item()
    assert torch.equal(s.cpu(), rs)


def test_quant_edge_values(cuda_dev):
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    x[1, 0], x[1, 1], x[1, 2] = 127.0, 0.5, 1.5  # ties to even at scale 1
    x[2, :] = -3.0
    x[3, ::2] = 1e-30  # subnormal-scale values: the 1e-8 floor applies
    for grouped in (0, 64):
        q, s = quantize_rows(x.to(cuda_dev), grouped)
        rq, rs = oracle.quant_groups_ref(x) if grouped else oracle.quant_rows_ref(x)
        assert torch.equal(q.cpu(), rq) and torch.equal(s.cpu(), rs)


def test_quant_golden(cuda_dev):
    d = golden("quant_rows")
    for i in range(3):
        x = to_t(d[f"x{i}"], bf16=True)
        q, s = quantize_rows(x.to(cuda_dev))
        assert torch.equal(q.cpu(), to_t(d[f"q{i}"])) and torch.equal(s.cpu(), to_t(d[f"s{i}"]))
        x = to_t(d[f"gx{i}"], bf16=True)
        q, s = quantize_rows(x.to(cuda_dev), 64)
        assert torch.equal(q.cpu(), to_t(d[f"gq{i}"])) and torch.equal(s.cpu(), to_t(d[f"gs{i}"]))
