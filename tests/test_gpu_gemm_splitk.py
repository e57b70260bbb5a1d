"""Split-K W8A8 GEMM for few rows (decode batches) on the B200.

A cluster of S CTAs computes one 128 x 128 output tile, each over 1/S of K; the exact int32 partial tiles are summed
in distributed shared memory and the per-token epilogue runs on the sum. Integer sums are exact in any order, so the
output must equal the one-CTA tile's bit for bit, and the oracle's (0 ulp without GELU).
"""

import pytest
import torch

import oracle
from lfm2opt import _capi
from lfm2opt.int8 import quantize_rows
from lfm2opt.kernels import int8_ext
from lfm2opt.quant import quantize_int8
from test_gpu_gemm import assert_close_bf16

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def run(xq, sx, wq, sw, b, gelu, tile):
    _capi.lib().lfm2q_set_gemm_tile(tile)
    try:
        y = torch.full((xq.shape[0], wq.shape[0]), float("nan"), device=xq.device, dtype=BF)
        int8_ext().gemm_i8(xq, sx, wq, sw, b, y, gelu)
        torch.cuda.synchronize()
    finally:
        _capi.lib().lfm2q_set_gemm_tile(0)
    return y


def operands(M, K, N, bias, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(BF)
    x[:, 3] *= 25
    wq, sw = quantize_int8((torch.randn(N, K, generator=g) * 0.02).to(BF))
    b = torch.randn(N, generator=g).to(BF).to(dev) if bias else None
    xq, sx = quantize_rows(x.to(dev), 0)
    return xq, sx, wq.to(dev), sw.to(dev), b


CASES = [(17, 2048, 8192), (33, 2048, 2048), (64, 2048, 8192), (64, 8192, 2048), (100, 2048, 6144), (128, 8192, 2048),
         (128, 2048, 16384), (200, 2048, 2048), (256, 4096, 3072), (1, 2048, 2048), (48, 1040, 1000), (96, 1152, 4352),
         (65, 8192, 264)]


@pytest.mark.parametrize("M,K,N", CASES)
@pytest.mark.parametrize("bias,gelu", [(False, False), (True, True)])
def test_splitk_equals_one_cta_tile(cuda_dev, M, K, N, bias, gelu):
    xq, sx, wq, sw, b = operands(M, K, N, bias, M * 7 + K + N, cuda_dev)
    ys = run(xq, sx, wq, sw, b, gelu, 1)
    yt = run(xq, sx, wq, sw, b, gelu, 128)
    assert torch.equal(ys, yt), (M, K, N)
    if M * N * K <= 2**31:
        r = oracle.gemm_i8_ref(xq.cpu(), sx.cpu(), wq.cpu(), sw.cpu(), None if b is None else b.cpu(), gelu)
        assert_close_bf16(ys.cpu(), r, gelu)


@pytest.mark.parametrize("M,K,N", [(64, 2048, 8192), (128, 8192, 2048), (40, 2048, 6144)])
def test_splitk_automatic_route(cuda_dev, M, K, N):
    """With the automatic choice, decode-batch shapes whose tiles fill fewer than half the SMs take split-K (or the
    A8 GEMV); every route gives the same bits."""
    xq, sx, wq, sw, b = operands(M, K, N, False, 5 + M, cuda_dev)
    ya = run(xq, sx, wq, sw, None, False, 0)
    yt = run(xq, sx, wq, sw, None, False, 128)
    assert torch.equal(ya, yt)


def test_splitk_repeated_and_graph(cuda_dev):
    """Back-to-back launches and a CUDA graph replay give the same bits (no state survives between calls)."""
    xq, sx, wq, sw, b = operands(64, 2048, 8192, True, 99, cuda_dev)
    ref = run(xq, sx, wq, sw, b, False, 1)
    _capi.lib().lfm2q_set_gemm_tile(1)
    try:
        ys = [torch.empty(64, 8192, device=cuda_dev, dtype=BF) for _ in range(3)]
        for y in ys:
            int8_ext().gemm_i8(xq, sx, wq, sw, b, y, False)
        torch.cuda.synchronize()
        for y in ys:
            assert torch.equal(y, ref)
        st = torch.cuda.Stream(cuda_dev)
        st.wait_stream(torch.cuda.current_stream(cuda_dev))
        yg = torch.empty(64, 8192, device=cuda_dev, dtype=BF)
        with torch.cuda.stream(st):
            int8_ext().gemm_i8(xq, sx, wq, sw, b, yg, False)
        torch.cuda.current_stream(cuda_dev).wait_stream(st)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            int8_ext().gemm_i8(xq, sx, wq, sw, b, yg, False)
        for _ in range(3):
            yg.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(yg, ref)
    finally:
        _capi.lib().lfm2q_set_gemm_tile(0)
    assert _capi.lib().lfm2q_check_device(0) == 0  # no pipeline wait gave up
