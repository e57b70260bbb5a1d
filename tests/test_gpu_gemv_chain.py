"""Chained decode GEMV (lfm2q_gemv_chain) on the B200.

Every layer's output is the weight-only GEMV y = bf16((x . W^T) * s) with the arithmetic of lfm2q_gemv's int8 tensor
path (tokens sliced into exact fixed-point bytes, exact int32 partial sums) wherever the slices fit, so:
  - against the oracle it meets the reference's own bound (tests/test_kernels.py:32) and the fp64 bound of the plain
    GEMV tests (relative error within 1.05x of the bf16 rounding of the exact value);
  - it equals lfm2q_gemv bit for bit wherever lfm2q_gemv takes that path for the same B;
  - a layer that reads an earlier layer's output sees that output complete: the chain equals running the same layers
    one single-layer chain at a time;
  - the L2 prefetch of the layers ahead changes no value: back-to-back calls give identical results.
"""

import pytest
import torch

from lfm2opt.kernels import GemvChain, ext
from lfm2opt.quant import quantize_int8
from test_gpu_gemv import check

pytestmark = pytest.mark.gpu
BF = torch.bfloat16

# the decode shapes (N, K) of the LFM2 stack and its head
STACK = [(3072, 2048), (2048, 2048), (6144, 2048), (2048, 2048), (16384, 2048), (2048, 8192), (65536, 2048)]


def weights(N, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    Wq, s = quantize_int8((torch.randn(N, K, generator=g) * 0.02).to(BF))
    return Wq.to(dev), s.to(dev)


def sliced_in_gemv(N, K, B):
    """Whether lfm2q_gemv runs an x-sliced int8 kernel for this shape on the default path (launch_gemv: the deep
    kernel up to 2 tokens whenever the slices fit, the ring kernel for 3-4 tokens from 8 M weights)."""
    fits = B <= 4 and B * 3 * (K + 64) <= 64 * 1024 and K <= 16384 // B
    return fits and (B <= 2 or N * K >= 8 * 1024 * 1024)


@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_chain_stack_matches_gemv_and_oracle(cuda_dev, B):
    g = torch.Generator().manual_seed(B)
    xs = {K: torch.randn(B, K, generator=g).to(BF).to(cuda_dev) for K in (2048, 8192)}
    layers = []
    for i, (N, K) in enumerate(STACK):
        W, s = weights(N, K, 100 + i, cuda_dev)
        y = torch.full((B, N), float("nan"), device=cuda_dev, dtype=BF)
        layers.append((W, s, xs[K], y))
    chain = GemvChain(layers)
    chain()
    torch.cuda.synchronize()
    for W, s, x, y in layers:
        N, K = W.shape
        check(y.cpu(), W.cpu(), s.cpu(), x.cpu())
        if sliced_in_gemv(N, K, B):
            r = torch.empty_like(y)
            ext().gemv(W, s, x, r)
            torch.cuda.synchronize()
            assert torch.equal(y, r), (N, K, B)
    # a second call gives the same values
    first = [y.clone() for _, _, _, y in layers]
    for _, _, _, y in layers:
        y.fill_(float("nan"))
    chain()
    torch.cuda.synchronize()
    for (_, _, _, y), f in zip(layers, first):
        assert torch.equal(y, f)


@pytest.mark.parametrize("B", [1, 2, 4])
def test_chain_dependencies(cuda_dev, B):
    """x of each layer is the previous layer's y (2048 -> 2048 -> 8192 -> 2048 -> 65536): the chain equals one-layer
    chains run in sequence, and every layer meets the oracle bound on the inputs it actually read."""
    dims = [2048, 2048, 8192, 2048, 65536]
    g = torch.Generator().manual_seed(40 + B)
    x0 = torch.randn(B, dims[0], generator=g).to(BF).to(cuda_dev)
    Ws = [weights(dims[i + 1], dims[i], 200 + i, cuda_dev) for i in range(len(dims) - 1)]
    ys = [torch.full((B, dims[i + 1]), float("nan"), device=cuda_dev, dtype=BF) for i in range(len(dims) - 1)]
    xin = [x0] + ys[:-1]
    chain = GemvChain([(W, s, xin[i], ys[i]) for i, (W, s) in enumerate(Ws)])
    chain()
    torch.cuda.synchronize()
    # one layer at a time, each on the previous one-layer result
    x = x0
    for i, (W, s) in enumerate(Ws):
        r = torch.full_like(ys[i], float("nan"))
        GemvChain([(W, s, x, r)])()
        torch.cuda.synchronize()
        assert torch.equal(ys[i], r), f"layer {i}"
        check(ys[i].cpu(), W.cpu(), s.cpu(), xin[i].cpu())
        x = r


def test_chain_small_and_ragged_shapes(cuda_dev):
    """N not a multiple of 16, K = 512, every layer with its own x."""
    B = 2
    shapes = [(40, 512), (1000, 1536), (17, 512), (3000, 4096), (2048, 2048)]
    g = torch.Generator().manual_seed(9)
    layers = []
    for i, (N, K) in enumerate(shapes):
        W, s = weights(N, K, 300 + i, cuda_dev)
        x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
        layers.append((W, s, x, torch.empty(B, N, device=cuda_dev, dtype=BF)))
    GemvChain(layers)()
    torch.cuda.synchronize()
    for W, s, x, y in layers:
        check(y.cpu(), W.cpu(), s.cpu(), x.cpu())


@pytest.mark.parametrize("B", [4])
def test_chain_wide_k_takes_bf16_path(cuda_dev, B):
    """B = 4 at K = 8192: the token slices do not fit, the layer runs on the bf16 path inside the chain."""
    W, s = weights(2048, 8192, 7, cuda_dev)
    x = torch.randn(B, 8192, device=cuda_dev).to(BF)
    y = torch.empty(B, 2048, device=cuda_dev, dtype=BF)
    r = torch.empty_like(y)
    GemvChain([(W, s, x, y)])()
    ext().gemv(W, s, x, r)
    torch.cuda.synchronize()
    assert torch.equal(y, r)
    check(y.cpu(), W.cpu(), s.cpu(), x.cpu())
