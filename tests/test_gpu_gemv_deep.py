"""Deep-prefetch x-sliced decode GEMV (gemv path 2 / 3) on the B200.

The deep kernel computes exactly what the ring x-sliced kernel computes (exact int32 partial sums of the sliced
tokens, the same fp32 combination), with another schedule: one block per SM, each warp's weight steps over all of its
row groups streamed through one ring requested before the dependency wait, the dependent launch triggered at the start
(path 2) or after the last row group (path 3). So:
  - it equals the ring kernel bit for bit (a one-layer GemvChain on path 4 always runs the ring kernel);
  - it meets the oracle bound of the plain GEMV tests;
  - in a chain of dependent GEMVs (each x the previous y) launched with PDL and early triggers, every layer reads
    its input complete: the chain equals the same layers run one at a time on the ring kernel.
"""

import pytest
import torch

from lfm2opt import _capi
from lfm2opt.kernels import GemvChain, ext
from lfm2opt.quant import quantize_int8
from test_gpu_gemv import check

pytestmark = pytest.mark.gpu
BF = torch.bfloat16

SHAPES = [(3072, 2048), (2048, 2048), (6144, 2048), (16384, 2048), (2048, 8192), (65536, 2048), (40, 512),
          (1000, 1536), (17, 4096), (4096, 16384)]


@pytest.fixture(params=[2, 3], ids=["early", "late"])
def deep(request):
    _capi.lib().lfm2q_set_gemv_path(request.param)
    yield request.param
    _capi.lib().lfm2q_set_gemv_path(0)


def weights(N, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    Wq, s = quantize_int8((torch.randn(N, K, generator=g) * 0.02).to(BF))
    return Wq.to(dev), s.to(dev)


def ring_result(W, s, x):
    """The ring x-sliced kernel's values (path 4, one-layer chain)."""
    _capi.lib().lfm2q_set_gemv_path(4)
    y = torch.full((x.shape[0], W.shape[0]), float("nan"), device=x.device, dtype=BF)
    GemvChain([(W, s, x, y)])()
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_deep_equals_ring_kernel(cuda_dev, deep, N, K, B):
    if K * B > 16384:
        pytest.skip("the slices do not fit: not the sliced path")
    W, s = weights(N, K, N + 7 * K + B, cuda_dev)
    g = torch.Generator().manual_seed(B * 131 + K)
    x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
    x[:, :: max(1, K // 7)] *= 300  # outlier channels
    r = ring_result(W, s, x)
    _capi.lib().lfm2q_set_gemv_path(deep)
    y = torch.full_like(r, float("nan"))
    ext().gemv(W, s, x, y)
    torch.cuda.synchronize()
    assert torch.equal(y, r), (N, K, B)
    if N * K <= 64 * 2**20:
        check(y.cpu(), W.cpu(), s.cpu(), x.cpu())


@pytest.mark.parametrize("B", [1, 2, 4])
def test_deep_dependent_chain(cuda_dev, deep, B):
    """2048 -> 6144 -> 2048 -> 16384 -> 2048 -> 8192 -> 2048 -> 65536, each layer reading the previous output, as
    consecutive launches (PDL) and as one GemvChain, both on the deep kernel, equal to one-at-a-time ring results."""
    dims = [2048, 6144, 2048, 16384, 2048, 8192, 2048, 65536]
    g = torch.Generator().manual_seed(50 + B)
    x0 = torch.randn(B, dims[0], generator=g).to(BF).to(cuda_dev)
    Ws = [weights(dims[i + 1], dims[i], 400 + i, cuda_dev) for i in range(len(dims) - 1)]
    ok_shapes = [B * dims[i] <= 16384 for i in range(len(dims) - 1)]
    # reference: one layer at a time on the ring kernel
    ref, x = [], x0
    for W, s in Ws:
        x = ring_result(W, s, x)
        ref.append(x)
    _capi.lib().lfm2q_set_gemv_path(deep)
    for attempt in range(2):  # consecutive launches, then the chain API
        ys = [torch.full((B, dims[i + 1]), float("nan"), device=cuda_dev, dtype=BF) for i in range(len(Ws))]
        xin = [x0] + ys[:-1]
        if attempt == 0:
            for i, (W, s) in enumerate(Ws):
                ext().gemv(W, s, xin[i], ys[i])
        else:
            GemvChain([(W, s, xin[i], ys[i]) for i, (W, s) in enumerate(Ws)])()
        torch.cuda.synchronize()
        for i in range(len(Ws)):
            if ok_shapes[i]:
                assert torch.equal(ys[i], ref[i]), (attempt, i)
            else:  # the bf16 path for this layer: the oracle bound on the input it read
                check(ys[i].cpu(), Ws[i][0].cpu(), Ws[i][1].cpu(), xin[i].cpu())


def test_deep_graph_replay(cuda_dev, deep):
    """A CUDA graph of 12 dependent deep GEMVs (ping-pong buffers, the decode pattern) replayed 5 times gives the
    same values as eager launches."""
    B = 1
    g = torch.Generator().manual_seed(3)
    Ws = [weights(2048, 2048, 900 + i, cuda_dev) for i in range(12)]
    x0 = torch.randn(B, 2048, generator=g).to(BF).to(cuda_dev)
    bufs = [torch.empty(B, 2048, device=cuda_dev, dtype=BF) for _ in range(2)]

    def run():
        x = x0
        for i, (W, s) in enumerate(Ws):
            y = bufs[i % 2]
            ext().gemv(W, s, x, y)
            x = y
        return x

    eager = run().clone()
    torch.cuda.synchronize()
    st = torch.cuda.Stream(cuda_dev)
    st.wait_stream(torch.cuda.current_stream(cuda_dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        run()
    torch.cuda.current_stream(cuda_dev).wait_stream(st)
    with torch.cuda.graph(graph):
        out = run()
    for _ in range(5):
        bufs[0].fill_(float("nan"))
        bufs[1].fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
