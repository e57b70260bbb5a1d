"""Decode GEMV on the B200 against the oracle.

The reference's own bound (tests/test_kernels.py:32): max|err| <= 2e-2 * max(max|ref|, 1) against
F.linear(x.float(), Wq.float() * scale).to(bf16). Tighter here: against the fp64 value, the relative Frobenius error
stays within 1.05x of the bf16 rounding error of the exact result (fp32 accumulation adds ~1e-6 relative).
"""

import pytest
import torch

import oracle
from conftest import golden, to_t
from lfm2opt.kernels import ext
from lfm2opt.quant import quantize_int8

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def check(y, W, s, x):
    ref = oracle.gemv_ref(W, s, x)
    err = (y.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * max(ref.float().abs().max().item(), 1.0), err
    r64 = oracle.gemv_f64(W, s, x)
    e = ((y.double() - r64).norm() / r64.norm()).item()
    e_round = ((r64.to(BF).double() - r64).norm() / r64.norm()).item()
    assert e <= 1.05 * e_round + 1e-6, (e, e_round)


SHAPES = [(3072, 2048), (6144, 2048), (2048, 2048), (16384, 2048), (2048, 8192), (65536, 2048), (40, 512),
          (1000, 1536)]


@pytest.fixture(params=[0, 1, 2, 4], ids=["auto", "bf16path", "deep", "ring"])
def gemv_path(request):
    """0: the int8 path with the tokens sliced into exact fixed-point bytes (deep kernel up to 2 tokens, ring kernel
    for 3-4 from 8 M weights), else bf16; 1: always bf16; 2: the deep kernel wherever the slices fit; 4: the ring
    kernel from 8 M weights."""
    from lfm2opt import _capi
    _capi.lib().lfm2q_set_gemv_path(request.param)
    yield request.param
    _capi.lib().lfm2q_set_gemv_path(0)


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("B", [1, 2, 3, 4, 7, 8, 13, 16, 19])
def test_gemv_int8(cuda_dev, gemv_path, N, K, B):
    if N * K > 40_000_000 and B not in (1, 8, 16):
        pytest.skip("large shape: a few batch sizes suffice")
    if gemv_path in (1, 2, 4) and B > 4:
        pytest.skip("the path knob only matters for B <= 4")
    g = torch.Generator().manual_seed(N + K + B)
    W = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    Wq, s = quantize_int8(W)
    x = torch.randn(B, K, generator=g).to(BF)
    y = torch.empty(B, N, device=cuda_dev, dtype=BF)
    ext().gemv(Wq.to(cuda_dev), s.to(cuda_dev), x.to(cuda_dev), y)
    check(y.cpu(), Wq, s, x)


def _token_scales():
    """Tokens spanning the fp range: plain, outlier channels x1000, tiny (1e-30), huge (1e30), all zero, one nonzero
    element, bf16 subnormals."""
    g = torch.Generator().manual_seed(11)
    K = 2048
    x = torch.randn(7, K, generator=g)
    x[1, ::97] *= 1000.0
    x[2] *= 1e-30
    x[3] *= 1e30
    x[4] = 0.0
    x[5] = 0.0
    x[5, 1234] = -3.5
    x[6] = torch.randn(K, generator=g) * 2.0 ** -130
    return x.to(BF)


@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_gemv_int8_sliced_extremes(cuda_dev, B):
    """The x-sliced int8 path picks a power-of-two scale per token from its absmax: tokens of very different
    magnitude, zero tokens and subnormal tokens are each within the rounding bound of their own exact result."""
    xs = _token_scales()
    g = torch.Generator().manual_seed(B)
    N = 4096  # N * K = 8 M weights: the sliced path
    Wq = torch.randint(-127, 128, (N, 2048), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 1e-3 + 1e-4
    for i0 in range(0, xs.shape[0], B):
        x = xs[i0:i0 + B]
        y = torch.empty(x.shape[0], N, device=cuda_dev, dtype=BF)
        ext().gemv(Wq.to(cuda_dev), s.to(cuda_dev), x.to(cuda_dev), y)
        r64 = oracle.gemv_f64(Wq, s, x)
        for b in range(x.shape[0]):
            if r64[b].abs().max() == 0:
                assert (y[b].cpu() == 0).all()
                continue
            e = ((y[b].cpu().double() - r64[b]).norm() / r64[b].norm()).item()
            e_round = ((r64[b].to(BF).double() - r64[b]).norm() / r64[b].norm()).item()
            assert e <= 1.05 * e_round + 1e-6, (i0 + b, e, e_round)


@pytest.mark.parametrize("N", [3072, 4096], ids=["bf16path", "sliced"])
@pytest.mark.parametrize("rows", [1, 2, 4, 8])
def test_gemv_kslices_agree(cuda_dev, rows, N):
    """The K-split tuning knob changes only the fp32 summation order (bf16 path) or nothing at all (ring sliced
    kernel: exact int32 partial sums)."""
    from lfm2opt import _capi
    _capi.lib().lfm2q_set_gemv_path(1 if N == 3072 else 4)
    try:
        _kslices_case(cuda_dev, rows, N)
    finally:
        _capi.lib().lfm2q_set_gemv_path(0)


def _kslices_case(cuda_dev, rows, N):
    g = torch.Generator().manual_seed(rows)
    Wq = torch.randint(-127, 128, (N, 2048), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 1e-3
    x = torch.randn(2, 2048, generator=g).to(BF)
    y = torch.empty(2, N, device=cuda_dev, dtype=BF)
    ext().gemv(Wq.to(cuda_dev), s.to(cuda_dev), x.to(cuda_dev), y, rows)
    check(y.cpu(), Wq, s, x)
    if N == 4096:
        y1 = torch.empty_like(y)
        ext().gemv(Wq.to(cuda_dev), s.to(cuda_dev), x.to(cuda_dev), y1, 1)
        assert torch.equal(y, y1)


@pytest.mark.parametrize("B", [1, 5])
def test_gemv_bf16_weights(cuda_dev, B):
    g = torch.Generator().manual_seed(B)
    W = (torch.randn(2048, 1024, generator=g) * 0.02).to(BF)
    x = torch.randn(B, 1024, generator=g).to(BF)
    y = torch.empty(B, 2048, device=cuda_dev, dtype=BF)
    ext().gemv(W.to(cuda_dev), None, x.to(cuda_dev), y)
    check(y.cpu(), W, None, x)


def test_gemv_golden(cuda_dev):
    d = golden("gemv")
    n = len([k for k in d.files if k.startswith("name")])
    for i in range(n):
        name = str(d[f"name{i}"])
        W = to_t(d[f"W{i}"], bf16="bf16" in name)
        s = to_t(d[f"s{i}"]) if d[f"s{i}"].size else None
        x = to_t(d[f"x{i}"], bf16=True)
        y = torch.empty(x.shape[0], W.shape[0], device=cuda_dev, dtype=BF)
        ext().gemv(W.to(cuda_dev), None if s is None else s.to(cuda_dev), x.to(cuda_dev), y)
        ref = to_t(d[f"y{i}"], bf16=True)
        err = (y.cpu().float() - ref.float()).abs().max().item()
        assert err <= 2e-2 * max(ref.float().abs().max().item(), 1.0), name


@pytest.mark.parametrize("int8", [True, False])
def test_gemv_epi_swiglu(cuda_dev, int8):
    """Epilogue 0 equals the plain GEMV's bf16 outputs (same K-slicing) followed by silu_mul (<= 1 bf16 ulp: the
    GPU uses __expf)."""
    g = torch.Generator().manual_seed(5)
    H, I = 2048, 8192
    x = torch.randn(1, H, generator=g).to(BF).to(cuda_dev)
    W = (torch.randn(2 * I, H, generator=g) * 0.02).to(BF)
    s = None
    if int8:
        W, s = quantize_int8(W)
        s = s.to(cuda_dev)
    W = W.to(cuda_dev)
    gout = torch.empty(1, 2 * I, device=cuda_dev, dtype=BF)
    ext().gemv(W, s, x, gout, 4)
    out = torch.empty(1, I, device=cuda_dev, dtype=BF)
    ext().gemv_epi(0, W, s, x, out)
    ref = oracle.gemm.silu_mul_ref(gout.cpu())
    ok, detail = oracle.silu_chain_close(out.cpu(), ref)
    assert ok, detail


@pytest.mark.parametrize("int8", [True, False])
@pytest.mark.parametrize("with_bias", [True, False])
def test_gemv_epi_shortconv(cuda_dev, int8, with_bias):
    """Epilogue 1 equals the plain GEMV's bf16 outputs followed by the short-conv step, bit for bit, state too."""
    g = torch.Generator().manual_seed(6)
    H = 2048
    x = torch.randn(1, H, generator=g).to(BF).to(cuda_dev)
    W = (torch.randn(3 * H, H, generator=g) * 0.02).to(BF)
    s = None
    if int8:
        W, s = quantize_int8(W)
        s = s.to(cuda_dev)
    W = W.to(cuda_dev)
    cw = (torch.randn(H, 3, generator=g) * 0.5).to(BF)
    cb = (torch.randn(H, generator=g) * 0.1).to(BF) if with_bias else None
    st0 = torch.randn(1, H, 3, generator=g).to(BF)
    parts = torch.empty(1, 3 * H, device=cuda_dev, dtype=BF)
    ext().gemv(W, s, x, parts, 2)
    st = st0.clone().to(cuda_dev)
    out = torch.empty(1, H, device=cuda_dev, dtype=BF)
    ext().gemv_epi(1, W, s, x, out, st, cw.to(cuda_dev), None if cb is None else cb.to(cuda_dev))
    p = parts.cpu().reshape(-1)
    b_, c_, x_ = p[:H].float(), p[H:2 * H].float(), p[2 * H:].float()
    bx = (b_ * x_).to(BF).float()
    s0 = st0.reshape(H, 3).float()
    wf = cw.float()
    acc = wf[:, 0] * s0[:, 1]
    acc = acc + wf[:, 1] * s0[:, 2]
    acc = acc + wf[:, 2] * bx
    if cb is not None:
        acc = acc + cb.float()
    ref = (c_ * acc.to(BF).float()).to(BF)
    assert torch.equal(out.cpu().reshape(-1), ref)
    new_state = torch.stack([s0[:, 1], s0[:, 2], bx], 1).to(BF)
    assert torch.equal(st.cpu().reshape(H, 3), new_state)


@pytest.mark.parametrize("N,K", [(3072, 2048), (2048, 8192), (65536, 2048), (16384, 2048), (40, 512), (264, 1152)])
@pytest.mark.parametrize("B", [1, 2, 7, 8, 9, 16, 19, 32, 33, 64, 100])
@pytest.mark.parametrize("gelu", [False, True])
def test_gemv_a8_bit_exact(cuda_dev, N, K, B, gelu):
    """A8 GEMV = the per-token W8A8 epilogue on the exact int32 sum: identical to the gemm_i8 oracle."""
    if N * K > 40_000_000 and (B not in (1, 16, 64) or gelu):
        pytest.skip("large shape: a few cases suffice")
    g = torch.Generator().manual_seed(N + K + B + gelu)
    W = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    Wq, sw = quantize_int8(W)
    x = torch.randn(B, K, generator=g).to(BF)
    b = (torch.randn(N, generator=g) * 0.1).to(BF) if gelu else None
    xq, sx = oracle.quant_rows_ref(x)
    y = torch.empty(B, N, device=cuda_dev, dtype=BF)
    ext().gemv_a8(Wq.to(cuda_dev), sw.to(cuda_dev), xq.to(cuda_dev), sx.to(cuda_dev), y,
                  None if b is None else b.to(cuda_dev), gelu)
    r = oracle.gemm_i8_ref(xq, sx, Wq, sw, b, gelu)
    from test_gpu_gemm import assert_close_bf16
    assert_close_bf16(y.cpu(), r, gelu)


@pytest.mark.parametrize("N,K", [(3072, 2048), (2048, 8192), (65536, 2048), (264, 1152), (40, 4352)])
@pytest.mark.parametrize("B", [1, 3, 8, 9, 16, 40])
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_a8_fused_quant(cuda_dev, N, K, B, gelu):
    """quant_rows fused into the A8 GEMV equals quant_rows followed by the gemm_i8 oracle, bit for bit."""
    if N * K > 40_000_000 and (B not in (1, 16) or gelu):
        pytest.skip("large shape: a few cases suffice")
    from lfm2opt.kernels import int8_ext
    g = torch.Generator().manual_seed(N + 3 * K + B)
    W = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    Wq, sw = quantize_int8(W)
    x = (torch.randn(B, K, generator=g) * (1 + torch.rand(B, 1, generator=g) * 4)).to(BF)
    b = (torch.randn(N, generator=g) * 0.1).to(BF) if gelu else None
    y = torch.empty(B, N, device=cuda_dev, dtype=BF)
    int8_ext().linear_a8(x.to(cuda_dev), Wq.to(cuda_dev), sw.to(cuda_dev), None if b is None else b.to(cuda_dev), y,
                         gelu)
    xq, sx = oracle.quant_rows_ref(x)
    r = oracle.gemm_i8_ref(xq, sx, Wq, sw, b, gelu)
    from test_gpu_gemm import assert_close_bf16
    assert_close_bf16(y.cpu(), r, gelu)
