"""W8A8 tcgen05 GEMMs on the B200 against the oracle.

Per-token: the int32 accumulator is exact and the fp32 epilogue has the reference's operation order, so the bf16
output must equal the oracle bit for bit (0 ulp); with GELU (tanhf on the GPU, torch's tanh on the CPU) within
1 bf16 ulp, the reference's own bound (tests/test_int8_gemm.py:174). Grouped: the fp32 fold is restated exactly
(fmaf per group, in order), so again 0 ulp, and the reference's 1.05x-of-bf16-rounding bound against fp64 holds.
"""

import pytest
import torch

import oracle
from conftest import golden, to_t
from lfm2opt import _capi
from lfm2opt.int8 import quantize_rows
from lfm2opt.kernels import int8_ext
from lfm2opt.quant import quantize_int8

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def assert_close_bf16(y, r, gelu):
    """0 ulp without GELU. With GELU <= 1 ulp, except in the fp32 cancellation region of 0.5 v (1 + tanh(u)) near
    tanh = -1 (v < ~ -4.5): there the fp32 value of 1 + tanh is a few units of 2^-24, CUDA's tanhf and the CPU's
    vectorised tanh may round it differently, and the outputs (|y| < 2e-7) may differ by up to 4e-7 absolute."""
    if not gelu:
        assert oracle.bf16_ulps(y, r) == 0
        return
    ia, ib = y.view(torch.int16).int(), r.view(torch.int16).int()
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    bad = ((ia - ib).abs() > 1) & ((y.float() - r.float()).abs() > 4e-7)
    assert not bad.any(), (bad.sum().item(), y[bad][:4], r[bad][:4])


def make(M, K, N, bias, seed, outlier_ch=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(BF)
    if outlier_ch:
        x[:, 5 % K] *= 30
    w = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    b = torch.randn(N, generator=g).to(BF) if bias else None
    return x, w, b


@pytest.fixture(params=[0, 128, 256, -192, -256, 1], ids=["auto", "bn128", "bn256", "pair192", "pair256", "splitk"])
def tile(request):
    """Tile override: 0 = automatic; 128 / 256 = one CTA per 128 x that many columns; -192 / -256 = a CTA pair
    (cluster of 2, tcgen05 cta_group::2) per 256 x that many columns; 1 = K split over a cluster of CTAs per 128 x 128
    tile (partials summed in distributed shared memory) wherever K has two 128-byte blocks per CTA."""
    _capi.lib().lfm2q_set_gemm_tile(request.param)
    yield request.param
    _capi.lib().lfm2q_set_gemm_tile(0)


TOKEN_CASES = [(9216, 1152, 3456, True, False), (9216, 1152, 4304, True, True), (2327, 2048, 16384, False, False),
               (272, 2048, 3072, False, False), (17, 2048, 2048, False, False), (1, 1152, 1152, True, False),
               (300, 1152, 1152, True, True), (16, 2048, 8192, False, False), (130, 4304, 1152, False, False),
               (129, 144, 264, True, False), (5, 16, 8, False, False), (4096, 8192, 2048, False, False),
               (383, 1152, 200, True, True), (640, 2048, 1152, True, False), (48, 2048, 6144, True, True),
               (64, 8192, 2048, False, False), (24, 2048, 3072, False, False), (65, 2048, 2048, True, False)]


@pytest.mark.parametrize("M,K,N,bias,gelu", TOKEN_CASES)
def test_gemm_i8_per_token(cuda_dev, tile, M, K, N, bias, gelu):
    if tile and M * N > 40_000_000:
        pytest.skip("forced tiles: the automatic run covers the big shapes")
    x, w, b = make(M, K, N, bias, M + K + N)
    xq, sx = quantize_rows(x.to(cuda_dev))
    wq, sw = quantize_int8(w)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8(xq, sx, wq.to(cuda_dev), sw.to(cuda_dev), None if b is None else b.to(cuda_dev), y, gelu)
    r = oracle.gemm_i8_ref(xq.cpu(), sx.cpu(), wq, sw, b, gelu)
    assert_close_bf16(y.cpu(), r, gelu)
    assert _capi.lib().lfm2q_check_device(0) == 0


def test_gemm_i8_int32_accumulator_exact(cuda_dev):
    """With unit scales and no bias the output is bf16(float(acc)): the int32 accumulator is checked through it on
    magnitudes where bf16 is exact (|acc| <= 256) and on the full range through the fp32 rounding."""
    g = torch.Generator().manual_seed(9)
    M, K, N = 257, 512, 384
    xq = torch.randint(-2, 3, (M, K), generator=g, dtype=torch.int8)
    wq = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    ones_m, ones_n = torch.ones(M), torch.ones(N)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8(xq.to(cuda_dev), ones_m.to(cuda_dev), wq.to(cuda_dev), ones_n.to(cuda_dev), None, y, False)
    acc = oracle.int_mm_exact(xq, wq)
    small = acc.abs() <= 256
    assert torch.equal(y.cpu().float()[small], acc.float()[small])
    assert torch.equal(y.cpu(), acc.float().to(BF))


def test_gemm_i8_golden(cuda_dev):
    d = golden("gemm_i8")
    for i in range(4):
        M, K, N, bias, gelu = (int(v) for v in d[f"meta{i}"])
        b = to_t(d[f"b{i}"], bf16=True).to(cuda_dev) if bias else None
        y = torch.empty(M, N, device=cuda_dev, dtype=BF)
        int8_ext().gemm_i8(to_t(d[f"xq{i}"]).to(cuda_dev), to_t(d[f"sx{i}"]).to(cuda_dev),
                           to_t(d[f"wq{i}"]).to(cuda_dev), to_t(d[f"sw{i}"]).to(cuda_dev), b, y, bool(gelu))
        assert_close_bf16(y.cpu(), to_t(d[f"y{i}"], bf16=True), gelu)


GROUP_CASES = [(9216, 1152, 3456, True, False), (9216, 4352, 1152, True, False), (2327, 8192, 2048, False, False),
               (1024, 1152, 4352, True, True), (17, 2048, 2048, False, False), (1, 1152, 1152, True, False),
               (33, 192, 136, True, False)]


@pytest.mark.parametrize("M,K,N,bias,gelu", GROUP_CASES)
def test_gemm_i8_grouped(cuda_dev, M, K, N, bias, gelu):
    x, w, b = make(M, K, N, bias, 3 * M + K + N, outlier_ch=True)
    xq, sxT = quantize_rows(x.to(cuda_dev), 64)
    wq, sw = quantize_int8(w)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8(xq, sxT, wq.to(cuda_dev), sw.to(cuda_dev), None if b is None else b.to(cuda_dev), y, gelu)
    xq, sxT = xq.cpu(), sxT.cpu()
    r = oracle.gemm_i8_grouped_ref(xq, sxT, wq, sw, b, gelu)
    assert_close_bf16(y.cpu(), r, gelu)
    if M * N <= 4_000_000:  # the reference's own acceptance bound against fp64
        r64 = oracle.gemm_i8_grouped_f64(xq, sxT, wq, sw, b, gelu)
        e_ours = ((y.cpu().double() - r64).norm() / r64.norm()).item()
        e_round = ((r64.to(BF).double() - r64).norm() / r64.norm()).item()
        assert e_ours <= 1.05 * e_round + 1e-6


def test_gemm_i8_grouped_golden(cuda_dev):
    d = golden("gemm_i8_grouped")
    for i in range(3):
        M, K, N, bias, gelu = (int(v) for v in d[f"meta{i}"])
        b = to_t(d[f"b{i}"], bf16=True) if bias else None
        y = torch.empty(M, N, device=cuda_dev, dtype=BF)
        int8_ext().gemm_i8(to_t(d[f"xq{i}"]).to(cuda_dev), to_t(d[f"sx{i}"]).to(cuda_dev),
                           to_t(d[f"wq{i}"]).to(cuda_dev), to_t(d[f"sw{i}"]).to(cuda_dev),
                           None if b is None else b.to(cuda_dev), y, bool(gelu))
        r = to_t(d[f"r{i}"])
        e_ours = ((y.cpu().double() - r).norm() / r.norm()).item()
        e_round = ((r.to(BF).double() - r).norm() / r.norm()).item()
        assert e_ours <= 1.05 * e_round + 1e-6, (i, e_ours, e_round)


@pytest.mark.parametrize("M,K,N,bias,gelu", [(9216, 1152, 4352, True, True), (1024, 1152, 4352, True, True),
                                             (37, 2048, 2048, False, False), (300, 4352, 1152, True, False)])
def test_gemm_i8_q(cuda_dev, M, K, N, bias, gelu):
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, K, generator=g).to(BF)
    w = (torch.randn(N, K, generator=g) * 0.05).to(BF)
    b = torch.randn(N, generator=g).to(BF).to(cuda_dev) if bias else None
    xq, sxT = quantize_rows(x.to(cuda_dev), 64)
    wq, sw = quantize_int8(w.to(cuda_dev))
    E = int8_ext()
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    E.gemm_i8(xq, sxT, wq, sw, b, y, gelu)
    rq, rs = quantize_rows(y, 64)  # the reference's definition: gemm_i8 -> grouped quant_rows, exactly
    q, s = torch.empty_like(rq), torch.empty_like(rs)
    E.gemm_i8_q(xq, sxT, wq, sw, b, q, s, gelu)
    assert torch.equal(q, rq) and torch.equal(s, rs)
    if not gelu:
        oq, os_ = oracle.gemm_i8_q_ref(xq.cpu(), sxT.cpu(), wq.cpu(), sw.cpu(), None if b is None else b.cpu())
        assert torch.equal(q.cpu(), oq) and torch.equal(s.cpu(), os_)


@pytest.fixture(params=[0, 256, -256], ids=["auto", "one_cta", "pair"])
def silu_tile(request):
    _capi.lib().lfm2q_set_gemm_tile(request.param)
    yield request.param
    _capi.lib().lfm2q_set_gemm_tile(0)


@pytest.mark.parametrize("M,K,I,bias", [(4096, 2048, 8192, False), (1024, 2048, 8192, True), (17, 2048, 8192, False),
                                        (300, 1152, 264, True), (1, 64, 8, False), (385, 2048, 200, True)])
def test_gemm_i8_silu(cuda_dev, silu_tile, M, K, I, bias):
    if silu_tile and M * I > 20_000_000:
        pytest.skip("forced tiles: the automatic run covers the big shapes")
    x, w, b = make(M, K, 2 * I, bias, M * 3 + I)
    xq, sx = quantize_rows(x.to(cuda_dev))
    wq, sw = quantize_int8(w)
    y = torch.empty(M, I, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8_silu(xq, sx, wq.to(cuda_dev), sw.to(cuda_dev), None if b is None else b.to(cuda_dev), y)
    r = oracle.gemm_i8_silu_ref(xq.cpu(), sx.cpu(), wq, sw, b)
    ok, detail = oracle.silu_chain_close(y.cpu(), r)
    assert ok, detail


def test_device_error_word_clear(cuda_dev):
    torch.cuda.synchronize()
    assert _capi.lib().lfm2q_check_device(1) == 0


# ------------------------------------------------------------------------------------------------ W8A16
W8_CASES = [(9216, 4304, 1152, True, False), (2327, 8192, 2048, False, False), (272, 8192, 2048, False, False),
            (9, 2048, 6144, False, False), (1, 2048, 2048, False, False), (1024, 1152, 4304, True, True),
            (4096, 2048, 8192, False, False), (300, 1152, 264, True, False), (517, 16, 40, True, True)]


@pytest.fixture(params=[0, 128, 64, -256], ids=["auto", "one_cta", "narrow", "pair"])
def w8_tile(request):
    _capi.lib().lfm2q_set_gemm_tile(request.param)
    yield request.param
    _capi.lib().lfm2q_set_gemm_tile(0)


@pytest.mark.parametrize("M,K,N,bias,gelu", W8_CASES)
def test_gemm_w8(cuda_dev, w8_tile, M, K, N, bias, gelu):
    """W8A16 (bf16 x, int8 W converted exactly to bf16, fp32 accumulation): products are exact, so against fp64 the
    relative error is the bf16 output rounding plus fp32 summation (<= 1.05x the rounding error); the reference's own
    acceptance, <= 1.5x the error of a bf16 GEMM on dequantized weights (tests/test_int8_gemm.py:178-196), follows."""
    if w8_tile and M * N > 12_000_000:
        pytest.skip("forced tiles: the automatic run covers the big shapes")
    g = torch.Generator().manual_seed(M + 7 * N + K)
    x = torch.randn(M, K, generator=g).to(BF)
    w = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    b = torch.randn(N, generator=g).to(BF) if bias else None
    wq, sw = quantize_int8(w)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    int8_ext().gemm_w8(x.to(cuda_dev), wq.to(cuda_dev), sw.to(cuda_dev), None if b is None else b.to(cuda_dev), y, gelu)
    assert _capi.lib().lfm2q_check_device(0) == 0
    r64 = oracle.gemm_w8_f64(x, wq, sw, b, gelu)
    yc = y.cpu().double()
    e_ours = ((yc - r64).norm() / r64.norm()).item()
    e_round = ((r64.to(BF).double() - r64).norm() / r64.norm()).item()
    assert e_ours <= 1.05 * e_round + 1e-6, (e_ours, e_round)
    if M * N * K <= 4e9:
        wd = (wq.float() * sw[:, None]).to(BF)
        rc = torch.nn.functional.linear(x.float(), wd.float(), None if b is None else b.float())
        if gelu:
            rc = torch.nn.functional.gelu(rc, approximate="tanh")
        e_cub = ((rc.to(BF).double() - r64).norm() / r64.norm()).item()
        assert e_ours <= 1.5 * e_cub + 1e-4, (e_ours, e_cub)


@pytest.mark.parametrize("epi", ["none", "gelu", "silu"])
def test_gemm_i8_accumulators_beyond_2p22(cuda_dev, epi):
    """Rows whose int32 sums reach 127 * 127 * K (all codes +-127), far beyond 2^24: (float)acc must round to nearest
    even exactly as the oracle's float(acc) does, in every epilogue."""
    M, K, N = 300, 2048, 1024
    g = torch.Generator().manual_seed(77)
    x = torch.randn(M, K, generator=g)
    x[::3] = 1.0          # every third row quantizes to 127 everywhere
    x[1::3] = torch.sign(torch.randn(K, generator=g))  # +-1 rows: +-127
    x = x.to(BF)
    w = (torch.randn(N, K, generator=g) * 0.02)
    w[: N // 4] = 0.02    # a quarter of the weight rows quantize to 127 everywhere
    w = w.to(BF)
    wq, sw = quantize_int8(w)
    b = (torch.randn(N, generator=g) * 0.1).to(BF)
    xq, sx = oracle.quant_rows_ref(x)
    assert int(oracle.int_mm_exact(xq, wq).abs().max()) >= 1 << 22
    dev = cuda_dev
    if epi == "silu":
        y = torch.empty(M, N // 2, device=dev, dtype=BF)
        int8_ext().gemm_i8_silu(xq.to(dev), sx.to(dev), wq.to(dev), sw.to(dev), b.to(dev), y)
        ok, detail = oracle.silu_chain_close(y.cpu(), oracle.gemm_i8_silu_ref(xq, sx, wq, sw, b))
        assert ok, detail
    else:
        y = torch.empty(M, N, device=dev, dtype=BF)
        int8_ext().gemm_i8(xq.to(dev), sx.to(dev), wq.to(dev), sw.to(dev), b.to(dev), y, epi == "gelu")
        assert_close_bf16(y.cpu(), oracle.gemm_i8_ref(xq, sx, wq, sw, b, epi == "gelu"), epi == "gelu")
