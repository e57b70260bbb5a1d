"""INT4 weight-only decode GEMV (lfm2q_gemv_w4, ext().gemv_w4) on the B200.

Parity: the reference's own bound (tests/test_kernels.py:32, applied to its INT4 case at :148-150): max|err| <=
2e-2 * max(max|ref|, 1) against F.linear(x.float(), dequantize_int4(Wp, S)).to(bf16); tighter, against the fp64
value of the dequantized product, the relative Frobenius error within 1.05x of the bf16 rounding error of the exact
result. The kernel's partial sums are exact integers per group (tokens sliced into exact fixed-point bytes), scaled
and summed in fp32. Also the golden vectors made by the reference's own code, and the reference's kernel on the
same GPU."""

import ctypes
from pathlib import Path

import pytest
import torch

import oracle
from conftest import golden, to_t
from lfm2opt import _capi
from lfm2opt.kernels import ext
from lfm2opt.quant import quantize_int4

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def check(y, Wp, S, x):
    ref = oracle.gemv_w4_ref(Wp, S, x)
    err = (y.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * max(ref.float().abs().max().item(), 1.0), err
    r64 = oracle.gemv_w4_f64(Wp, S, x)
    e = ((y.double() - r64).norm() / r64.norm()).item()
    e_round = ((r64.to(BF).double() - r64).norm() / r64.norm()).item()
    assert e <= 1.05 * e_round + 1e-6, (e, e_round)


def run(Wp, S, x, group, dev):
    """lfm2q_gemv_w4 through the C ABI for B = x.shape[0] tokens."""
    B, K = x.shape
    N = Wp.shape[0]
    y = torch.full((B, N), float("nan"), device=dev, dtype=BF)
    Wd, Sd, xd = Wp.to(dev), S.to(dev), x.to(dev)
    _capi.call("lfm2q_gemv_w4", Wd.data_ptr(), Sd.data_ptr(), xd.data_ptr(), y.data_ptr(), N, K, group, B,
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return y.cpu()


SHAPES = [(3072, 2048), (2048, 2048), (6144, 2048), (16384, 2048), (2048, 8192), (65536, 2048), (40, 512),
          (1000, 1536), (17, 128)]


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_gemv_w4(cuda_dev, N, K, B):
    if B * K > 16384:
        pytest.skip("B * K <= 16384")
    if N * K > 40_000_000 and B not in (1, 4):
        pytest.skip("large shape: a few batch sizes suffice")
    g = torch.Generator().manual_seed(N + K + B)
    W = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    Wp, S = quantize_int4(W)
    x = torch.randn(B, K, generator=g).to(BF)
    check(run(Wp, S, x, 128, cuda_dev), Wp, S, x)


@pytest.mark.parametrize("group", [128, 256, 512])
def test_gemv_w4_groups_and_clip_search(cuda_dev, group):
    g = torch.Generator().manual_seed(group)
    W = (torch.randn(3000, 4096, generator=g) * 0.02).to(BF)
    W[5, :group] = 0  # an all-zero group
    W[7, 3] = 0.5  # an outlier
    Wp, S = quantize_int4(W, group, clip_search=True)
    for B in (1, 2, 4):
        x = torch.randn(B, 4096, generator=g).to(BF)
        check(run(Wp, S, x, group, cuda_dev), Wp, S, x)


def test_gemv_w4_extreme_tokens(cuda_dev):
    """Tokens spanning the fp range (x1000 outlier channels, 1e-30, 1e30, all zero, one nonzero, bf16 subnormals):
    the slicing takes each token's own exponent."""
    g = torch.Generator().manual_seed(8)
    N, K = 2048, 2048
    Wp, S = quantize_int4((torch.randn(N, K, generator=g) * 0.02).to(BF))
    base = torch.randn(6, K, generator=g)
    base[0, ::97] *= 1000
    base[1] *= 1e-30
    base[2] *= 1e30
    base[3] = 0
    base[4] = 0
    base[4, 5] = 3.0
    base[5] = torch.randn(K, generator=g) * 1e-39  # subnormal in bf16
    for b in range(6):
        x = base[b:b + 1].to(BF)
        y = run(Wp, S, x, 128, cuda_dev)
        if b == 3:
            assert (y == 0).all()
            continue
        check(y, Wp, S, x)


def test_gemv_w4_matches_reference_golden(cuda_dev):
    d = golden("gemv_w4")
    for i in range(len([k for k in d.files if k.startswith("name")])):
        Wp, S, x = to_t(d[f"p{i}"]), to_t(d[f"s{i}"]), to_t(d[f"x{i}"], bf16=True)
        y = torch.empty(1, Wp.shape[0], device=cuda_dev, dtype=BF)
        ext().gemv_w4(Wp.to(cuda_dev), S.to(cuda_dev), x.to(cuda_dev), y)  # the reference's binding signature
        torch.cuda.synchronize()
        ref = to_t(d[f"y{i}"]).view(BF)
        assert (y.cpu().float() - ref.float()).abs().max().item() <= 2e-2 * max(ref.float().abs().max().item(), 1.0)
        check(y.cpu(), Wp, S, x)


REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librefk.so"


@pytest.mark.parametrize("N,K", [(3072, 2048), (65536, 2048), (2048, 8192)])
def test_gemv_w4_against_reference_kernel(cuda_dev, N, K):
    """The reference's own INT4 kernel on the same GPU and inputs meets the same bounds; both are timed."""
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    L = ctypes.CDLL(str(REF_LIB))
    if not hasattr(L, "refk_gemv_w4"):
        pytest.skip("oracle/_ref/librefk.so predates the INT4 wrapper")
    L.refk_gemv_w4.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    L.refk_gemv_w4.restype = ctypes.c_int
    g = torch.Generator().manual_seed(N + K)
    Wp, S = quantize_int4((torch.randn(N, K, generator=g) * 0.02).to(BF))
    x = torch.randn(1, K, generator=g).to(BF)
    Wd, Sd, xd = Wp.to(cuda_dev), S.to(cuda_dev), x.to(cuda_dev)
    y = torch.empty(1, N, device=cuda_dev, dtype=BF)
    ry = torch.empty_like(y)
    st = torch.cuda.current_stream().cuda_stream
    assert L.refk_gemv_w4(Wd.data_ptr(), Sd.data_ptr(), xd.data_ptr(), ry.data_ptr(), N, K, 128, st) == 0
    ext().gemv_w4(Wd, Sd, xd, y)
    torch.cuda.synchronize()
    check(y.cpu(), Wp, S, x)
    check(ry.cpu(), Wp, S, x)

    def t(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps
    ours = t(lambda: ext().gemv_w4(Wd, Sd, xd, y))
    ref = t(lambda: L.refk_gemv_w4(Wd.data_ptr(), Sd.data_ptr(), xd.data_ptr(), ry.data_ptr(), N, K, 128, st))
    print(f"\n[vs reference kernel] gemv_w4 {N}x{K}: lfm2q {ours:.1f} us, reference {ref:.1f} us ({ref / ours:.2f}x)")


@pytest.mark.parametrize("B", [1, 2, 3, 4])
def test_gemv_w4_outlier_channels_batched(cuda_dev, B):
    """Outlier channels (x300) in every token of a batch: each token keeps 3 exact slice bytes whatever B, so the
    small elements beside the outliers keep their bits and the result stays within the fp64 rounding bound."""
    g = torch.Generator().manual_seed(70 + B)
    N, K = 3072, 2048
    Wp, S = quantize_int4((torch.randn(N, K, generator=g) * 0.02).to(BF))
    x = torch.randn(B, K, generator=g)
    x[:, :: K // 7] *= 300
    x = x.to(BF)
    check(run(Wp, S, x, 128, cuda_dev), Wp, S, x)
