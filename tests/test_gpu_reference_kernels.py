"""lfm2q against the reference's own CUDA kernels, on the same B200 and the same device buffers.

The reference's kernels/int8_gemm.cu and kernels/lfm2_decode.cu are compiled for sm_100a from its source tree into
oracle/_ref/librefk.so (oracle/Makefile, target `ref`; built by __graft_entry__.build() where the source tree is
present) and called through a small C shim. Parity: the W8A8 paths are exact at int32 with the same fp32 epilogue
order on both sides, so the bf16 outputs must match bit for bit (GELU: within 1 ulp, the two sides evaluate tanh
differently); the quantizer must match code for code; the weight-only GEMV accumulates in fp32 in different orders,
so it is held to the reference's own tolerance. Speed: both sides timed with CUDA events on the same stream over
back-to-back launches (weights resident), printed per shape; lfm2q must not be slower.
"""

import ctypes
from pathlib import Path

import pytest
import torch

import oracle
from lfm2opt.int8 import quantize_rows
from lfm2opt.kernels import ext, int8_ext
from lfm2opt.quant import quantize_int8
from test_gpu_gemm import assert_close_bf16

pytestmark = pytest.mark.gpu

BF = torch.bfloat16
LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librefk.so"
_p, _i = ctypes.c_void_p, ctypes.c_int


@pytest.fixture(scope="module")
def refk(cuda_dev):
    if not LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built (the reference's source tree was absent at build time)")
    L = ctypes.CDLL(str(LIB))
    L.refk_gemm_i8.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]
    L.refk_gemm_w8.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p]
    L.refk_quant_rows.argtypes = [_p, _p, _p, _i, _i, _p]
    L.refk_gemv.argtypes = [_p, _i, _p, _p, _p, _i, _i, _i, _p]
    L.refk_set_pdl.argtypes = [_i]
    for f in (L.refk_gemm_i8, L.refk_gemm_w8, L.refk_quant_rows, L.refk_gemv):
        f.restype = _i
    L.refk_set_pdl.restype = None
    return L


def stream():
    return torch.cuda.current_stream().cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def call(status):
    assert status == 0, f"reference kernel launch failed: CUDA error {status}"


def inputs(M, K, N, bias, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(BF)
    w = (torch.randn(N, K, generator=g) * 0.02).to(BF)
    wq, sw = quantize_int8(w)
    b = (torch.randn(N, generator=g) * 0.1).to(BF).to(dev) if bias else None
    return x.to(dev), wq.to(dev), sw.to(dev), b


@pytest.mark.parametrize("rows,K", [(1, 1152), (300, 1152), (4097, 2048), (64, 2048)])
def test_quant_rows_matches_reference(cuda_dev, refk, rows, K):
    x = (torch.randn(rows, K, generator=torch.Generator().manual_seed(rows + K)) * 3).to(BF).to(cuda_dev)
    q, s = quantize_rows(x)
    rq = torch.empty_like(q)
    rs = torch.empty_like(s)
    call(refk.refk_quant_rows(ptr(x), ptr(rq), ptr(rs), rows, K, stream()))
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(s, rs)


GEMM_CASES = [(300, 1152, 1152, True, False), (2327, 2048, 3072, False, False), (4096, 2048, 2048, False, False),
              (16, 2048, 8192, False, False), (48, 2048, 6144, True, False), (1024, 1152, 4304, True, True),
              (9216, 4304, 1152, True, False), (517, 8192, 2048, False, False)]


@pytest.mark.parametrize("M,K,N,bias,gelu", GEMM_CASES)
@pytest.mark.parametrize("grouped", [False, True], ids=["per_token", "grouped"])
def test_gemm_i8_matches_reference(cuda_dev, refk, M, K, N, bias, gelu, grouped):
    if grouped and K % 128:
        pytest.skip("grouped scales need K % 128 == 0 in the reference")
    x, wq, sw, b = inputs(M, K, N, bias, M + K + N, cuda_dev)
    xq, sx = quantize_rows(x, 64 if grouped else 0)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    ry = torch.empty_like(y)
    int8_ext().gemm_i8(xq, sx, wq, sw, b, y, gelu)
    call(refk.refk_gemm_i8(ptr(xq), ptr(sx), ptr(wq), ptr(sw), ptr(b), ptr(ry), M, N, K, int(gelu), int(grouped),
                           stream()))
    torch.cuda.synchronize()
    assert_close_bf16(y.cpu(), ry.cpu(), gelu)


@pytest.mark.parametrize("M,K,N,bias,gelu", [(300, 1152, 1152, True, False), (2327, 2048, 3072, False, False),
                                             (1024, 1152, 4304, True, True)])
def test_gemm_w8_matches_reference(cuda_dev, refk, M, K, N, bias, gelu):
    """W8A16 accumulates bf16 x bf16 products in fp32 on both sides, in different orders: both within 1.05x of the
    bf16 rounding error of the fp64 product, and within a few bf16 ulps of each other."""
    x, wq, sw, b = inputs(M, K, N, bias, 3 * M + K, cuda_dev)
    y = torch.empty(M, N, device=cuda_dev, dtype=BF)
    ry = torch.empty_like(y)
    int8_ext().gemm_w8(x, wq, sw, b, y, gelu)
    call(refk.refk_gemm_w8(ptr(x), ptr(wq), ptr(sw), ptr(b), ptr(ry), M, N, K, int(gelu), stream()))
    torch.cuda.synchronize()
    r64 = oracle.gemm_w8_f64(x.cpu(), wq.cpu(), sw.cpu(), None if b is None else b.cpu(), gelu)
    e_round = ((r64.to(BF).double() - r64).norm() / r64.norm()).item()
    for out in (y, ry):
        e = ((out.cpu().double() - r64).norm() / r64.norm()).item()
        assert e <= 1.05 * e_round + 1e-6, (e, e_round)


@pytest.mark.parametrize("N,K,B", [(3072, 2048, 1), (65536, 2048, 1), (16384, 2048, 4), (2048, 8192, 8),
                                   (6144, 2048, 16)])
def test_gemv_matches_reference(cuda_dev, refk, N, K, B):
    g = torch.Generator().manual_seed(N + K + B)
    W = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(cuda_dev)
    s = (torch.rand(N, generator=g) * 1e-3 + 1e-4).to(cuda_dev)
    x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
    y = torch.empty(B, N, device=cuda_dev, dtype=BF)
    ry = torch.empty_like(y)
    ext().gemv(W, s, x, y)
    call(refk.refk_gemv(ptr(W), 1, ptr(s), ptr(x), ptr(ry), N, K, B, stream()))
    torch.cuda.synchronize()
    ref = oracle.gemv_ref(W.cpu(), s.cpu(), x.cpu())
    tol = 2e-2 * max(ref.float().abs().max().item(), 1.0)  # the reference's own bound (tests/test_kernels.py:32)
    for out in (y, ry):
        assert (out.cpu().float() - ref.float()).abs().max().item() <= tol


def _time(fn, reps=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3  # us


SPEED_CASES = [("gemm_i8", 16384, 2048, 6144), ("gemm_i8", 16384, 1152, 3456), ("gemm_i8", 16384, 8192, 2048),
               ("gemm_i8 grouped", 16384, 2048, 2048), ("gemm_w8", 16384, 2048, 6144), ("quant_rows", 65536, 2048, 0),
               ("gemv B=1", 1, 2048, 65536)]


@pytest.mark.parametrize("op,M,K,N", SPEED_CASES, ids=[f"{c[0]}-{c[1]}x{c[2]}x{c[3]}" for c in SPEED_CASES])
def test_not_slower_than_reference(cuda_dev, refk, op, M, K, N):
    dev = cuda_dev
    if op == "quant_rows":
        x = torch.randn(M, K, device=dev).to(BF)
        q, s = torch.empty(M, K, device=dev, dtype=torch.int8), torch.empty(M, device=dev)
        ours = _time(lambda: int8_ext().quant_rows(x, q, s))
        ref = _time(lambda: call(refk.refk_quant_rows(ptr(x), ptr(q), ptr(s), M, K, stream())))
        work, unit = 3 * M * K / 1e3, "GB/s"
    elif op.startswith("gemv"):
        W = torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8)
        s = torch.rand(N, device=dev) * 1e-3
        x = torch.randn(M, K, device=dev).to(BF)
        y = torch.empty(M, N, device=dev, dtype=BF)
        ours = _time(lambda: ext().gemv(W, s, x, y))
        ref = _time(lambda: call(refk.refk_gemv(ptr(W), 1, ptr(s), ptr(x), ptr(y), N, K, M, stream())))
        work, unit = N * K / 1e3, "GB/s"
    else:
        x, wq, sw, b = inputs(M, K, N, False, 11, dev)
        y = torch.empty(M, N, device=dev, dtype=BF)
        if op == "gemm_w8":
            ours = _time(lambda: int8_ext().gemm_w8(x, wq, sw, None, y, False))
            ref = _time(lambda: call(refk.refk_gemm_w8(ptr(x), ptr(wq), ptr(sw), None, ptr(y), M, N, K, 0, stream())))
        else:
            grouped = op.endswith("grouped")
            xq, sx = quantize_rows(x, 64 if grouped else 0)
            ours = _time(lambda: int8_ext().gemm_i8(xq, sx, wq, sw, None, y, False))
            ref = _time(lambda: call(refk.refk_gemm_i8(ptr(xq), ptr(sx), ptr(wq), ptr(sw), None, ptr(y), M, N, K, 0,
                                                       int(grouped), stream())))
        work, unit = 2 * M * N * K / 1e6, "TOPS"
    print(f"\n[vs reference kernel] {op} {M}x{K}x{N}: lfm2q {ours:.1f} us ({work / ours:.0f} {unit}), "
          f"reference {ref:.1f} us ({work / ref:.0f} {unit}), speed-up {ref / ours:.2f}x")
    assert ours <= ref * 1.02, (ours, ref)
