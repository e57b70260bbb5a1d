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
    if not hasattr(L, "refk_silu_mul"):
        pytest.skip("oracle/_ref/librefk.so predates the producer wrappers: rebuild it (oracle/Makefile, target ref)")
    L.refk_gemm_i8.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]
    L.refk_gemm_w8.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p]
    L.refk_quant_rows.argtypes = [_p, _p, _p, _i, _i, _p]
    L.refk_gemv.argtypes = [_p, _i, _p, _p, _p, _i, _i, _i, _p]
    L.refk_set_pdl.argtypes = [_i]
    L.refk_gemm_i8_q.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]
    L.refk_quant_groups.argtypes = [_p, _p, _p, _i, _i, _p]
    L.refk_add_layernorm_q.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, ctypes.c_float, _i, _p]
    L.refk_add_rmsnorm_q.argtypes = [_p, _p, _p, _p, _p, _i, _i, ctypes.c_float, _i, _p]
    L.refk_silu_mul_q.argtypes = [_p, _p, _p, _i, _i, _i, _p]
    L.refk_silu_mul.argtypes = [_p, _p, _i, _i, _p]
    for f in (L.refk_gemm_i8, L.refk_gemm_w8, L.refk_quant_rows, L.refk_gemv, L.refk_gemm_i8_q, L.refk_quant_groups,
              L.refk_add_layernorm_q, L.refk_add_rmsnorm_q, L.refk_silu_mul_q, L.refk_silu_mul):
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


# ------------------------------------------------------------------ fused producers and the SiLU gate, bit for bit
# The reference's own acceptance test for these is torch.equal (tests/test_int8_gemm.py:123-155); here the equality is
# with the reference's kernels themselves, run on the same GPU on the same inputs.

PRODUCER_ROWS = [(300, 1152), (257, 2048), (1, 1152), (4099, 1152), (64, 768)]


@pytest.mark.parametrize("grouped", [0, 1], ids=["per_row", "grouped"])
@pytest.mark.parametrize("with_y", [True, False], ids=["add", "noadd"])
@pytest.mark.parametrize("rows,D", PRODUCER_ROWS)
def test_add_layernorm_q_equals_reference(cuda_dev, refk, grouped, with_y, rows, D):
    g = torch.Generator().manual_seed(rows + D + grouped)
    h0 = (torch.randn(rows, D, generator=g) + 0.2).to(BF).to(cuda_dev)
    y = torch.randn(rows, D, generator=g).to(BF).to(cuda_dev) if with_y else None
    w = (torch.rand(D, generator=g) + 0.5).to(BF).to(cuda_dev)
    b = torch.randn(D, generator=g).to(BF).to(cuda_dev)
    h, rh = h0.clone(), h0.clone()
    from lfm2opt.int8 import qbuf
    q, s = qbuf(rows, D, 64 if grouped else 0, cuda_dev)
    rq, rs = torch.full_like(q, 99), torch.full_like(s, -1.0)
    int8_ext().add_layernorm_q(h, y, w, b, q, s, 1e-6)
    call(refk.refk_add_layernorm_q(ptr(rh), ptr(y), ptr(w), ptr(b), ptr(rq), ptr(rs), rows, D, 1e-6, grouped,
                                   stream()))
    torch.cuda.synchronize()
    assert torch.equal(h, rh)
    assert torch.equal(q, rq), f"{(q != rq).sum().item()} codes differ"
    assert torch.equal(s, rs), f"{(s != rs).sum().item()} scales differ"


@pytest.mark.parametrize("grouped", [0, 1], ids=["per_row", "grouped"])
@pytest.mark.parametrize("with_y", [True, False], ids=["add", "noadd"])
@pytest.mark.parametrize("rows,H", [(257, 2048), (1, 2048), (1000, 2048), (33, 1024), (5, 8192)])
def test_add_rmsnorm_q_equals_reference(cuda_dev, refk, grouped, with_y, rows, H):
    g = torch.Generator().manual_seed(rows + H + grouped + 7)
    h0 = torch.randn(rows, H, generator=g).to(BF).to(cuda_dev)
    y = torch.randn(rows, H, generator=g).to(BF).to(cuda_dev) if with_y else None
    w = (torch.rand(H, generator=g) + 0.5).to(BF).to(cuda_dev)
    h, rh = h0.clone(), h0.clone()
    from lfm2opt.int8 import qbuf
    q, s = qbuf(rows, H, 64 if grouped else 0, cuda_dev)
    rq, rs = torch.full_like(q, 99), torch.full_like(s, -1.0)
    int8_ext().add_rmsnorm_q(h, y, w, q, s, 1e-5)
    call(refk.refk_add_rmsnorm_q(ptr(rh), ptr(y), ptr(w), ptr(rq), ptr(rs), rows, H, 1e-5, grouped, stream()))
    torch.cuda.synchronize()
    assert torch.equal(h, rh)
    assert torch.equal(q, rq), f"{(q != rq).sum().item()} codes differ"
    assert torch.equal(s, rs), f"{(s != rs).sum().item()} scales differ"


@pytest.mark.parametrize("grouped", [0, 1], ids=["per_row", "grouped"])
@pytest.mark.parametrize("rows,I", [(257, 8192), (1, 8192), (64, 4096)])
def test_silu_mul_q_equals_reference(cuda_dev, refk, grouped, rows, I):
    g = torch.Generator().manual_seed(rows + I + grouped + 3)
    gg = (torch.randn(rows, 2 * I, generator=g) * 2).to(BF).to(cuda_dev)
    from lfm2opt.int8 import qbuf
    q, s = qbuf(rows, I, 64 if grouped else 0, cuda_dev)
    rq, rs = torch.full_like(q, 99), torch.full_like(s, -1.0)
    int8_ext().silu_mul_q(gg, q, s)
    call(refk.refk_silu_mul_q(ptr(gg), ptr(rq), ptr(rs), rows, I, grouped, stream()))
    # the reference's unfused chain: its silu_mul kernel (bf16 out), then the oracle's quantizer
    a = torch.empty(rows, I, device=cuda_dev, dtype=BF)
    call(refk.refk_silu_mul(ptr(gg), ptr(a), rows, I, stream()))
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(s, rs)
    uq, us = (oracle.quant_groups_ref if grouped else oracle.quant_rows_ref)(a.cpu())
    assert torch.equal(q.cpu(), uq) and torch.equal(s.cpu(), us)


@pytest.mark.parametrize("M,K,N,bias,gelu", [(300, 1152, 4352, True, True), (1024, 2048, 2048, False, False),
                                             (77, 4352, 1152, True, False)])
def test_gemm_i8_q_equals_reference(cuda_dev, refk, M, K, N, bias, gelu):
    x, wq, sw, b = inputs(M, K, N, bias, M + 2 * K + N, cuda_dev)
    xq, sxT = quantize_rows(x, 64)
    q = torch.empty(M, N, device=cuda_dev, dtype=torch.int8)
    s = torch.empty(N // 64, M, device=cuda_dev)
    rq, rs = torch.full_like(q, 99), torch.full_like(s, -1.0)
    int8_ext().gemm_i8_q(xq, sxT, wq, sw, b, q, s, gelu)
    call(refk.refk_gemm_i8_q(ptr(xq), ptr(sxT), ptr(wq), ptr(sw), ptr(b), ptr(rq), ptr(rs), M, N, K, int(gelu),
                             stream()))
    torch.cuda.synchronize()
    if gelu:  # the two sides evaluate tanh differently: codes within one, scales within 2^-7 relative
        assert (q.int() - rq.int()).abs().max().item() <= 1
        assert ((s - rs).abs() <= rs.abs() * 2 ** -7).all()
    else:
        assert torch.equal(q, rq) and torch.equal(s, rs)


@pytest.mark.parametrize("M,K,I,gate_bias", [(300, 2048, 8192, None), (1024, 1152, 2048, None),
                                             (256, 2048, 1024, -88.0), (130, 2048, 512, -87.5)])
def test_silu_gate_equals_reference_composition(cuda_dev, refk, M, K, I, gate_bias):
    """gemm_i8_silu equals the reference's gemm_i8 (bf16 [M, 2I]) followed by its silu_mul, bit for bit. With a gate
    bias near -88 the gate values land in [-89, -87], where 1 + exp(-g) passes 2^126: the IEEE quotient the reference
    takes is still a normal float there (a fast reciprocal-based division would return 0)."""
    x, wq, sw, _ = inputs(M, K, 2 * I, False, M + K + I, cuda_dev)
    b = None
    if gate_bias is not None:
        b = torch.zeros(2 * I, dtype=BF)
        b[:I] = gate_bias
        b[I:] = 1.0
        b = b.to(cuda_dev)
        sw = sw * 0.05  # gate = bias + a small product: every gate value lies within one unit of the bias
    xq, sx = quantize_rows(x)
    y = torch.empty(M, I, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8_silu(xq, sx, wq, sw, b, y)
    gu = torch.empty(M, 2 * I, device=cuda_dev, dtype=BF)
    call(refk.refk_gemm_i8(ptr(xq), ptr(sx), ptr(wq), ptr(sw), ptr(b), ptr(gu), M, 2 * I, K, 0, 0, stream()))
    ry = torch.empty_like(y)
    call(refk.refk_silu_mul(ptr(gu), ptr(ry), M, I, stream()))
    torch.cuda.synchronize()
    if gate_bias is not None:
        gate = gu[:, :I].float()
        assert gate.min().item() >= -89.0 and gate.max().item() <= -87.0
        assert (ry != 0).float().mean().item() > 0.5  # the reference's values there are not flushed to zero
    assert torch.equal(y, ry), f"{(y != ry).sum().item()} of {y.numel()} outputs differ"


def test_silu_gate_every_gate_value_equals_reference(cuda_dev, refk):
    """With all-zero activations every gate of the fused SiLU epilogue equals its bias, so the bias can enumerate gate
    values: every bf16 value with 2^-8 <= |g| < 2^8 (both signs, 16 binades x 128 mantissas), zero, subnormals, tiny
    and large values, the region around -88 where 1 + exp(-g) passes 2^126, and random bf16 values. The result must
    equal the reference's gemm_i8 -> silu_mul composition bit for bit. The up half is 1, so y = bf16(silu(g))."""
    table = [((s << 15) | (e << 7) | m) for s in (0, 1) for e in range(119, 135) for m in range(128)]
    extra = [0x0000, 0x8000, 0x0001, 0x8001, 0x0080, 0x3B00, 0xBB00, 0x3BFF, 0xBBFF, 0x4380, 0xC380, 0x43FF, 0xC3FF,
             0x4700, 0xC2B0, 0xC2B1, 0xC2AF, 0xC2B2, 0xC2C0, 0x7F7F, 0xFF7F]
    g = torch.Generator().manual_seed(13)
    rand = torch.randint(0, 0x7F80, (8192 - len(table) - len(extra),), generator=g)
    rand = rand | (torch.randint(0, 2, rand.shape, generator=g) << 15)
    bits = torch.tensor(table + extra, dtype=torch.int32)
    bits = torch.cat([bits, rand.to(torch.int32)])
    I, K, M = bits.numel(), 64, 3
    gate_bias = bits.to(torch.int16).view(BF)
    b = torch.cat([gate_bias, torch.ones(I, dtype=BF)]).to(cuda_dev)
    x = torch.zeros(M, K, dtype=BF, device=cuda_dev)
    w = (torch.randn(2 * I, K, generator=g) * 0.02).to(BF)
    wq, sw = quantize_int8(w)
    wq, sw = wq.to(cuda_dev), sw.to(cuda_dev)
    xq, sx = quantize_rows(x)
    y = torch.empty(M, I, device=cuda_dev, dtype=BF)
    int8_ext().gemm_i8_silu(xq, sx, wq, sw, b, y)
    gu = torch.empty(M, 2 * I, device=cuda_dev, dtype=BF)
    call(refk.refk_gemm_i8(ptr(xq), ptr(sx), ptr(wq), ptr(sw), ptr(b), ptr(gu), M, 2 * I, K, 0, 0, stream()))
    ry = torch.empty_like(y)
    call(refk.refk_silu_mul(ptr(gu), ptr(ry), M, I, stream()))
    torch.cuda.synchronize()
    assert torch.equal(gu[:, :I].cpu(), gate_bias.expand(M, I)), "gates are the biases"
    bad = (y != ry).any(0).nonzero().flatten()
    assert bad.numel() == 0, [hex(int(bits[i]) & 0xFFFF) for i in bad[:10]]


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
