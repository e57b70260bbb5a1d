"""The decode step's small kernels (lfm2q_add_rmsnorm, lfm2q_shortconv_step, lfm2q_qk_norm_rope_kv) on the B200.

  - against the CPU oracle (the reference's own test expressions, tests/test_kernels.py:26-90), with the reference
    test's bar: max |err| <= 2e-2 * max(|ref|, 1) (the kernels sum squares in fp32 in another order than torch's
    CPU mean, and a 1-ulp change of a normalised value can move the bf16 products after it);
  - against the reference's own kernels on the same device buffers (oracle/_ref/librefk.so): bit for bit, outputs
    and every in-place update (h, the conv state, the cache rows);
  - at the reference test's shapes (H 2048, 32 q / 8 KV heads, B = 2, max_len 512, pos 137) and at ragged ones.
"""

import ctypes
from pathlib import Path

import pytest
import torch

from lfm2opt.kernels import ext
from oracle.decode import add_rmsnorm_ref, qk_norm_rope_kv_ref, shortconv_step_ref

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
EPS = 1e-5
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librefk.so"


def refk():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    L = ctypes.CDLL(str(REF_LIB))
    if not hasattr(L, "refk_qk_norm_rope_kv"):
        pytest.skip("oracle/_ref/librefk.so predates the decode-step wrappers")
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.refk_add_rmsnorm.argtypes = [P, P, P, P, I, I, F, P]
    L.refk_shortconv_step.argtypes = [P, P, P, P, P, I, I, P]
    L.refk_qk_norm_rope_kv.argtypes = [P, P, P, P, F, P, P, P, P, I, I, I, I, F, P]
    return L


def st():
    return torch.cuda.current_stream().cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def close(out, ref):
    """tests/test_kernels.py:32-36: max |err| <= 2e-2 * max(|ref|, 1)."""
    err = (out.cpu().float() - ref.float()).abs().max().item()
    return err <= 2e-2 * max(ref.float().abs().max().item(), 1.0)


def gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("rows,H", [(2, 2048), (1, 2048), (3, 1000), (5, 8192), (1, 64)])
@pytest.mark.parametrize("add", [True, False])
def test_add_rmsnorm(cuda_dev, rows, H, add):
    g = gen(rows * 7 + H)
    h = torch.randn(rows, H, generator=g).to(BF)
    y = torch.randn(rows, H, generator=g).to(BF) if add else None
    w = (torch.rand(H, generator=g) + 0.5).to(BF)
    hd, yd, wd = h.to(cuda_dev), (y.to(cuda_dev) if add else None), w.to(cuda_dev)
    x = torch.empty(rows, H, device=cuda_dev, dtype=BF)
    hk = hd.clone()
    ext().add_rmsnorm(hk, yd, wd, x, EPS)
    rh, rx = add_rmsnorm_ref(h, y, w, EPS)
    torch.cuda.synchronize()
    assert torch.equal(hk.cpu(), rh)
    assert close(x, rx)
    L = refk()
    hr, xr = hd.clone(), torch.empty_like(x)
    assert L.refk_add_rmsnorm(ptr(hr), ptr(yd), ptr(wd), ptr(xr), rows, H, EPS, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(hk, hr) and torch.equal(x, xr)


@pytest.mark.parametrize("B,H", [(2, 2048), (1, 2048), (3, 1000), (4, 300)])
@pytest.mark.parametrize("bias", [False, True])
def test_shortconv_step(cuda_dev, B, H, bias):
    g = gen(B * 13 + H)
    bcx = torch.randn(B, 3 * H, generator=g).to(BF)
    state = torch.randn(B, H, 3, generator=g).to(BF)
    w = (torch.randn(H, 3, generator=g) * 0.5).to(BF)
    bb = (torch.randn(H, generator=g) * 0.1).to(BF) if bias else None
    d = [t.to(cuda_dev) if t is not None else None for t in (bcx, state, w, bb)]
    sk, yk = d[1].clone(), torch.empty(B, H, device=cuda_dev, dtype=BF)
    ext().shortconv_step(d[0], sk, d[2], d[3], yk)
    ry, rs = shortconv_step_ref(bcx, state, w, bb)
    torch.cuda.synchronize()
    assert torch.equal(sk.cpu(), rs)
    assert close(yk, ry)
    L = refk()
    sr, yr = d[1].clone(), torch.empty_like(yk)
    assert L.refk_shortconv_step(ptr(d[0]), ptr(sr), ptr(d[2]), ptr(d[3]), ptr(yr), B, H, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(sk, sr) and torch.equal(yk, yr)


@pytest.mark.parametrize("B,NQ,NKV,max_len,pos,scaling", [(2, 32, 8, 512, 137, 1.0), (1, 32, 8, 4096, 4000, 1.0),
                                                          (3, 8, 2, 64, 0, 1.0), (2, 32, 8, 512, 511, 0.7)])
def test_qk_norm_rope_kv(cuda_dev, B, NQ, NKV, max_len, pos, scaling):
    g = gen(B + NQ + pos)
    qkv = torch.randn(B, (NQ + 2 * NKV) * 64, generator=g).to(BF)
    qw, kw = (torch.rand(64, generator=g) + 0.5).to(BF), (torch.rand(64, generator=g) + 0.5).to(BF)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float) / 64))
    d = [t.to(cuda_dev) for t in (qkv, qw, kw, inv_freq)]
    p = torch.tensor([pos], device=cuda_dev)
    kc = torch.zeros(B, NKV, max_len, 64, device=cuda_dev, dtype=BF)
    vc = torch.zeros_like(kc)
    qo = torch.empty(B, NQ, 64, device=cuda_dev, dtype=BF)
    ext().qk_norm_rope_kv(d[0], d[1], d[2], d[3], scaling, p, qo, kc, vc, EPS)
    rq, rk, rv = qk_norm_rope_kv_ref(qkv, qw, kw, inv_freq, scaling, pos, NQ, NKV, EPS)
    torch.cuda.synchronize()
    assert close(qo, rq)
    assert close(kc[:, :, pos], rk)
    assert torch.equal(vc[:, :, pos].cpu(), rv)
    untouched = torch.ones(max_len, dtype=torch.bool)
    untouched[pos] = False
    assert not kc[:, :, untouched].any() and not vc[:, :, untouched].any()
    L = refk()
    kr, vr, qr = torch.zeros_like(kc), torch.zeros_like(vc), torch.empty_like(qo)
    assert L.refk_qk_norm_rope_kv(ptr(d[0]), ptr(d[1]), ptr(d[2]), ptr(d[3]), scaling, ptr(p), ptr(qr), ptr(kr),
                                  ptr(vr), B, NQ, NKV, max_len, EPS, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(qo, qr) and torch.equal(kc, kr) and torch.equal(vc, vr)


@pytest.mark.parametrize("B,V", [(1, 65536), (3, 65536), (1, 1001), (2, 8), (4, 4096)])
def test_argmax_next_equals_torch_argmax(cuda_dev, B, V):
    g = gen(B * 7 + V)
    logits = torch.randn(B, V, generator=g).to(BF)
    logits[0, V // 3] = 50.0  # ties: the first index wins
    logits[0, V // 2] = 50.0
    if B > 1:
        logits[1, V - 1] = float("nan")  # NaN counts as the largest, as in torch.argmax
        logits[1, 0] = float("nan")
    ld = logits.to(cuda_dev)
    tok = torch.full((B,), -1, device=cuda_dev, dtype=torch.int64)
    pos = torch.tensor([41], device=cuda_dev)
    ext().argmax_next(ld, tok, pos)
    torch.cuda.synchronize()
    assert torch.equal(tok.cpu(), torch.argmax(logits.float(), dim=-1))
    assert int(pos) == 42
    ext().argmax_next(ld, tok)  # no position to advance
    torch.cuda.synchronize()
    assert int(pos) == 42


@pytest.mark.parametrize("rows,H", [(1, 2048), (3, 2048), (2, 1000)])
def test_embed_rmsnorm_equals_embedding_then_add_rmsnorm(cuda_dev, rows, H):
    g = gen(rows + H)
    embed = torch.randn(300, H, generator=g).to(BF).to(cuda_dev)
    w = (torch.rand(H, generator=g) + 0.5).to(BF).to(cuda_dev)
    tok = torch.tensor([5, 299, 0][:rows], device=cuda_dev)
    h, x = torch.empty(rows, H, device=cuda_dev, dtype=BF), torch.empty(rows, H, device=cuda_dev, dtype=BF)
    ext().embed_rmsnorm(tok, embed, w, h, x, EPS)
    h_ref = embed[tok].clone()
    x_ref = torch.empty_like(x)
    L = refk()
    assert L.refk_add_rmsnorm(ptr(h_ref), None, ptr(w), ptr(x_ref), rows, H, EPS, st()) == 0
    torch.cuda.synchronize()
    assert torch.equal(h, embed[tok]) and torch.equal(x, x_ref)
