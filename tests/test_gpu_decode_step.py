"""A whole LFM2 decode step (lfm2opt.decode_step.DecodeStep, batch 1) on the B200.

  - replayed from a CUDA graph it produces the same bits as eager steps;
  - with lfm2q's int8 GEMVs (gemv, gemv_epi) swapped into a step built from the reference's own kernels
    (oracle/_ref/librefk.so: its add_rmsnorm, qk_norm_rope_kv, decode_attention_split), the two steps are
    bit-identical;
  - the step built entirely from the reference's kernels (its GEMVs too) on the same weights and forced tokens gives
    logits, residual stream, cache rows and conv states within max |err| <= 5e-2 and mean |err| <= 1e-2 of the
    largest magnitude: the GEMVs differ only in fp32 summation order (at most a bf16 ulp per output), and those
    differences go through 16 layers of bf16 norms and residual adds over several positions;
  - both are timed as graph replays at 1001 cached positions (printed).
"""

import ctypes
from pathlib import Path

import pytest
import torch

from lfm2opt.decode_step import DecodeStep, Lfm2Config, Lfm2Weights

pytestmark = pytest.mark.gpu
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librefk.so"


class RefOps:
    """The reference extension's op names over its own kernels (test infrastructure)."""

    def __init__(self):
        L = ctypes.CDLL(str(REF_LIB))
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.refk_gemv.argtypes = [P, I, P, P, P, I, I, I, P]
        L.refk_gemv_epi.argtypes = [I, P, I, P, P, P, I, I, P, P, P, P]
        L.refk_add_rmsnorm.argtypes = [P, P, P, P, I, I, F, P]
        L.refk_qk_norm_rope_kv.argtypes = [P, P, P, P, F, P, P, P, P, I, I, I, I, F, P]
        L.refk_decode_attention_split.argtypes = [P] * 6 + [I] * 5 + [F, P]
        self.L = L

    @staticmethod
    def _st():
        return torch.cuda.current_stream().cuda_stream

    def gemv(self, W, s, x, y):
        assert self.L.refk_gemv(W.data_ptr(), 1, s.data_ptr(), x.data_ptr(), y.data_ptr(), W.shape[0], W.shape[1], 1,
                                self._st()) == 0

    def gemv_epi(self, epi, W, s, x, y, state=None, cw=None, cbias=None):
        S = W.shape[0] // (2 if epi == 0 else 3)
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        assert self.L.refk_gemv_epi(epi, W.data_ptr(), 1, s.data_ptr(), x.data_ptr(), y.data_ptr(), S, W.shape[1],
                                    p(state), p(cw), p(cbias), self._st()) == 0

    def add_rmsnorm(self, h, y, w, x, eps):
        H = h.shape[-1]
        assert self.L.refk_add_rmsnorm(h.data_ptr(), None if y is None else y.data_ptr(), w.data_ptr(), x.data_ptr(),
                                       h.numel() // H, H, eps, self._st()) == 0

    def qk_norm_rope_kv(self, qkv, qw, kw, inv_freq, scaling, pos, q, kc, vc, eps):
        assert self.L.refk_qk_norm_rope_kv(qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), inv_freq.data_ptr(), scaling,
                                           pos.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), qkv.shape[0],
                                           q.shape[1], kc.shape[1], kc.shape[2], eps, self._st()) == 0

    def decode_attention_split(self, q, kc, vc, pos, out, ws, scale):
        assert self.L.refk_decode_attention_split(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                                                  out.data_ptr(), ws.data_ptr(), q.shape[0], q.shape[1], kc.shape[1],
                                                  kc.shape[2], ws.shape[2], scale, self._st()) == 0


@pytest.fixture(scope="module")
def weights(cuda_dev):
    return Lfm2Weights(Lfm2Config(), cuda_dev, seed=5)


def close_stack(a, b, what):
    """After 16 layers: the GEMVs' last-bit differences (the only difference, see the test above) go through bf16
    norms and residual adds at every layer, so the bar is max |err| <= 5e-2 and mean |err| <= 1e-2 of the largest
    magnitude."""
    ref = b.float()
    err = (a.float() - ref).abs()
    m = max(ref.abs().max().item(), 1.0)
    print(f"  {what}: max |err| / max |ref| = {err.max().item() / m:.4f}, mean = {err.mean().item() / m:.5f}")
    return err.max().item() <= 5e-2 * m and err.mean().item() <= 1e-2 * m


def test_graph_replay_equals_eager_steps(cuda_dev, weights):
    eager = DecodeStep(weights, max_len=512)
    for _ in range(3):
        eager.step()
    g = DecodeStep(weights, max_len=512).capture()  # warm-up step = step 1
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(g.logits, eager.logits) and torch.equal(g.h, eager.h)
    assert int(g.pos) == int(eager.pos) == 3
    assert all(torch.equal(g.kc[i], eager.kc[i]) for i in eager.kc)
    assert all(torch.equal(g.conv[i], eager.conv[i]) for i in eager.conv)


class HybridOps(RefOps):
    """The reference's kernels for everything but the int8 GEMVs (gemv and the fused gemv_epi), which are lfm2q's."""

    def gemv(self, W, s, x, y):
        from lfm2opt.kernels import ext
        ext().gemv(W, s, x, y)

    def gemv_epi(self, epi, W, s, x, y, state=None, cw=None, cbias=None):
        from lfm2opt.kernels import ext
        ext().gemv_epi(epi, W, s, x, y, state, cw, cbias)


def test_step_equals_reference_kernels_given_the_same_gemv(cuda_dev, weights):
    """With the GEMVs in common, the step on lfm2q's kernels and the step on the reference's are bit-identical: every
    other kernel (norms, q/k norm + RoPE + cache write, split attention) gives the reference's bits in context, under
    programmatic dependent launch."""
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    ours, hyb = DecodeStep(weights, max_len=512), DecodeStep(weights, max_len=512, ops=HybridOps())
    for t in (3, 9000, 17):
        for s in (ours, hyb):
            s.tok.fill_(t)
            s.step()
        torch.cuda.synchronize()
        assert torch.equal(ours.logits, hyb.logits) and torch.equal(ours.h, hyb.h), t
    assert all(torch.equal(ours.kc[i], hyb.kc[i]) and torch.equal(ours.vc[i], hyb.vc[i]) for i in ours.kc)
    assert all(torch.equal(ours.conv[i], hyb.conv[i]) for i in ours.conv)


def test_step_matches_the_reference_kernels(cuda_dev, weights):
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    ours, ref = DecodeStep(weights, max_len=512), DecodeStep(weights, max_len=512, ops=RefOps())
    for t in (1, 70, 4000, 65535, 12):  # forced tokens: both see the same inputs whatever their argmax
        for s in (ours, ref):
            s.tok.fill_(t)
            s.step()
        torch.cuda.synchronize()
        assert close_stack(ours.logits, ref.logits, f"logits (token {t})"), t
        assert close_stack(ours.h, ref.h, f"residual (token {t})"), t
    for i in ours.kc:
        assert close_stack(ours.kc[i][:, :, :5], ref.kc[i][:, :, :5], f"k cache {i}")
        assert close_stack(ours.vc[i][:, :, :5], ref.vc[i][:, :, :5], f"v cache {i}")
    for i in ours.conv:
        assert close_stack(ours.conv[i], ref.conv[i], f"conv state {i}")


def test_decode_step_time_vs_reference_kernels(cuda_dev, weights):
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    out = {}
    for name, ops in (("lfm2q", None), ("reference kernels", RefOps())):
        s = DecodeStep(weights, max_len=1024, ops=ops)
        s.pos.fill_(999)
        s.capture()
        for _ in range(3):
            s.replay()
        torch.cuda.synchronize()
        s.pos.fill_(1000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 20
        e0.record()
        for _ in range(n):
            s.replay()
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) * 1e3 / n
        del s
    print(f"\n[decode step, B=1, ~1010 cached positions] lfm2q {out['lfm2q']:.1f} us/token, reference kernels "
          f"{out['reference kernels']:.1f} us/token ({out['reference kernels'] / out['lfm2q']:.2f}x)")
