"""Split-over-positions decode attention (lfm2q_decode_attention_split) on the B200.

The kernel keeps the reference kernel's per-position arithmetic (kernels/lfm2_decode.cu:284-416) with another memory
schedule (a producer warp stages K and V rows in shared memory by bulk copies). So:
  - out meets the fp64 oracle within bf16 rounding plus fp32 / fast-exponential slack, on the reference test's cases
    (B = 2, max_len 3072, pos 2300, S = 16 and 4, and length 1; tests/test_kernels.py:94-115) and on ragged ones;
  - the partials in ws meet the oracle's per-split (m, l, acc);
  - out and ws equal the reference kernel's, bit for bit, on the same device buffers (oracle/_ref/librefk.so);
  - repeated calls and a CUDA-graph replay give the same bits.
"""

import ctypes
from pathlib import Path

import pytest
import torch

from lfm2opt.kernels import check_device, ext
from oracle.attention import decode_attention_f64, split_partials_f64

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librefk.so"

# (B, NKV, max_len, pos, S)
CASES = [(2, 8, 3072, 2300, 16), (2, 8, 3072, 2300, 4), (2, 8, 3072, 0, 16), (1, 2, 300, 299, 3),
         (3, 1, 129, 128, 2), (1, 8, 8192, 8191, 32), (4, 8, 1024, 63, 8), (1, 1, 64, 10, 64), (2, 4, 200, 130, 1),
         (1, 2, 256, 200, 80)]  # the last: more splits than the combine stages at once


def make(B, NKV, max_len, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, 4 * NKV, 64, generator=g).to(BF)
    kc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF)
    vc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF)
    return q, kc, vc, q.to(dev), kc.to(dev), vc.to(dev)


def run(qd, kcd, vcd, pos, S, scale):
    B, NQ = qd.shape[:2]
    out = torch.full_like(qd, float("nan"))
    ws = torch.full((B, NQ, S, 66), float("nan"), device=qd.device)
    ext().decode_attention_split(qd, kcd, vcd, torch.tensor([pos], device=qd.device), out, ws, scale)
    torch.cuda.synchronize()
    return out, ws


def check_out(out, ref64):
    """bf16 rounding (half an ulp, 2^-9 relative) plus 1e-3 of the row's largest value for the fp32 sums and the fast
    exponential."""
    r = ref64.float()
    tol = r.abs() * 2.0 ** -8 + 1e-3 * r.abs().amax(dim=-1, keepdim=True) + 1e-6
    assert ((out.cpu().float() - r).abs() <= tol).all(), (out.cpu().float() - r).abs().max().item()


@pytest.mark.parametrize("B,NKV,max_len,pos,S", CASES)
def test_decode_attention_split_vs_oracle(cuda_dev, B, NKV, max_len, pos, S):
    q, kc, vc, qd, kcd, vcd = make(B, NKV, max_len, pos + S, cuda_dev)
    scale = 64 ** -0.5
    out, ws = run(qd, kcd, vcd, pos, S, scale)
    check_device()
    check_out(out, decode_attention_f64(q, kc, vc, pos, scale))
    w64 = split_partials_f64(q, kc, vc, pos, scale, S)
    w = ws.cpu().double()
    live = w64[..., 1] > 0
    assert torch.equal(live, w[..., 1] > 0)
    assert torch.isinf(w[..., 0][~live]).all() and (w[..., 0][~live] < 0).all()
    assert (w[..., 0][live] - w64[..., 0][live]).abs().max().item() < 1e-4
    assert ((w[..., 1][live] - w64[..., 1][live]).abs() <= 1e-4 * w64[..., 1][live] + 1e-5).all()
    acc, acc64 = w[..., 2:][live], w64[..., 2:][live]
    assert ((acc - acc64).abs() <= 1e-4 * acc64.abs().amax(dim=-1, keepdim=True) + 1e-5).all()


def test_positions_past_the_cache_are_not_read(cuda_dev):
    """pos >= max_len attends the whole cache (the reference reads past it; this build clamps)."""
    q, kc, vc, qd, kcd, vcd = make(1, 2, 256, 5, cuda_dev)
    out, _ = run(qd, kcd, vcd, 1000, 4, 0.125)
    check_out(out, decode_attention_f64(q, kc, vc, 255, 0.125))


def _refk():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/librefk.so not built")
    L = ctypes.CDLL(str(REF_LIB))
    if not hasattr(L, "refk_decode_attention_split"):
        pytest.skip("oracle/_ref/librefk.so predates the attention wrapper")
    f = L.refk_decode_attention_split
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


@pytest.mark.parametrize("B,NKV,max_len,pos,S", [c for c in CASES])
def test_decode_attention_split_equals_reference_kernel(cuda_dev, B, NKV, max_len, pos, S):
    f = _refk()
    _, _, _, qd, kcd, vcd = make(B, NKV, max_len, 3 * pos + S, cuda_dev)
    scale = 64 ** -0.5
    out, ws = run(qd, kcd, vcd, pos, S, scale)
    NQ = 4 * NKV
    rout = torch.full_like(qd, float("nan"))
    rws = torch.full((B, NQ, S, 66), float("nan"), device=cuda_dev)
    p = torch.tensor([pos], device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert f(qd.data_ptr(), kcd.data_ptr(), vcd.data_ptr(), p.data_ptr(), rout.data_ptr(), rws.data_ptr(), B, NQ, NKV,
             max_len, S, scale, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, rout)
    live = rws[..., 1] > 0
    assert torch.equal(ws[..., :2], rws[..., :2])
    assert torch.equal(ws[..., 2:][live], rws[..., 2:][live])

    def t(fn, reps=20, replays=10):
        """Device time per call: `reps` calls captured in a CUDA graph, replayed (no host launch cost inside)."""
        side = torch.cuda.Stream(cuda_dev)
        side.wait_stream(torch.cuda.current_stream(cuda_dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(cuda_dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(replays):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * replays)
    ours = t(lambda: ext().decode_attention_split(qd, kcd, vcd, p, out, ws, scale))
    ref = t(lambda: f(qd.data_ptr(), kcd.data_ptr(), vcd.data_ptr(), p.data_ptr(), rout.data_ptr(), rws.data_ptr(),
                      B, NQ, NKV, max_len, S, scale, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(out, rout)
    print(f"\n[vs reference kernel] decode_attention_split B={B} NKV={NKV} len={pos + 1} S={S}: "
          f"lfm2q {ours:.1f} us, reference {ref:.1f} us ({ref / ours:.2f}x)")


def test_repeated_and_graph_replay(cuda_dev):
    _, _, _, qd, kcd, vcd = make(2, 8, 3072, 11, cuda_dev)
    p = torch.tensor([2300], device=cuda_dev)
    out = torch.empty_like(qd)
    ws = torch.empty(2, 32, 16, 66, device=cuda_dev)
    ext().decode_attention_split(qd, kcd, vcd, p, out, ws, 0.125)
    first = out.clone()
    ext().decode_attention_split(qd, kcd, vcd, p, out, ws, 0.125)
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    st = torch.cuda.Stream(cuda_dev)
    st.wait_stream(torch.cuda.current_stream(cuda_dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        ext().decode_attention_split(qd, kcd, vcd, p, out, ws, 0.125)
    for i in range(3):
        out.fill_(float("nan"))
        ws.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    p.fill_(1000)  # the graph reads pos from the device at replay
    graph.replay()
    torch.cuda.synchronize()
    assert not torch.equal(out, first)
    check_device()
