"""lfm2q_decode_attention_split_noalloc: decode attention for callers that cannot allocate device memory.

Some hosts of this library cannot call cudaMalloc: an FFI caller that is handed device pointers by another runtime
and holds no allocator, or a decode loop where an allocation would synchronize the device. This entry point takes no
workspace; the per-split partials go to a static 8 MiB array inside the library. The test calls it through the C ABI,
twice in a row with different inputs (the second call finds the first call's partials in the shared array), and checks
each output against lfm2q_decode_attention_split with a caller-allocated workspace on the same inputs: the same kernels
run, so the outputs must be equal bit for bit (tighter than the tolerance of the other attention tests). It also
checks that a size beyond the static workspace is refused before anything is launched.

The file is named to be collected last, so a run that stops at the first failure has run every other test first.
"""

import pytest
import torch

from lfm2opt import _capi

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
MAX_WS = 1 << 21  # LFM2Q_ATTN_NOALLOC_MAX_WS_FLOATS (include/lfm2q.h)


def inputs(B, NKV, max_len, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, 4 * NKV, 64, generator=g).to(BF).to(dev)
    kc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF).to(dev)
    vc = torch.randn(B, NKV, max_len, 64, generator=g).to(BF).to(dev)
    return q, kc, vc


def with_ws(q, kc, vc, pos, S, scale):
    B, NQ = q.shape[:2]
    out = torch.full_like(q, float("nan"))
    ws = torch.empty(B, NQ, S, 66, device=q.device)
    st = _capi.lib().lfm2q_decode_attention_split(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                                                  out.data_ptr(), ws.data_ptr(), B, NQ, kc.size(1), kc.size(2), S,
                                                  scale, torch.cuda.current_stream().cuda_stream)
    assert st == _capi.OK, _capi.lib().lfm2q_last_error()
    return out


def no_alloc(q, kc, vc, pos, S, scale):
    B, NQ = q.shape[:2]
    out = torch.full_like(q, float("nan"))
    st = _capi.lib().lfm2q_decode_attention_split_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                                                          out.data_ptr(), B, NQ, kc.size(1), kc.size(2), S, scale,
                                                          torch.cuda.current_stream().cuda_stream)
    assert st == _capi.OK, _capi.lib().lfm2q_last_error()
    return out


@pytest.mark.parametrize("first,second", [
    ((2, 8, 3072, 2300, 16), (2, 8, 3072, 2300, 16)),   # same shape, new inputs
    ((8, 8, 4096, 4000, 16), (1, 2, 300, 299, 3)),      # a small call after a large one: stale partials beyond it
    ((1, 2, 300, 0, 64), (3, 1, 129, 128, 2)),          # length 1 (mostly empty splits), then a ragged tail
])
def test_noalloc_equals_caller_workspace_on_two_calls_in_a_row(cuda_dev, first, second):
    outs = []
    for i, (B, NKV, max_len, pos, S) in enumerate((first, second)):
        q, kc, vc = inputs(B, NKV, max_len, 100 * i + pos + S, cuda_dev)
        p = torch.tensor([pos], device=cuda_dev)
        scale = 64 ** -0.5
        outs.append((no_alloc(q, kc, vc, p, S, scale), with_ws(q, kc, vc, p, S, scale)))
    torch.cuda.synchronize()
    for got, want in outs:
        assert not torch.isnan(got).any()
        assert torch.equal(got, want)
    assert _capi.lib().lfm2q_check_device(0) == _capi.OK


def test_noalloc_refuses_sizes_beyond_its_workspace(cuda_dev):
    q, kc, vc = inputs(1, 8, 1024, 5, cuda_dev)
    p = torch.tensor([1000], device=cuda_dev)
    out = torch.zeros_like(q)
    B, NQ = 64, 32
    S = MAX_WS // (B * NQ * 66) + 1  # one split more than fits
    st = _capi.lib().lfm2q_decode_attention_split_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(),
                                                          out.data_ptr(), B, NQ, 8, 1024, S, 0.125,
                                                          torch.cuda.current_stream().cuda_stream)
    assert st == _capi.EINVAL
    assert b"static workspace" in _capi.lib().lfm2q_last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing ran
