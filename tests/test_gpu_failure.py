"""Failure detection on the GPU without a fault: a kernel whose bounded pipeline wait can never be satisfied gives up
after a short limit, records the device error word and ends normally; the host reads LFM2Q_ETIMEOUT, clears the word,
and the context keeps working."""

import pytest
import torch

from lfm2opt import _capi
from lfm2opt.int8 import quantize_rows
from lfm2opt.kernels import int8_ext
from lfm2opt.quant import quantize_int8

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    L = _capi.lib()
    torch.cuda.synchronize()
    assert L.lfm2q_check_device(1) == _capi.OK
    stream = torch.cuda.current_stream(cuda_dev).cuda_stream
    assert L.lfm2q_selftest_wait_timeout(24, stream) == _capi.OK  # 2^24 cycles: ~10 ms
    torch.cuda.synchronize()
    assert L.lfm2q_check_device(1) == _capi.ETIMEOUT
    assert b"timed out" in L.lfm2q_last_error()
    assert L.lfm2q_check_device(0) == _capi.OK  # cleared
    # the context is intact: a normal GEMM still runs and is still exact
    g = torch.Generator().manual_seed(3)
    x = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    w = (torch.randn(384, 512, generator=g) * 0.02).to(torch.bfloat16)
    xq, sx = quantize_rows(x.to(cuda_dev))
    wq, sw = quantize_int8(w)
    y = torch.empty(256, 384, device=cuda_dev, dtype=torch.bfloat16)
    int8_ext().gemm_i8(xq, sx, wq.to(cuda_dev), sw.to(cuda_dev), None, y, False)
    import oracle
    r = oracle.gemm_i8_ref(xq.cpu(), sx.cpu(), wq, sw)
    assert oracle.bf16_ulps(y.cpu(), r) == 0
    assert L.lfm2q_check_device(0) == _capi.OK

