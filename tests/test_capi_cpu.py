"""The C-ABI library on CPU: it loads without a GPU, exports every entry point include/lfm2q.h declares, and rejects
bad arguments with LFM2Q_EINVAL and the reference bindings' messages before touching a device."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from lfm2opt import _capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "lfm2q.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lfm2q_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _capi.lib()
    names = declared()
    assert len(names) >= 18
    for n in names:
        assert hasattr(L, n), n
        assert n in _capi.SIGNATURES, n  # the Python binding covers every entry point


def test_version_and_no_error():
    L = _capi.lib()
    assert L.lfm2q_version().decode().startswith("lfm2q")
    assert isinstance(L.lfm2q_last_error(), bytes)


def _st(name, *args):
    return getattr(_capi.lib(), name)(*args)


def test_validation_runs_before_the_device():
    fake = 1 << 20  # 16-byte aligned, never dereferenced: the calls below fail validation first
    assert _st("lfm2q_gemm_i8", fake, fake, 0, fake, fake, None, fake, 16, 8, 24, 0, None) == _capi.EINVAL
    assert b"K % 16 == 0" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_gemm_i8", fake, fake, 0, fake, fake, None, fake, 16, 12, 32, 0, None) == _capi.EINVAL
    assert _st("lfm2q_gemm_i8", fake, fake, 1, fake, fake, None, fake, 16, 8, 32, 0, None) == _capi.EINVAL
    assert b"K % 64" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_gemm_i8", fake + 4, fake, 0, fake, fake, None, fake, 16, 8, 32, 0, None) == _capi.EINVAL
    assert b"aligned" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_gemm_i8_q", fake, fake, fake, fake, None, fake, fake, 16, 64, 64, 0, None) == _capi.EINVAL
    assert b"N % 128" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_quant_rows", fake, fake, fake, 4, 12, None) == _capi.EINVAL
    assert _st("lfm2q_quant_rows", fake, fake, fake, 4, 16392, None) == _capi.EINVAL
    assert _st("lfm2q_quant_groups", fake, fake, fake, 4, 96, None) == _capi.EINVAL
    assert _st("lfm2q_gemv", fake, 1, fake, fake, fake, 64, 256, 0, 1, None) == _capi.EINVAL
    assert b"512 (int8)" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_gemv", fake, 1, None, fake, fake, 64, 512, 0, 1, None) == _capi.EINVAL
    assert b"int8 W needs fp32 scale" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_gemv_epi", 2, fake, 1, fake, fake, fake, 64, 512, None, None, None, None) == _capi.EINVAL
    assert _st("lfm2q_gemv_epi", 1, fake, 1, fake, fake, fake, 64, 512, None, None, None, None) == _capi.EINVAL
    assert b"state" in _capi.lib().lfm2q_last_error()
    att = "lfm2q_decode_attention_split"
    assert _st(att, fake, fake, fake, fake, fake, fake, 0, 32, 8, 3072, 16, 0.125, None) == _capi.OK  # B = 0: nothing to do
    assert _st(att, fake, fake, fake, fake, fake, fake, 2, 24, 8, 3072, 16, 0.125, None) == _capi.EINVAL
    assert b"4 query heads per KV head" in _capi.lib().lfm2q_last_error()
    assert _st(att, fake, fake, fake, fake, fake, fake, 2, 32, 8, 3072, 0, 0.125, None) == _capi.EINVAL
    assert b"ws [B, NQ, S, 66]" in _capi.lib().lfm2q_last_error()
    assert _st(att, fake + 8, fake, fake, fake, fake, fake, 2, 32, 8, 3072, 16, 0.125, None) == _capi.EINVAL
    assert b"aligned" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_argmax_next", fake, fake, None, 2, 1001, None) == _capi.EINVAL  # rows not 16-byte aligned
    assert b"multiple of 8" in _capi.lib().lfm2q_last_error()
    assert _st("lfm2q_embed_rmsnorm", fake, fake, fake, fake, fake, 1, 16384, 1e-5, None) == _capi.EINVAL
    na = "lfm2q_decode_attention_split_noalloc"
    assert _st(na, fake, fake, fake, fake, fake, 64, 32, 8, 3072, 16, 0.125, None) == _capi.EINVAL  # 8.65 M floats
    assert b"static workspace" in _capi.lib().lfm2q_last_error()
    assert _st(na, fake, fake, fake, fake, fake, 0, 32, 8, 3072, 16, 0.125, None) == _capi.OK
    assert _st("lfm2q_gemm_i8_silu", fake, fake, fake, fake, None, fake, 16, 12, 32, None) == _capi.EINVAL
    assert _st("lfm2q_silu_mul_q", fake, fake, fake, 4, 100, 0, None) == _capi.EINVAL
    assert _st("lfm2q_add_rmsnorm_q", fake, None, fake, fake, fake, 4, 20, ctypes.c_float(1e-5), 0, None) \
        == _capi.EINVAL


def test_empty_batches_are_noops_without_a_device():
    fake = 1 << 20
    assert _st("lfm2q_quant_rows", fake, fake, fake, 0, 128, None) == _capi.OK
    assert _st("lfm2q_gemm_i8", fake, fake, 0, fake, fake, None, fake, 0, 64, 128, 0, None) == _capi.OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_valid_call_without_a_device_is_not_supported():
    fake = 1 << 20
    assert _st("lfm2q_quant_rows", fake, fake, fake, 4, 128, None) == _capi.ENOTSUP
    assert b"sm_100" in _capi.lib().lfm2q_last_error()
    assert _capi.lib().lfm2q_device_supported() == 0


def test_python_binding_raises_with_reference_messages():
    from lfm2opt.kernels import int8_ext, ext
    E = int8_ext()
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    q = torch.zeros(4, 128, dtype=torch.int8)
    s = torch.zeros(4)
    with pytest.raises(RuntimeError, match="x must be contiguous CUDA"):
        E.quant_rows(x, q, s)
    with pytest.raises(RuntimeError, match="must be contiguous CUDA"):
        ext().gemv(q, s, x, x)
    with pytest.raises(RuntimeError, match="xq must be contiguous CUDA"):
        E.gemm_i8(q, s, q, s, None, x, False)


def test_selftest_rejects_bad_limits():
    L = _capi.lib()
    assert L.lfm2q_selftest_wait_timeout(5, None) == _capi.EINVAL
    assert L.lfm2q_selftest_wait_timeout(40, None) == _capi.EINVAL


def test_gemv_chain_rejects_bad_layers_without_a_gpu():
    """lfm2q_gemv_chain validates every layer on the host before touching a device."""
    L = _capi.lib()
    fake = ctypes.c_void_p(1 << 20)
    ok = _capi.GemvLayer(1 << 20, 1 << 20, 2 << 20, 3 << 20, 256, 2048)
    arr = (_capi.GemvLayer * 2)(ok, ok)
    assert L.lfm2q_gemv_chain(arr, 0, 1, None) == _capi.EINVAL  # no layers
    assert L.lfm2q_gemv_chain(arr, 97, 1, None) == _capi.EINVAL  # too many
    assert L.lfm2q_gemv_chain(arr, 2, 5, None) == _capi.EINVAL  # B > 4
    assert L.lfm2q_gemv_chain(None, 1, 1, None) == _capi.EINVAL
    arr[1] = _capi.GemvLayer(1 << 20, 1 << 20, 2 << 20, 3 << 20, 256, 2000)  # K % 512
    assert L.lfm2q_gemv_chain(arr, 2, 1, None) == _capi.EINVAL
    assert b"layer 1" in L.lfm2q_last_error()
    arr[1] = _capi.GemvLayer(1 << 20, 1 << 20, 2 << 20, (2 << 20) + 64, 256, 2048)  # y overlaps x
    assert L.lfm2q_gemv_chain(arr, 2, 1, None) == _capi.EINVAL
    arr[1] = _capi.GemvLayer(1 << 20, 1 << 20, (2 << 20) + 8, 3 << 20, 256, 2048)  # x not 16-byte aligned
    assert L.lfm2q_gemv_chain(arr, 2, 1, None) == _capi.EINVAL
    del fake


def test_gemv_w4_rejects_bad_shapes_without_a_gpu():
    L = _capi.lib()
    p = 1 << 20
    assert L.lfm2q_gemv_w4(p, p, p, p, 256, 2048, 64, 1, None) == _capi.EINVAL  # group % 128
    assert L.lfm2q_gemv_w4(p, p, p, p, 256, 2000, 128, 1, None) == _capi.EINVAL  # K % group
    assert L.lfm2q_gemv_w4(p, p, p, p, 256, 2048, 128, 5, None) == _capi.EINVAL  # B > 4
    assert L.lfm2q_gemv_w4(p, p, p, p, 256, 8192, 128, 4, None) == _capi.EINVAL  # B * K > 16384
    assert L.lfm2q_gemv_w4(None, p, p, p, 256, 2048, 128, 1, None) == _capi.EINVAL
