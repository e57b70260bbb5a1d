"""ctypes binding of liblfm2q.so (the C ABI in include/lfm2q.h).

Loading fails loudly when the library has not been built: there is no CPU or PyTorch fallback for any op.
"""

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblfm2q.so"

OK, EINVAL, ENOTSUP, ECUDA, ETIMEOUT = 0, -22, -95, -5, -62

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float

# name -> argument types (all entry points return int unless listed in _VOID / _STR)
SIGNATURES = {
    "lfm2q_last_error": [],
    "lfm2q_version": [],
    "lfm2q_device_supported": [],
    "lfm2q_check_device": [_i],
    "lfm2q_quant_rows": [_p, _p, _p, _i, _i, _p],
    "lfm2q_quant_groups": [_p, _p, _p, _i, _i, _p],
    "lfm2q_gemm_i8": [_p, _p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_gemm_i8_q": [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_gemm_i8_silu": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "lfm2q_gemm_w8": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_add_layernorm_q": [_p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _p],
    "lfm2q_add_rmsnorm_q": [_p, _p, _p, _p, _p, _i, _i, _f, _i, _p],
    "lfm2q_silu_mul_q": [_p, _p, _p, _i, _i, _i, _p],
    "lfm2q_gemv": [_p, _i, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_gemv_epi": [_i, _p, _i, _p, _p, _p, _i, _i, _p, _p, _p, _p],
    "lfm2q_gemv_a8": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_linear_a8": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_set_pdl": [_i],
    "lfm2q_set_gemv_impl": [_i],
    "lfm2q_set_gemm_tile": [_i],
    "lfm2q_set_gemv_trigger": [_i],
    "lfm2q_set_gemv_path": [_i],
    "lfm2q_selftest_wait_timeout": [_i, _p],
    "lfm2q_gemv_chain": [_p, _i, _i, _p],
    "lfm2q_gemv_w4": [_p, _p, _p, _p, _i, _i, _i, _i, _p],
    "lfm2q_add_rmsnorm": [_p, _p, _p, _p, _i, _i, _f, _p],
    "lfm2q_shortconv_step": [_p, _p, _p, _p, _p, _i, _i, _p],
    "lfm2q_embed_rmsnorm": [_p, _p, _p, _p, _p, _i, _i, _f, _p],
    "lfm2q_argmax_next": [_p, _p, _p, _i, _i, _p],
    "lfm2q_qk_norm_rope_kv": [_p, _p, _p, _p, _f, _p, _p, _p, _p, _i, _i, _i, _i, _f, _p],
    "lfm2q_decode_attention_split": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p],
    "lfm2q_decode_attention_split_noalloc": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p],
}
_VOID = {"lfm2q_set_pdl", "lfm2q_set_gemv_impl", "lfm2q_set_gemm_tile", "lfm2q_set_gemv_trigger",
         "lfm2q_set_gemv_path"}
_STR = {"lfm2q_last_error", "lfm2q_version"}


class GemvLayer(ctypes.Structure):
    """lfm2q_gemv_layer (include/lfm2q.h)."""

    _fields_ = [("W", _p), ("scale", _p), ("x", _p), ("y", _p), ("N", _i), ("K", _i)]

_LIB = None


def lib():
    """The loaded library (ctypes.CDLL), with argument and return types set."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"lfm2q: {LIB_PATH} is not built. Build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(or python lfm2.5-vl-optimization_b200/build.py); there is no fallback implementation.")
        L = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None if name in _VOID else (ctypes.c_char_p if name in _STR else ctypes.c_int)
        _LIB = L
    return _LIB


def call(name, *args):
    """Call entry point `name`; raise RuntimeError with the library's message on a non-OK status."""
    st = getattr(lib(), name)(*args)
    if st != OK:
        msg = lib().lfm2q_last_error().decode()
        raise RuntimeError(msg or f"{name} failed with status {st}")
    return st
