"""TEST INFRASTRUCTURE ONLY: oracle fused producers (add_layernorm_q, add_rmsnorm_q, silu_mul_q), CPU.

Semantics: the reference's kernels/int8_gemm.cu:529-682 (bf16 rounding points, quantization). The fp32 reductions
follow the reduction order of the lfm2q kernels (one 256-thread block per row: thread t sums elements t, t+256, ...
in order, an xor butterfly per warp, then the 8 warp sums in warp order), so sums match bit for bit. The GPU's
rsqrtf / __expf intrinsics are approximations; here they are 1/sqrt and exp, so a bf16 result can differ by one
ulp (and an int8 code by one) on rare elements.
"""

import numpy as np
import torch

from . import _c
from .gemm import silu_mul_ref
from .quant import quant_groups_ref, quant_rows_ref

_T = 256


def _block_sum(vals: np.ndarray, fma_square=False) -> np.float32:
    """Sum of a fp32 row in the kernel's order (optionally of squares, each step a fused multiply-add)."""
    D = vals.shape[0]
    part = np.zeros(_T, dtype=np.float32)
    for j in range(0, D, _T):
        chunk = vals[j:j + _T]
        n = chunk.shape[0]
        if fma_square:
            part[:n] = _c.fmaf(chunk, chunk, part[:n])
        else:
            part[:n] = (part[:n] + chunk).astype(np.float32)
    warp = part.reshape(_T // 32, 32).copy()
    lane = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        warp = (warp + warp[:, lane ^ o]).astype(np.float32)
    t = np.float32(0)
    for w in range(_T // 32):
        t = np.float32(t + warp[w, 0])
    return t


def _residual(h, y):
    if y is None:
        return h.clone()
    return (h.float() + y.float()).to(torch.bfloat16)


def _quant(x_bf16, grouped):
    return quant_groups_ref(x_bf16) if grouped else quant_rows_ref(x_bf16)


@torch.no_grad()
def add_layernorm_q_ref(h, y, w, b, eps, grouped):
    """Returns (h_new, q, s)."""
    hn = _residual(h, y)
    X = hn.float().numpy()
    out = np.empty_like(X)
    wf, bf = w.float().numpy(), b.float().numpy()
    D = X.shape[1]
    for r in range(X.shape[0]):
        x = X[r]
        mean = np.float32(_block_sum(x) / np.float32(D))
        d = (x - mean).astype(np.float32)
        var = np.float32(_block_sum(d, fma_square=True) / np.float32(D))
        rstd = np.float32(1.0 / np.sqrt(np.float64(np.float32(var + np.float32(eps)))))
        t = (d * rstd).astype(np.float32)
        out[r] = _c.fmaf(t, wf, bf)
    xb = torch.from_numpy(out).to(torch.bfloat16)
    q, s = _quant(xb, grouped)
    return hn, q, s


@torch.no_grad()
def add_rmsnorm_q_ref(h, y, w, eps, grouped):
    """Returns (h_new, q, s)."""
    hn = _residual(h, y)
    X = hn.float().numpy()
    out = np.empty_like(X)
    wf = w.float().numpy()
    H = X.shape[1]
    for r in range(X.shape[0]):
        x = X[r]
        ss = _block_sum(x, fma_square=True)
        rs = np.float32(1.0 / np.sqrt(np.float64(np.float32(np.float32(ss / np.float32(H)) + np.float32(eps)))))
        n = torch.from_numpy((x * rs).astype(np.float32)).to(torch.bfloat16).float().numpy()
        out[r] = (wf * n).astype(np.float32)
    xb = torch.from_numpy(out).to(torch.bfloat16)
    q, s = _quant(xb, grouped)
    return hn, q, s


@torch.no_grad()
def silu_mul_q_ref(g, grouped):
    """Returns (q, s) of bf16(bf16(silu(g1)) * g3)."""
    return _quant(silu_mul_ref(g), grouped)
