"""TEST INFRASTRUCTURE ONLY: oracle fused producers (add_layernorm_q, add_rmsnorm_q, silu_mul_q), CPU.

Restates the reference's kernels operation by operation, reductions included:
  add_layernorm_q  kernels/int8_gemm.cu:529-585. One warp per row: lane l holds the 4-element chunks l, l + 32, ...
                   (elements (c * 32 + l) * 4 + j) and adds ((v0 + v1) + v2) + v3 of each chunk to its running sum in
                   chunk order; the lane sums meet in an xor butterfly (16, 8, 4, 2, 1) (`wsum`, :483-488); mean =
                   total / D. The squared deviations accumulate per lane, element by element, as fused multiply-adds
                   (nvcc contracts `qs += d * d`); rstd = rsqrt(total / D + eps); x = bf16(fma((v - mean) * rstd, w,
                   b)) (the contraction of `(v - mean) * rstd * w + b`).
  add_rmsnorm_q    kernels/int8_gemm.cu:589-642. One 256-thread block per row: thread t accumulates fma(v, v, ss) over
                   elements t, t + 256, ...; xor butterfly per warp; the 8 warp sums go through a second 32-lane
                   butterfly with zeros in lanes 8..31 (block_sum, kernels/lfm2_decode.cu:79-90); rs = rsqrt(ss / H +
                   eps); x = bf16(w * bf16(h * rs)).
  silu_mul_q       kernels/int8_gemm.cu:646-682: a = bf16(bf16(g1 / (1 + exp(-g1))) * g3).
Then quantization (order-free: maxima) as quant_rows / quant_groups.

The GPU evaluates rsqrt and exp with the hardware approximations rsqrtf / __expf; here they are the correctly rounded
1/sqrt and exp, so a row's rstd (and a SiLU value) can differ in the last bit from the GPU's, and an int8 code can then
differ by one. The bit-for-bit pin of the CUDA producers is the reference's own kernels run on the same GPU
(tests/test_gpu_reference_kernels.py); this oracle pins the reduction order and the rounding points, and is itself
checked against a direct per-lane / per-thread loop in tests/test_oracle.py.
"""

import numpy as np
import torch

from . import _c
from .gemm import silu_mul_ref
from .quant import quant_groups_ref, quant_rows_ref

_T = 256  # threads per row block (rmsnorm)


def _butterfly(lanes: np.ndarray) -> np.ndarray:
    """xor-butterfly sum over the last axis (32 lanes), fp32, returns lane 0's total (every lane ends equal)."""
    v = lanes.astype(np.float32, copy=True)
    idx = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        v = (v + v[..., idx ^ o]).astype(np.float32)
    return v[..., 0]


def _ln_chunks(X: np.ndarray):
    """[R, D] fp32 -> [R, rounds, 32, 4] chunks in the warp's lane layout, and the validity mask [rounds, 32]."""
    R, D = X.shape
    nc = D // 4
    rounds = -(-nc // 32)
    pad = np.zeros((R, rounds * 32 * 4), dtype=np.float32)
    pad[:, :D] = X
    valid = (np.arange(rounds * 32).reshape(rounds, 32) < nc)
    return pad.reshape(R, rounds, 32, 4), valid


def layernorm_stats(X: np.ndarray, eps: float):
    """(mean [R], rstd [R]) of fp32 rows X [R, D] in the reference's warp order (rstd correctly rounded)."""
    R, D = X.shape
    ch, valid = _ln_chunks(X)
    s = np.zeros((R, 32), dtype=np.float32)
    for r in range(ch.shape[1]):
        c = ch[:, r]
        t = (((c[..., 0] + c[..., 1]).astype(np.float32) + c[..., 2]).astype(np.float32) + c[..., 3]).astype(np.float32)
        s = np.where(valid[r], (s + t).astype(np.float32), s)
    mean = (_butterfly(s) / np.float32(D)).astype(np.float32)
    qs = np.zeros((R, 32), dtype=np.float32)
    for r in range(ch.shape[1]):
        for j in range(4):
            d = (ch[:, r, :, j] - mean[:, None]).astype(np.float32)
            qs = np.where(valid[r], _c.fmaf(d, d, qs), qs)
    var = (_butterfly(qs) / np.float32(D)).astype(np.float32)
    rstd = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float32).astype(np.float64))).astype(np.float32)
    return mean, rstd


def rmsnorm_rs(X: np.ndarray, eps: float) -> np.ndarray:
    """rs [R] = rsqrt(sum(x^2) / H + eps) of fp32 rows X [R, H] in the reference's block order (correctly rounded)."""
    R, H = X.shape
    part = np.zeros((R, _T), dtype=np.float32)
    for j in range(0, H, _T):
        chunk = X[:, j:j + _T]
        n = chunk.shape[1]
        part[:, :n] = _c.fmaf(chunk, chunk, part[:, :n])
    warp = _butterfly(part.reshape(R, _T // 32, 32))  # [R, 8]
    lanes = np.zeros((R, 32), dtype=np.float32)
    lanes[:, :_T // 32] = warp
    ss = _butterfly(lanes)
    v = ((ss / np.float32(H)).astype(np.float32) + np.float32(eps)).astype(np.float32)
    return (1.0 / np.sqrt(v.astype(np.float64))).astype(np.float32)


def _residual(h, y):
    if y is None:
        return h.clone()
    return (h.float() + y.float()).to(torch.bfloat16)


def _quant(x_bf16, grouped):
    return quant_groups_ref(x_bf16) if grouped else quant_rows_ref(x_bf16)


def _ulp_shift(v: np.ndarray, k: int) -> np.ndarray:
    """v moved by k fp32 ulps (k < 0: towards -inf)."""
    v = v.astype(np.float32, copy=True)
    for _ in range(abs(k)):
        v = np.nextafter(v, np.float32(np.inf if k > 0 else -np.inf)).astype(np.float32)
    return v


@torch.no_grad()
def add_layernorm_q_ref(h, y, w, b, eps, grouped, rstd_ulps=0):
    """Returns (h_new, q, s). rstd_ulps moves every row's rstd by that many fp32 ulps from the correctly rounded value
    (the GPU's rsqrtf is within 2 ulps of it)."""
    hn = _residual(h, y)
    X = hn.float().numpy()
    mean, rstd = layernorm_stats(X, eps)
    rstd = _ulp_shift(rstd, rstd_ulps)
    t = ((X - mean[:, None]).astype(np.float32) * rstd[:, None]).astype(np.float32)
    wf, bf = w.float().numpy(), b.float().numpy()
    out = _c.fmaf(t, np.broadcast_to(wf, t.shape).copy(), np.broadcast_to(bf, t.shape).copy())
    xb = torch.from_numpy(out).to(torch.bfloat16)
    q, s = _quant(xb, grouped)
    return hn, q, s


@torch.no_grad()
def add_rmsnorm_q_ref(h, y, w, eps, grouped, rs_ulps=0):
    """Returns (h_new, q, s). rs_ulps: as add_layernorm_q_ref's rstd_ulps."""
    hn = _residual(h, y)
    X = hn.float().numpy()
    rs = _ulp_shift(rmsnorm_rs(X, eps), rs_ulps)
    n = torch.from_numpy((X * rs[:, None]).astype(np.float32)).to(torch.bfloat16).float().numpy()
    out = (w.float().numpy()[None, :] * n).astype(np.float32)
    xb = torch.from_numpy(out).to(torch.bfloat16)
    q, s = _quant(xb, grouped)
    return hn, q, s


@torch.no_grad()
def silu_mul_q_ref(g, grouped):
    """Returns (q, s) of bf16(bf16(silu(g1)) * g3)."""
    return _quant(silu_mul_ref(g), grouped)
