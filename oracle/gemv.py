"""TEST INFRASTRUCTURE ONLY: oracle decode GEMVs (CPU)."""

import torch
import torch.nn.functional as F

from .gemm import silu_mul_ref


@torch.no_grad()
def gemv_ref(W, scale, x):
    """The reference's GEMV check expression (tests/test_kernels.py:134-138): F.linear(x.float(), Wq.float() *
    scale[:, None]).to(bf16) for int8 W; F.linear(x, W) (bf16) for bf16 W without a scale."""
    if W.dtype == torch.int8:
        return F.linear(x.float(), W.float() * scale.float()[:, None]).to(torch.bfloat16)
    if scale is None:
        return F.linear(x.float(), W.float()).to(torch.bfloat16)
    return (F.linear(x.float(), W.float()) * scale.float()).to(torch.bfloat16)


@torch.no_grad()
def gemv_f64(W, scale, x):
    """fp64 value of the GEMV before the final bf16 rounding: (x . W^T) * scale."""
    r = x.double() @ W.double().t()
    return r * scale.double() if scale is not None else r


@torch.no_grad()
def gemv_epi_ref(epi, W, scale, x, state=None, cw=None, cbias=None):
    """Batch-1 GEMV + epilogue (the reference's gemv_epi_kernel, kernels/lfm2_decode.cu:724-805), starting from the
    bf16 values the plain GEMV stores (computed here in fp64 and rounded: the GPU's fp32 accumulation may differ by
    one bf16 ulp). epi 0: bf16(bf16(silu(g)) * u). epi 1: short-conv step, conv = w0*s1 + w1*s2 + w2*bx (+ bias)
    with every product and sum rounded to fp32 in that order; returns (y, new_state)."""
    part = gemv_f64(W, scale, x).reshape(-1).to(torch.bfloat16)
    if epi == 0:
        return silu_mul_ref(part[None, :])[0]
    S = part.numel() // 3
    b_, c_, x_ = part[:S].float(), part[S:2 * S].float(), part[2 * S:].float()
    bx = (b_ * x_).to(torch.bfloat16).float()
    st = state.reshape(S, 3).float()
    s1, s2 = st[:, 1], st[:, 2]
    new_state = torch.stack([st[:, 1], st[:, 2], bx], dim=1).to(torch.bfloat16)
    w = cw.reshape(S, 3).float()
    acc = w[:, 0] * s1
    acc = acc + w[:, 1] * s2
    acc = acc + w[:, 2] * bx
    if cbias is not None:
        acc = acc + cbias.float()
    y = (c_ * acc.to(torch.bfloat16).float()).to(torch.bfloat16)
    return y, new_state


@torch.no_grad()
def dequantize_int4_ref(packed, scale):
    """int4 codes (low nibble = input 2j, high nibble = 2j + 1, stored + 8) times the group scales, fp32 [N, K] (the
    reference's dequantize_int4, src/lfm2opt/quant.py:43-48)."""
    p = packed.to(torch.int32)
    q = torch.stack([(p & 0xF) - 8, (p >> 4) - 8], dim=-1).reshape(packed.shape[0], -1).float()
    group = q.shape[1] // scale.shape[1]
    return (q.reshape(q.shape[0], -1, group) * scale.float()[..., None]).reshape(q.shape[0], -1)


@torch.no_grad()
def gemv_w4_ref(packed, scale, x):
    """The reference's INT4 GEMV check expression (tests/test_kernels.py:148-150): F.linear(x.float(),
    dequantize_int4(Wp, S)).to(bf16)."""
    return F.linear(x.float(), dequantize_int4_ref(packed, scale)).to(torch.bfloat16)


@torch.no_grad()
def gemv_w4_f64(packed, scale, x):
    """fp64 value of the INT4 GEMV before the final bf16 rounding."""
    return x.double() @ dequantize_int4_ref(packed, scale).double().t()
