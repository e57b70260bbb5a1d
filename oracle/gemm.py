"""TEST INFRASTRUCTURE ONLY: oracle W8A8 / W8A16 GEMMs (CPU).

The int32 accumulator is computed exactly (torch._int_mm on CPU, equal to the fp64 product for every shape here);
the epilogues restate the reference's fp32 operation order.
"""

import numpy as np
import torch
import torch.nn.functional as F

from . import _c
from .quant import quant_groups_ref


@torch.no_grad()
def int_mm_exact(xq: torch.Tensor, wq: torch.Tensor) -> torch.Tensor:
    """int32 [M, N] = xq [M, K] . wq [N, K]^T, exact (the value the tensor cores must produce)."""
    if xq.shape[0] == 0:
        return torch.zeros(0, wq.shape[0], dtype=torch.int32)
    return torch._int_mm(xq.contiguous(), wq.contiguous().t())


def bf16_ulps(a: torch.Tensor, b: torch.Tensor) -> int:
    """Max distance in bf16 units in the last place (the reference's tests/test_int8_gemm.py:41-47)."""
    ia = a.view(torch.int16).int()
    ib = b.view(torch.int16).int()
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return int((ia - ib).abs().max().item()) if ia.numel() else 0


@torch.no_grad()
def gemm_i8_ref(xq, sx, wq, sw, bias=None, gelu=False, out_f32=False):
    """Per-token W8A8 (the reference's test_i8 reference, tests/test_int8_gemm.py:166-172, and the store_tile
    epilogue, kernels/int8_gemm.cu:93-115): r = (float(acc) * sx[m]) * sw[n] (+ bias[n]) (GELU tanh), rounded to
    bf16. float(acc) rounds the exact int32 to fp32 (round to nearest even), as the GPU's cvt.rn does."""
    acc = int_mm_exact(xq, wq).float()
    r = acc * sx.float()[:, None] * sw.float()[None, :]
    if bias is not None:
        r = r + bias.float()
    if gelu:
        r = F.gelu(r, approximate="tanh")
    return r if out_f32 else r.to(torch.bfloat16)


@torch.no_grad()
def gemm_i8_grouped_f64(xq, sxT, wq, sw, bias=None, gelu=False):
    """fp64 reference of the grouped W8A8 (the reference's test_i8_grouped, tests/test_int8_gemm.py:90-98)."""
    M, K = xq.shape
    r = torch.zeros(M, wq.shape[0], dtype=torch.float64)
    for g in range(K // 64):
        part = xq[:, g * 64:(g + 1) * 64].double() @ wq[:, g * 64:(g + 1) * 64].double().t()
        r = r + part * sxT[g].double()[:, None]
    r = r * sw.double()[None, :]
    if bias is not None:
        r = r + bias.double()
    if gelu:
        r = F.gelu(r, approximate="tanh")
    return r


@torch.no_grad()
def gemm_i8_grouped_ref(xq, sxT, wq, sw, bias=None, gelu=False, round_bf16=True):
    """Grouped W8A8 with the kernel's exact fp32 operation order (kernels/int8_gemm.cu:202-230, :286-296):
    f = 0; for every 64-wide group g in order: f = fmaf(float(part_g), sxT[g][m], f); y = f * sw[n] (+ bias[n])
    (GELU); the int32 group sums are exact and |part_g| < 2^24, so float(part_g) is exact."""
    M, K = xq.shape
    N = wq.shape[0]
    acc = np.zeros((M, N), dtype=np.float32)
    for g in range(K // 64):
        part = int_mm_exact(xq[:, g * 64:(g + 1) * 64], wq[:, g * 64:(g + 1) * 64]).numpy()
        _c.fold_group(part, sxT[g].float().numpy(), acc)
    r = torch.from_numpy(acc) * sw.float()[None, :]
    if bias is not None:
        r = r + bias.float()
    if gelu:
        r = F.gelu(r, approximate="tanh")
    return r.to(torch.bfloat16) if round_bf16 else r


@torch.no_grad()
def gemm_i8_q_ref(xq, sxT, wq, sw, bias=None, gelu=False):
    """gemm_i8_q = grouped gemm_i8 (bf16 out) followed by the grouped quantizer (the reference's test_i8_qout,
    tests/test_int8_gemm.py:107-120; kernel kernels/int8_gemm.cu:234-285). Returns (yq [M, N], ysT [N/64, M])."""
    y = gemm_i8_grouped_ref(xq, sxT, wq, sw, bias, gelu)
    return quant_groups_ref(y)


@torch.no_grad()
def silu_mul_ref(g: torch.Tensor) -> torch.Tensor:
    """g bf16 [M, 2I] -> bf16(bf16(silu(a)) * b), the reference's silu_mul (kernels/lfm2_decode.cu:954-963);
    silu(a) = a / (1 + exp(-a)) in fp32 (the GPU kernels use the __expf / __fdividef intrinsics: see
    silu_chain_close for how far apart the two may be)."""
    I = g.shape[-1] // 2
    a, u = g[..., :I].float(), g[..., I:].float()
    s = (a / (1.0 + torch.exp(-a))).to(torch.bfloat16).float()
    return (s * u).to(torch.bfloat16)


def silu_chain_close(y: torch.Tensor, r: torch.Tensor, frac: float = 1e-3):
    """Acceptance check for bf16(bf16(silu(g)) * u) computed on the GPU (`__expf`, `__fdividef`) against
    silu_mul_ref on the CPU (torch's vectorised exp, whose last fp32 bit depends on the host's instruction set).
    The chain rounds twice: one bf16 ulp of difference in the inner bf16(silu(g)) moves the product by up to one
    ulp before its own rounding, so an output may differ by 2 ulps; differences stay rare. Returns (ok, detail)."""
    u = bf16_ulps(y, r)
    f = (y != r).float().mean().item() if y.numel() else 0.0
    return u <= 2 and f < frac, f"max {u} ulps, {f:.2e} of the elements differ"


def gelu_close(y: torch.Tensor, r: torch.Tensor):
    """Acceptance check for the GELU epilogue against gemm_i8_ref(..., gelu=True): <= 1 bf16 ulp, except in the fp32
    cancellation region of 0.5 v (1 + tanh(u)) near tanh = -1 (v < ~ -4.5), where the outputs are below 2e-7 in
    magnitude and the GPU's and the CPU's tanh may round 1 + tanh differently: there <= 4e-7 absolute.
    Returns (ok, detail)."""
    ia, ib = y.view(torch.int16).int(), r.view(torch.int16).int()
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    bad = ((ia - ib).abs() > 1) & ((y.float() - r.float()).abs() > 4e-7)
    return (not bool(bad.any())), f"{int(bad.sum())} outside the GELU bar, max {bf16_ulps(y, r)} ulps"


@torch.no_grad()
def gemm_i8_silu_ref(xq, sx, w13, sw13, bias=None):
    """The fused SiLU-gate GEMM's parity target: gemm_i8 (bf16 out, per token) over [w1 | w3], then silu_mul."""
    return silu_mul_ref(gemm_i8_ref(xq, sx, w13, sw13, bias))


@torch.no_grad()
def gemm_w8_f64(x, wq, sw, bias=None, gelu=False):
    """fp64 reference of W8A16 (the reference's test_w8, tests/test_int8_gemm.py:185-191)."""
    r = (x.double() @ wq.double().t()) * sw.double()[None, :]
    if bias is not None:
        r = r + bias.double()
    if gelu:
        r = F.gelu(r, approximate="tanh")
    return r
