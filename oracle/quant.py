"""TEST INFRASTRUCTURE ONLY: oracle quantizers (CPU, torch)."""

import torch


@torch.no_grad()
def quantize_int8_ref(w: torch.Tensor):
    """Per-output-row symmetric weight quantization; the reference's src/lfm2opt/quant.py:14-18."""
    wf = w.float()
    scale = (wf.abs().amax(1) / 127).clamp_min(1e-12)
    q = torch.round(wf / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.contiguous()


@torch.no_grad()
def quant_rows_ref(x: torch.Tensor):
    """Per-row activation quantization; the reference's ref_quant (tests/test_int8_gemm.py:35-38), which its
    quant_rows kernel (kernels/int8_gemm.cu:393-432) must equal bit for bit: scale = max(|x|, 1e-8) / 127 by true
    division, q = round-half-even(x / scale) clamped to +-127."""
    a = x.float().abs().amax(-1).clamp_min(1e-8)
    s = a / torch.full_like(a, 127.0)
    return torch.round(x.float() / s[:, None]).clamp(-127, 127).to(torch.int8), s


@torch.no_grad()
def quant_groups_ref(x: torch.Tensor):
    """Per-row, per-64-channel activation quantization with transposed scales [K/64, M]; the reference's
    ref_quant_groups (tests/test_int8_gemm.py:64-69) / quant_groups_kernel (kernels/int8_gemm.cu:435-474)."""
    xg = x.float().unflatten(-1, (-1, 64))
    a = xg.abs().amax(-1).clamp_min(1e-8)
    s = a / torch.full_like(a, 127.0)
    q = torch.round(xg / s[..., None]).clamp(-127, 127).to(torch.int8).flatten(-2)
    return q, s.t().contiguous()
