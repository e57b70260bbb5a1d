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


@torch.no_grad()
def quantize_int4_ref(w: torch.Tensor, group: int = 128, clip_search: bool = False):
    """Group-wise symmetric INT4 with two codes per byte; the reference's quantize_int4 (src/lfm2opt/quant.py:22-40):
    scale = max(amax, 1e-12) / 7 per row and group (optionally the clipped scale amax * a / 7, a on 16 steps of
    [0.70, 1.00], with the smallest squared error, first best kept); q = clamp(round(w / scale), -8, 7); byte j of a
    row = (q[2j] + 8) | (q[2j + 1] + 8) << 4. Returns (packed uint8 [N, K/2], scale fp32 [N, K/group])."""
    N, K = w.shape
    wg = w.float().reshape(N, K // group, group)
    amax = wg.abs().amax(-1).clamp_min(1e-12)
    scale = amax / 7
    if clip_search:
        best = torch.full_like(amax, float("inf"))
        for a in torch.linspace(0.70, 1.00, 16).tolist():
            s = amax * a / 7
            err = (torch.round(wg / s[..., None]).clamp(-8, 7) * s[..., None] - wg).pow(2).sum(-1)
            scale = torch.where(err < best, s, scale)
            best = torch.minimum(err, best)
    q = (torch.round(wg / scale[..., None]).clamp(-8, 7) + 8).to(torch.int32).reshape(N, K)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8), scale
