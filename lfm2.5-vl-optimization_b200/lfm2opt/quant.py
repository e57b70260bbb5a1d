"""Weight-only quantization for the decode GEMVs and the W8A8 GEMMs; done once at load time.

INT8: one fp32 scale per output row, W ~= q * s[n], q in [-127, 127], round-to-nearest (half to even), symmetric.
Same expression as the reference's quantize_int8 (src/lfm2opt/quant.py:14-18): scale = max(amax / 127, 1e-12),
q = clamp(round(w / scale), -127, 127).

INT4: one fp32 scale per row and group of `group` inputs (128 by default), q in [-8, 7], packed two per byte for the
INT4 GEMV (lfm2q_gemv_w4): input 2j in the low nibble and 2j + 1 in the high nibble of byte j, each stored as q + 8.
Same expressions as the reference's quantize_int4 / dequantize_int4 (src/lfm2opt/quant.py:22-48), including its
optional clipping search (per group, the scale amax * a / 7 with a on 16 steps from 0.70 to 1.00 that gives the
smallest squared error, first best kept), so the packed bytes and scales are bit-identical.

These are load-time tensor transforms (not kernels of the hot path) and run as PyTorch ops on whatever device holds
the weight, exactly as in the reference.
"""

import torch

GROUP = 128


@torch.no_grad()
def quantize_int8(w: torch.Tensor):
    wf = w.float()
    scale = (wf.abs().amax(1) / 127).clamp_min(1e-12)
    q = torch.round(wf / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.contiguous()


@torch.no_grad()
def quantize_int4(w: torch.Tensor, group: int = GROUP, clip_search: bool = False):
    """[N, K] weight -> (packed uint8 [N, K / 2], scales fp32 [N, K / group])."""
    N, K = w.shape
    if K % group:
        raise ValueError(f"K = {K} is not a multiple of the group size {group}")
    blocks = w.float().view(N, K // group, group)
    amax = blocks.abs().amax(-1).clamp_min(1e-12)
    scale = amax / 7
    if clip_search:
        best_err = torch.full_like(amax, float("inf"))
        for a in torch.linspace(0.70, 1.00, 16).tolist():
            cand = amax * a / 7
            err = (torch.round(blocks / cand[..., None]).clamp(-8, 7) * cand[..., None] - blocks).pow(2).sum(-1)
            take = err < best_err
            best_err = torch.where(take, err, best_err)
            scale = torch.where(take, cand, scale)
    codes = torch.round(blocks / scale[..., None]).clamp(-8, 7).to(torch.int16).view(N, K) + 8
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), scale.contiguous()


@torch.no_grad()
def dequantize_int4(packed: torch.Tensor, scale: torch.Tensor):
    """(packed uint8 [N, K / 2], scales [N, K / group]) -> fp32 [N, K]."""
    p = packed.to(torch.int16)
    q = torch.stack([(p & 0xF) - 8, (p >> 4) - 8], dim=-1).view(packed.shape[0], -1).float()
    group = q.shape[1] // scale.shape[1]
    return (q.view(q.shape[0], -1, group) * scale[..., None]).view(q.shape[0], -1)
