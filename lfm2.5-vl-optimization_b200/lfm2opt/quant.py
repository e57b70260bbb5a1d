"""Weight-only INT8 quantization for the decode GEMVs and the W8A8 GEMMs; done once at load time.

INT8: one fp32 scale per output row, W ~= q * s[n], q in [-127, 127], round-to-nearest (half to even), symmetric.
Same expression as the reference's quantize_int8 (src/lfm2opt/quant.py:14-18): scale = max(amax / 127, 1e-12),
q = clamp(round(w / scale), -127, 127). It is a load-time tensor transform (not a kernel of the hot path) and runs
as these PyTorch ops on whatever device holds the weight, exactly as in the reference.
"""

import torch


@torch.no_grad()
def quantize_int8(w: torch.Tensor):
    wf = w.float()
    scale = (wf.abs().amax(1) / 127).clamp_min(1e-12)
    q = torch.round(wf / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.contiguous()
