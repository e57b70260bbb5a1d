"""TEST INFRASTRUCTURE ONLY: oracle for the decode step's small kernels (CPU, torch).

Each function restates the PyTorch expression the reference's own tests check its kernels against
(tests/test_kernels.py:26-90: the ops of transformers' modeling_lfm2.py in bf16), evaluated on CPU."""

import torch
import torch.nn.functional as F

BF = torch.bfloat16


def rms(x, w, eps):
    """tests/test_kernels.py:26-29: n = bf16(x * rsqrt(mean(x^2) + eps)) in fp32, then w * n in bf16."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(BF)
    return w * n


@torch.no_grad()
def add_rmsnorm_ref(h, y, w, eps):
    """tests/test_kernels.py:40-50: h' = h + y (bf16), x = rms(h', w). Returns (h', x)."""
    hn = h + y if y is not None else h.clone()
    return hn, rms(hn, w, eps)


@torch.no_grad()
def shortconv_step_ref(bcx, state, w, bias=None):
    """tests/test_kernels.py:53-70 (transformers' causal_conv1d_update path): returns (y [B, H], new state)."""
    B, H3 = bcx.shape
    H = H3 // 3
    b_, c_, x_ = bcx.view(B, 1, H3).transpose(-1, -2).chunk(3, dim=-2)
    hx = b_ * x_
    new = torch.cat([state, hx], dim=-1)
    st = new[:, :, -3:].clone()
    conv = F.conv1d(new.float(), w.float().unsqueeze(1), None if bias is None else bias.float(), groups=H)
    conv = conv[:, :, -1:].to(BF)
    y = (c_ * conv).transpose(-1, -2).reshape(B, H)
    return y, st


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


@torch.no_grad()
def qk_norm_rope_kv_ref(qkv, qw, kw, inv_freq, scaling, pos, NQ, NKV, eps):
    """tests/test_kernels.py:73-90: per-head rms of q and k, RoPE as transformers' apply_rotary_pos_emb in bf16
    (q * cos + rotate_half(q) * sin, cos / sin = bf16(cos / sin(pos * inv_freq) * scaling)). Returns (q [B, NQ, 64],
    k [B, NKV, 64], v [B, NKV, 64])."""
    B = qkv.shape[0]
    q, k, v = qkv.view(B, NQ + 2 * NKV, 64).split([NQ, NKV, NKV], dim=1)
    q, k = rms(q, qw, eps), rms(k, kw, eps)
    freqs = float(pos) * inv_freq.float()
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = (emb.cos() * scaling).to(BF), (emb.sin() * scaling).to(BF)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin, v.clone()
