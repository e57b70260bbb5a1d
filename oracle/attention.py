"""TEST INFRASTRUCTURE ONLY: oracle decode attention (CPU)."""

import torch
import torch.nn.functional as F


@torch.no_grad()
def decode_attention_f64(q, kc, vc, pos, scale):
    """fp64 value of one decode step of grouped-query attention before the final bf16 rounding, the quantity the
    reference's split kernel computes (kernels/lfm2_decode.cu:284-416): for each sequence b and query head h (KV head
    h // (NQ / NKV)), out = softmax_t((q . k_t) * scale) . v over positions t = 0 .. min(pos, max_len - 1).
    q [B, NQ, D], kc / vc [B, NKV, max_len, D]."""
    B, NQ, D = q.shape
    NKV, max_len = kc.shape[1], kc.shape[2]
    n = min(int(pos) + 1, max_len)
    k = kc[:, :, :n].double().repeat_interleave(NQ // NKV, 1)  # [B, NQ, n, D]
    v = vc[:, :, :n].double().repeat_interleave(NQ // NKV, 1)
    s = torch.einsum("bhd,bhtd->bht", q.double() * scale, k)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bht,bhtd->bhd", p, v)


@torch.no_grad()
def decode_attention_sdpa(q, kc, vc, pos, scale):
    """The reference's own check expression (tests/test_kernels.py:94-101): F.scaled_dot_product_attention over the
    cache prefix with grouped-query heads, in the dtype of the inputs."""
    n = int(pos) + 1
    return F.scaled_dot_product_attention(q.unsqueeze(2), kc[:, :, :n], vc[:, :, :n], scale=scale,
                                          enable_gqa=True).squeeze(2)


@torch.no_grad()
def split_partials_f64(q, kc, vc, pos, scale, S):
    """fp64 per-split partials (m, l, acc[D]) of the reference's workspace layout ws [B, NQ, S, D + 2]
    (kernels/lfm2_decode.cu:284-383): split s covers positions [s * chunk, (s + 1) * chunk) of 0 .. min(pos,
    max_len - 1), chunk = ceil(max_len / S); an empty split has m = -inf, l = 0 (acc not defined: NaN here)."""
    B, NQ, D = q.shape
    NKV, max_len = kc.shape[1], kc.shape[2]
    n = min(int(pos) + 1, max_len)
    chunk = -(-max_len // S)
    k = kc.double().repeat_interleave(NQ // NKV, 1)
    v = vc.double().repeat_interleave(NQ // NKV, 1)
    ws = torch.full((B, NQ, S, D + 2), float("nan"), dtype=torch.float64)
    for s in range(S):
        t0, t1 = s * chunk, min(n, (s + 1) * chunk)
        if t0 >= t1:
            ws[:, :, s, 0] = float("-inf")
            ws[:, :, s, 1] = 0.0
            continue
        sc = torch.einsum("bhd,bhtd->bht", q.double() * scale, k[:, :, t0:t1])
        m = sc.max(dim=-1).values
        e = torch.exp(sc - m[..., None])
        ws[:, :, s, 0] = m
        ws[:, :, s, 1] = e.sum(-1)
        ws[:, :, s, 2:] = torch.einsum("bht,bhtd->bhd", e, v[:, :, t0:t1])
    return ws
