"""The decode-step oracle (oracle/decode.py) on CPU: the reference test expressions behave as the model's ops."""

import torch

from oracle.decode import add_rmsnorm_ref, qk_norm_rope_kv_ref, rotate_half, shortconv_step_ref

BF = torch.bfloat16


def test_rmsnorm_scales_rows_to_unit_rms():
    g = torch.Generator().manual_seed(0)
    h = torch.randn(3, 2048, generator=g).to(BF)
    hn, x = add_rmsnorm_ref(h, None, torch.ones(2048, dtype=BF), 1e-5)
    assert torch.equal(hn, h)
    r = x.float().pow(2).mean(-1).sqrt()
    assert ((r - 1).abs() < 1e-2).all()


def test_shortconv_state_shifts_and_output_is_the_window_dot():
    g = torch.Generator().manual_seed(1)
    B, H = 2, 16
    bcx = torch.randn(B, 3 * H, generator=g).to(BF)
    st = torch.randn(B, H, 3, generator=g).to(BF)
    w = torch.randn(H, 3, generator=g).to(BF)
    y, st2 = shortconv_step_ref(bcx, st, w)
    bx = (bcx[:, :H] * bcx[:, 2 * H:])
    assert torch.equal(st2[:, :, :2], st[:, :, 1:]) and torch.equal(st2[:, :, 2], bx)
    conv = (w.float() * st2.float()).sum(-1)
    assert ((y.float() - (bcx[:, H:2 * H].float() * conv)).abs() <= 0.05 * conv.abs().max() + 0.05).all()


def test_rope_at_position_zero_is_the_norm_and_rotation_is_a_rotation():
    g = torch.Generator().manual_seed(2)
    qkv = torch.randn(1, 48 * 64, generator=g).to(BF)
    qw = kw = torch.ones(64, dtype=BF)
    inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float) / 64))
    q0, k0, v0 = qk_norm_rope_kv_ref(qkv, qw, kw, inv, 1.0, 0, 32, 8, 1e-5)
    q1, _, _ = qk_norm_rope_kv_ref(qkv, qw, kw, inv, 1.0, 1000, 32, 8, 1e-5)
    assert torch.equal(v0, qkv.view(1, 48, 64)[:, 40:])
    # pos 0: cos = 1, sin = 0 -> the normed vector; any pos keeps each (d, d + 32) pair's length
    n0 = q0.float().pow(2)
    n1 = q1.float().pow(2)
    pair = lambda t: t[..., :32] + t[..., 32:]  # noqa: E731
    assert ((pair(n0) - pair(n1)).abs() <= 0.05 * pair(n0) + 1e-2).all()
    assert torch.equal(rotate_half(rotate_half(q0)), -q0)
