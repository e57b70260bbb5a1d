"""DecodeStep's host logic on CPU with a recording stand-in for the kernels: the op sequence is the reference's fused
decode step (src/lfm2opt/runtime.py:247-294), every op sees the tensors of its layer, and the step's two ends use
the fused lfm2q ops when the backend has them (else torch's embedding / argmax, as the reference)."""

import torch

from lfm2opt.decode_step import DecodeStep, Lfm2Config, Lfm2Weights

CFG = Lfm2Config(hidden=256, layers=4, attn_layers=(1, 3), n_heads=4, n_kv=1, inter=512, vocab=64)


class Recorder:
    def __init__(self, fused_ends):
        self.calls = []
        if fused_ends:
            self.embed_rmsnorm = lambda tok, embed, w, h, x, eps: self.calls.append(("embed_rmsnorm", w))
            self.argmax_next = lambda logits, tok, pos: self.calls.append(("argmax_next", logits.shape))

    def gemv(self, W, s, x, y):
        assert x.shape[-1] == W.shape[1] and y.numel() == W.shape[0]
        self.calls.append(("gemv", tuple(W.shape)))

    def gemv_epi(self, epi, W, s, x, y, state=None, cw=None, cbias=None):
        self.calls.append(("gemv_epi", epi, tuple(W.shape)))

    def add_rmsnorm(self, h, y, w, x, eps):
        self.calls.append(("add_rmsnorm", y is not None, w))

    def qk_norm_rope_kv(self, qkv, qw, kw, inv_freq, scaling, pos, q, kc, vc, eps):
        self.calls.append(("qk_norm_rope_kv", tuple(kc.shape)))

    def decode_attention_split(self, q, kc, vc, pos, out, ws, scale):
        assert ws.shape[-1] == 66 and abs(scale - 0.125) < 1e-9
        self.calls.append(("decode_attention_split", tuple(ws.shape)))


def expected(W, fused_ends):
    c, H = CFG, CFG.hidden
    qkv = ((c.n_heads + 2 * c.n_kv) * c.head_dim, H)
    seq = [("embed_rmsnorm", W.norm[0])] if fused_ends else [("add_rmsnorm", False, W.norm[0])]
    for i in range(c.layers):
        if i in c.attn_layers:
            seq += [("gemv", qkv), ("qk_norm_rope_kv", (1, c.n_kv, 128, c.head_dim)),
                    ("decode_attention_split", (1, c.n_heads, 16, 66)), ("gemv", (H, c.n_heads * c.head_dim))]
        else:
            seq += [("gemv_epi", 1, (3 * H, H)), ("gemv", (H, H))]
        seq += [("add_rmsnorm", True, W.ffn_norm[i]), ("gemv_epi", 0, (2 * c.inter, H)), ("gemv", (H, c.inter)),
                ("add_rmsnorm", True, W.norm[i + 1])]
    seq += [("gemv", (c.vocab, H))]
    if fused_ends:
        seq += [("argmax_next", (1, c.vocab))]
    return seq


def same(a, b):
    if len(a) != len(b):
        return False
    for x, y in zip(a, b):
        if len(x) != len(y) or x[0] != y[0]:
            return False
        for u, v in zip(x[1:], y[1:]):
            if isinstance(u, torch.Tensor) or isinstance(v, torch.Tensor):
                if u is not v:
                    return False
            elif u != v:
                return False
    return True


def test_step_issues_the_reference_sequence():
    W = Lfm2Weights(CFG, torch.device("cpu"), seed=1)
    for fused_ends in (True, False):
        rec = Recorder(fused_ends)
        s = DecodeStep(W, max_len=128, ops=rec)
        s.tok.fill_(5)
        s.logits.zero_()
        s.step()
        assert same(rec.calls, expected(W, fused_ends)), rec.calls[:6]
        if not fused_ends:  # torch ends: the argmax of the (zero) logits, position advanced
            assert int(s.tok) == 0 and int(s.pos) == 1


def test_weights_have_the_config_shapes():
    W = Lfm2Weights(CFG, torch.device("cpu"), seed=2)
    assert W.embed.shape == (CFG.vocab, CFG.hidden) and len(W.norm) == CFG.layers + 1
    for i, L in enumerate(W.layer):
        assert L["w13"][0].dtype == torch.int8 and L["w13"][0].shape == (2 * CFG.inter, CFG.hidden)
        assert ("qkv" in L) == (i in CFG.attn_layers)
    assert W.inv_freq.shape == (CFG.head_dim // 2,)
