"""One LFM2 decode step (batch 1) on the lfm2q kernels, replayable as one CUDA graph.

The sequence of kernels is the reference's fused decode step (src/lfm2opt/runtime.py:247-294, with its
`_linear` decode GEMVs, :223-244, on int8 weight-only weights): embedding -> rmsnorm; per layer either
  attention:  qkv GEMV -> qk_norm_rope_kv (k, v into the cache at pos) -> decode_attention_split -> o GEMV
  short conv: in_proj GEMV with the conv step fused (gemv_epi 1) -> out_proj GEMV
then residual add + ffn norm -> w1|w3 GEMV with the SwiGLU fused (gemv_epi 0) -> w2 GEMV -> residual add + next norm;
finally the lm_head GEMV, argmax, the token and the position advanced on the device. Every buffer is allocated once,
so the step captures into a CUDA graph (`DecodeStep.capture`), as the reference's runtime does.

`ops` is the kernel backend: by default lfm2q's (`lfm2opt.kernels.ext()`); any object with the reference
extension's op names and signatures (gemv, gemv_epi, add_rmsnorm, qk_norm_rope_kv, decode_attention_split) works.
"""

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .quant import quantize_int8

BF = torch.bfloat16


@dataclass(frozen=True)
class Lfm2Config:
    """The LM of LFM2.5-VL-1.6B (LFM2-1.2B): the decode GEMV shapes qkv 3072x2048, o 2048x2048, in_proj 6144x2048,
    out_proj 2048x2048, w1|w3 16384x2048, w2 2048x8192, lm_head 65536x2048."""
    hidden: int = 2048
    layers: int = 16
    attn_layers: tuple = (2, 5, 8, 10, 12, 14)
    n_heads: int = 32
    n_kv: int = 8
    head_dim: int = 64
    inter: int = 8192
    vocab: int = 65536
    eps: float = 1e-5
    rope_theta: float = 1e6
    conv_len: int = 3


class Lfm2Weights:
    """Random-init int8 weight-only decode weights of an Lfm2Config (per-row scales, quantize_int8), bf16 norms,
    conv kernels and embedding, generated on `device` from `seed` (no checkpoint is available offline)."""

    def __init__(self, cfg: Lfm2Config, device, seed=0):
        g = torch.Generator(device=device).manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim

        def lin(n, k):
            return quantize_int8((torch.randn(n, k, generator=g, device=device) * 0.02).to(BF))

        def norm(n):
            return (torch.rand(n, generator=g, device=device) + 0.5).to(BF)

        self.cfg = cfg
        self.embed = (torch.randn(cfg.vocab, H, generator=g, device=device) * 0.5).to(BF)
        self.norm = [norm(H) for _ in range(cfg.layers + 1)]  # operator norm of layer 0 .. final norm
        self.ffn_norm = [norm(H) for _ in range(cfg.layers)]
        self.layer = []
        for i in range(cfg.layers):
            if i in cfg.attn_layers:
                self.layer.append({"qkv": lin((cfg.n_heads + 2 * cfg.n_kv) * D, H), "o": lin(H, cfg.n_heads * D),
                                   "qw": norm(D), "kw": norm(D)})
            else:
                self.layer.append({"in": lin(3 * H, H), "out": lin(H, H),
                                   "cw": (torch.randn(H, cfg.conv_len, generator=g, device=device) * 0.5).to(BF)})
            self.layer[-1]["w13"] = lin(2 * cfg.inter, H)
            self.layer[-1]["w2"] = lin(H, cfg.inter)
        self.head = lin(cfg.vocab, H)
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))


class DecodeStep:
    """State (KV caches, conv states, token, position) and buffers of batch-1 decode for `weights`; `step()` runs
    one token. max_len: cache slots; attn_splits: the split count of decode_attention_split (the reference's
    default, 16)."""

    def __init__(self, weights: Lfm2Weights, max_len=4096, attn_splits=16, ops=None):
        if ops is None:
            from .kernels import ext
            ops = ext()
        self.w, self.ops, self.cfg = weights, ops, weights.cfg
        c, dev = self.cfg, weights.embed.device
        H = c.hidden
        self.max_len, self.S = max_len, attn_splits
        self.kc = {i: torch.zeros(1, c.n_kv, max_len, c.head_dim, device=dev, dtype=BF) for i in c.attn_layers}
        self.vc = {i: torch.zeros_like(self.kc[i]) for i in c.attn_layers}
        self.conv = {i: torch.zeros(1, H, c.conv_len, device=dev, dtype=BF)
                     for i in range(c.layers) if i not in c.attn_layers}
        self.tok = torch.zeros(1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.h = torch.empty(1, H, device=dev, dtype=BF)
        self.x = torch.empty_like(self.h)
        self.y = torch.empty_like(self.h)
        self.cy = torch.empty_like(self.h)
        self.qkv = torch.empty(1, (c.n_heads + 2 * c.n_kv) * c.head_dim, device=dev, dtype=BF)
        self.q = torch.empty(1, c.n_heads, c.head_dim, device=dev, dtype=BF)
        self.o = torch.empty_like(self.q)
        self.ws = torch.empty(1, c.n_heads, attn_splits, c.head_dim + 2, device=dev, dtype=torch.float32)
        self.act = torch.empty(1, c.inter, device=dev, dtype=BF)
        self.logits = torch.empty(1, c.vocab, device=dev, dtype=BF)
        self.graph = None

    @torch.no_grad()
    def step(self):
        K, W, c = self.ops, self.w, self.cfg
        fused_ends = hasattr(K, "embed_rmsnorm") and hasattr(K, "argmax_next")  # lfm2q's backend
        if fused_ends:  # embedding lookup + first norm in one launch
            K.embed_rmsnorm(self.tok, W.embed, W.norm[0], self.h, self.x, c.eps)
        else:
            self.h.copy_(F.embedding(self.tok, W.embed))
            K.add_rmsnorm(self.h, None, W.norm[0], self.x, c.eps)
        for i, L in enumerate(W.layer):
            if i in c.attn_layers:
                K.gemv(L["qkv"][0], L["qkv"][1], self.x, self.qkv)
                K.qk_norm_rope_kv(self.qkv, L["qw"], L["kw"], W.inv_freq, 1.0, self.pos, self.q, self.kc[i],
                                  self.vc[i], c.eps)
                K.decode_attention_split(self.q, self.kc[i], self.vc[i], self.pos, self.o, self.ws,
                                         c.head_dim ** -0.5)
                K.gemv(L["o"][0], L["o"][1], self.o.view(1, -1), self.y)
            else:
                K.gemv_epi(1, L["in"][0], L["in"][1], self.x, self.cy, self.conv[i], L["cw"], None)
                K.gemv(L["out"][0], L["out"][1], self.cy, self.y)
            K.add_rmsnorm(self.h, self.y, W.ffn_norm[i], self.x, c.eps)
            K.gemv_epi(0, L["w13"][0], L["w13"][1], self.x, self.act)
            K.gemv(L["w2"][0], L["w2"][1], self.act, self.y)
            K.add_rmsnorm(self.h, self.y, W.norm[i + 1], self.x, c.eps)
        K.gemv(W.head[0], W.head[1], self.x, self.logits)
        if fused_ends:  # argmax, next token and position advance in one launch
            K.argmax_next(self.logits, self.tok, self.pos)
        else:
            self.tok.copy_(torch.argmax(self.logits, dim=-1))
            self.pos.add_(1)

    def capture(self):
        """Capture one step into a CUDA graph (after one eager warm-up step on a side stream, which advances the
        position by one). `replay()` then runs a step."""
        dev = self.h.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        return self

    def replay(self):
        self.graph.replay()
